"""The multi-GPU partitioning logic on CPU gloo ranks (world size 2 and 3):
row sharding, length-balanced decode rows, and the long-row key split. The
long row runs long_decode's all-gather branch, the one a gloo group (and any
group that cannot map its peers' memory) takes: each rank's split partials,
their merge into one partial in the rank's chunk of the shared buffer, the
in-place all-gather, the grouped merge, with the GPU calls it makes
(ops.partials_plan, ops.stream_partials, ops.merge_partial,
ops.merge_groups) replaced by CPU restatements, since this suite has no
GPU; the kernels themselves are checked by the gpu tests. The peer
exchange's set-up (multi.PeerExchange) runs with its library calls faked, to
show that a failure on one rank fails every rank together."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oat
from wpt_b200 import multi


def test_shard_rows_covers_every_row_once():
    for n in (1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            rows = [r for rank in range(world) for r in range(n)[multi.shard_rows(n, world, rank)]]
            assert rows == list(range(n))


def test_balanced_rows_balances_lengths():
    g = torch.Generator().manual_seed(0)
    lengths = torch.randint(1024, 32769, (64,), generator=g).tolist()
    for world in (2, 4, 8):
        parts = multi.balanced_rows(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)
        assert max(loads) / (sum(lengths) / world) < 1.05


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SPLITS = 3  # partials per rank in the CPU stand-ins


def _cpu_partials_plan(q_shape, N, device, window=0):
    return SPLITS, 1


def _cpu_stream_partials(q, k, v, local, scale, window=0, into=None, splits=None):
    """The key-stream kernel's partials-only mode restated on the CPU: the
    shard's keys cut into `splits` equal chunks, each chunk's output
    normalised by its own sum and that sum's log (-inf for no key)."""
    B, T, H, C = q.shape
    n = k.shape[1]
    per = -(-n // splits)
    part_o, part_lse = into
    for s in range(splits):
        a, b = s * per, min(n, (s + 1) * per)
        if a >= b:
            part_o[s] = 0.0
            part_lse[s] = float("-inf")
            continue
        out, lse = oat.range_attention(q.numpy(), k[:, a:b].numpy(), v[:, a:b].numpy(), (local - a).numpy(), scale)
        part_o[s] = torch.from_numpy(np.nan_to_num(out)).reshape(B * T * H, C)
        part_lse[s] = torch.from_numpy(lse).reshape(B * T * H)
    return part_o, part_lse


def _cpu_merge_partial(part_o, part_lse, out_o=None, out_lse=None):
    """The merge kernel's partial mode restated: the splits' normalised
    output and log-sum together, no sink."""
    o, total = oat.merge_partials(part_o.double().numpy(), part_lse.double().numpy(), np.ones(part_lse.shape))
    out_o.copy_(torch.from_numpy(np.nan_to_num(o)).float())
    out_lse.copy_(torch.from_numpy(total).float())
    return out_o, out_lse


def _cpu_merge_groups(parts, per, rows, H, C, sink=None):
    """The grouped merge kernel restated: chunk g = per splits' outputs
    (per, rows, C) then their log-sums (per, rows)."""
    G = parts.shape[0]
    o = parts[:, :per * rows * C].reshape(G * per, rows, C).double().numpy()
    lse = parts[:, per * rows * C:per * rows * (C + 1)].reshape(G * per, rows).double().numpy()
    out, total = oat.merge_partials(o, lse, np.ones(lse.shape),
                                    None if sink is None else np.tile(sink.numpy(), rows // H))
    return torch.from_numpy(out).float(), torch.from_numpy(total).float()


def _long_rank(rank, world, port, result, with_sink):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # the production branch of long_decode, with the three GPU calls it
    # makes replaced by their CPU restatements (no GPU in this suite)
    from wpt_b200 import ops
    ops.partials_plan = _cpu_partials_plan
    ops.stream_partials = _cpu_stream_partials
    ops.merge_partial = _cpu_merge_partial
    ops.merge_groups = _cpu_merge_groups
    try:
        g = torch.Generator().manual_seed(5)
        B, T, H, C, N = 1, 2, 4, 16, 1000
        q = torch.randn(B, T, H, C, generator=g, dtype=torch.float64)
        k = torch.randn(B, N, C, generator=g, dtype=torch.float64)
        v = torch.randn(B, N, C, generator=g, dtype=torch.float64)
        sink = torch.randn(H, generator=g, dtype=torch.float64) if with_sink else None
        positions = torch.tensor([[700, 999]])
        start, stop = multi.key_shard(N, world, rank)
        for _ in range(2):  # the second call reuses the plan and its buffer
            out, lse = multi.long_decode(q.float(), k[:, start:stop].float(), v[:, start:stop].float(), start,
                                         positions, 0.25, sink=None if sink is None else sink.float())
        if rank == 0:
            result["out"], result["lse"] = out.numpy(), lse.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,with_sink", [(2, False), (3, True)])
def test_long_row_split_over_gloo_ranks_equals_whole(world, with_sink):
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_long_rank, args=(world, port, result, with_sink), nprocs=world, start_method="spawn",
                       join=True)
    g = torch.Generator().manual_seed(5)
    B, T, H, C, N = 1, 2, 4, 16, 1000
    q = torch.randn(B, T, H, C, generator=g, dtype=torch.float64)
    k = torch.randn(B, N, C, generator=g, dtype=torch.float64)
    v = torch.randn(B, N, C, generator=g, dtype=torch.float64)
    sink = torch.randn(H, generator=g, dtype=torch.float64).numpy() if with_sink else None
    q, k, v = (x.float().double() for x in (q, k, v))
    ref, ref_lse = oat.range_attention(q.numpy(), k.numpy(), v.numpy(), np.array([[700, 999]]), 0.25, sink=sink)
    assert np.abs(result["out"] - ref).max() < 1e-5
    assert np.abs(result["lse"] - ref_lse).max() < 1e-5


class _FakePeerLib:
    """Stands in for the library's peer-buffer calls on a CPU rank: `fail`
    names the call that fails on this rank ("alloc", "open" or None)."""

    def __init__(self, rank, fail):
        self.rank, self.fail, self.closed = rank, fail, []

    def wpt_peer_bytes(self, world, rows, C):
        return 4096

    def wpt_peer_alloc(self, nbytes, buffer, handle):
        if self.fail == "alloc":
            return 3
        buffer._obj.value = 256 * (self.rank + 1)
        handle.raw = bytes([self.rank]) * 64
        return 0

    def wpt_peer_open(self, handle, buffer):
        if self.fail == "open":
            return 3
        buffer._obj.value = 4096 * (handle[0] + 1)
        return 0

    def wpt_peer_close(self, buffer, opened):
        self.closed.append((buffer, opened))
        return 0

    def wpt_last_error(self):
        return b"no peer memory here"


def _peer_setup_rank(rank, world, port, fail_rank, fail, result):
    import contextlib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = _FakePeerLib(rank, fail if rank == fail_rank else None)
        multi._lib.lib = lambda: fake
        multi.torch.cuda.device = lambda device: contextlib.nullcontext()
        try:
            multi.PeerExchange(8, 128, world, rank, None, "cpu")
            result[rank] = ("built", fake.closed)
        except multi.PeerSetupFailed:
            result[rank] = ("failed", fake.closed)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail", ["alloc", "open", None])
def test_peer_setup_fails_on_every_rank_together(fail):
    """A rank that cannot allocate or map an exchange buffer makes every rank
    raise PeerSetupFailed (so all of them take the all-gather exchange), each
    having unmapped what it mapped and freed its own buffer; with no failure
    every rank builds it."""
    world = 3
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_peer_setup_rank, args=(world, _free_port(), 1, fail, result), nprocs=world,
                       start_method="spawn", join=True)
    for rank in range(world):
        state, closed = result[rank]
        if fail is None:
            assert state == "built" and closed == []
            continue
        assert state == "failed"
        own = [c for c in closed if c[1] == 0]
        assert own == ([] if (fail == "alloc" and rank == 1) else [(256 * (rank + 1), 0)])
        mapped = [c for c in closed if c[1] == 1]
        if fail == "open" and rank != 1:  # the ranks that mapped their peers unmapped them
            assert len(mapped) == world - 1
