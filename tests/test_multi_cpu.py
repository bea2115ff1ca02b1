"""The multi-GPU partitioning logic on CPU gloo ranks (world size 2 and 3):
row sharding, length-balanced decode rows, and the long-row key split whose
partials are all-gathered and merged by log-sum-exp. The per-shard
attention and the merge are the CPU oracle here (no GPU in this suite); on
the GPU they are the key-stream and merge kernels, checked by the gpu tests."""

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


def _oracle_partial(q, k, v, local, scale):
    out, lse = oat.range_attention(q.numpy(), k.numpy(), v.numpy(), local.numpy(), scale)
    return torch.from_numpy(out).float(), torch.from_numpy(lse).float()


def _oracle_merge(parts_o, parts_lse, H, sink):
    out, lse = oat.merge_partials(parts_o.double().numpy(), parts_lse.double().numpy(),
                                  np.ones(parts_lse.shape), None if sink is None else np.tile(sink.numpy(), parts_lse.shape[1] // H))
    return torch.from_numpy(out).float(), torch.from_numpy(lse).float()


def _long_rank(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        B, T, H, C, N = 1, 2, 4, 16, 1000
        q = torch.randn(B, T, H, C, generator=g, dtype=torch.float64)
        k = torch.randn(B, N, C, generator=g, dtype=torch.float64)
        v = torch.randn(B, N, C, generator=g, dtype=torch.float64)
        positions = torch.tensor([[700, 999]])
        start, stop = multi.key_shard(N, world, rank)
        out, lse = multi.long_decode(q, k[:, start:stop], v[:, start:stop], start, positions, 0.25,
                                     partial=_oracle_partial, merge=_oracle_merge)
        if rank == 0:
            result["out"], result["lse"] = out.numpy(), lse.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_long_row_split_over_gloo_ranks_equals_whole(world):
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    result = manager.dict()
    mp.start_processes(_long_rank, args=(world, port, result), nprocs=world, start_method="spawn", join=True)
    g = torch.Generator().manual_seed(5)
    B, T, H, C, N = 1, 2, 4, 16, 1000
    q = torch.randn(B, T, H, C, generator=g, dtype=torch.float64)
    k = torch.randn(B, N, C, generator=g, dtype=torch.float64)
    v = torch.randn(B, N, C, generator=g, dtype=torch.float64)
    ref, ref_lse, _ = oat.exact_attention(q.numpy(), k.numpy(), v.numpy(), np.array([[700, 999]]), 0.25, 0, 0)
    assert np.abs(result["out"] - ref).max() < 1e-5
    assert np.abs(result["lse"] - ref_lse).max() < 1e-5
