"""Multi-GPU partitioning of the attention hot path, one process per GPU.

The reference has no multi-GPU inference (its collectives serve training
only: packages/wpt-model/src/wpt_model/sequence.py:143-185,
packages/wpt-training/src/wpt_training/strategies/ddp.py:40-55). Two
partitions fit this path:

  * independent rows (prefill batches, decode rows, verification rows): each
    rank takes its own rows and no data crosses NVLink (shard_rows,
    balanced_rows, which balances decode rows by their cached lengths);
  * one long row (long-context decode): its keys are split into contiguous
    shards, one per rank. Each rank's kernel computes split partials of the
    query over its shard (output normalised by each split's softmax sum, and
    that sum's log); one exchange kernel merges them, stores the result into
    every rank's exchange buffer over NVLink (CUDA IPC mappings, set up once
    per shape), waits for every rank's result of the same call and merges
    the ranks' partials by log-sum-exp: H x (C + 1) floats per rank and
    query, latency-bound, so two launches and no collective per call. Where
    that cannot run (a gloo group, ranks sharing a GPU, more than 8 ranks,
    WPT_B200_PEER=0), the partials are merged into this rank's chunk of a
    shared buffer, one in-place all-gather exchanges the chunks and a merge
    kernel combines them.
"""

import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_rows(n, world, rank):
    """The contiguous slice of n rows that `rank` of `world` takes."""
    per, extra = divmod(n, world)
    start = rank * per + min(rank, extra)
    return slice(start, start + per + (1 if rank < extra else 0))


def balanced_rows(lengths, world):
    """Rows split over `world` ranks so that each rank's total length is
    about equal (longest first, each to the least loaded rank): a list of
    row-index lists, each sorted."""
    lengths = [int(x) for x in lengths]
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    load = [0] * world
    parts = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        parts[r].append(i)
        load[r] += lengths[i]
    return [sorted(p) for p in parts]


def key_shard(n_rows, world, rank):
    """The contiguous key rows [start, stop) of a long row that `rank` holds."""
    s = shard_rows(n_rows, world, rank)
    return s.start, s.stop


_PLANS = {}  # (shape, shard length, world, device, group) -> the long row's buffers on this rank


class PeerSetupFailed(RuntimeError):
    """Some rank could not allocate or map an exchange buffer; every rank
    raises it together (and has released what it made), so the ranks fall
    back to the all-gather exchange together."""


class PeerExchange:
    """This rank's exchange buffer for one long-row shape and the other
    ranks' buffers mapped into this process (wpt_peer_alloc / wpt_peer_open
    over CUDA IPC). Built by every rank of `group` together: the handles are
    gathered, every rank reports whether it could allocate and map, and the
    set-up ends with a barrier, so no rank writes into a buffer before its
    owner has zeroed it. A failure on any rank raises PeerSetupFailed on
    every rank. Kept for the life of the process."""

    def __init__(self, rows, C, world, rank, group, device):
        lib = _lib.lib()
        nbytes = lib.wpt_peer_bytes(world, rows, C)
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        self.peers = (ctypes.c_void_p * world)()
        opened = []
        with torch.cuda.device(device):
            ok = nbytes > 0 and lib.wpt_peer_alloc(nbytes, ctypes.byref(own), handle) == _lib.OK
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw if ok else None, group=group)
            ok = ok and all(h is not None for h in handles)
            if ok:
                for g in range(world):
                    if g == rank:
                        self.peers[g] = own.value
                        continue
                    mapped = ctypes.c_void_p()
                    if lib.wpt_peer_open(handles[g], ctypes.byref(mapped)) != _lib.OK:
                        ok = False
                        break
                    self.peers[g] = mapped.value
                    opened.append(mapped.value)
            flags = [None] * world
            dist.all_gather_object(flags, bool(ok), group=group)
            if not all(flags):
                for ptr in opened:
                    lib.wpt_peer_close(ptr, 1)
                dist.barrier(group=group)  # every rank has unmapped before any buffer is freed
                if own.value:
                    lib.wpt_peer_close(own.value, 0)
                raise PeerSetupFailed("a rank could not set up its exchange buffer: " +
                                      lib.wpt_last_error().decode(errors="replace"))
            dist.barrier(group=group)
        self.world, self.rank = world, rank


def _peer_capable(q, world, rows, group):
    """Whether the ranks can exchange through peer mappings: CUDA tensors, an
    NCCL group of 2 to 8 ranks on distinct GPUs (the ranks' exchange kernels
    wait for one another, so two ranks must never share a GPU), at most 4,096
    rows, and WPT_B200_PEER not 0. Every rank reaches the same answer (the
    GPU identities are gathered)."""
    if os.environ.get("WPT_B200_PEER", "1") == "0" or not q.is_cuda or not 2 <= world <= 8:
        return False
    if dist.get_backend(group) != "nccl" or _lib.lib().wpt_peer_bytes(world, rows, q.shape[-1]) == 0:
        return False
    ids = [None] * world
    dist.all_gather_object(ids, str(torch.cuda.get_device_properties(q.device).uuid), group=group)
    return len(set(ids)) == world


def _long_plan(q, n_local, world, group):
    """The buffers of one long-row shape on this rank, allocated once: this
    rank's split partials (its kernel's splits for its own shard) and the
    exchanged buffer (world, chunk), chunk = one partial (rows, C) and its
    log-sums (rows), padded to 16 bytes."""
    B, T, H, C = q.shape
    key = (tuple(q.shape), n_local, world, q.device, id(group))
    plan = _PLANS.get(key)
    if plan is None:
        rows = B * T * H
        splits, _ = ops.partials_plan(q.shape, n_local, q.device)
        part_o = torch.empty(splits, rows, C, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(splits, rows, dtype=torch.float32, device=q.device)
        parts = None
        if _peer_capable(q, world, rows, group):
            try:
                parts = PeerExchange(rows, C, world, dist.get_rank(group), group, q.device)
            except PeerSetupFailed:
                parts = None  # every rank takes the all-gather exchange
        if parts is None:
            chunk = (rows * (C + 1) + 3) // 4 * 4
            parts = torch.empty(world, chunk, dtype=torch.float32, device=q.device)
        plan = _PLANS[key] = (splits, part_o, part_lse, parts)
    return plan


def long_decode(q, k_shard, v_shard, shard_start, positions, scale, sink=None, group=None):
    """Attention of q (B, T, H, C) over a long row whose keys are split over
    the ranks of `group`: this rank holds rows [shard_start, shard_start + n)
    as k_shard, v_shard (B, n, C). positions (B, T) are positions in the whole
    row. Returns (out (B, T, H, C) bf16, lse (B, T, H)) on every rank.

    Each rank's key-stream kernel computes split partials of its shard;
    then, with peer mappings (an NCCL group on distinct GPUs, set up on the
    first call of a shape, which every rank must make together and outside
    any graph capture), one exchange kernel merges them, stores the result
    into every rank's buffer over NVLink, waits for every rank's result of
    the same call and merges them with the sink. Otherwise a merge kernel
    combines them into one partial (normalised output and log-sum, fp32)
    written straight into this rank's chunk of the exchanged buffer, one
    in-place all-gather brings every rank's chunk to every rank (rows x
    (C + 1) floats each, whatever the split counts), and one merge kernel
    combines the ranks' partials with the sink. Buffers are allocated once
    per shape and reused, and nothing synchronises the host, so the call can
    be captured in a CUDA graph; calls on one stream are ordered, calls that
    overlap on several streams would share the buffers."""
    B, T, H, C = q.shape
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    # rows of this shard the query sees: 0 .. local (none when negative)
    local = positions if shard_start == 0 else positions - shard_start
    if world == 1:  # the whole row is here: one kernel call
        return ops.stream_forward(q, k_shard, v_shard, local, scale, sink=sink)
    rank = dist.get_rank(group)
    splits, part_o, part_lse, parts = _long_plan(q, k_shard.shape[1], world, group)
    rows = B * T * H
    ops.stream_partials(q, k_shard, v_shard, local, scale, into=(part_o, part_lse), splits=splits)
    if isinstance(parts, PeerExchange):
        merged, merged_lse = ops.exchange(part_o, part_lse, parts.peers, world, rank, H, sink)
        return merged.reshape(B, T, H, C), merged_lse.reshape(B, T, H)
    mine = parts[rank]
    ops.merge_partial(part_o, part_lse, out_o=mine[:rows * C].view(rows, C), out_lse=mine[rows * C:rows * (C + 1)])
    dist.all_gather_into_tensor(parts.view(-1), mine, group=group)  # in place: every rank's chunk to every rank
    merged, merged_lse = ops.merge_groups(parts, 1, rows, H, C, sink)
    return merged.reshape(B, T, H, C), merged_lse.reshape(B, T, H)
