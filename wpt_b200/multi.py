"""Multi-GPU partitioning of the attention hot path, one process per GPU.

The reference has no multi-GPU inference (its collectives serve training
only: packages/wpt-model/src/wpt_model/sequence.py:143-185,
packages/wpt-training/src/wpt_training/strategies/ddp.py:40-55). Two
partitions fit this path:

  * independent rows (prefill batches, decode rows, verification rows): each
    rank takes its own rows and no data crosses NVLink (shard_rows,
    balanced_rows, which balances decode rows by their cached lengths);
  * one long row (long-context decode): its keys are split into contiguous
    shards, one per rank. Each rank computes the partial attention of the
    query over its shard (output normalised by its own softmax sum, and that
    sum's log), the ranks all-gather those partials over NCCL, and each
    merges them by log-sum-exp (the merge kernel): H x (C + 1) floats per rank
    and query, latency-bound.
"""

import torch
import torch.distributed as dist

from . import ops


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


def long_decode(q, k_shard, v_shard, shard_start, positions, scale, sink=None, group=None, partial=None,
                merge=None):
    """Attention of q (B, T, H, C) over a long row whose keys are split over
    the ranks of `group`: this rank holds rows [shard_start, shard_start + n)
    as k_shard, v_shard (B, n, C). positions (B, T) are positions in the whole
    row. Returns (out (B, T, H, C) bf16, lse (B, T, H)) on every rank.

    partial(q, k, v, local_positions, scale) -> (out, lse) computes this rank's
    share (default: the key-stream kernel); merge(parts_o, parts_lse, H,
    sink) -> (out rows, lse rows) combines the gathered shares (default: the
    merge kernel). Tests substitute CPU versions to check the partitioning
    with gloo ranks."""
    B, T, H, C = q.shape
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    local = positions - shard_start  # rows of this shard the query sees: 0 .. local (none when negative)
    if partial is None and merge is None:
        if world == 1:  # the whole row is here: one kernel call
            return ops.stream_forward(q, k_shard, v_shard, local, scale, sink=sink)
        # the kernel's own split partials go straight into the collective and
        # one merge combines every rank's splits (no local merge, no copies)
        part_o, part_lse = ops.stream_partials(q, k_shard, v_shard, local, scale)
        S = part_o.shape[0]
        parts_o = torch.empty(world * S, B * T * H, C, dtype=torch.float32, device=q.device)
        parts_s = torch.empty(world * S, B * T * H, dtype=torch.float32, device=q.device)
        dist.all_gather_into_tensor(parts_o, part_o, group=group)
        dist.all_gather_into_tensor(parts_s, part_lse, group=group)
        merged, merged_lse = ops.merge_partials(parts_o, parts_s, H, sink)
        return merged.reshape(B, T, H, C), merged_lse.reshape(B, T, H)
    partial = partial or (lambda q_, k_, v_, p_, s_: ops.stream_forward(q_, k_, v_, p_, s_))
    merge = merge or ops.merge_partials
    out, lse = partial(q, k_shard, v_shard, local, scale)
    o = out.float().reshape(1, B * T * H, C)
    s = lse.float().reshape(1, B * T * H)
    if world > 1:  # one collective: each rank's (output, log-sum) rows packed side by side
        packed = torch.cat([o, s.unsqueeze(-1)], dim=-1).contiguous()
        gathered = torch.empty(world, B * T * H, C + 1, dtype=torch.float32, device=o.device)
        dist.all_gather_into_tensor(gathered, packed, group=group)
        parts_o = gathered[..., :C].contiguous()
        parts_s = gathered[..., C].contiguous()
    else:
        parts_o, parts_s = o, s
    merged, merged_lse = merge(parts_o, parts_s, H, sink)
    return merged.reshape(B, T, H, C), merged_lse.reshape(B, T, H)
