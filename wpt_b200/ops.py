"""Forward operations over the C ABI (include/wpt_attn.h): tensor checks,
output and scratch allocation through torch's caching allocator, and the
choice of kernel and split count. Every function here launches CUDA
kernels of libwpt_b200.so on the current stream; none has a CPU path.

Kernel choice: queries x heads of one batch row fill the 128 rows of the
prefill kernel's tiles (tcgen05, M = 128 rows); with few queries per row
(decode, short extends) the key-stream kernel computes S^T = K Q^T with the
keys as M instead, and splits long rows over many CTAs.
"""

import math
import os

import torch

from . import _lib

LAUNCHES = [0]  # kernels this module has launched (read by bench.py around its timed region)
# key tiles per key-stream CTA when set (WPT_B200_CHUNK, read once): overrides the split heuristic
CHUNK_TILES = int(os.environ.get("WPT_B200_CHUNK", "0"))
# the prefill kernel's 2-split cluster combine (WPT_B200_PREFILL_CLUSTER=0 turns it off)
PREFILL_CLUSTER = os.environ.get("WPT_B200_PREFILL_CLUSTER", "1") != "0"


def _need_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("wpt_b200 computes on a CUDA device only; got a tensor on " + str(t.device))


_SMS = {}


def sm_count(device):
    """The streaming multiprocessors of `device`, asked of the runtime once."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    n = _SMS.get(index)
    if n is None:
        n = _SMS[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return n


def _bf16(x):
    """The kernels compute in bf16 (WPT's compute dtype under autocast,
    packages/wpt-model/src/wpt_model/layers.py:13-17). Other dtypes are
    refused rather than rounded: the reference computes in the inputs'
    dtype, so silently rounding float32 inputs would return float32
    tensors of bf16 accuracy. NotImplementedError is what the reference's
    kernel tests skip on (tests/test_kernels.py:149-154)."""
    if x.dtype != torch.bfloat16:
        raise NotImplementedError(f"wpt_b200 computes attention in bfloat16; got {x.dtype} "
                                  "(cast q, k and v to bfloat16, as WPT's autocast does)")
    return x


def _table(x):
    """A (B, N, C) table whose last dimension is contiguous, strides in
    multiples of 8 elements (16 bytes), at a 16-byte aligned address."""
    x = _bf16(x)
    sb, sn, sc = x.stride()
    ok = sc == 1 and sn % 8 == 0 and (sb % 8 == 0 or x.shape[0] == 1) and x.data_ptr() % 16 == 0
    return x if ok else x.contiguous()


def _rows(x):
    if x.dtype == torch.int64 and x.is_contiguous():
        return x
    return x.to(torch.int64).contiguous()


def _splits_for(ctas, tiles, sms):
    """Split count for a grid of `ctas` work items over `tiles` key tiles
    each: the persistent kernel runs the ctas * splits items in waves of
    one per SM, so the estimate is waves x (tiles per item + about 2 tiles'
    worth of per-item cost), plus half a tile per split for the merge; the
    cheapest count up to 32 (never more than the tiles) wins."""
    if ctas >= sms or tiles <= 1:
        return 1
    best, best_cost = 1, None
    for s in range(1, min(tiles, 32) + 1):
        cost = math.ceil(ctas * s / sms) * (tiles / s + 2) + (0.5 * s if s > 1 else 0.0)
        if best_cost is None or cost < best_cost:
            best, best_cost = s, cost
    return best


def prefill_forward(q, k, v, positions, scale, window=0, floor=None, tree_bits=None, tree_base=None, sink=None,
                    splits=None):
    """(out (B, T, H, C) bf16, lse (B, T, H) fp32) from the tcgen05 prefill
    kernel: each query reads rows max(0, p - window + 1, floor) ..
    min(p, N - 1) of k and v, p its position; tree_bits/tree_base give the
    tree mask; sink (H,) joins each head's denominator."""
    _need_cuda(q, k, v, positions, floor, tree_bits, tree_base, sink)
    q = _bf16(q).contiguous()
    k, v = _table(k), _table(v)
    B, T, H, C = q.shape
    N = k.shape[1]
    positions = _rows(positions)
    floor = None if floor is None else _rows(floor)
    if tree_bits is not None:
        tree_bits = tree_bits.to(torch.int64).contiguous()
        tree_base = _rows(tree_base)
    if sink is not None:
        sink = sink.float().contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B, T, H, dtype=torch.float32, device=q.device)
    TQ = max(1, 128 // H)
    if splits is None:
        tiles = window // 128 + 2 if window else (N + 127) // 128
        splits = _splits_for(B * math.ceil(T / (2 * TQ)), tiles, sm_count(q.device))  # one item per tile pair
    part_o = part_lse = None
    # two splits with one work item per SM: the pair's splits combine as one
    # 2-CTA cluster in shared memory (no partials, no merge launch)
    cluster = (splits == 2 and PREFILL_CLUSTER and 2 * B * math.ceil(T / (2 * TQ)) <= sm_count(q.device))
    if splits > 1 and not cluster:
        part_o = torch.empty(splits, B * T * H, C, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(splits, B * T * H, dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().wpt_attn_prefill(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        _lib.ptr(positions), _lib.ptr(floor), _lib.ptr(tree_bits), _lib.ptr(tree_base), _lib.ptr(sink),
        _lib.ptr(out), _lib.ptr(lse), _lib.ptr(part_o), _lib.ptr(part_lse), int(splits),
        B, T, H, C, N, int(window), float(scale), _lib.stream(q.device)))
    LAUNCHES[0] += 1 + (splits > 1 and not cluster)
    return out, lse


def _stream_shape(T, H, gather):
    """(columns per CTA, queries per CTA) of the key-stream kernel, as the C
    launcher derives them."""
    cols = H if gather else min(T * H, 64)
    ncol = 16 if cols <= 16 else 32 if cols <= 32 else 64
    return ncol, (1 if gather else ncol // H)


def uses_stream(T, H, C):
    """Whether the key-stream kernel computes this shape (few queries per row)."""
    return C == 128 and H <= 64 and T * H <= 64


_PLAN_CACHE = {}


def _stream_plan(B, T, H, N, K, window, gather, sms, chunk_tiles=None):
    """(chunk_tiles, splits, cluster) of a key-stream call: each query
    group's key slots are cut into chunks of chunk_tiles key tiles, one CTA
    per chunk; cluster: the splits of a group combine in shared memory as one
    thread-block cluster (2 to 8 splits on a grid of one wave) instead of
    through partials and a merge kernel. Remembered per shape (a decode loop
    asks the same question every step)."""
    key = (B, T, H, N, K, window, gather, sms, chunk_tiles)
    plan = _PLAN_CACHE.get(key)
    if plan is None:
        if len(_PLAN_CACHE) > 4096:
            _PLAN_CACHE.clear()
        plan = _PLAN_CACHE[key] = _stream_plan_for(B, T, H, N, K, window, gather, sms, chunk_tiles)
    return plan


def _stream_plan_for(B, T, H, N, K, window, gather, sms, chunk_tiles):
    _, TQ = _stream_shape(T, H, gather)
    groups = B * math.ceil(T / TQ)
    if gather:
        slots = K + max(window, 0)
    else:
        slots = min(N, window + TQ - 1) if window > 0 else N
    tiles = max(1, math.ceil(slots / 128))
    if chunk_tiles is None:
        chunk_tiles = CHUNK_TILES
    auto = not chunk_tiles
    if not chunk_tiles and gather:
        # every query gathers exactly `tiles` tiles: its slots split so that
        # the grid is about one CTA per SM
        chunk_tiles = math.ceil(tiles / max(1, sms // groups))
    elif not chunk_tiles:
        # at least 16 key tiles per CTA (a CTA's start-up costs about as much
        # as streaming a few tiles), more when that still gives two CTAs per
        # SM for rows of the table's full length (most rows are shorter)
        chunk_tiles = max(min(16, tiles), 16 * math.ceil(tiles * groups / (2 * sms) / 16))
        if tiles >= 64 and 2 * math.ceil(tiles / chunk_tiles) * groups < sms:
            # a few long rows (a GPU's shard of a long-context decode) that
            # would leave most SMs idle: about one CTA per SM
            chunk_tiles = max(2, math.ceil(tiles * groups / sms))
    chunk_tiles = max(1, min(int(chunk_tiles), tiles))
    splits = math.ceil(tiles / chunk_tiles)
    if auto and splits == 1 and tiles >= 2 and 2 * groups <= sms:
        # short rows (window rows) on fewer CTAs than SMs: each row's tiles
        # over a cluster of up to 8 CTAs, still one wave
        splits = min(8, tiles, sms // groups)
        chunk_tiles = math.ceil(tiles / splits)
        splits = math.ceil(tiles / chunk_tiles)
    return chunk_tiles, splits, 1 < splits <= 8 and groups * splits <= sms


def stream_forward(q, k, v, positions, scale, window=0, floor=None, idx=None, sink=None, chunk_tiles=None):
    """(out (B, T, H, C) bf16, lse (B, T, H) fp32) from the key-stream
    kernel. Range mode (idx None): as prefill_forward. Gather mode: each
    query reads rows idx[b, t, :] (-1 for none) and its last `window` rows."""
    _need_cuda(q, k, v, positions, floor, idx, sink)
    q = _bf16(q).contiguous()
    k, v = _table(k), _table(v)
    B, T, H, C = q.shape
    N = k.shape[1]
    positions = _rows(positions)
    floor = None if floor is None else _rows(floor)
    gather = idx is not None
    K = 0
    if gather:
        idx = _rows(idx)
        K = idx.shape[-1]
    if sink is not None and (sink.dtype != torch.float32 or not sink.is_contiguous()):
        sink = sink.float().contiguous()
    dev = q.device
    chunk_tiles, splits, cluster = _stream_plan(B, T, H, N, K, window, gather, sm_count(dev), chunk_tiles)
    out = torch.empty_like(q)
    lse = torch.empty((B, T, H), dtype=torch.float32, device=dev)
    part_o = part_lse = None
    if splits > 1 and not cluster:
        part_o = torch.empty((splits, B * T * H, C), dtype=torch.float32, device=dev)
        part_lse = torch.empty((splits, B * T * H), dtype=torch.float32, device=dev)
    ks, vs = k.stride(), v.stride()
    _lib.check(_lib.lib().wpt_attn_decode(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), ks[0], ks[1], vs[0], vs[1],
        positions.data_ptr(), _lib.ptr(floor), _lib.ptr(idx), K, _lib.ptr(sink), out.data_ptr(), lse.data_ptr(),
        _lib.ptr(part_o), _lib.ptr(part_lse), splits, chunk_tiles, B, T, H, C, N, int(window), float(scale),
        _lib.stream(dev)))
    LAUNCHES[0] += 1 + (splits > 1 and not cluster)
    return out, lse


def partials_plan(q_shape, N, device, window=0):
    """(splits, chunk_tiles) the key-stream kernel uses for partials of a
    (B, T, H, C) query block over N keys: at least two splits."""
    B, T, H, C = q_shape
    chunk_tiles, splits, _ = _stream_plan(B, T, H, N, 0, window, False, sm_count(device), None)
    if splits < 2:  # at least two partials, so that the caller always has partials to merge
        chunk_tiles, splits = max(1, math.ceil(chunk_tiles / 2)), 2
    return splits, chunk_tiles


def stream_partials(q, k, v, positions, scale, window=0, into=None, splits=None):
    """The key-stream kernel's split partials without the merge: (part_o
    (S, B*T*H, C) fp32, each split's output normalised by its own sum;
    part_lse (S, B*T*H) fp32, the natural log of that sum, -inf for a split
    with no visible row), S >= 2 (partials_plan). For callers that merge
    them with partials computed elsewhere (merge_partials, merge_groups),
    e.g. on the other GPUs of a long row. into=(part_o, part_lse): write
    there (contiguous fp32 of those shapes) instead of new tensors.
    splits: this many partials (>= 2) instead of partials_plan's count, the
    keys cut into that many equal chunks of whole tiles (splits with no key
    give -inf log-sums): ranks whose shards differ in length then still
    produce chunks of one layout."""
    _need_cuda(q, k, v, positions)
    q = _bf16(q).contiguous()
    k, v = _table(k), _table(v)
    B, T, H, C = q.shape
    N = k.shape[1]
    positions = _rows(positions)
    if splits is None:
        splits, chunk_tiles = partials_plan(q.shape, N, q.device, window)
    else:
        splits = max(2, int(splits))
        slots = min(N, window + 63) if window > 0 else N
        chunk_tiles = max(1, math.ceil(math.ceil(slots / 128) / splits))
    if into is None:
        part_o = torch.empty(splits, B * T * H, C, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(splits, B * T * H, dtype=torch.float32, device=q.device)
    else:
        part_o, part_lse = into
        if (part_o.shape != (splits, B * T * H, C) or part_lse.shape != (splits, B * T * H)
                or not part_o.is_contiguous() or not part_lse.is_contiguous()):
            raise ValueError("stream_partials: `into` does not match partials_plan's shapes")
    _lib.check(_lib.lib().wpt_attn_decode(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        _lib.ptr(positions), None, None, 0, None, None, None, _lib.ptr(part_o), _lib.ptr(part_lse), splits,
        chunk_tiles, B, T, H, C, N, int(window), float(scale), _lib.stream(q.device)))
    LAUNCHES[0] += 1
    return part_o, part_lse


def merge_partial(part_o, part_lse, out_o=None, out_lse=None):
    """Merge of S split partials (part_o (S, rows, C), part_lse (S, rows)
    fp32) into one partial of the same kind, no sink: (out_o (rows, C) fp32,
    the splits' output normalised by their common sum; out_lse (rows,), its
    log). out_o / out_lse: write there (contiguous fp32) instead."""
    _need_cuda(part_o, part_lse, out_o, out_lse)
    S, rows, C = part_o.shape
    out_o = torch.empty(rows, C, dtype=torch.float32, device=part_o.device) if out_o is None else out_o
    out_lse = torch.empty(rows, dtype=torch.float32, device=part_o.device) if out_lse is None else out_lse
    _lib.check(_lib.lib().wpt_attn_merge_partial(_lib.ptr(part_o), _lib.ptr(part_lse), S, rows, rows, C,
                                                 _lib.ptr(out_o), _lib.ptr(out_lse), _lib.stream(part_o.device)))
    LAUNCHES[0] += 1
    return out_o, out_lse


def merge_groups(parts, per, rows, H, C, sink=None, out=None, lse=None):
    """Merge of partials gathered side by side: parts (G, group_floats) fp32,
    chunk g = `per` splits' output partials (per, rows, C) then their
    log-sums (per, rows). Returns (out (rows, C) bf16, lse (rows,) fp32)."""
    _need_cuda(parts, sink)
    G, group_floats = parts.shape
    if sink is not None:
        sink = sink.float().contiguous()
    out = torch.empty(rows, C, dtype=torch.bfloat16, device=parts.device) if out is None else out
    lse = torch.empty(rows, dtype=torch.float32, device=parts.device) if lse is None else lse
    _lib.check(_lib.lib().wpt_attn_merge_groups(_lib.ptr(parts), G, per, rows, group_floats, H, C, _lib.ptr(sink),
                                                _lib.ptr(out), _lib.ptr(lse), _lib.stream(parts.device)))
    LAUNCHES[0] += 1
    return out, lse


def exchange(part_o, part_lse, peers, world, rank, H, sink=None):
    """The long row's combine across GPUs in one kernel (wpt_attn_exchange):
    this rank's split partials (part_o (S, rows, C), part_lse (S, rows)
    fp32) are merged, stored into every rank's exchange buffer (peers: a
    ctypes array of the world buffers as mapped here), and, once every
    rank's result of the same call has landed, merged with the sink into
    (out (rows, C) bf16, lse (rows,) fp32)."""
    _need_cuda(part_o, part_lse, sink)
    S, rows, C = part_o.shape
    if sink is not None:
        sink = sink.float().contiguous()
    out = torch.empty(rows, C, dtype=torch.bfloat16, device=part_o.device)
    lse = torch.empty(rows, dtype=torch.float32, device=part_o.device)
    _lib.check(_lib.lib().wpt_attn_exchange(_lib.ptr(part_o), _lib.ptr(part_lse), S, rows, H, C, _lib.ptr(sink),
                                            peers, world, rank, _lib.ptr(out), _lib.ptr(lse),
                                            _lib.stream(part_o.device)))
    LAUNCHES[0] += 1
    return out, lse


def attention_forward(q, k, v, positions, scale, window=0, floor=None, sink=None):
    """Range attention by the kernel that suits the shape: the key-stream
    kernel for few queries per row, the prefill kernel otherwise."""
    B, T, H, C = q.shape
    if uses_stream(T, H, C):
        return stream_forward(q, k, v, positions, scale, window=window, floor=floor, sink=sink)
    return prefill_forward(q, k, v, positions, scale, window=window, floor=floor, sink=sink)


def select_rows(q, k, positions, lse, scale, K, window):
    """Each query's K chosen rows (B, T, K) int64 (pytorch_kernels.py:112-117):
    the top K by max_h (q_h . k_n * scale - lse_h) among rows 0 .. p - window,
    -1 padded. lse is the forward pass's (B, T, H)."""
    _need_cuda(q, k, positions, lse)
    q = _bf16(q).contiguous()
    k = _table(k)
    B, T, H, C = q.shape
    N = k.shape[1]
    positions = _rows(positions)
    lse = lse.float().contiguous()
    chosen = torch.empty(B, T, K, dtype=torch.int64, device=q.device)
    if K == 0:
        return chosen
    ld = (N + 3) // 4 * 4
    scores = torch.empty(B * T, ld, dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().wpt_attn_topk(
        _lib.ptr(q), _lib.ptr(k), k.stride(0), k.stride(1), _lib.ptr(positions), _lib.ptr(lse), _lib.ptr(scores),
        ld, _lib.ptr(chosen), int(K), B, T, H, C, N, int(window), float(scale), _lib.stream(q.device)))
    LAUNCHES[0] += 2
    return chosen


def merge_partials(part_o, part_lse, H, sink=None, out=None, lse=None):
    """Log-sum-exp merge of split partials: part_o (S, rows, C) fp32,
    part_lse (S, rows) -> (out (rows, C) bf16, lse (rows,) fp32)."""
    _need_cuda(part_o, part_lse, sink)
    S, rows, C = part_o.shape
    part_o, part_lse = part_o.float().contiguous(), part_lse.float().contiguous()
    if sink is not None:
        sink = sink.float().contiguous()
    out = torch.empty(rows, C, dtype=torch.bfloat16, device=part_o.device) if out is None else out
    lse = torch.empty(rows, dtype=torch.float32, device=part_o.device) if lse is None else lse
    _lib.check(_lib.lib().wpt_attn_merge(_lib.ptr(part_o), _lib.ptr(part_lse), S, rows, rows, H, C, _lib.ptr(sink),
                                         _lib.ptr(out), _lib.ptr(lse), _lib.stream(part_o.device)))
    LAUNCHES[0] += 1
    return out, lse


def attention_backward(q, k, v, positions, out, lse, d_out, scale, window=0, floor=None, sink=None, idx=None,
                       f32=False):
    """Gradients of range attention (each query reads rows max(0, p - window
    + 1, floor) .. min(p, N - 1)), plus its chosen rows idx (B, T, K) when
    given (sparse attention), sink (H,) in the denominators, from the forward
    pass's out (bf16) and lse: (dq (B, T, H, C), dk, dv (B, N, C) in bf16, or
    fp32 when f32; d_sink (H,) fp32 or None). Tensor-core kernels (bwd_prep,
    bwd_kv, bwd_q, and bwd_gather for chosen rows) on the current stream."""
    _need_cuda(q, k, v, positions, out, lse, d_out, floor, sink, idx)
    q = _bf16(q).contiguous()
    k, v = _table(k), _table(v)
    B, T, H, C = q.shape
    N = k.shape[1]
    positions = _rows(positions)
    floor = None if floor is None else _rows(floor)
    K = 0
    if idx is not None and idx.shape[-1] > 0:
        idx = _rows(idx)
        K = idx.shape[-1]
    else:
        idx = None
    out = _bf16(out).contiguous()
    d_out = d_out.to(torch.bfloat16).contiguous()
    lse = lse.float().contiguous()
    if sink is not None:
        sink = sink.float().contiguous()
    wide = f32 or K > 0  # chosen rows are added by fp32 atomics
    dtype = torch.float32 if wide else torch.bfloat16
    dq = torch.empty(B, T, H, C, dtype=dtype, device=q.device)
    dk = torch.empty(B, N, C, dtype=dtype, device=q.device)
    dv = torch.empty(B, N, C, dtype=dtype, device=q.device)
    d_sink = None if sink is None else torch.empty(H, dtype=torch.float32, device=q.device)
    nbytes = _lib.lib().wpt_attn_backward_scratch_bytes(B, T, H, C, N)
    if nbytes == 0:
        raise NotImplementedError(f"attention backward for B={B} T={T} H={H} C={C} N={N}: the kernels take "
                                  "head width 128 and up to 128 heads")
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _lib.check(_lib.lib().wpt_attn_backward(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        _lib.ptr(positions), _lib.ptr(floor), _lib.ptr(idx), K, _lib.ptr(sink), _lib.ptr(out), _lib.ptr(lse),
        _lib.ptr(d_out), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(d_sink), _lib.ptr(scratch),
        1 if wide else 0, B, T, H, C, N, int(window), float(scale), _lib.stream(q.device)))
    LAUNCHES[0] += 3 + (sink is not None) + (K > 0)
    if wide and not f32:
        dq, dk, dv = (to_bf16(x) for x in (dq, dk, dv))
    return dq, dk, dv, d_sink


def to_bf16(x):
    """A contiguous fp32 tensor rounded to bf16 by the library's kernel."""
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.lib().wpt_f32_to_bf16(_lib.ptr(x), x.numel(), _lib.ptr(y), _lib.stream(x.device)))
    LAUNCHES[0] += 1
    return y


def cache_append(held, new, first, counts, need=None):
    """The generation cache's entries write (cache.py:110-128): row b's new
    entries new[b, :counts[b]] go to rows first[b] .. of the held table
    (B, capacity, ...), grown to max(need, 2 * capacity) rows (zeros) when
    `need` rows do not fit, as the reference grows it. Returns (held, the
    first `need` rows of it). need = max_b(first[b] + counts[b]) is what the
    reference reads back to the host; a caller that knows it (its own count
    of each row's tokens) passes it, and the call then launches one kernel
    and synchronises nothing."""
    _need_cuda(new, first, counts)
    B, n = new.shape[:2]
    first, counts = _rows(first), _rows(counts)
    if need is None:
        need = int((first + counts).max()) if B else 0  # the reference's own host read
    if held is None:
        held = new.new_zeros((B, 0) + tuple(new.shape[2:]))
    cap = held.shape[1]
    if need > cap:
        held = torch.cat([held, held.new_zeros((B, max(need, 2 * cap) - cap) + tuple(held.shape[2:]))], 1)
    held = held.to(new.dtype)
    if B and n:
        es = new.element_size()
        row_bytes = es * math.prod(new.shape[2:])
        if new.stride(-1) != 1 or (new.dim() > 3 and not new[0, 0].is_contiguous()):
            new = new.contiguous()
        _lib.check(_lib.lib().wpt_cache_append(
            _lib.ptr(new), new.stride(0) * es, new.stride(1) * es, _lib.ptr(held), held.stride(0) * es,
            held.stride(1) * es, _lib.ptr(first), _lib.ptr(counts), B, n, row_bytes, held.shape[1],
            _lib.stream(new.device)))
        LAUNCHES[0] += 1
    return held, held[:, :need]


def tree_bits(parents, B, base=None):
    """(n,) or (B, n) int64 parent indices on the GPU (-1 for a root,
    parents[i] < i) -> ((B, n) int64 ancestor masks: bit j of node i is set
    when node j is i or one of its ancestors; (B, n) positions base[b] + i
    when base (B,) is given, else None). One small kernel on the current
    stream: no host synchronisation, so verification can be captured in a
    CUDA graph. A parent that is not before its child ends that node's walk
    (the mask then holds the nodes met so far)."""
    n = parents.shape[-1]
    if n > 64:
        raise NotImplementedError(f"a tree of {n} nodes: the kernels take up to 64")
    _need_cuda(parents, base)
    par = _rows(parents)
    stride = 0 if par.dim() == 1 else n
    if stride and par.shape != (B, n):
        par = par.expand(B, n).contiguous()
    bits = torch.empty(B, n, dtype=torch.int64, device=par.device)
    positions = None if base is None else torch.empty(B, n, dtype=torch.int64, device=par.device)
    _lib.check(_lib.lib().wpt_tree_bits(_lib.ptr(par), stride, B, n, _lib.ptr(bits), _lib.ptr(base),
                                        _lib.ptr(positions), _lib.stream(par.device)))
    LAUNCHES[0] += 1
    return bits, positions


def head_scores(h, weight, round_bf16=True):
    """(R, V) fp32 scores = h (R, D) @ weight (V, D)^T from the tcgen05 head
    kernel (model.py:267,471: the output head, bias-free; with round_bf16 each
    score is rounded to bf16 first, as the reference's autocast head returns
    it). h and weight bf16 with contiguous rows; D a multiple of 64."""
    _need_cuda(h, weight)
    if h.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise NotImplementedError("the head kernel takes bf16 hidden states and weights")
    if h.stride(-1) != 1:
        h = h.contiguous()
    if weight.stride(-1) != 1:
        weight = weight.contiguous()
    R, D = h.shape
    V = weight.shape[0]
    if weight.shape[1] != D:
        raise ValueError(f"hidden width {D} against a head weight of {tuple(weight.shape)}")
    scores = torch.empty(R, V, dtype=torch.float32, device=h.device)
    _lib.check(_lib.lib().wpt_head_scores(h.data_ptr(), h.stride(0), weight.data_ptr(), weight.stride(0), R, D, V,
                                          1 if round_bf16 else 0, scores.data_ptr(), _lib.stream(h.device)))
    LAUNCHES[0] += math.ceil(R / 128)
    return scores


def accept(scores, drafted, q, uniforms, resample, temperature=1.0, top_k=None, lengths=None):
    """The acceptance step for R rows (wpt_inference/__init__.py:173-179,
    210-222) with explicit draws: returns (tokens (R, n + 1) int64, -1
    padded: each row's kept drafts then its drawn token; accepted (R,)
    int64: the drafts each row kept)."""
    _need_cuda(scores, drafted, q, uniforms, resample, lengths)
    scores = scores.float().contiguous()
    R, n1, V = scores.shape
    n = n1 - 1
    drafted = drafted.to(torch.int64).contiguous()
    q = q.float().contiguous()
    uniforms = uniforms.float().contiguous()
    resample = resample.float().reshape(R).contiguous()
    lengths = None if lengths is None else lengths.to(torch.int64).contiguous()
    scratch = torch.empty(_lib.lib().wpt_accept_scratch_bytes(R, n, V), dtype=torch.uint8, device=scores.device)
    tokens = torch.empty(R, n + 1, dtype=torch.int64, device=scores.device)
    accepted = torch.empty(R, dtype=torch.int64, device=scores.device)
    _lib.check(_lib.lib().wpt_accept(
        _lib.ptr(scores), _lib.ptr(drafted), _lib.ptr(q), _lib.ptr(uniforms), _lib.ptr(resample), _lib.ptr(lengths),
        _lib.ptr(scratch), _lib.ptr(tokens), _lib.ptr(accepted), R, n, V, float(temperature),
        0 if top_k is None else int(top_k), _lib.stream(scores.device)))
    LAUNCHES[0] += 2
    return tokens, accepted
