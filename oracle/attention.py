"""CPU restatement of WPT's MQA attention operations, in numpy.

TEST INFRASTRUCTURE ONLY. This module is the checker: only `tests/`,
`__graft_entry__.smoke()` and the CPU legs of `bench.py` (`cpu_baseline`,
`--impl reference`) may import it. The product path (`wpt_b200`) never
calls it and has no CPU fallback.

Every function restates the reference's algorithm from its source and cites
the lines it follows (paths relative to the reference repository):

    exact_attention   packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-121,142-146
                      (selection :112-117, column count chosen_columns :73-77)
    sparse_attention  pytorch_kernels.py:149-153,171-187,213-217
    window_attention  packages/wpt-model/src/wpt_model/attention.py:85-107
    dense_attention   attention.py:74-82 (used for the tree-masked verification)
    drafter_attention packages/wpt-model/src/wpt_model/drafter.py:141-151,
                      its visible mask :189-195

Differences from the reference that are deliberate and harmless:
  * arithmetic is float64 by default (the reference computes in float32);
    `dtype=np.float32` reproduces the reference's precision for timing;
  * the log-sum-exp is returned, not only saved for the backward pass
    (pytorch_kernels.py:109 computes it, :118 saves it);
  * top-k ties: the reference takes "whichever row topk returns first"
    (pytorch_kernels.py:31-32), this takes whichever argpartition returns;
    tests compare choices up to ties, as the reference's own tests do
    (tests/test_kernels.py:175-180).
"""

import numpy as np

NEG_INF = -np.inf


def chosen_columns(top_k, window, N):
    """pytorch_kernels.py:73-77: columns of the chosen rows for a table of N rows."""
    return max(0, min(top_k, N - window))


def _logsumexp(z, axis=-1):
    m = np.max(z, axis=axis, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    s = np.sum(np.exp(z - m_safe), axis=axis, keepdims=True)
    with np.errstate(divide="ignore"):
        return np.squeeze(np.log(s) + m_safe, axis=axis)


def _query_block(H, N, budget=1 << 24):
    return max(1, budget // max(1, H * N))


def exact_attention(q, k, v, positions, scale, top_k, window, dtype=np.float64):
    """Causal MQA attention by positions, plus each query's top_k rows.

    q (B, T, H, c); k, v (B, N, c); positions (B, T) int, each query's row:
    a query at position p reads rows 0..min(p, N - 1) (pytorch_kernels.py:18-26,
    66-70). Returns (out (B, T, H, c), lse (B, T, H), chosen (B, T, K) int64,
    -1 padded), K = chosen_columns(top_k, window, N). A row's score is its
    largest log-weight over the heads (:113); rows at least `window` tokens
    back compete (:114-115); -inf scores become -1 (:117).
    """
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    positions = np.asarray(positions, np.int64)
    B, T, H, c = q.shape
    N = k.shape[1]
    K = chosen_columns(top_k, window, N)
    out = np.empty((B, T, H, c), dtype)
    lse = np.empty((B, T, H), dtype)
    chosen = np.full((B, T, K), -1, np.int64)
    rows = np.arange(N)
    step = _query_block(H, N)
    for b in range(B):
        for t0 in range(0, T, step):
            part = slice(t0, min(T, t0 + step))
            p = positions[b, part]                                   # (R,)
            z = np.einsum("rhc,nc->rhn", q[b, part], k[b]) * dtype(scale)
            z = np.where(rows[None, None, :] > p[:, None, None], NEG_INF, z)
            l = _logsumexp(z)                                        # (R, H)
            lse[b, part] = l
            w = np.exp(z - l[..., None])
            out[b, part] = np.einsum("rhn,nc->rhc", w, v[b])
            if K:
                score = (z - l[..., None]).max(axis=1)               # (R, N)
                near = rows[None, :] > (p[:, None] - window)
                score = np.where(near, NEG_INF, score)
                take = min(K, N)
                idx = np.argpartition(-score, take - 1, axis=-1)[:, :take]
                best = np.take_along_axis(score, idx, -1)
                chosen[b, part, :take] = np.where(best == NEG_INF, -1, idx)
    return out, lse, chosen


def range_attention(q, k, v, positions, scale, window=0, sink=None, dtype=np.float64):
    """Attention over contiguous rows, the exact path (pytorch_kernels.py
    :98-121, no choice) and the window path (sparse_attention with no chosen
    rows, :171-187 over the rows of :149-153) in one: query at position p
    reads rows max(0, p - window + 1) .. min(p, N - 1) (every row up to p when
    window is 0), sink (H,) or None in each head's denominator. Blocks of
    queries go through matrix products (BLAS), so this is also the timed CPU
    baseline. Returns (out, lse)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    positions = np.asarray(positions, np.int64)
    B, T, H, c = q.shape
    N = k.shape[1]
    out = np.empty((B, T, H, c), dtype)
    lse = np.empty((B, T, H), dtype)
    step = max(1, (1 << 22) // max(1, H * (window if window else N)))
    for b in range(B):
        for t0 in range(0, T, step):
            part = slice(t0, min(T, t0 + step))
            p = positions[b, part]
            hi = np.minimum(p, N - 1)
            lo = np.maximum(p - window + 1, 0) if window else np.zeros_like(p)
            a, e = int(lo.min()), int(hi.max()) + 1
            R = len(p)
            if e <= a:
                out[b, part] = 0
                lse[b, part] = -np.inf if sink is None else np.asarray(sink, dtype)[None, :]
                continue
            rows = np.arange(a, e)
            z = (q[b, part].reshape(R * H, c) @ k[b, a:e].T).reshape(R, H, e - a) * dtype(scale)
            seen = (rows[None, :] >= lo[:, None]) & (rows[None, :] <= hi[:, None])
            z = np.where(seen[:, None, :], z, NEG_INF)
            l = _logsumexp(z)
            if sink is not None:
                l = np.logaddexp(l, np.asarray(sink, dtype)[None, :])
            lse[b, part] = l
            w = np.exp(z - l[..., None])
            out[b, part] = (w.reshape(R * H, e - a) @ v[b, a:e]).reshape(R, H, c)
    return out, lse


def window_rows(positions, window, N):
    """pytorch_kernels.py:149-153: (B, T, window) each query's last window
    rows, -1 before the text and past the table."""
    positions = np.asarray(positions, np.int64)
    rows = positions[..., None] - window + 1 + np.arange(window)
    return np.where((rows < 0) | (rows >= N), -1, rows)


def sparse_over_rows(q, k, v, sink, rows, scale, dtype=np.float64):
    """pytorch_kernels.py:171-187: attention of each query over its rows
    (B, T, R) (-1 masked), sink (H,) in every head's denominator. Returns
    (out, lse)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    sink = np.asarray(sink, dtype)
    rows = np.asarray(rows, np.int64)
    B, T, H, c = q.shape
    safe = np.clip(rows, 0, None)
    out = np.empty((B, T, H, c), dtype)
    lse = np.empty((B, T, H), dtype)
    for b in range(B):
        keys = k[b][safe[b]]                                         # (T, R, c)
        vals = v[b][safe[b]]
        z = np.einsum("thc,trc->thr", q[b], keys) * dtype(scale)
        z = np.where(rows[b][:, None, :] < 0, NEG_INF, z)
        l = np.logaddexp(_logsumexp(z), sink[None, :])               # :183
        lse[b] = l
        out[b] = np.einsum("thr,trc->thc", np.exp(z - l[..., None]), vals)
    return out, lse


def sparse_attention(q, k, v, sink, idx, positions, scale, window, dtype=np.float64):
    """pytorch_kernels.py:213-217: over each query's chosen rows idx (B, T, K)
    and its last `window` rows (concatenated, duplicates kept), with the
    sink. Returns (out, lse)."""
    N = np.asarray(k).shape[1]
    rows = np.concatenate([np.asarray(idx, np.int64), window_rows(positions, window, N)], -1)
    return sparse_over_rows(q, k, v, sink, rows, scale, dtype)


def window_attention(q, k, v, sink, positions, scale, window=128, dtype=np.float64):
    """attention.py:85-107. k, v (B, window - 1 + T, c): the window - 1 rows
    before the pass, then its own. Query t reads table rows t .. t + window - 1
    whose positions are not before the text: row j holds position
    p_t - (t + window - 1 - j), visible when that is >= 0 (:105-106).
    positions (T,) or (B, T). Returns (out, lse)."""
    q = np.asarray(q, dtype)
    B, T, H, c = q.shape
    positions = np.broadcast_to(np.asarray(positions, np.int64), (B, T))
    t = np.arange(T)
    j = t[:, None] + np.arange(window)[None, :]                      # (T, W) table rows
    back = (t[:, None] + window - 1) - j                             # distance back
    rows = np.where(positions[:, :, None] - back[None] >= 0, j[None], -1)
    return sparse_over_rows(q, k, v, sink, rows, scale, dtype)


def ancestors_mask(parents):
    """(n, n) bool: node i sees node j when j is i or one of its ancestors.
    parents[i] < i, -1 for a root (a child of the last cache row)."""
    parents = np.asarray(parents, np.int64)
    n = parents.shape[-1]
    seen = np.zeros((n, n), bool)
    for i in range(n):
        j = i
        while j >= 0:
            seen[i, j] = True
            j = int(parents[j])
    return seen


def tree_attention(q, k, v, cache_len, parents, scale, sink=None, dtype=np.float64):
    """Tree-masked verification attention, dense_attention's math
    (attention.py:74-82) with the mask of a draft tree. q (B, n, H, c): the n
    tree nodes of each row, node i's key and value at table row
    cache_len[b] + i; node i sees rows < cache_len[b] and the rows of its
    ancestors and itself. parents (n,) or (B, n). For a chain
    (parents[i] = i - 1) this equals exact_attention at positions
    cache_len + i. Returns (out, lse)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    B, n, H, c = q.shape
    cache_len = np.asarray(cache_len, np.int64).reshape(B)
    parents = np.broadcast_to(np.asarray(parents, np.int64), (B, n))
    out = np.empty((B, n, H, c), dtype)
    lse = np.empty((B, n, H), dtype)
    for b in range(B):
        L = int(cache_len[b])
        seen = ancestors_mask(parents[b])
        visible = np.concatenate([np.ones((n, L), bool), seen], 1)  # (n, L + n)
        keys, vals = k[b, :L + n], v[b, :L + n]
        z = np.einsum("ihc,jc->ihj", q[b], keys) * dtype(scale)
        z = np.where(visible[:, None, :], z, NEG_INF)
        l = _logsumexp(z)
        if sink is not None:
            l = np.logaddexp(l, np.asarray(sink, dtype)[None, :])
        lse[b] = l
        out[b] = np.einsum("ihj,jc->ihc", np.exp(z - l[..., None]), vals)
    return out, lse


def merge_partials(o, m, l, sink=None):
    """Log-sum-exp merge of split-KV partial results: o (S, ..., c) each
    split's normalised output, lse (S, ...) each split's log-sum-exp (m + log l
    in natural units). Returns (out, lse) over the union of the splits, the
    sink (broadcast over the trailing dims of lse) added to the denominator."""
    lse_s = np.asarray(m, np.float64) + np.log(np.asarray(l, np.float64))
    total = _logsumexp(lse_s, axis=0)
    if sink is not None:
        total = np.logaddexp(total, sink)
    w = np.exp(lse_s - total[None])
    return np.sum(w[..., None] * np.asarray(o, np.float64), axis=0), total


def dense_attention(q, k, v, sink, visible, scale, dtype=np.float64):
    """attention.py:74-82: q (..., Q, H, c) over k, v (..., K, c), each query
    reading the keys visible (..., Q, K) shows it, sink (H,) in each head's
    denominator. Returns (out (..., Q, H, c), lse (..., Q, H))."""
    q, k, v = (np.asarray(x, dtype) for x in (q, k, v))
    z = np.einsum("...qhc,...kc->...qhk", q, k) * dtype(scale)
    z = np.where(np.asarray(visible, bool)[..., :, None, :], z, NEG_INF)
    l = np.logaddexp(_logsumexp(z), np.asarray(sink, dtype))
    return np.einsum("...qhk,...kc->...qhc", np.exp(z - l[..., None]), v), l


def drafter_visible(lengths, count, window):
    """drafter.py:189-195: (R, count, count + window) bool over the table
    [block; context]: every place reads the whole block, and context entry j
    (position lengths - window + j) when it is not before the text and within
    `window` tokens of the place (position lengths + i)."""
    lengths = np.asarray(lengths, np.int64)
    positions = lengths[:, None] + np.arange(count)[None]
    context_positions = lengths[:, None] - window + np.arange(window)[None]
    seen = (context_positions[:, None, :] >= 0) & (context_positions[:, None, :] > positions[..., None] - window)
    return np.concatenate([np.ones((len(lengths), count, count), bool), seen], -1)


def drafter_attention(q, block, context, sink, lengths, scale, dtype=np.float64):
    """The drafter backbone's attention (drafter.py:141-151): q (R, count, H,
    c), block (R, count, 2c) and context (R, window, 2c) entries (keys then
    values), table [block; context] read through drafter_visible. Returns
    (out, lse)."""
    block, context = np.asarray(block, dtype), np.asarray(context, dtype)
    c = block.shape[-1] // 2
    table = np.concatenate([block, context], 1)
    visible = drafter_visible(lengths, block.shape[1], context.shape[1])
    return dense_attention(q, table[..., :c], table[..., c:], sink, visible, scale, dtype)
