"""CPU restatement of the gradients of WPT's MQA attention, in numpy.

TEST INFRASTRUCTURE ONLY (the checker): only `tests/`, `__graft_entry__.smoke()`
and the CPU legs of `bench.py` may import it; the product package never does.

Follows the reference's backward passes (paths relative to the reference
repository, packages/wpt-model/src/wpt_model/):

    exact_backward    pytorch_kernels.py:123-139 (_Exact.backward)
    rows_backward     pytorch_kernels.py:189-210 (_Sparse.backward), over
                      each query's rows (B, T, R), -1 masked, with the sink
    sparse_backward   the rows of sparse_attention (:213-217): chosen rows
                      then the last `window` rows (:149-153)
    window_backward   attention.py:85-107's layout (window_attention), whose
                      gradient the reference leaves to autograd; the same
                      formulas over its visible rows

The formulas, for one query and head with softmax weights p_n over the rows
it reads (the sink, if any, only in the denominator):

    delta   = sum_c d_out[c] * out[c]          (= sum_n p_n dp_n)
    dp_n    = d_out . v_n
    dz_n    = p_n (dp_n - delta) * scale
    dq      = sum_n dz_n k_n;   dk_n += dz_n q;   dv_n += p_n d_out
    d_sink  = -exp(sink - lse) * delta         (summed over queries)

p_n is recomputed from the saved log-sum-exp (p_n = exp(z_n - lse)), as the
reference does. Arithmetic is float64 by default.
"""

import numpy as np

from .attention import window_rows

NEG_INF = -np.inf


def exact_backward(q, k, v, positions, out, lse, d_out, scale, dtype=np.float64):
    """Gradients (dq, dk, dv) of causal MQA attention by positions: a query
    at position p read rows 0 .. min(p, N - 1); lse (B, T, H) is the
    forward pass's log-sum-exp, out its output."""
    q, k, v, out, d_out = (np.asarray(x, dtype) for x in (q, k, v, out, d_out))
    lse = np.asarray(lse, dtype)
    positions = np.asarray(positions, np.int64)
    B, T, H, c = q.shape
    N = k.shape[1]
    delta = (d_out * out).sum(-1)                                      # (B, T, H)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    rows = np.arange(N)
    step = max(1, (1 << 22) // max(1, H * N))
    for b in range(B):
        for t0 in range(0, T, step):
            part = slice(t0, min(T, t0 + step))
            R = part.stop - part.start
            z = (q[b, part].reshape(R * H, c) @ k[b].T).reshape(R, H, N) * dtype(scale)
            seen = rows[None, :] <= positions[b, part][:, None]              # (R, N)
            p = np.where(seen[:, None, :], np.exp(z - lse[b, part][..., None]), 0.0)
            dp = (d_out[b, part].reshape(R * H, c) @ v[b].T).reshape(R, H, N)
            dz = p * (dp - delta[b, part][..., None]) * dtype(scale)
            dq[b, part] = (dz.reshape(R * H, N) @ k[b]).reshape(R, H, c)
            dk[b] += dz.reshape(R * H, N).T @ q[b, part].reshape(R * H, c)
            dv[b] += p.reshape(R * H, N).T @ d_out[b, part].reshape(R * H, c)
    return dq, dk, dv


def rows_backward(q, k, v, sink, rows, out, lse, d_out, scale, dtype=np.float64):
    """Gradients (dq, dk, dv, d_sink) of attention of each query over its
    rows (B, T, R) (-1 masked) with sink (H,) in each head's denominator."""
    q, k, v, out, d_out = (np.asarray(x, dtype) for x in (q, k, v, out, d_out))
    lse = np.asarray(lse, dtype)
    sink = np.asarray(sink, dtype)
    rows = np.asarray(rows, np.int64)
    B, T, H, c = q.shape
    delta = (d_out * out).sum(-1)                                      # (B, T, H)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    safe = np.clip(rows, 0, None)
    for b in range(B):
        keys, vals = k[b][safe[b]], v[b][safe[b]]                      # (T, R, c)
        z = np.einsum("thc,trc->thr", q[b], keys) * dtype(scale)
        live = (rows[b] >= 0)[:, None, :]
        p = np.where(live, np.exp(z - lse[b][..., None]), 0.0)         # (T, H, R)
        dp = np.einsum("thc,trc->thr", d_out[b], vals)
        dz = p * (dp - delta[b][..., None]) * dtype(scale)
        dq[b] = np.einsum("thr,trc->thc", dz, keys)
        gk = np.einsum("thr,thc->trc", dz, q[b])                       # each (query, row) pair's share
        gv = np.einsum("thr,thc->trc", p, d_out[b])
        flat = safe[b].reshape(-1)
        mask = (rows[b] >= 0).reshape(-1, 1)
        np.add.at(dk[b], flat, gk.reshape(-1, c) * mask)
        np.add.at(dv[b], flat, gv.reshape(-1, c) * mask)
    d_sink = -(np.exp(sink[None, None, :] - lse) * delta).sum((0, 1))
    return dq, dk, dv, d_sink


def sparse_backward(q, k, v, sink, idx, positions, out, lse, d_out, scale, window, dtype=np.float64):
    """Gradients of sparse_attention: each query's chosen rows idx (B, T, K)
    (-1 for none) and its last `window` rows, concatenated."""
    N = np.asarray(k).shape[1]
    rows = np.concatenate([np.asarray(idx, np.int64), window_rows(positions, window, N)], -1)
    return rows_backward(q, k, v, sink, rows, out, lse, d_out, scale, dtype)


def window_backward(q, k, v, sink, positions, out, lse, d_out, scale, window, dtype=np.float64):
    """Gradients of window_attention's layout: k, v (B, window - 1 + T, c),
    query t reads table rows t .. t + window - 1 not before the text."""
    B, T = np.asarray(q).shape[:2]
    positions = np.broadcast_to(np.asarray(positions, np.int64), (B, T))
    t = np.arange(T)
    j = t[:, None] + np.arange(window)[None, :]
    back = (t[:, None] + window - 1) - j
    rows = np.where(positions[:, :, None] - back[None] >= 0, j[None], -1)
    return rows_backward(q, k, v, sink, rows, out, lse, d_out, scale, dtype)
