"""Backward passes of the attention operations: the reference's own
gradient formulas (packages/wpt-model/src/wpt_model/pytorch_kernels.py
:123-139 for exact attention, :189-210 for sparse attention) evaluated with
torch on the GPU, in FP32, one block of queries at a time, from the
forward pass's saved log-sum-exp. Native backward kernels are a later step;
this keeps the module differentiable, as the reference's kernel decision
requires (kernels.py:123-144)."""

import torch

BLOCK_VALUES = 1 << 24


def _block_rows(B, H, N):
    return max(1, BLOCK_VALUES // max(1, B * H * N))


def exact_backward(q, k, v, positions, out, lse, d_out, scale):
    """pytorch_kernels.py:123-139."""
    given = (q, k, v)
    q, k, v = q.float(), k.float(), v.float()
    B, T, H, c = q.shape
    N = k.shape[1]
    d_out, out = d_out.float(), out.float()
    delta = (d_out * out).sum(-1)
    dq, dk, dv = torch.empty_like(q), torch.zeros_like(k), torch.zeros_like(v)
    rows = _block_rows(B, H, N)
    ends = positions.amax(0)
    for start in range(0, T, rows):
        part = slice(start, start + rows)
        seen = min(int(ends[part].max()) + 1, N)
        z = torch.einsum("brhc,bnc->brhn", q[:, part], k[:, :seen]) * scale
        later = torch.arange(seen, device=q.device) > positions[:, part, None]
        z = z.masked_fill(later[:, :, None], float("-inf"))
        p = (z - lse[:, part, :, None]).exp()
        dp = torch.einsum("brhc,bnc->brhn", d_out[:, part], v[:, :seen])
        dz = p * (dp - delta[:, part, :, None]) * scale
        dq[:, part] = torch.einsum("brhn,bnc->brhc", dz, k[:, :seen])
        dk[:, :seen] += torch.einsum("brhn,brhc->bnc", dz, q[:, part])
        dv[:, :seen] += torch.einsum("brhn,brhc->bnc", p, d_out[:, part])
    return tuple(g.to(x.dtype) for g, x in zip((dq, dk, dv), given))


def _gather(table, idx):
    B, N, c = table.shape
    flat = idx.clamp(min=0) + torch.arange(B, device=idx.device)[:, None, None] * N
    return table.reshape(B * N, c)[flat]


def _scatter_add(table_grad, idx, values):
    B, N, c = table_grad.shape
    flat = idx.clamp(min=0) + torch.arange(B, device=idx.device)[:, None, None] * N
    table_grad.view(B * N, c).index_add_(0, flat.reshape(-1), values.reshape(-1, c))


def sparse_backward(q, k, v, sink, rows_idx, out, lse, d_out, scale):
    """pytorch_kernels.py:189-210; rows_idx (B, T, R): the chosen rows then
    the window rows, -1 for none; lse includes the sink."""
    given = (q, k, v, sink)
    q, k, v, sink = q.float(), k.float(), v.float(), sink.float()
    B, T, H, c = q.shape
    d_out, out = d_out.float(), out.float()
    delta = (d_out * out).sum(-1)
    dq, dk, dv = torch.empty_like(q), torch.zeros_like(k), torch.zeros_like(v)
    rows = _block_rows(B, rows_idx.shape[-1], max(c, H))
    for start in range(0, T, rows):
        part = slice(start, start + rows)
        keys, values = _gather(k, rows_idx[:, part]), _gather(v, rows_idx[:, part])
        z = torch.einsum("brhc,brkc->brhk", q[:, part], keys) * scale
        z = z.masked_fill(rows_idx[:, part, None, :] < 0, float("-inf"))
        p = (z - lse[:, part, :, None]).exp()
        dp = torch.einsum("brhc,brkc->brhk", d_out[:, part], values)
        dz = p * (dp - delta[:, part, :, None]) * scale
        dq[:, part] = torch.einsum("brhk,brkc->brhc", dz, keys)
        _scatter_add(dk, rows_idx[:, part], torch.einsum("brhk,brhc->brkc", dz, q[:, part]))
        _scatter_add(dv, rows_idx[:, part], torch.einsum("brhk,brhc->brkc", p, d_out[:, part]))
    d_sink = -((sink - lse).exp() * delta).sum((0, 1))
    return tuple(g.to(x.dtype) for g, x in zip((dq, dk, dv, d_sink), given))
