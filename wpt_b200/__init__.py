"""wpt_b200: WPT's attention hot path on B200 (sm_100a).

A kernel-form module with the reference's contract (packages/wpt-model/src/
wpt_model/pytorch_kernels.py:18-26; chosen by kernels.py:86-112), so that

    from wpt_model import kernels
    import wpt_b200
    kernels._kernels, kernels._form = wpt_b200, "b200"

makes WPT's exact and sparse layers run on these kernels. It exposes

    NAME
    exact_attention(q, k, v, positions, scale, top_k, window) -> (out, chosen)
    sparse_attention(q, k, v, sink, idx, positions, scale, window) -> out
    window_attention(q, k, v, sink, positions, scale)   (attention.py:85-107)
    drafter_attention(q, block, context, sink, lengths, scale)   (drafter.py:141-151)
    tree_attention(q, k, v, cache_len, parents, scale, sink=None) -> (out, lse)
    accept(scores, drafted, q, uniforms, resample, temperature, top_k)

with the reference's argument meanings, dtypes, -1 conventions and errors.
Forward passes run hand-written CUDA kernels (libwpt_b200.so, C ABI in
include/wpt_attn.h); there is no CPU path and no other backend: a missing
library or a CPU tensor raises. The backward passes (exact, sparse and
window attention; pytorch_kernels.py:123-139,189-210) are hand-written
tensor-core kernels too, from the saved output and log-sum-exp.
"""

import torch

from . import ops
from ._lib import LibraryMissing, device_status  # noqa: F401

NAME = "B200"
WINDOW = 128  # attention.py:53, what window_attention reads when not given a window


def chosen_columns(top_k, window, N):
    """pytorch_kernels.py:73-77."""
    return max(0, min(top_k, N - window))


def _positions(positions, B):
    """positions (T,) or (B, T) -> (B, T) int64, contiguous (kernels.py:155-157)."""
    if positions.dtype == torch.int64 and positions.dim() == 2 and positions.shape[0] == B and \
            positions.is_contiguous():
        return positions
    return positions.to(torch.int64).expand(B, -1).contiguous()


def _needs_grad(*tensors):
    """Whether autograd would record this call (grad mode on and an input
    that requires a gradient): when not, the forward runs without the
    autograd Function's bookkeeping, a few microseconds a call."""
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _bf16_only(*tensors):
    """The kernels compute in bfloat16, WPT's compute dtype under autocast
    (layers.py:13-17). The reference computes in its inputs' dtype, so
    float32 or float16 inputs are refused, not silently rounded; the
    reference's kernel tests skip on NotImplementedError
    (tests/test_kernels.py:149-154)."""
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise NotImplementedError(f"wpt_b200 computes attention in bfloat16; got {t.dtype} "
                                      "(cast q, k and v to bfloat16, as WPT's autocast does)")


# ------------------------------------------------------------ exact attention

def _exact_forward(q, k, v, positions, scale, top_k, window):
    B, T, H, c = q.shape
    positions = _positions(positions, B)
    out, lse = ops.attention_forward(q, k, v, positions, scale)
    chosen = ops.select_rows(q, k, positions, lse, scale, chosen_columns(top_k, window, k.shape[1]), window)
    return out, chosen, positions, lse


class _Exact(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, positions, scale, top_k, window):
        out, chosen, positions, lse = _exact_forward(q, k, v, positions, scale, top_k, window)
        ctx.save_for_backward(q, k, v, positions, out, lse)
        ctx.scale = scale
        ctx.mark_non_differentiable(chosen)
        return out.to(q.dtype), chosen

    @staticmethod
    def backward(ctx, d_out, _d_chosen):
        q, k, v, positions, out, lse = ctx.saved_tensors
        dq, dk, dv, _ = ops.attention_backward(q, k, v, positions, out, lse, d_out, ctx.scale)
        return dq, dk, dv, None, None, None, None


def exact_attention(q, k, v, positions, scale, top_k, window):
    """pytorch_kernels.exact_attention's result: (output (B, T, H, c) in q's
    dtype, chosen rows (B, T, K) int64, -1 padded)."""
    _bf16_only(q, k, v)
    if not _needs_grad(q, k, v):
        return _exact_forward(q, k, v, positions, scale, top_k, window)[:2]
    return _Exact.apply(q, k, v, positions, scale, top_k, window)


def forward_with_lse(q, k, v, positions, scale, window=0, sink=None):
    """Forward only, with the log-sum-exp: (out bf16, lse fp32)."""
    _bf16_only(q, k, v)
    return ops.attention_forward(q, k, v, _positions(positions, q.shape[0]), scale, window=window, sink=sink)


# ----------------------------------------------------------- sparse attention

def _sparse_forward(q, k, v, sink, idx, positions, scale, window):
    B, T, H, c = q.shape
    positions = _positions(positions, B)
    if idx.shape[-1] == 0:
        out, lse = ops.attention_forward(q, k, v, positions, scale, window=window, sink=sink)
    elif ops.uses_stream(1, H, c):
        out, lse = ops.stream_forward(q, k, v, positions, scale, window=window, idx=idx, sink=sink)
    else:
        raise NotImplementedError(f"sparse attention with {H} heads of width {c}: the gather kernel takes "
                                  "head width 128 and up to 64 heads")
    return out, positions, lse


class _Sparse(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, sink, idx, positions, scale, window):
        out, positions, lse = _sparse_forward(q, k, v, sink, idx, positions, scale, window)
        ctx.save_for_backward(q, k, v, sink, idx, positions, out, lse)
        ctx.scale, ctx.window = scale, window
        return out.to(q.dtype)

    @staticmethod
    def backward(ctx, d_out):
        q, k, v, sink, idx, positions, out, lse = ctx.saved_tensors
        # the window rows by the range kernels, the chosen rows by the gather kernel
        dq, dk, dv, d_sink = ops.attention_backward(q, k, v, positions, out, lse, d_out, ctx.scale,
                                                    window=ctx.window, sink=sink, idx=idx)
        return dq, dk, dv, None if d_sink is None else d_sink.to(sink.dtype), None, None, None, None


def sparse_attention(q, k, v, sink, idx, positions, scale, window):
    """pytorch_kernels.sparse_attention's result: the output (B, T, H, c), in
    q's dtype, over each query's rows idx (B, T, K) (-1 for none) and its
    last `window` rows, with sink (H,) in each head's denominator."""
    _bf16_only(q, k, v)
    if not _needs_grad(q, k, v, sink):
        return _sparse_forward(q, k, v, sink, idx, positions, scale, window)[0]
    return _Sparse.apply(q, k, v, sink, idx, positions, scale, window)


# ----------------------------------------------------------- window attention

class _Range(torch.autograd.Function):
    """Attention of each query over the contiguous table rows max(0, p -
    window + 1, floor) .. min(p, N - 1), p its entry of `rows`, with the
    sink; backward by the library's kernels."""

    @staticmethod
    def forward(ctx, q, k, v, sink, rows, floor, scale, W):
        out, lse = ops.attention_forward(q, k, v, rows, scale, window=W, floor=floor, sink=sink)
        ctx.save_for_backward(q, k, v, sink, rows, floor, out, lse)
        ctx.scale, ctx.window = scale, W
        return out

    @staticmethod
    def backward(ctx, d_out):
        q, k, v, sink, rows, floor, out, lse = ctx.saved_tensors
        dq, dk, dv, d_sink = ops.attention_backward(q, k, v, rows, out, lse, d_out, ctx.scale, window=ctx.window,
                                                    floor=floor, sink=sink)
        return dq, dk, dv, None if d_sink is None else d_sink.to(sink.dtype), None, None, None, None


def _range_attention(q, k, v, sink, rows, floor, scale, W):
    if not _needs_grad(q, k, v, sink):
        return ops.attention_forward(q, k, v, rows, scale, window=W, floor=floor, sink=sink)[0]
    return _Range.apply(q, k, v, sink, rows, floor, scale, W)


def window_attention(q, k, v, sink, positions, scale, window=None):
    """attention.py:85-107: q (B, T, H, c) at positions (T,) or (B, T); k, v
    (B, window - 1 + T, c), the window - 1 rows before the pass then its own;
    query t reads table rows t .. t + window - 1 that are not before the
    text, with the sink in each head's denominator. window defaults to
    WINDOW (128, attention.py:53). Differentiable in q, k, v and sink, as
    the reference's (plain autograd there; the backward kernels here)."""
    _bf16_only(q, k, v)
    W = WINDOW if window is None else int(window)
    B, T, H, c = q.shape
    positions = _positions(positions, B)
    t = torch.arange(T, device=q.device, dtype=torch.int64)
    rows = (t + W - 1).expand(B, T).contiguous()  # each query's own row in the table
    floor = rows - positions  # the row of position 0: rows before it are before the text
    return _range_attention(q, k, v, sink, rows, floor, scale, W)


# ---------------------------------------------------------- drafter attention

def drafter_attention(q, block, context, sink, lengths, scale):
    """The drafter backbone's attention (packages/wpt-model/src/wpt_model/
    drafter.py:141-151): q (R, count, H, c) for the count places
    of R blocks at positions lengths[r] + i; block (R, count, 2c) the places'
    entries and context (R, W, 2c) the injected context's, at positions
    lengths[r] - W + j (keys then values in each). Place i reads the whole
    block (both directions) and the context entries within W tokens of it
    that are not before the text (the visible mask of drafter.py:189-195),
    with the sink in each head's denominator. Returns (R, count, H, c).

    With the table ordered [context; block], place i's rows are one
    contiguous range, max(i + 1, W - lengths[r]) .. W + count - 1, so the
    range kernels compute it (forward and backward)."""
    _bf16_only(q, block, context)
    R, count, H, c = q.shape
    W = context.shape[1]
    table = torch.cat([context, block], 1)
    lengths = torch.as_tensor(lengths, dtype=torch.int64, device=q.device).reshape(R, 1)
    i = torch.arange(count, device=q.device, dtype=torch.int64)
    rows = torch.full((R, count), W + count - 1, dtype=torch.int64, device=q.device)
    floor = torch.maximum(i[None] + 1, W - lengths).contiguous()
    return _range_attention(q, table[..., :c], table[..., c:], sink, rows, floor, scale, 0)


# ----------------------------------------------------------- tree attention

def tree_attention(q, k, v, cache_len, parents, scale, sink=None):
    """Verification attention of a draft tree: q (B, n, H, c) for n nodes
    whose keys and values sit at table rows cache_len[b] + i; node i reads
    the rows before cache_len[b] and those of its ancestors and itself
    (parents (n,) or (B, n), -1 for a root). A chain (parents[i] = i - 1) is
    exact_attention at positions cache_len + i. Returns (out bf16, lse)."""
    _bf16_only(q, k, v)
    B, n, H, c = q.shape
    cache_len = torch.as_tensor(cache_len, dtype=torch.int64, device=q.device).reshape(-1).expand(B).contiguous()
    bits, positions = ops.tree_bits(torch.as_tensor(parents, dtype=torch.int64, device=q.device), B, cache_len)
    return ops.prefill_forward(q, k, v, positions, scale, tree_bits=bits, tree_base=cache_len, sink=sink)


# ------------------------------------------------------------ acceptance step

def accept(scores, drafted, q, uniforms, resample, temperature=1.0, top_k=None, lengths=None):
    """WPT's speculative acceptance (wpt_inference/__init__.py:173-179,
    210-222) for R rows on the GPU, with the draws as inputs: scores
    (R, n + 1, V) target logits, drafted (R, n), q (R, n, V) the drafter's
    probabilities, uniforms (R, n) the accept tests' draws, resample (R,) the
    last token's draw (inverse CDF). Returns (tokens (R, n + 1), -1 padded;
    accepted (R,))."""
    return ops.accept(scores, drafted, q, uniforms, resample, temperature, top_k, lengths)


def sample(scores, resample, temperature=1.0, top_k=None):
    """The writer's sampling step without drafts (wpt_inference/__init__.py:
    173-182: softmax of the top_k-masked scores / temperature, then a draw;
    SURVEY F3's sampling, the output head's product left to the caller):
    scores (R, V) fp32 logits, resample (R,) the draws, each turned into a
    token by inverse CDF (the first index whose float64 running sum of the
    probabilities exceeds resample[i] times their total). top_k 1 is argmax.
    Returns (R,) int64 tokens. The acceptance kernels with no drafts."""
    R, V = scores.shape
    empty = scores.new_empty(R, 0, V)
    tokens, _ = ops.accept(scores[:, None], torch.empty(R, 0, dtype=torch.int64, device=scores.device), empty,
                           scores.new_empty(R, 0), resample, temperature, top_k)
    return tokens[:, 0]


def head_sample(h, weight, resample, temperature=1.0, top_k=None, round_bf16=True):
    """The writer's step from the last hidden state of each row:
    the output head's scores on the tensor cores (model.py:267,471,
    ops.head_scores; rounded to bf16 as the reference's autocast head gives
    them), then sample(): softmax of the top_k-masked scores / temperature and
    the inverse-CDF draw with resample (wpt_inference/__init__.py:173-182).
    h (R, D) bf16 (final-normed), weight (V, D) bf16, resample (R,).
    Returns (tokens (R,) int64, scores (R, V) fp32)."""
    scores = ops.head_scores(h, weight, round_bf16)
    return sample(scores, resample, temperature, top_k), scores


# ------------------------------------------------------------ cache append

def cache_append(held, new, first, counts, need=None):
    """The generation cache's entries write (packages/wpt-model/src/
    wpt_model/cache.py:110-128, Reading.everything): row b's new
    entries new[b, :counts[b]] are written after its first[b] earlier ones,
    the table growing as the reference's does. Returns (held, held[:, :need]).
    Given need (max_b(first[b] + counts[b]), which a caller keeping its own
    count of each row's tokens knows), the call is one kernel with no host
    synchronisation, where the reference reads the size and the written
    rows back to the host on every exact layer of every step."""
    return ops.cache_append(held, new, first, counts, need)


# ------------------------------------------------------------- installation

def install(kernels, attention=None, device=None, check=True):
    """Makes this module the attention form of the WPT process that imported
    `kernels` (wpt_model.kernels, kernels.py:62-112) and, given `attention`
    (wpt_model.attention), its window layers' window_attention too
    (attention.py:85, which WPT calls directly rather than through a form).

    check: first runs the reference's own install check on this module,
    kernels._try (kernels.py:115-144: both operations forward and backward
    on a small input on `device`), which raises if the kernels cannot work.
    The window wrapper reads attention.WINDOW at each call and casts q, k and
    v to the compute dtype (autocast's bf16), as kernels.exact_attention
    does for the form's operations (kernels.py:160-171)."""
    import sys
    me = sys.modules[__name__]
    if check:
        kernels._try(me, device if device is not None else torch.device("cuda", torch.cuda.current_device()))
    kernels._kernels, kernels._form = me, "b200"
    if attention is not None:
        def window(q, k, v, sink, positions, scale):
            dtype = kernels.compute_dtype(q)
            with torch.autocast(q.device.type, enabled=False):
                return window_attention(q.to(dtype), k.to(dtype), v.to(dtype), sink.float(), positions, scale,
                                        window=attention.WINDOW)
        attention.window_attention = window
    return me


__all__ = ["install", "drafter_attention", "cache_append", "sample", "accept", "NAME", "WINDOW", "chosen_columns", "exact_attention", "sparse_attention", "window_attention",
           "tree_attention",
           "forward_with_lse", "device_status", "LibraryMissing"]
