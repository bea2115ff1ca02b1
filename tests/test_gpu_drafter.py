"""The drafter backbone's attention (packages/wpt-model/src/
wpt_model/drafter.py:141-151 with the visible mask of :189-195) on the range
kernels, against the CPU oracle: the forward pass against oracle
dense_attention over the reference's [block; context] table and mask
(oracle.attention.drafter_attention), the gradients of q, the block's and
the context's entries and the sink against the oracle's gradient formulas.
Contexts partly before the text (lengths below the window) included.
Tolerances: outputs within max-abs 2e-2 (bf16), gradients within 2% of
their largest magnitude and 1% relative Frobenius error."""

import numpy as np
import pytest
import torch

from oracle import attention as oat
from oracle import backward as ob

pytestmark = pytest.mark.gpu

C, W = 128, 128


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _np(x):
    return x.detach().float().cpu().numpy().astype(np.float64)


def _close_grad(got, want, name):
    got = _np(got)
    scale = max(np.abs(want).max(), 1e-6)
    assert np.abs(got - want).max() <= 2e-2 * scale, name
    assert np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-12) < 1e-2, name


def _case(R, count, H, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(R, count, H, C, generator=g) * 0.5).bfloat16().cuda()
    block = (torch.randn(R, count, 2 * C, generator=g) * 0.5).bfloat16().cuda()
    context = (torch.randn(R, W, 2 * C, generator=g) * 0.5).bfloat16().cuda()
    sink = (torch.randn(H, generator=g) * 0.5).cuda()
    lengths = torch.tensor([3, 50, 127, 128, 500, 2000][:R]).cuda()
    return q, block, context, sink, lengths


@pytest.mark.parametrize("R,count,H", [(6, 4, 16), (6, 16, 16), (4, 8, 32), (5, 2, 4)])
def test_drafter_attention_matches_the_reference_mask(wb, R, count, H):
    q, block, context, sink, lengths = _case(R, count, H, seed=count * 10 + H)
    out = wb.drafter_attention(q, block, context, sink, lengths, C ** -0.5)
    assert wb.device_status() == 0
    ref, _ = oat.drafter_attention(_np(q), _np(block), _np(context), _np(sink), lengths.cpu().numpy(), C ** -0.5)
    assert np.abs(_np(out) - ref).max() < 2e-2


def test_drafter_attention_gradients_match_oracle(wb):
    R, count, H = 6, 8, 16
    q, block, context, sink, lengths = _case(R, count, H, seed=5)
    q, block, context, sink = (x.requires_grad_() for x in (q, block, context, sink))
    d_out = torch.randn(R, count, H, C, generator=torch.Generator().manual_seed(6)).bfloat16().cuda()
    out = wb.drafter_attention(q, block, context, sink, lengths, C ** -0.5)
    out.backward(d_out)
    assert wb.device_status() == 0
    # the oracle over the table [context; block] with each place's rows listed
    table = np.concatenate([_np(context), _np(block)], 1)
    L = lengths.cpu().numpy()
    rows = np.full((R, count, W + count), -1, np.int64)
    for r in range(R):
        for i in range(count):
            seen = np.arange(max(i + 1, W - int(L[r])), W + count)
            rows[r, i, :len(seen)] = seen
    ref_out, ref_lse = oat.sparse_over_rows(_np(q), table[..., :C], table[..., C:], _np(sink), rows, C ** -0.5)
    assert np.abs(_np(out) - ref_out).max() < 2e-2
    dq, dk, dv, ds = ob.rows_backward(_np(q), table[..., :C], table[..., C:], _np(sink), rows, _np(out), ref_lse,
                                      _np(d_out), C ** -0.5)
    dtable = np.concatenate([dk, dv], -1)
    _close_grad(q.grad, dq, "dq")
    _close_grad(context.grad, dtable[:, :W], "d context")
    _close_grad(block.grad, dtable[:, W:], "d block")
    assert np.abs(_np(sink.grad) - ds).max() <= 1e-2 * max(1.0, np.abs(ds).max())
