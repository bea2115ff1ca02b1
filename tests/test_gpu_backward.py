"""The backward kernels (bwd_prep, bwd_kv, bwd_q; gathered rows by
bwd_gather) against the CPU oracle's gradients (oracle/backward.py, which
the reference's own autograd pins, tests/test_oracle.py), through the C ABI.

The oracle is given the GPU forward pass's own output and log-sum-exp, so
the comparison isolates the backward pass. P and dS enter the tensor-core
products as bf16 and the gradients leave as bf16, so the bound is relative
to each gradient's size: max-abs error within 2% of the gradient's largest
magnitude, and a relative Frobenius error under 1%."""

import numpy as np
import pytest
import torch

from oracle import attention as oat
from oracle import backward as ob

pytestmark = pytest.mark.gpu

C = 128


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _np(x):
    return x.float().cpu().numpy().astype(np.float64)


def _close_grad(got, want, name):
    got = got.float().cpu().numpy().astype(np.float64) if torch.is_tensor(got) else got
    scale = max(np.abs(want).max(), 1e-6)
    err = np.abs(got - want).max()
    fro = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-12)
    assert np.isfinite(got).all(), name
    assert err <= 2e-2 * scale, f"{name}: max-abs error {err:.3g} against a largest gradient of {scale:.3g}"
    assert fro < 1e-2, f"{name}: relative Frobenius error {fro:.3g}"


def _case(B, T, H, N, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, T, H, C, generator=g) * 0.5).bfloat16().cuda()
    e = (torch.randn(B, N, 2 * C, generator=g) * 0.5).bfloat16().cuda()
    d_out = torch.randn(B, T, H, C, generator=g).bfloat16().cuda()
    return q, e, d_out


@pytest.mark.parametrize("B,T,H", [(2, 300, 16), (1, 257, 4), (2, 130, 12), (1, 64, 32), (3, 40, 8)])
def test_exact_backward_matches_oracle(wb, B, T, H):
    from wpt_b200 import ops
    q, e, d_out = _case(B, T, H, T, seed=B * 100 + T + H)
    k, v = e[..., :C], e[..., C:]
    positions = torch.arange(T).expand(B, T).contiguous().cuda()
    out, lse = ops.attention_forward(q, k, v, positions, C ** -0.5)
    dq, dk, dv, ds = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5)
    assert wb.device_status() == 0 and ds is None
    rq, rk, rv = ob.exact_backward(_np(q), _np(k), _np(v), positions.cpu().numpy(), _np(out), _np(lse), _np(d_out),
                                   C ** -0.5)
    _close_grad(dq, rq, "dq")
    _close_grad(dk, rk, "dk")
    _close_grad(dv, rv, "dv")


def test_exact_backward_generation_pass_and_padding_past_table(wb):
    # ragged rows at different places in a longer table, one row's later
    # queries past the table (they read up to its last row), stale rows
    # past each row's length that must get zero gradients
    from wpt_b200 import ops
    B, T, H, N = 3, 24, 16, 700
    q, e, d_out = _case(B, T, H, N, seed=9)
    k, v = e[..., :C], e[..., C:]
    positions = torch.stack([680 + torch.arange(T), 100 + torch.arange(T), 690 + torch.arange(T)]).cuda()
    out, lse = ops.attention_forward(q, k, v, positions, C ** -0.5)
    dq, dk, dv, _ = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5)
    assert wb.device_status() == 0
    rq, rk, rv = ob.exact_backward(_np(q), _np(k), _np(v), positions.cpu().numpy(), _np(out), _np(lse), _np(d_out),
                                   C ** -0.5)
    _close_grad(dq, rq, "dq")
    _close_grad(dk, rk, "dk")
    _close_grad(dv, rv, "dv")
    assert dk[1, 124:].abs().max().item() == 0 and dv[1, 124:].abs().max().item() == 0


@pytest.mark.parametrize("T,H,window", [(600, 16, 128), (300, 8, 1024), (520, 32, 200)])
def test_window_sink_backward_matches_oracle(wb, T, H, window):
    from wpt_b200 import ops
    B = 2
    q, e, d_out = _case(B, T, H, T, seed=T + window)
    k, v = e[..., :C], e[..., C:]
    sink = (torch.randn(H, generator=torch.Generator().manual_seed(4)) * 0.5).cuda()
    positions = torch.arange(T).expand(B, T).contiguous().cuda()
    out, lse = ops.attention_forward(q, k, v, positions, C ** -0.5, window=window, sink=sink)
    dq, dk, dv, ds = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5, window=window, sink=sink)
    assert wb.device_status() == 0
    rows = oat.window_rows(positions.cpu().numpy(), window, T)
    rq, rk, rv, rs = ob.rows_backward(_np(q), _np(k), _np(v), _np(sink), rows, _np(out), _np(lse), _np(d_out),
                                      C ** -0.5)
    _close_grad(dq, rq, "dq")
    _close_grad(dk, rk, "dk")
    _close_grad(dv, rv, "dv")
    assert np.abs(ds.cpu().numpy() - rs).max() <= 1e-2 * max(1.0, np.abs(rs).max())


def test_fp32_gradients_equal_bf16_ones_before_rounding(wb):
    from wpt_b200 import ops
    B, T, H = 1, 200, 16
    q, e, d_out = _case(B, T, H, T, seed=77)
    k, v = e[..., :C], e[..., C:]
    positions = torch.arange(T).expand(B, T).contiguous().cuda()
    out, lse = ops.attention_forward(q, k, v, positions, C ** -0.5)
    g16 = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5)
    g32 = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5, f32=True)
    for a, b in zip(g16[:3], g32[:3]):
        assert b.dtype == torch.float32
        assert torch.equal(a, b.bfloat16())
