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
    return x.detach().float().cpu().numpy().astype(np.float64)


def _close_grad(got, want, name):
    got = got.detach().float().cpu().numpy().astype(np.float64) if torch.is_tensor(got) else got
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


@pytest.mark.parametrize("B,T,H,N,K,window", [(2, 40, 16, 600, 300, 64), (1, 9, 32, 2000, 1024, 128),
                                              (2, 5, 4, 300, 40, 8), (1, 3, 64, 500, 130, 16)])
def test_sparse_backward_with_chosen_rows_matches_oracle(wb, B, T, H, N, K, window):
    from wpt_b200 import ops
    g = torch.Generator().manual_seed(N + K + H)
    q, e, d_out = _case(B, T, H, N, seed=N + K)
    k, v = e[..., :C], e[..., C:]
    sink = (torch.randn(H, generator=g) * 0.5).cuda()
    positions = (N - T + torch.arange(T)).expand(B, T).contiguous()
    # each query's chosen rows: distinct rows at least `window` back, some -1
    idx = torch.stack([torch.stack([torch.randperm(int(p) - window + 1, generator=g)[:K] for p in row])
                       for row in positions])
    idx[:, ::2, -K // 5:] = -1
    positions, idx = positions.cuda(), idx.cuda()
    out, lse = ops.stream_forward(q, k, v, positions, C ** -0.5, window=window, idx=idx, sink=sink)
    dq, dk, dv, ds = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5, window=window,
                                            sink=sink, idx=idx)
    assert wb.device_status() == 0
    assert dq.dtype == torch.bfloat16 and dk.dtype == torch.bfloat16
    rq, rk, rv, rs = ob.sparse_backward(_np(q), _np(k), _np(v), _np(sink), idx.cpu().numpy(),
                                        positions.cpu().numpy(), _np(out), _np(lse), _np(d_out), C ** -0.5, window)
    _close_grad(dq, rq, "dq")
    _close_grad(dk, rk, "dk")
    _close_grad(dv, rv, "dv")
    assert np.abs(ds.cpu().numpy() - rs).max() <= 1e-2 * max(1.0, np.abs(rs).max())


def test_window_attention_autograd_matches_oracle(wb):
    B, T, H, W = 2, 300, 16, 128
    g = torch.Generator().manual_seed(12)
    q = (torch.randn(B, T, H, C, generator=g) * 0.5).bfloat16().cuda().requires_grad_()
    k = (torch.randn(B, W - 1 + T, C, generator=g) * 0.5).bfloat16().cuda().requires_grad_()
    v = (torch.randn(B, W - 1 + T, C, generator=g) * 0.5).bfloat16().cuda().requires_grad_()
    sink = (torch.randn(H, generator=g) * 0.5).cuda().requires_grad_()
    positions = torch.stack([5 + torch.arange(T), 900 + torch.arange(T)]).cuda()
    d_out = torch.randn(B, T, H, C, generator=g).bfloat16().cuda()
    out = wb.window_attention(q, k, v, sink, positions, C ** -0.5, window=W)
    out.backward(d_out)
    assert wb.device_status() == 0
    ref_out, ref_lse = oat.window_attention(_np(q), _np(k), _np(v), _np(sink), positions.cpu().numpy(), C ** -0.5, W)
    rq, rk, rv, rs = ob.window_backward(_np(q), _np(k), _np(v), _np(sink), positions.cpu().numpy(), _np(out),
                                        ref_lse, _np(d_out), C ** -0.5, W)
    _close_grad(q.grad, rq, "dq")
    _close_grad(k.grad, rk, "dk")
    _close_grad(v.grad, rv, "dv")
    assert np.abs(sink.grad.cpu().numpy() - rs).max() <= 1e-2 * max(1.0, np.abs(rs).max())


def test_reference_try_both_sequence_forward_and_backward(wb):
    # the reference's install check (kernels.py:123-144): bf16 leaves B=1,
    # T=8, H=4, c=128, window 2, top_k 4; exact attention, then sparse
    # attention over its choice, then one backward through both
    generator = torch.Generator().manual_seed(0)
    B, T, H, c, window, top_k = 1, 8, 4, 128, 2, 4

    def leaf(*shape):
        return torch.randn(*shape, generator=generator).to("cuda", torch.bfloat16).requires_grad_()
    q, k, v = leaf(B, T, H, c), leaf(B, T, c), leaf(B, T, c)
    sink = torch.zeros(H, device="cuda", requires_grad=True)
    positions = torch.arange(T, device="cuda").expand(B, T)
    with torch.enable_grad():
        out, chosen = wb.exact_attention(q, k, v, positions, c ** -0.5, top_k, window)
        sparse = wb.sparse_attention(q, k, v, sink, chosen, positions, c ** -0.5, window)
        (out.float().sum() + sparse.float().sum()).backward()
    torch.cuda.synchronize()
    assert wb.device_status() == 0
    pos = positions.cpu().numpy()
    qn, kn, vn = _np(q), _np(k), _np(v)
    ones = np.ones((B, T, H, c))
    ref_out, ref_lse, _ = oat.exact_attention(qn, kn, vn, pos, c ** -0.5, 0, 0)
    eq, ek, ev = ob.exact_backward(qn, kn, vn, pos, _np(out), ref_lse, ones, c ** -0.5)
    idx = chosen.cpu().numpy()
    s_out, s_lse = oat.sparse_attention(qn, kn, vn, np.zeros(H), idx, pos, c ** -0.5, window)
    sq, sk, sv, ss = ob.sparse_backward(qn, kn, vn, np.zeros(H), idx, pos, _np(sparse), s_lse, ones, c ** -0.5,
                                        window)
    _close_grad(q.grad, eq + sq, "dq")
    _close_grad(k.grad, ek + sk, "dk")
    _close_grad(v.grad, ev + sv, "dv")
    assert np.abs(sink.grad.cpu().numpy() - ss).max() <= 1e-2 * max(1.0, np.abs(ss).max())
    assert q.grad.dtype == torch.bfloat16 and sink.grad.dtype == torch.float32


def test_a_wait_that_runs_out_reports_and_leaves_the_context_usable(wb):
    # failure detection without a fault: the query-tile kernel's loader does
    # not issue key tile 0's copy (nothing is in flight for it) and its waits
    # give up after 1 ms; the call returns, status bit 0 is set, and after a
    # reset the next call (hook off) is correct
    from wpt_b200 import _lib, ops
    B, T, H = 1, 16, 16
    q, e, d_out = _case(B, T, H, T, seed=3)
    k, v = e[..., :C], e[..., C:]
    positions = torch.arange(T).expand(B, T).contiguous().cuda()
    out, lse = ops.attention_forward(q, k, v, positions, C ** -0.5)
    assert wb.device_status() == 0
    _lib.check(_lib.lib().wpt_debug_backward_fault(0, 1_000_000))
    try:
        ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5)
        assert wb.device_status(reset=True) & 1  # a bounded wait ran out, and the status says so
    finally:
        _lib.check(_lib.lib().wpt_debug_backward_fault(-1, 0))
    assert wb.device_status() == 0
    dq, dk, dv, _ = ops.attention_backward(q, k, v, positions, out, lse, d_out, C ** -0.5)
    assert wb.device_status() == 0
    rq, rk, rv = ob.exact_backward(_np(q), _np(k), _np(v), positions.cpu().numpy(), _np(out), _np(lse), _np(d_out),
                                   C ** -0.5)
    _close_grad(dq, rq, "dq")
    _close_grad(dk, rk, "dk")
    _close_grad(dv, rv, "dv")
