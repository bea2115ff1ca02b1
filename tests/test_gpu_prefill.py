"""The tcgen05 prefill kernel against the CPU oracle (which the reference's
own outputs pin, tests/test_oracle.py), through the C ABI: causal exact
attention, window + sink, window_attention's tail layout, tree-masked
verification, split-KV, ragged generation passes and padding queries past
the table. Tolerances (BASELINE): bf16 outputs within max-abs 2e-2, LSE
within 1e-3."""

import numpy as np
import pytest
import torch

from oracle import attention as oat

pytestmark = pytest.mark.gpu

OUT_TOL, LSE_TOL = 2e-2, 1e-3


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _inputs(B, T, H, C, N, seed, spread=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, T, H, C, generator=g) * spread).bfloat16()
    entries = (torch.randn(B, N, 2 * C, generator=g) * spread).bfloat16()
    return q, entries


def _np(x):
    return x.float().cpu().numpy().astype(np.float64)


def _check(wb, out, lse, ref_out, ref_lse):
    assert wb.device_status() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref_out).max() < OUT_TOL
    if lse is not None:
        assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_TOL


@pytest.mark.parametrize("B,T,H,C", [(2, 300, 4, 128), (1, 257, 16, 128), (2, 130, 8, 64), (1, 64, 32, 128),
                                     (3, 40, 12, 128), (1, 700, 2, 128)])
def test_causal_prefill_matches_oracle(wb, B, T, H, C):
    q, e = _inputs(B, T, H, C, T, seed=B * 1000 + T)
    qd, ed = q.cuda(), e.cuda()
    positions = torch.arange(T).expand(B, T).contiguous()
    out, lse = wb.forward_with_lse(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


def test_exact_attention_drop_in_returns_q_dtype_and_empty_choice(wb):
    B, T, H, C = 2, 200, 8, 128
    q, e = _inputs(B, T, H, C, T, seed=5)
    qd, ed = q.cuda(), e.cuda()
    positions = torch.arange(T).cuda()  # (T,) is expanded as kernels.py:_positions does
    out, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions, C ** -0.5, 0, 128)
    assert out.dtype == torch.bfloat16 and chosen.shape == (B, T, 0) and chosen.dtype == torch.int64
    ref_out, _, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]),
                                        np.broadcast_to(np.arange(T), (B, T)), C ** -0.5, 0, 128)
    _check(wb, out, None, ref_out, None)


def test_generation_pass_ragged_rows_and_padding_past_table(wb):
    # rows at different places; the last row's later queries sit past the
    # table (they read up to its last row); rows past a row's own length
    # hold stale values that must not be read
    B, T, H, C, N = 3, 4, 16, 128, 400
    q, e = _inputs(B, T, H, C, N, seed=7)
    positions = torch.tensor([[396, 397, 398, 399], [100, 101, 102, 103], [398, 399, 400, 401]])
    e[1, 104:] = 77.0  # stale rows of row 1: large values that would show if read
    out, lse = wb.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("T,H,window", [(600, 16, 128), (1100, 8, 256), (300, 4, 1024)])
def test_window_with_sink_matches_sparse_oracle(wb, T, H, window):
    # sparse_attention with no chosen rows = each query's last `window` rows + sink
    B, C = 2, 128
    q, e = _inputs(B, T, H, C, T, seed=T + window)
    sink = torch.randn(H, generator=torch.Generator().manual_seed(1)) * 0.5
    positions = torch.arange(T).expand(B, T).contiguous()
    out, lse = wb.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                   window=window, sink=sink.cuda())
    ref_out, ref_lse = oat.sparse_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().numpy(),
                                            np.zeros((B, T, 0), np.int64), positions.numpy(), C ** -0.5, window)
    _check(wb, out, lse, ref_out, ref_lse)


def test_window_attention_tail_layout_matches_oracle(wb):
    # attention.py:85-107's layout: window - 1 tail rows, then the pass; the
    # first row starts near the text's start, so some tail rows are before it
    B, T, H, C, W = 2, 300, 16, 128, 128
    g = torch.Generator().manual_seed(11)
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    k = torch.randn(B, W - 1 + T, C, generator=g).bfloat16()
    v = torch.randn(B, W - 1 + T, C, generator=g).bfloat16()
    sink = torch.randn(H, generator=g) * 0.5
    positions = torch.stack([5 + torch.arange(T), 900 + torch.arange(T)])
    out = wb.window_attention(q.cuda(), k.cuda(), v.cuda(), sink.cuda(), positions.cuda(), C ** -0.5, window=W)
    ref_out, _ = oat.window_attention(_np(q), _np(k), _np(v), sink.double().numpy(), positions.numpy(), C ** -0.5, W)
    _check(wb, out, None, ref_out, None)


def test_tree_verification_matches_oracle(wb):
    B, L, n, H, C = 4, 1000, 16, 32, 128
    q, e = _inputs(B, n, H, C, L + n + 5, seed=21)
    parents = torch.tensor([-1, 0, 0, 0, 1, 1, 2, 2, 3, 4, 4, 5, 6, 7, 8, 9])
    cache_len = torch.tensor([1000, 700, 999, 3])
    out, lse = wb.tree_attention(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], cache_len.cuda(), parents,
                                 C ** -0.5)
    ref_out, ref_lse = oat.tree_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), cache_len.numpy(),
                                          parents.numpy(), C ** -0.5)
    _check(wb, out, lse, ref_out, ref_lse)


def test_tree_bits_on_the_device_match_the_ancestor_masks(wb):
    from wpt_b200 import ops
    parents = torch.tensor([[-1, 0, 0, 1, 1, 2, 4], [-1, 0, 1, 2, 3, 4, 5]])
    bits, pos = ops.tree_bits(parents.cuda(), 2, torch.tensor([10, 500]).cuda())
    bits = bits.cpu()
    assert pos.cpu().tolist() == [[10 + i for i in range(7)], [500 + i for i in range(7)]]
    assert bits[0].tolist() == [0b1, 0b11, 0b101, 0b1011, 0b10011, 0b100101, 0b1010011]
    assert bits[1].tolist() == [(1 << (i + 1)) - 1 for i in range(7)]
    chain = ops.tree_bits(torch.arange(64).cuda() - 1, 3)[0].cpu()
    assert chain.shape == (3, 64) and chain[0, 0].item() == 1 and chain[2, -1].item() == -1  # all 64 bits
    masks = oat.ancestors_mask(np.array([-1, 0, 0, 1, 1, 2, 4]))
    want = [(masks[i] * (1 << np.arange(7))).sum() for i in range(7)]
    assert bits[0].tolist() == [int(w) for w in want]
    # a parent that is not before its child ends that node's walk (no fault, no endless loop)
    bad = ops.tree_bits(torch.tensor([-1, 2, 0]).cuda(), 1)[0].cpu()
    assert bad.tolist() == [[0b1, 0b10, 0b101]]
    assert wb.device_status() == 0


def test_chain_tree_equals_exact_attention(wb):
    B, L, n, H, C = 2, 513, 6, 32, 128
    q, e = _inputs(B, n, H, C, L + n, seed=22)
    qd, ed = q.cuda(), e.cuda()
    out, lse = wb.tree_attention(qd, ed[..., :C], ed[..., C:], torch.tensor([L, L]).cuda(), torch.arange(n) - 1,
                                 C ** -0.5)
    positions = (L + torch.arange(n)).expand(B, n).contiguous().cuda()
    out2, lse2 = wb.forward_with_lse(qd, ed[..., :C], ed[..., C:], positions, C ** -0.5)
    assert (out.float() - out2.float()).abs().max().item() < 1e-6
    assert (lse - lse2).abs().max().item() < 1e-6


@pytest.mark.parametrize("splits", [2, 5])
def test_split_kv_equals_unsplit(wb, splits):
    from wpt_b200 import ops
    B, T, H, C, N = 2, 8, 16, 128, 3000
    q, e = _inputs(B, T, H, C, N, seed=splits)
    positions = (N - T + torch.arange(T)).expand(B, T).contiguous().cuda()
    sink = (torch.randn(H, generator=torch.Generator().manual_seed(3)) * 0.5).cuda()
    qd, ed = q.cuda(), e.cuda()
    whole = ops.prefill_forward(qd, ed[..., :C], ed[..., C:], positions, C ** -0.5, sink=sink, splits=1)
    parts = ops.prefill_forward(qd, ed[..., :C], ed[..., C:], positions, C ** -0.5, sink=sink, splits=splits)
    assert (whole[0].float() - parts[0].float()).abs().max().item() < 1e-2
    assert (whole[1] - parts[1]).abs().max().item() < 1e-4
    seen = np.arange(N)[None, None, :] <= positions.cpu().numpy()[..., None]
    rows = np.where(seen, np.arange(N)[None, None, :], -1)
    ref_out, ref_lse = oat.sparse_over_rows(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().cpu().numpy(),
                                            rows, C ** -0.5)
    _check(wb, parts[0], parts[1], ref_out, ref_lse)


@pytest.mark.parametrize("splits", [2, 4])
def test_split_kv_with_a_partly_filled_last_query_tile(wb, splits):
    # the last query tile of each row holds 12 of 16 tokens (H = 8): every
    # split's partial must be complete before its epilogue reads it
    from wpt_b200 import ops
    B, T, H, C = 2, 700, 8, 128
    q, e = _inputs(B, T, H, C, T, seed=708)
    positions = torch.arange(T).expand(B, T).contiguous()
    out, lse = ops.prefill_forward(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                   splits=splits)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


def test_growing_scores_force_rescales(wb):
    # scores that grow along the row raise each row's running maximum by far
    # more than the lazy threshold in every tile, so O is rescaled each time
    B, T, H, C = 1, 640, 16, 128
    g = torch.Generator().manual_seed(31)
    u = torch.randn(C, generator=g)
    u = u / u.norm()
    q = (u * 3.0 + 0.1 * torch.randn(B, T, H, C, generator=g)).bfloat16()
    k = (u * (torch.arange(T)[:, None] / 16.0) + 0.1 * torch.randn(B, T, C, generator=g)).bfloat16()
    v = torch.randn(B, T, C, generator=g).bfloat16()
    positions = torch.arange(T).expand(B, T).contiguous()
    out, lse = wb.forward_with_lse(q.cuda(), k.cuda(), v.cuda(), positions.cuda(), C ** -0.5)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(k), _np(v), positions.numpy(), C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)
