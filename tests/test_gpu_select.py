"""Exact attention's choice of rows (pytorch_kernels.py:112-117) on the GPU
against the CPU oracle, judged the way the reference's own kernel tests
judge its GPU forms (packages/wpt-model/tests/test_kernels.py:157-199,
test_triton_kernels.py:36-48): the same number of rows per query, -1 in
the same places, and every chosen row weighted within 1e-2 (log) of the
reference's own top_k-th, since bf16 products may order near ties
differently. The reference's SHAPES, a decode row, a generation pass and
rows of equal scores are covered."""

import numpy as np
import pytest
import torch

from oracle import attention as oat

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _np(x):
    return x.float().cpu().numpy().astype(np.float64)


def _score(q, k, positions, scale):
    """(B, T, N): each row's largest log-weight over the heads (the reference's score)."""
    z = np.einsum("bthc,bnc->bthn", q, k) * scale
    N = k.shape[1]
    z = np.where(np.arange(N)[None, None, None, :] > positions[:, :, None, None], -np.inf, z)
    m = z.max(-1, keepdims=True)
    lse = np.log(np.exp(z - m).sum(-1, keepdims=True)) + m
    return (z - lse).max(2)


def _assert_chosen_alike(q, k, positions, scale, chosen, expected):
    score = _score(q, k, positions, scale)
    kth = np.where(expected < 0, np.inf, np.take_along_axis(score, np.clip(expected, 0, None), -1)).min(-1)
    picked = np.where(chosen < 0, np.inf, np.take_along_axis(score, np.clip(chosen, 0, None), -1))
    assert chosen.shape == expected.shape
    assert ((chosen >= 0) == (expected >= 0)).all()
    assert (picked >= kth[..., None] - 1e-2).all()
    for row in chosen.reshape(-1, chosen.shape[-1]):
        kept = row[row >= 0]
        assert len(set(kept.tolist())) == len(kept)


# (heads, width, tokens, top k, window): the reference's SHAPES (test_kernels.py:139-140)
SHAPES = [(2, 128, 700, 64, 128), (4, 128, 300, 16, 32), (12, 128, 300, 16, 32), (8, 128, 700, 64, 128),
          (8, 128, 2000, 1024, 128)]


@pytest.mark.parametrize("H,C,T,top_k,window", SHAPES)
def test_choice_matches_reference_rule(wb, H, C, T, top_k, window):
    g = torch.Generator().manual_seed(T + H)
    B = 2
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    k = torch.randn(B, T, C, generator=g).bfloat16()
    v = torch.randn(B, T, C, generator=g).bfloat16()
    positions = torch.arange(T).expand(B, T).contiguous()
    out, chosen = wb.exact_attention(q.cuda(), k.cuda(), v.cuda(), positions.cuda(), C ** -0.5, top_k, window)
    assert wb.device_status() == 0
    _, _, expected = oat.exact_attention(_np(q), _np(k), _np(v), positions.numpy(), C ** -0.5, top_k, window)
    _assert_chosen_alike(_np(q), _np(k), positions.numpy(), C ** -0.5, chosen.cpu().numpy(), expected)
    ref_out, _, _ = oat.exact_attention(_np(q), _np(k), _np(v), positions.numpy(), C ** -0.5, 0, window)
    assert np.abs(out.float().cpu().numpy() - ref_out).max() < 2e-2


def test_decode_choice_over_a_long_row(wb):
    g = torch.Generator().manual_seed(1)
    B, T, H, C, N = 3, 1, 32, 128, 9000
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    positions = torch.tensor([[8999], [4000], [900]])
    qd, ed = q.cuda(), e.cuda()
    _, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5, 1024, 128)
    assert wb.device_status() == 0
    k = _np(e[..., :C])
    _, _, expected = oat.exact_attention(_np(q), k, _np(e[..., C:]), positions.numpy(), C ** -0.5, 1024, 128)
    _assert_chosen_alike(_np(q), k, positions.numpy(), C ** -0.5, chosen.cpu().numpy(), expected)


def test_generation_pass_choice(wb):
    # ragged rows, a query past the table, halves of an entries table (test_triton_kernels.py:51-77)
    g = torch.Generator().manual_seed(0)
    B, T, H, C, N, top_k, window = 3, 4, 4, 128, 400, 64, 16
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    positions = torch.tensor([[396, 397, 398, 399], [100, 101, 102, 103], [398, 399, 400, 401]])
    _, chosen = wb.exact_attention(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                   top_k, window)
    k = _np(e[..., :C])
    _, _, expected = oat.exact_attention(_np(q), k, _np(e[..., C:]), positions.numpy(), C ** -0.5, top_k, window)
    pos_clipped = np.minimum(positions.numpy(), N - 1)
    _assert_chosen_alike(_np(q), k, pos_clipped, C ** -0.5, chosen.cpu().numpy(), expected)


def test_rows_of_equal_scores_are_chosen_as_many_as_wanted(wb):
    # every key one of two vectors (test_triton_kernels.py:100-120): distinct rows, as many as top_k
    g = torch.Generator().manual_seed(3)
    B, T, H, C, top_k, window = 1, 400, 2, 128, 64, 8
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    pair = torch.randn(2, C, generator=g)
    k = pair[(torch.arange(T) % 7 == 0).long()][None].bfloat16()
    v = torch.randn(B, T, C, generator=g).bfloat16()
    positions = torch.arange(T).expand(B, T).contiguous()
    _, chosen = wb.exact_attention(q.cuda(), k.cuda(), v.cuda(), positions.cuda(), C ** -0.5, top_k, window)
    _, _, expected = oat.exact_attention(_np(q), _np(k), _np(v), positions.numpy(), C ** -0.5, top_k, window)
    _assert_chosen_alike(_np(q), _np(k), positions.numpy(), C ** -0.5, chosen.cpu().numpy(), expected)


def test_choice_feeds_sparse_attention(wb):
    # the exact layer's choice read by a sparse layer (attention.py:187,215)
    g = torch.Generator().manual_seed(9)
    B, T, H, C, top_k, window = 2, 300, 16, 128, 32, 32
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, T, 2 * C, generator=g).bfloat16()
    sink = torch.randn(H, generator=g) * 0.5
    positions = torch.arange(T).expand(B, T).contiguous()
    qd, ed = q.cuda(), e.cuda()
    _, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5, top_k, window)
    out = wb.sparse_attention(qd, ed[..., :C], ed[..., C:], sink.cuda(), chosen, positions.cuda(), C ** -0.5,
                              window)
    ref, _ = oat.sparse_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().numpy(),
                                  chosen.cpu().numpy(), positions.numpy(), C ** -0.5, window)
    assert np.abs(out.float().cpu().numpy() - ref).max() < 2e-2


@pytest.mark.parametrize("tied", [False, True])
def test_decode_choice_over_ragged_rows(wb, tied):
    """Decode rows of many lengths, some with no row to choose from (the
    balanced split of the scoring over the SMs, with ranges that cross
    rows); with tied keys (two distinct key vectors) thousands of equal
    scores crowd the threshold's bin and the radix passes decide."""
    g = torch.Generator().manual_seed(5 + tied)
    B, T, H, C, N, top_k, window = 40, 1, 32, 128, 6000, 256, 128
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    if tied:
        pair = torch.randn(2, C, generator=g)
        e[..., :C] = pair[(torch.arange(N) % 5 == 0).long()][None].bfloat16()
    positions = torch.randint(100, N + 200, (B, 1), generator=g)
    qd, ed = q.cuda(), e.cuda()
    _, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5, top_k, window)
    assert wb.device_status() == 0
    k = _np(e[..., :C])
    _, _, expected = oat.exact_attention(_np(q), k, _np(e[..., C:]), positions.numpy(), C ** -0.5, top_k, window)
    pos_clipped = np.minimum(positions.numpy(), N - 1)
    _assert_chosen_alike(_np(q), k, pos_clipped, C ** -0.5, chosen.cpu().numpy(), expected)


def test_decode_choice_over_rows_longer_than_the_key_cache(wb):
    """Rows of more candidates than the select kernel caches in shared
    memory: the passes read the scores from global memory."""
    g = torch.Generator().manual_seed(11)
    B, T, H, C, N, top_k, window = 2, 1, 32, 128, 60000, 1024, 128
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    positions = torch.tensor([[59999], [50000]])
    qd, ed = q.cuda(), e.cuda()
    _, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5, top_k, window)
    assert wb.device_status() == 0
    k = _np(e[..., :C])
    _, _, expected = oat.exact_attention(_np(q), k, _np(e[..., C:]), positions.numpy(), C ** -0.5, top_k, window)
    _assert_chosen_alike(_np(q), k, positions.numpy(), C ** -0.5, chosen.cpu().numpy(), expected)


@pytest.mark.parametrize("top_k", [64, 1])
def test_decode_choice_with_a_few_more_rows_than_top_k(wb, top_k):
    """Decode rows with top_k + 1 .. top_k + 16 candidates and a few about
    twice top_k: with fewer queries than SMs each query's candidates are cut
    into two slices (the second from the row's rounded middle), so the
    second slice is small, or empty (2 candidates, top_k 1), and the bin's
    keys come from both."""
    g = torch.Generator().manual_seed(13 + top_k)
    B, T, H, C, N, window = 20, 1, 32, 128, 1024, 8
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    counts = torch.tensor(list(range(top_k + 1, top_k + 17)) + [2 * top_k - 1, 2 * top_k, 2 * top_k + 3, 5])
    positions = (counts + window - 1).view(B, 1)  # count = position - window + 1 candidates
    qd, ed = q.cuda(), e.cuda()
    _, chosen = wb.exact_attention(qd, ed[..., :C], ed[..., C:], positions.cuda(), C ** -0.5, top_k, window)
    assert wb.device_status() == 0
    k = _np(e[..., :C])
    _, _, expected = oat.exact_attention(_np(q), k, _np(e[..., C:]), positions.numpy(), C ** -0.5, top_k, window)
    _assert_chosen_alike(_np(q), k, positions.numpy(), C ** -0.5, chosen.cpu().numpy(), expected)
