"""Parity at the shapes bench.py measures, through the public calls, with
the bench's own seeded inputs (bench.config2_inputs, config3_inputs,
config4_inputs): every number bench.py reports is a throughput of output
checked here against the CPU oracle (which the reference's own outputs pin,
tests/test_oracle.py).

  config 2  B=8, T=4096, 16q/1kv, c=128: the causal pass (exact_attention,
            top_k 0) and the window-1024 pass with a sink (sparse_attention
            with no chosen rows); two whole batch rows against the oracle.
  config 3  the 64 seed-0 ragged rows up to 32,768 keys (rows past each
            length hold random values): global, window-1024 + sink, exact
            attention with its top-1024 choice (window 128) judged by the
            reference's rule (tests/test_kernels.py:157-199 of the reference),
            and sparse attention over the chosen rows.
  config 4  B=32, L=8192, the 16-node draft tree through tree_attention.

Tolerances (BASELINE): bf16 outputs within max-abs 2e-2, LSE within 1e-3."""

import numpy as np
import pytest
import torch

import bench
from oracle import attention as oat

pytestmark = pytest.mark.gpu

OUT_TOL, LSE_TOL = 2e-2, 1e-3
C = 128


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _f32(x):
    return x.float().cpu().numpy()


def _close(out, lse, ref_out, ref_lse):
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref_out).max() < OUT_TOL
    if lse is not None:
        assert np.abs(lse.float().cpu().numpy() - ref_lse).max() < LSE_TOL


@pytest.fixture(scope="module")
def config2():
    q, entries, positions, sink = bench.config2_inputs(torch.device("cuda", 0), 0)
    return q, entries, positions, sink


@pytest.mark.parametrize("window", [0, 1024])
def test_config2_prefill_passes_match_oracle(wb, config2, window):
    q, entries, positions, sink = config2
    k, v = entries[..., :C], entries[..., C:]
    B, T = q.shape[:2]
    if window:
        empty = torch.empty(B, T, 0, dtype=torch.int64, device=q.device)
        out = wb.sparse_attention(q, k, v, sink, empty, positions, C ** -0.5, window)
        _, lse = wb.forward_with_lse(q, k, v, positions, C ** -0.5, window=window, sink=sink)
    else:
        out, chosen = wb.exact_attention(q, k, v, positions, C ** -0.5, 0, 1024)
        assert chosen.shape == (B, T, 0)
        _, lse = wb.forward_with_lse(q, k, v, positions, C ** -0.5)
    assert wb.device_status() == 0
    for b in (0, B - 1):  # two whole batch rows; float32 BLAS oracle, about a second a row
        ref_out, ref_lse = oat.range_attention(_f32(q[b:b + 1]), _f32(k[b:b + 1]), _f32(v[b:b + 1]),
                                               positions[b:b + 1].cpu().numpy(), C ** -0.5, window=window,
                                               sink=_f32(sink) if window else None, dtype=np.float32)
        _close(out[b:b + 1], lse[b:b + 1], ref_out, ref_lse)


@pytest.fixture(scope="module")
def config3():
    return bench.config3_inputs(torch.device("cuda", 0), 0)


@pytest.mark.parametrize("window", [0, 1024])
def test_config3_decode_rows_match_oracle(wb, config3, window):
    L, table, q, sink, pos = config3
    k, v = table[..., :C], table[..., C:]
    if window:
        empty = torch.empty(64, 1, 0, dtype=torch.int64, device=q.device)
        out = wb.sparse_attention(q, k, v, sink, empty, pos, C ** -0.5, window)
        _, lse = wb.forward_with_lse(q, k, v, pos, C ** -0.5, window=window, sink=sink)
    else:
        out, _ = wb.exact_attention(q, k, v, pos, C ** -0.5, 0, 128)
        _, lse = wb.forward_with_lse(q, k, v, pos, C ** -0.5)
    assert wb.device_status() == 0
    Lmax = int(L.max())
    ref_out, ref_lse = oat.range_attention(_f32(q), _f32(k[:, :Lmax]), _f32(v[:, :Lmax]), pos.cpu().numpy(),
                                           C ** -0.5, window=window, sink=_f32(sink) if window else None,
                                           dtype=np.float32)
    _close(out, lse, ref_out, ref_lse)  # all 64 rows


def _row_scores(q, k, position, scale):
    """(N,): each row's largest log-weight over the heads, the reference's
    selection score (pytorch_kernels.py:112-113), rows past `position` -inf."""
    z = (q.reshape(-1, q.shape[-1]).astype(np.float64) @ k.T.astype(np.float64)) * scale  # (H, N)
    z[:, position + 1:] = -np.inf
    m = z.max(-1, keepdims=True)
    lse = np.log(np.exp(z - m).sum(-1, keepdims=True)) + m
    return (z - lse).max(0)


def test_config3_top1024_choice_and_sparse_pass_match_oracle(wb, config3):
    L, table, q, sink, pos = config3
    k, v = table[..., :C], table[..., C:]
    top_k, window = 1024, 128
    out, chosen = wb.exact_attention(q, k, v, pos, C ** -0.5, top_k, window)
    sparse = wb.sparse_attention(q, k, v, sink, chosen, pos, C ** -0.5, 1024)
    assert wb.device_status() == 0
    assert chosen.shape == (64, 1, top_k)
    chosen_h = chosen.cpu().numpy()
    rows = [int(torch.argmax(L)), int(torch.argmin(L)), 0, 17, 63]
    for b in rows:
        p = int(pos[b, 0])
        score = _row_scores(_f32(q[b, 0]), _f32(k[b, :p + 1]), p, C ** -0.5)
        cand = score[:max(0, p - window + 1)]  # rows at least `window` back compete (:114-115)
        picked = chosen_h[b, 0]
        if len(cand) <= top_k:  # every candidate is chosen, the rest of the columns are -1
            assert sorted(picked[picked >= 0].tolist()) == list(range(len(cand)))
            assert (picked[len(cand):] == -1).all()
            continue
        kth = np.sort(cand)[::-1][top_k - 1]
        assert (picked >= 0).all() and len(set(picked.tolist())) == top_k
        assert (picked <= p - window).all()
        # the reference's rule: every pick weighs within 1e-2 (log) of the reference's own top_k-th
        assert (score[picked] >= kth - 1e-2).all()
    # the sparse pass over the GPU's own choice, against the oracle over the same rows
    idx = chosen_h[rows][:, :, :]
    ref_out, ref_lse = oat.sparse_attention(_f32(q[rows]), _f32(k[rows]), _f32(v[rows]), _f32(sink), idx,
                                            pos[rows].cpu().numpy(), C ** -0.5, 1024, dtype=np.float32)
    _close(sparse[rows], None, ref_out, None)
    ref_exact, _ = oat.range_attention(_f32(q[rows]), _f32(k[rows]), _f32(v[rows]), pos[rows].cpu().numpy(),
                                       C ** -0.5, dtype=np.float32)
    _close(out[rows], None, ref_exact, None)


def test_config4_tree_verification_matches_oracle(wb):
    t4, q4, cl, parents, depth = bench.config4_inputs(torch.device("cuda", 0), 0)
    out, lse = wb.tree_attention(q4, t4[..., :C], t4[..., C:], cl, torch.tensor(parents).cuda(), C ** -0.5)
    assert wb.device_status() == 0
    rows = [0, 13, 31]
    ref_out, ref_lse = oat.tree_attention(_f32(q4[rows]), _f32(t4[rows, :, :C]), _f32(t4[rows, :, C:]),
                                          cl[rows].cpu().numpy(), np.array(parents), C ** -0.5, dtype=np.float32)
    _close(out[rows], lse[rows], ref_out, ref_lse)
