"""The CPU oracle against the golden vectors the reference itself produced
(tests/golden/make_golden.py). This pins the oracle before any GPU result is
compared with it."""

import numpy as np
import torch

from oracle import accept as oa
from oracle import attention as oat


def _chosen_sets(chosen):
    return [[set(r[r >= 0].tolist()) for r in row] for row in chosen]


def test_exact_small_matches_reference(gold):
    d = gold("exact_small.npz")
    out, lse, chosen = oat.exact_attention(d["q"], d["k"], d["v"], d["positions"], float(d["scale"]),
                                           int(d["top_k"]), int(d["window"]))
    assert np.abs(out - d["out"]).max() < 1e-5
    assert np.abs(lse - d["lse"]).max() < 1e-5
    assert chosen.shape == d["chosen"].shape
    assert _chosen_sets(chosen) == _chosen_sets(d["chosen"])


def test_exact_generation_pass_matches_reference(gold):
    # ragged rows, one query past the table's last row, k/v halves of one table
    d = gold("exact_generation.npz")
    c = d["q"].shape[-1]
    e = d["entries"]
    out, lse, chosen = oat.exact_attention(d["q"], e[..., :c], e[..., c:], d["positions"], float(d["scale"]),
                                           int(d["top_k"]), int(d["window"]))
    assert np.abs(out - d["out"]).max() < 1e-5
    assert np.abs(lse - d["lse"]).max() < 1e-5
    assert _chosen_sets(chosen) == _chosen_sets(d["chosen"])


def test_sparse_small_matches_reference(gold):
    d = gold("sparse_small.npz")
    out, lse = oat.sparse_attention(d["q"], d["k"], d["v"], d["sink"], d["idx"], d["positions"], float(d["scale"]),
                                    int(d["window"]))
    assert np.abs(out - d["out"]).max() < 1e-5
    assert np.abs(lse - d["lse"]).max() < 1e-5


def test_window_attention_matches_reference(gold):
    d = gold("window_small.npz")
    out, _ = oat.window_attention(d["q"], d["k"], d["v"], d["sink"], d["positions"], float(d["scale"]),
                                  int(d["window"]))
    assert np.abs(out - d["out"]).max() < 1e-5


def _config1_inputs():
    g = torch.Generator().manual_seed(0)
    B, T, H, c = 2, 512, 8, 64
    q = torch.randn(B, T, H, c, generator=g).numpy()
    k = torch.randn(B, T, c, generator=g).numpy()
    v = torch.randn(B, T, c, generator=g).numpy()
    sink = (torch.randn(H, generator=g) * 0.5).numpy()
    return q, k, v, sink


def test_config1_window_exact_sparse_match_reference(gold):
    # B=2, T=512, 8 heads, c=64, window 128, fp32
    d = gold("config1.npz")
    q, k, v, sink = _config1_inputs()
    assert np.array_equal(sink, d["sink"])
    B, T, H, c = q.shape
    W, scale, keep = 128, c ** -0.5, slice(None, None, int(d["keep_step"]))
    positions = np.broadcast_to(np.arange(T), (B, T))
    tail = np.zeros((B, W - 1, c), np.float32)
    kt, vt = np.concatenate([tail, k], 1), np.concatenate([tail, v], 1)
    out, _ = oat.window_attention(q[:1], kt[:1], vt[:1], np.zeros(H), positions[:1], scale, W)
    assert np.abs(out[0, keep] - d["window_sink0"]).max() < 1e-5
    out, _ = oat.window_attention(q[:1], kt[:1], vt[:1], sink, positions[:1], scale, W)
    assert np.abs(out[0, keep] - d["window_sink"]).max() < 1e-5
    out, _, _ = oat.exact_attention(q[:1], k[:1], v[:1], positions[:1], scale, 0, W)
    assert np.abs(out[0, keep] - d["exact"]).max() < 1e-5
    out, _ = oat.sparse_attention(q[:1], k[:1], v[:1], sink, np.zeros((1, T, 0), np.int64), positions[:1], scale, W)
    assert np.abs(out[0, keep] - d["sparse_window"]).max() < 1e-5
    # the window pass equals the sparse pass over the same rows (tail rows are before the text)
    assert np.abs(d["window_sink"] - d["sparse_window"]).max() < 1e-5


def test_tree_attention_matches_reference_dense_and_chain(gold):
    d = gold("tree.npz")
    B, n = d["q"].shape[:2]
    L = int(d["cache_len"])
    out, _ = oat.tree_attention(d["q"], d["k"], d["v"], np.full(B, L), d["parents"], float(d["scale"]), d["sink"])
    assert np.abs(out - d["out_tree"]).max() < 1e-5
    chain = np.arange(n) - 1
    out, _ = oat.tree_attention(d["q"], d["k"], d["v"], np.full(B, L), chain, float(d["scale"]))
    assert np.abs(out - d["out_chain"]).max() < 1e-5


def test_merge_partials_equals_whole():
    rng = np.random.default_rng(0)
    B, T, H, c, N = 1, 3, 2, 8, 40
    q, k, v = rng.normal(size=(B, T, H, c)), rng.normal(size=(B, N, c)), rng.normal(size=(B, N, c))
    sink = rng.normal(size=H)
    positions = np.full((B, T), N - 1)
    whole, lse = oat.sparse_over_rows(q, k, v, sink, np.broadcast_to(np.arange(N), (B, T, N)), 0.3)
    parts = [np.arange(0, 13), np.arange(13, 29), np.arange(29, 40)]
    os_, ls_ = [], []
    for rows in parts:
        o, l = oat.sparse_over_rows(q, k, v, np.full(H, -np.inf), np.broadcast_to(rows, (B, T, len(rows))), 0.3)
        os_.append(o)
        ls_.append(l)
    merged, mlse = oat.merge_partials(np.stack(os_), np.stack(ls_), np.ones_like(np.stack(ls_)), sink)
    assert np.abs(merged - whole).max() < 1e-10 and np.abs(mlse - lse).max() < 1e-10
    del positions


def test_accept_matches_reference_writer(gold):
    # the reference's own Writer._speculate, with explicit draws, gave these
    for name in ("stochastic", "topk", "greedy"):
        d = gold(f"accept_{name}.npz")
        top_k = None if int(d["top_k"]) < 0 else int(d["top_k"])
        tokens, accepted = oa.accept(d["scores"], d["drafted"], d["q"], d["uniforms"], d["resample"],
                                     float(d["temperature"]), top_k)
        assert np.array_equal(accepted, d["accepted"]), name
        assert np.array_equal(tokens, d["tokens"]), name


def test_greedy_accept_is_argmax_agreement():
    rng = np.random.default_rng(1)
    R, n, V = 4, 5, 64
    scores = rng.normal(size=(R, n + 1, V)).astype(np.float32)
    q = oa.probabilities(rng.normal(size=(R, n, V)), 1.0, 1)
    drafted = scores[:, :n].argmax(-1)
    drafted[1, 2] = (drafted[1, 2] + 1) % V
    tokens, accepted = oa.accept(scores, drafted, q, rng.random((R, n)), rng.random(R), 1.0, 1)
    assert accepted.tolist() == [n, 2, n, n]
    assert tokens[1, 2] == scores[1, 2].argmax()


def test_range_attention_equals_exact_and_sparse_window():
    # the BLAS range path (the timed CPU baseline) against the two pinned restatements
    rng = np.random.default_rng(2)
    B, T, H, c, N = 2, 90, 3, 16, 130
    q, k, v = rng.normal(size=(B, T, H, c)), rng.normal(size=(B, N, c)), rng.normal(size=(B, N, c))
    sink = rng.normal(size=H)
    positions = np.stack([N - T + np.arange(T), 7 + np.arange(T)])
    out, lse = oat.range_attention(q, k, v, positions, 0.3)
    ref_out, ref_lse, _ = oat.exact_attention(q, k, v, positions, 0.3, 0, 0)
    assert np.abs(out - ref_out).max() < 1e-10 and np.abs(lse - ref_lse).max() < 1e-10
    out, lse = oat.range_attention(q, k, v, positions, 0.3, window=17, sink=sink)
    ref_out, ref_lse = oat.sparse_attention(q, k, v, sink, np.zeros((B, T, 0), np.int64), positions, 0.3, 17)
    assert np.abs(out - ref_out).max() < 1e-10 and np.abs(lse - ref_lse).max() < 1e-10


def _grad_case(d, name):
    return {key[len(name) + 1:]: d[key] for key in d.files if key.startswith(name + "_")}


def test_exact_backward_matches_reference_autograd(gold):
    from oracle import backward as ob
    g = _grad_case(gold("grads.npz"), "exact")
    dq, dk, dv = ob.exact_backward(g["q"], g["k"], g["v"], g["positions"], g["out"], g["lse"], g["d_out"],
                                   float(g["scale"]))
    for got, want in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())


def test_sparse_backward_matches_reference_autograd(gold):
    from oracle import backward as ob
    g = _grad_case(gold("grads.npz"), "sparse")
    dq, dk, dv, ds = ob.sparse_backward(g["q"], g["k"], g["v"], g["sink"], g["idx"], g["positions"], g["out"],
                                        g["lse"], g["d_out"], float(g["scale"]), int(g["window"]))
    for got, want in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"]), (ds, g["d_sink"])):
        assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())


def test_window_backward_matches_reference_autograd(gold):
    from oracle import backward as ob
    g = _grad_case(gold("grads.npz"), "window")
    out, lse = oat.window_attention(g["q"], g["k"], g["v"], g["sink"], g["positions"], float(g["scale"]),
                                    int(g["window"]))
    assert np.abs(out - g["out"]).max() < 1e-5
    dq, dk, dv, ds = ob.window_backward(g["q"], g["k"], g["v"], g["sink"], g["positions"], out, lse, g["d_out"],
                                        float(g["scale"]), int(g["window"]))
    for got, want in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"]), (ds, g["d_sink"])):
        assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())


def test_dense_attention_restatement_matches_the_tree_golden(gold):
    # the tree golden was made by the reference's own dense_attention
    # (attention.py:74-82) with a visible mask of the cache rows and each
    # node's ancestors; the generic restatement gives the same outputs
    d = gold("tree.npz")
    q, k, v, sink = d["q"], d["k"], d["v"], d["sink"]
    B, n = q.shape[:2]
    parents = np.broadcast_to(d["parents"], (B, n))
    for b in range(B):
        L = int(np.broadcast_to(np.asarray(d["cache_len"]).reshape(-1), (B,))[b])
        visible = np.concatenate([np.ones((n, L), bool), oat.ancestors_mask(parents[b])], 1)
        out, _ = oat.dense_attention(q[b], k[b, :L + n], v[b, :L + n], sink, visible, float(d["scale"]))
        assert np.abs(out - d["out_tree"][b]).max() < 1e-5


def test_drafter_visible_mask_follows_the_reference_formula():
    # place i reads the whole block, and context entry j when j > i (within
    # the window) and its position is not before the text (j >= window - L)
    vis = oat.drafter_visible([3, 200], 4, 8)
    assert vis.shape == (2, 4, 12)
    assert vis[:, :, :4].all()
    for r, L in enumerate([3, 200]):
        for i in range(4):
            for j in range(8):
                assert vis[r, i, 4 + j] == (j > i and j >= 8 - L)


def test_drafter_attention_restatement_matches_the_reference_backbone(gold):
    # drafter.npz: the reference's own Drafter.backbone, its first layer's
    # dense_attention call recorded (mask, table, output)
    d = gold("drafter.npz")
    lengths, W = d["lengths"], int(d["window"])
    count = d["q"].shape[1]
    assert np.array_equal(oat.drafter_visible(lengths, count, W), d["visible"])
    block = np.concatenate([d["k"][:, :count], d["v"][:, :count]], -1)
    context = np.concatenate([d["k"][:, count:], d["v"][:, count:]], -1)
    out, _ = oat.drafter_attention(d["q"], block, context, d["sink"], lengths, float(d["scale"]))
    assert np.abs(out - d["out"]).max() < 1e-5


def test_cache_append_restatement_matches_the_reference_rows(gold):
    from oracle import cache as oc
    d = gold("cache_append.npz")
    held, lengths = None, np.zeros(3, np.int64)
    for step in range(3):
        counts = d[f"counts{step}"]
        held, table = oc.cache_append(held, d[f"new{step}"], lengths, counts)
        assert table.shape == d[f"table{step}"].shape
        assert np.array_equal(table, d[f"table{step}"])
        lengths = lengths + counts


def test_head_scores_rounding_is_bf16_nearest_even():
    # the reference's head under bf16 autocast returns bf16 scores (model.py:471)
    from oracle import accept as oa
    x = np.array([[1.0, 3.14159265, -2.718281828, 1e-3, 65504.5, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8]])
    want = torch.tensor(x).float().bfloat16().float().numpy()
    assert np.array_equal(oa.head_scores(x, np.eye(x.shape[1])), want)
