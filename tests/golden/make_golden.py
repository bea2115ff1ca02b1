"""Writes the golden fixtures under tests/golden/ by running the REFERENCE's
own code (imported from the reference checkout named by --reference or the
WPT_REFERENCE environment variable) on seeded inputs. Run once, in a machine
that has the reference; the fixtures are committed and the tests read only
them:

    python tests/golden/make_golden.py --reference <the reference repository>

What each fixture pins (paths relative to the reference repository):
  cache_append.npz      the generation cache's entries table after ragged reads,
                        through the reference's Rows/Reading (cache.py:54-134)
  grads.npz             gradients from the reference's autograd: exact attention
                        (pytorch_kernels.py:123-139), sparse attention with a
                        sink (:189-210), window_attention (attention.py:85-107)
  exact_small.npz       pytorch_kernels.exact_attention (+ top-k choice, LSE
                        read from the autograd node's saved tensors),
                        packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-146
  exact_generation.npz  the same on a generation pass: ragged rows, a query past
                        the table, k/v halves of one entries table
                        (tests/test_triton_kernels.py:51-77's case)
  sparse_small.npz      pytorch_kernels.sparse_attention, :171-217
  window_small.npz      attention.window_attention with WINDOW patched to 8,
                        attention.py:85-107
  config1.npz           BASELINE config 1 (B=2, T=512, H=8, c=64, window 128,
                        fp32): window_attention (sink 0 and sink ~ N(0, .5)),
                        causal exact_attention, sparse_attention with no chosen
                        rows; a strided subset of row 0's queries is stored
  tree.npz              attention.dense_attention with an ancestor mask
                        (attention.py:74-82), and exact_attention for a chain
  drafter.npz           the drafter backbone's attention: Drafter.backbone's
                        visible mask and dense_attention call (drafter.py:141-151,
                        179-204) on a tiny random model
  accept_*.npz          wpt_inference.Writer._speculate (__init__.py:196-233)
                        with a fake model and drafter, torch.rand and
                        torch.multinomial replaced by explicit draws
"""

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root):
    for package in ("wpt-model", "wpt-utils", "wpt-inference"):
        sys.path.insert(0, os.path.join(root, "packages", package, "src"))
    from wpt_model import attention, pytorch_kernels  # noqa: E402
    import wpt_inference  # noqa: E402
    return attention, pytorch_kernels, wpt_inference


def _np(x):
    return x.detach().cpu().numpy()


def _lse_of(out):
    """The LSE the reference's _Exact/_Sparse saved for its backward pass."""
    return _np(out.grad_fn.saved_tensors[-1])


def _inputs(B, T, H, c, N, seed):
    g = torch.Generator().manual_seed(seed)

    def rand(*shape):
        return torch.randn(*shape, generator=g).requires_grad_()
    positions = (N - T + torch.arange(T)).expand(B, T).contiguous()
    return rand(B, T, H, c), rand(B, N, c), rand(B, N, c), rand(H), positions


def exact_small(pk):
    q, k, v, _, positions = _inputs(2, 30, 3, 16, 50, 0)
    out, chosen = pk.exact_attention(q, k, v, positions, 0.3, 5, 8)
    np.savez(os.path.join(HERE, "exact_small.npz"), q=_np(q), k=_np(k), v=_np(v), positions=_np(positions),
             scale=0.3, top_k=5, window=8, out=_np(out), lse=_lse_of(out), chosen=_np(chosen))


def exact_generation(pk):
    g = torch.Generator().manual_seed(0)
    B, T, H, c, N, top_k, window = 3, 4, 4, 32, 60, 8, 4
    q = torch.randn(B, T, H, c, generator=g).requires_grad_()
    entries = torch.randn(B, N, 2 * c, generator=g)
    k, v = entries[..., :c], entries[..., c:]
    positions = torch.tensor([[56, 57, 58, 59], [20, 21, 22, 23], [58, 59, 60, 61]])
    out, chosen = pk.exact_attention(q, k, v, positions, c ** -0.5, top_k, window)
    np.savez(os.path.join(HERE, "exact_generation.npz"), q=_np(q), entries=_np(entries), positions=_np(positions),
             scale=c ** -0.5, top_k=top_k, window=window, out=_np(out), lse=_lse_of(out), chosen=_np(chosen))


def sparse_small(pk):
    q, k, v, sink, positions = _inputs(2, 30, 3, 16, 50, 1)
    g = torch.Generator().manual_seed(2)
    idx = torch.stack([torch.stack([torch.randperm(int(p) - 4, generator=g)[:6] if int(p) >= 10
                                    else torch.full((6,), -1) for p in row]) for row in positions])
    idx[:, ::3, -2:] = -1
    out = pk.sparse_attention(q, k, v, sink, idx, positions, 0.3, 5)
    np.savez(os.path.join(HERE, "sparse_small.npz"), q=_np(q), k=_np(k), v=_np(v), sink=_np(sink), idx=_np(idx),
             positions=_np(positions), scale=0.3, window=5, out=_np(out), lse=_lse_of(out))


def grads(at, pk):
    """Gradients of the reference's autograd: exact attention (the backward
    of pytorch_kernels.py:123-139) on a causal pass and a generation pass,
    sparse attention with chosen rows, -1 padding and a sink
    (:189-210), and window_attention (attention.py:85-107, plain autograd),
    each with a seeded d_out."""
    g = torch.Generator().manual_seed(11)
    cases = {}
    # exact, causal prefill with ragged positions in row 1
    B, T, H, c, N = 2, 40, 4, 16, 40
    q = torch.randn(B, T, H, c, generator=g).requires_grad_()
    k = torch.randn(B, N, c, generator=g).requires_grad_()
    v = torch.randn(B, N, c, generator=g).requires_grad_()
    positions = torch.stack([torch.arange(T), torch.clamp(torch.arange(T) - 5, min=0)])
    d_out = torch.randn(B, T, H, c, generator=g)
    out, _ = pk.exact_attention(q, k, v, positions, 0.3, 0, 8)
    lse = _lse_of(out)
    out.backward(d_out)
    cases["exact"] = dict(q=_np(q), k=_np(k), v=_np(v), positions=_np(positions), scale=0.3, d_out=_np(d_out),
                          out=_np(out), lse=lse, dq=_np(q.grad), dk=_np(k.grad), dv=_np(v.grad))
    # sparse: chosen rows (some -1) plus the last `window` rows, with a sink
    B, T, H, c, N, W = 2, 24, 4, 16, 60, 6
    q = torch.randn(B, T, H, c, generator=g).requires_grad_()
    k = torch.randn(B, N, c, generator=g).requires_grad_()
    v = torch.randn(B, N, c, generator=g).requires_grad_()
    sink = (torch.randn(H, generator=g) * 0.5).requires_grad_()
    positions = (N - T + torch.arange(T)).expand(B, T).contiguous()
    idx = torch.stack([torch.stack([torch.randperm(int(p) - W + 1, generator=g)[:7] for p in row])
                       for row in positions])
    idx[:, ::4, -3:] = -1
    d_out = torch.randn(B, T, H, c, generator=g)
    out = pk.sparse_attention(q, k, v, sink, idx, positions, 0.25, W)
    lse = _lse_of(out)
    out.backward(d_out)
    cases["sparse"] = dict(q=_np(q), k=_np(k), v=_np(v), sink=_np(sink), idx=_np(idx), positions=_np(positions),
                           scale=0.25, window=W, d_out=_np(d_out), out=_np(out), lse=lse, dq=_np(q.grad),
                           dk=_np(k.grad), dv=_np(v.grad), d_sink=_np(sink.grad))
    # window_attention's tail layout, through plain autograd
    W, B, T, H, c = 8, 2, 20, 3, 16
    q = torch.randn(B, T, H, c, generator=g).requires_grad_()
    k = torch.randn(B, W - 1 + T, c, generator=g).requires_grad_()
    v = torch.randn(B, W - 1 + T, c, generator=g).requires_grad_()
    sink = (torch.randn(H, generator=g) * 0.5).requires_grad_()
    positions = torch.stack([3 + torch.arange(T), 40 + torch.arange(T)])
    d_out = torch.randn(B, T, H, c, generator=g)
    saved = at.WINDOW
    at.WINDOW = W
    try:
        out = at.window_attention(q, k, v, sink, positions, 0.25)
    finally:
        at.WINDOW = saved
    out.backward(d_out)
    cases["window"] = dict(q=_np(q), k=_np(k), v=_np(v), sink=_np(sink), positions=_np(positions), scale=0.25,
                           window=W, d_out=_np(d_out), out=_np(out), dq=_np(q.grad), dk=_np(k.grad),
                           dv=_np(v.grad), d_sink=_np(sink.grad))
    np.savez(os.path.join(HERE, "grads.npz"), **{f"{case}_{key}": value for case, d in cases.items()
                                                 for key, value in d.items()})


def cache_append(root):
    """The generation cache's entries of an exact layer through the
    reference's own Rows/Reading (cache.py:54-134, Reading.everything
    :110-128): a prompt of ragged counts, then two extends that grow the
    table and write each row at its own length."""
    from wpt_model.cache import Rows
    from wpt_model.carry import Entries

    class Layer:  # a module that passes on one entries table, as ExactAttention does
        def passes_on(self):
            return {"entries": Entries()}

    g = torch.Generator().manual_seed(21)
    B, width = 3, 16
    layer, rows = Layer(), Rows(B, torch.device("cpu"))
    steps = {}
    for step, counts in enumerate(([5, 2, 7], [1, 4, 0], [9, 1, 3])):
        counts = torch.tensor(counts)
        n = int(counts.max())
        new = torch.randn(B, n, width, generator=g)
        reading = rows.reading(counts, undoable=False)
        table = reading.everything(layer, "entries", new)
        reading.finish()
        steps.update({f"new{step}": _np(new).copy(), f"counts{step}": _np(counts).copy(),
                      f"table{step}": _np(table).copy()})  # copies: later reads write the held table in place
    np.savez(os.path.join(HERE, "cache_append.npz"), **steps)


def drafter():
    """The drafter backbone's attention through the reference's own
    Drafter.backbone (drafter.py:179-204: the visible mask of :189-195, each
    layer's DrafterLayer.attend of :141-151) on a tiny random model on the
    CPU: what its dense_attention receives (queries, the [block; context]
    table's keys and values, sink, visible mask, scale) and returns, for the
    first layer call. Contexts partly before the text included."""
    from types import SimpleNamespace

    import torch.nn as nn
    from wpt_model import drafter as dr
    from wpt_model.config import ModelConfig

    torch.manual_seed(31)
    config = ModelConfig(vocab_size=64, block_size=16, window_layers=1, sparse_groups=1, sparse_layers=1,
                         d_model=32, attention_heads=4, attention_head_dim=64, n_experts=4, top_k=2,
                         expert_width=16, latent_width=16, shared_width=32, engram_layers=(), engram_order=2,
                         engram_heads=1, engram_dim=8, engram_table_size=97, residual_groups=2)
    drafter = dr.Drafter(config, dr.DrafterConfig(features=(1,), layers=1, block=4, markov_rank=4)).eval()
    model = SimpleNamespace(embedding=nn.Embedding(config.vocab_size, config.d_model),
                            head=nn.Linear(config.d_model, config.vocab_size, bias=False))
    calls = []
    inner = dr.dense_attention

    def recording(q, k, v, sink, visible, scale):
        out = inner(q, k, v, sink, visible, scale)
        calls.append({"q": _np(q).copy(), "k": _np(k).copy(), "v": _np(v).copy(), "sink": _np(sink).copy(),
                      "visible": _np(visible).copy(), "scale": np.float64(scale), "out": _np(out).copy()})
        return out

    lengths = torch.tensor([3, 50, 127, 128, 500])
    R, count = len(lengths), 4
    context = torch.randn(R, dr.WINDOW, config.d_model)
    anchors = torch.randint(0, config.vocab_size, (R,))
    dr.dense_attention = recording
    try:
        with torch.no_grad():
            drafter.backbone(model, context, lengths, anchors, count)
    finally:
        dr.dense_attention = inner
    np.savez(os.path.join(HERE, "drafter.npz"), lengths=_np(lengths), window=np.int64(dr.WINDOW), **calls[0])


def window_small(at):
    g = torch.Generator().manual_seed(3)
    W, B, T, H, c = 8, 2, 20, 3, 16
    q = torch.randn(B, T, H, c, generator=g)
    k = torch.randn(B, W - 1 + T, c, generator=g)
    v = torch.randn(B, W - 1 + T, c, generator=g)
    sink = torch.randn(H, generator=g) * 0.5
    positions = torch.stack([3 + torch.arange(T), 40 + torch.arange(T)])  # row 0 starts near the text's start
    saved = at.WINDOW
    at.WINDOW = W
    try:
        out = at.window_attention(q, k, v, sink, positions, 0.25)
    finally:
        at.WINDOW = saved
    np.savez(os.path.join(HERE, "window_small.npz"), q=_np(q), k=_np(k), v=_np(v), sink=_np(sink),
             positions=_np(positions), scale=0.25, window=W, out=_np(out))


def config1(at, pk):
    """BASELINE config 1; a strided subset of row 0's queries is stored."""
    g = torch.Generator().manual_seed(0)
    B, T, H, c, W = 2, 512, 8, 64, 128
    q = torch.randn(B, T, H, c, generator=g)
    k = torch.randn(B, T, c, generator=g)
    v = torch.randn(B, T, c, generator=g)
    sink = torch.randn(H, generator=g) * 0.5
    positions = torch.arange(T).expand(B, T).contiguous()
    scale = c ** -0.5
    tail = torch.zeros(B, W - 1, c)
    kt, vt = torch.cat([tail, k], 1), torch.cat([tail, v], 1)
    keep = slice(None, None, 8)
    results = {}
    with torch.no_grad():
        results["window_sink0"] = at.window_attention(q, kt, vt, torch.zeros(H), positions, scale)
        results["window_sink"] = at.window_attention(q, kt, vt, sink, positions, scale)
        results["exact"], _ = pk.exact_attention(q, k, v, positions, scale, 0, W)
        empty = torch.zeros(B, T, 0, dtype=torch.long)
        results["sparse_window"] = pk.sparse_attention(q, k, v, sink, empty, positions, scale, W)
    np.savez(os.path.join(HERE, "config1.npz"), seed=0, sink=_np(sink), keep_step=8,
             **{name: _np(x[0, keep]) for name, x in results.items()})


def tree(at, pk):
    g = torch.Generator().manual_seed(4)
    B, L, n, H, c = 2, 40, 7, 4, 32
    q = torch.randn(B, n, H, c, generator=g)
    k = torch.randn(B, L + n + 3, c, generator=g)  # 3 stale rows past the tree
    v = torch.randn(B, L + n + 3, c, generator=g)
    sink = torch.randn(H, generator=g) * 0.5
    parents = torch.tensor([-1, 0, 0, 1, 1, 2, 4])
    seen = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        j = i
        while j >= 0:
            seen[i, j] = True
            j = int(parents[j])
    visible = torch.cat([torch.ones(n, L, dtype=torch.bool), seen], 1)
    scale = c ** -0.5
    out_tree = at.dense_attention(q, k[:, :L + n], v[:, :L + n], sink, visible.expand(B, n, L + n), scale)
    positions = (L + torch.arange(n)).expand(B, n).contiguous()
    out_chain, _ = pk.exact_attention(q, k, v, positions, scale, 0, 1)
    np.savez(os.path.join(HERE, "tree.npz"), q=_np(q), k=_np(k), v=_np(v), sink=_np(sink), parents=_np(parents),
             cache_len=L, scale=scale, out_tree=_np(out_tree), out_chain=_np(out_chain))


class _FakeModel(torch.nn.Module):
    """Hands the Writer fixed target scores for one speculative step."""

    def __init__(self, scores):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.zeros(1))
        self.scores = scores
        self.kept = None

    def new_cache(self, rows, routes=False):
        return _FakeCache(rows)

    def extend(self, ids, cache, counts, undoable=False, features=()):
        return (self.scores[:, :ids.shape[1]],)

    def undo(self, cache, kept):
        self.kept = list(kept)


class _FakeCache:
    def __init__(self, rows):
        self.lengths = torch.zeros(rows, dtype=torch.long)

    def select(self, index):
        return _FakeCache(len(index))


class _FakeDrafter:
    features, window = (), 0

    def __init__(self, tokens, q):
        self.tokens, self.q = tokens, q

    def draft(self, model, histories, context, count, probabilities, generator):
        return self.tokens[:, :count], self.q[:, :count], None


def accept_case(wi, name, R, n, V, temperature, top_k, seed):
    g = torch.Generator().manual_seed(seed)
    scores = torch.randn(R, n + 1, V, generator=g) * 2.0
    q_logits = torch.randn(R, n, V, generator=g) * 2.0
    # half of the rows draft near the target (many accepted), half far (early rejections)
    q_logits[: R // 2] = scores[: R // 2, :n] + 0.3 * q_logits[: R // 2]
    writer_probs = wi.Writer.__dict__["_probabilities"]

    class _P:
        pass
    holder = _P()
    holder.temperature, holder.top_k = temperature, top_k
    q = writer_probs(holder, q_logits)
    drafted = torch.multinomial(q.reshape(-1, V), 1, generator=g).view(R, n)
    uniforms = torch.rand(R, n, generator=g)
    resample = torch.rand(R, generator=g)

    state = {"row": 0, "j": 0}
    real_rand, real_multinomial = torch.rand, torch.multinomial

    def rand(*args, **kwargs):
        u = uniforms[state["row"], state["j"]].clone()
        state["j"] += 1
        return u

    def multinomial(weights, num, generator=None):
        cs = torch.cumsum(weights.double(), -1)
        target = float(resample[state["row"]]) * float(cs[-1])
        token = min(int(torch.searchsorted(cs, torch.tensor([target], dtype=torch.float64), right=True)), V - 1)
        state["row"] += 1
        state["j"] = 0
        return torch.tensor([token])

    model = _FakeModel(scores)
    writer = wi.Writer(model, [1], R, temperature=temperature, top_k=top_k, generator=torch.Generator(),
                       drafter=_FakeDrafter(drafted, q), draft=n)
    torch.rand, torch.multinomial = rand, multinomial
    try:
        written = writer.write({}, {row: n + 10 for row in range(R)})
    finally:
        torch.rand, torch.multinomial = real_rand, real_multinomial
    tokens = np.full((R, n + 1), -1, np.int64)
    for row, toks in written.items():
        tokens[row, :len(toks)] = toks
    accepted = np.array([len(written[row]) - 1 for row in range(R)], np.int64)
    np.savez(os.path.join(HERE, f"accept_{name}.npz"), scores=_np(scores), q=_np(q), drafted=_np(drafted),
             uniforms=_np(uniforms), resample=_np(resample), temperature=temperature,
             top_k=-1 if top_k is None else top_k, tokens=tokens, accepted=accepted,
             kept=np.array(model.kept, np.int64))


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("WPT_REFERENCE"), required="WPT_REFERENCE" not in os.environ,
                        help="the reference repository's root (or set WPT_REFERENCE)")
    parser.add_argument("--only", default=None, help="comma-separated fixtures to write (default: all)")
    args = parser.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    at, pk, wi = _import_reference(args.reference)
    if args.only:
        for name in args.only.split(","):
            {"grads": lambda: grads(at, pk), "cache_append": lambda: cache_append(args.reference),
             "drafter": drafter}[name]()
        return
    grads(at, pk)
    cache_append(args.reference)
    drafter()
    exact_small(pk)
    exact_generation(pk)
    sparse_small(pk)
    window_small(at)
    config1(at, pk)
    tree(at, pk)
    accept_case(wi, "stochastic", R=8, n=6, V=1000, temperature=1.0, top_k=None, seed=5)
    accept_case(wi, "topk", R=8, n=6, V=1000, temperature=0.8, top_k=40, seed=6)
    accept_case(wi, "greedy", R=8, n=6, V=1000, temperature=1.0, top_k=1, seed=7)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
