"""The drop-in on the reference's own model code: with this library
installed as WPT's attention form (wpt_b200.install: the reference's
kernels._try check on this module, then its exact, sparse and window layers
on these kernels), each kind of attention layer read through a generation
cache in pieces gives what the same layer gives over the whole text in the
reference's PyTorch form, within the 3e-2 share of the largest output the
reference's own tests allow a GPU form (packages/wpt-model/tests/
test_cache.py:71,75-101). The whole model (WPT.extend, model.py:456-473)
runs through the cache on these kernels with finite scores; its scores are
not compared across forms because, as the reference's test_cache.py:120-126
says, bf16 rounding sends some tokens of a random model to other experts.

Needs the reference installed in baseline/_ref (baseline/install_ref.py);
skipped without it."""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "wpt_model")),
                                 reason="the reference is not installed in baseline/_ref")]

# a prompt, single tokens, a few, a long piece and the rest: 300 tokens, past
# the window (128), pieces ending inside and across the window's blocks
PIECES = [37, 1, 1, 5, 100, 1, 155]


def _reference():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    from wpt_model import WPT, ModelConfig, attention, kernels
    from wpt_model.cache import Rows
    from wpt_model.sequence import WHOLE
    return WPT, ModelConfig, attention, kernels, Rows, WHOLE


def _config(ModelConfig):
    return ModelConfig(vocab_size=50, block_size=16, window_layers=1, sparse_groups=1, sparse_layers=2, d_model=64,
                       attention_heads=4, attention_head_dim=128, n_experts=4, top_k=2, expert_width=8,
                       latent_width=8, shared_width=16, engram_layers=[2], engram_order=3, engram_heads=2,
                       engram_dim=4, engram_table_size=31, residual_groups=3)


def _randomized(module):
    torch.manual_seed(1)
    with torch.no_grad():
        for p in module.parameters():  # the zero-started parameters (sinks, ...) made to count
            if p.abs().max() == 0:
                p.normal_(std=0.5)
    return module


def _in_pieces(Rows, read, x):
    """read(piece, reading) over x (B, T, ...) piece by piece, each piece
    read through a cache's rows; the outputs joined."""
    rows, out, start = Rows(x.shape[0], x.device), [], 0
    for size in PIECES:
        reading = rows.reading(torch.full((x.shape[0],), size, device=x.device), undoable=False)
        out.append(read(x[:, start:start + size], reading))
        reading.finish()
        start += size
    return torch.cat(out, 1)


@pytest.fixture
def reference():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    WPT, ModelConfig, attention, kernels, Rows, WHOLE = _reference()
    saved = (attention.TOP_K, attention.window_attention, kernels._kernels, kernels._form)
    attention.TOP_K = 16  # exact layers pick 16 rows, so that the choice matters within 300 tokens
    try:
        yield wpt_b200, WPT, _config(ModelConfig), attention, kernels, Rows, WHOLE
    finally:
        attention.TOP_K, attention.window_attention, kernels._kernels, kernels._form = saved


def _share(got, want):
    return ((got.float() - want.float()).abs().max() / want.float().abs().max()).item()


def test_window_layer_through_the_cache_matches_the_pytorch_form(reference):
    wb, WPT, config, attention, kernels, Rows, WHOLE = reference
    torch.manual_seed(0)
    layer = _randomized(attention.WindowAttention(config)).eval().cuda()
    x = torch.randn(2, sum(PIECES), config.d_model, device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        kernels._kernels, kernels._form = None, "pytorch"
        want = layer(x, WHOLE)
        wb.install(kernels, attention)
        got = _in_pieces(Rows, lambda piece, reading: layer(piece, reading), x)
        whole = layer(x, WHOLE)
    assert wb.device_status() == 0
    assert _share(got, want) <= 3e-2 and _share(whole, want) <= 3e-2


def test_exact_and_sparse_layers_through_the_cache_match_the_pytorch_form(reference):
    wb, WPT, config, attention, kernels, Rows, WHOLE = reference
    torch.manual_seed(0)
    exact, sparse = (_randomized(kind(config)).eval().cuda()
                     for kind in (attention.ExactAttention, attention.SparseAttention))
    x = torch.randn(2, sum(PIECES), config.d_model, device="cuda")

    def both(piece, place):
        out, handoff = exact(piece, piece, place)
        return torch.cat([out, sparse(piece, handoff, place)], -1)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        kernels._kernels, kernels._form = None, "pytorch"
        want = both(x, WHOLE)
        wb.install(kernels, attention)
        got = _in_pieces(Rows, both, x)
        whole = both(x, WHOLE)
    assert wb.device_status() == 0
    assert _share(got, want) <= 3e-2 and _share(whole, want) <= 3e-2


def test_the_whole_model_generates_through_this_form(reference):
    wb, WPT, config, attention, kernels, Rows, WHOLE = reference
    torch.manual_seed(0)
    model = _randomized(WPT(config)).eval().cuda()
    ids = torch.randint(config.vocab_size, (2, sum(PIECES)), generator=torch.Generator().manual_seed(1)).cuda()
    wb.install(kernels, attention)  # runs kernels._try on this module first
    assert kernels.kernels(ids.device) is wb
    cache = model.new_cache(2)
    start = 0
    for size in PIECES:
        scores, _ = model.extend(ids[:, start:start + size], cache)
        assert scores.shape == (2, size, config.vocab_size) and torch.isfinite(scores).all()
        start += size
    assert cache.lengths.tolist() == [sum(PIECES)] * 2
    assert wb.device_status() == 0
