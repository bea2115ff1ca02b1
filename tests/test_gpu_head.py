"""The output head's product and the writer's sampling step from it (SURVEY
F3; packages/wpt-model/src/wpt_model/model.py:267,471 the head,
packages/wpt-inference/src/wpt_inference/__init__.py:173-182 the sampling)
on the GPU: the tcgen05 head kernel against the float64 oracle (oracle.accept
.head_scores), rounded to bf16 as the reference's autocast head returns its
scores (each score within half a bf16 step of the exact product, plus the
fp32 accumulation's error) and unrounded (within 1e-4 of the product's
scale), over one and several 128-row launches, ragged vocabulary tiles and
the config-5 decode shape (64 rows, width 2,048, vocabulary 65,536); then
head_sample's tokens equal the oracle's draw over the kernel's own scores."""

import numpy as np
import pytest
import torch

from oracle import accept as oa

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def _case(R, D, V, seed):
    g = torch.Generator().manual_seed(seed)
    h = (torch.randn(R, D, generator=g)).bfloat16()
    w = (torch.randn(V, D, generator=g) * D ** -0.5).bfloat16()
    return h, w


def _exact(h, w):
    return oa.head_scores(h.float().numpy(), w.float().numpy(), round_bf16=False).astype(np.float64)


@pytest.mark.parametrize("R,D,V", [(64, 2048, 65536), (37, 256, 1000), (130, 128, 777), (1, 64, 129)])
def test_head_scores_match_the_oracle(wb, R, D, V):
    from wpt_b200 import ops
    h, w = _case(R, D, V, seed=R + D + V)
    exact = _exact(h, w)
    got = ops.head_scores(h.cuda(), w.cuda()).cpu().numpy().astype(np.float64)
    assert wb.device_status() == 0
    # bf16 rounding: half a step (2^-8 relative), plus fp32 accumulation over D products
    assert (np.abs(got - exact) <= np.abs(exact) * 2.0 ** -8 + 1e-4).all()
    raw = ops.head_scores(h.cuda(), w.cuda(), round_bf16=False).cpu().numpy().astype(np.float64)
    assert np.abs(raw - exact).max() < 1e-4
    # rounding the kernel's own fp32 products to bf16 (nearest even) gives exactly its rounded scores
    assert np.array_equal(torch.from_numpy(raw).float().bfloat16().float().numpy(), got.astype(np.float32))


@pytest.mark.parametrize("temperature,top_k", [(1.0, None), (0.8, 40), (1.0, 1)])
def test_head_sample_draws_from_its_scores(wb, temperature, top_k):
    R, D, V = 64, 2048, 65536
    h, w = _case(R, D, V, seed=7)
    resample = torch.rand(R, generator=torch.Generator().manual_seed(8))
    tokens, scores = wb.head_sample(h.cuda(), w.cuda(), resample.cuda(), temperature, top_k)
    assert wb.device_status() == 0
    s = scores.cpu().numpy()
    assert (np.abs(s.astype(np.float64) - _exact(h, w)) <= np.abs(_exact(h, w)) * 2.0 ** -8 + 1e-4).all()
    want, accepted = oa.accept(s[:, None], np.zeros((R, 0), np.int64), np.zeros((R, 0, V), np.float32),
                               np.zeros((R, 0), np.float32), resample.numpy(), temperature, top_k)
    assert np.array_equal(tokens.cpu().numpy(), want[:, 0])
    if top_k == 1:  # a maximum (bf16 scores tie often; the reference's top-1 mask keeps ties and draws among them)
        assert np.array_equal(s[np.arange(R), tokens.cpu().numpy()], s.max(-1))
