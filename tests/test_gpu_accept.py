"""The acceptance step on the GPU (wpt_inference/__init__.py:173-179,210-222):
accepted counts and tokens bit-exact against the reference's own
Writer._speculate (the golden fixtures, made with explicit draws) and
against the CPU oracle at BASELINE config 4's shape (32 rows, 16 drafts,
vocabulary 65536, logits ~ N(0, 2)): stochastic, greedy (top_k 1) and top_k
40 at temperature 0.8, and rows verifying fewer drafts."""

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


@pytest.mark.parametrize("name", ["stochastic", "topk", "greedy"])
def test_accept_matches_reference_writer(wb, gold, name):
    d = gold(f"accept_{name}.npz")
    top_k = None if int(d["top_k"]) < 0 else int(d["top_k"])
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    tokens, accepted = wb.accept(dev(d["scores"]), dev(d["drafted"]), dev(d["q"]), dev(d["uniforms"]),
                                 dev(d["resample"]), float(d["temperature"]), top_k)
    assert np.array_equal(accepted.cpu().numpy(), d["accepted"])
    assert np.array_equal(tokens.cpu().numpy(), d["tokens"])


def _config4(seed, temperature, top_k, near=True):
    g = torch.Generator().manual_seed(seed)
    R, n, V = 32, 16, 65536
    scores = torch.randn(R, n + 1, V, generator=g) * 2.0
    q_logits = torch.randn(R, n, V, generator=g) * 2.0
    if near:  # half of the rows draft close to the target, so that drafts are kept
        q_logits[: R // 2] = scores[: R // 2, :n] + 0.3 * q_logits[: R // 2]
    q = torch.from_numpy(oa.probabilities(q_logits.numpy(), temperature, top_k))
    drafted = torch.multinomial(q.reshape(-1, V), 1, generator=g).view(R, n)
    uniforms = torch.rand(R, n, generator=g)
    resample = torch.rand(R, generator=g)
    return scores, drafted, q, uniforms, resample


@pytest.mark.parametrize("temperature,top_k", [(1.0, None), (1.0, 1), (0.8, 40)])
def test_accept_matches_oracle_at_config4(wb, temperature, top_k):
    scores, drafted, q, uniforms, resample = _config4(4, temperature, top_k)
    tokens, accepted = wb.accept(scores.cuda(), drafted.cuda(), q.cuda(), uniforms.cuda(), resample.cuda(),
                                 temperature, top_k)
    ref_tokens, ref_accepted = oa.accept(scores.numpy(), drafted.numpy(), q.numpy(), uniforms.numpy(),
                                         resample.numpy(), temperature, top_k)
    assert np.array_equal(accepted.cpu().numpy(), ref_accepted)
    assert np.array_equal(tokens.cpu().numpy(), ref_tokens)
    assert ref_accepted.max() > 0 and ref_accepted.min() < 16  # both outcomes exercised


def test_rows_verifying_fewer_drafts(wb):
    scores, drafted, q, uniforms, resample = _config4(5, 1.0, None)
    lengths = torch.randint(0, 17, (32,), generator=torch.Generator().manual_seed(6))
    tokens, accepted = wb.accept(scores.cuda(), drafted.cuda(), q.cuda(), uniforms.cuda(), resample.cuda(), 1.0,
                                 None, lengths=lengths.cuda())
    ref_tokens, ref_accepted = oa.accept(scores.numpy(), drafted.numpy(), q.numpy(), uniforms.numpy(),
                                         resample.numpy(), 1.0, None, lengths=lengths.numpy())
    assert np.array_equal(accepted.cpu().numpy(), ref_accepted)
    assert np.array_equal(tokens.cpu().numpy(), ref_tokens)


@pytest.mark.parametrize("V,temperature", [(1000, 1.0), (50257, 0.7), (152067, 1.0), (4096, 1.3)])
def test_vocabularies_of_any_size(wb, V, temperature):
    """Vocabularies that are not a multiple of the statistics segment, the
    draw chunk or four entries (the scalar path), with masked (-inf) logits."""
    g = torch.Generator().manual_seed(V)
    R, n = 6, 5
    scores = torch.randn(R, n + 1, V, generator=g) * 2.0
    scores[:, :, V // 3: V // 3 + 17] = float("-inf")
    q_logits = scores[:, :n] + 0.5 * torch.randn(R, n, V, generator=g)
    q = torch.from_numpy(oa.probabilities(q_logits.numpy(), temperature, None))
    drafted = torch.multinomial(q.reshape(-1, V), 1, generator=g).view(R, n)
    uniforms = torch.rand(R, n, generator=g)
    resample = torch.rand(R, generator=g)
    tokens, accepted = wb.accept(scores.cuda(), drafted.cuda(), q.cuda(), uniforms.cuda(), resample.cuda(),
                                 temperature, None)
    ref_tokens, ref_accepted = oa.accept(scores.numpy(), drafted.numpy(), q.numpy(), uniforms.numpy(),
                                         resample.numpy(), temperature, None)
    assert np.array_equal(accepted.cpu().numpy(), ref_accepted)
    assert np.array_equal(tokens.cpu().numpy(), ref_tokens)
    assert wb.device_status() == 0


@pytest.mark.parametrize("V,top_k,tied", [(1000, 5, False), (65536, 1500, False), (65536, 40, True),
                                          (32000, 200, False)])
def test_top_k_thresholds(wb, V, top_k, tied):
    """The top-k threshold's paths: a bound from the thread maxima and a
    sort of the few entries above it; and the radix passes over the whole
    row when top_k exceeds the thread count or thousands of entries tie
    (logits rounded to halves) at the bound."""
    g = torch.Generator().manual_seed(top_k)
    R, n = 4, 6
    scores = torch.randn(R, n + 1, V, generator=g) * 2.0
    if tied:
        scores = torch.round(scores * 2.0) / 2.0
    q_logits = scores[:, :n] + 0.5 * torch.randn(R, n, V, generator=g)
    q = torch.from_numpy(oa.probabilities(q_logits.numpy(), 0.9, top_k))
    drafted = torch.multinomial(q.reshape(-1, V), 1, generator=g).view(R, n)
    uniforms = torch.rand(R, n, generator=g)
    resample = torch.rand(R, generator=g)
    tokens, accepted = wb.accept(scores.cuda(), drafted.cuda(), q.cuda(), uniforms.cuda(), resample.cuda(),
                                 0.9, top_k)
    ref_tokens, ref_accepted = oa.accept(scores.numpy(), drafted.numpy(), q.numpy(), uniforms.numpy(),
                                         resample.numpy(), 0.9, top_k)
    assert np.array_equal(accepted.cpu().numpy(), ref_accepted)
    assert np.array_equal(tokens.cpu().numpy(), ref_tokens)
    assert wb.device_status() == 0


@pytest.mark.parametrize("temperature", [0.7, 0.8, 0.9, 1.3, 0.3, 2.5, 0.123456])
def test_temperature_scaling_is_ieee_division(wb, temperature):
    """The kernels' x / temperature (reciprocal, product and Markstein's
    correction) against numpy's IEEE float32 division on 2^22 random bit
    patterns plus logits' usual range, +-0 and +-inf: bit for bit for
    quotients of magnitude 2^-100 and up and for zeros and infinities,
    within one unit in the last place below."""
    from wpt_b200 import _lib
    rng = np.random.default_rng(int(temperature * 1e6))
    bits = rng.integers(0, 2 ** 32, 1 << 22, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    x = np.concatenate([x, rng.normal(0.0, 4.0, 1 << 20).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore", under="ignore"):
        ref = x / np.float32(temperature)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    _lib.check(_lib.lib().wpt_temperature_scale(_lib.ptr(xd), xd.numel(), float(temperature), _lib.ptr(out),
                                                _lib.stream(xd.device)))
    got = out.cpu().numpy()
    normal = (np.abs(ref) >= np.float32(2.0 ** -100)) | (x == 0)
    differ = got[normal].view(np.uint32) != ref[normal].view(np.uint32)
    assert not differ.any(), (x[normal][differ][:8], got[normal][differ][:8], ref[normal][differ][:8])
    ulps = np.abs(got[~normal].view(np.int32).astype(np.int64) - ref[~normal].view(np.int32).astype(np.int64))
    assert ulps.max(initial=0) <= 1


@pytest.mark.parametrize("V,temperature,top_k", [(65536, 1.0, None), (1000, 0.8, 40), (65536, 1.0, 1), (777, 1.3, None)])
def test_sampling_without_drafts_matches_the_oracle(wb, V, temperature, top_k):
    # the writer's plain sampling step (wpt_inference/__init__.py:173-182):
    # the acceptance rule with no drafts draws every row's token from p_0
    g = torch.Generator().manual_seed(V + (top_k or 0))
    R = 16
    scores = torch.randn(R, V, generator=g) * 2
    resample = torch.rand(R, generator=g)
    got = wb.sample(scores.cuda(), resample.cuda(), temperature, top_k)
    assert wb.device_status() == 0
    tokens, accepted = oa.accept(scores[:, None].numpy(), np.zeros((R, 0), np.int64), np.zeros((R, 0, V), np.float32),
                                 np.zeros((R, 0), np.float32), resample.numpy(), temperature, top_k)
    assert (accepted == 0).all()
    assert np.array_equal(got.cpu().numpy(), tokens[:, 0])
    if top_k == 1:
        assert np.array_equal(got.cpu().numpy(), scores.argmax(-1).numpy())
