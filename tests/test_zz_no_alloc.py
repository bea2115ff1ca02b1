"""wpt_attn_decode_noalloc, the decode entry point that allocates nothing:
its split partials live in the library's static device array instead of
caller buffers. It is for callers that cannot allocate device memory on
the hot path (an FFI host without a caching allocator, a serving loop that
must not synchronise on cudaMalloc/cudaFree or grow its footprint).

Called through the C ABI, twice in a row with different inputs, its output
must match wpt_attn_decode's (given torch-allocated scratch) within the
tolerances of the other GPU tests; an oversized call must be refused before
anything launches. This file is collected last so that a run stopping at
its first failure has already run every other test; it also passes alone
in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

OUT_TOL, LSE_TOL = 2e-2, 1e-3


@pytest.fixture(scope="module")
def lib():
    from wpt_b200 import _lib, build
    build.build()
    return _lib


def _case(seed, B=6, H=32, C=128, N=5000):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, 1, H, C, generator=g) * 0.5).bfloat16().cuda()
    e = (torch.randn(B, N, 2 * C, generator=g) * 0.5).bfloat16().cuda()
    lengths = torch.randint(1, N + 1, (B,), generator=g)
    positions = (lengths - 1)[:, None].contiguous().cuda()
    sink = (torch.randn(H, generator=g) * 0.5).cuda()
    return q, e, positions, sink


def _decode(L, q, e, positions, sink, splits, chunk, noalloc, idx=None, window=0, outputs=True):
    B, T, H, C = q.shape
    N = e.shape[1]
    k, v = e[..., :C], e[..., C:]
    out = torch.empty_like(q) if outputs else None
    lse = torch.empty(B, T, H, dtype=torch.float32, device=q.device) if outputs else None
    K = 0 if idx is None else idx.shape[-1]
    common = (L.ptr(q), L.ptr(k), L.ptr(v), k.stride(0), k.stride(1), v.stride(0), v.stride(1), L.ptr(positions),
              None, L.ptr(idx), K, L.ptr(sink), L.ptr(out), L.ptr(lse))
    tail = (splits, chunk, B, T, H, C, N, window, C ** -0.5, L.stream(q.device))
    if noalloc:
        rc = L.lib().wpt_attn_decode_noalloc(*common, *tail)
    else:
        part_o = torch.empty(splits, B * T * H, C, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(splits, B * T * H, dtype=torch.float32, device=q.device)
        rc = L.lib().wpt_attn_decode(*common, L.ptr(part_o), L.ptr(part_lse), *tail)
    L.check(rc)
    torch.cuda.synchronize()
    return out, lse


def _same(want, want_lse, got, got_lse):
    assert np.isfinite(got.float().cpu().numpy()).all()
    assert (got.float() - want.float()).abs().max().item() < OUT_TOL
    assert (got_lse - want_lse).abs().max().item() < LSE_TOL


def test_noalloc_decode_matches_the_allocating_entry_point_twice(lib):
    splits, chunk = 5, 8  # 5 x 8 x 128 = 5120 rows per query, more than N
    for seed in (1, 2):  # two calls in a row share (and overwrite) the static scratch
        q, e, positions, sink = _case(seed)
        want, want_lse = _decode(lib, q, e, positions, sink, splits, chunk, noalloc=False)
        got, got_lse = _decode(lib, q, e, positions, sink, splits, chunk, noalloc=True)
        _same(want, want_lse, got, got_lse)
    assert lib.device_status() == 0


def test_noalloc_decode_with_one_split_uses_no_scratch(lib):
    q, e, positions, sink = _case(4)
    want, want_lse = _decode(lib, q, e, positions, sink, 1, 40, noalloc=False)
    got, got_lse = _decode(lib, q, e, positions, sink, 1, 40, noalloc=True)
    _same(want, want_lse, got, got_lse)
    assert lib.device_status() == 0


def test_noalloc_sparse_gather_matches_twice(lib):
    # gather mode: each query's 300 chosen rows (some -1) then its last 128 rows
    for seed in (5, 6):
        q, e, positions, sink = _case(seed, B=4, N=3000)
        g = torch.Generator().manual_seed(seed)
        idx = torch.randint(0, 1000, (4, 1, 300), generator=g)
        idx[:, :, ::7] = -1
        idx = idx.cuda()
        positions = torch.full_like(positions, 2999)
        want, want_lse = _decode(lib, q, e, positions, sink, 2, 2, noalloc=False, idx=idx, window=128)
        got, got_lse = _decode(lib, q, e, positions, sink, 2, 2, noalloc=True, idx=idx, window=128)
        _same(want, want_lse, got, got_lse)
    assert lib.device_status() == 0


def test_noalloc_decode_at_its_largest_size(lib):
    # splits x B x T x H = 127 x 4 x 1 x 32 = 16256 rows of 129 floats, the most
    # that fit in 2^21 floats (2^21 / 129 is not whole, so no call fills it
    # exactly); one split more is refused
    q, e, positions, sink = _case(7, B=4, N=127 * 128)
    positions = torch.tensor([[127 * 128 - 1], [9000], [128], [5]]).cuda()
    want, want_lse = _decode(lib, q, e, positions, sink, 127, 1, noalloc=False)
    got, got_lse = _decode(lib, q, e, positions, sink, 127, 1, noalloc=True)
    _same(want, want_lse, got, got_lse)
    assert lib.device_status() == 0
    with pytest.raises(NotImplementedError, match="static scratch"):
        _decode(lib, q, e, positions, sink, 128, 1, noalloc=True)


def test_noalloc_decode_refuses_more_than_its_scratch(lib):
    # 64 rows x 32 heads x 129 floats per split: 1024 splits need far more than 8 MiB
    q, e, positions, sink = _case(3, B=64, N=1000)
    with pytest.raises(NotImplementedError, match="static scratch"):
        _decode(lib, q, e, positions, sink, 1024, 1, noalloc=True)


def test_noalloc_decode_refuses_the_partials_only_mode(lib):
    # out == lse == NULL would leave the partials in the library's private
    # array, where the caller cannot read them
    q, e, positions, sink = _case(8)
    with pytest.raises(ValueError, match="out and lse are required"):
        _decode(lib, q, e, positions, sink, 5, 8, noalloc=True, outputs=False)
