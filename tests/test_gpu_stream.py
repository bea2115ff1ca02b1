"""The key-stream kernel (decode, short extends, sparse gathers) against the
CPU oracle, through the C ABI: ragged decode rows with stale rows past each
length, window + sink decode, a long row over many splits, extends of a few
queries, and sparse attention over chosen rows with -1 padding
(pytorch_kernels.py:171-187,213-217). Tolerances: bf16 outputs within
max-abs 2e-2, LSE within 1e-3."""

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


def _np(x):
    return x.float().cpu().numpy().astype(np.float64)


def _check(wb, out, lse, ref_out, ref_lse):
    assert wb.device_status() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref_out).max() < OUT_TOL
    if lse is not None:
        assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_TOL


def _decode_case(B, T, H, N, seed, lengths=None):
    g = torch.Generator().manual_seed(seed)
    C = 128
    q = (torch.randn(B, T, H, C, generator=g) * 0.5).bfloat16()
    e = (torch.randn(B, N, 2 * C, generator=g) * 0.5).bfloat16()
    if lengths is None:
        lengths = torch.randint(T, N + 1, (B,), generator=g)
    positions = lengths[:, None] - T + torch.arange(T)[None]
    for b in range(B):  # stale rows past each row's length: finite, large, never to be read
        e[b, int(lengths[b]):] = 50.0
    return q, e, positions


@pytest.mark.parametrize("B,T,H,N", [(8, 1, 32, 5000), (4, 1, 16, 3000), (3, 2, 32, 2000), (5, 3, 4, 900),
                                     (2, 1, 64, 1000)])
def test_decode_matches_oracle(wb, B, T, H, N):
    q, e, positions = _decode_case(B, T, H, N, seed=B * 100 + T * 10 + H)
    C = 128
    out, lse = wb.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("chunk", [1, 3, 4, 16, 100])  # 32, 11 splits merged by a kernel; 8, 2 in a cluster; 1
def test_decode_split_chunks_agree(wb, chunk):
    from wpt_b200 import ops
    q, e, positions = _decode_case(4, 1, 32, 4000, seed=chunk)
    C = 128
    out, lse = ops.stream_forward(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                  chunk_tiles=chunk)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


def test_decode_window_with_sink(wb):
    B, H, N, W, C = 6, 32, 6000, 1024, 128
    q, e, positions = _decode_case(B, 1, H, N, seed=9, lengths=torch.tensor([5, 600, 1024, 1025, 4000, 6000]))
    sink = torch.randn(H, generator=torch.Generator().manual_seed(2)) * 0.5
    out, lse = wb.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                   window=W, sink=sink.cuda())
    ref_out, ref_lse = oat.sparse_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().numpy(),
                                            np.zeros((B, 1, 0), np.int64), positions.numpy(), C ** -0.5, W)
    _check(wb, out, lse, ref_out, ref_lse)


def test_long_single_row_over_many_splits(wb):
    q, e, positions = _decode_case(1, 1, 32, 40000, seed=4, lengths=torch.tensor([39999]))
    C = 128
    out, lse = wb.forward_with_lse(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("chunk", [2, 7])
def test_long_row_merged_from_many_splits(wb, chunk):
    # 157 or 23 splits of one 32-head row: the merge's one-CTA-per-row form
    from wpt_b200 import ops
    q, e, positions = _decode_case(1, 1, 32, 40000, seed=6, lengths=torch.tensor([39999]))
    C = 128
    out, lse = ops.stream_forward(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                  chunk_tiles=chunk)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out, lse, ref_out, ref_lse)


def _sparse_case(B, T, H, N, K, W, seed):
    g = torch.Generator().manual_seed(seed)
    C = 128
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    sink = torch.randn(H, generator=g) * 0.5
    positions = (N - T + torch.arange(T)).expand(B, T).contiguous()
    idx = torch.full((B, T, K), -1, dtype=torch.long)
    for b in range(B):
        for t in range(T):
            far = int(positions[b, t]) - W + 1  # rows before the window
            if far > 0:
                pick = torch.randperm(far, generator=g)[:K]
                idx[b, t, :len(pick)] = pick
    idx[:, ::3, -2:] = -1
    return q, e, sink, idx, positions


@pytest.mark.parametrize("B,T,H,N,K,W", [(2, 40, 16, 700, 64, 128), (2, 30, 2, 700, 64, 128),
                                         (1, 8, 32, 3000, 1024, 128), (2, 16, 12, 2000, 16, 32),
                                         (1, 4, 16, 5000, 300, 1024)])
def test_sparse_gather_matches_oracle(wb, B, T, H, N, K, W):
    q, e, sink, idx, positions = _sparse_case(B, T, H, N, K, W, seed=T * 7 + H)
    C = 128
    out = wb.sparse_attention(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], sink.cuda(), idx.cuda(),
                              positions.cuda(), C ** -0.5, W)
    ref_out, _ = oat.sparse_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().numpy(), idx.numpy(),
                                      positions.numpy(), C ** -0.5, W)
    assert out.dtype == torch.bfloat16
    _check(wb, out, None, ref_out, None)


def test_sparse_golden_shape_through_both_paths_agree(wb):
    # the same sparse call computed by gathers and, with no chosen rows, by ranges
    q, e, sink, idx, positions = _sparse_case(2, 20, 16, 900, 0, 128, seed=3)
    C = 128
    from wpt_b200 import ops
    qd, kd, vd = q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:]
    window_rows = oat.window_rows(positions.numpy(), 128, 900)
    a, la = ops.stream_forward(qd, kd, vd, positions.cuda(), C ** -0.5, window=128, sink=sink.cuda())
    b, lb = ops.stream_forward(qd, kd, vd, positions.cuda(), C ** -0.5, window=0,
                               idx=torch.from_numpy(window_rows).cuda(), sink=sink.cuda())
    assert (a.float() - b.float()).abs().max().item() < 1e-2
    assert (la - lb).abs().max().item() < 1e-4


def test_decode_growing_scores_force_rescales(wb):
    # the running maximum is raised by far more than the lazy threshold in
    # every tile, so the key-stream kernel rescales O^T each time
    from wpt_b200 import ops
    B, H, C, N = 4, 32, 128, 3000
    g = torch.Generator().manual_seed(32)
    u = torch.randn(C, generator=g)
    u = u / u.norm()
    q = (u * 3.0 + 0.1 * torch.randn(B, 1, H, C, generator=g)).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g)
    e[..., :C] = u * (torch.arange(N)[:, None] / 16.0) + 0.1 * e[..., :C]
    e = e.bfloat16()
    positions = torch.tensor([[2999], [2000], [1300], [300]])
    for chunk in (1, 4, 100):
        out, lse = ops.stream_forward(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], positions.cuda(), C ** -0.5,
                                      chunk_tiles=chunk)
        ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                                  C ** -0.5, 0, 0)
        _check(wb, out, lse, ref_out, ref_lse)


def test_partials_merged_by_the_caller_equal_the_whole_call(wb):
    # out = lse = NULL: the kernel stops at its split partials; merging two
    # halves' partials (as two GPUs of a long row would) gives the whole row
    from wpt_b200 import ops
    q, e, positions = _decode_case(1, 1, 32, 20000, seed=7, lengths=torch.tensor([19999]))
    C = 128
    qd, ed, pd = q.cuda(), e.cuda(), positions.cuda()
    half = 10240
    parts = [ops.stream_partials(qd, ed[:, a:b, :C], ed[:, a:b, C:], pd - a, C ** -0.5)
             for a, b in ((0, half), (half, 20000))]
    part_o = torch.cat([p[0] for p in parts])
    part_lse = torch.cat([p[1] for p in parts])
    out, lse = ops.merge_partials(part_o, part_lse, 32)
    ref_out, ref_lse, _ = oat.exact_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), positions.numpy(),
                                              C ** -0.5, 0, 0)
    _check(wb, out.reshape(1, 1, 32, C), lse.reshape(1, 1, 32), ref_out, ref_lse)


def test_sparse_window_rows_outside_the_table(wb):
    """Gather mode's window tiles come by TMA: windows that start before row
    0 (early positions) or run past the table's end (a position beyond it)
    read zeros there and mask those rows, as the reference's -1 rows are."""
    B, T, H, N, K, W = 4, 1, 32, 1500, 256, 1024
    g = torch.Generator().manual_seed(77)
    C = 128
    q = torch.randn(B, T, H, C, generator=g).bfloat16()
    e = torch.randn(B, N, 2 * C, generator=g).bfloat16()
    sink = torch.randn(H, generator=g) * 0.5
    positions = torch.tensor([[5], [700], [1499], [1540]])
    idx = torch.full((B, T, K), -1, dtype=torch.long)
    for b in range(B):
        far = int(positions[b, 0]) - W + 1
        if far > 0:
            pick = torch.randperm(far, generator=g)[:K]
            idx[b, 0, :len(pick)] = pick
    out = wb.sparse_attention(q.cuda(), e.cuda()[..., :C], e.cuda()[..., C:], sink.cuda(), idx.cuda(),
                              positions.cuda(), C ** -0.5, W)
    ref_out, _ = oat.sparse_attention(_np(q), _np(e[..., :C]), _np(e[..., C:]), sink.double().numpy(), idx.numpy(),
                                      positions.numpy(), C ** -0.5, W)
    _check(wb, out, None, ref_out, None)


@pytest.mark.parametrize("shards,with_sink", [(2, False), (3, True), (8, True)])
def test_long_row_shards_packed_and_merged_equal_one_call(wb, shards, with_sink):
    # the kernel path of the multi-GPU long row on one GPU: each shard's
    # split partials, merged into one partial in its own chunk of one buffer
    # (as the in-place all-gather leaves them on every rank), then one
    # grouped merge of the chunks with the sink
    from wpt_b200 import multi, ops
    g = torch.Generator().manual_seed(40 + shards)
    H, C, N = 32, 128, 20000
    q = (torch.randn(1, 1, H, C, generator=g) * 0.5).bfloat16().cuda()
    e = (torch.randn(1, N, 2 * C, generator=g) * 0.5).bfloat16().cuda()
    sink = (torch.randn(H, generator=g) * 0.5).cuda() if with_sink else None
    positions = torch.tensor([[N - 1]]).cuda()
    rows = H
    chunk = (rows * (C + 1) + 3) // 4 * 4
    parts = torch.empty(shards, chunk, dtype=torch.float32, device="cuda")
    for r in range(shards):
        a, b = multi.key_shard(N, shards, r)
        part_o, part_lse = ops.stream_partials(q, e[:, a:b, :C], e[:, a:b, C:], positions - a, C ** -0.5)
        ops.merge_partial(part_o, part_lse, out_o=parts[r, :rows * C].view(rows, C),
                          out_lse=parts[r, rows * C:rows * (C + 1)])
    out, lse = ops.merge_groups(parts, 1, rows, H, C, sink)
    whole, whole_lse = ops.stream_forward(q, e[..., :C], e[..., C:], positions, C ** -0.5, sink=sink)
    assert wb.device_status() == 0
    assert (out.float().reshape(whole.shape) - whole.float()).abs().max().item() < 1e-2
    assert (lse.reshape(whole_lse.shape) - whole_lse).abs().max().item() < 1e-4
    ref, ref_lse = oat.range_attention(_np(q.cpu()), _np(e[..., :C].cpu()), _np(e[..., C:].cpu()),
                                       np.array([[N - 1]]), C ** -0.5,
                                       sink=None if sink is None else sink.double().cpu().numpy())
    _check(wb, out.reshape(whole.shape), lse.reshape(whole_lse.shape), ref, ref_lse)
