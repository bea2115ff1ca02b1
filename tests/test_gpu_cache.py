"""The generation cache's entries write (packages/wpt-model/src/
wpt_model/cache.py:110-128) on the GPU: the reference's own Rows/Reading
sequence recorded in tests/golden/cache_append.npz (ragged counts, growth)
replayed bit for bit, a bf16 (B, N, 2c) entries table against the oracle
with the size given by the host (one kernel, no host synchronisation), and
a destination past the table refused on the device (status bit 1) instead
of written."""

import numpy as np
import pytest
import torch

from oracle import cache as oc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wb():
    import wpt_b200
    from wpt_b200 import build
    build.build()
    return wpt_b200


def test_cache_append_replays_the_reference_rows(wb, gold):
    d = gold("cache_append.npz")
    held, lengths = None, torch.zeros(3, dtype=torch.int64, device="cuda")
    for step in range(3):
        counts = torch.from_numpy(d[f"counts{step}"]).cuda()
        held, table = wb.cache_append(held, torch.from_numpy(d[f"new{step}"]).cuda(), lengths, counts)
        assert table.shape == d[f"table{step}"].shape
        assert np.array_equal(table.cpu().numpy(), d[f"table{step}"])
        lengths = lengths + counts
    assert wb.device_status() == 0


def test_cache_append_bf16_entries_with_the_size_from_the_host(wb):
    g = torch.Generator().manual_seed(3)
    B, C = 5, 128
    held_np, held = None, None
    first = np.zeros(B, np.int64)
    for counts in ([300, 17, 1, 0, 64], [1, 1, 1, 1, 1], [5, 200, 0, 33, 2]):
        counts = np.array(counts)
        n = int(counts.max())
        new = (torch.randn(B, n, 2 * C, generator=g)).bfloat16()
        need = int((first + counts).max())  # known to the host: its own count of each row's tokens
        held, table = wb.cache_append(held, new.cuda(), torch.from_numpy(first).cuda(),
                                      torch.from_numpy(counts).cuda(), need=need)
        held_np, ref = oc.cache_append(held_np, new.float().numpy(), first, counts)
        assert np.array_equal(table.float().cpu().numpy(), ref)
        first = first + counts
    assert wb.device_status() == 0


def test_cache_append_past_the_table_is_refused_on_the_device(wb):
    from wpt_b200 import _lib
    held = torch.zeros(2, 8, 16, device="cuda")
    new = torch.ones(2, 3, 16, device="cuda")
    first = torch.tensor([6, 0], device="cuda")  # row 0's third entry would land at row 8, past the table
    counts = torch.tensor([3, 3], device="cuda")
    es = 4
    _lib.check(_lib.lib().wpt_cache_append(_lib.ptr(new), new.stride(0) * es, new.stride(1) * es, _lib.ptr(held),
                                           held.stride(0) * es, held.stride(1) * es, _lib.ptr(first),
                                           _lib.ptr(counts), 2, 3, 16 * es, 8, _lib.stream(held.device)))
    assert wb.device_status(reset=True) & 2
    got = held.cpu()
    assert (got[0, 6:8] == 1).all() and (got[1, :3] == 1).all() and got[1, 3:].abs().sum() == 0
