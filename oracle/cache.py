"""CPU restatement of the generation cache's entries write, in numpy.

TEST INFRASTRUCTURE ONLY (the checker): only `tests/`, `__graft_entry__.smoke()`
and the CPU legs of `bench.py` may import it; the product package never does.

Follows packages/wpt-model/src/wpt_model/cache.py:110-128 (Reading.everything):
row b's new entries new[b, j] (j < counts[b]) go to rows first[b] + j of
the held table; the table grows to max(need, 2 * capacity) rows (zeros)
when need = max_b(first[b] + counts[b]) exceeds it; the call returns the
held table and its first `need` rows.
"""

import numpy as np


def cache_append(held, new, first, counts):
    new = np.asarray(new)
    first = np.asarray(first, np.int64)
    counts = np.asarray(counts, np.int64)
    B = new.shape[0]
    held = np.zeros((B, 0) + new.shape[2:], new.dtype) if held is None else np.asarray(held, new.dtype).copy()
    need = int((first + counts).max()) if B else 0
    if need > held.shape[1]:
        grown = max(need, 2 * held.shape[1])
        held = np.concatenate([held, np.zeros((B, grown - held.shape[1]) + held.shape[2:], held.dtype)], 1)
    for b in range(B):
        for j in range(int(counts[b])):
            held[b, first[b] + j] = new[b, j]
    return held, held[:, :need]
