"""The long row's exchange protocol (wpt_b200/csrc/exchange.cuh), modelled
on the CPU: `world` ranks each make a sequence of calls; in call e a rank
stores its partial into slot `rank` of buffer half e % 2 of every rank, then
adds one arrival to that half's counter on every rank, waits until its own
counter reaches world * (e // 2 + 1), and reads every rank's slot of the
half. Stores, arrivals and reads of all ranks interleave at random. Every
read must see the partial of the same call (no rank overwrites a half that
another still has to read, and no wait ends before all partials of its call
are in); with a single half instead of two the model must find a schedule
that breaks this, which shows that it can."""

import random

import pytest


def _run(world, calls, seed, halves=2):
    rnd = random.Random(seed)
    data = [[[None] * world for _ in range(halves)] for _ in range(world)]
    count = [[0] * halves for _ in range(world)]

    def rank(r):
        for e in range(calls):
            h = e % halves
            for d in rnd.sample(range(world), world):  # the stores, in any order
                data[d][h][r] = e
                yield
            for d in range(world):  # then the arrivals (after the barrier, a release each)
                count[d][h] += 1
                yield
            while count[r][h] < world * (e // halves + 1):
                yield
            for g in range(world):  # the reads of this call's partials
                if data[r][h][g] != e:
                    raise AssertionError(f"rank {r} call {e} read slot {g} of call {data[r][h][g]}")
                yield
    procs = {r: rank(r) for r in range(world)}
    while procs:
        r = rnd.choice(list(procs))
        try:
            next(procs[r])
        except StopIteration:
            del procs[r]


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_two_halves_never_read_a_stale_or_missing_partial(world):
    for seed in range(500):
        _run(world, 7, seed * 10 + world)


def test_one_half_is_not_enough():
    found = False
    for seed in range(500):
        try:
            _run(2, 7, seed, halves=1)
        except AssertionError:
            found = True
            break
    assert found
