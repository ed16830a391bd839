"""CPU: the hot-store replacement policy of the tiered expert store.

The reference ships its policy as include/tier.h:30-58 (LFRU score, pick,
decay).  tier_cases.npz holds cases run through the reference's own compiled
functions (tests/golden/make_golden.py).  Here:
  * the oracle restatement (oracle/moe_oracle.c) equals them on every case;
  * the library's rule (omc_tier_pick, exported for exactly this check; no
    device involved) equals them on every case;
  * where the reference harness is built, both equal it on fresh random cases;
  * the oracle's per-forward heat accounting equals a direct count.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tier_cases.npz")


def _cases():
    z = np.load(GOLDEN)
    for c in range(z["E"].size):
        E, npin = int(z["E"][c]), int(z["npin"][c])
        yield (z["heat"][c, :E], z["last"][c, :E], int(z["clock"][c]), z["pinned"][c, :npin],
               z["lfru"][c], z["swap"][c], z["score"][c, :E], z["decay"][c, :E])


def _tuple(r):
    return (int(r[1]), int(r[2]), int(r[3])) if r[0] else None


def test_golden_covers_the_edges():
    z = np.load(GOLDEN)
    assert z["E"].size >= 400
    assert 0 < int(z["lfru"][:, 0].sum()) < z["E"].size   # both outcomes present
    assert int(z["swap"][:, 0].sum()) > 0


def test_oracle_matches_reference_golden(oracle):
    o = oracle.Tier("oracle")
    for heat, last, clock, pinned, lfru, swap, score, decay in _cases():
        assert o.pick_lfru(heat, last, clock, pinned) == _tuple(lfru)
        assert o.pick_heat(heat, pinned) == _tuple(swap)
        assert [o.score(int(h), int(l), clock) for h, l in zip(heat, last)] == [int(v) for v in score]
        assert np.array_equal(o.decay(heat), decay)


def test_library_rule_matches_reference_golden(omc_lib):
    n = 0
    for heat, last, clock, pinned, lfru, _, _, _ in _cases():
        assert omc_lib.tier_pick(heat, last, clock, pinned) == _tuple(lfru)
        n += 1
    assert n >= 400


def test_random_against_compiled_reference(oracle, omc_lib):
    if oracle.ref_lib("tier") is None:
        pytest.skip("reference tier.h harness not built here")
    o, r = oracle.Tier("oracle"), oracle.Tier("ref")
    rng = np.random.default_rng(77)
    for it in range(3000):
        E = int(rng.integers(1, 129))
        npin = int(rng.integers(1, E + 1))
        pinned = rng.choice(E, npin, replace=False).astype(np.int32)
        heat = rng.integers(0, [8, 300, 2**32 - 1][it % 3], E, dtype=np.uint64).astype(np.uint32)
        clock = int(rng.integers(0, 2**32))
        last = ((clock - rng.integers(0, 400, E)) & 0xFFFFFFFF).astype(np.uint32)
        want = r.pick_lfru(heat, last, clock, pinned)
        assert o.pick_lfru(heat, last, clock, pinned) == want
        assert omc_lib.tier_pick(heat, last, clock, pinned) == want
        assert o.pick_heat(heat, pinned) == r.pick_heat(heat, pinned)


def test_no_swap_without_outsider_or_slots(omc_lib):
    heat = np.array([5, 9, 1], np.uint32)
    last = np.zeros(3, np.uint32)
    assert omc_lib.tier_pick(heat, last, 0, np.array([0, 1, 2], np.int32)) is None   # all resident
    assert omc_lib.tier_pick(heat, last, 0, np.array([], np.int32)) is None           # no slot


def test_heat_accounting(oracle):
    o = oracle.Tier("oracle")
    E = 12
    rng = np.random.default_rng(5)
    heat, last, clock = np.zeros(E, np.uint32), np.zeros(E, np.uint32), 0
    want_h, want_l = np.zeros(E, np.uint64), np.zeros(E, np.uint32)
    for step in range(1, 41):
        idx = rng.integers(0, E, (int(rng.integers(1, 9)), 3)).astype(np.int32)
        heat, last, clock = o.account(idx, E, heat, last, clock, decay_every=8)
        cnt = np.bincount(idx.ravel(), minlength=E)
        want_h += cnt.astype(np.uint64)
        want_l[cnt > 0] = step
        if step % 8 == 0:
            want_h >>= 1
        assert clock == step
        assert np.array_equal(heat, want_h.astype(np.uint32))
        assert np.array_equal(last, want_l)
    # saturation instead of wrap-around
    h, _, _ = o.account(np.zeros(4, np.int32), E, np.full(E, 2**32 - 2, np.uint32), np.zeros(E, np.uint32), 0)
    assert int(h[0]) == 2**32 - 1
