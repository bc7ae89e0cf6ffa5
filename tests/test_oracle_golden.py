"""Pin the CPU oracle against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).  CPU only."""

import math

import numpy as np
import pytest

import cases as C
from oracle import schedule as S
from oracle_runner import load_golden, oracle_case

# The oracle computes in float64; the fixtures are the reference in float32.
RTOL = ATOL = 1e-5          # reference suite's forward tolerance (test_reference.py:118)
GRAD_RTOL = GRAD_ATOL = 1e-4  # reference suite's gradient tolerance (test_reference.py:119)

GRAD_KEYS = {"dq", "dk_packed", "dv_packed", "dpos", "dsinks", "dlse", "dout_pre", "dk", "dv", "dx",
             "dw_proj", "dkcw", "dvcw"}


@pytest.mark.parametrize("name", [c["name"] for c in C.CASES])
def test_oracle_matches_reference(name):
    c = C.CASE_BY_NAME[name]
    gold = load_golden(name)
    got = oracle_case(c)
    for key, want in gold.items():
        if key in ("case", "ring_live", "caps", "offsets"):
            continue
        have = got[key]
        if key.startswith("ring_"):
            live = gold["ring_live"]
            want, have = want[:, live], have[:, live]
        tol = GRAD_RTOL if key in GRAD_KEYS else RTOL
        # the fixtures accumulate in float32 over up to a few hundred entries on
        # the longer geometries: allow 3x the suite's tolerance there
        if C.GEOS[c["geo"]]["N"] >= 512:
            tol *= 3.0
        np.testing.assert_allclose(have, want, rtol=tol, atol=tol, err_msg=f"{name}:{key}")
    if "caps" in gold:
        assert tuple(got["caps"]) == tuple(gold["caps"])
    if "offsets" in gold:
        assert tuple(got["offsets"]) == tuple(gold["offsets"])


@pytest.mark.parametrize("sched", [s[0] for s in C.SCHEDULES])
def test_schedule_oracle_matches_reference(sched):
    name, N, cache, fmap = next(s for s in C.SCHEDULES if s[0] == sched)
    gold = load_golden("sched_" + name)
    a = S.activation_times(fmap)
    assert tuple(a) == tuple(gold["a"])
    assert S.level_offsets(N, len(a)) == list(gold["offsets"])
    for q, row in zip(gold["qs"], gold["bounds"]):
        assert [tuple(r) for r in S.row_ranges(int(q), a, cache)] == [tuple(r) for r in row], q
    assert S.decode_caps(a, cache) == tuple(gold["caps"])
    if N <= 20000:
        assert S.coarsest_span(a, cache, N) == int(gold["span"])
    if N <= 1024:
        rows = S.all_row_ranges(N, a, cache)
        for lv, s, e, lo, hi in gold["fwd_hulls"]:
            assert S.fwd_hull(s, e, lv, rows) == (lo, hi)
        by_level = {}
        for lv, s, e, lo, hi in gold["bwd_hulls"]:
            if lv not in by_level:
                by_level[lv] = S.node_queries(N, lv, rows)
            assert S.bwd_hull(s, e, by_level[lv]) == (lo, hi)


def test_readme_tiny_hand_golden():
    """The reference suite's hand-derived table (test_reference.py:482-491)."""
    golden = {0: [(0, 1), (0, 0), (0, 0)], 1: [(0, 2), (0, 0), (0, 0)],
              2: [(0, 3), (0, 0), (0, 0)], 3: [(2, 4), (0, 1), (0, 0)],
              4: [(2, 5), (0, 1), (0, 0)], 5: [(4, 6), (0, 2), (0, 0)],
              6: [(4, 7), (0, 0), (0, 1)], 7: [(6, 8), (2, 3), (0, 1)]}
    a = S.activation_times({1: 2, 2: 3})
    for q, want in golden.items():
        assert S.row_ranges(q, a, 6) == want
    # bin-distance golden at q = 7 (test_reference.py:1099-1101)
    d = S.bin_distances(7, a, 6)
    assert d[(2, 0)] == 3 and d[(1, 2)] == 2 and d[(0, 6)] == 1 and d[(0, 7)] == 0
    # activation times golden (test_reference.py:272)
    assert S.activation_times({1: 64, 2: 72, 3: 80}) == (0, 65, 82, 116)


def test_activation_time_errors():
    with pytest.raises(ValueError):
        S.activation_times({1: 2, 3: 4})
    with pytest.raises(ValueError):
        S.activation_times({1: 3})  # a[1] = 4, phase 0 mod 2


def test_visible_set_is_cache_bounded_and_chronological():
    for name, N, cache, fmap in C.SCHEDULES[:6]:
        a = S.activation_times(fmap)
        for q in range(N):
            ent = S.visible_entries(q, a, cache)
            assert len(ent) <= cache
            assert ent[-1] == (0, q)
            starts = [j << lv for lv, j in ent]
            ends = [(j + 1) << lv for lv, j in ent]
            assert all(e == s for e, s in zip(ends, starts[1:]))  # contiguous, disjoint
            assert ends[-1] == q + 1
            # coarse-before-fine in time: levels never increase going newer
            lvls = [lv for lv, _ in ent]
            assert all(x >= y for x, y in zip(lvls, lvls[1:]))
