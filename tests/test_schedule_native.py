"""CPU tests of the integer schedule: the C library's host closed forms and
the Python range_spec API, bit-exact against the reference's golden tables
and the oracle.  No GPU needed (host-only library calls)."""

import ctypes

import numpy as np
import pytest

import cases as C
from oracle import schedule as S
from oracle_runner import load_golden
from telescope_cache_b200 import _lib
from telescope_cache_b200 import range_spec as R
from telescope_cache_b200.telescoping_attn.decode_state import decode_capacities


def _native(fmap, cache, N):
    return R.native_schedule(R.RangeSpec.from_fmap(fmap, cache, N))


def _host_bounds(sched, qs):
    qs = np.ascontiguousarray(qs, dtype=np.int32)
    out = np.zeros((len(qs), sched.num_levels, 2), dtype=np.int32)
    _lib.check(_lib.lib().tc_range_bounds_host(ctypes.byref(sched), qs.ctypes.data, len(qs),
                                               out.ctypes.data), "tc_range_bounds_host")
    return out


def _host_hulls(sched, kind, level, lo, hi):
    lo = np.ascontiguousarray(lo, dtype=np.int32)
    hi = np.ascontiguousarray(hi, dtype=np.int32)
    out = np.zeros((len(lo), 2), dtype=np.int32)
    _lib.check(_lib.lib().tc_hulls_host(ctypes.byref(sched), kind, level, lo.ctypes.data,
                                        hi.ctypes.data, len(lo), out.ctypes.data), "tc_hulls_host")
    return out


@pytest.mark.parametrize("sched", [s[0] for s in C.SCHEDULES])
def test_native_schedule_matches_golden(sched):
    name, N, cache, fmap = next(s for s in C.SCHEDULES if s[0] == sched)
    g = load_golden("sched_" + name)
    ns = _native(fmap, cache, N)
    assert list(ns.act)[:ns.num_levels] == list(g["a"])
    assert list(ns.offsets)[:ns.num_levels + 1] == list(g["offsets"])
    assert ns.coarsest_span == int(g["span"])
    got = _host_bounds(ns, g["qs"])
    assert np.array_equal(got, g["bounds"])
    fh = g["fwd_hulls"]
    for lv in np.unique(fh[:, 0]):
        sel = fh[fh[:, 0] == lv]
        got = _host_hulls(ns, 0, int(lv), sel[:, 1], sel[:, 2])
        assert np.array_equal(got, sel[:, 3:5]), (name, lv)
    bh = g["bwd_hulls"]
    for lv in np.unique(bh[:, 0]):
        sel = bh[bh[:, 0] == lv]
        got = _host_hulls(ns, 1, int(lv), sel[:, 1], sel[:, 2])
        assert np.array_equal(got, sel[:, 3:5]), (name, lv)
    assert decode_capacities(tuple(g["a"]), cache) == tuple(g["caps"])


@pytest.mark.parametrize("sched", [s[0] for s in C.SCHEDULES])
def test_python_range_spec_matches_golden(sched):
    name, N, cache, fmap = next(s for s in C.SCHEDULES if s[0] == sched)
    g = load_golden("sched_" + name)
    spec = R.RangeSpec.from_fmap(fmap, cache, N)
    assert spec.activation_times == tuple(g["a"])
    assert spec.level_offsets() == tuple(g["offsets"])
    assert R.coarsest_lifetime_span(spec) == int(g["span"])
    for q, row in zip(g["qs"][:600], g["bounds"][:600]):
        assert [R.range_bounds(spec, int(q), lv) for lv in range(spec.num_levels)] == \
            [tuple(r) for r in row]
    for lv, s, e, lo, hi in g["fwd_hulls"][:400]:
        assert R.fwd_bounds(spec, int(s), int(e), int(lv)) == (lo, hi)
    for lv, s, e, lo, hi in g["bwd_hulls"][:400]:
        assert R.bwd_bounds(spec, int(s), int(e), int(lv)) == (lo, hi)


def test_exhaustive_small_schedules_vs_oracle():
    """Every query of the small schedules: C closed form == oracle's analytic
    ruler/slot ranges, including eviction and odd lengths."""
    for name, N, cache, fmap in C.SCHEDULES[:7]:
        ns = _native(fmap, cache, N)
        a = S.activation_times(fmap)
        got = _host_bounds(ns, np.arange(N))
        want = np.array([S.row_ranges(q, a, cache) for q in range(N)])
        assert np.array_equal(got, want), name


def test_visible_stats():
    spec = R.RangeSpec.from_fmap({1: 128, 2: 256, 3: 384}, 512, 1024)
    mn, mx, tot = R.visible_stats(spec)
    a = S.activation_times({1: 128, 2: 256, 3: 384})
    counts = [len(S.visible_entries(q, a, 512)) for q in range(1024)]
    assert (mn, mx, tot) == (min(counts), max(counts), sum(counts))
    # config 1: sum_q |A(q)| = 271,872 per head, the FLOP basis of the CPU config
    assert tot == 271872


def test_schedule_errors():
    with pytest.raises(ValueError):
        R.activation_times_from_fmap({1: 2, 3: 4})
    with pytest.raises(ValueError):
        R.activation_times_from_fmap({1: 3})
    with pytest.raises(ValueError):
        R.RangeSpec((1, 3), 6, 8)
    spec = R.RangeSpec.from_fmap({1: 2, 2: 3}, 6, 8)
    for bad in (lambda: R.range_bounds(spec, 8, 0), lambda: R.range_bounds(spec, -1, 0),
                lambda: R.range_bounds(spec, 0, 3), lambda: R.elem_mask(spec, 0, 8, 0),
                lambda: R.fwd_bounds(spec, 0, 9, 0), lambda: R.fwd_bounds(spec, 2, 1, 0),
                lambda: R.node_query_bounds(spec, 2, 2), lambda: R.bwd_bounds(spec, 0, 9, 0)):
        with pytest.raises(ValueError):
            bad()
    assert R.fwd_bounds(spec, 3, 3, 0) == R.EMPTY
    assert R.bwd_bounds(spec, 0, 0, 0) == R.EMPTY
    with pytest.raises(ValueError):
        decode_capacities((1, 3), 6)


def test_node_query_bounds_vs_oracle():
    for name, N, cache, fmap in C.SCHEDULES[:6]:
        spec = R.RangeSpec.from_fmap(fmap, cache, N)
        a = S.activation_times(fmap)
        rows = S.all_row_ranges(N, a, cache)
        for lv in range(spec.num_levels):
            nq = S.node_queries(N, lv, rows)
            for k in range(spec.level_len(lv)):
                want = (nq[k][0], nq[k][-1] + 1) if nq[k] else (0, 0)
                assert R.node_query_bounds(spec, k, lv) == want, (name, lv, k)
