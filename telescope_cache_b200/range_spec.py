"""Integer schedule of telescoping attention: the host-side API of
``telescoping_attn/range_spec.py`` (same names, arguments, results and
errors).

Node j of level l summarises tokens [j 2^l, (j+1) 2^l).  A schedule ``fmap``
yields activation times a[l]; every query sees one contiguous node interval
per level.  The closed forms here use only ``+ - * >> min max`` so that the
same code runs on Python ints and on integer tensors (``IntOps``).  The CUDA
kernels evaluate the identical closed forms (``csrc/common.cuh``); the O(N)
schedule scans (coarsest lifetime span, decode capacities) run in the C
library.
"""

import ctypes
from dataclasses import dataclass
from typing import Callable, Dict, NamedTuple, Sequence, Tuple

EMPTY: Tuple[int, int] = (0, 0)


def activation_times_from_fmap(fmap: Dict[int, int]) -> Tuple[int, ...]:
    """a[0..L] for a schedule {level: slots}; a[1] = fmap[1] + 1 and each
    level adds 2^(l-1) (fmap[l] - fmap[l-1]) + 2^(l-2).  Raises ValueError
    for non-consecutive keys or a level whose phase a[l] mod 2^l is not
    2^(l-1) (range_spec.py:26-54)."""
    if not fmap:
        return (0,)
    top = max(fmap)
    keys = sorted(fmap)
    if keys != list(range(1, top + 1)):
        raise ValueError(f"fmap keys must be consecutive 1..L; got {keys}")
    times = [0, fmap[1] + 1]
    for lv in range(2, top + 1):
        times.append(times[-1] + ((fmap[lv] - fmap[lv - 1]) << (lv - 1)) + (1 << (lv - 2)))
    for lv in range(1, top + 1):
        phase = times[lv] % (1 << lv)
        if phase != 1 << (lv - 1):
            raise ValueError(
                f"fmap not dyadically aligned at level {lv}: a[{lv}]={times[lv]} has phase "
                f"{phase} mod {1 << lv}, expected {1 << (lv - 1)}.")
    return tuple(times)


@dataclass(frozen=True)
class RangeSpec:
    """Activation times a[0..L], cache size C and sequence length N
    (range_spec.py:57-126)."""

    activation_times: Tuple[int, ...]
    cache_size: int
    seq_len: int

    @classmethod
    def from_fmap(cls, fmap: Dict[int, int], cache_size: int, seq_len: int) -> "RangeSpec":
        return cls(activation_times_from_fmap(fmap), cache_size, seq_len)

    def __post_init__(self):
        if self.cache_size <= 0 or self.seq_len <= 0:
            raise ValueError("cache_size and seq_len must be positive")
        if len(self.activation_times) < 1 or self.activation_times[0] != 0:
            raise ValueError("activation_times must start with a[0] = 0")

    @property
    def num_levels(self) -> int:
        return len(self.activation_times)

    @property
    def coarsest(self) -> int:
        return len(self.activation_times) - 1

    def level_len(self, level: int) -> int:
        self._check_level(level)
        return self.seq_len >> level

    def level_offsets(self) -> Tuple[int, ...]:
        return level_offsets(self.seq_len, self.num_levels)

    @property
    def total_len(self) -> int:
        return self.level_offsets()[-1]

    def _check_level(self, level: int) -> None:
        if not 0 <= level <= self.coarsest:
            raise ValueError(f"level {level} out of range [0, {self.coarsest}]")

    def _check_q(self, q: int) -> None:
        if not 0 <= q < self.seq_len:
            raise ValueError(f"q={q} out of range [0, {self.seq_len})")

    def _check_k(self, k: int, level: int) -> None:
        n = self.level_len(level)
        if not 0 <= k < n:
            raise ValueError(f"k={k} out of range [0, {n}) at level {level}")


class IntOps(NamedTuple):
    """The backend-specific pair (min, max); everything else is + - * >>."""

    minimum: Callable
    maximum: Callable


PY_OPS = IntOps(minimum=min, maximum=max)


def level_row_bounds(q, activation_times: Sequence[int], cache_size: int, ops: IntOps = PY_OPS):
    """[lo, hi) of every level for query q (empty as lo >= hi).  A fine level
    holds the nodes created since its last completed parent pair; the
    coarsest holds what the fine levels leave of the cache, newest first
    (range_spec.py:142-171)."""
    a = tuple(activation_times)
    top = len(a) - 1
    mx = ops.maximum
    out = []
    used = 0
    for lv in range(top):
        newest_end = mx(q - a[lv] + (1 << lv), 0) >> lv
        first_live = (mx(q - a[lv + 1] + (2 << lv), 0) >> (lv + 1)) * 2
        out.append((first_live, newest_end))
        used = used + mx(newest_end - first_live, 0)
    end_top = mx(q - a[top] + (1 << top), 0) >> top
    out.append((mx(end_top - (cache_size - used), 0), end_top))
    return tuple(out)


def level_row_bounds_one(q, level: int, activation_times: Sequence[int], cache_size: int,
                         ops: IntOps = PY_OPS):
    return level_row_bounds(q, activation_times, cache_size, ops)[level]


def block_hull(q_lo: int, q_hi: int, level: int, activation_times: Sequence[int], cache_size: int,
               ops: IntOps = PY_OPS):
    """Hull of the level ranges over [q_lo, q_hi): both bounds are monotone in
    q, so it is [lo(q_lo), hi(q_hi - 1)) (range_spec.py:187-202)."""
    lo = level_row_bounds_one(q_lo, level, activation_times, cache_size, ops)[0]
    hi = level_row_bounds_one(q_hi - 1, level, activation_times, cache_size, ops)[1]
    return lo, hi


def normalize_empty(bounds: Tuple[int, int]) -> Tuple[int, int]:
    lo, hi = bounds
    return (lo, hi) if lo < hi else (0, 0)


def level_lens(seq_len: int, num_levels: int) -> Tuple[int, ...]:
    return tuple(seq_len >> lv for lv in range(num_levels))


def level_offsets(seq_len: int, num_levels: int) -> Tuple[int, ...]:
    acc, out = 0, [0]
    for n in level_lens(seq_len, num_levels):
        acc += n
        out.append(acc)
    return tuple(out)


def node_query_hull(k, level: int, activation_times: Sequence[int], coarsest_span: int,
                    seq_len: int, ops: IntOps = PY_OPS):
    """Queries that can see node k of `level`: from its creation to its
    parent's creation (fine levels) or `coarsest_span` later (coarsest),
    clamped to N (range_spec.py:230-253)."""
    a = tuple(activation_times)
    top = len(a) - 1
    born = a[level] + (k << level)
    if level < top:
        gone = a[level + 1] + ((k >> 1) << (level + 1))
    else:
        gone = born + coarsest_span
    return born, ops.minimum(gone, seq_len)


def tile_query_hull(k_lo: int, k_hi: int, level: int, activation_times: Sequence[int],
                    coarsest_span: int, seq_len: int, ops: IntOps = PY_OPS):
    """Hull of node_query_hull over nodes [k_lo, k_hi), the last node clamped
    to the newest one created before N (range_spec.py:256-281)."""
    last_created = (seq_len - activation_times[level] - 1) >> level
    k_last = ops.minimum(k_hi - 1, last_created)
    lo = node_query_hull(k_lo, level, activation_times, coarsest_span, seq_len, ops)[0]
    hi = node_query_hull(k_last, level, activation_times, coarsest_span, seq_len, ops)[1]
    return lo, hi


_SPAN_CACHE: Dict[Tuple, int] = {}


def coarsest_lifetime_span(spec) -> int:
    """Longest lifetime of a coarsest node evicted before N (N if none is);
    one O(N) scan per schedule in the C library, memoised
    (range_spec.py:287-317)."""
    key = (tuple(spec.activation_times), spec.cache_size, spec.seq_len)
    hit = _SPAN_CACHE.get(key)
    if hit is None:
        hit = int(native_schedule(spec).coarsest_span)
        _SPAN_CACHE[key] = hit
    return hit


def range_bounds(spec: RangeSpec, q: int, level: int) -> Tuple[int, int]:
    """Exact level-local range of query q (range_spec.py:324-336)."""
    spec._check_q(q)
    spec._check_level(level)
    lo, hi = normalize_empty(level_row_bounds_one(q, level, spec.activation_times, spec.cache_size))
    if hi > spec.level_len(level):
        raise AssertionError(
            f"range [{lo},{hi}) exceeds level_len={spec.level_len(level)} at q={q}, level={level}")
    return lo, hi


def packed_bounds(spec: RangeSpec, q: int, level: int) -> Tuple[int, int]:
    lo, hi = range_bounds(spec, q, level)
    if lo == hi:
        return EMPTY
    base = spec.level_offsets()[level]
    return base + lo, base + hi


def elem_mask(spec: RangeSpec, q: int, k_local: int, level: int) -> bool:
    spec._check_k(k_local, level)
    lo, hi = range_bounds(spec, q, level)
    return lo <= k_local < hi


def fwd_bounds(spec: RangeSpec, q_lo: int, q_hi: int, level: int) -> Tuple[int, int]:
    if not 0 <= q_lo <= q_hi <= spec.seq_len:
        raise ValueError(f"[q_lo, q_hi)=[{q_lo},{q_hi}) not within [0, {spec.seq_len}]")
    spec._check_level(level)
    if q_lo == q_hi:
        return EMPTY
    return normalize_empty(block_hull(q_lo, q_hi, level, spec.activation_times, spec.cache_size))


def node_query_bounds(spec: RangeSpec, k: int, level: int) -> Tuple[int, int]:
    spec._check_k(k, level)
    return normalize_empty(node_query_hull(k, level, spec.activation_times,
                                           coarsest_lifetime_span(spec), spec.seq_len))


def bwd_bounds(spec: RangeSpec, k_lo: int, k_hi: int, level: int) -> Tuple[int, int]:
    spec._check_level(level)
    n = spec.level_len(level)
    if not 0 <= k_lo <= k_hi <= n:
        raise ValueError(f"[k_lo, k_hi)=[{k_lo},{k_hi}) not within [0, {n}]")
    if k_lo == k_hi:
        return EMPTY
    return normalize_empty(tile_query_hull(k_lo, k_hi, level, spec.activation_times,
                                           coarsest_lifetime_span(spec), spec.seq_len))


# ---------------------------------------------------------------------------
# native schedule (the C struct the kernels consume)
# ---------------------------------------------------------------------------

_NATIVE_CACHE: Dict[Tuple, object] = {}


def native_schedule(spec):
    """The tc_schedule struct of a RangeSpec (activation times, level
    lengths, packed offsets, coarsest span), memoised per schedule."""
    from . import _lib

    key = (tuple(spec.activation_times), spec.cache_size, spec.seq_len)
    hit = _NATIVE_CACHE.get(key)
    if hit is None:
        if len(spec.activation_times) > _lib.MAX_LEVELS:
            raise NotImplementedError(f"at most {_lib.MAX_LEVELS} levels are supported")
        act = (ctypes.c_int32 * len(spec.activation_times))(*spec.activation_times)
        hit = _lib.Schedule()
        _lib.check(_lib.lib().tc_schedule_from_times(
            ctypes.cast(act, ctypes.c_void_p), len(spec.activation_times), spec.cache_size,
            spec.seq_len, ctypes.byref(hit)), "tc_schedule_from_times")
        _NATIVE_CACHE[key] = hit
    return hit


_STATS_CACHE: Dict[Tuple, Tuple[int, int, int]] = {}


def visible_stats(spec) -> Tuple[int, int, int]:
    """(min, max, sum) over queries of the visible-entry count |A(q)|."""
    from . import _lib

    key = (tuple(spec.activation_times), spec.cache_size, spec.seq_len)
    hit = _STATS_CACHE.get(key)
    if hit is None:
        out = (ctypes.c_int64 * 3)()
        _lib.check(_lib.lib().tc_schedule_stats(ctypes.byref(native_schedule(spec)),
                                                ctypes.cast(out, ctypes.c_void_p)),
                   "tc_schedule_stats")
        hit = (int(out[0]), int(out[1]), int(out[2]))
        _STATS_CACHE[key] = hit
    return hit


__all__ = [
    "EMPTY", "RangeSpec", "IntOps", "PY_OPS", "activation_times_from_fmap", "level_row_bounds",
    "level_row_bounds_one", "block_hull", "normalize_empty", "level_lens", "level_offsets",
    "node_query_hull", "tile_query_hull", "coarsest_lifetime_span", "range_bounds",
    "packed_bounds", "elem_mask", "fwd_bounds", "node_query_bounds", "bwd_bounds",
]
