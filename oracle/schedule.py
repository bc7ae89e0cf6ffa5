"""Integer schedule oracle (TEST INFRASTRUCTURE, see ``oracle/__init__.py``).

Restates, in deliberately naive form, the schedule semantics of the
reference:

* activation times ``a[l]`` and the dyadic alignment check --
  ``telescoping_attn/range_spec.py:26-54``;
* per-query level ranges from the ruler/slot policy (newest/oldest node per
  level, coarsest level fills the remaining cache and evicts oldest first) --
  the analytic formulation of ``test/test_reference.py:322-395``, which the
  reference's branch-free closed form (``range_spec.py:142-171``) must equal;
* hulls by brute force over those ranges (``range_spec.py:187-281``,
  ``:360-402``);
* the coarsest-level lifetime span (``range_spec.py:287-317``);
* decode ring capacities (``reference.py:1739-1772``) and ring slots
  (``reference.py:1775-1784``);
* chronological bin distances by sorting the visible entries
  (``reference.py:327-371``; ``minimal_reference.py:53-69``).

Everything here is plain Python on ints.  It is slow on purpose: the product
computes the same quantities with O(1) closed forms.
"""

from typing import Dict, List, Sequence, Tuple


def activation_times(fmap: Dict[int, int]) -> Tuple[int, ...]:
    """a[0..L] from a schedule map {level: slots}; raises on a bad map.

    range_spec.py:26-54 -- a[1] = fmap[1] + 1 and
    a[l] = a[l-1] + 2^(l-1) (fmap[l] - fmap[l-1]) + 2^(l-2), with the phase
    check a[l] mod 2^l == 2^(l-1).
    """
    if not fmap:
        return (0,)
    top = max(fmap)
    if sorted(fmap) != list(range(1, top + 1)):
        raise ValueError("fmap keys must be consecutive 1..L")
    a = [0, fmap[1] + 1]
    for lv in range(2, top + 1):
        a.append(a[-1] + 2 ** (lv - 1) * (fmap[lv] - fmap[lv - 1]) + 2 ** (lv - 2))
    for lv in range(1, top + 1):
        if a[lv] % 2 ** lv != 2 ** (lv - 1):
            raise ValueError(f"fmap not dyadically aligned at level {lv}")
    return tuple(a)


def level_lens(seq_len: int, num_levels: int) -> List[int]:
    """Node count per level: N, N//2, N//4, ... (range_spec.py:85-91)."""
    out, n = [], seq_len
    for _ in range(num_levels):
        out.append(n)
        n //= 2
    return out


def level_offsets(seq_len: int, num_levels: int) -> List[int]:
    """Prefix sums of level_lens, len num_levels + 1 (range_spec.py:93-102)."""
    off = [0]
    for n in level_lens(seq_len, num_levels):
        off.append(off[-1] + n)
    return off


def row_ranges(q: int, a: Sequence[int], cache: int) -> List[Tuple[int, int]]:
    """Visible [lo, hi) per level for query q, EMPTY as (0, 0).

    Ruler/slot policy (test_reference.py:322-395): at fine level l the newest
    node is (q - a[l]) // 2^l once q >= a[l]; every parent completed at level
    l+1 removes its two children, so the oldest live node is
    2 * (newest_parent + 1) once q >= a[l+1].  The coarsest level holds what
    the fine levels leave of the cache, newest first.
    """
    top = len(a) - 1
    out = []
    used = 0
    for lv in range(top):
        if q < a[lv]:
            out.append((0, 0))
            continue
        newest = (q - a[lv]) // 2 ** lv
        oldest = 0
        if q >= a[lv + 1]:
            oldest = 2 * ((q - a[lv + 1]) // 2 ** (lv + 1) + 1)
        if oldest > newest:
            out.append((0, 0))
        else:
            out.append((oldest, newest + 1))
            used += newest + 1 - oldest
    remaining = cache - used
    if q < a[top] or remaining <= 0:
        out.append((0, 0))
    else:
        newest = (q - a[top]) // 2 ** top
        count = min(remaining, newest + 1)
        out.append((newest - count + 1, newest + 1))
    return out


def all_row_ranges(seq_len: int, a: Sequence[int], cache: int):
    """row_ranges for every query: list indexed [q][level] -> (lo, hi)."""
    return [row_ranges(q, a, cache) for q in range(seq_len)]


def visible_entries(q: int, a: Sequence[int], cache: int) -> List[Tuple[int, int]]:
    """(level, j) visible to q, oldest -> newest by interval start j * 2^level
    (minimal_reference.py:53-69)."""
    ent = []
    for lv, (lo, hi) in enumerate(row_ranges(q, a, cache)):
        ent.extend((lv, j) for j in range(lo, hi))
    ent.sort(key=lambda e: e[1] * 2 ** e[0])
    return ent


def bin_distances(q: int, a: Sequence[int], cache: int) -> Dict[Tuple[int, int], int]:
    """Chronological bin distance of every visible entry: 0 = the query's own
    token, M-1 = the oldest entry (reference.py:327-371, computed here by
    sorting rather than by the reference's rank formula)."""
    ent = visible_entries(q, a, cache)
    m = len(ent)
    return {e: m - 1 - r for r, e in enumerate(ent)}


def fwd_hull(q_lo: int, q_hi: int, level: int, rows) -> Tuple[int, int]:
    """Hull of the level ranges over queries [q_lo, q_hi) (range_spec.py:360-373)."""
    nz = [rows[q][level] for q in range(q_lo, q_hi) if rows[q][level][0] < rows[q][level][1]]
    if not nz:
        return (0, 0)
    return (min(r[0] for r in nz), max(r[1] for r in nz))


def node_queries(seq_len: int, level: int, rows) -> List[List[int]]:
    """For each node of `level`, the sorted queries that see it."""
    n = seq_len >> level
    qs = [[] for _ in range(n)]
    for q in range(seq_len):
        lo, hi = rows[q][level]
        for k in range(lo, hi):
            qs[k].append(q)
    return qs


def bwd_hull(k_lo: int, k_hi: int, node_qs) -> Tuple[int, int]:
    """Hull of the inverse sets over nodes [k_lo, k_hi) (range_spec.py:386-402)."""
    vis = [node_qs[k] for k in range(k_lo, k_hi) if node_qs[k]]
    if not vis:
        return (0, 0)
    return (min(v[0] for v in vis), max(v[-1] for v in vis) + 1)


def coarsest_span(a: Sequence[int], cache: int, seq_len: int) -> int:
    """Longest lifetime of a coarsest node that is evicted before the sequence
    ends; seq_len when nothing is evicted (range_spec.py:287-317)."""
    # Node k of the coarsest level is evicted at the first q whose oldest
    # coarsest node is past k.  "Oldest" is the un-normalised value
    # newest + 1 - remaining (clamped at 0), as the reference's sweep uses it,
    # so a query whose fine levels fill the cache evicts everything older.
    top = len(a) - 1
    n_nodes = seq_len >> top
    span = 0
    evicted = 0
    for q in range(seq_len):
        rr = row_ranges(q, a, cache)
        used = sum(hi - lo for lo, hi in rr[:top])
        hi_top = (q - a[top]) // 2 ** top + 1 if q >= a[top] else 0
        oldest = max(hi_top - (cache - used), 0)
        while evicted < oldest and evicted < n_nodes:
            born = a[top] + evicted * 2 ** top
            if born < seq_len:
                span = max(span, q - born)
            evicted += 1
    return span if span else seq_len


def decode_caps(a: Sequence[int], cache: int) -> Tuple[int, ...]:
    """Per-level ring capacities: the peak live count of each level over two
    schedule periods past the last activation (reference.py:1739-1772)."""
    top = len(a) - 1
    horizon = 2 * (a[top] + 2 ** (top + 1)) + 1
    caps = [0] * (top + 1)
    for q in range(horizon):
        rr = row_ranges(q, a, cache)
        used = 0
        for lv in range(top):
            caps[lv] = max(caps[lv], rr[lv][1] - rr[lv][0])
            used += rr[lv][1] - rr[lv][0]
        if used > cache:
            raise ValueError("fine levels exceed cache_size")
        caps[top] = max(caps[top], cache - used)
    return tuple(caps)


def ring_offsets(caps: Sequence[int]) -> List[int]:
    off = [0]
    for c in caps:
        off.append(off[-1] + c)
    return off


def ring_slot(offsets: Sequence[int], caps: Sequence[int], level: int, j: int) -> int:
    """Physical ring slot of node j at `level` (reference.py:1775-1784)."""
    return offsets[level] + j % caps[level]
