"""Host-side index arithmetic of the prefill hand-off (tc_decode_init): for
every schedule and a spread of prefill lengths, the live ranges the wrapper
passes (range_bounds of query N-1) equal the oracle's, each level's live
count fits its ring, and the kernel's slot -> node rule (the one node j in
[lo, hi) with j mod cap = slot - ring_off[l]) reproduces the oracle's
placement (node j at ring_off[l] + j mod cap, reference.py:1900-1930) slot for
slot.  The kernel itself is checked on the GPU in test_gpu_decode_init.py."""

import pytest

import cases as C
from oracle import schedule as S
from telescope_cache_b200.range_spec import RangeSpec, range_bounds


def kernel_rule(slot, offs, caps, lo, hi):
    """decode_init_kernel's mapping, restated: (level, node) or (level, None)."""
    l = 0
    while l + 1 < len(caps) and slot >= offs[l + 1]:
        l += 1
    cap, r = caps[l], slot - offs[l]
    if lo[l] < hi[l]:
        j = lo[l] + ((r - lo[l] % cap) % cap + cap) % cap
        if j < hi[l]:
            return l, j
    return l, None


@pytest.mark.parametrize("sched", [s[0] for s in C.SCHEDULES])
def test_slot_rule_matches_oracle_placement(sched):
    _, n_max, cache, fmap = next(s for s in C.SCHEDULES if s[0] == sched)
    a = S.activation_times(fmap)
    caps = S.decode_caps(a, cache)
    offs = S.ring_offsets(caps)
    lens = sorted({1, 2, 3, 7, max(a) + 1, n_max // 3, n_max // 2 + 5, n_max - 1, n_max} - {0})
    for n in (x for x in lens if 1 <= x <= n_max):
        rr = S.row_ranges(n - 1, a, cache)
        spec = RangeSpec(a, cache, n)
        lo, hi = [], []
        for lv in range(len(a)):
            got = range_bounds(spec, n - 1, lv)
            want = rr[lv] if rr[lv][0] < rr[lv][1] else (0, 0)
            assert tuple(got) == tuple(want), (sched, n, lv)
            assert got[1] - got[0] <= caps[lv], (sched, n, lv)
            lo.append(got[0])
            hi.append(got[1])
        placed = {}
        for lv in range(len(a)):
            for j in range(lo[lv], hi[lv]):
                s = S.ring_slot(offs, caps, lv, j)
                assert s not in placed, (sched, n, lv, j)
                placed[s] = (lv, j)
        for s in range(offs[-1]):
            lv, j = kernel_rule(s, offs, caps, lo, hi)
            assert placed.get(s, (lv, None)) == (lv, j), (sched, n, s)


def test_cpu_levels_raise_no_fallback():
    """The hand-off computes on CUDA tensors only: CPU level tensors raise
    before any launch instead of taking a CPU path."""
    import torch

    import telescope_cache_b200 as T
    n, fmap, cache = 40, {1: 8, 2: 16, 3: 24}, 32
    kl = [torch.zeros(1, n >> l, 2, 8) for l in range(4)]
    wl = [torch.zeros(1, n >> l, 2, 1) for l in range(4)]
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        T.init_decode_state(kl, kl, wl, fmap, cache)


@pytest.mark.parametrize("bad", ["k_batch", "k_heads", "v_dim", "w_heads"])
def test_mismatched_level_raises_before_launch(bad):
    """A level with live nodes whose batch, head count or head dim differs
    from level 0's raises ValueError before anything is launched (the kernel
    would copy level 0's row size from it); the reference fails on the ring
    write of that level instead."""
    import torch

    import telescope_cache_b200 as T
    n, fmap, cache = 40, {1: 8, 2: 16, 3: 24}, 32
    kl = [torch.zeros(2, n >> l, 2, 8) for l in range(4)]
    vl = [torch.zeros(2, n >> l, 2, 8) for l in range(4)]
    wl = [torch.zeros(2, n >> l, 2, 1) for l in range(4)]
    if bad == "k_batch":
        kl[1] = torch.zeros(1, n >> 1, 2, 8)
    elif bad == "k_heads":
        kl[2] = torch.zeros(2, n >> 2, 1, 8)
    elif bad == "v_dim":
        vl[1] = torch.zeros(2, n >> 1, 2, 4)
    else:
        wl[2] = torch.zeros(2, n >> 2, 3, 1)
    with pytest.raises(ValueError, match="shape"):
        T.init_decode_state(kl, vl, wl, fmap, cache)


def test_conv_history_segments():
    """The hand-off's conv history (last K-1 pre-conv rows, zero-padded on the
    left) with segment ids: rows of an earlier packed example than the last
    row's are zeroed; without ids, or with one example, it is the plain tail."""
    import torch

    from telescope_cache_b200.telescoping_attn.decode_state import _conv_history

    x = torch.arange(2 * 6 * 3, dtype=torch.float32).reshape(2, 6, 3) + 1
    seq = torch.tensor([[0, 0, 0, 1, 1, 1], [0, 0, 0, 0, 2, 2]])
    h = _conv_history(x, 4, seq)
    assert torch.equal(h[0], x[0, 3:])                       # the last example covers all K-1 rows
    assert torch.equal(h[1, 0], torch.zeros(3)) and torch.equal(h[1, 1:], x[1, 4:])
    assert torch.equal(_conv_history(x, 4), x[:, 3:])
    assert torch.equal(_conv_history(x, 4, torch.zeros(2, 6, dtype=torch.long)), x[:, 3:])
    # shorter prefill than K-1: left zero padding, then the segment rule
    short = _conv_history(x[:, :2], 4, seq[:, :2])
    assert short.shape == (2, 3, 3) and torch.equal(short[:, 0], torch.zeros(2, 3))
    assert torch.equal(short[:, 1:], x[:, :2])
    # a history is a copy: updating it leaves the prefill rows alone
    h[0, 0, 0] = -1.0
    assert x[0, 3, 0] != -1.0
