"""Prefill hand-off on the device (tc_decode_init behind init_decode_state):
the rings equal, bit for bit, the reference's placement -- zero rings, then
for every level the nodes live at query N-1 written to
ring_offsets[l] + j % caps[l] (reference.py:1900-1930) -- for level tensors
that are views of one packed buffer, contiguous, or offset so that only
narrow vector copies are aligned, in f32 and bf16, with empty levels."""

import pytest
import torch

import telescope_cache_b200 as T
from telescope_cache_b200 import _lib
from telescope_cache_b200.range_spec import RangeSpec, activation_times_from_fmap, range_bounds

pytestmark = pytest.mark.gpu


def placed_by_index_put(k_levels, v_levels, w_levels, fmap, cache, n):
    """The reference's ring placement, restated with torch indexing on the
    same device (the checker, not the product path)."""
    a = activation_times_from_fmap(fmap)
    caps = T.decode_capacities(a, cache)
    offs = [0]
    for c in caps:
        offs.append(offs[-1] + c)
    B, _, H, Dk = k_levels[0].shape
    Dv = v_levels[0].shape[-1]
    k = k_levels[0].new_zeros(B, offs[-1], H, Dk)
    v = v_levels[0].new_zeros(B, offs[-1], H, Dv)
    w = w_levels[0].new_zeros(B, offs[-1], H, 1)
    spec = RangeSpec(a, cache, n)
    for level in range(len(a)):
        lo, hi = range_bounds(spec, n - 1, level)
        if lo == hi:
            continue
        slots = offs[level] + torch.remainder(torch.arange(lo, hi, device=k.device), caps[level])
        k[:, slots] = k_levels[level][:, lo:hi]
        v[:, slots] = v_levels[level][:, lo:hi]
        w[:, slots] = w_levels[level][:, lo:hi]
    return k, v, w


def make_levels(B, n, H, Dk, Dv, L, dtype, layout, gen):
    lens = [n >> l for l in range(L + 1)]
    total = sum(lens)

    def buf(D):
        x = torch.randn(B, total, H, D, generator=gen).to("cuda", dtype)
        if layout == "odd":
            # the same values one element past an aligned allocation: only
            # element-wide vector copies are aligned
            flat = torch.empty(x.numel() + 1, device="cuda", dtype=dtype)
            flat[1:] = x.reshape(-1)
            x = flat[1:].view(B, total, H, D)
        return x

    kp, vp = buf(Dk), buf(Dv)
    wp = torch.randn(B, total, H, 1, generator=gen).to("cuda", dtype)
    out = ([], [], [])
    off = 0
    for m in lens:
        for lst, p in zip(out, (kp, vp, wp)):
            view = p[:, off:off + m]
            lst.append(view.contiguous() if layout == "contiguous" else view)
        off += m
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("layout", ["views", "contiguous", "odd"])
@pytest.mark.parametrize("shape", [(3, 100, 2, 16, 16), (2, 7, 3, 24, 40), (1, 333, 1, 8, 8)])
def test_rings_equal_reference_placement(dtype, layout, shape):
    B, n, H, Dk, Dv = shape
    fmap, cache = {1: 8, 2: 16, 3: 24}, 32
    gen = torch.Generator().manual_seed(n * 7 + H)
    kl, vl, wl = make_levels(B, n, H, Dk, Dv, 3, dtype, layout, gen)
    before = _lib.launch_count()
    st = T.init_decode_state(kl, vl, wl, fmap, cache)
    assert _lib.launch_count() > before  # the placement ran in the library
    k, v, w = placed_by_index_put(kl, vl, wl, fmap, cache, n)
    assert st.t == n
    assert torch.equal(st.k, k) and torch.equal(st.v, v) and torch.equal(st.w, w)


def test_rings_after_garbage_are_rewritten_whole():
    """The rings come from torch.empty: a slot with no live node must read
    zero even when the allocator hands back memory that held other data."""
    gen = torch.Generator().manual_seed(5)
    kl, vl, wl = make_levels(2, 40, 2, 16, 16, 3, torch.bfloat16, "views", gen)
    fmap, cache = {1: 8, 2: 16, 3: 24}, 32
    for _ in range(2):
        junk = torch.full((1 << 20,), float("nan"), device="cuda")
        del junk
        st = T.init_decode_state(kl, vl, wl, fmap, cache)
        k, v, w = placed_by_index_put(kl, vl, wl, fmap, cache, 40)
        assert torch.equal(st.k, k) and torch.equal(st.v, v) and torch.equal(st.w, w)
