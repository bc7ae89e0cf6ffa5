"""The oracle's segment-reset short conv (the seq_idx extension; the
reference leaves the resets as a TODO at reference.py:186-189, so no
reference golden exists for it).  Pinned by properties instead: packed
examples convolved together equal each example convolved alone, one
segment per row equals the reference conv, and the VJP is the adjoint of
the forward (<dy, J dx> = <J^T dy, dx>)."""

import numpy as np

from oracle import numerics as O


def _seq(rng, B, N, n_cut):
    seq = np.zeros((B, N), np.int32)
    for b in range(B):
        for i, c in enumerate(np.sort(rng.choice(np.arange(1, N), n_cut, replace=False))):
            seq[b, c:] = i + 1
    return seq


def test_segments_equal_separate_examples():
    rng = np.random.Generator(np.random.PCG64(3))
    B, N, C, K = 2, 97, 6, 4
    x = rng.standard_normal((B, N, C))
    w = rng.standard_normal((C, K))
    seq = _seq(rng, B, N, 7)
    y = O.short_conv(x, w, seq)
    for b in range(B):
        cuts = [0] + list(np.flatnonzero(np.diff(seq[b])) + 1) + [N]
        for s0, s1 in zip(cuts[:-1], cuts[1:]):
            np.testing.assert_array_equal(O.short_conv(x[b:b + 1, s0:s1], w), y[b:b + 1, s0:s1])
    np.testing.assert_array_equal(O.short_conv(x, w, np.full((B, N), 5)), O.short_conv(x, w))


def test_segment_vjp_is_the_adjoint():
    rng = np.random.Generator(np.random.PCG64(4))
    B, N, C, K = 2, 64, 5, 3
    x = rng.standard_normal((B, N, C))
    w = rng.standard_normal((C, K))
    dy = rng.standard_normal((B, N, C))
    seq = _seq(rng, B, N, 5)
    dx, dw = O.short_conv_vjp(x, w, dy, seq)
    # the conv is linear in x for fixed w and linear in w for fixed x
    ux = rng.standard_normal(x.shape)
    uw = rng.standard_normal(w.shape)
    jx = O.short_conv(ux, w, seq)  # J_x ux (residual included)
    jw = O.short_conv(x, w + uw, seq) - O.short_conv(x, w, seq)
    np.testing.assert_allclose((dy * jx).sum(), (dx * ux).sum(), rtol=1e-12)
    np.testing.assert_allclose((dy * jw).sum(), (dw * uw).sum(), rtol=1e-10)
    # no segments: the reference conv's VJP
    dx0, dw0 = O.short_conv_vjp(x, w, dy)
    dx1, dw1 = O.short_conv_vjp(x, w, dy, np.zeros((B, N), np.int32))
    np.testing.assert_array_equal(dx0, dx1)
    np.testing.assert_array_equal(dw0, dw1)
