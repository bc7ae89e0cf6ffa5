"""Gradients through the standalone differentiable helpers of the reference
API -- short_conv (reference.py:167-211), compute_summary_weights
(reference.py:117-145) and apply_rope (reference.py:267-302) -- against
torch autograd of the reference's formulas in fp32 on the same inputs, and
the segment resets of short_conv (the seq_idx extension; the reference
leaves them as a TODO at reference.py:186-189) against the CPU oracle and
against each packed example convolved on its own.
Tolerance: fp32 normwise 1e-5; bf16 normwise 2e-2."""

import numpy as np
import pytest
import torch

import telescope_cache_b200 as T
from oracle import numerics as O

pytestmark = pytest.mark.gpu


def _close(got, want, dtype):
    got, want = got.detach().double().cpu(), want.detach().double().cpu()
    rel = ((got - want).norm() / max(want.norm().item(), 1e-30)).item()
    assert rel <= (1e-5 if dtype == torch.float32 else 2e-2), f"normwise {rel:.3e}"


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _conv_formula(x, w):
    """The reference's short_conv in fp32 torch ops (autograd-able)."""
    K = w.shape[1]
    xf = x.float()
    xp = torch.nn.functional.pad(xf, (0, 0, K - 1, 0))
    acc = sum(w.float()[:, j] * xp[:, j:j + x.shape[1]] for j in range(K))
    return xf + acc


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K", [1, 3, 4])
def test_short_conv_gradients(dtype, K):
    torch.cuda.set_device(0)
    g = _gen(20 + K)
    B, N, C = 2, 300, 48
    x = torch.randn(B, N, C, generator=g, device="cuda").to(dtype)
    w = (torch.randn(C, K, generator=g, device="cuda") / K).to(dtype)
    dy = torch.randn(B, N, C, generator=g, device="cuda").to(dtype)
    x1, w1 = _leaf(x), _leaf(w)
    y = T.short_conv(x1, w1)
    assert y.grad_fn is not None
    dx, dw = torch.autograd.grad(y, (x1, w1), dy)
    x2, w2 = _leaf(x.float()), _leaf(w.float())
    y2 = _conv_formula(x2, w2)
    dx2, dw2 = torch.autograd.grad(y2, (x2, w2), dy.float())
    assert dx.dtype == dtype and dw.dtype == dtype
    _close(y.detach(), y2.detach(), dtype)
    _close(dx, dx2, dtype)
    _close(dw, dw2, dtype)
    # without gradients: the same values, no graph
    with torch.no_grad():
        assert torch.equal(T.short_conv(x, w), y.detach())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_summary_weights_gradients(dtype):
    torch.cuda.set_device(0)
    g = _gen(31)
    for (B, N, Hq, Hkv, Dk) in ((2, 70, 8, 2, 64), (1, 33, 4, 4, 128), (2, 17, 6, 3, 256)):
        q = torch.randn(B, N, Hq, Dk, generator=g, device="cuda").to(dtype)
        k = torch.randn(B, N, Hkv, Dk, generator=g, device="cuda").to(dtype)
        dw = torch.randn(B, N, Hkv, 1, generator=g, device="cuda").to(dtype)
        q1, k1 = _leaf(q), _leaf(k)
        w = T.compute_summary_weights(q1, k1)
        dq, dk = torch.autograd.grad(w, (q1, k1), dw)
        q2, k2 = _leaf(q.float()), _leaf(k.float())
        s = (q2.reshape(B, N, Hkv, Hq // Hkv, Dk) * k2.unsqueeze(3)).sum(-1) / Dk ** 0.5
        w2 = torch.logsumexp(s, dim=3, keepdim=True)
        dq2, dk2 = torch.autograd.grad(w2, (q2, k2), dw.float())
        _close(w.detach(), w2.detach(), dtype)
        _close(dq, dq2, dtype)
        _close(dk, dk2, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("inverse", [False, True])
def test_rope_gradients(dtype, inverse):
    torch.cuda.set_device(0)
    g = _gen(41)
    B, N, H, D = 2, 50, 3, 64
    cos, sin = T.rope_tables(N, D, device="cuda")
    x = torch.randn(B, N, H, D, generator=g, device="cuda").to(dtype)
    dy = torch.randn(B, N, H, D, generator=g, device="cuda").to(dtype)
    pos = torch.arange(N, device="cuda")[None, :, None]
    x1 = _leaf(x)
    y = T.apply_rope(x1, pos, cos, sin, inverse=inverse)
    (dx,) = torch.autograd.grad(y, (x1,), dy)
    x2 = _leaf(x.float())
    c, s = cos[pos], sin[pos]
    if inverse:
        s = -s
    a, b = x2[..., : D // 2], x2[..., D // 2:]
    y2 = torch.cat([a * c - b * s, b * c + a * s], dim=-1)
    (dx2,) = torch.autograd.grad(y2, (x2,), dy.float())
    assert dx.dtype == dtype
    _close(y.detach(), y2.detach(), dtype)
    _close(dx, dx2, dtype)
    with pytest.raises(NotImplementedError):
        T.apply_rope(x1, pos, cos.clone().requires_grad_(True), sin)


def _segments(B, N, seed):
    """Segment ids [B, N]: ragged packed examples, one of length 1, one row
    a single example."""
    r = np.random.Generator(np.random.PCG64(seed))
    seq = np.zeros((B, N), np.int32)
    for b in range(B - 1):
        cuts = np.sort(r.choice(np.arange(1, N), size=5, replace=False))
        cuts[1] = cuts[0] + 1  # a one-row example
        for i, c0 in enumerate(cuts):
            seq[b, c0:] = i + 1
    return seq


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_short_conv_segments_match_oracle_and_separate_examples(dtype):
    torch.cuda.set_device(0)
    B, N, C, K = 3, 600, 40, 4
    r = np.random.Generator(np.random.PCG64(7))
    x_np = r.standard_normal((B, N, C)).astype(np.float32)
    w_np = (r.standard_normal((C, K)) / K).astype(np.float32)
    dy_np = r.standard_normal((B, N, C)).astype(np.float32)
    seq_np = _segments(B, N, 8)
    x = torch.from_numpy(x_np).cuda().to(dtype)
    w = torch.from_numpy(w_np).cuda().to(dtype)
    seq = torch.from_numpy(seq_np).cuda()
    x1, w1 = _leaf(x), _leaf(w)
    y = T.short_conv(x1, w1, seq_idx=seq)
    dyt = torch.from_numpy(dy_np).cuda().to(dtype)
    dx, dw = torch.autograd.grad(y, (x1, w1), dyt)
    xf, wf = x.float().cpu().numpy(), w.float().cpu().numpy()
    want_y = O.short_conv(xf, wf, seq_np)
    want_dx, want_dw = O.short_conv_vjp(xf, wf, dyt.float().cpu().numpy(), seq_np)
    _close(y.detach(), torch.from_numpy(want_y), dtype)
    _close(dx, torch.from_numpy(want_dx), dtype)
    _close(dw, torch.from_numpy(want_dw), dtype)
    # each example on its own (zero history at its first row): the same bits
    # for y and dx (the taps run in the same order)
    with torch.no_grad():
        for b in range(B):
            ids = seq_np[b]
            starts = [0] + [i for i in range(1, N) if ids[i] != ids[i - 1]] + [N]
            for s0, s1 in zip(starts[:-1], starts[1:]):
                alone = T.short_conv(x[b:b + 1, s0:s1], w)
                assert torch.equal(alone, y.detach()[b:b + 1, s0:s1])
    # one segment id per row = no resets
    same = torch.full((B, N), 3, dtype=torch.int32, device="cuda")
    with torch.no_grad():
        assert torch.equal(T.short_conv(x, w, seq_idx=same), T.short_conv(x, w))
    with pytest.raises(ValueError):
        T.short_conv(x, w, seq_idx=seq[:, :-1])


def test_builder_and_decode_hand_off_with_segments():
    """build_dyadic_summaries(seq_idx=...) equals the builder on keys and
    values convolved per example; gradients reach the conv weights; the
    decode hand-off zeroes history rows of earlier examples."""
    torch.cuda.set_device(0)
    g = _gen(51)
    B, N, Hq, Hkv, D, K, L = 2, 256, 4, 2, 64, 4, 4
    q = torch.randn(B, N, Hq, D, generator=g, device="cuda")
    k = torch.randn(B, N, Hkv, D, generator=g, device="cuda")
    v = torch.randn(B, N, Hkv, D, generator=g, device="cuda")
    kcw = torch.randn(Hkv * D, K, generator=g, device="cuda") / K
    vcw = torch.randn(Hkv * D, K, generator=g, device="cuda") / K
    seq = torch.from_numpy(_segments(B, N, 9)).cuda()
    with torch.no_grad():
        kl, vl, wl = T.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw, v_conv_weight=vcw, seq_idx=seq)
        kc = T.short_conv(k.reshape(B, N, -1), kcw, seq).reshape(B, N, Hkv, D)
        vc = T.short_conv(v.reshape(B, N, -1), vcw, seq).reshape(B, N, Hkv, D)
        kl2, vl2, wl2 = T.build_dyadic_summaries(q, kc, vc, L)
        for a, b_ in zip(kl + vl + wl, kl2 + vl2 + wl2):
            assert torch.equal(a, b_)
        # all one segment: the fused-conv builder's values
        one = torch.zeros(B, N, dtype=torch.int32, device="cuda")
        kl3, _, wl3 = T.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw, v_conv_weight=vcw, seq_idx=one)
        kl4, _, wl4 = T.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw, v_conv_weight=vcw)
        for a, b_ in zip(kl3 + wl3, kl4 + wl4):
            _close(a, b_, torch.float32)
    kcw1 = _leaf(kcw)
    kl, vl, wl = T.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw1, v_conv_weight=vcw, seq_idx=seq)
    (gk,) = torch.autograd.grad(sum(t.float().sum() for t in kl) + sum(t.sum() for t in wl), (kcw1,))
    assert torch.isfinite(gk).all() and gk.abs().sum() > 0
    # hand-off: the last example of row 0 starts two rows before the end
    seq_h = torch.zeros(B, N, dtype=torch.int32, device="cuda")
    seq_h[0, N - 2:] = 1
    with torch.no_grad():
        kl, vl, wl = T.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw, v_conv_weight=vcw, seq_idx=seq_h)
        st = T.init_decode_state(kl, vl, wl, {1: 8, 2: 16, 3: 24}, 32, k_pre_conv=k, v_pre_conv=v, conv_kernel_size=K,
                                 seq_idx=seq_h)
        kf = k.reshape(B, N, -1)
        assert torch.equal(st.conv_k[0, 0], torch.zeros_like(kf[0, 0]))
        assert torch.equal(st.conv_k[0, 1:], kf[0, N - 2:])
        assert torch.equal(st.conv_k[1], kf[1, N - K + 1:])
