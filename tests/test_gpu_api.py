"""The remaining reference API on CUDA: standalone helpers (weights, conv,
RoPE, relative states), attend-only / advance-only decode, and autograd
through the differentiable forward, sink and gate -- each against the CPU
oracle or an explicit composition (reference suite tolerances)."""

import math

import numpy as np
import pytest
import torch

import cases as C
import telescope_cache_b200 as T
from oracle import numerics as O
from oracle import schedule as S

pytestmark = pytest.mark.gpu


def t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def test_standalone_weights_conv_rope():
    r = rng(1)
    q = r.standard_normal((2, 9, 4, 8)).astype(np.float32)
    k = r.standard_normal((2, 9, 2, 8)).astype(np.float32)
    x = r.standard_normal((2, 9, 16)).astype(np.float32)
    wp = r.standard_normal((2, 16)).astype(np.float32)
    w = r.standard_normal((16, 3)).astype(np.float32)
    np.testing.assert_allclose(T.compute_summary_weights(t(q), t(k))[..., 0].cpu().numpy(),
                               O.qk_weights(q, k), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(T.compute_linear_weights(t(x), t(wp))[..., 0].cpu().numpy(),
                               O.linear_weights(x, wp), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(T.short_conv(t(x), t(w)).cpu().numpy(), O.short_conv(x, w),
                               rtol=1e-5, atol=1e-5)
    cos, sin = T.rope_tables(9, 8, device="cuda")
    c_np, s_np = O.rope_tables(9, 8)
    np.testing.assert_allclose(cos.cpu().numpy(), c_np, rtol=1e-6, atol=1e-6)
    pos = torch.arange(9, device="cuda")[None, :, None]
    got = T.apply_rope(t(q), pos, cos, sin).cpu().numpy()
    np.testing.assert_allclose(got, O.rotate(q, np.arange(9)[None, :, None], c_np, s_np),
                               rtol=1e-5, atol=1e-5)
    back = T.apply_rope(t(got), pos, cos, sin, inverse=True).cpu().numpy()
    np.testing.assert_allclose(back, q, rtol=1e-5, atol=1e-5)
    # bf16 conv: fp32 residual then one cast (reference.py:167-211)
    xb = (t(x) * 100).to(torch.bfloat16)
    want = (xb.float() + torch.from_numpy(O.short_conv(xb.float().cpu().numpy(), w) -
                                          xb.float().cpu().numpy()).float().cuda()).to(torch.bfloat16)
    assert torch.equal(T.short_conv(xb, t(w)), want)


def test_decode_attend_only_and_advance_only():
    """multilevel_attention_decode (state untouched) and advance_decode_state
    reproduce decode_step, and the stats list the oracle's visible set."""
    c = C.CASE_BY_NAME["dec_plain_four"]
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c)
    d = {k: t(v) for k, v in inp.items()}
    n0 = g["N"] - 5
    kl, vl, wl = T.build_dyadic_summaries(d["q"][:, :n0], d["k"][:, :n0], d["v"][:, :n0], 3)
    st_a = T.init_decode_state(kl, vl, wl, g["fmap"], g["cache"])
    st_b = T.init_decode_state(kl, vl, wl, g["fmap"], g["cache"])
    for i in range(5):
        ti = n0 + i
        sl = slice(ti, ti + 1)
        out_a, lse_a = T.decode_step(d["x"][:, sl], d["q"][:, sl], d["k"][:, sl], d["v"][:, sl], st_a)
        T.advance_decode_state(st_b, d["q"][:, sl], d["k"][:, sl], d["v"][:, sl])
        out_b, lse_b, stats = T.multilevel_attention_decode(d["q"][:, sl], st_b)
        torch.testing.assert_close(out_b, out_a, rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(lse_b, lse_a, rtol=1e-6, atol=1e-6)
        a = S.activation_times(g["fmap"])
        want = S.visible_entries(ti, a, g["cache"])
        assert sorted(stats["entries"], key=lambda e: e[1] << e[0]) == want
    assert st_a.t == st_b.t == g["N"]


def test_autograd_forward_matches_explicit_backward():
    """Gradients through multilevel_attention_forward + sink (autograd) equal
    the explicit sink-backward + multilevel_attention_backward composition."""
    c = C.CASE_BY_NAME["bwd_rel_sink_tiny"]
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c)
    d = {k: t(v) for k, v in inp.items()}
    with torch.no_grad():
        kl, vl, _ = T.build_dyadic_summaries(d["q"], d["k"], d["v"], len(g["fmap"]))
        packed = T.pack_levels(kl, vl)
    q = d["q"].clone().requires_grad_(True)
    pk = packed.k.clone().requires_grad_(True)
    pv = packed.v.clone().requires_grad_(True)
    st = d["states"].clone().requires_grad_(True)
    pj = d["rel_proj"].clone().requires_grad_(True)
    sinks = d["sinks"].clone().requires_grad_(True)
    pk_ = T.PackedKV(pk, pv, packed.level_offsets)
    out, lse = T.multilevel_attention_forward(q, pk_, g["fmap"], g["cache"], softcap=c["softcap"],
                                              position_mode="relative", relative_states=st,
                                              relative_proj=pj)
    final = T.apply_attention_sink(out, lse, sinks)
    grads = torch.autograd.grad(final, (q, pk, pv, st, pj, sinks), d["dout"])
    dout_pre, dlse, dsinks = T.attention_sink_backward(out.detach(), lse.detach(), sinks.detach(),
                                                       d["dout"])
    dq, dk, dv, dpos, _ = T.multilevel_attention_backward(
        q.detach(), T.PackedKV(pk.detach(), pv.detach(), packed.level_offsets), out.detach(),
        lse.detach(), dout_pre, g["fmap"], g["cache"], softcap=c["softcap"], dlse=dlse,
        position_mode="relative", relative_states=st.detach(), relative_proj=pj.detach())
    for got, want in ((grads[0], dq), (grads[1], dk), (grads[2], dv), (grads[5], dsinks)):
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(grads[3], torch.einsum("bnhr,dr->bnhd", dpos, pj.detach()),
                               rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(grads[4], torch.einsum("bnhd,bnhr->dr", st.detach(), dpos),
                               rtol=1e-5, atol=1e-5)


def test_gate_autograd_matches_torch():
    r = rng(3)
    out = t(r.standard_normal((2, 5, 4, 8)).astype(np.float32)).requires_grad_(True)
    x = t(r.standard_normal((2, 5, 12)).astype(np.float32)).requires_grad_(True)
    wg = t(r.standard_normal((32, 12)).astype(np.float32) / 4).requires_grad_(True)
    y = T.apply_output_gate(out, x, wg)
    want = torch.nn.functional.silu(x.matmul(wg.t())).reshape(2, 5, 4, 8) * out
    torch.testing.assert_close(y, want, rtol=1e-6, atol=1e-6)
    gy = torch.randn_like(y)
    g1 = torch.autograd.grad(y, (out, x, wg), gy)
    g2 = torch.autograd.grad(want, (out, x, wg), gy)
    for a, b in zip(g1, g2):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


def test_never_visible_nodes_get_zero_gradient():
    """Packed nodes no query sees get exactly zero dk/dv
    (test_reference.py:1575-1600)."""
    c = C.CASE_BY_NAME["bwd_none_four"]
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c)
    d = {k: t(v) for k, v in inp.items()}
    kl, vl, _ = T.build_dyadic_summaries(d["q"], d["k"], d["v"], len(g["fmap"]))
    packed = T.pack_levels(kl, vl)
    out, lse = T.multilevel_attention_forward(d["q"], packed, g["fmap"], g["cache"])
    _, dk, dv, _, _ = T.multilevel_attention_backward(d["q"], packed, out, lse, d["dout"],
                                                      g["fmap"], g["cache"])
    spec = T.range_spec.RangeSpec.from_fmap(g["fmap"], g["cache"], g["N"])
    off = spec.level_offsets()
    nv = []
    for lv in range(spec.num_levels):
        for kk in range(spec.level_len(lv)):
            if T.range_spec.node_query_bounds(spec, kk, lv) == (0, 0):
                nv.append(off[lv] + kk)
    assert nv, "geometry has no never-visible nodes"
    assert bool((dk[:, nv] == 0).all()) and bool((dv[:, nv] == 0).all())
