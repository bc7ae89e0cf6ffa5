"""Bit-for-bit repeatability of the deterministic kernels: the builder and
its VJP (conv, qk weights, eight levels), the tensor-core attention forward
and backward with the relative band and the drel tail write-out over many
tiles, the split-K projection and the decode step (split entries, conv,
rope, sink, gate).  None of them accumulates with atomics or depends on
scheduling order, so two runs on the same inputs must give the same bits;
a difference points at a race (a shared-memory or mbarrier hazard)."""

import pytest
import torch

import telescope_cache_b200 as T
from oracle import schedule as S
from telescope_cache_b200.telescoping_attn.attention import multilevel_attention_forward
from telescope_cache_b200.telescoping_attn.linear import linear
from telescope_cache_b200.telescoping_attn.packing import PackedKV

pytestmark = pytest.mark.gpu


def _same(a, b, what):
    for i, (x, y) in enumerate(zip(a, b)):
        assert torch.equal(x, y), f"{what}: output {i} differs between two runs"


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def test_builder_and_vjp_repeat():
    torch.cuda.set_device(0)
    g = _gen(61)
    B, N, Hq, Hkv, D, L, K = 2, 1500, 4, 2, 128, 7, 4
    q = torch.randn(B, N, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, N, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, N, Hkv, D, generator=g, device="cuda").bfloat16()
    kcw = (torch.randn(Hkv * D, K, generator=g, device="cuda") / K).bfloat16()
    vcw = (torch.randn(Hkv * D, K, generator=g, device="cuda") / K).bfloat16()

    def run():
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v, kcw, vcw)]
        kl, vl, wl = T.build_dyadic_summaries(leaves[0], leaves[1], leaves[2], L, k_conv_weight=leaves[3],
                                              v_conv_weight=leaves[4])
        packed = T.pack_levels(kl, vl)
        gk = torch.ones_like(packed.k)
        loss = (packed.k.float() * gk.float()).sum() + packed.v.float().square().sum() + \
            sum(w.float().sum() for w in wl)
        return [packed.k.detach(), packed.v.detach()] + list(torch.autograd.grad(loss, leaves))

    _same(run(), run(), "builder / VJP")


def test_tensor_core_attention_relative_repeats():
    torch.cuda.set_device(0)
    g = _gen(62)
    B, N, Hq, Hkv, D = 1, 4096, 4, 2, 128
    fmap, cache, bins = {l: 256 * l for l in range(1, 5)}, 1280, 1536
    L = len(fmap)
    offs = tuple(S.level_offsets(N, L + 1))
    q = torch.randn(B, N, Hq, D, generator=g, device="cuda").bfloat16()
    kp = torch.randn(B, offs[-1], Hkv, D, generator=g, device="cuda").bfloat16()
    vp = torch.randn(B, offs[-1], Hkv, D, generator=g, device="cuda").bfloat16()
    st = (torch.randn(B, N, Hq, 16, generator=g, device="cuda") * 0.5).bfloat16()
    pj = (torch.randn(16, bins, generator=g, device="cuda") * 0.5).bfloat16()
    dout = torch.randn(B, N, Hq, D, generator=g, device="cuda").bfloat16()
    dlse = torch.randn(B, N, Hq, generator=g, device="cuda")

    def run():
        out, lse = multilevel_attention_forward(q, PackedKV(kp, vp, offs), fmap, cache, softcap=20.0,
                                                position_mode="relative", relative_states=st, relative_proj=pj)
        dq, dk, dv, drel, _ = T.multilevel_attention_backward(
            q, PackedKV(kp, vp, offs), out, lse, dout, fmap, cache, softcap=20.0, dlse=dlse,
            position_mode="relative", relative_states=st, relative_proj=pj)
        return [out, lse, dq, dk, dv, drel]

    _same(run(), run(), "relative attention")


def test_split_k_projection_repeats():
    torch.cuda.set_device(0)
    g = _gen(63)
    x = torch.randn(64, 2048, generator=g, device="cuda").bfloat16()
    w = (torch.randn(2048, 2048, generator=g, device="cuda") / 45).bfloat16()
    _same([linear(x, w), linear(x, w, out_dtype=torch.float32)],
          [linear(x, w), linear(x, w, out_dtype=torch.float32)], "split-K projection")


def test_decode_repeats():
    torch.cuda.set_device(0)
    g = _gen(64)
    B, N, Hq, Hkv, D, K, steps = 2, 900, 2, 2, 128, 4, 6
    fmap, cache = {1: 128, 2: 256, 3: 384, 4: 512}, 640  # entries split over CTAs
    L = len(fmap)
    E = 64
    x = torch.randn(B, N + steps, E, generator=g, device="cuda").bfloat16()
    q = torch.randn(B, N + steps, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, N + steps, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, N + steps, Hkv, D, generator=g, device="cuda").bfloat16()
    kcw = (torch.randn(Hkv * D, K, generator=g, device="cuda") / K).bfloat16()
    vcw = (torch.randn(Hkv * D, K, generator=g, device="cuda") / K).bfloat16()
    sinks = torch.randn(Hq, generator=g, device="cuda")
    gate = (torch.randn(Hq * D, E, generator=g, device="cuda") / 8).bfloat16()
    cos, sin = T.rope_tables(N + steps + 1, D, device="cuda")

    def run():
        with torch.no_grad():
            kl, vl, wl = T.build_dyadic_summaries(q[:, :N], k[:, :N], v[:, :N], L, k_conv_weight=kcw,
                                                  v_conv_weight=vcw)
            st = T.init_decode_state(kl, vl, wl, fmap, cache, k_pre_conv=k[:, :N], v_pre_conv=v[:, :N],
                                     conv_kernel_size=K)
            outs = []
            for t in range(N, N + steps):
                sl = slice(t, t + 1)
                out, lse = T.decode_step(x[:, sl], q[:, sl], k[:, sl], v[:, sl], st, k_conv_weight=kcw,
                                         v_conv_weight=vcw, position_mode="rope", rope_cos=cos, rope_sin=sin,
                                         sinks=sinks, gate_weight=gate)
                outs += [out, lse]
            return outs + [st.k, st.v, st.w, st.conv_k, st.conv_v]

    _same(run(), run(), "decode")
