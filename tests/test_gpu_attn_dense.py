"""Autograd of multilevel_attention_forward (out and lse, the sink's dlse
seam included) against torch autograd of a dense fp32 restatement of
reference.py:771-1071 -- softmax over exactly each query's visible set
(the CPU oracle's schedule), softcap, RoPE at summary positions, relative
bias states . proj at the bin distance -- on geometries whose node tiles'
query hulls span several query blocks (the backward's node-owned pass then
walks more than one block per tile).  Gradients of q, packed k / v,
relative_states and relative_proj.  Tolerance: fp32 normwise 1e-5; bf16
normwise 1e-2 (measured on B200: at most 7e-7 and 3.6e-3, the bf16 rounding
floor), tighter than the 2e-2 bar so that an error of a few percent in one
pass cannot hide under it.  The product is also run twice and must repeat
bit for bit (no pass accumulates with atomics, so a difference means a
race)."""

import math

import pytest
import torch

from oracle import schedule as S
from telescope_cache_b200.telescoping_attn.attention import multilevel_attention_forward
from telescope_cache_b200.telescoping_attn.packing import PackedKV
from telescope_cache_b200.telescoping_attn.position import rope_tables
from test_gpu_fms_attention import _close, _rot, _visible

pytestmark = pytest.mark.gpu


def _dense(q, kp, vp, st, pj, N, fmap, cache, softcap, mode, cos=None, sin=None):
    B, _, H, Dk = q.shape
    E = H // kp.shape[2]
    idx, dist, ok, kpos, _ = _visible(N, fmap, cache)
    dev = q.device
    idx, dist, ok, kpos = idx.to(dev), dist.to(dev), ok.to(dev), kpos.to(dev)
    if mode == "rope":
        q = _rot(q, torch.arange(N, device=dev)[None, :, None], cos, sin)
        kp = _rot(kp, kpos[None, :, None], cos, sin)
    Kg = kp[:, idx].repeat_interleave(E, dim=3)
    Vg = vp[:, idx].repeat_interleave(E, dim=3)
    X = torch.einsum("bthd,btmhd->bthm", q, Kg) / math.sqrt(Dk)
    if mode == "relative":
        X = X + torch.gather(st @ pj, 3, dist[None, :, None, :].expand(B, N, H, -1))
    Sx = softcap * torch.tanh(X / softcap) if softcap is not None else X
    Sx = Sx.masked_fill(~ok[None, :, None, :], float("-inf"))
    lse = torch.logsumexp(Sx, -1)
    return torch.einsum("bthm,btmhd->bthd", torch.exp(Sx - lse.unsqueeze(-1)), Vg), lse


GEOS = [
    # fp32 (SIMT kernels): four levels, cache 12, GQA 2 and 3
    dict(dtype=torch.float32, B=2, N=96, H=4, Hkv=2, D=16, fmap={1: 4, 2: 6, 3: 8}, cache=12, bins=12),
    dict(dtype=torch.float32, B=1, N=200, H=6, Hkv=2, D=32, fmap={1: 8, 2: 16, 3: 24}, cache=32, bins=40),
    # bf16 head dim 128 (tensor-core kernels)
    dict(dtype=torch.bfloat16, B=1, N=512, H=4, Hkv=2, D=128, fmap={1: 64, 2: 128, 3: 192}, cache=256,
         bins=256),
]


@pytest.mark.parametrize("gi", range(len(GEOS)))
@pytest.mark.parametrize("mode", ["none", "rope", "relative"])
@pytest.mark.parametrize("softcap", [20.0, None])
def test_attention_autograd_matches_dense_restatement(gi, mode, softcap):
    c = GEOS[gi]
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(500 + 10 * gi + (mode == "rope") + 2 * (mode == "relative") + 5 * (softcap is None))
    B, N, H, Hkv, D, dt = c["B"], c["N"], c["H"], c["Hkv"], c["D"], c["dtype"]
    L = len(c["fmap"])
    offs = tuple(S.level_offsets(N, L + 1))
    total = offs[-1]

    def rnd(*shape, s=1.0):
        return (torch.randn(*shape, generator=g, device="cuda") * s).to(dt)

    q, kp, vp = rnd(B, N, H, D), rnd(B, total, Hkv, D), rnd(B, total, Hkv, D)
    st, pj = rnd(B, N, H, 16, s=0.5), rnd(16, c["bins"], s=0.5)
    dout, dlse = rnd(B, N, H, D), torch.randn(B, N, H, generator=g, device="cuda")
    kw, cos, sin = {}, None, None
    if mode == "relative":
        kw = dict(relative_states=st, relative_proj=pj)
    elif mode == "rope":
        cos, sin = rope_tables(N, D, device="cuda")
        kw = dict(rope_cos=cos, rope_sin=sin)

    def product():
        leaves = [t.clone().requires_grad_(True) for t in (q, kp, vp)]
        rel = [t.clone().requires_grad_(True) for t in (st, pj)] if mode == "relative" else []
        kwr = dict(relative_states=rel[0], relative_proj=rel[1]) if rel else kw
        out, lse = multilevel_attention_forward(leaves[0], PackedKV(leaves[1], leaves[2], offs), c["fmap"],
                                                c["cache"], softcap=softcap, position_mode=mode, **kwr)
        grads = torch.autograd.grad((out.float() * dout.float()).sum() + (lse * dlse).sum(), leaves + rel)
        return out, lse, grads

    out, lse, got = product()
    out_b, lse_b, got_b = product()
    assert torch.equal(out, out_b) and torch.equal(lse, lse_b)
    assert all(torch.equal(a, b_) for a, b_ in zip(got, got_b)), "the backward does not repeat bit for bit"
    ref = [t.float().clone().requires_grad_(True) for t in (q, kp, vp, st, pj)]
    o2, l2 = _dense(ref[0], ref[1], ref[2], ref[3], ref[4], N, c["fmap"], c["cache"], softcap, mode, cos, sin)
    want = torch.autograd.grad((o2 * dout.float()).sum() + (l2 * dlse).sum(),
                               ref[:3] + (ref[3:] if mode == "relative" else []))
    tol = 1e-5 if dt == torch.float32 else 1e-2
    _close(out, o2, tol, "out")
    _close(lse, l2, tol, "lse")
    for n, a, b_ in zip(["dq", "dk_packed", "dv_packed", "drelative_states", "drelative_proj"], got, want):
        _close(a, b_, tol, n)
