"""The relative bias band of a forward is reused by the backward of the same
call (same lse, same unmodified relative_states / relative_proj objects) and
recomputed otherwise; results agree bit for bit either way, and the kept band
goes away with the forward's lse."""

import gc

import pytest
import torch

import telescope_cache_b200 as T
from telescope_cache_b200.telescoping_attn import attention as A

pytestmark = pytest.mark.gpu


def _case(dev):
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    B, N, H, D, L, W = 1, 1024, 2, 128, 4, 64
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    bf = torch.bfloat16
    q, k, v, dout = (torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf) for _ in range(4))
    states = (0.02 * torch.randn(B, N, H, 6, generator=g, device=dev)).to(bf)
    proj = (0.02 * torch.randn(6, cache, generator=g, device=dev)).to(bf)
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1)
    return q, T.pack_levels(kl, vl), dout, states, proj, fmap, cache


def test_backward_reuses_the_forward_band():
    dev = torch.device("cuda")
    q, packed, dout, states, proj, fmap, cache = _case(dev)
    pos = dict(position_mode="relative", relative_states=states, relative_proj=proj)
    out, lse = T.multilevel_attention_forward(q, packed, fmap, cache, softcap=30.0, **pos)
    assert id(lse) in A._BANDS
    mx = A.visible_stats(A.RangeSpec.from_fmap(fmap, cache, q.shape[1]))[1]
    assert A._cached_band(lse, states, proj, mx, torch.bfloat16) is not None
    reused = T.multilevel_attention_backward(q, packed, out, lse, dout, fmap, cache, softcap=30.0, **pos)
    # a copy of lse has no kept band: the backward recomputes it
    lse2 = lse.clone()
    assert A._cached_band(lse2, states, proj, mx, torch.bfloat16) is None
    fresh = T.multilevel_attention_backward(q, packed, out, lse2, dout, fmap, cache, softcap=30.0, **pos)
    for a, b in zip(reused[:4], fresh[:4]):
        assert torch.equal(a, b)
    # an in-place change of the states (even to the same values) invalidates it
    states.mul_(1.0)
    assert A._cached_band(lse, states, proj, mx, torch.bfloat16) is None
    again = T.multilevel_attention_backward(q, packed, out, lse, dout, fmap, cache, softcap=30.0, **pos)
    for a, b in zip(again[:4], fresh[:4]):
        assert torch.equal(a, b)
    # other states objects never reuse it
    other = states.clone()
    assert A._cached_band(lse, other, proj, mx, torch.bfloat16) is None
    # the kept band lives as long as the forward's lse
    key = id(lse)
    del lse, reused, again
    gc.collect()
    assert key not in A._BANDS
