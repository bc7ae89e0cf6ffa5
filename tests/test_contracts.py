"""The reference suite's API contracts, replayed on this build.

- Error matrix (test_reference.py:1888-2079): every case raises the same
  exception type with the same message as the reference; the expected
  outcomes were recorded by running the reference itself
  (golden/make_contract_golden.py -> golden/contract_errors.json).
- No mutation (test_reference.py:1797-1816): the default forward equals the
  explicit position_mode="none" bit for bit, and no position mode mutates the
  packed buffers.
- Never-visible nodes (test_reference.py:1575-1596): packed nodes no query
  sees get exactly zero dK / dV, from the explicit backward and from autograd,
  on the reference's geometries (SIMT path) and on a bf16 Dk = Dv = 128
  schedule with eviction (tensor-core path).
"""

import json
import os
import types

import pytest
import torch

import contract_cases as CC
from telescope_cache_b200 import reference as R
from telescope_cache_b200.range_spec import EMPTY, RangeSpec, node_query_bounds
from telescope_cache_b200.telescoping_attn.position import check_relative_bins

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = {d["label"]: d for d in json.load(open(os.path.join(HERE, "golden", "contract_errors.json")))}


def product_api():
    api = types.SimpleNamespace(**{n: getattr(R, n) for n in R.__all__})
    api.RangeSpec = RangeSpec
    return api


def test_golden_records_every_case():
    """The recorded reference outcomes cover exactly the case list, and the
    reference raised ValueError in every one (as its suite asserts)."""
    labels = [lab for lab, _ in CC.error_cases(types.SimpleNamespace(**_shape_only_api()), "cpu")]
    assert labels == list(GOLDEN)
    assert all(d["type"] == "ValueError" for d in GOLDEN.values())


def _shape_only_api():
    """Enough of an API to list the cases on CPU (the thunks are not run)."""
    api = {n: getattr(R, n) for n in R.__all__}
    api["RangeSpec"] = RangeSpec

    def bds(q, k, v, L, **kw):
        B, N = k.shape[:2]
        return ([torch.zeros(B, N >> l, k.shape[2], k.shape[3]) for l in range(L + 1)],
                [torch.zeros(B, N >> l, v.shape[2], v.shape[3]) for l in range(L + 1)],
                [torch.zeros(B, N >> l, k.shape[2], 1) for l in range(L + 1)])
    api["build_dyadic_summaries"] = bds
    return api


def test_bin_overflow_messages_host():
    """The too-small relative table is reported at the reference's tile: the
    forward / backward query blocks of block_m = 3 with block_n = 2 tiles,
    and the decode query 7 over its exact ranges (host replay of the
    reference loop, no GPU)."""
    g = CC.TINY
    spec = RangeSpec.from_fmap(g["fmap"], g["cache"], g["N"])
    with pytest.raises(ValueError) as e:
        check_relative_bins(spec, 2, block_m=3, block_n=2)
    assert str(e.value) == GOLDEN["table too small"]["message"]
    assert str(e.value) == GOLDEN["backward table too small"]["message"]
    dspec = RangeSpec.from_fmap(g["fmap"], g["cache"], 8)
    with pytest.raises(ValueError) as e:
        check_relative_bins(dspec, 2, block_n=32, query=7)
    assert str(e.value) == GOLDEN["decode table too small"]["message"]
    check_relative_bins(spec, g["cache"], block_m=3, block_n=2)  # cache_size bins always suffice


@pytest.mark.gpu
def test_error_matrix_matches_reference():
    torch.cuda.set_device(0)
    mismatches = []
    for label, fn in CC.error_cases(product_api(), "cuda"):
        etype, msg = CC.run_case(fn)
        want = GOLDEN[label]
        if (etype, msg) != (want["type"], want["message"]):
            mismatches.append(f"{label}: got {etype}: {msg!r}; reference {want['type']}: {want['message']!r}")
    assert not mismatches, "\n".join(mismatches)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,geo", [(torch.float32, "tiny"), (torch.bfloat16, "d128")])
def test_no_mutation_and_default_none_bitwise(dtype, geo):
    torch.cuda.set_device(0)
    dev = "cuda"
    if geo == "tiny":
        g = dict(CC.TINY)
    else:
        g = dict(B=1, N=512, Hq=2, Hkv=2, Dk=128, Dv=128, fmap={1: 64, 2: 128}, cache=192)
    B, N, Hq, Hkv, Dk, Dv = (g[s] for s in ("B", "N", "Hq", "Hkv", "Dk", "Dv"))
    L = len(g["fmap"])
    torch.manual_seed(455)
    q = torch.randn(B, N, Hq, Dk, device=dev).to(dtype)
    k = torch.randn(B, N, Hkv, Dk, device=dev).to(dtype)
    v = torch.randn(B, N, Hkv, Dv, device=dev).to(dtype)
    kl, vl, _ = R.build_dyadic_summaries(q, k, v, L)
    packed = R.pack_levels(kl, vl)

    def fwd(**kw):
        return R.multilevel_attention_forward(q, packed, g["fmap"], g["cache"], **kw)

    out_a, lse_a = fwd()
    out_b, lse_b = fwd(position_mode="none")
    assert torch.equal(out_a, out_b) and torch.equal(lse_a, lse_b)
    k_snap, v_snap, q_snap = packed.k.clone(), packed.v.clone(), q.clone()
    cos, sin = R.rope_tables(N, Dk, device=dev)
    states = torch.randn(B, N, Hq, CC.DREL, device=dev)
    proj = torch.randn(CC.DREL, g["cache"], device=dev)
    for kw in (dict(position_mode="none"), dict(position_mode="rope", rope_cos=cos, rope_sin=sin),
               dict(position_mode="relative", relative_states=states, relative_proj=proj)):
        out, lse = fwd(**kw)
        R.multilevel_attention_backward(q, packed, out, lse, torch.ones_like(out), g["fmap"], g["cache"], **kw)
        assert torch.equal(packed.k, k_snap) and torch.equal(packed.v, v_snap), kw["position_mode"]
        assert torch.equal(q, q_snap), kw["position_mode"]


def _never_visible(spec):
    nv = torch.zeros(spec.total_len, dtype=torch.bool)
    off = spec.level_offsets()
    for lv in range(spec.num_levels):
        for kk in range(spec.level_len(lv)):
            if node_query_bounds(spec, kk, lv) == EMPTY:
                nv[off[lv] + kk] = True
    return nv


NV_GEOS = {
    "evict": dict(B=1, N=64, Hq=4, Hkv=2, Dk=8, Dv=16, fmap={1: 2, 2: 3}, cache=6, dtype=torch.float32),
    "four_levels": dict(B=1, N=96, Hq=8, Hkv=4, Dk=16, Dv=16, fmap={1: 4, 2: 6, 3: 8}, cache=12,
                        dtype=torch.float32),
    # tensor-core path: bf16, Dk = Dv = 128, a schedule that evicts coarse nodes
    "d128_evict": dict(B=1, N=1024, Hq=2, Hkv=2, Dk=128, Dv=128, fmap={1: 64, 2: 96, 3: 128}, cache=160,
                       dtype=torch.bfloat16),
}


@pytest.mark.gpu
@pytest.mark.parametrize("geo,seed", [("evict", 340), ("four_levels", 344), ("d128_evict", 346)])
def test_never_visible_nodes_get_zero_gradient(geo, seed):
    torch.cuda.set_device(0)
    dev = "cuda"
    g = NV_GEOS[geo]
    B, N, Hq, Hkv, Dk, Dv = (g[s] for s in ("B", "N", "Hq", "Hkv", "Dk", "Dv"))
    spec = RangeSpec.from_fmap(g["fmap"], g["cache"], N)
    nv = _never_visible(spec).to(dev)
    assert nv.any(), "the geometry must have never-visible nodes"
    torch.manual_seed(seed)
    q = torch.randn(B, N, Hq, Dk, device=dev).to(g["dtype"])
    k = torch.randn(B, N, Hkv, Dk, device=dev).to(g["dtype"])
    v = torch.randn(B, N, Hkv, Dv, device=dev).to(g["dtype"])
    with torch.no_grad():
        kl, vl, _ = R.build_dyadic_summaries(q, k, v, spec.num_levels - 1)
        packed = R.pack_levels(kl, vl)
    q_leaf = q.detach().clone().requires_grad_(True)
    k_leaf = packed.k.detach().clone().requires_grad_(True)
    v_leaf = packed.v.detach().clone().requires_grad_(True)
    pl = R.PackedKV(k_leaf, v_leaf, packed.level_offsets)
    out, lse = R.multilevel_attention_forward(q_leaf, pl, g["fmap"], g["cache"], softcap=20.0)
    dout = torch.randn_like(out)
    dq_a, dk_a, dv_a = torch.autograd.grad(out, (q_leaf, k_leaf, v_leaf), dout)
    _, dk_p, dv_p, _, _ = R.multilevel_attention_backward(
        q, packed, out.detach(), lse.detach(), dout, g["fmap"], g["cache"], softcap=20.0)
    for name, t in (("dk_p", dk_p), ("dv_p", dv_p), ("dk_auto", dk_a), ("dv_auto", dv_a)):
        assert bool((t[:, nv] == 0).all()), f"{geo}/{name}: nonzero gradient on never-visible nodes"
        assert bool((t[:, ~nv] != 0).any()), f"{geo}/{name}: no gradient at all"
