"""The no-allocation backward entry point, tc_attn_bwd_noalloc.

It serves callers that cannot call cudaMalloc themselves (their framework or
serving engine already reserved the device memory in its own pool, or their
host runtime only hands out buffers it owns): it takes the same inputs and
outputs as tc_attn_bwd, but keeps the one scratch buffer tc_attn_bwd needs
(the per-row Delta) in a fixed array inside the library.

This test calls it through the C ABI twice in a row and checks both results
against the allocating entry point (reached through the public API), with the
tolerances the other GPU tests use.  The file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

import cases as C
import telescope_cache_b200 as T
from telescope_cache_b200 import _lib
from telescope_cache_b200.telescoping_attn import attention as A

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-4   # fp32 gradient tolerance of the reference suite
BF16_REL = 2e-2   # bf16: within 2e-2 relative of the reference


def _close(got, want, dtype):
    got, want = got.double().cpu().numpy(), want.double().cpu().numpy()
    if dtype == "bf16":
        scale = np.abs(want).max()
        assert (np.abs(got - want) <= BF16_REL * (np.abs(want) + scale)).all()
    else:
        np.testing.assert_allclose(got, want, rtol=GRAD_TOL, atol=GRAD_TOL)


def _inputs(name):
    c = C.CASE_BY_NAME[name]
    g = C.GEOS[c["geo"]]
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    d = {k: torch.from_numpy(v).to("cuda", dt) for k, v in C.make_inputs(c).items()}
    kl, vl, _ = T.build_dyadic_summaries(d["q"], d["k"], d["v"], len(g["fmap"]))
    packed = T.pack_levels(kl, vl)
    pos = {}
    if c["position"] == "rope":
        cos, sin = T.rope_tables(g["N"], g["Dk"], device="cuda")
        pos = dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    elif c["position"] == "relative":
        pos = dict(position_mode="relative", relative_states=d["states"],
                   relative_proj=d["rel_proj"])
    out, lse = T.multilevel_attention_forward(d["q"], packed, g["fmap"], g["cache"],
                                              softcap=c["softcap"], **pos)
    dout, dlse = d["dout"], None
    if c["sink"]:
        dout, dlse, _ = T.attention_sink_backward(out, lse, d["sinks"], d["dout"])
    return c, g, d, packed, pos, out, lse, dout, dlse


def _noalloc_call(c, g, d, packed, pos, out, lse, dout, dlse):
    """One tc_attn_bwd_noalloc call with caller-owned inputs and outputs."""
    args, sched, _, keep, dims = A._prepare(
        d["q"], packed, g["fmap"], g["cache"], c["softcap"], pos.get("position_mode", "none"),
        pos.get("rope_cos"), pos.get("rope_sin"), pos.get("relative_states"),
        pos.get("relative_proj"))
    B, N, Hq, Hkv, Dk, Dv, dtype = dims
    o, g_, l = out.contiguous(), dout.to(dtype).contiguous(), lse.contiguous()
    dl = None if dlse is None else dlse.float().contiguous()
    dq = torch.empty(B, N, Hq, Dk, device="cuda", dtype=dtype)
    dk = torch.empty(packed.k.shape, device="cuda", dtype=dtype)
    dv = torch.empty(packed.v.shape, device="cuda", dtype=dtype)
    drel = None
    if args.position_mode == _lib.POS["relative"]:
        drel = torch.zeros(B, N, Hq, args.rel_bins, device="cuda", dtype=torch.float32)
    args.lse, args.o, args.dout = l.data_ptr(), o.data_ptr(), g_.data_ptr()
    args.dlse = None if dl is None else dl.data_ptr()
    args.delta = None
    args.dq, args.dk, args.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    args.drel = None if drel is None else drel.data_ptr()
    rc = _lib.lib().tc_attn_bwd_noalloc(ctypes.byref(args), ctypes.byref(sched),
                                        _lib.stream_of(d["q"]))
    assert rc == _lib.TC_OK, rc
    torch.cuda.synchronize()
    del keep
    return dq, dk, dv, drel


@pytest.mark.parametrize("name", ["bwd_rel_sink_tiny", "bwd_rope_sink_tiny", "bwd_none_gqa3",
                                  "bwd_rel_sink_d128_bf16", "bwd_rope_sink_d128_bf16"])
def test_noalloc_backward_matches_allocating_entry_point(name):
    c, g, d, packed, pos, out, lse, dout, dlse = _inputs(name)
    want = T.multilevel_attention_backward(d["q"], packed, out, lse, dout, g["fmap"], g["cache"],
                                           softcap=c["softcap"], dlse=dlse, **pos)
    for _ in range(2):  # two calls in a row share (and fully rewrite) the scratch
        got = _noalloc_call(c, g, d, packed, pos, out, lse, dout, dlse)
        for gt, wt in zip(got, want[:4]):
            if wt is None:
                assert gt is None
            else:
                # the rope wrapper rotates dq/dk back in the same kernels
                _close(gt.to(wt.dtype), wt, c["dtype"])


def test_noalloc_rejects_sizes_beyond_its_scratch():
    buf = torch.zeros(16, device="cuda")
    spec = T.range_spec.RangeSpec.from_fmap({1: 2, 2: 3}, 6, 1 << 16)
    sched = T.range_spec.native_schedule(spec)
    p = buf.data_ptr()
    args = _lib.AttnArgs(B=8, N=1 << 16, Hq=16, Hkv=16, Dk=8, Dv=8, dtype=_lib.TC_F32, q=p, k=p,
                         v=p, out=p, lse=p, o=p, dout=p, dq=p, dk=p, dv=p)
    rc = _lib.lib().tc_attn_bwd_noalloc(ctypes.byref(args), ctypes.byref(sched),
                                        _lib.stream_of(buf))
    assert rc == 5  # TC_ERR_SCRATCH_LIMIT: 8 * 65536 * 16 rows > 2^22
