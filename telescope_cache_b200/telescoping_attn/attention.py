"""Phase-2 multilevel attention over the packed level-major K/V
(``reference.py:671-1071`` forward, ``:1222-1672`` backward).

The forward is one CUDA launch (tensor-core kernel for bf16/f16 at
Dk = Dv = 128, SIMT kernel otherwise); the backward is a Delta pass, a
Q-owned dQ pass and a KV-owned dK/dV pass.  RoPE rotates Q rows and packed K
once into rotated copies before the launch (the reference rounds rotated
operands to the input dtype the same way); the relative bias is formed in
the kernel from relative_states and relative_proj and is never materialised.

``multilevel_attention_forward`` is differentiable: its autograd backward is
``multilevel_attention_backward`` (with the lse gradient as the dlse seed).
"""

import ctypes
import math
import weakref
from typing import Dict, Optional

import torch

from .. import _lib
from .linear import linear
from ..range_spec import RangeSpec, native_schedule, visible_stats
from .packing import PackedKV
from .position import _rope_into, check_relative_bins, positional_args

_STATUS = {}


def device_status(device) -> torch.Tensor:
    """The int32 device status word the kernels OR error bits into."""
    key = torch.device(device).index
    t = _STATUS.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[key] = t
    return t


def read_device_status(device, reset=True) -> int:
    """Synchronise and read (and clear) the device status word."""
    t = device_status(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


def _impl_code(impl: Optional[str]) -> int:
    return {None: 0, "auto": 0, "simt": 1, "tensor": 2}[impl]


REL_PAD = 136  # zero bins on each side of the relative band (>= one 128-node tile + 8)


def _relative_band(st, pj, max_visible, dtype):
    """Bias logits rel[row, REL_PAD + d] = states[row] . proj[:, d] for every
    distance d a query can reach (< max_visible), in the kernels' element
    type, with REL_PAD zero columns on both sides -- the operand of the
    tensor-core relative path.  One tc_linear launch: states [rows, d_rel]
    times the padded table (as [width, d_rel] rows), fp32 accumulation,
    rounded once to the kernels' type."""
    d_rel, bins = pj.shape
    reach = min(bins, max_visible)
    width = (reach + 2 * REL_PAD + 7) // 8 * 8
    proj_pad = torch.zeros(d_rel, width, device=pj.device, dtype=pj.dtype)
    proj_pad[:, REL_PAD:REL_PAD + reach] = pj[:, :reach]
    rows = st.reshape(-1, d_rel)
    band = linear(rows, proj_pad.t().contiguous(), out_dtype=dtype)
    return band, width


# The relative band of a forward, kept for the backward of the same call:
# id(lse) -> (weak lse, weak states, weak proj, their versions and shapes,
# band, width).  An entry lives as long as the forward's lse output; it is
# reused only for the same states / proj objects, unmodified (version
# counters), so a backward with other or changed tensors recomputes the band.
_BANDS: Dict[int, tuple] = {}


def _band_key(states, proj, reach, dtype):
    return (states._version, tuple(states.shape), states.dtype, proj._version, tuple(proj.shape), proj.dtype,
            reach, dtype)


def _cached_band(lse, states, proj, reach, dtype):
    e = _BANDS.get(id(lse)) if lse is not None else None
    if e is None or e[0]() is not lse or e[1]() is not states or e[2]() is not proj:
        return None
    if e[3] != _band_key(states, proj, reach, dtype):
        return None
    return e[4], e[5]


def _keep_band(lse, states, proj, reach, dtype, band, width):
    k = id(lse)
    _BANDS[k] = (weakref.ref(lse, lambda _r, k=k: _BANDS.pop(k, None)), weakref.ref(states), weakref.ref(proj),
                 _band_key(states, proj, reach, dtype), band, width)


def _tensor_core_shape(dtype, Dk, Dv):
    return dtype in (torch.bfloat16, torch.float16) and Dk == 128 and Dv == 128


def _prepare(q, packed, fmap, cache_size, softcap, position_mode, rope_cos, rope_sin,
             relative_states, relative_proj, impl=None, band_of=None, block_m=16, block_n=32):
    """Shared validation + operand preparation of forward and backward.
    band_of: the forward's lse in a backward, whose relative band is reused
    when it was kept for the same, unmodified states and proj."""
    B, N, Hq, Dk = q.shape
    Hkv = packed.k.shape[2]
    Dv = packed.v.shape[-1]
    if Hq % Hkv != 0:
        raise ValueError(f"Hq={Hq} must be divisible by Hkv={Hkv}.")
    spec = RangeSpec.from_fmap(fmap, cache_size, N)
    if tuple(packed.level_offsets) != spec.level_offsets():
        raise ValueError(
            f"packed level_offsets {tuple(packed.level_offsets)} != spec {spec.level_offsets()}")
    bins = positional_args(position_mode, rope_cos, rope_sin, relative_states, relative_proj,
                           B=B, N=N, Hq=Hq, Dk=Dk, spec=spec, rope_positions=N)
    mn, mx, _ = visible_stats(spec)
    if position_mode == "relative":
        check_relative_bins(spec, bins, mx, block_m=block_m, block_n=block_n)
    if mn == 0:
        raise RuntimeError("Found query rows with no attended KV entries.")
    _lib.require_cuda(q, packed.k, packed.v)
    dtype = packed.v.dtype
    qc = q.to(dtype).contiguous()
    kc = packed.k.to(dtype).contiguous()
    vc = packed.v.contiguous()
    sched = native_schedule(spec)
    cos = sin = None
    if position_mode == "rope":
        cos = rope_cos.to(device=q.device, dtype=torch.float32).contiguous()
        sin = rope_sin.to(device=q.device, dtype=torch.float32).contiguous()
        qc = _rope_into(qc, torch.empty_like(qc), cos, sin, 0)
        kc = _rope_into(kc, torch.empty_like(kc), cos, sin, 1, sched=sched)
    st = pj = None
    rel_dt = 0
    if position_mode == "relative":
        rdt = torch.result_type(relative_states, relative_proj)
        if rdt not in (torch.float32, torch.bfloat16, torch.float16):
            rdt = torch.float32
        st = relative_states.to(device=q.device, dtype=rdt).contiguous()
        pj = relative_proj.to(device=q.device, dtype=rdt).contiguous()
        rel_dt = _lib.dtype_code(rdt)
    args = _lib.AttnArgs(
        B=B, N=N, Hq=Hq, Hkv=Hkv, Dk=Dk, Dv=Dv, dtype=_lib.dtype_code(dtype),
        has_softcap=0 if softcap is None else 1, softcap=0.0 if softcap is None else float(softcap),
        position_mode=_lib.POS[position_mode], q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(),
        rel_states=None if st is None else st.data_ptr(), rel_proj=None if pj is None else pj.data_ptr(),
        rel_dtype=rel_dt, d_rel=0 if st is None else st.shape[-1], rel_bins=bins,
        rope_cos=None if cos is None else cos.data_ptr(), rope_sin=None if sin is None else sin.data_ptr(),
        rope_npos=0 if cos is None else cos.shape[0],
        dev_status=device_status(q.device).data_ptr())
    band = None
    if position_mode == "relative" and impl != "simt" and _tensor_core_shape(dtype, Dk, Dv):
        hit = _cached_band(band_of, relative_states, relative_proj, mx, dtype)
        band, width = hit if hit is not None else _relative_band(st, pj, mx, dtype)
        args.rel_logits = band.data_ptr()
        args.rel_logits_stride = width
        args.rel_logits_pad = REL_PAD
    keep = (qc, kc, vc, cos, sin, st, pj, band)
    if band is not None:
        args._band = (mx, band, width)  # for _keep_band after the forward
    return args, sched, spec, keep, (B, N, Hq, Hkv, Dk, Dv, dtype)


def _forward(q, packed, fmap, cache_size, softcap, position_mode, rope_cos, rope_sin,
             relative_states, relative_proj, impl=None, block_m=16, block_n=32):
    args, sched, spec, keep, dims = _prepare(q, packed, fmap, cache_size, softcap, position_mode,
                                             rope_cos, rope_sin, relative_states, relative_proj,
                                             impl, block_m=block_m, block_n=block_n)
    B, N, Hq, Hkv, Dk, Dv, dtype = dims
    out = torch.empty(B, N, Hq, Dv, device=q.device, dtype=dtype)
    lse = torch.empty(B, N, Hq, device=q.device, dtype=torch.float32)
    args.out = out.data_ptr()
    args.lse = lse.data_ptr()
    args.impl = _impl_code(impl)
    _lib.launch("tc_attn_fwd", q.device, ctypes.byref(args), ctypes.byref(sched), _lib.stream_of(q))
    band = getattr(args, "_band", None)
    if band is not None:
        _keep_band(lse, relative_states, relative_proj, band[0], dims[-1], band[1], band[2])
    del keep
    return out, lse


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, pk, pv, relative_states, relative_proj, offsets, fmap, cache_size, softcap,
                position_mode, rope_cos, rope_sin, impl, blocks):
        packed = PackedKV(pk, pv, offsets)
        out, lse = _forward(q, packed, fmap, cache_size, softcap, position_mode, rope_cos, rope_sin,
                            relative_states, relative_proj, impl, *blocks)
        ctx.save_for_backward(q, pk, pv, out, lse, relative_states, relative_proj, rope_cos, rope_sin)
        ctx.cfg = (offsets, fmap, cache_size, softcap, position_mode, impl, blocks)
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, pk, pv, out, lse, st, pj, cos, sin = ctx.saved_tensors
        offsets, fmap, cache_size, softcap, position_mode, impl, blocks = ctx.cfg
        if dout is None:
            dout = torch.zeros_like(out)
        dq, dk, dv, dpos, _ = multilevel_attention_backward(
            q, PackedKV(pk, pv, offsets), out, lse, dout.to(out.dtype), fmap, cache_size, *blocks,
            softcap=softcap, dlse=dlse, position_mode=position_mode, rope_cos=cos, rope_sin=sin,
            relative_states=st, relative_proj=pj, impl=impl)
        dst = dpj = None
        if dpos is not None:
            if ctx.needs_input_grad[3]:
                dst = torch.einsum("bnhr,dr->bnhd", dpos, pj.float()).to(st.dtype)
            if ctx.needs_input_grad[4]:
                dpj = torch.einsum("bnhd,bnhr->dr", st.float(), dpos).to(pj.dtype)
        return (dq.to(q.dtype), dk.to(pk.dtype), dv.to(pv.dtype), dst, dpj,
                None, None, None, None, None, None, None, None, None)


def multilevel_attention_forward(
    q: torch.Tensor,
    packed: PackedKV,
    fmap: Dict[int, int],
    cache_size: int,
    block_m: int = 16,
    block_n: int = 32,
    softcap: float = 20.0,
    *,
    position_mode: str = "none",
    rope_cos: Optional[torch.Tensor] = None,
    rope_sin: Optional[torch.Tensor] = None,
    relative_states: Optional[torch.Tensor] = None,
    relative_proj: Optional[torch.Tensor] = None,
    impl: Optional[str] = None,
):
    """(out [B, N, Hq, Dv] in V's dtype, lse [B, N, Hq] fp32 natural-log,
    pre-sink) with S = c tanh(X / c) (or X when softcap is None),
    X = q.k / sqrt(Dk) [+ relative bias], softmax over exactly each query's
    multiresolution set (reference.py:771-1071).  Tiling is the kernel's
    choice; block_m / block_n only name the query blocks and node tiles at
    which a too-small relative table is reported, as the reference's loop
    does.  ``impl`` ('simt' | 'tensor' | None) pins a kernel family for
    testing."""
    grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (q, packed.k, packed.v, relative_states, relative_proj))
    if not grad:
        return _forward(q, packed, fmap, cache_size, softcap, position_mode, rope_cos, rope_sin,
                        relative_states, relative_proj, impl, block_m, block_n)
    return _Attention.apply(q, packed.k, packed.v, relative_states, relative_proj,
                            tuple(packed.level_offsets), fmap, cache_size, softcap, position_mode,
                            rope_cos, rope_sin, impl, (block_m, block_n))


@torch.no_grad()
def multilevel_attention_backward(
    q: torch.Tensor,
    packed: PackedKV,
    out: torch.Tensor,
    lse: torch.Tensor,
    dout: torch.Tensor,
    fmap: Dict[int, int],
    cache_size: int,
    block_m: int = 16,
    block_n: int = 32,
    softcap: float = 20.0,
    *,
    dlse: Optional[torch.Tensor] = None,
    position_mode: str = "none",
    rope_cos: Optional[torch.Tensor] = None,
    rope_sin: Optional[torch.Tensor] = None,
    relative_states: Optional[torch.Tensor] = None,
    relative_proj: Optional[torch.Tensor] = None,
    impl: Optional[str] = None,
):
    """Explicit Phase-2 backward at the packed boundary
    (reference.py:1308-1672): P = exp(S - lse) from the saved lse,
    Delta = rowsum(dO O) - dlse, dS = P (dP - Delta), dX = dS softcap',
    dQ = scale dX K, dK = scale dX^T Q, dV = P^T dO; RoPE gradients are
    rotated back by R(-p) in fp32.  Returns the fixed 5-tuple
    (dq, dk_packed, dv_packed, dposition, stats); dposition is drel_logits
    [B, N, Hq, max_relative_bins] fp32 in relative mode, else None.
    block_m / block_n only name where a too-small relative table is
    reported (the reference's query blocks and node tiles)."""
    if position_mode not in ("none", "rope", "relative"):
        raise ValueError(
            f"position_mode must be 'none', 'rope' or 'relative', got {position_mode!r}")
    B, N, Hq, Dk = q.shape
    Hkv = packed.k.shape[2]
    Dv = packed.v.shape[-1]
    if Hq % Hkv != 0:
        raise ValueError(f"Hq={Hq} must be divisible by Hkv={Hkv}.")
    if tuple(out.shape) != (B, N, Hq, Dv):
        raise ValueError(f"out shape {tuple(out.shape)} != {(B, N, Hq, Dv)}")
    if tuple(dout.shape) != (B, N, Hq, Dv):
        raise ValueError(f"dout shape {tuple(dout.shape)} != {(B, N, Hq, Dv)}")
    if tuple(lse.shape) != (B, N, Hq) or lse.dtype != torch.float32:
        raise ValueError("lse must be float32 [B, N, Hq]")
    spec = RangeSpec.from_fmap(fmap, cache_size, N)
    if tuple(packed.level_offsets) != spec.level_offsets():
        raise ValueError("packed level_offsets do not match the schedule")
    positional_args(position_mode, rope_cos, rope_sin, relative_states, relative_proj,
                    B=B, N=N, Hq=Hq, Dk=Dk, spec=spec, rope_positions=N)
    if dlse is not None:
        if tuple(dlse.shape) != (B, N, Hq):
            raise ValueError(f"dlse shape {tuple(dlse.shape)} != {(B, N, Hq)}")
        if not dlse.dtype.is_floating_point:
            raise ValueError("dlse must have floating dtype")
    args, sched, spec, keep, dims = _prepare(q, packed, fmap, cache_size, softcap, position_mode,
                                             rope_cos, rope_sin, relative_states, relative_proj,
                                             impl, band_of=lse, block_m=block_m, block_n=block_n)
    dtype = dims[-1]
    _lib.require_cuda(out, lse, dout, dlse)
    oc = out.to(dtype).contiguous()
    gc = dout.to(dtype).contiguous()
    lc = lse.contiguous()
    dl = None if dlse is None else dlse.float().contiguous()
    delta = torch.empty(B, N, Hq, device=q.device, dtype=torch.float32)
    dq = torch.empty(B, N, Hq, Dk, device=q.device, dtype=dtype)
    dk = torch.empty(packed.k.shape, device=q.device, dtype=dtype)
    dv = torch.empty(packed.v.shape, device=q.device, dtype=dtype)
    drel = None
    if position_mode == "relative":
        # the tensor-core path writes every element (zeros past each row's
        # visible count); the SIMT path writes visible bins only
        alloc = torch.empty if args.rel_logits else torch.zeros
        drel = alloc(B, N, Hq, args.rel_bins, device=q.device, dtype=torch.float32)
    args.lse = lc.data_ptr()
    args.o = oc.data_ptr()
    args.dout = gc.data_ptr()
    args.dlse = None if dl is None else dl.data_ptr()
    args.delta = delta.data_ptr()
    args.dq = dq.data_ptr()
    args.dk = dk.data_ptr()
    args.dv = dv.data_ptr()
    args.drel = None if drel is None else drel.data_ptr()
    args.impl = _impl_code(impl)
    _lib.launch("tc_attn_bwd", q.device, ctypes.byref(args), ctypes.byref(sched), _lib.stream_of(q))
    del keep
    stats = {"softcap_used": softcap is not None, "kernel": "cuda"}
    return (dq.to(q.dtype), dk.to(packed.k.dtype), dv.to(packed.v.dtype), drel, stats)


__all__ = ["multilevel_attention_forward", "multilevel_attention_backward"]
