"""Decode-time attention and the full one-token block
(``reference.py:2093-2317``): ``multilevel_attention_decode`` reads the ring
cache for the newest query, ``decode_step`` advances the cache and attends in
one fused CUDA launch, with the sink and gate applied in its epilogue."""

from typing import Optional, Tuple

import torch

from .. import _lib
from .linear import linear
from .decode_state import (DecodeState, _check_tick, _decode_launch, _ensure_rotated_ring, _rot_key,
                           _validate_advance)
from .position import check_relative_bins, compute_relative_states, positional_args


def _decode_positional(state, q_t, t, position_mode, rope_cos, rope_sin, relative_states,
                       relative_proj, block_n=32):
    B, _, Hq, Dk = q_t.shape
    spec = state.spec(t + 1)
    bins = positional_args(position_mode, rope_cos, rope_sin, relative_states, relative_proj,
                           B=B, N=1, Hq=Hq, Dk=Dk, spec=spec, rope_positions=t + 1)
    cos = sin = st = pj = None
    if position_mode == "rope":
        cos = rope_cos.to(device=q_t.device, dtype=torch.float32).contiguous()
        sin = rope_sin.to(device=q_t.device, dtype=torch.float32).contiguous()
    elif position_mode == "relative":
        from ..range_spec import range_bounds
        visible = sum(hi - lo for lo, hi in (range_bounds(spec, t, lv) for lv in range(spec.num_levels)))
        check_relative_bins(spec, bins, visible, block_n=block_n, query=t)
        rdt = torch.result_type(relative_states, relative_proj)
        if rdt not in (torch.float32, torch.bfloat16, torch.float16):
            rdt = torch.float32
        st = relative_states.to(device=q_t.device, dtype=rdt).reshape(B, Hq, -1).contiguous()
        pj = relative_proj.to(device=q_t.device, dtype=rdt).contiguous()
    return cos, sin, st, pj


def _decode_stats(state, t, position_mode):
    """The reference's diagnostic dict: entries in gather order (level by
    level, ascending node), with rope positions / bin distances."""
    from ..range_spec import range_bounds
    spec = state.spec(t + 1)
    bounds = [range_bounds(spec, t, lv) for lv in range(spec.num_levels)]
    stats = {"entries": [], "positions": [], "distances": []}
    finer = 0
    for lv, (lo, hi) in enumerate(bounds):
        for j in range(lo, hi):
            stats["entries"].append((lv, j))
            if position_mode == "rope":
                stats["positions"].append(((j + 1) << lv) - 1)
            elif position_mode == "relative":
                stats["distances"].append(finer + hi - 1 - j)
        finer += hi - lo
    return stats


def multilevel_attention_decode(
    q_t: torch.Tensor,
    state: DecodeState,
    *,
    block_n: int = 32,
    softcap: float = 20.0,
    position_mode: str = "none",
    rope_cos: Optional[torch.Tensor] = None,
    rope_sin: Optional[torch.Tensor] = None,
    relative_states: Optional[torch.Tensor] = None,
    relative_proj: Optional[torch.Tensor] = None,
):
    """Attention of query t = state.t - 1 over its ring entries
    (reference.py:2093-2239) -> (out [B, 1, Hq, Dv], lse [B, 1, Hq] fp32, stats)."""
    if q_t.dim() != 4 or q_t.shape[1] != 1:
        raise ValueError(f"q_t must be [B, 1, Hq, Dk], got {tuple(q_t.shape)}")
    if state.t < 1:
        raise ValueError("no token has been consumed yet")
    B, _, Hq, Dk = q_t.shape
    Bs, _, Hkv, Dks = state.k.shape
    if Bs != B or Dks != Dk:
        raise ValueError(
            f"q_t {tuple(q_t.shape)} incompatible with the state's keys {tuple(state.k.shape)}")
    if Hq % Hkv != 0:
        raise ValueError(f"Hq={Hq} must be divisible by Hkv={Hkv}.")
    t = state.t - 1
    cos, sin, st, pj = _decode_positional(state, q_t, t, position_mode, rope_cos, rope_sin,
                                          relative_states, relative_proj, block_n)
    k_rot = _ensure_rotated_ring(state, cos, sin) if position_mode == "rope" else None
    out, lse, _, _ = _decode_launch(state, _lib.DECODE_ATTEND, q_t, softcap=softcap,
                                    position_mode=position_mode, cos=cos, sin=sin, rel_states=st,
                                    rel_proj=pj, t=t, k_rot=k_rot)
    return out, lse, _decode_stats(state, t, position_mode)


def decode_step(
    x_t: torch.Tensor,
    q_t: torch.Tensor,
    k_t: torch.Tensor,
    v_t: torch.Tensor,
    state: DecodeState,
    *,
    weight_mode: str = "qk",
    w_proj: Optional[torch.Tensor] = None,
    k_conv_weight: Optional[torch.Tensor] = None,
    v_conv_weight: Optional[torch.Tensor] = None,
    block_n: int = 32,
    softcap: float = 20.0,
    position_mode: str = "none",
    rope_cos: Optional[torch.Tensor] = None,
    rope_sin: Optional[torch.Tensor] = None,
    relative_weight: Optional[torch.Tensor] = None,
    relative_proj: Optional[torch.Tensor] = None,
    sinks: Optional[torch.Tensor] = None,
    gate_weight: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """The telescope block for one token after the Q/K/V projections: advance
    the cache, attend, sink, gate (reference.py:2242-2317).  Returns
    (out [B, 1, Hq, Dv] post-sink/gate, lse [B, 1, Hq] pre-sink fp32)."""
    if weight_mode == "qk":
        if w_proj is not None:
            raise ValueError("w_proj provided with weight_mode='qk'")
        wx, wp = None, None
    elif weight_mode == "linear":
        if w_proj is None:
            raise ValueError("weight_mode='linear' requires w_proj")
        wx, wp = x_t, w_proj
    else:
        raise ValueError(f"unknown weight_mode {weight_mode!r}")
    w_t = _validate_advance(state, q_t, k_t, v_t, wx, wp, k_conv_weight, v_conv_weight)
    B, _, Hq, Dk = q_t.shape
    Dv = state.v.shape[-1]
    relative_states = None
    if position_mode == "relative":
        if relative_weight is None or relative_proj is None:
            raise ValueError("position_mode='relative' requires relative_weight and relative_proj")
        relative_states = compute_relative_states(x_t, relative_weight, Hq)
    elif relative_weight is not None:
        raise ValueError(f"relative_weight provided with position_mode={position_mode!r}")
    t = state.t
    cos, sin, st, pj = _decode_positional(state, q_t, t, position_mode, rope_cos, rope_sin,
                                          relative_states, relative_proj, block_n)
    if sinks is not None and tuple(sinks.shape) != (Hq,):
        raise ValueError(f"sinks shape {tuple(sinks.shape)} != {(Hq,)} (one logit per query head)")
    gate_pre = None
    if gate_weight is not None:
        if x_t.dim() != 3 or x_t.shape[0] != B or x_t.shape[1] != 1:
            raise ValueError(f"x shape {tuple(x_t.shape)} incompatible with out; expected [B, 1, emb_dim]")
        if tuple(gate_weight.shape) != (Hq * Dv, x_t.shape[-1]):
            raise ValueError(
                f"gate_weight shape {tuple(gate_weight.shape)} != {(Hq * Dv, x_t.shape[-1])}")
        gate_pre = linear(x_t, gate_weight).reshape(B, Hq * Dv)
    _check_tick(state, t)
    k_rot = _ensure_rotated_ring(state, cos, sin) if position_mode == "rope" else None
    out, lse, _, _ = _decode_launch(
        state, _lib.DECODE_FULL, q_t, k_t, v_t, w_t=w_t, kcw=k_conv_weight, vcw=v_conv_weight,
        softcap=softcap, position_mode=position_mode, cos=cos, sin=sin, rel_states=st, rel_proj=pj,
        sinks=None if sinks is None else sinks.contiguous(), gate_pre=gate_pre, k_rot=k_rot)
    state.t = t + 1
    # the step wrote the rotated copies of the rows it created (rope), so the
    # ring stays current for these tables; other modes leave it stale
    state.k_rot_key = _rot_key(state, cos, sin) if k_rot is not None else None
    if gate_pre is not None:
        out = out.to(torch.result_type(out, gate_pre))
    return out, lse


__all__ = ["multilevel_attention_decode", "decode_step"]
