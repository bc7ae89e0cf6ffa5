"""Positional helpers: post-summary RoPE and the summary-bin relative bias
(reference ``telescoping_attn/position.py`` / ``reference.py:214-462``), plus
the positional-argument validation shared by forward, backward and decode
(``reference.py:675-768``)."""

import ctypes
from typing import Optional, Tuple

import torch

from .. import _lib
from .linear import project
from ..range_spec import IntOps, RangeSpec, elem_mask, range_bounds, visible_stats


def summary_token_position(level: int, local_index: int) -> int:
    """RoPE anchor of node (level, j): the right endpoint (j + 1) 2^level - 1
    of the tokens it summarises (reference.py:219-237)."""
    if level < 0 or local_index < 0:
        raise ValueError(
            f"level and local_index must be nonnegative, got ({level}, {local_index})")
    return ((local_index + 1) << level) - 1


def rope_tables(n_pos: int, dim: int, base: float = 10000.0, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [n_pos, dim // 2] float32, theta_i = base^(-2i/dim), GPT-NeoX
    rotate-half convention (reference.py:240-264)."""
    if dim <= 0 or dim % 2 != 0:
        raise ValueError(f"dim must be positive and even, got {dim}")
    if n_pos <= 0:
        raise ValueError(f"n_pos must be positive, got {n_pos}")
    freqs = base ** (-torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim)
    ang = torch.arange(n_pos, device=device, dtype=torch.float32)[:, None] * freqs[None, :]
    return torch.cos(ang), torch.sin(ang)


def _rope_into(x, y, cos, sin, kind, sched=None, positions=None, inverse=False):
    """tc_rope_apply over x viewed as [B, S, H, D]."""
    B, S, H, D = x.shape
    cos = cos if cos.dtype == torch.float32 and cos.is_contiguous() else cos.float().contiguous()
    sin = sin if sin.dtype == torch.float32 and sin.is_contiguous() else sin.float().contiguous()
    _lib.launch("tc_rope_apply", x.device,
        B, S, H, D, _lib.dtype_code(x.dtype), _lib.ptr(x), _lib.ptr(y), _lib.ptr(cos), _lib.ptr(sin),
        cos.shape[0], kind, None if sched is None else ctypes.byref(sched),
        _lib.ptr(positions), 1 if inverse else 0, _lib.stream_of(x))
    return y


def _rope_rows(x, pos, cos, sin, inverse):
    """tc_rope_apply at per-row positions pos (int32, x.shape[:-1])."""
    D = x.shape[-1]
    xc = x.contiguous()
    y = torch.empty_like(xc)
    if xc.numel():
        _rope_into(xc.reshape(1, 1, -1, D), y.reshape(1, 1, -1, D), cos, sin, 2,
                   positions=pos.reshape(-1), inverse=inverse)
    return y


class _Rope(torch.autograd.Function):
    """apply_rope with its VJP as backward: R(p) is orthogonal, so the
    gradient of y = R(p) x is R(p)^T dy = R(-p) dy, rotated in fp32 and cast
    to x's dtype as autograd does through the reference's x.float()."""

    @staticmethod
    def forward(ctx, x, pos, cos, sin, inverse):
        ctx.save_for_backward(pos, cos, sin)
        ctx.inverse = inverse
        ctx.x_dtype = x.dtype
        return _rope_rows(x, pos, cos, sin, inverse)

    @staticmethod
    def backward(ctx, gy):
        pos, cos, sin = ctx.saved_tensors
        g = gy if gy.dtype == ctx.x_dtype else gy.float()
        dx = _rope_rows(g, pos, cos, sin, not ctx.inverse).to(ctx.x_dtype)
        return dx, None, None, None, None


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               inverse: bool = False) -> torch.Tensor:
    """Rotate-half RoPE of x [..., D] at integer `positions` (broadcastable to
    x.shape[:-1]) in fp32, cast back; inverse=True applies R(-p)
    (reference.py:267-302).  Differentiable in x; the tables are constants
    (a cos / sin that requires gradients raises)."""
    if cos.shape != sin.shape:
        raise ValueError(f"cos shape {tuple(cos.shape)} != sin shape {tuple(sin.shape)}")
    D = x.shape[-1]
    if 2 * cos.shape[-1] != D:
        raise ValueError(f"rope tables cover dim {2 * cos.shape[-1]}, x has dim {D}")
    _lib.require_cuda(x, cos, sin)
    if not torch.is_tensor(positions):
        positions = torch.tensor(positions, device=x.device)
    pos = positions.to(device=x.device).expand(x.shape[:-1]).to(torch.int32).contiguous()
    if pos.numel() and (int(pos.min()) < 0 or int(pos.max()) >= cos.shape[0]):
        raise IndexError("rope position outside the tables")
    if torch.is_grad_enabled() and (x.requires_grad or cos.requires_grad or sin.requires_grad):
        if cos.requires_grad or sin.requires_grad:
            raise NotImplementedError("gradients with respect to the rope tables are not supported")
        return _Rope.apply(x, pos, cos, sin, bool(inverse))
    return _rope_rows(x, pos, cos, sin, inverse)


def validate_summary_causality(spec: RangeSpec) -> None:
    """Positional modes need a[l] >= 2^l - 1: a summary becomes visible only
    after its newest token (reference.py:305-324)."""
    for level in range(1, spec.num_levels):
        if spec.activation_times[level] < (1 << level) - 1:
            raise ValueError(
                f"schedule makes a level-{level} summary visible before its interval completes "
                f"(a[{level}]={spec.activation_times[level]} < {(1 << level) - 1}); positional "
                f"semantics undefined")


def relative_bin_distance(spec: RangeSpec, q: int, level: int, k_local: int) -> int:
    """0-based chronological bin distance of visible entry (level, k_local)
    from query q: the number of visible entries whose interval starts later
    (reference.py:327-371).  Raises ValueError if it is not visible."""
    if not elem_mask(spec, q, k_local, level):
        raise ValueError(f"entry (level={level}, k_local={k_local}) is not visible to query {q}")
    start = k_local << level
    total = older = 0
    for lv in range(spec.num_levels):
        lo, hi = range_bounds(spec, q, lv)
        total += hi - lo
        first_not_older = (start + (1 << lv) - 1) >> lv
        older += min(max(first_not_older, lo), hi) - lo
    return total - 1 - older


def compute_relative_states(x: torch.Tensor, relative_weight: torch.Tensor, Hq: int) -> torch.Tensor:
    """relative_states [B, N, Hq, d_rel] = x @ relative_weight^T, reshaped
    (reference.py:374-395), on tc_linear (gradients included)."""
    B, N, E = x.shape
    rows, Ew = relative_weight.shape
    if Ew != E or rows % Hq != 0:
        raise ValueError(
            f"relative_weight shape {tuple(relative_weight.shape)} incompatible with "
            f"emb_dim={E}, Hq={Hq}")
    return project(x, relative_weight).reshape(B, N, Hq, rows // Hq)


def positional_args(position_mode, rope_cos, rope_sin, relative_states, relative_proj, *,
                    B, N, Hq, Dk, spec, rope_positions):
    """Validate the positional arguments exactly like the reference
    (reference.py:675-768).  Returns max_relative_bins (0 unless relative).
    Unlike the reference, rel_logits are never materialised: the kernels
    form each bias from relative_states and relative_proj on the fly."""
    if position_mode not in ("none", "rope", "relative"):
        raise ValueError(
            f"position_mode must be 'none', 'rope' or 'relative', got {position_mode!r}")
    bins = 0
    if position_mode == "none":
        if any(t is not None for t in (rope_cos, rope_sin, relative_states, relative_proj)):
            raise ValueError("positional arguments provided with position_mode='none'")
    elif position_mode == "rope":
        if rope_cos is None or rope_sin is None:
            raise ValueError("position_mode='rope' requires rope_cos and rope_sin")
        if relative_states is not None or relative_proj is not None:
            raise ValueError("relative_* arguments provided with position_mode='rope'")
        if Dk % 2 != 0:
            raise ValueError(f"RoPE requires an even Dk, got {Dk}")
        if rope_cos.shape != rope_sin.shape:
            raise ValueError(
                f"rope_cos shape {tuple(rope_cos.shape)} != rope_sin shape {tuple(rope_sin.shape)}")
        if rope_cos.dim() != 2 or rope_cos.shape[-1] * 2 != Dk:
            raise ValueError(f"rope tables must be [n_pos, {Dk // 2}], got {tuple(rope_cos.shape)}")
        if rope_cos.shape[0] < rope_positions:
            raise ValueError(
                f"rope tables cover {rope_cos.shape[0]} positions; summary positions reach "
                f"N-1={rope_positions - 1}")
        validate_summary_causality(spec)
    else:
        if relative_states is None or relative_proj is None:
            raise ValueError(
                "position_mode='relative' requires relative_states and relative_proj")
        if rope_cos is not None or rope_sin is not None:
            raise ValueError("rope_* arguments provided with position_mode='relative'")
        if relative_states.dim() != 4 or tuple(relative_states.shape[:3]) != (B, N, Hq):
            raise ValueError(
                f"relative_states shape {tuple(relative_states.shape)} != [{B}, {N}, {Hq}, d_rel]")
        if relative_proj.dim() != 2 or relative_proj.shape[0] != relative_states.shape[-1]:
            raise ValueError(
                f"relative_proj shape {tuple(relative_proj.shape)} incompatible with "
                f"d_rel={relative_states.shape[-1]}")
        bins = relative_proj.shape[1]
        if bins < 1:
            raise ValueError("relative_proj must have >= 1 bins")
        validate_summary_causality(spec)
    return bins


def _first_bin_overflow(spec: RangeSpec, bins: int, q_blocks, block_n: int, exact: bool):
    """(distance, q_start, q_end, level) of the first tile at which the
    reference's loop meets a visible entry whose bin distance reaches
    `bins`, or None.  The reference walks query blocks in order, then
    levels, then block_n-node tiles (of the block's hull, or of the row's
    exact range when `exact`), and raises at the first tile holding an
    offending visible lane, reporting that tile's largest visible distance
    (reference.py:398-452, :959-1000, :1497-1545, :2175-2206).  A visible
    node j of level l has distance prefix(l) + hi(l) - 1 - j, prefix(l)
    counting the finer levels' entries."""
    import numpy as np

    from ..range_spec import fwd_bounds, level_row_bounds, normalize_empty

    a, cache = spec.activation_times, spec.cache_size
    nl = spec.num_levels
    np_ops = IntOps(minimum=np.minimum, maximum=np.maximum)
    for q_start, q_end in q_blocks:
        qs = np.arange(q_start, q_end, dtype=np.int64)
        raw = level_row_bounds(qs, a, cache, np_ops)
        lo = np.stack([np.where(l_ < h_, l_, 0) for l_, h_ in raw], 1)
        hi = np.stack([np.where(l_ < h_, h_, 0) for l_, h_ in raw], 1)
        cnt = hi - lo
        if int(cnt.sum(1).max()) - 1 < bins:
            continue
        prefix = np.cumsum(cnt, 1) - cnt
        for level in range(nl):
            if exact:
                k_lo, k_hi = int(lo[0, level]), int(hi[0, level])
            else:
                k_lo, k_hi = fwd_bounds(spec, q_start, q_end, level)
            if k_lo == k_hi:
                continue
            for k_start in range(k_lo, k_hi, block_n):
                k_end = min(k_start + block_n, k_hi)
                first = np.maximum(lo[:, level], k_start)
                vis = first < np.minimum(hi[:, level], k_end)
                if not vis.any():
                    continue
                dmax = int((prefix[:, level] + hi[:, level] - 1 - first)[vis].max())
                if dmax >= bins:
                    return dmax, q_start, q_end, level
    return None


def check_relative_bins(spec: RangeSpec, bins: int, max_visible: Optional[int] = None, *,
                        block_m: int = 16, block_n: int = 32, query: Optional[int] = None):
    """The reference raises when a visible entry's distance reaches the table
    size (reference.py:441-452).  Distances run to |A(q)| - 1, so whether it
    raises is max_q |A(q)| > bins, decided once per schedule; only then is
    the reference's tile loop replayed on the host (query blocks of block_m,
    or the single decode query `query` over its exact ranges, and block_n
    tiles) to raise with the same message at the same tile."""
    mx = visible_stats(spec)[1] if max_visible is None else max_visible
    if mx - 1 < bins:
        return
    if query is None:
        blocks = ((q, min(q + block_m, spec.seq_len)) for q in range(0, spec.seq_len, max(block_m, 1)))
    else:
        blocks = ((query, query + 1),)
    hit = _first_bin_overflow(spec, bins, blocks, max(block_n, 1), query is not None)
    if hit is None:
        return
    dist, q_start, q_end, level = hit
    raise ValueError(
        f"relative bin distance {dist} in query block [{q_start},{q_end}) at level {level} exceeds "
        f"max_relative_bins={bins}; no silent clamping -- a table with >= cache_size={spec.cache_size} "
        f"bins always suffices")


__all__ = ["summary_token_position", "rope_tables", "apply_rope", "validate_summary_causality",
           "relative_bin_distance", "compute_relative_states"]
