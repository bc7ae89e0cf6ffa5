"""Incremental decode: per-level modular rings driven by the schedule
(reference ``telescoping_attn/decode_state.py`` / ``reference.py:1675-2317``).

Node j of level l lives at ring slot ring_offsets[l] + j % caps[l]; the
schedule's ranges alone say which nodes are live.  A decode step (conv step,
merge weight, the single ruler-tick merge, the level-0 write, the attention
read of the new query, sink and gate) is one CUDA launch
(``tc_decode_step``); the gate and linear-weight projections of the token's
hidden state run first as one GEMM / GEMV each.
"""

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from .. import _lib
from ..range_spec import (RangeSpec, activation_times_from_fmap, level_row_bounds,
                          range_bounds)
from .position import compute_relative_states, positional_args, check_relative_bins
from .summaries import _check_conv_weight, compute_linear_weights, short_conv


@dataclass
class DecodeState:
    """One layer's decode cache (reference.py:1703-1736):
    k [B, sum(caps), Hkv, Dk] unrotated post-conv keys, v [B, sum(caps), Hkv, Dv],
    w [B, sum(caps), Hkv, 1] merge log-weights, conv_k/conv_v [B, K-1, Hkv*D]
    (last K-1 pre-conv rows, newest last) or None, t = tokens consumed.

    k_rot / k_rot_key are this build's derived cache for rope decode: the ring
    keys rotated at their summary positions, valid for the rope tables named by
    the key.  Every decode call keeps it current or marks it stale; it is
    rebuilt from k when needed, so it never changes results."""

    k: torch.Tensor
    v: torch.Tensor
    w: torch.Tensor
    conv_k: Optional[torch.Tensor]
    conv_v: Optional[torch.Tensor]
    t: int
    activation_times: Tuple[int, ...]
    cache_size: int
    caps: Tuple[int, ...]
    ring_offsets: Tuple[int, ...]
    k_rot: Optional[torch.Tensor] = None
    k_rot_key: Optional[tuple] = None

    @property
    def num_levels(self) -> int:
        return len(self.activation_times)

    def spec(self, seq_len: int) -> RangeSpec:
        return RangeSpec(self.activation_times, self.cache_size, seq_len)


_CAPS: Dict[Tuple, Tuple[int, ...]] = {}


def decode_capacities(activation_times: Tuple[int, ...], cache_size: int) -> Tuple[int, ...]:
    """Ring capacity per level: the peak live count of each fine level and
    the most the coarsest can be left over two schedule periods
    (reference.py:1739-1772); one scan in the C library, memoised."""
    a = tuple(activation_times)
    if not a or a[0] != 0:
        raise ValueError("activation_times must start with a[0] = 0")
    if cache_size <= 0:
        raise ValueError("cache_size must be positive")
    key = (a, cache_size)
    hit = _CAPS.get(key)
    if hit is None:
        if len(a) > _lib.MAX_LEVELS:
            raise NotImplementedError(f"at most {_lib.MAX_LEVELS} levels are supported")
        act = (ctypes.c_int32 * len(a))(*a)
        caps = (ctypes.c_int32 * len(a))()
        rc = _lib.lib().tc_decode_caps(ctypes.cast(act, ctypes.c_void_p), len(a), cache_size,
                                       ctypes.cast(caps, ctypes.c_void_p))
        if rc == _lib.TC_ERR_ARG:
            raise ValueError(f"fine levels need more slots than cache_size={cache_size}")
        _lib.check(rc, "tc_decode_caps")
        hit = tuple(int(c) for c in caps)
        _CAPS[key] = hit
    return hit


def ring_slot(state: DecodeState, level: int, j: int) -> int:
    """Physical slot of node j at `level` (reference.py:1775-1784)."""
    if not 0 <= level < state.num_levels:
        raise ValueError(f"level {level} out of range [0, {state.num_levels - 1}]")
    if j < 0:
        raise ValueError(f"node index must be nonnegative, got {j}")
    return state.ring_offsets[level] + j % state.caps[level]


def _dense_rows(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """t [B, n, ...] in `dtype` with every token's trailing block dense (the
    layout tc_decode_init copies rows from); batch and token strides stay free."""
    t = t.to(dtype)
    want = 1
    for size, stride in zip(reversed(t.shape[2:]), reversed(t.stride()[2:])):
        if size != 1 and stride != want:
            return t.contiguous()
        want *= size
    return t


def _conv_history(x_pre: torch.Tensor, kernel_size: int, seq_idx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Last K-1 rows of x_pre [B, N, C], zero-padded on the left when N < K-1
    (reference.py:1796-1807).  With segment ids seq_idx [B, N], rows of an
    earlier example than the last row's are zeroed: decoding continues the
    last packed example only."""
    hist = kernel_size - 1
    if hist == 0:
        return x_pre[:, :0].clone()
    # slice before padding: only the last K-1 rows are copied, not the prefill
    tail = x_pre[:, -hist:]
    if seq_idx is not None:
        same = seq_idx[:, -tail.shape[1]:] == seq_idx[:, -1:]
        tail = torch.where(same.unsqueeze(-1), tail, torch.zeros((), dtype=tail.dtype, device=tail.device))
    pad = hist - tail.shape[1]
    if pad > 0:
        return torch.nn.functional.pad(tail, (0, 0, pad, 0)).contiguous()
    # a copy, never a view: decode steps update the history in place
    return tail.clone(memory_format=torch.contiguous_format)


def short_conv_step(x: torch.Tensor, state: torch.Tensor, weight: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """One-token short conv: full = [state, x], y = x + sum_j w[:, j] full[j]
    with fp32 taps and residual (reference.py:1810-1845).  Returns
    (y [B, 1, C], new_state = full[:, 1:])."""
    if x.dim() != 3 or x.shape[1] != 1:
        raise ValueError(f"x must be [B, 1, C], got {tuple(x.shape)}")
    B, _, C = x.shape
    _check_conv_weight(weight, C)
    K = weight.shape[1]
    if tuple(state.shape) != (B, K - 1, C):
        raise ValueError(f"conv state shape {tuple(state.shape)} != {(B, K - 1, C)}")
    full = torch.cat([state, x], dim=1)
    # the causal conv at the last of K rows sees exactly the K taps
    y = short_conv(full, weight)[:, -1:]
    return y, full[:, 1:]


def init_decode_state(
    k_levels: List[torch.Tensor],
    v_levels: List[torch.Tensor],
    w_levels: List[torch.Tensor],
    fmap: Dict[int, int],
    cache_size: int,
    *,
    k_pre_conv: Optional[torch.Tensor] = None,
    v_pre_conv: Optional[torch.Tensor] = None,
    conv_kernel_size: Optional[int] = None,
    seq_idx: Optional[torch.Tensor] = None,
) -> DecodeState:
    """Prefill hand-off: the nodes live at query N-1 go to their ring slots and
    t = N; the last K-1 pre-conv rows seed the conv history
    (reference.py:1848-1945).  seq_idx (an extension, as for short_conv):
    segment ids [B, N] of a packed prefill; history rows of earlier examples
    than the last row's are zeroed."""
    if (k_pre_conv is None) != (v_pre_conv is None):
        raise ValueError("k_pre_conv and v_pre_conv must both be provided or both be None")
    if (k_pre_conv is None) != (conv_kernel_size is None):
        raise ValueError("conv_kernel_size must accompany the pre-conv rows (and vice versa)")
    a = activation_times_from_fmap(fmap)
    L = len(a) - 1
    if min(len(k_levels), len(v_levels), len(w_levels)) < L + 1:
        raise ValueError(
            f"need {L + 1} levels, got {len(k_levels)}/{len(v_levels)}/{len(w_levels)}")
    B, N, Hkv, Dk = k_levels[0].shape
    Dv = v_levels[0].shape[-1]
    if N < 1:
        raise ValueError("prefill must contain at least one token")
    if tuple(w_levels[0].shape) != (B, N, Hkv, 1):
        raise ValueError(f"w_levels[0] shape {tuple(w_levels[0].shape)} != {(B, N, Hkv, 1)}")
    caps = decode_capacities(a, cache_size)
    offs = [0]
    for c in caps:
        offs.append(offs[-1] + c)
    total = offs[-1]
    dev = k_levels[0].device
    # the kernel copies (Hkv, D) rows of B batch rows from every level with live
    # nodes: their batch and trailing sizes must match level 0's
    spec = RangeSpec(a, cache_size, N)
    for level in range(L + 1):
        lo, hi = range_bounds(spec, N - 1, level)
        if lo == hi:
            continue
        for name, t, tail in (("k_levels", k_levels[level], (Hkv, Dk)), ("v_levels", v_levels[level], (Hkv, Dv)),
                              ("w_levels", w_levels[level], (Hkv, 1))):
            if t.dim() != 4 or t.shape[0] != B or tuple(t.shape[2:]) != tail:
                raise ValueError(
                    f"{name}[{level}] shape {tuple(t.shape)} != [{B}, n, {tail[0]}, {tail[1]}]")
    _lib.require_cuda(*k_levels[:L + 1], *v_levels[:L + 1], *w_levels[:L + 1])
    kdt, vdt, wdt = k_levels[0].dtype, v_levels[0].dtype, w_levels[0].dtype
    if kdt != vdt:
        raise NotImplementedError(f"key and value levels must share a dtype ({kdt} vs {vdt})")
    if L + 1 > _lib.MAX_LEVELS:
        raise NotImplementedError(f"at most {_lib.MAX_LEVELS} levels are supported")
    # every slot is written by tc_decode_init (live node or zeros)
    state = DecodeState(
        k=torch.empty(B, total, Hkv, Dk, device=dev, dtype=kdt),
        v=torch.empty(B, total, Hkv, Dv, device=dev, dtype=vdt),
        w=torch.empty(B, total, Hkv, 1, device=dev, dtype=wdt),
        conv_k=None, conv_v=None, t=N, activation_times=a, cache_size=cache_size, caps=caps,
        ring_offsets=tuple(offs))
    args = _lib.DecodeInitArgs()
    args.B, args.Hkv, args.Dk, args.Dv = B, Hkv, Dk, Dv
    args.dtype, args.w_dtype = _lib.dtype_code(kdt), _lib.dtype_code(wdt)
    args.num_levels = L + 1
    args.ring_off[0] = 0
    keep = []  # level tensors converted for the kernel stay alive until the launch
    for level in range(L + 1):
        lo, hi = range_bounds(spec, N - 1, level)
        args.caps[level] = caps[level]
        args.ring_off[level + 1] = offs[level + 1]
        args.lo[level], args.hi[level] = lo, hi
        if lo == hi:
            continue
        if hi > k_levels[level].shape[1] or hi > v_levels[level].shape[1] or hi > w_levels[level].shape[1]:
            raise ValueError(f"level {level}: live range [{lo},{hi}) exceeds the given level tensors")
        if hi - lo > caps[level]:
            raise AssertionError(f"level {level} has {hi - lo} live nodes > cap {caps[level]} at q={N - 1}")
        kl, vl = _dense_rows(k_levels[level], kdt), _dense_rows(v_levels[level], vdt)
        wl = _dense_rows(w_levels[level].squeeze(-1), wdt)
        keep += [kl, vl, wl]
        args.k_lv[level], args.v_lv[level], args.w_lv[level] = kl.data_ptr(), vl.data_ptr(), wl.data_ptr()
        args.k_stride_b[level], args.k_stride_n[level] = kl.stride(0), kl.stride(1)
        args.v_stride_b[level], args.v_stride_n[level] = vl.stride(0), vl.stride(1)
        args.w_stride_b[level], args.w_stride_n[level] = wl.stride(0), wl.stride(1)
    args.ring_k, args.ring_v, args.ring_w = state.k.data_ptr(), state.v.data_ptr(), state.w.data_ptr()
    _lib.launch("tc_decode_init", state.k.device, ctypes.byref(args), _lib.stream_of(state.k))
    del keep
    if k_pre_conv is not None:
        if conv_kernel_size <= 0:
            raise ValueError(f"conv kernel size must be positive, got {conv_kernel_size}")
        if k_pre_conv.shape[:2] != (B, N) or v_pre_conv.shape[:2] != (B, N):
            raise ValueError(
                f"pre-conv rows must be [B={B}, N={N}, ...], got {tuple(k_pre_conv.shape)} / "
                f"{tuple(v_pre_conv.shape)}")
        seq = None
        if seq_idx is not None:
            if tuple(seq_idx.shape) != (B, N) or seq_idx.dtype.is_floating_point:
                raise ValueError(f"seq_idx must be an integer tensor [{B}, {N}], got {tuple(seq_idx.shape)}")
            seq = seq_idx.to(k_pre_conv.device)
        state.conv_k = _conv_history(k_pre_conv.reshape(B, N, -1), conv_kernel_size, seq)
        state.conv_v = _conv_history(v_pre_conv.reshape(B, N, -1), conv_kernel_size, seq)
    return state


def _check_tick(state: DecodeState, t: int):
    """The schedule invariants the reference asserts at every step
    (reference.py:2036-2082): at most one level fires, its children are live
    at t-1, and no level exceeds its ring capacity at t.  Every level's range
    of a row comes from one pass of the closed forms; the ranges of query t
    are memoised for the next step's check of t - 1."""
    a = state.activation_times
    fired = None
    for level in range(1, len(a)):
        if t >= a[level] and (t - a[level]) % (1 << level) == 0:
            if fired is not None:
                raise AssertionError(
                    f"levels {fired} and {level} both activate at t={t}; the schedule is not "
                    f"dyadically aligned")
            fired = level
    if fired is not None:
        j = (t - a[fired]) >> fired
        lo_c, hi_c = _checked_bounds(state, t - 1, t)[fired - 1]
        if not (lo_c <= 2 * j and 2 * j + 1 < hi_c):
            raise AssertionError(
                f"children of node ({fired}, {j}) not live at t-1={t - 1}: level-{fired - 1} "
                f"range [{lo_c},{hi_c})")
    for level, (lo, hi) in enumerate(_checked_bounds(state, t, t + 1)):
        if hi - lo > state.caps[level]:
            raise AssertionError(
                f"level {level} needs {hi - lo} live slots > cap {state.caps[level]} at t={t}")


_BOUNDS_MEMO: Dict[Tuple, list] = {}


def _checked_bounds(state: DecodeState, q: int, seq_len: int):
    """range_bounds(spec(seq_len), q, level) for every level at once: the
    normalised ranges of query q with the reference's level-length check.
    The last two results per schedule are memoised (a step checks t - 1 and
    t; the next step checks t and t + 1)."""
    if not 0 <= q < seq_len:
        raise ValueError(f"q={q} out of range [0, {seq_len})")
    key = (state.activation_times, state.cache_size, q, seq_len)
    hit = _BOUNDS_MEMO.get(key)
    if hit is not None:
        return hit
    out = []
    for level, (lo, hi) in enumerate(level_row_bounds(q, state.activation_times, state.cache_size)):
        if lo >= hi:
            lo = hi = 0
        if hi > seq_len >> level:
            raise AssertionError(
                f"range [{lo},{hi}) exceeds level_len={seq_len >> level} at q={q}, level={level}")
        out.append((lo, hi))
    if len(_BOUNDS_MEMO) >= 64:
        _BOUNDS_MEMO.clear()
    _BOUNDS_MEMO[key] = out
    return out


DECODE_MAX_SPLITS = 8


def _rot_key(state: DecodeState, cos, sin):
    return (cos.data_ptr(), sin.data_ptr(), tuple(cos.shape), state.k.data_ptr(), state.t)


def _ensure_rotated_ring(state: DecodeState, cos, sin):
    """Make state.k_rot hold the live keys rotated with these tables (rebuilt
    from state.k by one launch when stale).  Returns the ring."""
    if state.k_rot is None or state.k_rot.shape != state.k.shape or state.k_rot.dtype != state.k.dtype \
            or state.k_rot.device != state.k.device:
        state.k_rot = torch.empty_like(state.k)
        state.k_rot_key = None
    if state.k_rot_key != _rot_key(state, cos, sin):
        if state.t >= 1:
            B, _, Hkv, Dk = state.k.shape
            dummy = torch.empty(B, 1, Hkv, Dk, device=state.k.device, dtype=state.k.dtype)
            _decode_launch(state, _lib.DECODE_ROTATE, dummy, position_mode="rope", cos=cos, sin=sin,
                           t=state.t - 1, k_rot=state.k_rot)
        state.k_rot_key = _rot_key(state, cos, sin)
    return state.k_rot


_WORKSPACE: Dict[Tuple, torch.Tensor] = {}


def _workspace(device, stream, numel):
    """The split-attention scratch (partial softmax states): one buffer per
    device, stream and size, reused by the steps issued on that stream (which
    run in issue order, so they never overlap)."""
    key = (device, stream.value, numel)
    ws = _WORKSPACE.get(key)
    if ws is None:
        if len(_WORKSPACE) >= 32:
            _WORKSPACE.clear()
        ws = torch.empty(numel, device=device, dtype=torch.float32)
        _WORKSPACE[key] = ws
    return ws


def _static_args(state: DecodeState, Hq: int):
    """The fields of tc_decode_args that depend only on the state (dims,
    dtypes, schedule, ring pointers), built once per state and copied into
    each call's struct."""
    key = (Hq, state.k.data_ptr(), state.v.data_ptr(), state.w.data_ptr(), state.k.dtype, state.w.dtype,
           tuple(state.k.shape), tuple(state.v.shape))
    cached = getattr(state, "_args_proto", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    B, _, Hkv, Dk = state.k.shape
    proto = _lib.DecodeArgs(
        B=B, Hq=Hq, Hkv=Hkv, Dk=Dk, Dv=state.v.shape[-1], dtype=_lib.dtype_code(state.k.dtype),
        w_dtype=_lib.dtype_code(state.w.dtype), num_levels=state.num_levels, cache_size=state.cache_size,
        act=(ctypes.c_int32 * _lib.MAX_LEVELS)(*state.activation_times),
        caps=(ctypes.c_int32 * _lib.MAX_LEVELS)(*state.caps),
        ring_off=(ctypes.c_int32 * (_lib.MAX_LEVELS + 1))(*state.ring_offsets),
        ring_k=state.k.data_ptr(), ring_v=state.v.data_ptr(), ring_w=state.w.data_ptr())
    object.__setattr__(state, "_args_proto", (key, proto))
    return proto


def _decode_launch(state: DecodeState, mode, q_t, k_t=None, v_t=None, w_t=None, kcw=None, vcw=None,
                   softcap=None, position_mode="none", cos=None, sin=None, rel_states=None,
                   rel_proj=None, sinks=None, gate_pre=None, t=None, want_kv=False, k_rot=None):
    B, _, Hq, Dk = q_t.shape
    Hkv = state.k.shape[2]
    Dv = state.v.shape[-1]
    dtype = state.k.dtype
    _lib.require_cuda(q_t, state.k, state.v, state.w)
    for name, ring in (("k", state.k), ("v", state.v), ("w", state.w)):
        if not ring.is_contiguous():
            raise ValueError(f"decode ring {name} must be contiguous (it is updated in place)")
    qc = q_t.to(dtype).contiguous()
    kc = None if k_t is None else k_t.to(dtype).contiguous()
    vc = None if v_t is None else v_t.to(dtype).contiguous()
    out = torch.empty(B, 1, Hq, Dv, device=q_t.device, dtype=dtype)
    lse = torch.empty(B, 1, Hq, device=q_t.device, dtype=torch.float32)
    k_new = torch.empty(B, 1, Hkv, Dk, device=q_t.device, dtype=dtype) if want_kv else None
    v_new = torch.empty(B, 1, Hkv, Dv, device=q_t.device, dtype=dtype) if want_kv else None
    stream = _lib.stream_of(q_t)
    ws = None
    if Dk == 128 and Dv == 128 and dtype in (torch.bfloat16, torch.float16):
        # scratch for splitting each (batch, KV head)'s entries over CTAs
        ws = _workspace(q_t.device, stream, B * Hkv * DECODE_MAX_SPLITS * (Hq // Hkv) * 130)
    conv_w = 0 if kcw is None else kcw.shape[1]
    if kcw is not None:
        kcw = kcw.contiguous()
        vcw = vcw.to(kcw.dtype).contiguous()
        for name, cs in (("conv_k", state.conv_k), ("conv_v", state.conv_v)):
            if not cs.is_contiguous() or cs.dtype != dtype:
                setattr(state, name, cs.to(dtype).contiguous())
    keep = []

    def p(t_):
        if t_ is None:
            return None
        keep.append(t_)
        return t_.data_ptr()

    args = _lib.DecodeArgs()
    ctypes.pointer(args)[0] = _static_args(state, Hq)
    args.mode = mode
    args.t = state.t if t is None else t
    if conv_w:
        args.conv_k, args.conv_v = p(state.conv_k), p(state.conv_v)
        args.k_conv_w, args.v_conv_w = p(kcw), p(vcw)
        args.conv_dtype = _lib.dtype_code(kcw.dtype)
        args.conv_k_width = conv_w
    args.q_t, args.k_t, args.v_t, args.w_t = p(qc), p(kc), p(vc), p(w_t)
    args.has_softcap = 0 if softcap is None else 1
    args.softcap = 0.0 if softcap is None else float(softcap)
    args.position_mode = _lib.POS[position_mode]
    args.rope_cos, args.rope_sin = p(cos), p(sin)
    if rel_states is not None:
        args.rel_states, args.rel_proj = p(rel_states), p(rel_proj)
        args.rel_dtype = _lib.dtype_code(rel_states.dtype)
        args.d_rel = rel_states.shape[-1]
        args.rel_bins = rel_proj.shape[1]
    if sinks is not None:
        args.sinks, args.sink_dtype = p(sinks), _lib.dtype_code(sinks.dtype)
    if gate_pre is not None:
        args.gate_pre, args.gate_dtype = p(gate_pre), _lib.dtype_code(gate_pre.dtype)
    args.out, args.lse = out.data_ptr(), lse.data_ptr()
    args.k_new, args.v_new = p(k_new), p(v_new)
    if ws is not None:
        args.workspace, args.workspace_floats = ws.data_ptr(), ws.numel()
    args.ring_k_rot = p(k_rot)
    _lib.launch("tc_decode_step", q_t.device, ctypes.byref(args), stream)
    del keep
    return out, lse, k_new, v_new


def _validate_advance(state, q_t, k_t, v_t, x_t, w_proj, k_conv_weight, v_conv_weight):
    B, _, Hkv, Dk = state.k.shape
    Dv = state.v.shape[-1]
    if q_t.dim() != 4 or q_t.shape[0] != B or q_t.shape[1] != 1 or q_t.shape[-1] != Dk \
            or q_t.shape[2] % Hkv != 0:
        raise ValueError(
            f"q_t shape {tuple(q_t.shape)} incompatible with [B={B}, 1, Hq (multiple of {Hkv}), "
            f"Dk={Dk}]")
    if tuple(k_t.shape) != (B, 1, Hkv, Dk):
        raise ValueError(f"k_t shape {tuple(k_t.shape)} != {(B, 1, Hkv, Dk)}")
    if tuple(v_t.shape) != (B, 1, Hkv, Dv):
        raise ValueError(f"v_t shape {tuple(v_t.shape)} != {(B, 1, Hkv, Dv)}")
    if (k_conv_weight is None) != (v_conv_weight is None):
        raise ValueError("k_conv_weight and v_conv_weight must both be provided or both be None")
    if k_conv_weight is not None:
        if state.conv_k is None or state.conv_v is None:
            raise ValueError(
                "conv weights given but the state was initialised without pre-conv rows "
                "(init_decode_state k_pre_conv/v_pre_conv)")
        _check_conv_weight(k_conv_weight, Hkv * Dk)
        _check_conv_weight(v_conv_weight, Hkv * Dv)
        K = k_conv_weight.shape[1]
        if v_conv_weight.shape[1] != K:
            raise NotImplementedError("K and V conv widths must match")
        if tuple(state.conv_k.shape) != (B, K - 1, Hkv * Dk):
            raise ValueError(f"conv state shape {tuple(state.conv_k.shape)} != {(B, K - 1, Hkv * Dk)}")
    elif state.conv_k is not None:
        raise ValueError("the state carries a conv state but no conv weights were given")
    if (x_t is None) != (w_proj is None):
        raise ValueError(
            "x_t and w_proj must both be provided (linear weight mode) or both be None (QK weight mode)")
    w_t = None
    if x_t is not None:
        w_t = compute_linear_weights(x_t, w_proj)
        if tuple(w_t.shape) != (B, 1, Hkv, 1):
            raise ValueError(f"linear weights shape {tuple(w_t.shape)} != {(B, 1, Hkv, 1)}")
        w_t = w_t.to(state.w.dtype).contiguous()
    return w_t


def advance_decode_state(state: DecodeState, q_t: torch.Tensor, k_t: torch.Tensor, v_t: torch.Tensor,
                         *, x_t: Optional[torch.Tensor] = None, w_proj: Optional[torch.Tensor] = None,
                         k_conv_weight: Optional[torch.Tensor] = None,
                         v_conv_weight: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Consume token t = state.t in place: conv step, merge weight, the ruler-
    tick merge, then the level-0 write; state.t becomes t + 1
    (reference.py:1948-2090).  Returns (k_t, v_t) as stored (post-conv)."""
    w_t = _validate_advance(state, q_t, k_t, v_t, x_t, w_proj, k_conv_weight, v_conv_weight)
    _check_tick(state, state.t)
    _, _, k_new, v_new = _decode_launch(state, _lib.DECODE_ADVANCE, q_t, k_t, v_t, w_t=w_t,
                                        kcw=k_conv_weight, vcw=v_conv_weight, want_kv=True)
    state.t += 1
    state.k_rot_key = None  # no rope tables here: the rotated ring is stale
    return k_new, v_new


__all__ = ["DecodeState", "decode_capacities", "ring_slot", "short_conv_step", "init_decode_state",
           "advance_decode_state"]
