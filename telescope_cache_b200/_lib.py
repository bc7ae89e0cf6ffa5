"""ctypes binding of ``libtelescope_b200.so`` (declared in
``include/telescope_cache.h``).

The library is the only compute path: if it is missing or a CUDA tensor is
not available the calls raise; there is no CPU fallback.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libtelescope_b200.so")

MAX_LEVELS = 16

TC_OK, TC_ERR_ARG, TC_ERR_UNSUPPORTED, TC_ERR_CUDA, TC_ERR_SCHEDULE = 0, 1, 2, 3, 4
TC_F32, TC_BF16, TC_F16 = 0, 1, 2
TC_LIN_STORE, TC_LIN_GATE = 0, 1
POS = {"none": 0, "rope": 1, "relative": 2}
DECODE_FULL, DECODE_ADVANCE, DECODE_ATTEND, DECODE_ROTATE = 0, 1, 2, 3

_c_i32, _c_i64, _c_f32, _c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class Schedule(ctypes.Structure):
    _fields_ = [
        ("num_levels", _c_i32), ("cache_size", _c_i32), ("seq_len", _c_i32),
        ("coarsest_span", _c_i32), ("act", _c_i32 * MAX_LEVELS),
        ("level_len", _c_i32 * MAX_LEVELS), ("offsets", _c_i64 * (MAX_LEVELS + 1)),
    ]


class TreeArgs(ctypes.Structure):
    _fields_ = [
        ("B", _c_i32), ("N", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("Dk", _c_i32),
        ("Dv", _c_i32), ("num_summary_levels", _c_i32), ("dtype", _c_i32), ("w_dtype", _c_i32),
        ("q", _c_vp), ("k", _c_vp), ("v", _c_vp), ("w0", _c_vp), ("k_conv_w", _c_vp),
        ("v_conv_w", _c_vp), ("conv_dtype", _c_i32), ("conv_k", _c_i32), ("k_packed", _c_vp),
        ("v_packed", _c_vp), ("w_packed", _c_vp), ("total", _c_i64),
    ]


class TreeBwdArgs(ctypes.Structure):
    _fields_ = [
        ("B", _c_i32), ("N", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("Dk", _c_i32),
        ("Dv", _c_i32), ("num_summary_levels", _c_i32), ("dtype", _c_i32), ("w_dtype", _c_i32),
        ("detach", _c_i32), ("q", _c_vp), ("k_packed", _c_vp), ("v_packed", _c_vp), ("w_packed", _c_vp),
        ("gk_packed", _c_vp), ("gv_packed", _c_vp), ("gw_packed", _c_vp), ("dq", _c_vp),
        ("dq_dtype", _c_i32), ("d0_dtype", _c_i32), ("dk0", _c_vp), ("dv0", _c_vp), ("dw0", _c_vp),
        ("scratch", _c_vp), ("scratch_bytes", _c_i64), ("total", _c_i64),
    ]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("B", _c_i32), ("N", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("Dk", _c_i32),
        ("Dv", _c_i32), ("dtype", _c_i32), ("has_softcap", _c_i32), ("softcap", _c_f32),
        ("position_mode", _c_i32), ("q", _c_vp), ("k", _c_vp), ("v", _c_vp),
        ("rel_states", _c_vp), ("rel_proj", _c_vp), ("rel_dtype", _c_i32), ("d_rel", _c_i32),
        ("rel_bins", _c_i32), ("rope_cos", _c_vp), ("rope_sin", _c_vp), ("rope_npos", _c_i32),
        ("out", _c_vp), ("lse", _c_vp), ("o", _c_vp), ("dout", _c_vp), ("dlse", _c_vp),
        ("delta", _c_vp), ("dq", _c_vp), ("dk", _c_vp), ("dv", _c_vp), ("drel", _c_vp),
        ("dev_status", _c_vp), ("impl", _c_i32), ("rel_logits", _c_vp),
        ("rel_logits_stride", _c_i64), ("rel_logits_pad", _c_i32), ("tile_n", _c_i32),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("mode", _c_i32), ("B", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("Dk", _c_i32),
        ("Dv", _c_i32), ("dtype", _c_i32), ("w_dtype", _c_i32), ("t", _c_i32),
        ("num_levels", _c_i32), ("cache_size", _c_i32), ("act", _c_i32 * MAX_LEVELS),
        ("caps", _c_i32 * MAX_LEVELS), ("ring_off", _c_i32 * (MAX_LEVELS + 1)),
        ("ring_k", _c_vp), ("ring_v", _c_vp), ("ring_w", _c_vp), ("conv_k", _c_vp),
        ("conv_v", _c_vp), ("k_conv_w", _c_vp), ("v_conv_w", _c_vp), ("conv_dtype", _c_i32),
        ("conv_k_width", _c_i32), ("q_t", _c_vp), ("k_t", _c_vp), ("v_t", _c_vp), ("w_t", _c_vp),
        ("has_softcap", _c_i32), ("softcap", _c_f32), ("position_mode", _c_i32),
        ("rope_cos", _c_vp), ("rope_sin", _c_vp), ("rel_states", _c_vp), ("rel_proj", _c_vp),
        ("rel_dtype", _c_i32), ("d_rel", _c_i32), ("rel_bins", _c_i32), ("sinks", _c_vp),
        ("sink_dtype", _c_i32), ("gate_pre", _c_vp), ("gate_dtype", _c_i32), ("out", _c_vp),
        ("lse", _c_vp), ("k_new", _c_vp), ("v_new", _c_vp), ("workspace", _c_vp),
        ("workspace_floats", _c_i64), ("ring_k_rot", _c_vp),
    ]


class DecodeInitArgs(ctypes.Structure):
    _fields_ = [
        ("B", _c_i32), ("Hkv", _c_i32), ("Dk", _c_i32), ("Dv", _c_i32), ("dtype", _c_i32),
        ("w_dtype", _c_i32), ("num_levels", _c_i32), ("caps", _c_i32 * MAX_LEVELS),
        ("ring_off", _c_i32 * (MAX_LEVELS + 1)), ("lo", _c_i32 * MAX_LEVELS),
        ("hi", _c_i32 * MAX_LEVELS), ("k_lv", _c_vp * MAX_LEVELS), ("v_lv", _c_vp * MAX_LEVELS),
        ("w_lv", _c_vp * MAX_LEVELS), ("k_stride_b", _c_i64 * MAX_LEVELS),
        ("k_stride_n", _c_i64 * MAX_LEVELS), ("v_stride_b", _c_i64 * MAX_LEVELS),
        ("v_stride_n", _c_i64 * MAX_LEVELS), ("w_stride_b", _c_i64 * MAX_LEVELS),
        ("w_stride_n", _c_i64 * MAX_LEVELS), ("ring_k", _c_vp), ("ring_v", _c_vp), ("ring_w", _c_vp),
    ]


# (name, argtypes) of every exported symbol; the CPU test checks that each one
# exists and that this list matches include/telescope_cache.h.
SIGNATURES = {
    "tc_version": [],
    "tc_schedule_init": [_c_vp, _c_i32, _c_i32, _c_i32, ctypes.POINTER(Schedule)],
    "tc_schedule_from_times": [_c_vp, _c_i32, _c_i32, _c_i32, ctypes.POINTER(Schedule)],
    "tc_schedule_stats": [ctypes.POINTER(Schedule), _c_vp],
    "tc_decode_caps": [_c_vp, _c_i32, _c_i32, _c_vp],
    "tc_range_bounds_host": [ctypes.POINTER(Schedule), _c_vp, _c_i32, _c_vp],
    "tc_hulls_host": [ctypes.POINTER(Schedule), _c_i32, _c_i32, _c_vp, _c_vp, _c_i32, _c_vp],
    "tc_range_bounds_device": [ctypes.POINTER(Schedule), _c_vp, _c_i32, _c_vp, _c_vp],
    "tc_build_tree": [ctypes.POINTER(TreeArgs), _c_vp],
    "tc_build_tree_bwd": [ctypes.POINTER(TreeBwdArgs), _c_vp],
    "tc_tree_bwd_scratch_bytes": [ctypes.POINTER(TreeBwdArgs)],
    "tc_short_conv_bwd": [_c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_i32, _c_vp, _c_vp, _c_vp, _c_vp,
                          _c_vp, _c_i64, _c_vp],
    "tc_linear_weights": [_c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_vp, _c_i32, _c_vp, _c_vp],
    "tc_linear": [_c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp, _c_i64,
                  _c_i32, _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_vp],
    "tc_linear_scratch_floats": [_c_i64, _c_i32, _c_i32, _c_i32],
    "tc_linear_wgrad": [_c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp, _c_i64, _c_i32, _c_vp,
                        _c_i64, _c_vp, _c_i64, _c_vp, _c_vp],
    "tc_linear_wgrad_scratch_floats": [_c_i64, _c_i32, _c_i32],
    "tc_qk_weights": [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp, _c_i32, _c_vp,
                      _c_vp],
    "tc_short_conv": [_c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_i32, _c_vp, _c_vp, _c_vp],
    "tc_short_conv_seg": [_c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_i32, _c_vp, _c_vp, _c_vp, _c_vp],
    "tc_short_conv_seg_bwd": [_c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_i32, _c_vp, _c_vp, _c_vp, _c_vp,
                              _c_vp, _c_vp, _c_i64, _c_vp],
    "tc_qk_weights_bwd": [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp, _c_i32, _c_vp, _c_vp,
                          _c_vp, _c_vp],
    "tc_rope_apply": [_c_i32, _c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp, _c_vp, _c_vp, _c_i32,
                      _c_i32, ctypes.POINTER(Schedule), _c_vp, _c_i32, _c_vp],
    "tc_attn_fwd": [ctypes.POINTER(AttnArgs), ctypes.POINTER(Schedule), _c_vp],
    "tc_attn_bwd": [ctypes.POINTER(AttnArgs), ctypes.POINTER(Schedule), _c_vp],
    "tc_attn_bwd_noalloc": [ctypes.POINTER(AttnArgs), ctypes.POINTER(Schedule), _c_vp],
    "tc_selftest_wait_timeout": [_c_vp, _c_vp],
    "tc_sink_fwd": [_c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp, _c_i32, _c_vp, _c_vp, _c_vp],
    "tc_sink_bwd": [_c_i64, _c_i32, _c_i32, _c_i32, _c_vp, _c_vp, _c_i32, _c_vp, _c_vp, _c_vp,
                    _c_vp, _c_vp, _c_vp],
    "tc_gate_apply": [_c_i64, _c_i32, _c_vp, _c_i32, _c_vp, _c_i32, _c_vp, _c_vp],
    "tc_decode_step": [ctypes.POINTER(DecodeArgs), _c_vp],
    "tc_decode_init": [ctypes.POINTER(DecodeInitArgs), _c_vp],
}

_LIB = None


def lib():
    """Load the library once.  Raises (no fallback) when it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"telescope_cache_b200: CUDA library {LIB_PATH} is missing; build it with "
                "`python -m telescope_cache_b200.build_lib` (no CPU fallback exists)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        handle.tc_launch_count.argtypes = []
        handle.tc_launch_count.restype = ctypes.c_int64
        handle.tc_tree_bwd_scratch_bytes.restype = ctypes.c_int64
        handle.tc_linear_wgrad_scratch_floats.restype = ctypes.c_int64
        handle.tc_linear_scratch_floats.restype = ctypes.c_int64
        _LIB = handle
    return _LIB


_ERRORS = {
    TC_ERR_ARG: ValueError,
    TC_ERR_UNSUPPORTED: NotImplementedError,
    TC_ERR_CUDA: RuntimeError,
    TC_ERR_SCHEDULE: ValueError,
}


def launch_count():
    """CUDA kernels launched by the library so far (tc_launch_count)."""
    return int(lib().tc_launch_count())


def check(rc, what):
    if rc != TC_OK:
        exc = _ERRORS.get(rc, RuntimeError)
        raise exc(f"telescope_cache_b200: {what} failed with status {rc}")


def launch(name, device, *args):
    """Call the entry point `name` with `device` current, so that its kernels
    launch on the device that owns the tensors and their stream whatever device
    the caller has current (the caller's current device is restored).  Raises
    on a nonzero status."""
    fn = getattr(lib(), name)
    if device is not None and device.type == "cuda" and device.index != torch.cuda.current_device():
        with torch.cuda.device(device):
            rc = fn(*args)
    else:
        rc = fn(*args)
    check(rc, name)


def dtype_code(dt):
    if dt == torch.float32:
        return TC_F32
    if dt == torch.bfloat16:
        return TC_BF16
    if dt == torch.float16:
        return TC_F16
    raise TypeError(f"telescope_cache_b200: unsupported dtype {dt}")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    """The product path runs on CUDA tensors only."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "telescope_cache_b200 computes on CUDA tensors only (got a tensor on "
                f"{t.device}); there is no CPU fallback")
