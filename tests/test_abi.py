"""The C-ABI library loads on a machine without a GPU and exports exactly the
functions ``include/telescope_cache.h`` declares (no compute calls)."""

import ctypes
import os
import re

from telescope_cache_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "telescope_cache.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t)\s+(tc_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    # tc_launch_count (no arguments, int64 result) is bound outside SIGNATURES
    assert set(names) - {"tc_launch_count"} == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert lib.tc_version() == 1
    assert hasattr(lib, "tc_launch_count") and _lib.launch_count() >= 0


def test_struct_sizes_match_header():
    # tc_schedule: 4 int32 + 2 * 16 int32 + 17 int64
    assert ctypes.sizeof(_lib.Schedule) == 4 * 4 + 2 * 16 * 4 + 17 * 8
    # tc_decode_init_args: 7 int32, caps, ring_off, lo, hi; 3 x 16 level pointers,
    # 6 x 16 int64 strides, 3 ring pointers
    assert ctypes.sizeof(_lib.DecodeInitArgs) == 7 * 4 + 16 * 4 + 17 * 4 + 2 * 16 * 4 + 3 * 16 * 8 + \
        6 * 16 * 8 + 3 * 8
    assert _lib.DecodeInitArgs.ring_k.offset == 1440


def test_bad_arguments_return_status_codes():
    lib = _lib.lib()
    assert lib.tc_schedule_init(None, 2, 6, 8, None) == _lib.TC_ERR_ARG
    # no ring pointers: rejected before any launch
    assert lib.tc_decode_init(ctypes.byref(_lib.DecodeInitArgs()), None) == _lib.TC_ERR_ARG
    vals = (ctypes.c_int32 * 1)(3)  # a[1] = 4: wrong phase
    s = _lib.Schedule()
    assert lib.tc_schedule_init(ctypes.cast(vals, ctypes.c_void_p), 1, 6, 8, ctypes.byref(s)) == \
        _lib.TC_ERR_SCHEDULE
    assert lib.tc_attn_fwd(None, None, None) == _lib.TC_ERR_ARG
    assert lib.tc_build_tree(None, None) == _lib.TC_ERR_ARG
    assert lib.tc_decode_step(None, None) == _lib.TC_ERR_ARG
    assert lib.tc_build_tree_bwd(None, None) == _lib.TC_ERR_ARG
    assert lib.tc_tree_bwd_scratch_bytes(None) == -1


def test_tree_bwd_scratch_plan():
    """Scratch holds fp32 copies of levels 6..L (the levels above the 64-leaf
    tiles), each region rounded up to 256 bytes; none when L <= 6."""
    lib = _lib.lib()
    B, N, H, D = 2, 4096, 3, 64

    def args(L):
        total = sum(N >> l for l in range(L + 1))
        return _lib.TreeBwdArgs(B=B, N=N, Hq=H, Hkv=H, Dk=D, Dv=D, num_summary_levels=L, dtype=_lib.TC_BF16,
                                w_dtype=_lib.TC_F32, k_packed=16, v_packed=16, w_packed=16, dk0=16, dv0=16,
                                d0_dtype=_lib.TC_BF16, total=total)

    assert lib.tc_tree_bwd_scratch_bytes(ctypes.byref(args(6))) == 0
    rows = B * sum(N >> l for l in range(6, 9)) * H
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    assert lib.tc_tree_bwd_scratch_bytes(ctypes.byref(args(8))) == 2 * up(rows * D * 4) + up(rows * 4)
    bad = args(8)
    bad.total += 1
    assert lib.tc_tree_bwd_scratch_bytes(ctypes.byref(bad)) == -1
