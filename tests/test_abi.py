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
    return sorted(set(re.findall(r"^\s*int\s+(tc_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert lib.tc_version() == 1
    assert hasattr(lib, "tc_launch_count") and _lib.launch_count() >= 0


def test_struct_sizes_match_header():
    # tc_schedule: 4 int32 + 2 * 16 int32 + 17 int64
    assert ctypes.sizeof(_lib.Schedule) == 4 * 4 + 2 * 16 * 4 + 17 * 8


def test_bad_arguments_return_status_codes():
    lib = _lib.lib()
    assert lib.tc_schedule_init(None, 2, 6, 8, None) == _lib.TC_ERR_ARG
    vals = (ctypes.c_int32 * 1)(3)  # a[1] = 4: wrong phase
    s = _lib.Schedule()
    assert lib.tc_schedule_init(ctypes.cast(vals, ctypes.c_void_p), 1, 6, 8, ctypes.byref(s)) == \
        _lib.TC_ERR_SCHEDULE
    assert lib.tc_attn_fwd(None, None, None) == _lib.TC_ERR_ARG
    assert lib.tc_build_tree(None, None) == _lib.TC_ERR_ARG
    assert lib.tc_decode_step(None, None) == _lib.TC_ERR_ARG
