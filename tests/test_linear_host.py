"""Host-side rules of the projection entry points (no GPU needed): the
scratch queries, argument checks before any launch."""

import ctypes

from telescope_cache_b200 import _lib


def test_split_k_scratch_only_for_few_rows_and_long_k():
    lib = _lib.lib()
    bf = _lib.TC_BF16
    # decode gate: 64 rows, N = K = 2048 -> split K, fp32 partial sums per part
    need = lib.tc_linear_scratch_floats(64, 2048, 2048, bf)
    assert need > 0 and need % (64 * 2048) == 0
    # many row blocks (the config-2 gate) or a short K (the band) -> no split
    assert lib.tc_linear_scratch_floats(16384, 2048, 2048, bf) == 0
    assert lib.tc_linear_scratch_floats(1 << 20, 2848, 16, bf) == 0
    assert lib.tc_linear_scratch_floats(64, 2048, 256, bf) == 0  # 4 K-blocks
    assert lib.tc_linear_scratch_floats(-1, 16, 16, bf) == -1


def test_wgrad_scratch_covers_partials_and_transpose():
    lib = _lib.lib()
    M, N1, N2 = 131072, 32, 2048
    need = lib.tc_linear_wgrad_scratch_floats(M, N1, N2)
    chunks = (M + 4095) // 4096
    # per-chunk partial tiles plus the 16-bit transposed A rows (two per float)
    assert need >= chunks * N1 * N2 + N1 * M // 2
    assert lib.tc_linear_wgrad_scratch_floats(0, 0, 16) == -1


def test_invalid_arguments_are_rejected_before_launch():
    lib = _lib.lib()
    null = ctypes.c_void_p(0)
    # null pointers / bad strides / bad epilogue -> TC_ERR_ARG, nothing launched
    rc = lib.tc_linear(4, 8, 8, _lib.TC_BF16, null, 8, _lib.TC_BF16, null, 8, _lib.TC_BF16, null, 8,
                       _lib.TC_LIN_STORE, null, 0, null, 0, null, null)
    assert rc == _lib.TC_ERR_ARG
    rc = lib.tc_linear(4, 8, 8, _lib.TC_BF16, ctypes.c_void_p(16), 4, _lib.TC_BF16, ctypes.c_void_p(16), 8,
                       _lib.TC_BF16, ctypes.c_void_p(16), 8, _lib.TC_LIN_STORE, null, 0, null, 0, null, null)
    assert rc == _lib.TC_ERR_ARG  # lda < K
    rc = lib.tc_linear(4, 8, 8, _lib.TC_BF16, ctypes.c_void_p(16), 8, _lib.TC_BF16, ctypes.c_void_p(16), 8,
                       _lib.TC_BF16, ctypes.c_void_p(16), 8, 7, null, 0, null, 0, null, null)
    assert rc == _lib.TC_ERR_ARG  # unknown epilogue
    rc = lib.tc_linear_wgrad(4, 8, 8, _lib.TC_BF16, null, 8, _lib.TC_BF16, null, 8, _lib.TC_F32, null, 8,
                             null, 0, null, null)
    assert rc == _lib.TC_ERR_ARG
