"""The C-ABI library builds, loads without a GPU, and exports every entry point include/geoattn.h declares."""
import ctypes
import os
import re

import pytest

from foreswe_gpu_optimization_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "geoattn.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(geoattn_[a-z_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    build.build()
    return _lib.lib()


def test_header_declares_the_binding_surface():
    assert set(declared()) == set(_lib.EXPORTED)


def test_every_declared_symbol_is_exported(L):
    for name in declared():
        assert hasattr(L, name), name


def test_version_and_error_strings(L):
    assert L.geoattn_version() == 2
    unknown = L.geoattn_error_string(99)
    assert b"unknown" in unknown
    msgs = [L.geoattn_error_string(code) for code in range(8)]  # GEOATTN_OK .. GEOATTN_ERR_SCRATCH
    assert all(msgs) and unknown not in msgs and len(set(msgs)) == 8
    assert b"other-device" in msgs[1]


def test_size_queries_without_gpu(L):
    sh = _lib.Shape(32, 8, 512, 64, _lib.DTYPE_BF16, 1)
    assert L.geoattn_prior_bytes(ctypes.byref(sh)) == 2 * 512 * 512 * 4
    assert L.geoattn_stats_bytes(ctypes.byref(sh)) == 3 * 32 * 8 * 512 * 4
    assert L.geoattn_bwd_workspace_bytes(ctypes.byref(sh)) > 32 * 8 * 512 * 16   # 4 float row records per row
    bad = _lib.Shape(1, 1, 16, 256, _lib.DTYPE_BF16, 0)
    assert L.geoattn_prior_bytes(ctypes.byref(bad)) == 0
    # fp32 head_dim 128: status word, hi/lo planes of q and k ([2][N][DP]), transposed v ([DP][N padded to 128])
    fp = _lib.Shape(1, 1, 16, 128, _lib.DTYPE_FP32, 0)
    assert L.geoattn_fwd_workspace_bytes(ctypes.byref(fp)) == 256 + 2 * (2 * 16 * 128 * 4) + 128 * 128 * 4
    for dtype in (_lib.DTYPE_FP32, _lib.DTYPE_BF16):  # head_dim above 192 has no kernel
        assert L.geoattn_fwd_workspace_bytes(ctypes.byref(_lib.Shape(1, 1, 16, 200, dtype, 0))) == 0
    # fp32 backward (N = 16: N_pad 128, one row block): status word, row records (4 floats per row; 5 above head dim
    # 64, where b = sum P2 P1 joins them), partials, hi/lo planes of q, k, v, dO, transposed hi planes of k, q, dO,
    # each rounded up to 256 bytes, and the fp32 dS scratch (N_pad^2 per b*h) for the dQ GEMM
    f64 = _lib.Shape(1, 1, 16, 64, _lib.DTYPE_FP32, 0)
    assert L.geoattn_bwd_workspace_bytes(ctypes.byref(f64)) == (256 + 128 * 16 + 256 + 4 * (2 * 16 * 64 * 4)
                                                                + 3 * (64 * 128 * 4) + 128 * 128 * 4)
    f128 = _lib.Shape(1, 1, 16, 128, _lib.DTYPE_FP32, 0)
    assert L.geoattn_bwd_workspace_bytes(ctypes.byref(f128)) == (256 + 128 * 20 + 256 + 4 * (2 * 16 * 128 * 4)
                                                                 + 3 * (128 * 128 * 4) + 128 * 128 * 4)


def test_invalid_arguments_rejected_before_any_launch(L):
    sh = _lib.Shape(1, 1, 16, 64, _lib.DTYPE_BF16, 0)
    assert L.geoattn_fwd(None, None) == 1
    args = _lib.FwdArgs()
    args.shape = sh
    assert L.geoattn_fwd(ctypes.byref(args), None) == 1          # null pointers
    args.shape = _lib.Shape(1, 1, 16, 300, _lib.DTYPE_BF16, 0)
    assert L.geoattn_fwd(ctypes.byref(args), None) == 2          # head_dim without a kernel
    assert L.geoattn_prior_from_dense(ctypes.byref(sh), None, 16, None, 16, None, None) == 1
