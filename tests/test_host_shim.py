"""The C++ drop-in `linear()` (qwen3-vl-2b-inference_b200/host/linear_shim.cpp):
the reference's signature over host buffers, backed by the C ABI.  Compared
with the reference's own compiled `linear()` on the same host buffers."""
import ctypes
import os

import numpy as np
import pytest

import oracle
from conftest import PKG_DIR, make_linear_inputs

SHIM = os.path.join(PKG_DIR, "lib", "libqvl_b200_linear_shim.so")


def _shim():
    L = ctypes.CDLL(SHIM)
    P, Z = ctypes.c_void_p, ctypes.c_size_t
    L.qvl_shim_linear_i8.argtypes = [P, P, P, P, Z, Z, Z, ctypes.c_int, Z]
    L.qvl_shim_release_weights.argtypes = []
    return L


def test_shim_library_exports_linear():
    L = _shim()
    assert hasattr(L, "qvl_shim_linear_i8")
    assert hasattr(L, "_ZN8qvl_shim6linearEPKvS1_S1_S1_S1_PvmmmbNS_5DType4TypeES4_S4_S4_bm")


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,gq,g", [(1, 2048, 2048, 1, 128), (1, 6144, 2048, 1, 128), (4, 512, 1024, 1, 64),
                                        (1, 1024, 2048, 0, 0)])
def test_shim_matches_reference_linear(cuda, M, N, K, gq, g):
    L = _shim()
    x, w, ws = make_linear_inputs(M + N + g, M, N, K, g if gq else K)
    y = np.zeros((M, N), np.float32)
    for _ in range(2):   # second call reuses the uploaded weights
        L.qvl_shim_linear_i8(x.ctypes.data, w.ctypes.data, ws.ctypes.data, y.ctypes.data, M, N, K, gq, g)
        if gq:
            ref = oracle.ref_linear(x, w, ws, True, g) if oracle.ref_available() else oracle.linear_i8(x, w, ws, g)
        else:
            # per-row scales: the reference's own row-quant branch reads B as [K, N]
            # (cpu_wrapper.cpp:172-215); the intended product is its kernel with g = K
            ref = oracle.ref_i8_kernel(x, w, ws, K) if oracle.ref_available() else oracle.linear_i8(x, w, ws, K)
        np.testing.assert_array_equal(y, ref)
    # the host weights go away with this test: drop their device copies
    L.qvl_shim_release_weights()
