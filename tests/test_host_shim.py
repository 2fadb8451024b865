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
    # the reference's own mangled name of linear() (its global `linear` with
    # `struct DType`), so reference objects bind to it at link time
    assert hasattr(L, "_Z6linearPKvS0_S0_S0_S0_PvmmmbN5DType4TypeES3_S3_S3_bm")


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


def _ref_object_symbol(name):
    """Mangled names the reference's compiled forward_text object references."""
    import subprocess
    obj = os.path.join(os.path.dirname(oracle.REF_SO), "obj", "model", "src", "forward.o")
    if not os.path.exists(obj):
        pytest.skip("reference objects not built")
    out = subprocess.run(["nm", "-u", obj], capture_output=True, text=True, check=True).stdout
    return name in out


def test_reference_call_sites_bind_to_the_shim_symbol():
    """The reference's forward_text object calls exactly the symbol the shim
    defines."""
    assert _ref_object_symbol("_Z6linearPKvS0_S0_S0_S0_PvmmmbN5DType4TypeES3_S3_S3_bm")


@pytest.mark.gpu
def test_reference_forward_text_on_the_shim(qvl, cuda, tmp_path):
    """The reference's own decoder (loader, forward_text, classifier_gemm)
    linked with the shim in place of its linear(): every INT8 product runs on
    the B200 kernels and the logits equal the reference's CPU build (per-row
    products through its own kernel with group K) bit for bit."""
    import qvl_b200.modelfile as MF
    if not (os.path.exists(oracle.REF_B200_SO) and oracle.ref_model_available()):
        pytest.skip("reference model libraries not built")
    hdr = MF.qwen3vl_2b_header(num_hidden_layers=2, vision_hidden_size=32, vision_intermediate_size=64,
                               vision_num_heads=2)
    p = str(tmp_path / "m.bin")
    MF.write_model_bin(p, hdr, MF.synthetic_text(hdr, seed=9))
    gpu = oracle.RefModel(p, fp16_kv=False, dropin=True)
    cpu = oracle.RefModel(p, fp16_kv=False)
    try:
        tok = 99
        for pos in range(6):
            a = gpu.forward(tok, pos)
            b = cpu.forward(tok, pos)
            np.testing.assert_array_equal(a, b, err_msg=f"pos {pos}")
            tok = oracle.argmax(b)
    finally:
        gpu.close()
        cpu.close()
