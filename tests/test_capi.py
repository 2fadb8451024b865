"""CPU-side checks of the product library: it loads and exports every symbol
include/qvl_b200.h declares, and argument validation needs no GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT, import_qvl

HEADER = os.path.join(ROOT, "include", "qvl_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qvl_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    assert "qvl_linear_i8" in names and "qvl_attention_decode" in names


def test_library_exports_every_declared_symbol():
    qvl = import_qvl()
    L = qvl.load_library()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert set(qvl.EXPORTED) <= set(declared_functions())


def test_status_strings_and_validation_without_gpu():
    qvl = import_qvl()
    L = qvl.load_library()
    assert L.qvl_status_string(0) == b"ok"
    assert L.qvl_version().startswith(b"qvl_b200")
    # null pointers and bad shapes are rejected before any CUDA call
    assert L.qvl_linear_i8(None, None, None, None, 1, 1, 16, 1, 16, 0, None, 0, None) == 1
    assert L.qvl_quantize_rows(None, None, None, 1, 16, 16, None) == 1
    assert L.qvl_linear_i8_workspace_bytes(4, 2048, 128) == 4 * 2048 * 2 + 256
    d = qvl.AttnDims(16, 8, 64, 64, 4, 256)   # head_dim 64 is not implemented
    assert L.qvl_attention_workspace_bytes(1, 256, ctypes.byref(d)) == 0
    assert L.qvl_argmax_rows(None, None, 1, 1, None) == 1


def test_unsupported_group_size_is_reported():
    qvl = import_qvl()
    L = qvl.load_library()
    fake = ctypes.c_void_p(256)   # never dereferenced: shape check fails first
    rc = L.qvl_linear_q16_i8(fake, fake, fake, fake, fake, 1, 16, 96 * 3, 96, 0, None)
    assert rc == 2


def test_text_decode_step_validation_without_gpu():
    """qvl_text_decode_step rejects bad arguments before any CUDA call."""
    qvl = import_qvl()
    L = qvl.load_library()
    fake = 4096                      # aligned, never dereferenced
    w = qvl.TextWeightsC()
    for name, _ in qvl.TextWeightsC._fields_[:26]:
        setattr(w, name, fake)
    w.layers, w.vocab, w.hidden, w.intermediate = 2, 4096, 2048, 6144
    w.heads, w.kv_heads, w.head_dim, w.norm_group, w.eps = 16, 8, 128, 128, 1e-6
    ws_bytes = L.qvl_text_decode_workspace_bytes()
    assert ws_bytes > 0

    def call(max_ctx=64, ws=fake, nbytes=ws_bytes, stride=8192, weights=w):
        return L.qvl_text_decode_step(ctypes.byref(weights), fake, fake, fake, fake, fake, fake, stride, fake, 64,
                                      fake, fake, max_ctx, ws, nbytes, None)

    assert call(max_ctx=8193) == 2            # context above 16 slices x 512
    assert call(nbytes=ws_bytes - 1) == 4     # workspace too small
    assert call(ws=fake + 16) == 4            # workspace not 256-byte aligned
    assert call(stride=12) == 1               # layer stride breaks 16-byte KV rows
    w.intermediate = 4096
    assert call() == 2                        # other model dims are not compiled in
    w.intermediate = 6144
    w.w_q = None
    assert call() == 1
    assert L.qvl_text_decode_step(None, *([None] * 6), 0, None, 0, None, None, 0, None, 0, None) == 1
