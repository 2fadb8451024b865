"""Test infrastructure only: ctypes bindings to the CPU checkers.

* ``liboracle.so`` -- the scalar C restatement of the reference's INT8 hot
  path (oracle.c), built by ``make -C oracle``.
* ``_ref/libqwen_ref.so`` -- the reference engine's own CPU operators,
  compiled from its unmodified sources by ``make -C oracle ref`` (only where
  the reference sources are present; the built file travels with the repo).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module.  The product library never links or calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqwen_ref.so")
REF_MODEL_SO = os.path.join(HERE, "_ref", "libqwen_ref_model.so")
# the same decoder with the product's linear() shim linked in place of the reference's
REF_B200_SO = os.path.join(HERE, "_ref", "libqwen_ref_b200.so")


def _reference_dir():
    """Where the reference sources are: $QVL_REFERENCE_DIR, else the
    `reference_path` that BASELINE.json at the repository root names (absent
    on machines without the sources; the built library then travels)."""
    d = os.environ.get("QVL_REFERENCE_DIR")
    if d:
        return d
    try:
        import json
        with open(os.path.join(HERE, "..", "BASELINE.json")) as f:
            return json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        return ""


REF_SRC = _reference_dir()

LANE8_DISPATCH, LANE8, TILED = 0, 1, 2

_P = ctypes.c_void_p
_Z = ctypes.c_size_t
_I = ctypes.c_int


def build(ref: bool = True) -> None:
    """Compile the restatement, and the reference library when its sources exist."""
    subprocess.run(["make", "-C", HERE, "-s", "all"], check=True)
    if ref and REF_SRC and os.path.isdir(REF_SRC):
        subprocess.run(["make", "-C", HERE, "-s", "-j8", "ref", f"REF={REF_SRC}"], check=True)


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data


_orc = None
_ref = None


def lib():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_quantize_row.argtypes = [_P, _Z, _Z, _P, _P]
        L.orc_linear_i8.argtypes = [_P, _P, _P, _P, _Z, _Z, _Z, _Z, _I]
        L.orc_group_sums.argtypes = [_P, _P, _P, _Z, _Z, _Z, _Z]
        L.orc_swiglu.argtypes = [_P, _P, _Z]
        L.orc_expf.argtypes = [_P, _P, _Z]
        L.orc_exp_ref.argtypes = [ctypes.c_float]
        L.orc_exp_ref.restype = ctypes.c_float
        L.orc_softmax.argtypes = [_P, _Z]
        L.orc_rope_inplace.argtypes = [_P, _P, _P, _I, _I]
        L.orc_attention.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _Z, _I]
        L.orc_argmax.argtypes = [_P, _Z]
        L.orc_argmax.restype = _I
        L.orc_rope_table.argtypes = [_P, _P, _Z, _I, ctypes.c_float]
        L.orc_rms_norm_i8.argtypes = [_P, _P, _P, _P, _Z, _Z, ctypes.c_float, _Z, _I]
        L.orc_embedding_i8.argtypes = [_P, _P, _P, _Z, _Z]
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_SO)
        L.ref_i8_kernel.argtypes = [_P, _P, _P, _P, _Z, _Z, _Z, _Z]
        L.ref_linear_i8.argtypes = [_P, _P, _P, _P, _Z, _Z, _Z, _I, _Z]
        L.ref_swiglu.argtypes = [_P, _P, _Z]
        L.ref_softmax.argtypes = [_P, _Z]
        L.ref_apply_rotary.argtypes = [_P, _P, _P, _Z, _I, _I, _I]
        L.ref_apply_rotary_cache.argtypes = [_P, _P, _P, _P, _Z, _I, _I, _I, _Z]
        L.ref_attention.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _Z, _I]
        L.ref_rms_norm_i8.argtypes = [_P, _P, _P, _P, _Z, _Z, ctypes.c_float, _Z]
        L.ref_rms_norm_inplace_i8.argtypes = [_P, _P, _P, _Z, _Z, ctypes.c_float, _Z]
        L.ref_embedding_i8.argtypes = [_P, _P, _P, _Z, _Z, _Z]
        _ref = L
    return _ref


class RefModel:
    """The reference's own text decoder end to end (oracle/ref_model.cpp):
    init_model_weights on a .bin model file, qwen_rope_precompute, and
    forward_text per token; per-row INT8 through the reference's INT8 kernel
    with group = K, and (fp16_kv) the new KV rows rounded to fp16 values as
    an FP16 cache holds them.  One model per library at a time.

    dropin=True loads the build whose linear() is the product's host shim
    (host/linear_shim.cpp): the reference's forward_text with every INT8
    product on the GPU."""

    _libs: dict = {}

    def __init__(self, path: str, fp16_kv: bool = True, dropin: bool = False):
        so = REF_B200_SO if dropin else REF_MODEL_SO
        if so not in RefModel._libs:
            L = ctypes.CDLL(so)
            L.refm_load.argtypes = [ctypes.c_char_p, _I]
            L.refm_load.restype = _I
            L.refm_config.argtypes = [_P]
            L.refm_forward.argtypes = [_I, _I]
            L.refm_forward.restype = ctypes.POINTER(ctypes.c_float)
            L.refm_rope.argtypes = [_P, _P, _I]
            L.refm_kv.argtypes = [_I]
            L.refm_kv.restype = ctypes.POINTER(ctypes.c_float)
            L.refm_free.argtypes = []
            L.refm_forward_img.argtypes = [_P, _I, _I, _I, _P, _P]
            L.refm_forward_img.restype = _I
            L.refm_set_vision.argtypes = [_P, _P, _I]
            RefModel._libs[so] = L
        L = self._lib = RefModel._libs[so]
        if L.refm_load(path.encode(), int(fp16_kv)) != 0:
            raise RuntimeError(f"reference loader failed on {path} (or a model is already loaded)")
        c = np.zeros(12, np.int32)
        L.refm_config(c.ctypes.data)
        self.vocab, self.hidden, self.inter, self.layers, self.heads, self.kv_heads, self.seq_len = map(int, c[:7])
        self.rope_theta, self.group_size, self.group_quantized = int(c[7]), int(c[9]), int(c[10])
        self.eps = float(c[11:12].view(np.float32)[0])
        self.head_dim = self.hidden // self.heads
        n = self.layers * self.kv_heads * self.seq_len * self.head_dim
        shape = (self.layers, self.kv_heads, self.seq_len, self.head_dim)
        self.k_cache = np.ctypeslib.as_array(L.refm_kv(0), shape=(n,)).reshape(shape)
        self.v_cache = np.ctypeslib.as_array(L.refm_kv(1), shape=(n,)).reshape(shape)

    def rope(self, rows: int):
        half = self.head_dim // 2
        c = np.empty((rows, half), np.float32)
        s = np.empty((rows, half), np.float32)
        self._lib.refm_rope(c.ctypes.data, s.ctypes.data, rows)
        return c, s

    def forward(self, token: int, pos: int) -> np.ndarray:
        """forward_text: the logits (a copy) for `token` at `pos`."""
        p = self._lib.refm_forward(int(token), int(pos))
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def forward_img(self, patches: np.ndarray, grid_h: int, grid_w: int, out_hidden: int = 2048):
        """forward_img on preprocessed patches [T, C*2*P*P]: (image embeddings
        [T/4, out_hidden] fp32, deep-stack rows [3, T/4, hidden] as float)."""
        patches = np.ascontiguousarray(patches, dtype=np.float32)
        T = patches.shape[0]
        d = T // 4
        x = np.zeros((d, out_hidden), np.float32)
        deep = np.zeros((3, d, self.hidden), np.float32)
        r = self._lib.refm_forward_img(patches.ctypes.data, T, grid_h, grid_w, x.ctypes.data, deep.ctypes.data)
        if r != d:
            raise RuntimeError("forward_img failed")
        return x, deep

    def set_vision(self, x: np.ndarray, deep: np.ndarray):
        """Image embeddings [n, out_hidden] and deep-stack rows [3, n, hidden]
        for the image tokens of the next prompt (in place of forward_img's)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        deep = np.ascontiguousarray(deep, dtype=np.float32)
        self._lib.refm_set_vision(x.ctypes.data, deep.ctypes.data, x.shape[0])

    def close(self):
        self._lib.refm_free()


def ref_model_available() -> bool:
    return os.path.exists(REF_MODEL_SO)


# ---------------------------------------------------------------- restatement
def quantize(x: np.ndarray, g: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    q = np.empty((M, K), np.int16)
    s = np.empty((M, K // g), np.float32)
    for i in range(M):
        lib().orc_quantize_row(x[i].ctypes.data, K, g, q[i].ctypes.data, s[i].ctypes.data)
    return q, s


def linear_i8(x, w, ws, g, mode=LANE8_DISPATCH, threads=1):
    """y = x . dequant(w)^T in the reference's order.  With an explicit mode
    (LANE8 or TILED) every output row depends on its own input row only, so
    `threads` > 1 splits the rows over host threads (ctypes drops the GIL)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    if threads > 1 and mode != LANE8_DISPATCH and M > 1:
        from concurrent.futures import ThreadPoolExecutor
        bounds = np.linspace(0, M, min(threads, M) + 1).astype(int)

        def part(i):
            a, b = bounds[i], bounds[i + 1]
            if b > a:
                lib().orc_linear_i8(x[a:b].ctypes.data, _ptr(w), _ptr(ws), y[a:b].ctypes.data, b - a, N, K, g, mode)
        with ThreadPoolExecutor(len(bounds) - 1) as ex:
            list(ex.map(part, range(len(bounds) - 1)))
        return y
    lib().orc_linear_i8(_ptr(x), _ptr(w), _ptr(ws), _ptr(y), M, N, K, g, mode)
    return y


def group_sums(q, w, g):
    M, K = q.shape
    N = w.shape[0]
    out = np.empty((M, N, K // g), np.int32)
    lib().orc_group_sums(_ptr(q), _ptr(w), _ptr(out), M, N, K, g)
    return out


def swiglu(gate, up):
    g = np.array(gate, dtype=np.float32, copy=True, order="C")
    u = np.ascontiguousarray(up, dtype=np.float32)
    lib().orc_swiglu(_ptr(g), _ptr(u), g.size)
    return g


def expf(x, threads=1):
    """The host C library's expf, elementwise (rows split over threads)."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    y = np.empty_like(x)
    if threads <= 1:
        lib().orc_expf(_ptr(x), _ptr(y), x.size)
        return y
    from concurrent.futures import ThreadPoolExecutor
    b = np.linspace(0, x.size, threads + 1).astype(np.int64)
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda i: lib().orc_expf(x[b[i]:].ctypes.data, y[b[i]:].ctypes.data, int(b[i + 1] - b[i])),
                    range(threads)))
    return y


def softmax(x):
    v = np.array(x, dtype=np.float32, copy=True)
    lib().orc_softmax(_ptr(v), v.size)
    return v


def exp_ref(x: float) -> float:
    return lib().orc_exp_ref(x)


def rope_inplace(x, cos_row, sin_row):
    """x: [n_heads, D] fp32, rotated in place (returns x)."""
    n, D = x.shape
    lib().orc_rope_inplace(_ptr(x), _ptr(cos_row), _ptr(sin_row), n, D)
    return x


def attention(key_cache, value_cache, q, pos):
    """key/value_cache: [NKV, S, D] fp32; q: [NH, D] (already rotated)."""
    NKV, S, D = key_cache.shape
    NH = q.shape[0]
    att = np.zeros((NH, S), np.float32)
    out = np.empty((NH, D), np.float32)
    lib().orc_attention(_ptr(key_cache), _ptr(value_cache), _ptr(q), _ptr(att), _ptr(out),
                        NH, NKV, D, S, pos)
    return out


def argmax(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().orc_argmax(_ptr(x), x.size))


def rope_table(S: int, D: int = 128, theta: float = 5e6):
    c = np.empty((S, D // 2), np.float32)
    s = np.empty((S, D // 2), np.float32)
    lib().orc_rope_table(_ptr(c), _ptr(s), S, D, theta)
    return c, s


def rms_norm_i8(x, wq, ws, group_size, eps, inplace=False):
    """x fp32 [batches, hidden] -> normalised copy (reference rms_norm /
    rms_norm_inplace arithmetic)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    B, H = x.shape
    out = np.empty_like(x)
    lib().orc_rms_norm_i8(_ptr(x), _ptr(wq), _ptr(ws), _ptr(out), H, group_size, eps, B, int(inplace))
    return out


def embedding_i8(table, scales, token):
    H = table.shape[1]
    out = np.empty(H, np.float32)
    lib().orc_embedding_i8(_ptr(table), _ptr(scales), _ptr(out), H, int(token))
    return out


# -------------------------------------------------------- compiled reference
def ref_rms_norm_i8(x, wq, ws, group_size, eps, inplace=False):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    B, H = x.shape
    if inplace:
        ref_lib().ref_rms_norm_inplace_i8(_ptr(x), _ptr(wq), _ptr(ws), H, group_size, eps, B)
        return x
    out = np.zeros_like(x)
    ref_lib().ref_rms_norm_i8(_ptr(x), _ptr(wq), _ptr(ws), _ptr(out), H, group_size, eps, B)
    return out


def ref_embedding_i8(table, scales, token):
    V, H = table.shape
    out = np.zeros(H, np.float32)
    ref_lib().ref_embedding_i8(_ptr(table), _ptr(scales), _ptr(out), V, H, int(token))
    return out

def ref_i8_kernel(x, w, ws, g):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    ref_lib().ref_i8_kernel(_ptr(x), _ptr(w), _ptr(ws), _ptr(y), M, N, K, g)
    return y


def ref_linear(x, w, ws, group_quantized, g):
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    ref_lib().ref_linear_i8(_ptr(x), _ptr(w), _ptr(ws), _ptr(y), M, N, K, int(group_quantized), g)
    return y


def ref_swiglu(gate, up):
    g = np.array(gate, dtype=np.float32, copy=True, order="C")
    u = np.ascontiguousarray(up, dtype=np.float32)
    ref_lib().ref_swiglu(_ptr(g), _ptr(u), g.size)
    return g


def ref_softmax(x):
    v = np.array(x, dtype=np.float32, copy=True)
    ref_lib().ref_softmax(_ptr(v), v.size)
    return v


def ref_rope(x, cos_tab, sin_tab, pos):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    n, D = x.shape
    ref_lib().ref_apply_rotary(_ptr(x), _ptr(cos_tab), _ptr(sin_tab), cos_tab.shape[0], n, D, pos)
    return x


def ref_attention(key_cache, value_cache, q, pos):
    NKV, S, D = key_cache.shape
    NH = q.shape[0]
    att = np.zeros((NH, S), np.float32)
    out = np.zeros((NH, D), np.float32)
    ref_lib().ref_attention(_ptr(key_cache), _ptr(value_cache), _ptr(q), _ptr(att), _ptr(out),
                            NH, NKV, D, S, pos)
    return out
