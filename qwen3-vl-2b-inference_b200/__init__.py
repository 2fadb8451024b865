"""Host-side mirror of the reference engine's INT8 hot-path operators, running
on the sm_100a kernels of ``lib/libqvl_b200.so`` through its C ABI
(include/qvl_b200.h).

The operator names and argument meanings follow the reference
(dangtruong-github/qwen3-vl-2b-inference):

=====================  ==========================================================
this module            reference
=====================  ==========================================================
``linear``             ``linear`` INT8 branch, matmul/src/cpu_wrapper.cpp:308-357
``quantize_rows``      activation prologue, cpu_f32a_i8f32sb_f32c_avx2.cpp:135-177
``swiglu``             ``swiglu``, layers/src/text_layer.cpp:420-434
``swiglu_mlp``         gate/up linear + swiglu + down linear, model/src/forward.cpp:621-654
``rope_kv_append``     ``apply_rotary`` + ``apply_rotary_cache`` + v copy,
                       layers/src/text_layer.cpp:712-824, model/src/forward.cpp:545-562
``attention``          ``attn_scores_all_heads`` + ``softmax`` +
                       ``attn_weighted_sum_all_heads``, layers/src/text_layer.cpp:436-710
``greedy_decode``      ``greedy_decode``, tokenizer/src/utils.cpp:34-44
=====================  ==========================================================

Tensors are torch CUDA tensors (torch supplies device memory and streams
only).  There is no CPU fallback: if the library is missing, importing this
module raises.  An unsupported combination raises ``QvlError`` (the
reference prints and calls ``exit(1)``, cpu_wrapper.cpp:394-395).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libqvl_b200.so")

SEM_REFERENCE, SEM_LANE8, SEM_TILED = 0, 1, 2
DTYPE_FP32, DTYPE_INT32, DTYPE_FP16, DTYPE_INT8, DTYPE_INT4 = 0, 1, 2, 3, 4

EXPORTED = (
    "qvl_status_string", "qvl_last_cuda_error", "qvl_version", "qvl_quantize_rows",
    "qvl_linear_i8_workspace_bytes", "qvl_linear_i8", "qvl_linear_q16_i8", "qvl_swiglu",
    "qvl_swiglu_mlp_workspace_bytes", "qvl_swiglu_mlp_i8", "qvl_rope_kv_append",
    "qvl_attention_workspace_bytes", "qvl_attention_decode", "qvl_argmax_rows",
    "qvl_qknorm_rope_kv_append", "qvl_rms_norm_i8", "qvl_embedding_lookup_i8",
    "qvl_swiglu_quantize_rows", "qvl_linear_q16_i8_multi", "qvl_gate_up_swiglu_q16_i8",
    "qvl_linear_q16_i8_tail", "qvl_linear_q16_i8_batched", "qvl_linear_q16_i8_batched_workspace_bytes",
    "qvl_attention_decode_q16", "qvl_text_decode_workspace_bytes", "qvl_text_decode_step",
    "qvl_text_decode_step_ex",
    "qvl_text_decode_abort_flag", "qvl_text_decode_trace", "qvl_tc_timeout_status",
    "qvl_attention_decode_static", "qvl_attention_ordered_workspace_bytes", "qvl_attention_decode_ordered",
    "qvl_rope_table", "qvl_quantize_rows_planes", "qvl_qknorm_rope_attention_decode_ordered", "qvl_rms_norm_i8_planes", "qvl_linear_planes_i8_batched",
)
SEM_ACCUMULATE = 0x100


class QvlError(RuntimeError):
    pass


class AttnDims(ctypes.Structure):
    _fields_ = [("num_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("page_size", ctypes.c_int),
                ("max_pages_per_seq", ctypes.c_int), ("max_pos", ctypes.c_int)]


class RowTail(ctypes.Structure):
    _fields_ = [("counter", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("norm_s", ctypes.c_void_p),
                ("norm_group", ctypes.c_size_t), ("eps", ctypes.c_float), ("inplace_form", ctypes.c_int),
                ("norm_out", ctypes.c_void_p), ("q", ctypes.c_void_p), ("q_scales", ctypes.c_void_p),
                ("quant_group", ctypes.c_size_t)]


class TextWeightsC(ctypes.Structure):
    """qvl_text_weights: stacked device pointers of the text decoder."""
    _fields_ = ([(n, ctypes.c_void_p) for n in (
        "w_q", "w_k", "w_v", "w_o", "w_gate", "w_up", "w_down", "s_q", "s_k", "s_v", "s_o", "s_gate", "s_up",
        "s_down", "in_norm", "post_norm", "q_norm", "k_norm", "in_norm_s", "post_norm_s", "q_norm_s",
        "k_norm_s", "final_norm", "final_norm_s", "embed", "embed_s")]
        + [(n, ctypes.c_int) for n in ("layers", "vocab", "hidden", "intermediate", "heads", "kv_heads",
                                       "head_dim", "norm_group")]
        + [("eps", ctypes.c_float)])


_P, _Z, _I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
_lib = None


def load_library(path: str = LIB_PATH):
    """Load libqvl_b200.so (build it with build.py); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"libqvl_b200.so not built ({path}); run `python {PKG_DIR}/build.py`")
    L = ctypes.CDLL(path)
    L.qvl_status_string.restype = ctypes.c_char_p
    L.qvl_status_string.argtypes = [_I]
    L.qvl_version.restype = ctypes.c_char_p
    L.qvl_quantize_rows.argtypes = [_P, _P, _P, _Z, _Z, _Z, _P]
    L.qvl_linear_i8_workspace_bytes.restype = _Z
    L.qvl_linear_i8_workspace_bytes.argtypes = [_Z, _Z, _Z]
    L.qvl_linear_i8.argtypes = [_P, _P, _P, _P, _Z, _Z, _Z, _I, _Z, _I, _P, _Z, _P]
    L.qvl_linear_q16_i8.argtypes = [_P, _P, _P, _P, _P, _Z, _Z, _Z, _Z, _I, _P]
    L.qvl_swiglu.argtypes = [_P, _P, _Z, _P]
    L.qvl_swiglu_mlp_workspace_bytes.restype = _Z
    L.qvl_swiglu_mlp_workspace_bytes.argtypes = [_Z, _Z, _Z, _Z]
    L.qvl_swiglu_mlp_i8.argtypes = [_P] * 8 + [_Z, _Z, _Z, _Z, _I, _P, _Z, _P]
    L.qvl_rope_kv_append.argtypes = [_P] * 8 + [_Z, _P, _P, ctypes.POINTER(AttnDims), _P]
    L.qvl_attention_workspace_bytes.restype = _Z
    L.qvl_attention_workspace_bytes.argtypes = [_Z, _I, ctypes.POINTER(AttnDims)]
    L.qvl_attention_decode.argtypes = [_P] * 6 + [_Z, _I, _P, ctypes.POINTER(AttnDims), _P, _Z, _P]
    L.qvl_attention_ordered_workspace_bytes.restype = _Z
    L.qvl_attention_ordered_workspace_bytes.argtypes = [_Z, _I, ctypes.POINTER(AttnDims)]
    L.qvl_attention_decode_ordered.argtypes = [_P] * 6 + [_Z, _I, _P, ctypes.POINTER(AttnDims), _P, _Z, _P]
    L.qvl_argmax_rows.argtypes = [_P, _P, _Z, _Z, _P]
    L.qvl_qknorm_rope_kv_append.argtypes = [_P] * 8 + [_Z, _P, _P, _P, _P, _P, _P, _Z, ctypes.c_float,
                                                       ctypes.POINTER(AttnDims), _P]
    L.qvl_rms_norm_i8.argtypes = [_P] * 6 + [_Z, _Z, _Z, ctypes.c_float, _I, _Z, _P]
    L.qvl_embedding_lookup_i8.argtypes = [_P] * 4 + [_Z, _Z, _Z, _P]
    L.qvl_swiglu_quantize_rows.argtypes = [_P] * 4 + [_Z, _Z, _Z, _P]
    L.qvl_gate_up_swiglu_q16_i8.argtypes = [_P] * 8 + [_Z, _Z, _Z, _Z, _I, _P]
    L.qvl_linear_q16_i8_tail.argtypes = [_P, _P, _Z, _P, _P, _P, _P, _Z, _Z, _Z, _I, _I,
                                         ctypes.POINTER(RowTail), _P]
    L.qvl_linear_q16_i8_batched_workspace_bytes.restype = _Z
    L.qvl_linear_q16_i8_batched_workspace_bytes.argtypes = [_Z, _Z]
    L.qvl_linear_q16_i8_batched.argtypes = [_P, _P, _Z, _P, _P, _P, _P, _Z, _Z, _I, _I, _P, _P, _Z, _P]
    L.qvl_attention_decode_q16.argtypes = [_P] * 6 + [_Z, _I, _P, _P, _P, _P, ctypes.POINTER(AttnDims), _P, _Z, _P]
    L.qvl_linear_q16_i8_multi.argtypes = [_P, _P, _Z, _P, _P, _P, _P, _Z, _Z, _Z, _I, _P]
    L.qvl_text_decode_workspace_bytes.restype = _Z
    L.qvl_text_decode_workspace_bytes.argtypes = []
    L.qvl_text_decode_step.argtypes = [ctypes.POINTER(TextWeightsC)] + [_P] * 6 + [ctypes.c_long, _P, _I, _P, _P,
                                                                                _I, _P, _Z, _P]
    L.qvl_text_decode_step_ex.argtypes = L.qvl_text_decode_step.argtypes[:-1] + [_I, _P]
    L.qvl_text_decode_abort_flag.restype = _P
    L.qvl_text_decode_abort_flag.argtypes = [_P]
    L.qvl_text_decode_trace.restype = _P
    L.qvl_text_decode_trace.argtypes = [_P]
    L.qvl_tc_timeout_status.argtypes = [ctypes.POINTER(_I), _I, _P]
    L.qvl_rope_table.argtypes = [_I, _I, _I, _P, _P]
    L.qvl_quantize_rows_planes.argtypes = [_P] * 5 + [_Z, _Z, _Z, _P]
    L.qvl_qknorm_rope_attention_decode_ordered.argtypes = ([_P] * 8 + [_Z, _I] + [_P] * 6 +
                                                           [_Z, ctypes.c_float, _P, _P, _P, _Z, _P])
    L.qvl_rms_norm_i8_planes.argtypes = [_P] * 8 + [_Z, _Z, _Z, ctypes.c_float, _I, _P]
    L.qvl_linear_planes_i8_batched.argtypes = [_P, _P, _P, _Z, _P, _P, _P, _P, _Z, _Z, _I, _P]
    L.qvl_internal_set_tc_timeout.argtypes = [_P]
    _lib = L
    return L


def _check(rc: int, what: str) -> None:
    if rc != 0:
        L = load_library()
        msg = L.qvl_status_string(rc).decode()
        cuda = L.qvl_last_cuda_error()
        raise QvlError(f"{what}: {msg} (status {rc}, last CUDA error {cuda})")


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise QvlError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise QvlError("expected a contiguous tensor")
    return t.data_ptr()


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Workspace:
    """Device scratch owned by the caller and reused across calls (the C ABI
    never allocates).  Grows on demand outside any timed or captured region."""

    def __init__(self, device=None):
        self.device = torch.device(device or "cuda")
        self.buf = torch.empty(0, dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        return self.buf


_default_ws: dict = {}


def _ws(ws, device):
    if ws is not None:
        return ws
    key = torch.device(device).index
    if key not in _default_ws:
        _default_ws[key] = Workspace(device)
    return _default_ws[key]


# --------------------------------------------------------------------------- ops
def quantize_rows(x: torch.Tensor, group_size: int, stream=None):
    """fp32 [M,K] -> (int16 [M,K], fp32 [M,K/g]); the reference's activation prologue."""
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int16, device=x.device)
    s = torch.empty((M, K // group_size), dtype=torch.float32, device=x.device)
    _check(load_library().qvl_quantize_rows(_ptr(x), _ptr(q), _ptr(s), M, K, group_size,
                                            _stream(stream)), "quantize_rows")
    return q, s


def linear(A: torch.Tensor, B: torch.Tensor, B_scale: torch.Tensor, C: torch.Tensor | None = None,
           group_quantized: bool = True, group_size: int = 0, semantics: int = SEM_REFERENCE,
           workspace: Workspace | None = None, stream=None) -> torch.Tensor:
    """C[M,N] = A[M,K] (fp32) x dequant(B[N,K] int8, B_scale fp32)^T.

    ``group_quantized=False`` is per-output-row scaling (group size K)."""
    M, K = A.shape
    N = B.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    g = group_size if group_quantized else K
    L = load_library()
    nbytes = L.qvl_linear_i8_workspace_bytes(M, K, g)
    ws = _ws(workspace, A.device).get(nbytes)
    _check(L.qvl_linear_i8(_ptr(A), _ptr(B), _ptr(B_scale), _ptr(C), M, N, K, int(group_quantized),
                           group_size, semantics, _ptr(ws), ws.numel(), _stream(stream)), "linear")
    return C


def linear_q16(q, q_scales, B, B_scale, group_size, C=None, semantics=SEM_REFERENCE, stream=None):
    M, K = q.shape
    N = B.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=q.device)
    _check(load_library().qvl_linear_q16_i8(_ptr(q), _ptr(q_scales), _ptr(B), _ptr(B_scale), _ptr(C),
                                            M, N, K, group_size, semantics, _stream(stream)),
           "linear_q16")
    return C


def swiglu(gate: torch.Tensor, up: torch.Tensor, stream=None) -> torch.Tensor:
    """In place: gate = silu(gate) * up."""
    _check(load_library().qvl_swiglu(_ptr(gate), _ptr(up), gate.numel(), _stream(stream)), "swiglu")
    return gate


def swiglu_mlp(x, w_gate, s_gate, w_up, s_up, w_down, s_down, group_size, out=None,
               semantics=SEM_REFERENCE, workspace=None, stream=None):
    """out[M,H] = down(swiglu(gate(x), up(x))) with int8 weights."""
    M, H = x.shape
    I = w_gate.shape[0]
    if out is None:
        out = torch.empty((M, H), dtype=torch.float32, device=x.device)
    L = load_library()
    ws = _ws(workspace, x.device).get(L.qvl_swiglu_mlp_workspace_bytes(M, H, I, group_size))
    _check(L.qvl_swiglu_mlp_i8(_ptr(x), _ptr(w_gate), _ptr(s_gate), _ptr(w_up), _ptr(s_up),
                               _ptr(w_down), _ptr(s_down), _ptr(out), M, H, I, group_size, semantics,
                               _ptr(ws), ws.numel(), _stream(stream)), "swiglu_mlp")
    return out


class PagedKV:
    """One layer's FP16 KV pages [num_pages, NKV, page_size, D] plus a page table
    [num_seqs, max_pages_per_seq] (identity-mapped unless given)."""

    def __init__(self, num_seqs, max_ctx, num_heads=16, num_kv_heads=8, head_dim=128,
                 page_size=64, max_pos=None, device="cuda", page_table=None, k=None, v=None):
        """k, v: optional preallocated page tensors (e.g. one layer of a
        stacked [layers, pages, ...] cache); zero-filled pages otherwise."""
        self.page_size = page_size
        self.maxp = (max_ctx + page_size - 1) // page_size
        num_pages = num_seqs * self.maxp
        shape = (num_pages, num_kv_heads, page_size, head_dim)
        self.k = torch.zeros(shape, dtype=torch.float16, device=device) if k is None else k
        self.v = torch.zeros(shape, dtype=torch.float16, device=device) if v is None else v
        if tuple(self.k.shape) != shape or tuple(self.v.shape) != shape:
            raise QvlError(f"KV pages must have shape {shape}")
        if page_table is None:
            page_table = torch.arange(num_pages, dtype=torch.int32, device=device).view(num_seqs, self.maxp)
        self.page_table = page_table.contiguous()
        self.dims = AttnDims(num_heads, num_kv_heads, head_dim, page_size, self.maxp,
                             max_pos if max_pos is not None else max_ctx)


def rope_kv_append(q, k_new, v_new, kv: PagedKV, seq_ids, positions, rope_cos, rope_sin, stream=None):
    """Rotate q in place; rotate k_new and write k/v (fp16) at each query's position."""
    nq = q.shape[0]
    _check(load_library().qvl_rope_kv_append(
        _ptr(q), _ptr(k_new), _ptr(v_new), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table),
        _ptr(seq_ids), _ptr(positions), nq, _ptr(rope_cos), _ptr(rope_sin), ctypes.byref(kv.dims),
        _stream(stream)), "rope_kv_append")
    return q


def attention(q, kv: PagedKV, seq_ids, positions, max_ctx, out=None, workspace=None, stream=None):
    """out[nq, NH, D] = softmax(q k^T / sqrt(D)) v over positions [0, pos] of each query."""
    nq = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    L = load_library()
    ws = _ws(workspace, q.device).get(L.qvl_attention_workspace_bytes(nq, max_ctx, ctypes.byref(kv.dims)))
    _check(L.qvl_attention_decode(_ptr(q), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table),
                                  _ptr(seq_ids), _ptr(positions), nq, max_ctx, _ptr(out),
                                  ctypes.byref(kv.dims), _ptr(ws), ws.numel(), _stream(stream)),
           "attention")
    return out


def attention_ordered(q, kv: PagedKV, seq_ids, positions, max_ctx, out=None, workspace=None, stream=None):
    """attention() in the reference's own summation order (bit-exact with
    attn_scores_all_heads + softmax + attn_weighted_sum_all_heads on the same
    fp16-valued cache); sequential over the context, so slower."""
    nq = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    L = load_library()
    ws = _ws(workspace, q.device).get(L.qvl_attention_ordered_workspace_bytes(nq, max_ctx, ctypes.byref(kv.dims)))
    _check(L.qvl_attention_decode_ordered(_ptr(q), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table),
                                          _ptr(seq_ids), _ptr(positions), nq, max_ctx, _ptr(out),
                                          ctypes.byref(kv.dims), _ptr(ws), ws.numel(), _stream(stream)),
           "attention_ordered")
    return out


def qknorm_rope_attention_ordered(q, k_new, v_new, kv: PagedKV, seq_ids, positions, max_ctx, rope_cos, rope_sin,
                                  q_norm_w, q_norm_s, k_norm_w, k_norm_s, norm_group, eps, out=None, workspace=None,
                                  stream=None):
    """qknorm_rope_kv_append + attention_ordered of one decode step in one
    pass (q is left unrotated); every query a different sequence."""
    nq = q.shape[0]
    if out is None:
        out = torch.empty_like(q)
    L = load_library()
    ws = _ws(workspace, q.device).get(L.qvl_attention_ordered_workspace_bytes(nq, max_ctx, ctypes.byref(kv.dims)))
    _check(L.qvl_qknorm_rope_attention_decode_ordered(
        _ptr(q), _ptr(k_new), _ptr(v_new), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table), _ptr(seq_ids),
        _ptr(positions), nq, max_ctx, _ptr(rope_cos), _ptr(rope_sin), _ptr(q_norm_w), _ptr(q_norm_s),
        _ptr(k_norm_w), _ptr(k_norm_s), norm_group, eps, _ptr(out), ctypes.byref(kv.dims), _ptr(ws), ws.numel(),
        _stream(stream)), "qknorm_rope_attention_ordered")
    return out


def text_weights_struct(t: dict, cfg) -> TextWeightsC:
    """qvl_text_weights for the stacked weight dict of decoder.TextWeights
    (the tensors must stay alive while the struct is used)."""
    names = {"w_q": "wq", "w_k": "wk", "w_v": "wv", "w_o": "wo", "w_gate": "wg", "w_up": "wu", "w_down": "wd"}
    w = TextWeightsC()
    for f, n in names.items():
        setattr(w, f, _ptr(t[n]))
        setattr(w, "s" + f[1:], _ptr(t[n + "_s"]))
    for n in ("in_norm", "post_norm", "q_norm", "k_norm", "final_norm", "embed"):
        setattr(w, n, _ptr(t[n]))
        setattr(w, n + "_s", _ptr(t[n + "_s"]))
    w.layers, w.vocab, w.hidden, w.intermediate = cfg.layers, cfg.vocab, cfg.hidden, cfg.intermediate
    w.heads, w.kv_heads, w.head_dim, w.norm_group = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.norm_group
    w.eps = cfg.eps
    return w


def text_decode_workspace(device) -> torch.Tensor:
    """Zero-filled workspace for text_decode_step (keep it between calls)."""
    n = load_library().qvl_text_decode_workspace_bytes()
    return torch.zeros(n, dtype=torch.uint8, device=device)


DECODE_REFERENCE_ORDER = 1


def text_decode_step(w: TextWeightsC, x, logits, token, pos, k_all, v_all, page_table, page_size, rope_cos,
                     rope_sin, max_ctx, workspace, stream=None, flags=0):
    """One whole decode token of one request in one launch: reads token[0] and
    pos[0], writes logits and x, replaces token[0] by the greedy token and
    advances pos[0].  k_all / v_all: [layers, pages, NKV, page_size, D] fp16.
    flags=DECODE_REFERENCE_ORDER: attention in the reference's summation order."""
    layer_stride = k_all[0].numel()
    _check(load_library().qvl_text_decode_step_ex(
        ctypes.byref(w), _ptr(x), _ptr(logits), _ptr(token), _ptr(pos), _ptr(k_all), _ptr(v_all), layer_stride,
        _ptr(page_table), page_size, _ptr(rope_cos), _ptr(rope_sin), max_ctx, _ptr(workspace),
        workspace.numel(), flags, _stream(stream)), "text_decode_step")


def tc_timed_out(clear: bool = False, stream=None) -> bool:
    """True if a bounded wait of the tensor-core GEMM gave up on this device
    since the word was last cleared (synchronises); clear=True resets it."""
    v = _I(0)
    _check(load_library().qvl_tc_timeout_status(ctypes.byref(v), int(clear), _stream(stream)), "tc_timeout_status")
    return bool(v.value)


def text_decode_aborted(workspace) -> bool:
    """True if a grid-barrier wait of text_decode_step timed out (synchronises)."""
    off = load_library().qvl_text_decode_abort_flag(_ptr(workspace)) - workspace.data_ptr()
    return bool(workspace[off:off + 4].view(torch.int32).item())


def text_decode_trace(workspace) -> np.ndarray:
    """Phase timestamps (ns) of the last text_decode_step on this workspace:
    [0] kernel start, [1 + i] opening of grid barrier i (synchronises)."""
    off = load_library().qvl_text_decode_trace(_ptr(workspace)) - workspace.data_ptr()
    return workspace[off:off + 1024 * 8].view(torch.int64).cpu().numpy()


def greedy_decode(logits: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    """int32 [rows]: first index of the row maximum."""
    rows = logits.shape[0] if logits.dim() == 2 else 1
    n = logits.shape[-1]
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _check(load_library().qvl_argmax_rows(_ptr(logits), _ptr(out), rows, n, _stream(stream)),
           "greedy_decode")
    return out


def rms_norm_i8(x, w, w_scales, norm_group, eps, out=None, q=None, q_scales=None, quant_group=0,
                inplace_form=False, stream=None):
    """rms_norm (inplace_form=False) / rms_norm_inplace rounding with an INT8
    group-quantised weight; writes `out` and/or the next linear's int16
    activations q, q_scales (group quant_group)."""
    rows, H = x.shape
    _check(load_library().qvl_rms_norm_i8(_ptr(x), _ptr(w), _ptr(w_scales), _ptr(out), _ptr(q),
                                          _ptr(q_scales), rows, H, norm_group, eps, int(inplace_form),
                                          quant_group, _stream(stream)), "rms_norm_i8")
    return out


def qknorm_rope_kv_append(q, k_new, v_new, kv: PagedKV, seq_ids, positions, rope_cos, rope_sin,
                          q_norm_w, q_norm_s, k_norm_w, k_norm_s, norm_group, eps, stream=None):
    nq = q.shape[0]
    _check(load_library().qvl_qknorm_rope_kv_append(
        _ptr(q), _ptr(k_new), _ptr(v_new), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table),
        _ptr(seq_ids), _ptr(positions), nq, _ptr(rope_cos), _ptr(rope_sin), _ptr(q_norm_w),
        _ptr(q_norm_s), _ptr(k_norm_w), _ptr(k_norm_s), norm_group, eps, ctypes.byref(kv.dims),
        _stream(stream)), "qknorm_rope_kv_append")
    return q


def embedding_lookup_i8(table, row_scales, token_ids, out, stream=None):
    V, H = table.shape
    _check(load_library().qvl_embedding_lookup_i8(_ptr(table), _ptr(row_scales), _ptr(token_ids), _ptr(out),
                                                  token_ids.numel(), V, H, _stream(stream)),
           "embedding_lookup_i8")
    return out


def swiglu_quantize_rows(gate, up, q, q_scales, group_size, stream=None):
    M, I = gate.shape
    _check(load_library().qvl_swiglu_quantize_rows(_ptr(gate), _ptr(up), _ptr(q), _ptr(q_scales), M, I,
                                                   group_size, _stream(stream)), "swiglu_quantize_rows")
    return q


def linear_q16_multi(q, q_scales, mats, outs, group_size, semantics=SEM_REFERENCE, stream=None):
    """outs[i] = q . dequant(mats[i])^T for up to three (W, scales) pairs in one launch."""
    n = len(mats)
    M, K = q.shape
    Bp = (ctypes.c_void_p * n)(*[_ptr(w) for w, _ in mats])
    Sp = (ctypes.c_void_p * n)(*[_ptr(s) for _, s in mats])
    Cp = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    Np = (ctypes.c_size_t * n)(*[w.shape[0] for w, _ in mats])
    _check(load_library().qvl_linear_q16_i8_multi(_ptr(q), _ptr(q_scales), n, Bp, Sp, Cp, Np, M, K,
                                                  group_size, semantics, _stream(stream)), "linear_q16_multi")
    return outs


def gate_up_swiglu(q, q_scales, w_gate, s_gate, w_up, s_up, h, group_size, up_scratch=None,
                   semantics=SEM_REFERENCE, stream=None):
    """h = swiglu(gate(q), up(q)) with the SwiGLU fused into the GEMV epilogue."""
    M, K = q.shape
    I = w_gate.shape[0]
    _check(load_library().qvl_gate_up_swiglu_q16_i8(_ptr(q), _ptr(q_scales), _ptr(w_gate), _ptr(s_gate),
                                                    _ptr(w_up), _ptr(s_up), _ptr(h), _ptr(up_scratch), M, I,
                                                    K, group_size, semantics, _stream(stream)),
           "gate_up_swiglu")
    return h


def linear_tail(q, q_scales, mats, outs, group_size, counter, q_out, q_out_scales, quant_group,
                norm=None, eps=1e-6, inplace_form=False, norm_out=None, swiglu_pair=False,
                semantics=SEM_REFERENCE, stream=None):
    """Products of `mats` (like linear_q16_multi; swiglu_pair=True: gate/up with
    SwiGLU into outs[0]) followed, in the same launch, by RMSNorm (norm=(w, s,
    group)) and/or quantisation of outs[0] into q_out/q_out_scales.
    `counter`: a zero-initialised int32 device tensor (left at zero)."""
    n = len(mats)
    M, K = q.shape
    Bp = (ctypes.c_void_p * n)(*[_ptr(w) for w, _ in mats])
    Sp = (ctypes.c_void_p * n)(*[_ptr(s) for _, s in mats])
    Cp = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    Np = (ctypes.c_size_t * n)(*[w.shape[0] for w, _ in mats])
    t = RowTail(_ptr(counter), _ptr(norm[0]) if norm else None, _ptr(norm[1]) if norm else None,
                norm[2] if norm else 0, eps, int(inplace_form), _ptr(norm_out), _ptr(q_out),
                _ptr(q_out_scales), quant_group)
    _check(load_library().qvl_linear_q16_i8_tail(_ptr(q), _ptr(q_scales), n, Bp, Sp, Cp, Np, M, K, group_size,
                                                 semantics, int(swiglu_pair), ctypes.byref(t), _stream(stream)),
           "linear_tail")
    return outs


def linear_batched(q, q_scales, mats, outs, workspace, semantics=SEM_TILED, swiglu_pair=False, up_scratch=None,
                   stream=None):
    """Tensor-core products of the same activations (split into hi/lo planes once)."""
    n = len(mats)
    M, K = q.shape
    Bp = (ctypes.c_void_p * n)(*[_ptr(w) for w, _ in mats])
    Sp = (ctypes.c_void_p * n)(*[_ptr(s) for _, s in mats])
    Cp = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    Np = (ctypes.c_size_t * n)(*[w.shape[0] for w, _ in mats])
    L = load_library()
    ws = workspace.get(L.qvl_linear_q16_i8_batched_workspace_bytes(M, K))
    _check(L.qvl_linear_q16_i8_batched(_ptr(q), _ptr(q_scales), n, Bp, Sp, Cp, Np, M, K, semantics,
                                       int(swiglu_pair), _ptr(up_scratch), _ptr(ws), ws.numel(), _stream(stream)),
           "linear_batched")
    return outs


class Planes:
    """The tensor cores' hi/lo activation planes (hi = q >> 8, lo = q & 255)
    of up to `rows` x `cols` quantised activations, reused across products."""

    def __init__(self, rows, cols, device):
        self.hi = torch.empty(rows * cols, dtype=torch.int8, device=device)
        self.lo = torch.empty(rows * cols, dtype=torch.uint8, device=device)


def quantize_rows_planes(x, q, q_scales, planes: Planes, group_size=0, stream=None):
    """quantize_rows into q/q_scales that also fills `planes` for linear_planes_batched."""
    M, K = x.shape
    _check(load_library().qvl_quantize_rows_planes(_ptr(x), _ptr(q), _ptr(q_scales), _ptr(planes.hi),
                                                   _ptr(planes.lo), M, K, group_size or K, _stream(stream)),
           "quantize_rows_planes")
    return q


def rms_norm_i8_planes(x, w, w_scales, norm_group, eps, q, q_scales, planes: Planes, out=None, inplace_form=False,
                       stream=None):
    """rms_norm_i8 with per-row quantisation that also fills `planes`."""
    rows, H = x.shape
    _check(load_library().qvl_rms_norm_i8_planes(_ptr(x), _ptr(w), _ptr(w_scales), _ptr(out), _ptr(q),
                                                 _ptr(q_scales), _ptr(planes.hi), _ptr(planes.lo), rows, H,
                                                 norm_group, eps, int(inplace_form), _stream(stream)),
           "rms_norm_i8_planes")
    return out


def linear_planes_batched(planes: Planes, q_scales, mats, outs, M, K, semantics=SEM_TILED, stream=None):
    """Tensor-core products of activations already in `planes`, one launch for all (<= 3) matrices."""
    n = len(mats)
    Bp = (ctypes.c_void_p * n)(*[_ptr(w) for w, _ in mats])
    Sp = (ctypes.c_void_p * n)(*[_ptr(s) for _, s in mats])
    Cp = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    Np = (ctypes.c_size_t * n)(*[w.shape[0] for w, _ in mats])
    _check(load_library().qvl_linear_planes_i8_batched(_ptr(planes.hi), _ptr(planes.lo), _ptr(q_scales), n, Bp, Sp,
                                                       Cp, Np, M, K, semantics, _stream(stream)),
           "linear_planes_batched")
    return outs


def attention_q16(q, kv: PagedKV, seq_ids, positions, max_ctx, out, q_out, q_out_scales, counter,
                  workspace=None, stream=None):
    """attention + per-row quantisation of its output (fused when single-launch)."""
    nq = q.shape[0]
    L = load_library()
    ws = _ws(workspace, q.device).get(L.qvl_attention_workspace_bytes(nq, max_ctx, ctypes.byref(kv.dims)))
    _check(L.qvl_attention_decode_q16(_ptr(q), kv.k.data_ptr(), kv.v.data_ptr(), _ptr(kv.page_table),
                                      _ptr(seq_ids), _ptr(positions), nq, max_ctx, _ptr(out), _ptr(q_out),
                                      _ptr(q_out_scales), _ptr(counter), ctypes.byref(kv.dims), _ptr(ws),
                                      ws.numel(), _stream(stream)), "attention_q16")
    return out
