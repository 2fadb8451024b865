"""The attention entry point for callers that cannot allocate device memory
when they call in (a plugin inside a framework that owns every device
allocation, or a serving loop that must not allocate): its scratch is a
fixed array inside the library.  It must give the same output as the
workspace-taking entry point, call after call.

Named to be collected last, so a run that stops at the first failure has run
everything else first."""
import ctypes

import numpy as np
import pytest
import torch

from test_gpu_parity import NH, NKV, D, _attn_setup, dev

pytestmark = pytest.mark.gpu

_P, _Z, _I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


def _static_fn(qvl):
    L = qvl.load_library()
    f = L.qvl_attention_decode_static
    f.argtypes = [_P] * 6 + [_Z, _I, _P, ctypes.POINTER(qvl.AttnDims), _P]
    f.restype = _I
    return f


def _run_both(qvl, cuda, ctxs, seed):
    kv, _, q, kn, vn, cos, sin = _attn_setup(qvl, cuda, ctxs, seed=seed)
    B = len(ctxs)
    qd = dev(q, cuda)
    seq = torch.arange(B, dtype=torch.int32, device=cuda)
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32, device=cuda)
    qvl.rope_kv_append(qd, dev(kn, cuda), dev(vn, cuda), kv, seq, pos, dev(cos, cuda), dev(sin, cuda))
    max_ctx = max(ctxs)
    expect = qvl.attention(qd, kv, seq, pos, max_ctx).cpu().numpy()
    out = torch.full_like(qd, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = _static_fn(qvl)(qd.data_ptr(), kv.k.data_ptr(), kv.v.data_ptr(), kv.page_table.data_ptr(),
                         seq.data_ptr(), pos.data_ptr(), B, max_ctx, out.data_ptr(),
                         ctypes.byref(kv.dims), stream)
    assert rc == 0, qvl.load_library().qvl_status_string(rc)
    return out.cpu().numpy(), expect


def test_static_scratch_attention_matches_workspace_path(qvl, cuda):
    # calls in a row on different shapes: each reuses the array the one before
    # left behind.  Contexts above 8192 tokens with few queries take the
    # split-K path, the one that uses the scratch; [300, 33] takes the cluster
    # path.  Both entry points run the same kernels, so the bytes must agree.
    for ctxs, seed in (([9000, 33], 1), ([12000], 2), ([300, 33], 3), ([9000, 33], 4)):
        got, expect = _run_both(qvl, cuda, ctxs, seed)
        assert np.isfinite(got).all()
        assert np.array_equal(got, expect)


def test_static_scratch_rejects_oversized_requests(qvl, cuda):
    d = qvl.AttnDims(NH, NKV, D, 64, 512, 32768)
    need = qvl.load_library().qvl_attention_workspace_bytes(64, 32768, ctypes.byref(d))
    assert need > (32 << 20)
    fake = 1 << 20          # 16-byte aligned; rejected before any access
    rc = _static_fn(qvl)(fake, fake, fake, fake, fake, fake, 64, 32768, fake, ctypes.byref(d), None)
    assert rc == 4          # QVL_ERR_WORKSPACE: larger than the built-in scratch
