"""GPU parity: the sm_100a kernels, called through the C ABI, against the CPU
oracle (itself pinned to the reference's compiled code) on the same seeded
inputs.

Bars: integer accumulation and everything built
only from it is bit-exact; fp32 outputs within a max relative error of 1e-3
(||a - b||_inf / ||b||_inf), fp16-cache attention included.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import make_linear_inputs

pytestmark = pytest.mark.gpu

REL_TOL_FP32 = 1e-3


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("M,K,g", [(1, 2048, 2048), (3, 2048, 128), (2, 6144, 6144), (5, 1024, 32),
                                   (1, 6144, 128), (4, 512, 16)])
def test_quantize_rows_bit_exact(qvl, cuda, M, K, g):
    x, _, _ = make_linear_inputs(M * 7 + g, M, 1, K, g)
    x[0, :5] = [0.0, -0.0, 1e-30, 3.5, -2.5]
    q, s = qvl.quantize_rows(dev(x, cuda), g)
    qo, so = oracle.quantize(x, g)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_quantize_zero_row(qvl, cuda):
    x = np.zeros((1, 256), np.float32)
    q, s = qvl.quantize_rows(dev(x, cuda), 128)
    qo, so = oracle.quantize(x, 128)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


LINEAR = [
    # (M, N, K, g): M=1 with N,K >= 1024 is the reference's GEMV order
    (1, 6144, 2048, 2048),   # config 0: gate/up per-row
    (1, 2048, 2048, 2048),   # q/o proj
    (1, 1024, 2048, 2048),   # k/v proj
    (1, 2048, 6144, 6144),   # down proj (K = 6144)
    (1, 6144, 2048, 128),
    (1, 1024, 1024, 64),
    (1, 1024, 1024, 32),
    (1, 1024, 1024, 256),
    (1, 1000, 1024, 1024),   # N below the GEMV threshold -> tiled order
    (3, 256, 512, 128),
    (8, 2048, 2048, 2048),
    (13, 300, 2048, 512),    # ragged row tile (8 + 5)
    (1, 17, 512, 512),       # odd N
    (4, 512, 1024, 64),      # generic kernel, TILED, 4-lane segments
    (2, 256, 512, 32),       # generic kernel, TILED, 2-lane segments
]


@pytest.mark.parametrize("M,N,K,g", LINEAR)
def test_linear_bit_exact(qvl, cuda, M, N, K, g):
    x, w, ws = make_linear_inputs(1000 + M + N + g, M, N, K, g)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=True, group_size=g)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, g))


def test_linear_rowwise_flag_means_group_K(qvl, cuda):
    x, w, ws = make_linear_inputs(3, 1, 2048, 2048, 2048)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=False)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, 2048))


@pytest.mark.parametrize("M,g", [(4, 2048), (32, 128), (9, 2048)])
def test_linear_batched_decode_rows_match_single_row(qvl, cuda, M, g):
    """LANE8: each row of a decode batch equals its own M=1 reference GEMV."""
    x, w, ws = make_linear_inputs(77 + M, M, 2048, 2048, g)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_size=g, semantics=qvl.SEM_LANE8)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, g, oracle.LANE8))


@pytest.mark.parametrize("M,g", [(16, 2048), (64, 128), (130, 2048)])
def test_linear_tiled_medium_m(qvl, cuda, M, g):
    x, w, ws = make_linear_inputs(5 + M, M, 1024, 2048, g)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_size=g, semantics=qvl.SEM_TILED)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, g, oracle.TILED))


def test_lm_head_gemv(qvl, cuda):
    x, w, ws = make_linear_inputs(9, 1, 151936, 2048, 2048)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_size=2048)
    yo = oracle.linear_i8(x, w, ws, 2048)
    np.testing.assert_array_equal(y.cpu().numpy(), yo)
    idx = qvl.greedy_decode(y)
    assert int(idx.item()) == oracle.argmax(yo[0])


@pytest.mark.parametrize("N,K", [(4096, 2048), (2048, 6144), (16, 2048)])
def test_ring_gemv_accumulate(qvl, cuda, N, K):
    """M=1 per-row GEMVs of >= 4 MiB stream through the ring kernel (the
    16-row case stays on the direct-load kernel): C += x.W^T bit-exact
    against the reference's product plus the separate add (add_vector)."""
    import torch
    x, w, ws = make_linear_inputs(321 + N + K, 1, N, K, K)
    q, qs = qvl.quantize_rows(dev(x, cuda), K)
    c0 = np.random.default_rng(N).standard_normal((1, N), dtype=np.float32)
    c = dev(c0.copy(), cuda)
    qvl.linear_q16(q, qs, dev(w, cuda), dev(ws, cuda), K, C=c, semantics=qvl.SEM_LANE8 | qvl.SEM_ACCUMULATE)
    want = (c0 + oracle.linear_i8(x, w, ws, K, oracle.LANE8)).astype(np.float32)
    np.testing.assert_array_equal(c.cpu().numpy(), want)


@pytest.mark.parametrize("M", [1, 64])
def test_swiglu_mlp_per_row(qvl, cuda, M):
    """group_size 0: per-row scales for gate/up (group 2048) and down (group
    6144); M=64 runs the products on the tensor cores (TILED order)."""
    H, I = 2048, 6144
    rng = np.random.default_rng(70 + M)
    x = rng.standard_normal((M, H), dtype=np.float32)
    wg = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wu = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wd = rng.integers(-127, 128, (H, I), dtype=np.int8)
    sg, su = (rng.uniform(0.001, 0.02, I).astype(np.float32) for _ in range(2))
    sd = rng.uniform(0.001, 0.02, H).astype(np.float32)
    out = qvl.swiglu_mlp(*(dev(a, cuda) for a in (x, wg, sg, wu, su, wd, sd)), group_size=0)
    mode = oracle.LANE8_DISPATCH
    h = oracle.swiglu(oracle.linear_i8(x, wg, sg, H, mode), oracle.linear_i8(x, wu, su, H, mode))
    ref = oracle.linear_i8(h, wd, sd, I, mode)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_swiglu_mlp_config2_m512(qvl, cuda):
    """Config 2 at M=512 (the tensor-core products, TILED order), per-row
    scales: bit-exact on a spread of 64 rows (rows are independent)."""
    H, I, M = 2048, 6144, 512
    rng = np.random.default_rng(512)
    x = rng.standard_normal((M, H), dtype=np.float32)
    wg = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wu = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wd = rng.integers(-127, 128, (H, I), dtype=np.int8)
    sg, su = (rng.uniform(0.001, 0.02, I).astype(np.float32) for _ in range(2))
    sd = rng.uniform(0.001, 0.02, H).astype(np.float32)
    out = qvl.swiglu_mlp(*(dev(a, cuda) for a in (x, wg, sg, wu, su, wd, sd)), group_size=0).cpu().numpy()
    rows = np.unique(np.concatenate([[0, 1, 255, 511], rng.choice(M, 60, replace=False)]))
    xs = x[rows]
    T = oracle.TILED
    h = oracle.swiglu(oracle.linear_i8(xs, wg, sg, H, T, threads=16), oracle.linear_i8(xs, wu, su, H, T, threads=16))
    ref = oracle.linear_i8(h, wd, sd, I, T, threads=16)
    np.testing.assert_array_equal(out[rows], ref)


def test_expf_matches_host_on_every_float(qvl, cuda):
    """The device expf used by SwiGLU equals the host C library's expf (what
    the reference calls) on all 2^32 inputs; NaN inputs give NaN."""
    import ctypes
    L = qvl.load_library()
    L.qvl_internal_expf.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    chunk = 1 << 28
    y = torch.empty(chunk, dtype=torch.float32, device=cuda)
    bad = 0
    for c in range(1 << 32 >> 28):
        xb = np.arange(c * chunk, (c + 1) * chunk, dtype=np.uint64).astype(np.uint32)
        x = xb.view(np.float32)
        xd = torch.from_numpy(x).to(cuda)
        assert L.qvl_internal_expf(xd.data_ptr(), y.data_ptr(), chunk, torch.cuda.current_stream().cuda_stream) == 0
        got = y.cpu().numpy()
        want = oracle.expf(x, threads=16)
        nan = np.isnan(x)
        assert np.isnan(got[nan]).all()
        bad += int((got.view(np.uint32)[~nan] != want.view(np.uint32)[~nan]).sum())
    assert bad == 0


def test_swiglu_matches(qvl, cuda):
    rng = np.random.default_rng(4)
    g = (rng.standard_normal(6144, dtype=np.float32) * 4)
    u = rng.standard_normal(6144, dtype=np.float32)
    gd = dev(g, cuda)
    qvl.swiglu(gd, dev(u, cuda))
    out = gd.cpu().numpy()
    ref = oracle.swiglu(g, u)
    np.testing.assert_array_equal(out, ref)


@pytest.mark.parametrize("M,g", [(1, 2048), (1, 128), (4, 2048), (64, 2048), (64, 128), (32, 64)])
def test_swiglu_mlp(qvl, cuda, M, g):
    H, I = 2048, 6144
    rng = np.random.default_rng(50 + M)
    x = rng.standard_normal((M, H), dtype=np.float32)
    wg = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wu = rng.integers(-127, 128, (I, H), dtype=np.int8)
    wd = rng.integers(-127, 128, (H, I), dtype=np.int8)
    sg = rng.uniform(0.001, 0.02, I * H // g).astype(np.float32)
    su = rng.uniform(0.001, 0.02, I * H // g).astype(np.float32)
    sd = rng.uniform(0.001, 0.02, I * H // g).astype(np.float32)
    out = qvl.swiglu_mlp(*(dev(a, cuda) for a in (x, wg, sg, wu, su, wd, sd)), group_size=g)
    gate = oracle.linear_i8(x, wg, sg, g)
    up = oracle.linear_i8(x, wu, su, g)
    h = oracle.swiglu(gate, up)
    ref = oracle.linear_i8(h, wd, sd, g)
    got = out.cpu().numpy()
    assert rel_err(got, ref) < REL_TOL_FP32
    assert (got == ref).mean() > 0.99   # bit-exact except where expf rounding differs


# ------------------------------------------------------------------ attention
NH, NKV, D = 16, 8, 128


def _attn_setup(qvl, cuda, ctxs, page_size=64, seed=0, theta=5e6):
    """Per sequence: a pre-filled cache of ctx-1 tokens (post-RoPE K, V as
    fp16) and a new token at pos = ctx-1 appended through rope_kv_append."""
    rng = np.random.default_rng(seed)
    B = len(ctxs)
    max_ctx = max(ctxs)
    kv = qvl.PagedKV(B, max_ctx, NH, NKV, D, page_size, max_pos=max_ctx, device=cuda)
    # shuffle the physical pages to exercise the page table
    perm = torch.randperm(kv.page_table.numel(), generator=torch.Generator().manual_seed(seed))
    kv.page_table = perm.to(torch.int32).view(B, kv.maxp).to(cuda).contiguous()
    cos, sin = oracle.rope_table(max_ctx, D, theta)
    caches = []
    for b, ctx in enumerate(ctxs):
        kc = rng.standard_normal((NKV, ctx, D), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((NKV, ctx, D), dtype=np.float32).astype(np.float16)
        pt = kv.page_table[b].cpu().numpy()
        t = np.arange(ctx - 1)
        pidx = torch.from_numpy(pt[t // page_size].astype(np.int64)).to(cuda)
        slot = torch.from_numpy((t % page_size).astype(np.int64)).to(cuda)
        kv.k[pidx, :, slot] = torch.from_numpy(np.ascontiguousarray(kc[:, :-1].transpose(1, 0, 2))).to(cuda)
        kv.v[pidx, :, slot] = torch.from_numpy(np.ascontiguousarray(vc[:, :-1].transpose(1, 0, 2))).to(cuda)
        caches.append((kc, vc))
    q = rng.standard_normal((B, NH, D), dtype=np.float32)
    kn = rng.standard_normal((B, NKV, D), dtype=np.float32)
    vn = rng.standard_normal((B, NKV, D), dtype=np.float32)
    return kv, caches, q, kn, vn, cos, sin


def _oracle_decode(caches, ctxs, q, kn, vn, cos, sin):
    outs = []
    for b, ctx in enumerate(ctxs):
        pos = ctx - 1
        kc, vc = caches[b]
        kc = kc.astype(np.float32).copy()
        vc = vc.astype(np.float32).copy()
        qb = oracle.rope_inplace(q[b].copy(), cos[pos], sin[pos])
        kb = oracle.rope_inplace(kn[b].copy(), cos[pos], sin[pos])
        kc[:, pos] = kb.astype(np.float16).astype(np.float32)   # cache stores fp16
        vc[:, pos] = vn[b].astype(np.float16).astype(np.float32)
        outs.append(oracle.attention(np.ascontiguousarray(kc), np.ascontiguousarray(vc), qb, pos))
    return np.stack(outs)


@pytest.mark.parametrize("ctxs", [[1], [512], [4096], [3, 77, 600], [32768], [130] * 8,
                                  [512] * 64, [4096] * 64, [32768] * 8])
def test_attention_decode(qvl, cuda, ctxs):
    kv, caches, q, kn, vn, cos, sin = _attn_setup(qvl, cuda, ctxs, seed=len(ctxs) + ctxs[0])
    B = len(ctxs)
    qd = dev(q, cuda)
    seq = torch.arange(B, dtype=torch.int32, device=cuda)
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32, device=cuda)
    qvl.rope_kv_append(qd, dev(kn, cuda), dev(vn, cuda), kv, seq, pos, dev(cos, cuda), dev(sin, cuda))
    out = qvl.attention(qd, kv, seq, pos, max(ctxs)).cpu().numpy()
    ref = _oracle_decode(caches, ctxs, q, kn, vn, cos, sin)
    for b in range(B):
        assert rel_err(out[b], ref[b]) < REL_TOL_FP32, (b, rel_err(out[b], ref[b]))


@pytest.mark.parametrize("ctxs", [[1], [8], [9], [452], [3, 77, 600, 16], [4096], [512] * 8])
def test_attention_ordered_bit_exact(qvl, cuda, ctxs):
    """The reference-order attention equals the oracle (pinned bit-exact to the
    reference's attn_scores_all_heads + softmax + attn_weighted_sum_all_heads)
    on the same fp16-valued cache, bit for bit."""
    kv, caches, q, kn, vn, cos, sin = _attn_setup(qvl, cuda, ctxs, seed=17 + len(ctxs) + ctxs[0])
    B = len(ctxs)
    qd = dev(q, cuda)
    seq = torch.arange(B, dtype=torch.int32, device=cuda)
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32, device=cuda)
    qvl.rope_kv_append(qd, dev(kn, cuda), dev(vn, cuda), kv, seq, pos, dev(cos, cuda), dev(sin, cuda))
    out = qvl.attention_ordered(qd, kv, seq, pos, max(ctxs)).cpu().numpy()
    ref = _oracle_decode(caches, ctxs, q, kn, vn, cos, sin)
    np.testing.assert_array_equal(out, ref)


@pytest.mark.parametrize("ctxs,with_norm", [([1, 128, 129, 452, 257], True), ([300, 1000], False),
                                             ([512] * 32, True)])
def test_qknorm_rope_attention_ordered_fused(qvl, cuda, ctxs, with_norm):
    """QK-norm + RoPE + KV append inside the reference-order score pass equals
    qknorm_rope_kv_append followed by attention_ordered bit for bit: the
    attention output and every page of the cache (positions at, before and
    after a 128-position block boundary, the first position, no QK-norm)."""
    kv, caches, q, kn, vn, cos, sin = _attn_setup(qvl, cuda, ctxs, seed=29 + len(ctxs))
    B, ng, eps = len(ctxs), 16, 1e-6
    rng = np.random.default_rng(5)
    nw = [dev(rng.integers(-127, 128, D, dtype=np.int8), cuda) if with_norm else None for _ in range(2)]
    ns = [dev(rng.uniform(0.001, 0.02, D // ng).astype(np.float32), cuda) if with_norm else None for _ in range(2)]
    seq = torch.arange(B, dtype=torch.int32, device=cuda)
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32, device=cuda)
    cd, sd, knd, vnd = dev(cos, cuda), dev(sin, cuda), dev(kn, cuda), dev(vn, cuda)
    k0, v0 = kv.k.clone(), kv.v.clone()
    qd = dev(q, cuda)
    if with_norm:
        qvl.qknorm_rope_kv_append(qd, knd, vnd, kv, seq, pos, cd, sd, nw[0], ns[0], nw[1], ns[1], ng, eps)
    else:
        qvl.rope_kv_append(qd, knd, vnd, kv, seq, pos, cd, sd)
    ref = qvl.attention_ordered(qd, kv, seq, pos, max(ctxs))
    k_ref, v_ref = kv.k.clone(), kv.v.clone()
    kv.k.copy_(k0)
    kv.v.copy_(v0)
    qraw = dev(q, cuda)
    out = qvl.qknorm_rope_attention_ordered(qraw, knd, vnd, kv, seq, pos, max(ctxs), cd, sd, nw[0], ns[0], nw[1],
                                            ns[1], ng, eps)
    assert torch.equal(out, ref)
    assert torch.equal(kv.k, k_ref) and torch.equal(kv.v, v_ref)
    np.testing.assert_array_equal(qraw.cpu().numpy(), q)


def test_attention_causal_prefill(qvl, cuda):
    """512 prompt tokens of one sequence: append all, then one causal pass."""
    T = 512
    rng = np.random.default_rng(8)
    kv = qvl.PagedKV(1, T, NH, NKV, D, 64, max_pos=T, device=cuda)
    cos, sin = oracle.rope_table(T, D, 5e6)
    q = rng.standard_normal((T, NH, D), dtype=np.float32)
    kn = rng.standard_normal((T, NKV, D), dtype=np.float32)
    vn = rng.standard_normal((T, NKV, D), dtype=np.float32)
    qd = dev(q, cuda)
    seq = torch.zeros(T, dtype=torch.int32, device=cuda)
    pos = torch.arange(T, dtype=torch.int32, device=cuda)
    qvl.rope_kv_append(qd, dev(kn, cuda), dev(vn, cuda), kv, seq, pos, dev(cos, cuda), dev(sin, cuda))
    out = qvl.attention(qd, kv, seq, pos, T).cpu().numpy()
    kc = np.zeros((NKV, T, D), np.float32)
    vc = np.zeros((NKV, T, D), np.float32)
    for t in range(T):
        kc[:, t] = oracle.rope_inplace(kn[t].copy(), cos[t], sin[t]).astype(np.float16).astype(np.float32)
        vc[:, t] = vn[t].astype(np.float16).astype(np.float32)
    for t in range(T):
        qt = oracle.rope_inplace(q[t].copy(), cos[t], sin[t])
        ref = oracle.attention(kc, vc, qt, t)
        assert rel_err(out[t], ref) < REL_TOL_FP32, t


def test_argmax_tie_and_nan(qvl, cuda):
    x = np.zeros((3, 5000), np.float32)
    x[0, [7, 4000]] = 5.0
    x[1, :] = np.nan
    x[1, 2] = 1.0
    x[2, :] = -np.inf
    idx = qvl.greedy_decode(dev(x, cuda)).cpu().numpy()
    assert list(idx) == [oracle.argmax(r) for r in x] == [7, 2, 0]


# ------------------------------------------------------------ tensor-core GEMM
@pytest.mark.parametrize("M,N,K", [(16, 128, 128), (32, 2048, 2048), (32, 1024, 2048), (32, 2048, 6144),
                                   (17, 256, 1024), (48, 6144, 2048), (512, 2048, 2048), (512, 1024, 2048), (512, 6144, 2048),
                                   (512, 2048, 6144), (130, 2048, 2048), (2048, 256, 2048), (77, 300, 1024),
                                   (454, 1024, 2048), (454, 6144, 2048),
                                   (1024, 6144, 2048), (600, 8192, 1024)])
def test_linear_prefill_tensor_core_bit_exact(qvl, cuda, M, N, K):
    """M >= 16 with per-row scales runs the tcgen05 kind::i8 GEMM (hi/lo split
    of the int16 activations); TILED order, bit-exact with the oracle.  The
    last two shapes have >= 2 waves of 128 x 128 tiles and take the
    persistent kernel (double-buffered accumulators; 600 rows: a ragged
    activation tile)."""
    x, w, ws = make_linear_inputs(7 * M + N, M, N, K, K)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=False)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, K, oracle.TILED, threads=16))


@pytest.mark.parametrize("M,N,K,g", [(16, 256, 1024, 32), (48, 2048, 2048, 64), (64, 2048, 2048, 128),
                                     (130, 1024, 2048, 64), (77, 300, 1024, 256), (200, 512, 2048, 512),
                                     (512, 2048, 2048, 128), (512, 6144, 2048, 128), (452, 2048, 6144, 128),
                                     (512, 1024, 2048, 32), (256, 2048, 2048, 64)])
def test_linear_grouped_tensor_core_bit_exact(qvl, cuda, M, N, K, g):
    """Group-wise scales at M >= 16 run the group-wise tcgen05 kernel: exact
    integer sums per group, acc = fma(float(S) * a_s, w_s, acc) over the
    groups in order (TILED), bit-exact with the oracle; ragged M and N."""
    x, w, ws = make_linear_inputs(11 * M + N + g, M, N, K, g)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=True, group_size=g)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, g, oracle.TILED, threads=16))


def test_linear_persistent_tensor_core_accumulate(qvl, cuda):
    """C += product on the persistent tensor-core path (the reference's
    add_vector after linear()), bit-exact."""
    M, N, K = 600, 8192, 1024
    x, w, ws = make_linear_inputs(99, M, N, K, K)
    q, qs = qvl.quantize_rows(dev(x, cuda), K)
    c0 = np.random.default_rng(5).standard_normal((M, N), dtype=np.float32)
    c = dev(c0.copy(), cuda)
    qvl.linear_batched(q, qs, [(dev(w, cuda), dev(ws, cuda))], [c], qvl.Workspace(cuda),
                       semantics=qvl.SEM_TILED | qvl.SEM_ACCUMULATE)
    want = (c0 + oracle.linear_i8(x, w, ws, K, oracle.TILED, threads=16)).astype(np.float32)
    np.testing.assert_array_equal(c.cpu().numpy(), want)


@pytest.mark.parametrize("M", [64, 512])
def test_linear_prefill_lm_head_rows(qvl, cuda, M):
    """LM head (N=151936) on the tensor cores: all columns of a spread of 64
    rows (config 1 at M=512), bit-exact against the TILED order."""
    x, w, ws = make_linear_inputs(3 + M, M, 151936, 2048, 2048)
    y = qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=False).cpu().numpy()
    rows = np.unique(np.concatenate([[0, M - 1], np.random.default_rng(M).choice(M, 62, replace=False)]))
    ref = oracle.linear_i8(x[rows], w, ws, 2048, oracle.TILED, threads=16)
    np.testing.assert_array_equal(y[rows], ref)


def test_tc_timeout_word_skips_and_reports(qvl, cuda):
    """A raised tensor-core timeout word (what a wait that gave up leaves):
    the next tensor-core product computes nothing and the host sees the word;
    cleared, the path computes again.  No wait is made to time out."""
    x, w, ws = make_linear_inputs(11, 32, 256, 1024, 1024)
    L = qvl.load_library()
    assert not qvl.tc_timed_out()
    assert L.qvl_internal_set_tc_timeout(torch.cuda.current_stream().cuda_stream) == 0
    y = torch.full((32, 256), float("nan"), device=cuda)
    qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=False, C=y)
    assert torch.isnan(y).all()
    assert qvl.tc_timed_out(clear=True)
    assert not qvl.tc_timed_out()
    qvl.linear(dev(x, cuda), dev(w, cuda), dev(ws, cuda), group_quantized=False, C=y)
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.linear_i8(x, w, ws, 1024, oracle.TILED))


@pytest.mark.parametrize("ctxs", [[300], [1, 700], [9000]])
def test_attention_with_fused_quantisation(qvl, cuda, ctxs):
    """attention_q16 == attention followed by quantize_rows (bit-exact),
    on the single-launch path and on the split-K path."""
    kv, _, q, kn, vn, cos, sin = _attn_setup(qvl, cuda, ctxs, seed=3)
    B = len(ctxs)
    qd = dev(q, cuda)
    seq = torch.arange(B, dtype=torch.int32, device=cuda)
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32, device=cuda)
    qvl.rope_kv_append(qd, dev(kn, cuda), dev(vn, cuda), kv, seq, pos, dev(cos, cuda), dev(sin, cuda))
    out = torch.empty_like(qd)
    q16 = torch.empty((B, NH * D), dtype=torch.int16, device=cuda)
    s16 = torch.empty((B, 1), dtype=torch.float32, device=cuda)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):
        qvl.attention_q16(qd, kv, seq, pos, max(ctxs), out, q16, s16, counter)
    ref = qvl.attention(qd, kv, seq, pos, max(ctxs))
    rq, rs = qvl.quantize_rows(ref.view(B, -1), NH * D)
    assert torch.equal(out, ref)
    assert torch.equal(q16, rq) and torch.equal(s16, rs)
    assert int(counter.item()) == 0


@pytest.mark.parametrize("M,K", [(32, 2048), (452, 6144), (16, 1024)])
def test_quantize_rows_planes(qvl, cuda, M, K):
    """The quantisation that also writes the tensor-core planes: q and the
    scales equal quantize_rows, hi = q >> 8 and lo = q & 255 exactly."""
    x = np.random.default_rng(M + K).standard_normal((M, K), dtype=np.float32)
    q0, s0 = qvl.quantize_rows(dev(x, cuda), K)
    q = torch.empty((M, K), dtype=torch.int16, device=cuda)
    s = torch.empty((M, 1), dtype=torch.float32, device=cuda)
    P = qvl.Planes(M, K, cuda)
    qvl.quantize_rows_planes(dev(x, cuda), q, s, P)
    np.testing.assert_array_equal(q.cpu().numpy(), q0.cpu().numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), s0.cpu().numpy())
    qn = q.cpu().numpy().astype(np.int32).reshape(-1)
    np.testing.assert_array_equal(P.hi.cpu().numpy()[:M * K].astype(np.int32), qn >> 8)
    np.testing.assert_array_equal(P.lo.cpu().numpy()[:M * K].astype(np.int32), qn & 255)


def test_rms_norm_planes_matches_rms_norm(qvl, cuda):
    M, H, ng = 32, 2048, 128
    rng = np.random.default_rng(77)
    x = rng.standard_normal((M, H), dtype=np.float32)
    w = rng.integers(-127, 128, H, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, H // ng).astype(np.float32)
    q0 = torch.empty((M, H), dtype=torch.int16, device=cuda)
    s0 = torch.empty((M, 1), dtype=torch.float32, device=cuda)
    qvl.rms_norm_i8(dev(x, cuda), dev(w, cuda), dev(ws, cuda), ng, 1e-6, q=q0, q_scales=s0, quant_group=H)
    q = torch.empty_like(q0)
    s = torch.empty_like(s0)
    P = qvl.Planes(M, H, cuda)
    qvl.rms_norm_i8_planes(dev(x, cuda), dev(w, cuda), dev(ws, cuda), ng, 1e-6, q, s, P)
    np.testing.assert_array_equal(q.cpu().numpy(), q0.cpu().numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), s0.cpu().numpy())
    qn = q.cpu().numpy().astype(np.int32).reshape(-1)
    np.testing.assert_array_equal(P.hi.cpu().numpy().astype(np.int32), qn >> 8)
    np.testing.assert_array_equal(P.lo.cpu().numpy().astype(np.int32), qn & 255)


@pytest.mark.parametrize("M,acc", [(32, False), (452, False), (32, True)])
def test_linear_planes_batched_three_matrices(qvl, cuda, M, acc):
    """q/k/v-shaped products of one set of planes in a single launch (weight
    tiles of the three matrices numbered one after the other), TILED order,
    bit-exact; with acc, C += product."""
    K = 2048
    rng = np.random.default_rng(M + 3)
    x = rng.standard_normal((M, K), dtype=np.float32)
    Ns = (2048, 1024, 1024)
    ws_ = [rng.integers(-127, 128, (n, K), dtype=np.int8) for n in Ns]
    ss = [rng.uniform(0.001, 0.02, n).astype(np.float32) for n in Ns]
    c0 = [rng.standard_normal((M, n), dtype=np.float32) for n in Ns]
    q = torch.empty((M, K), dtype=torch.int16, device=cuda)
    s = torch.empty((M, 1), dtype=torch.float32, device=cuda)
    P = qvl.Planes(M, K, cuda)
    qvl.quantize_rows_planes(dev(x, cuda), q, s, P)
    outs = [dev(c.copy(), cuda) if acc else torch.empty((M, n), device=cuda) for c, n in zip(c0, Ns)]
    qvl.linear_planes_batched(P, s, [(dev(w, cuda), dev(sc, cuda)) for w, sc in zip(ws_, ss)], outs, M, K,
                              semantics=qvl.SEM_TILED | (qvl.SEM_ACCUMULATE if acc else 0))
    for o, w, sc, c in zip(outs, ws_, ss, c0):
        want = oracle.linear_i8(x, w, sc, K, oracle.TILED, threads=16)
        if acc:
            want = (c + want).astype(np.float32)
        np.testing.assert_array_equal(o.cpu().numpy(), want)
