"""Pins the C restatement (oracle/oracle.c) to the reference engine: against
the committed golden vectors (made by tests/golden/make_golden.py from the
reference's own compiled code) and, where oracle/_ref was built, against the
compiled reference live on fresh seeds."""
import hashlib
import os

import numpy as np
import pytest

import oracle
from conftest import make_linear_inputs

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
from golden.make_golden import LINEAR_CASES, attention_case  # noqa: E402


def _sha(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.digest()


@pytest.mark.parametrize("case", LINEAR_CASES, ids=[c[0] for c in LINEAR_CASES])
def test_linear_golden_bit_exact(case):
    name, seed, M, N, K, g = case
    x, w, ws = make_linear_inputs(seed, M, N, K, g)
    assert _sha(x, w, ws) == GOLD[f"{name}/sha"].tobytes(), "input generator drifted"
    y = oracle.linear_i8(x, w, ws, g)
    np.testing.assert_array_equal(y, GOLD[f"{name}/y"])


def test_softmax_golden():
    np.testing.assert_array_equal(oracle.softmax(GOLD["softmax/x"]), GOLD["softmax/y"])


def test_swiglu_golden():
    np.testing.assert_array_equal(oracle.swiglu(GOLD["swiglu/gate"], GOLD["swiglu/up"]), GOLD["swiglu/y"])


def test_rope_golden():
    c, s = oracle.rope_table(256)
    y = oracle.rope_inplace(GOLD["rope/x"].copy(), c[201], s[201])
    np.testing.assert_array_equal(y, GOLD["rope/y"])


@pytest.mark.parametrize("seed", [31, 32, 33])
def test_attention_golden(seed):
    S, pos = GOLD[f"attn_{seed}/meta"]
    kc, vc, q = attention_case(seed, int(S), int(pos))
    y = oracle.attention(kc, vc, q, int(pos))
    np.testing.assert_array_equal(y, GOLD[f"attn_{seed}/y"])


def test_group_sums_exact():
    x, w, ws = make_linear_inputs(5, 2, 8, 256, 64)
    q, s = oracle.quantize(x, 64)
    gs = oracle.group_sums(q, w, 64)
    expect = (q.astype(np.int64)[:, None, :] * w.astype(np.int64)[None, :, :]).reshape(2, 8, 4, 64).sum(-1)
    np.testing.assert_array_equal(gs, expect)


def test_exp_ref_properties():
    # exact at 0, under-approximates e^x by < 8e-4 relative in the normal range
    assert oracle.exp_ref(0.0) == 1.0
    for x in np.linspace(-20, 20, 101):
        r = oracle.exp_ref(float(x))
        assert abs(r - np.exp(x)) / np.exp(x) < 8e-4


def test_argmax_first_index():
    v = np.array([1.0, 3.0, -1.0, 3.0, np.nan], np.float32)
    assert oracle.argmax(v) == 1
    assert oracle.argmax(np.full(5, -np.inf, np.float32)) == 0


ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


@ref
@pytest.mark.parametrize("M,N,K,g", [(1, 2048, 2048, 2048), (1, 6144, 2048, 128), (1, 2048, 6144, 6144),
                                     (4, 300, 1024, 128), (7, 64, 512, 32), (1, 70000, 2048, 2048)])
def test_linear_vs_compiled_reference(M, N, K, g):
    x, w, ws = make_linear_inputs(100 + M + g, M, N, K, g)
    np.testing.assert_array_equal(oracle.linear_i8(x, w, ws, g), oracle.ref_i8_kernel(x, w, ws, g))


@ref
def test_reference_tiled_kernel_zero_bug_is_real():
    """The reference's tiled M>1 kernel returns zeros when g > 256
    (cpu_f32a_i8f32sb_f32c_avx2.cpp:543); the restatement implements the
    intended arithmetic instead."""
    x, w, ws = make_linear_inputs(7, 2, 64, 512, 512)
    assert not oracle.ref_i8_kernel(x, w, ws, 512).any()
    assert oracle.linear_i8(x, w, ws, 512).any()


@ref
@pytest.mark.parametrize("pos", [0, 5, 7, 8, 15, 63, 200, 255])
def test_attention_vs_compiled_reference(pos):
    kc, vc, q = attention_case(pos, 256, pos)
    a = oracle.attention(kc, vc, q, pos)
    b = oracle.ref_attention(kc, vc, q, pos)
    np.testing.assert_array_equal(a, b)


@ref
def test_softmax_swiglu_vs_compiled_reference():
    rng = np.random.default_rng(3)
    for n in (1, 7, 8, 9, 4097):
        v = rng.standard_normal(n, dtype=np.float32) * 10
        np.testing.assert_array_equal(oracle.softmax(v), oracle.ref_softmax(v))
    g = rng.standard_normal(6144, dtype=np.float32) * 5
    u = rng.standard_normal(6144, dtype=np.float32)
    np.testing.assert_array_equal(oracle.swiglu(g, u), oracle.ref_swiglu(g, u))


@ref
@pytest.mark.parametrize("H,gs,B", [(2048, 128, 3), (128, 128, 24), (128, 64, 16), (6144, 128, 1)])
@pytest.mark.parametrize("inplace", [False, True])
def test_rms_norm_i8_vs_compiled_reference(H, gs, B, inplace):
    rng = np.random.default_rng(H + B)
    x = (rng.standard_normal((B, H)) * rng.uniform(0.1, 30)).astype(np.float32)
    wq = rng.integers(-127, 128, H).astype(np.int8)
    ws = rng.uniform(0.001, 0.02, H // gs).astype(np.float32)
    np.testing.assert_array_equal(oracle.rms_norm_i8(x, wq, ws, gs, 1e-6, inplace),
                                  oracle.ref_rms_norm_i8(x, wq, ws, gs, 1e-6, inplace))


@ref
def test_embedding_vs_compiled_reference():
    rng = np.random.default_rng(2)
    t = rng.integers(-127, 128, (100, 2048)).astype(np.int8)
    s = rng.uniform(0.001, 0.02, 100).astype(np.float32)
    np.testing.assert_array_equal(oracle.embedding_i8(t, s, 37), oracle.ref_embedding_i8(t, s, 37))
