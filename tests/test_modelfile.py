"""The .bin model-file reader (qvl_b200.modelfile) against the reference's
exporter and loader, and the end-to-end oracle (oracle.RefModel: the
reference's own init_model_weights + qwen_rope_precompute + forward_text)
against the operator-by-operator composition the GPU tests use
(oracle/decode.py).  CPU only."""
import os
import sys

import numpy as np
import pytest

import oracle
from oracle.decode import CpuDecoder

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_exporter_fixture as FX  # noqa: E402


def _mf(qvl):
    import qvl_b200.modelfile as MF
    return MF


def _exporter_quantize(x, name, group_quantized, group):
    """export_qwen_bin.py:242-275 (quantize_rowwise / quantize_groupwise), 8 bits."""
    if group_quantized or "norm" in name:
        x2 = x.reshape(-1, group)
    else:
        x2 = x.reshape(-1, x.shape[-1])
    scales = (np.max(np.abs(x2), axis=1, keepdims=True) + np.float32(1e-8)) / np.float32(127)
    q = np.clip(np.round(x2 / scales).astype(np.int8), -127, 127)
    return q.reshape(x.shape), scales.ravel().astype(np.float32)


_HF = {"embed": "embed_tokens.weight", "final_norm": "norm.weight", "in_norm": "input_layernorm.weight",
       "post_norm": "post_attention_layernorm.weight", "wd": "mlp.down_proj.weight", "wg": "mlp.gate_proj.weight",
       "wu": "mlp.up_proj.weight", "k_norm": "self_attn.k_norm.weight", "q_norm": "self_attn.q_norm.weight",
       "wk": "self_attn.k_proj.weight", "wo": "self_attn.o_proj.weight", "wq": "self_attn.q_proj.weight",
       "wv": "self_attn.v_proj.weight"}


@pytest.mark.parametrize("tag,gq", [("rowwise", 0), ("g32", 1)])
def test_reader_matches_reference_exporter(qvl, tag, gq):
    """A file written by the reference's own exporter (committed fixture, made
    by tests/golden/make_exporter_fixture.py): header and every text tensor's
    int8 values and scales read back as the exporter quantised them."""
    MF = _mf(qvl)
    tt = MF.map_text_tensors(os.path.join(HERE, "golden", f"exporter_small_{tag}.bin"))
    h = tt.header
    d = FX.DIMS
    assert (h["vocab_size"], h["hidden_size"], h["intermediate_size"], h["num_hidden_layers"]) == \
        (d["vocab_size"], d["hidden_size"], d["intermediate_size"], d["num_hidden_layers"])
    assert (h["text_bits"], h["group_size"], h["vision_bits"], h["group_quantized"]) == (8, 32, 16, gq)
    assert h["rope_theta"] == 5000000 and np.float32(h["rms_norm_eps"]) == np.float32(1e-6)
    st = FX.synthetic_state()
    for name, (data, scales, _) in tt.tensors.items():
        hf = _HF[name]
        if name in ("embed", "final_norm"):
            x = st["model.language_model." + hf]
        else:
            x = np.stack([st[f"model.language_model.layers.{i}.{hf}"] for i in range(d["num_hidden_layers"])])
        if x.ndim == 3 and not gq and "norm" not in name:
            parts = [_exporter_quantize(x[i], name, gq, 32) for i in range(x.shape[0])]
            q, s = np.stack([p[0] for p in parts]), np.concatenate([p[1] for p in parts])
        else:
            q, s = _exporter_quantize(x, name, gq, 32)
        np.testing.assert_array_equal(data, q, err_msg=name)
        np.testing.assert_array_equal(scales, s, err_msg=name)


def _small_header(MF, **over):
    return MF.qwen3vl_2b_header(vocab_size=1000, hidden_size=512, intermediate_size=768, num_hidden_layers=2,
                                num_attention_heads=4, num_key_value_heads=2, vision_hidden_size=32,
                                vision_intermediate_size=64, vision_num_heads=2, out_hidden_size=512,
                                group_size=32, **over)


def test_write_read_roundtrip(qvl, tmp_path):
    MF = _mf(qvl)
    hdr = _small_header(MF)
    text = MF.synthetic_text(hdr, seed=1)
    p = str(tmp_path / "m.bin")
    MF.write_model_bin(p, hdr, text)
    tt = MF.map_text_tensors(p)
    for k, (data, scales, _) in tt.tensors.items():
        np.testing.assert_array_equal(data, text[k][0])
        np.testing.assert_array_equal(scales, text[k][1])
    assert os.path.getsize(p) == MF.HEADER_BYTES + sum(a.nbytes + s.nbytes for a, s in text.values()) + \
        2 * sum(int(np.prod(s)) for s in MF.vision_shapes(hdr))


def test_rope_table_is_the_reference_precompute(qvl, tmp_path):
    """The product's RoPE table (host libm) equals qwen_rope_precompute's text
    section, and the C restatement equals both."""
    if not oracle.ref_model_available():
        pytest.skip("reference model library not built")
    import qvl_b200.decoder as D
    MF = _mf(qvl)
    hdr = _small_header(MF)
    p = str(tmp_path / "m.bin")
    MF.write_model_bin(p, hdr, MF.synthetic_text(hdr, seed=2))
    rm = oracle.RefModel(p)
    try:
        rc, rs = rm.rope(rm.seq_len)
        gc, gs = D.rope_table(rm.seq_len, rm.head_dim, rm.rope_theta)
        np.testing.assert_array_equal(gc, rc)
        np.testing.assert_array_equal(gs, rs)
        oc, os_ = oracle.rope_table(rm.seq_len, rm.head_dim, rm.rope_theta)
        np.testing.assert_array_equal(oc, rc)
        np.testing.assert_array_equal(os_, rs)
    finally:
        rm.close()


def test_forward_text_equals_operator_composition(qvl, tmp_path):
    """The reference's own forward_text (loaded from a .bin through its own
    loader) and the operator-by-operator composition of oracle/decode.py give
    bit-identical logits over 12 greedy steps: the composition the GPU tests
    use is the reference's decoder."""
    if not oracle.ref_model_available():
        pytest.skip("reference model library not built")
    import qvl_b200.decoder as D
    MF = _mf(qvl)
    hdr = _small_header(MF)
    p = str(tmp_path / "m.bin")
    MF.write_model_bin(p, hdr, MF.synthetic_text(hdr, seed=3))
    tt = MF.map_text_tensors(p)
    rm = oracle.RefModel(p)
    try:
        cfg = D.TextConfig(hidden=512, intermediate=768, layers=2, heads=4, kv_heads=2, head_dim=128, vocab=1000,
                           eps=rm.eps, norm_group=32)
        w = {}
        for k, (data, scales, stride) in tt.tensors.items():
            w[k] = np.ascontiguousarray(data)
            w[k + "_s"] = np.ascontiguousarray(scales.reshape(
                data.shape[:-1] + ((data.shape[-1] // stride,) if k.endswith("norm") else ())))
        cos, sin = rm.rope(rm.seq_len)
        cpu = CpuDecoder(cfg, w, rm.seq_len, cos, sin, backend="ref")
        tok = 17
        for pos in range(12):
            a = rm.forward(tok, pos)
            b, t = cpu.step(tok, pos)
            np.testing.assert_array_equal(a, b, err_msg=f"pos {pos}")
            assert oracle.argmax(a) == t
            tok = t
    finally:
        rm.close()
