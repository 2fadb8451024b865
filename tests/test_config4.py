"""BASELINE config 4 end to end: a synthetic 448x448 image and 256 text ids
through the whole Qwen3-VL-2B-shaped model read from one model file --
vision tower, prompt pass with the image embeddings and deep-stack rows, then
greedy decoding -- against the reference's own forward_text fed the same
prompt token by token.

The vision tower agrees with the reference's forward_img within 1e-2
(tests/test_vision.py); to compare the text side bit for bit, the
reference is given this tower's image embeddings and deep-stack rows
(oracle.RefModel.set_vision) in place of its own.  The prompt pass runs in
the reference's M=1 order (order="lane8") with reference-order attention, so
the logits of the last prompt position and of every generated token are
bit-identical."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_config4_image_prompt_then_greedy_decode(qvl, cuda, tmp_path):
    if not oracle.ref_model_available():
        pytest.skip("reference model library (oracle/_ref) not built")
    import qvl_b200.decoder as D
    import qvl_b200.modelfile as MF
    import qvl_b200.vision as V
    hdr = MF.qwen3vl_2b_header()
    path = str(tmp_path / "qwen3vl2b.bin")
    MF.write_model_bin(path, hdr, MF.synthetic_text(hdr, seed=4), rng=np.random.default_rng(8))
    rng = np.random.default_rng(12)
    img = rng.integers(0, 256, (448, 448, 3), dtype=np.uint8)
    patches, gh, gw = V.image_patches(img)
    enc = V.VisionEncoder.from_file(path, gh, gw, device=cuda)
    emb, deep = enc.forward(torch.from_numpy(patches).to(cuda))
    n_img = emb.shape[0]
    assert n_img == 196
    prompt = ([hdr["vision_start_token_id"]] + [hdr["image_token_id"]] * n_img + [hdr["vision_end_token_id"]] +
              rng.integers(0, 151643, 256).tolist())
    T = len(prompt)
    cfg, w = MF.load_text_weights(path, device=cuda)
    dec = D.TextDecoder(w, max_batch=1, max_ctx=1024, device=cuda, persistent=True)
    dec.prefill(torch.tensor(prompt, dtype=torch.int32, device=cuda), image_embeds=emb, deepstack=deep,
                order="lane8")
    torch.cuda.synchronize()
    rm = oracle.RefModel(path, fp16_kv=True)
    try:
        rm.set_vision(emb.cpu().numpy(), deep.float().cpu().numpy())
        for pos, tok in enumerate(prompt):
            ref = rm.forward(tok, pos)
        got = dec.logits[0].cpu().numpy()
        assert np.array_equal(got, ref), float(np.abs(got - ref).max())
        tok = oracle.argmax(ref)
        assert int(dec.tokens[0].item()) == tok
        ids = []
        for s in range(24):
            dec.step()
            torch.cuda.synchronize()
            ref = rm.forward(tok, T + s)
            got = dec.logits[0].cpu().numpy()
            assert np.array_equal(got, ref), (s, float(np.abs(got - ref).max()))
            tok = oracle.argmax(ref)
            assert int(dec.tokens[0].item()) == tok, s
            ids.append(tok)
        assert len(set(ids)) > 1
    finally:
        rm.close()
