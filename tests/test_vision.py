"""The vision tower (qvl_b200.vision) against the reference's own forward_img
(oracle.RefModel: the reference's loader and forward_img compiled from its
sources), and its kernels against plain fp32 PyTorch references.

Bars: the tensor-core FP16 product within fp32-accumulation rounding of an
fp32 product of the same fp16 operands (fp16 outputs within one fp16 ulp
plus accumulation error); the whole tower within 1e-2 relative (fp16
intermediates, sums in a different order)."""
import numpy as np
import pytest
import torch

import oracle


def _vis(qvl):
    import qvl_b200.vision as V
    return V


def test_image_patches_layout(qvl):
    """Patch (gy, gx) in merge order holds channel c, frame t, row py, col px
    of pixel (16*gy + py, 16*gx + px) normalised as (p - 127.5) / 127.5."""
    V = _vis(qvl)
    rng = np.random.default_rng(1)
    img = rng.integers(0, 256, (64, 96, 3), dtype=np.uint8)
    p, gh, gw = V.image_patches(img)
    assert (gh, gw) == (4, 6) and p.shape == (24, 1536)
    for k in (0, 5, 13, 23):
        bh, bw = divmod(k // 4, gw // 2)
        ih, iw = divmod(k % 4, 2)
        gy, gx = 2 * bh + ih, 2 * bw + iw
        for c, t, py, px in ((0, 0, 0, 0), (2, 1, 15, 3), (1, 0, 7, 15)):
            want = (np.float32(img[16 * gy + py, 16 * gx + px, c]) - np.float32(127.5)) / np.float32(127.5)
            assert p[k, ((c * 2 + t) * 16 + py) * 16 + px] == want




@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(784, 1024, 1024), (784, 4096, 1024), (196, 2048, 4096), (77, 256, 192),
                                   (1, 128, 64), (600, 384, 320)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_gemm_f16_tensor_cores(qvl, cuda, M, N, K, mode):
    V = _vis(qvl)
    g = torch.Generator(device=cuda).manual_seed(M + N + K + mode)
    A = torch.randn(M, K, device=cuda, generator=g).half()
    W = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).half()
    b = (0.1 * torch.randn(N, device=cuda, generator=g)).half()
    ref = A.float() @ W.float().t() + b.float()
    if mode in (0, 1):
        C = torch.empty(M, N, dtype=torch.float16, device=cuda)
    else:
        C = torch.randn(M, N, device=cuda, generator=g) if mode == 3 else torch.empty(M, N, device=cuda)
    C0 = C.clone()
    V._lib()
    rc = qvl.load_library().qvl_gemm_f16(A.data_ptr(), W.data_ptr(), b.data_ptr(), C.data_ptr(), M, N, K, mode,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    if mode == 0:
        want = ref
    elif mode == 1:
        h = ref.half().float()
        want = 0.5 * h * (1.0 + torch.tanh(0.7978845608028654 * (h + 0.044715 * h * h * h)))
    elif mode == 2:
        want = ref
    else:
        want = C0 + ref.half().float()
    err = (C.float() - want).abs().max().item()
    tol = 2e-3 * max(1.0, want.abs().max().item())
    assert err <= tol, (err, tol)


@pytest.mark.gpu
def test_vision_attention_matches_torch(qvl, cuda):
    V = _vis(qvl)
    T, NH, HD = 784, 16, 64
    g = torch.Generator(device=cuda).manual_seed(3)
    q, k, v = (torch.randn(T, NH, HD, device=cuda, generator=g).half() for _ in range(3))
    out = torch.empty_like(q)
    V._lib()
    rc = qvl.load_library().qvl_vision_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), T, NH, HD,
                                                 0.125, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    s = torch.einsum("thd,shd->hts", q.float(), k.float()) * 0.125
    ref = torch.einsum("hts,shd->thd", torch.softmax(s, dim=-1), v.float())
    assert (out.float() - ref).abs().max().item() < 2e-3


@pytest.mark.gpu
def test_vision_tower_matches_reference_forward_img(qvl, cuda, tmp_path):
    """A 448x448 image (784 patches -> 196 tokens) through the full 24-layer
    tower: the image embeddings and the three deep-stack outputs against the
    reference's forward_img on the same model file and patches, within 1e-2
    of each output's largest magnitude."""
    if not oracle.ref_model_available():
        pytest.skip("reference model library (oracle/_ref) not built")
    import qvl_b200.modelfile as MF
    V = _vis(qvl)
    hdr = MF.qwen3vl_2b_header(num_hidden_layers=1, intermediate_size=256, vocab_size=1024)
    path = str(tmp_path / "vision.bin")
    MF.write_model_bin(path, hdr, MF.synthetic_text(hdr, seed=1), rng=np.random.default_rng(7))
    img = np.random.default_rng(0).integers(0, 256, (448, 448, 3), dtype=np.uint8)
    patches, gh, gw = V.image_patches(img)
    enc = V.VisionEncoder.from_file(path, gh, gw, device=cuda)
    out, deep = enc.forward(torch.from_numpy(patches).to(cuda))
    torch.cuda.synchronize()
    rm = oracle.RefModel(path)
    try:
        rx, rdeep = rm.forward_img(patches, gh, gw)
    finally:
        rm.close()
    got, gdeep = out.cpu().numpy(), deep.float().cpu().numpy()
    assert np.isfinite(got).all() and np.isfinite(gdeep).all()
    ex = np.abs(got - rx).max() / np.abs(rx).max()
    assert ex < 1e-2, ex
    for d in range(3):
        ed = np.abs(gdeep[d] - rdeep[d]).max() / np.abs(rdeep[d]).max()
        assert ed < 1e-2, (d, ed)
