"""Vision tower of Qwen3-VL on the sm_100a kernels (the reference's
forward_img, model/src/forward.cpp:3-456) and the host-side image
preprocessing it takes.

Per image of grid_h x grid_w patches (T = grid_h * grid_w, merged tokens
D = T / 4):

    patch embed (conv_3d) -> + interpolated position table -> 24 x [
      layer_norm -> q, k, v linear (+ 2-D rotary on q, k) -> attention ->
      proj linear + residual -> layer_norm -> fc1 linear + gelu_tanh ->
      fc2 linear + residual -> (layers 5, 11, 17: deep-stack merger on the
      stream viewed as [D, 4*VH]) ] -> layer_norm -> merger fc1 + gelu_tanh ->
    merger fc2 -> image embeddings [D, out_hidden] (fp32)

Weights are the model file's FP16 vision tensors (modelfile.map_vision_tensors)
in the exporter's [out, in] layout; every linear layer is one FP16
tensor-core product (qvl_gemm_f16) with its bias and the following gelu_tanh
or residual add fused into the epilogue.  Intermediates are fp16 where the
reference keeps them fp16 (vision_t, q, k, v, the MLP activations, the deep
stack) and fp32 where it keeps fp32 (the residual stream vision_x, the final
embeddings).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _check, _ptr, _stream, load_library
from .modelfile import map_vision_tensors, read_header

_P, _I, _Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
GEMM_F16, GEMM_F16_GELU, GEMM_F32, GEMM_ADD_F32 = 0, 1, 2, 3
DEEP_LAYERS = {5: 0, 11: 1, 17: 2}          # model/src/load_model.cpp:109-112
VISION_THETA = 10000.0                      # load_model.cpp:99
VISION_SCALE = 0.125                        # load_model.cpp:100
POS_GRID = 48                               # sqrt(2304 position embeddings)


def _lib():
    L = load_library()
    if not getattr(L, "_vision_bound", False):
        L.qvl_vision_rot_table.argtypes = [ctypes.c_float, _I, _I, _I, _I, _P, _P]
        L.qvl_vision_pos_interp.argtypes = [_I, _I, _I, _I, _P, _P]
        L.qvl_vision_patch_embed.argtypes = [_P, _P, _P, _P, _I, _I, _I, _P]
        L.qvl_vision_pos_add.argtypes = [_P, _P, _P, _P, _I, _I, _P]
        L.qvl_layer_norm.argtypes = [_P, _I, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P]
        L.qvl_gemm_f16.argtypes = [_P, _P, _P, _P, _Z, _Z, _Z, _I, _P]
        L.qvl_vision_rotary.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.qvl_vision_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P]
        L._vision_bound = True
    return L


def image_patches(rgb: np.ndarray, patch: int = 16, merge: int = 2, temporal: int = 2):
    """Host preprocessing of an RGB image whose sides are multiples of
    patch*merge (so the reference's smart_resize keeps its size,
    tokenizer/src/img_processor.cpp:36-76): HWC -> CHW, (x - 127.5) / 127.5
    per channel (normalize_inplace, :107-125), the frame duplicated `temporal`
    times (duplicate_to_batch, :165-185), then permute_8d with order
    (2,5,3,6,1,0,4,7) (:127-163) -> patches [grid_h*grid_w, C*temporal*patch*patch]
    in merge order.  Returns (patches fp32, grid_h, grid_w)."""
    img = np.asarray(rgb)
    H, W, C = img.shape
    if H % (patch * merge) or W % (patch * merge):
        raise ValueError("image sides must be multiples of patch*merge (resizing is not implemented)")
    chw = img.astype(np.float32).transpose(2, 0, 1)
    m, s = np.float32(127.5), np.float32(127.5)
    chw = (chw - m) / s
    batch = np.broadcast_to(chw, (temporal, C, H, W))
    gh, gw = H // patch, W // patch
    x = batch.reshape(temporal, C, gh // merge, merge, patch, gw // merge, merge, patch)
    x = x.transpose(2, 5, 3, 6, 1, 0, 4, 7)
    return np.ascontiguousarray(x.reshape(gh * gw, C * temporal * patch * patch), dtype=np.float32), gh, gw


class VisionEncoder:
    """forward_img on the GPU for images of one grid size."""

    @classmethod
    def from_file(cls, path: str, grid_h: int, grid_w: int, device="cuda"):
        """Weights from a model file's vision tower (vision_bits 16)."""
        vt = map_vision_tensors(path)
        if vt["patch_w"].dtype != np.float16:
            raise ValueError("vision_bits must be 16")
        dev = torch.device(device)
        return cls(read_header(path), {k: torch.from_numpy(np.array(v, copy=True)).to(dev) for k, v in vt.items()},
                   grid_h, grid_w, device)

    @classmethod
    def random(cls, header: dict, grid_h: int, grid_w: int, device="cuda", seed: int = 0):
        """Synthetic fp16 weights at the header's sizes, drawn on the device
        with the model-file writer's scales (no checkpoint is available)."""
        from .modelfile import vision_tensors
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        t = {}
        for name, shape in vision_tensors(header):
            r = torch.randn(shape, generator=g, device=dev)
            if name in ("norm1_w", "norm2_w") or name.endswith("norm_w"):
                r = 1.0 + 0.05 * r
            elif name.endswith("_b"):
                r = 0.02 * r
            elif name == "pos_w":
                r = 0.5 * r
            else:
                fan_in = shape[-1] if name != "patch_w" else int(np.prod(shape[1:]))
                r = r / float(np.sqrt(fan_in))
            t[name] = r.half()
        return cls(header, t, grid_h, grid_w, device)

    def __init__(self, header: dict, tensors: dict, grid_h: int, grid_w: int, device="cuda"):
        """header: the model file's header values; tensors: name -> fp16
        device tensor of the vision tower (modelfile.vision_tensors names and
        shapes, [out, in] layout)."""
        h = header
        self.h = h
        self.dev = dev = torch.device(device)
        self.VH, self.VI, self.OH = h["vision_hidden_size"], h["vision_intermediate_size"], h["out_hidden_size"]
        self.NH = h["vision_num_heads"]
        self.HD = self.VH // self.NH
        self.depth = h["vision_depth"]
        self.merge = h["vision_spatial_merge_size"]
        self.eps = float(np.float32(h["rms_norm_eps"]))
        self.gh, self.gw = grid_h, grid_w
        self.T = grid_h * grid_w
        self.D = self.T // (self.merge * self.merge)
        if self.merge * self.merge * self.VH != self.VI:
            raise ValueError("the deep-stack and merger layers take merge^2 * vision_hidden = vision_intermediate")
        self.w = dict(tensors)
        self.w["patch_w"] = self.w["patch_w"].reshape(self.VH, -1)
        L = _lib()
        T, HD = self.T, self.HD
        cs = np.empty((T, HD), np.uint16)
        sn = np.empty((T, HD), np.uint16)
        _check(L.qvl_vision_rot_table(VISION_THETA, HD, grid_h, grid_w, self.merge, cs.ctypes.data, sn.ctypes.data),
               "vision_rot_table")
        idx = np.empty((T, 4), np.int32)
        wt = np.empty((T, 4), np.float32)
        _check(L.qvl_vision_pos_interp(grid_h, grid_w, POS_GRID, self.merge, idx.ctypes.data, wt.ctypes.data),
               "vision_pos_interp")
        self.rot_cos = torch.from_numpy(cs.view(np.float16)).to(dev)
        self.rot_sin = torch.from_numpy(sn.view(np.float16)).to(dev)
        self.pos_idx = torch.from_numpy(idx).to(dev)
        self.pos_wt = torch.from_numpy(wt).to(dev)
        f16, f32 = torch.float16, torch.float32
        self.x = torch.empty((T, self.VH), dtype=f32, device=dev)
        self.t = torch.empty((T, self.VH), dtype=f16, device=dev)
        self.q = torch.empty((T, self.VH), dtype=f16, device=dev)
        self.k = torch.empty((T, self.VH), dtype=f16, device=dev)
        self.v = torch.empty((T, self.VH), dtype=f16, device=dev)
        self.att = torch.empty((T, self.VH), dtype=f16, device=dev)
        self.mlp = torch.empty((T, self.VI), dtype=f16, device=dev)
        self.deep = torch.empty((3, self.D, self.OH), dtype=f16, device=dev)
        self.out = torch.empty((self.D, self.OH), dtype=f32, device=dev)

    def _gemm(self, A, W, b, C, M, N, K, mode, stream):
        _check(_lib().qvl_gemm_f16(_ptr(A), _ptr(W), _ptr(b), _ptr(C), M, N, K, mode, stream), "gemm_f16")

    def _norm(self, x, x_f16, g, b, out, out_f16, rows, H, stream):
        _check(_lib().qvl_layer_norm(_ptr(x), int(x_f16), _ptr(g), _ptr(b), _ptr(out), int(out_f16), rows, H,
                                     self.eps, stream), "layer_norm")

    def forward(self, patches: torch.Tensor, stream=None):
        """patches fp32 [T, C*2*P*P] on the device -> (embeddings fp32 [D, OH],
        deep-stack fp16 [3, D, OH]); device work only."""
        L = _lib()
        st = _stream(stream)
        w = self.w
        T, D, VH, VI, OH = self.T, self.D, self.VH, self.VI, self.OH
        _check(L.qvl_vision_patch_embed(_ptr(patches), _ptr(w["patch_w"]), _ptr(w["patch_b"]), _ptr(self.x), T, VH,
                                        patches.shape[1], st), "patch_embed")
        _check(L.qvl_vision_pos_add(_ptr(self.x), _ptr(w["pos_w"]), _ptr(self.pos_idx), _ptr(self.pos_wt), T, VH, st),
               "pos_add")
        for l in range(self.depth):
            self._norm(self.x, False, w["norm1_w"][l], w["norm1_b"][l], self.t, True, T, VH, st)
            for j, dst in enumerate((self.q, self.k, self.v)):
                self._gemm(self.t, w["qkv_w"][l, j], w["qkv_b"][l, j], dst, T, VH, VH, GEMM_F16, st)
            for dst in (self.q, self.k):
                _check(L.qvl_vision_rotary(_ptr(dst), _ptr(self.rot_cos), _ptr(self.rot_sin), T, self.NH, self.HD, st),
                       "vision_rotary")
            _check(L.qvl_vision_attention(_ptr(self.q), _ptr(self.k), _ptr(self.v), _ptr(self.att), T, self.NH,
                                          self.HD, VISION_SCALE, st), "vision_attention")
            self._gemm(self.att, w["proj_w"][l], w["proj_b"][l], self.x, T, VH, VH, GEMM_ADD_F32, st)
            self._norm(self.x, False, w["norm2_w"][l], w["norm2_b"][l], self.t, True, T, VH, st)
            self._gemm(self.t, w["mlp1_w"][l], w["mlp1_b"][l], self.mlp, T, VI, VH, GEMM_F16_GELU, st)
            self._gemm(self.mlp, w["mlp2_w"][l], w["mlp2_b"][l], self.x, T, VH, VI, GEMM_ADD_F32, st)
            if l in DEEP_LAYERS:
                d = DEEP_LAYERS[l]
                # the stream viewed as [D, merge^2 * VH]: four neighbouring patches per row
                self._norm(self.x, False, w["d_norm_w"][d], w["d_norm_b"][d], self.t, True, D, VI, st)
                self._gemm(self.t, w["d_mlp1_w"][d], w["d_mlp1_b"][d], self.mlp, D, VI, VI, GEMM_F16_GELU, st)
                self._gemm(self.mlp, w["d_mlp2_w"][d], w["d_mlp2_b"][d], self.deep[d], D, OH, VI, GEMM_F16, st)
        self._norm(self.x, False, w["merge_norm_w"], w["merge_norm_b"], self.t, True, T, VH, st)
        self._gemm(self.t, w["merge_mlp1_w"], w["merge_mlp1_b"], self.mlp, D, VI, VI, GEMM_F16_GELU, st)
        self._gemm(self.mlp, w["merge_mlp2_w"], w["merge_mlp2_b"], self.out, D, OH, VI, GEMM_F32, st)
        return self.out, self.deep
