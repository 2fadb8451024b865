"""Model files in the exporter's .bin layout, read into device memory.

Layout (written by export_bin/export_qwen_bin.py, read by the reference's
init_model_weights, model/src/load_model.cpp:50-246):

* header: 21 little-endian values in the exporter's KEYS order
  (export_qwen_bin.py:36-60) -- rms_norm_eps as float32, the others int32 --
  then text_bits, group_size, vision_bits, group_quantized as int32
  (:395-401; load_model.cpp:63-93).
* then one group per weight kind, in the exporter's key order
  (reorder_keys_for_write / reorder_keys_by_group, :84-212): the embedding;
  per layer kind, all layers stacked; the final norm; the vision tower.  For
  INT8 a group holds ALL its scales (fp32) first, then ALL its int8 data
  (write_weights_streaming, :297-357); FP16/FP32 tensors have data only.
* INT8 scales: per output row ([N] per layer) for a per-row export, per
  `group_size` consecutive values for a group-wise export; norm weights are
  always group-wise (:325; the loader's gq_force, load_model.cpp:185-196).

The text-weight order the loader maps (load_model.cpp:184-196) is
embed, input_layernorm (its rms_ffn_w), down, gate, up,
post_attention_layernorm (its rms_attn_w), k_norm, k, o, q_norm, q, v, norm.

`load_text_weights` reads the header and the text tensors straight from the
file (memory-mapped) into device buffers in the layout the kernels take; the
vision tower is skipped by size.  `write_model_bin` writes a synthetic model
in the same layout (int8 weights and scales given directly), e.g. for tests
and benchmarks without a checkpoint.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np
import torch

HEADER_KEYS = (
    "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
    "num_key_value_heads", "max_position_embeddings", "rope_theta", "rms_norm_eps",
    "vision_hidden_size", "vision_depth", "vision_patch_size", "vision_spatial_merge_size",
    "vision_temporal_patch_size", "vision_num_heads", "vision_intermediate_size", "out_hidden_size",
    "image_token_id", "vision_start_token_id", "vision_end_token_id", "video_token_id",
)
QUANT_KEYS = ("text_bits", "group_size", "vision_bits", "group_quantized")
HEADER_BYTES = 4 * (len(HEADER_KEYS) + len(QUANT_KEYS))

# text tensors in file order: (name used by the decoder, shape builder, is_norm)
_TEXT_ORDER = (
    ("embed", lambda c: (c["vocab_size"], c["hidden_size"]), False),
    ("in_norm", lambda c: (c["num_hidden_layers"], c["hidden_size"]), True),
    ("wd", lambda c: (c["num_hidden_layers"], c["hidden_size"], c["intermediate_size"]), False),
    ("wg", lambda c: (c["num_hidden_layers"], c["intermediate_size"], c["hidden_size"]), False),
    ("wu", lambda c: (c["num_hidden_layers"], c["intermediate_size"], c["hidden_size"]), False),
    ("post_norm", lambda c: (c["num_hidden_layers"], c["hidden_size"]), True),
    ("k_norm", lambda c: (c["num_hidden_layers"], _head_dim(c)), True),
    ("wk", lambda c: (c["num_hidden_layers"], c["num_key_value_heads"] * _head_dim(c), c["hidden_size"]), False),
    ("wo", lambda c: (c["num_hidden_layers"], c["hidden_size"], c["hidden_size"]), False),
    ("q_norm", lambda c: (c["num_hidden_layers"], _head_dim(c)), True),
    ("wq", lambda c: (c["num_hidden_layers"], c["num_attention_heads"] * _head_dim(c), c["hidden_size"]), False),
    ("wv", lambda c: (c["num_hidden_layers"], c["num_key_value_heads"] * _head_dim(c), c["hidden_size"]), False),
    ("final_norm", lambda c: (c["hidden_size"],), True),
)


def _head_dim(c):
    return c["hidden_size"] // c["num_attention_heads"]


class ModelFileError(ValueError):
    pass


def read_header(path: str) -> dict:
    with open(path, "rb") as f:
        raw = f.read(HEADER_BYTES)
    if len(raw) < HEADER_BYTES:
        raise ModelFileError(f"{path}: shorter than the {HEADER_BYTES}-byte header")
    vals = {}
    for i, k in enumerate(HEADER_KEYS + QUANT_KEYS):
        fmt = "<f" if k == "rms_norm_eps" else "<i"
        vals[k] = struct.unpack_from(fmt, raw, 4 * i)[0]
    return vals


def _scale_count(name, shape, hdr):
    n = int(np.prod(shape))
    stride = hdr["group_size"] if (hdr["group_quantized"] or _is_norm(name)) else shape[-1]
    if stride <= 0 or n % stride:
        raise ModelFileError(f"{name}: {n} values do not split into groups of {stride}")
    return n // stride, stride


def _is_norm(name):
    return name.endswith("norm")


@dataclasses.dataclass
class TextTensors:
    """Host views (memory-mapped) of the text tensors: name -> (int8 data
    shaped like the tensor, fp32 scales, values per scale)."""
    header: dict
    tensors: dict


def map_text_tensors(path: str) -> TextTensors:
    hdr = read_header(path)
    if hdr["text_bits"] != 8:
        raise ModelFileError(f"text_bits={hdr['text_bits']}: the B200 path runs INT8 text weights only")
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    off = HEADER_BYTES
    out = {}
    for name, shp, _ in _TEXT_ORDER:
        shape = tuple(int(v) for v in shp(hdr))
        count = int(np.prod(shape))
        ns, stride = _scale_count(name, shape, hdr)
        if off + 4 * ns + count > mm.size:
            raise ModelFileError(f"{path}: truncated at {name}")
        scales = mm[off:off + 4 * ns].view(np.float32)
        off += 4 * ns
        data = mm[off:off + count].view(np.int8).reshape(shape)
        off += count
        out[name] = (data, scales, stride)
    return TextTensors(hdr, out)


def load_text_weights(path: str, device="cuda"):
    """Text decoder of a .bin model file -> (TextConfig, TextWeights) on
    `device`.  Per-row exports give the per-output-row scale layout the
    decoder runs ([L, N] per matrix); norm weights keep their group scales."""
    from .decoder import TextConfig, TextWeights
    tt = map_text_tensors(path)
    hdr = tt.header
    if hdr["group_quantized"]:
        raise ModelFileError("group-quantised text weights: the decoder runs per-row INT8 exports "
                             "(group_quantized = 0); use map_text_tensors for the raw tensors")
    L = hdr["num_hidden_layers"]
    cfg = TextConfig(hidden=hdr["hidden_size"], intermediate=hdr["intermediate_size"], layers=L,
                     heads=hdr["num_attention_heads"], kv_heads=hdr["num_key_value_heads"],
                     head_dim=_head_dim(hdr), vocab=hdr["vocab_size"], eps=float(np.float32(hdr["rms_norm_eps"])),
                     rope_theta=float(hdr["rope_theta"]), norm_group=hdr["group_size"])
    t = {}
    for name, (data, scales, stride) in tt.tensors.items():
        dt = torch.from_numpy(np.array(data, copy=True)).to(device)
        if _is_norm(name):
            st = scales.reshape(data.shape[:-1] + (data.shape[-1] // stride,))
        else:
            st = scales.reshape(data.shape[:-1])                  # one scale per output row
        t[name] = dt
        t[name + "_s"] = torch.from_numpy(np.array(st, copy=True)).to(device)
    return cfg, TextWeights(cfg, t)


def write_model_bin(path: str, header: dict, text: dict, vision_bits: int = 16, rng=None):
    """Write a model in the exporter's layout.  `header`: the 21 KEYS values
    plus group_size and group_quantized (text_bits is 8).  `text`: decoder
    name -> (int8 array of the tensor's shape, fp32 scales) for every entry
    of the text order.  The vision tower (FP16 or FP32, vision_bits) is
    written with small random values drawn from `rng` at the header's vision
    sizes, in the loader's order (load_model.cpp:199-246)."""
    rng = rng or np.random.default_rng(0)
    hdr = dict(header)
    hdr["text_bits"] = 8
    hdr["vision_bits"] = vision_bits
    with open(path, "wb") as f:
        for k in HEADER_KEYS:
            f.write(struct.pack("<f" if k == "rms_norm_eps" else "<i", hdr[k]))
        for k in QUANT_KEYS:
            f.write(struct.pack("<i", int(hdr[k])))
        for name, shp, _ in _TEXT_ORDER:
            shape = tuple(int(v) for v in shp(hdr))
            data, scales = text[name]
            ns, _ = _scale_count(name, shape, hdr)
            data = np.ascontiguousarray(data, dtype=np.int8)
            scales = np.ascontiguousarray(scales, dtype=np.float32).ravel()
            if data.shape != shape or scales.size != ns:
                raise ModelFileError(f"{name}: expected {shape} / {ns} scales, got {data.shape} / {scales.size}")
            f.write(scales.tobytes())
            f.write(data.tobytes())
        fdt = np.float16 if vision_bits == 16 else np.float32
        for name, shape in vision_tensors(hdr):
            f.write(_vision_init(name, shape, rng).astype(fdt).tobytes())


_VISION_ORDER = ("patch_b", "patch_w", "pos_w", "proj_b", "proj_w", "qkv_b", "qkv_w", "mlp1_b", "mlp1_w",
                 "mlp2_b", "mlp2_w", "norm1_b", "norm1_w", "norm2_b", "norm2_w", "d_mlp1_b", "d_mlp1_w",
                 "d_mlp2_b", "d_mlp2_w", "d_norm_b", "d_norm_w", "merge_mlp1_b", "merge_mlp1_w",
                 "merge_mlp2_b", "merge_mlp2_w", "merge_norm_b", "merge_norm_w")


def vision_tensors(h: dict):
    """(name, shape) of the vision-tower tensors in file order
    (load_model.cpp:199-246; 2304 position embeddings, 3 channels and 3
    deep-stack mergers are fixed there).  Matrices keep the exporter's
    [out, in] layout."""
    return list(zip(_VISION_ORDER, vision_shapes(h)))


def _vision_init(name, shape, rng):
    """Synthetic values that keep activations O(1): matrices ~N(0, 1/fan_in),
    biases ~N(0, 0.02^2), norm weights ~1 + N(0, 0.05^2), position table ~N(0, 0.5^2)."""
    n = int(np.prod(shape))
    if name.endswith("norm_w") or name in ("norm1_w", "norm2_w"):
        return 1.0 + 0.05 * rng.standard_normal(n, dtype=np.float32)
    if name.endswith("_b"):
        return 0.02 * rng.standard_normal(n, dtype=np.float32)
    if name == "pos_w":
        return 0.5 * rng.standard_normal(n, dtype=np.float32)
    fan_in = shape[-1] if name != "patch_w" else int(np.prod(shape[1:]))
    return rng.standard_normal(n, dtype=np.float32) / np.float32(np.sqrt(fan_in))


def vision_shapes(h: dict):
    """Shapes of the vision-tower tensors in file order (load_model.cpp:199-246)."""
    VH, VD, VI = h["vision_hidden_size"], h["vision_depth"], h["vision_intermediate_size"]
    VP, VTP, OH = h["vision_patch_size"], h["vision_temporal_patch_size"], h["out_hidden_size"]
    VNPE, VC, VDSD = 2304, 3, 3
    return [(VH,), (VH, VC, VTP, VP, VP), (VNPE, VH),
            (VD, VH), (VD, VH, VH), (VD, 3, VH), (VD, 3, VH, VH),
            (VD, VI), (VD, VI, VH), (VD, VH), (VD, VH, VI),
            (VD, VH), (VD, VH), (VD, VH), (VD, VH),
            (VDSD, VI), (VDSD, VI, VI), (VDSD, OH), (VDSD, OH, VI), (VDSD, VI), (VDSD, VI),
            (VI,), (VI, VI), (OH,), (OH, VI), (VH,), (VH,)]


def text_bytes(hdr: dict) -> int:
    """Bytes of the header plus the text tensors (where the vision tower starts)."""
    off = HEADER_BYTES
    for name, shp, _ in _TEXT_ORDER:
        shape = tuple(int(v) for v in shp(hdr))
        ns, _ = _scale_count(name, shape, dict(hdr, text_bits=8))
        off += 4 * ns + int(np.prod(shape))
    return off


def map_vision_tensors(path: str) -> dict:
    """Host views (memory-mapped, fp16 or fp32 per vision_bits) of the vision
    tower: name -> array of its shape, in the exporter's [out, in] layout."""
    hdr = read_header(path)
    if hdr["text_bits"] != 8:
        raise ModelFileError("only INT8 text weights are read")
    dt = {16: np.float16, 32: np.float32}.get(hdr["vision_bits"])
    if dt is None:
        raise ModelFileError(f"vision_bits={hdr['vision_bits']}")
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    off = text_bytes(hdr)
    out = {}
    es = np.dtype(dt).itemsize
    for name, shape in vision_tensors(hdr):
        n = int(np.prod(shape))
        if off + n * es > mm.size:
            raise ModelFileError(f"{path}: truncated at vision tensor {name}")
        out[name] = mm[off:off + n * es].view(dt).reshape(shape)
        off += n * es
    return out


def synthetic_text(header: dict, seed: int = 0):
    """Random text weights with the benchmark's distributions: int8 ~U[-127,
    127], scales ~U(0.001, 0.02) (per output row for the matrices, per group
    for the norms)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shp, _ in _TEXT_ORDER:
        shape = tuple(int(v) for v in shp(header))
        ns, _ = _scale_count(name, shape, dict(header, text_bits=8))
        out[name] = (rng.integers(-127, 128, size=shape, dtype=np.int8),
                     rng.uniform(0.001, 0.02, ns).astype(np.float32))
    return out


def qwen3vl_2b_header(**over):
    """Header values of the Qwen3-VL-2B architecture (config 4)."""
    h = dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
             num_attention_heads=16, num_key_value_heads=8, max_position_embeddings=262144,
             rope_theta=5000000, rms_norm_eps=1e-6, vision_hidden_size=1024, vision_depth=24,
             vision_patch_size=16, vision_spatial_merge_size=2, vision_temporal_patch_size=2,
             vision_num_heads=16, vision_intermediate_size=4096, out_hidden_size=2048,
             image_token_id=151655, vision_start_token_id=151652, vision_end_token_id=151653,
             video_token_id=151656, group_size=128, group_quantized=0)
    h.update(over)
    return h
