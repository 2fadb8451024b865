"""Qwen3-VL-2B text decoder step on the sm_100a kernels.

Host orchestration of one decode token for B independent requests, in the
order of the reference's ``forward_text`` (model/src/forward.cpp:458-720):

    embedding_lookup -> 28 x [rms_norm -> q/k/v linear -> QK rms_norm_inplace
    -> RoPE + KV append -> attention -> o linear + residual -> rms_norm ->
    gate/up linear -> swiglu -> down linear + residual] -> rms_norm_inplace ->
    tied LM head -> greedy_decode

Every product runs through the C ABI (libqvl_b200.so).  Row i of every linear
is computed in the reference's M=1 summation order (QVL_SEM_LANE8), so each
request matches the reference run on that request alone.  Differences from
the reference, by design: the KV cache is FP16 and paged (the reference keeps
an FP32 contiguous cache, load_model.cpp:348-349) and attention is split-K
over the context (same exp polynomial and zeroing rules).

Weights use the reference layout (export_bin/export_qwen_bin.py): int8
[out, in] per matrix with per-output-row fp32 scales (per-row export), norm
weights int8 with fp32 group scales (group ``norm_group``).  ``random()``
draws them synthetically (no checkpoint is available): int8 ~U[-127,127],
scales ~U(0.001, 0.02).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import (SEM_ACCUMULATE, SEM_LANE8, SEM_TILED, PagedKV, linear_batched, Workspace, attention, embedding_lookup_i8,
               attention_ordered, DECODE_REFERENCE_ORDER,
               attention_q16, gate_up_swiglu, greedy_decode, linear_q16, linear_q16_multi, linear_tail,
               qknorm_rope_kv_append, rms_norm_i8, text_decode_step, text_decode_workspace, text_weights_struct,
               Planes, linear_planes_batched, quantize_rows_planes, rms_norm_i8_planes,
               qknorm_rope_attention_ordered)
from . import load_library
from . import swiglu as swiglu_


@dataclasses.dataclass
class TextConfig:
    hidden: int = 2048
    intermediate: int = 6144
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 5e6
    norm_group: int = 128


def rope_table(max_pos: int, head_dim: int = 128, theta: float = 5e6):
    """Text section of qwen_rope_precompute (model/src/load_model.cpp:413-490),
    computed on the host by qvl_rope_table with the host's single-precision
    libm exactly as the reference computes it (theta is an integer there)."""
    import ctypes
    c = np.empty((max_pos, head_dim // 2), np.float32)
    s = np.empty((max_pos, head_dim // 2), np.float32)
    L = load_library()
    rc = L.qvl_rope_table(int(theta), head_dim, max_pos, c.ctypes.data_as(ctypes.c_void_p),
                          s.ctypes.data_as(ctypes.c_void_p))
    if rc:
        raise ValueError(f"qvl_rope_table: status {rc}")
    return c, s


_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


class TextWeights:
    """Device copies of the text-decoder weights in the reference layout."""

    def __init__(self, cfg: TextConfig, tensors: dict):
        self.cfg = cfg
        self.t = tensors

    @staticmethod
    def shapes(cfg: TextConfig):
        H, I, L, D = cfg.hidden, cfg.intermediate, cfg.layers, cfg.head_dim
        return {"wq": (L, cfg.heads * D, H), "wk": (L, cfg.kv_heads * D, H), "wv": (L, cfg.kv_heads * D, H),
                "wo": (L, H, cfg.heads * D), "wg": (L, I, H), "wu": (L, I, H), "wd": (L, H, I)}

    @classmethod
    def random(cls, cfg: TextConfig, seed: int = 0, device="cuda"):
        g = torch.Generator(device=device).manual_seed(seed)
        t = {}

        def i8(shape):
            return torch.randint(-127, 128, shape, dtype=torch.int8, device=device, generator=g)

        def sc(shape):
            return (torch.rand(shape, dtype=torch.float32, device=device, generator=g) * 0.019 + 0.001)

        for name, shp in cls.shapes(cfg).items():
            t[name] = i8(shp)
            t[name + "_s"] = sc(shp[:2])                      # per-output-row scales
        H, L, D, ng = cfg.hidden, cfg.layers, cfg.head_dim, cfg.norm_group
        for name, n in (("in_norm", H), ("post_norm", H), ("q_norm", D), ("k_norm", D)):
            t[name] = i8((L, n))
            t[name + "_s"] = sc((L, n // ng))
        t["final_norm"] = i8((H,))
        t["final_norm_s"] = sc((H // ng,))
        t["embed"] = i8((cfg.vocab, H))                       # tied with the LM head
        t["embed_s"] = sc((cfg.vocab,))
        return cls(cfg, t)

    def numpy(self):
        return {k: v.cpu().numpy() for k, v in self.t.items()}


class TextDecoder:
    """Batched decode over a paged FP16 KV cache (one sequence per request)."""

    def __init__(self, weights: TextWeights, max_batch: int, max_ctx: int, page_size: int = 64,
                 device="cuda", batch_order: str = "auto", persistent: bool = False,
                 attn_order: str = "reference", tp_group=None):
        """batch_order: "lane8" computes every request row in the reference's
        M=1 decode order (CUDA-core GEMV, each request bit-matches the
        reference run on it alone); "tiled" runs the batch as one M=B product
        on the tensor cores in the reference's M>1 order (what the reference's
        linear() does for an M>1 call); "auto" = tiled for B >= 16.
        persistent: (max_batch 1 only) run each token as ONE cooperative
        launch (qvl_text_decode_step) instead of ~6 launches per layer.
        attn_order: "fast" splits each context over CTAs (fp32 partial sums
        grouped differently from the reference); "reference" runs the
        reference's own summation order, so that with the lane8 order every
        operation of a token is bit-identical to the reference's.
        tp_group: a torch.distributed group (NCCL) whose ranks run prefill()
        together: every product of the prompt pass is split by output column
        over the group and all-gathered (qvl_b200.parallel), so each column
        is computed once, by its owner, with unchanged arithmetic -- results
        are bit-identical to one GPU.  Decode steps stay per-rank."""
        self.tp = tp_group
        if attn_order not in ("fast", "reference"):
            raise ValueError(attn_order)
        self.attn_order = attn_order
        self.w = weights
        cfg = self.cfg = weights.cfg
        self.B = max_batch
        self.max_ctx = max_ctx
        dev = self.device = torch.device(device)
        H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim
        B = max_batch
        f32, i16 = torch.float32, torch.int16
        self.x = torch.zeros((B, H), dtype=f32, device=dev)
        self.qx = torch.zeros((B, H), dtype=i16, device=dev)
        self.qx_s = torch.zeros((B, 1), dtype=f32, device=dev)
        self.q = torch.zeros((B, cfg.heads * D), dtype=f32, device=dev)
        self.k = torch.zeros((B, cfg.kv_heads * D), dtype=f32, device=dev)
        self.v = torch.zeros((B, cfg.kv_heads * D), dtype=f32, device=dev)
        self.att = torch.zeros((B, cfg.heads * D), dtype=f32, device=dev)
        self.qa = torch.zeros((B, cfg.heads * D), dtype=i16, device=dev)
        self.qa_s = torch.zeros((B, 1), dtype=f32, device=dev)
        self.gate = torch.zeros((B, I), dtype=f32, device=dev)
        self.up = torch.zeros((B, I), dtype=f32, device=dev)
        self.qh = torch.zeros((B, I), dtype=i16, device=dev)
        self.qh_s = torch.zeros((B, 1), dtype=f32, device=dev)
        self.logits = torch.zeros((B, cfg.vocab), dtype=f32, device=dev)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int32, device=dev)
        self.seq_ids = torch.arange(B, dtype=torch.int32, device=dev)
        # one stacked cache (uniform layer stride), viewed per layer
        maxp = (max_ctx + page_size - 1) // page_size
        kv_shape = (cfg.layers, B * maxp, cfg.kv_heads, page_size, D)
        self.k_all = torch.zeros(kv_shape, dtype=torch.float16, device=dev)
        self.v_all = torch.zeros(kv_shape, dtype=torch.float16, device=dev)
        self.page_size = page_size
        self.kv = [PagedKV(B, max_ctx, cfg.heads, cfg.kv_heads, D, page_size, max_pos=max_ctx, device=dev,
                           k=self.k_all[l], v=self.v_all[l]) for l in range(cfg.layers)]
        if persistent and max_batch != 1:
            raise ValueError("persistent decode serves one request (max_batch 1)")
        self.persistent = persistent
        if persistent:
            self.pw = text_weights_struct(weights.t, cfg)
            self.pws = text_decode_workspace(dev)
        cos, sin = rope_table(max_ctx, D, cfg.rope_theta)
        self.set_rope_table(cos, sin)
        self.counters = torch.zeros(4, dtype=torch.int32, device=dev)   # fused-tail counters (stay 0)
        self.fuse_tails = max_batch == 1   # one CTA finishes each row: pays off for a single row
        if batch_order == "auto":
            batch_order = "tiled" if max_batch >= 16 else "lane8"
        self.use_tc = batch_order == "tiled"
        self.tc_ws = Workspace(dev)
        if self.use_tc:
            # hi/lo planes written by the quantising kernels, read by the products
            self.planes = Planes(max_batch, max(cfg.hidden, cfg.intermediate), dev)
        self.ws = Workspace(dev)
        self.ws.get(load_library().qvl_attention_workspace_bytes(B, max_ctx, self.kv[0].dims))
        if attn_order == "reference":
            self.ws.get(load_library().qvl_attention_ordered_workspace_bytes(B, max_ctx, self.kv[0].dims))

    def set_rope_table(self, cos: np.ndarray, sin: np.ndarray):
        self.rope_cos = torch.from_numpy(np.ascontiguousarray(cos)).to(self.device)
        self.rope_sin = torch.from_numpy(np.ascontiguousarray(sin)).to(self.device)

    def _lin(self, q, qs, name, l, out, acc=False):
        t = self.w.t
        W = t[name][l] if l is not None else t[name]
        S = t[name + "_s"][l] if l is not None else t[name + "_s"]
        return linear_q16(q, qs, W, S, q.shape[1], C=out, semantics=SEM_LANE8 | (SEM_ACCUMULATE if acc else 0))

    def _lin_multi(self, q, qs, names, l, outs):
        t = self.w.t
        mats = [(t[n][l], t[n + "_s"][l]) for n in names]
        return linear_q16_multi(q, qs, mats, outs, q.shape[1], semantics=SEM_LANE8)

    def step(self, B=None):
        """One decode token for requests 0..B-1: reads self.tokens and
        self.positions, leaves the logits in self.logits and the greedy
        tokens in self.tokens, and advances self.positions by one.  Only
        device work is issued (graph-capturable)."""
        B = B or self.B
        if self.persistent:
            text_decode_step(self.pw, self.x, self.logits, self.tokens, self.positions, self.k_all, self.v_all,
                             self.kv[0].page_table, self.page_size, self.rope_cos, self.rope_sin, self.max_ctx,
                             self.pws, flags=DECODE_REFERENCE_ORDER if self.attn_order == "reference" else 0)
            return
        cfg, t = self.cfg, self.w.t
        H, ng, eps = cfg.hidden, cfg.norm_group, cfg.eps
        x = self.x[:B]
        qx, qx_s = self.qx[:B], self.qx_s[:B]
        seq, pos = self.seq_ids[:B], self.positions[:B]
        embedding_lookup_i8(t["embed"], t["embed_s"], self.tokens[:B], x)
        if self.use_tc:
            self._step_tc(B)
            greedy_decode(self.logits[:B], out=self.tokens[:B])
            pos.add_(1)
            return
        if self.fuse_tails:
            rms_norm_i8(x, t["in_norm"][0], t["in_norm_s"][0], ng, eps, q=qx, q_scales=qx_s, quant_group=H)
        L = cfg.layers
        for l in range(L):
            if not self.fuse_tails:
                rms_norm_i8(x, t["in_norm"][l], t["in_norm_s"][l], ng, eps, q=qx, q_scales=qx_s, quant_group=H)
            self._lin_multi(qx, qx_s, ("wq", "wk", "wv"), l, (self.q[:B], self.k[:B], self.v[:B]))
            qknorm_rope_kv_append(self.q[:B], self.k[:B], self.v[:B], self.kv[l], seq, pos, self.rope_cos,
                                  self.rope_sin, t["q_norm"][l], t["q_norm_s"][l], t["k_norm"][l],
                                  t["k_norm_s"][l], ng, eps)
            if self.attn_order == "reference":
                attention_ordered(self.q[:B], self.kv[l], seq, pos, self.max_ctx, out=self.att[:B], workspace=self.ws)
                _quantize_into(self.att[:B], self.qa[:B], self.qa_s[:B])
            elif self.fuse_tails:
                attention_q16(self.q[:B], self.kv[l], seq, pos, self.max_ctx, self.att[:B], self.qa[:B],
                              self.qa_s[:B], self.counters[3], workspace=self.ws)
            else:
                attention(self.q[:B], self.kv[l], seq, pos, self.max_ctx, out=self.att[:B], workspace=self.ws)
                _quantize_into(self.att[:B], self.qa[:B], self.qa_s[:B])
            if self.fuse_tails:
                # o_proj + residual, then post-attention rms_norm -> gate/up input, one launch
                linear_tail(self.qa[:B], self.qa_s[:B], [(t["wo"][l], t["wo_s"][l])], [x], H, self.counters[0],
                            qx, qx_s, H, norm=(t["post_norm"][l], t["post_norm_s"][l], ng), eps=eps,
                            semantics=SEM_LANE8 | SEM_ACCUMULATE)
                # gate/up + SwiGLU, then quantisation of the SwiGLU row -> down input
                linear_tail(qx, qx_s, [(t["wg"][l], t["wg_s"][l]), (t["wu"][l], t["wu_s"][l])],
                            [self.gate[:B], self.up[:B]], H, self.counters[1], self.qh[:B], self.qh_s[:B],
                            cfg.intermediate, swiglu_pair=True, semantics=SEM_LANE8)
                # down + residual, then the next layer's input rms_norm (or the final norm) -> next input
                if l + 1 < L:
                    nrm, inpl, nout = (t["in_norm"][l + 1], t["in_norm_s"][l + 1], ng), False, None
                else:
                    nrm, inpl, nout = (t["final_norm"], t["final_norm_s"], ng), True, x
                linear_tail(self.qh[:B], self.qh_s[:B], [(t["wd"][l], t["wd_s"][l])], [x], cfg.intermediate,
                            self.counters[2], qx, qx_s, H, norm=nrm, eps=eps, inplace_form=inpl, norm_out=nout,
                            semantics=SEM_LANE8 | SEM_ACCUMULATE)
                continue
            self._lin(self.qa[:B], self.qa_s[:B], "wo", l, x, acc=True)
            rms_norm_i8(x, t["post_norm"][l], t["post_norm_s"][l], ng, eps, q=qx, q_scales=qx_s, quant_group=H)
            gate_up_swiglu(qx, qx_s, t["wg"][l], t["wg_s"][l], t["wu"][l], t["wu_s"][l], self.gate[:B], H,
                           up_scratch=self.up[:B], semantics=SEM_LANE8)
            _quantize_into(self.gate[:B], self.qh[:B], self.qh_s[:B])
            self._lin(self.qh[:B], self.qh_s[:B], "wd", l, x, acc=True)
        if not self.fuse_tails:
            rms_norm_i8(x, t["final_norm"], t["final_norm_s"], ng, eps, out=x, q=qx, q_scales=qx_s,
                        quant_group=H, inplace_form=True)
        self._lin(qx, qx_s, "embed", None, self.logits[:B])
        greedy_decode(self.logits[:B], out=self.tokens[:B])
        pos.add_(1)

    def _step_tc(self, B):
        """Tensor-core batch (reference M>1 order): every linear runs as one
        M=B tcgen05 product; the kernels that quantise an activation row also
        write its hi/lo planes, and q/k/v and gate/up are one launch each."""
        cfg, t = self.cfg, self.w.t
        H, I, ng, eps = cfg.hidden, cfg.intermediate, cfg.norm_group, cfg.eps
        x, qx, qx_s = self.x[:B], self.qx[:B], self.qx_s[:B]
        seq, pos = self.seq_ids[:B], self.positions[:B]
        P = self.planes
        acc = SEM_TILED | SEM_ACCUMULATE
        for l in range(cfg.layers):
            rms_norm_i8_planes(x, t["in_norm"][l], t["in_norm_s"][l], ng, eps, qx, qx_s, P)
            linear_planes_batched(P, qx_s, [(t[n][l], t[n + "_s"][l]) for n in ("wq", "wk", "wv")],
                                  [self.q[:B], self.k[:B], self.v[:B]], B, H)
            if self.attn_order == "reference":
                # QK-norm, RoPE and the KV append inside the score pass (one
                # request per sequence)
                qknorm_rope_attention_ordered(self.q[:B], self.k[:B], self.v[:B], self.kv[l], seq, pos, self.max_ctx,
                                              self.rope_cos, self.rope_sin, t["q_norm"][l], t["q_norm_s"][l],
                                              t["k_norm"][l], t["k_norm_s"][l], ng, eps, out=self.att[:B],
                                              workspace=self.ws)
            else:
                qknorm_rope_kv_append(self.q[:B], self.k[:B], self.v[:B], self.kv[l], seq, pos, self.rope_cos,
                                      self.rope_sin, t["q_norm"][l], t["q_norm_s"][l], t["k_norm"][l],
                                      t["k_norm_s"][l], ng, eps)
                attention(self.q[:B], self.kv[l], seq, pos, self.max_ctx, out=self.att[:B], workspace=self.ws)
            quantize_rows_planes(self.att[:B], self.qa[:B], self.qa_s[:B], P)
            linear_planes_batched(P, self.qa_s[:B], [(t["wo"][l], t["wo_s"][l])], [x], B, H, semantics=acc)
            rms_norm_i8_planes(x, t["post_norm"][l], t["post_norm_s"][l], ng, eps, qx, qx_s, P)
            linear_planes_batched(P, qx_s, [(t["wg"][l], t["wg_s"][l]), (t["wu"][l], t["wu_s"][l])],
                                  [self.gate[:B], self.up[:B]], B, H)
            swiglu_(self.gate[:B], self.up[:B])
            quantize_rows_planes(self.gate[:B], self.qh[:B], self.qh_s[:B], P)
            linear_planes_batched(P, self.qh_s[:B], [(t["wd"][l], t["wd_s"][l])], [x], B, I, semantics=acc)
        rms_norm_i8_planes(x, t["final_norm"], t["final_norm_s"], ng, eps, qx, qx_s, P, out=x, inplace_form=True)
        linear_planes_batched(P, qx_s, [(t["embed"], t["embed_s"])], [self.logits[:B]], B, H)

    def prefill(self, tokens: torch.Tensor, seq: int = 0, start: int = 0, image_embeds=None, deepstack=None,
                image_token_id: int = 151655, order: str = "tiled"):
        """Prompt of T tokens of request `seq` at positions start..start+T-1 as
        one M=T pass, attention causal over the paged cache (query t sees
        positions <= start+t).  Leaves the last token's logits and greedy id in
        self.logits[seq] / self.tokens[seq] and self.positions[seq] = start+T.

        order "tiled": every linear is one tensor-core product (the reference's
        M>1 order).  order "lane8": every row in the reference's M=1 order and
        attention in its summation order (with attn_order "reference"), i.e.
        exactly what the reference computes when it feeds the prompt one token
        at a time (model/src/utils.cpp:143-160).

        image_embeds fp32 [n, H] / deepstack fp16 [3, n, H] (the vision tower's
        outputs): the k-th prompt token equal to image_token_id takes row k of
        image_embeds instead of its embedding, and after layers 0..2 row k of
        deepstack[l] is added to it (forward_text, model/src/forward.cpp:476-485,
        665-673)."""
        cfg, t = self.cfg, self.w.t
        T = tokens.numel()
        H, I, D, ng, eps = cfg.hidden, cfg.intermediate, cfg.head_dim, cfg.norm_group, cfg.eps
        dev = self.device
        pf = getattr(self, "_pf", None)
        if pf is None or pf["T"] < T:
            f32, i16 = torch.float32, torch.int16
            pf = dict(T=T, x=torch.zeros((T, H), dtype=f32, device=dev), q16=torch.zeros((T, I), dtype=i16, device=dev),
                      qh=torch.zeros((T, H), dtype=i16, device=dev),
                      qs=torch.zeros((T, 1), dtype=f32, device=dev), q=torch.zeros((T, cfg.heads * D), dtype=f32, device=dev),
                      k=torch.zeros((T, cfg.kv_heads * D), dtype=f32, device=dev),
                      v=torch.zeros((T, cfg.kv_heads * D), dtype=f32, device=dev),
                      att=torch.zeros((T, cfg.heads * D), dtype=f32, device=dev),
                      gate=torch.zeros((T, I), dtype=f32, device=dev), up=torch.zeros((T, I), dtype=f32, device=dev),
                      logits=torch.zeros((1, cfg.vocab), dtype=f32, device=dev),
                      seq=torch.zeros(T, dtype=torch.int32, device=dev),
                      pos=torch.zeros(T, dtype=torch.int32, device=dev), ws=Workspace(dev))
            pf["ws"].get(load_library().qvl_linear_q16_i8_batched_workspace_bytes(T, I))
            pf["planes"] = Planes(T, I, dev)
            self._pf = pf
        x, q16, qs = pf["x"][:T], pf["q16"][:T], pf["qs"][:T]
        qh = pf["qh"][:T]
        pf["seq"][:T].fill_(seq)
        torch.arange(start, start + T, dtype=torch.int32, device=dev, out=pf["pos"][:T])
        sq, ps = pf["seq"][:T], pf["pos"][:T]
        ws = pf["ws"]
        embedding_lookup_i8(t["embed"], t["embed_s"], tokens.to(torch.int32), x)
        img_mask = img_idx = None
        if image_embeds is not None:
            # the k-th image token takes embedding row k: found on the device
            # (running count of image tokens), no host synchronisation, so
            # the pass can be enqueued while earlier work runs.  Image tokens
            # beyond the embedding rows repeat the last row (the reference
            # would read past its buffer).
            mask = tokens.reshape(-1) == image_token_id
            img_idx = (torch.cumsum(mask.to(torch.int32), 0) - 1).clamp_(0, image_embeds.shape[0] - 1).long()
            img_mask = mask[:, None]
            x.copy_(torch.where(img_mask, image_embeds.to(torch.float32)[img_idx], x))
        lane8 = order == "lane8"
        if order not in ("tiled", "lane8"):
            raise ValueError(order)
        prod = self._prefill_product_lane8 if lane8 else self._prefill_product
        attn = attention_ordered if self.attn_order == "reference" else attention
        if self.attn_order == "reference":
            ws.get(load_library().qvl_attention_ordered_workspace_bytes(T, self.max_ctx, self.kv[0].dims))
        # one process, tensor-core order: the quantising kernels write the
        # products' hi/lo planes, q/k/v and gate/up are one launch each
        planes = pf["planes"] if (not lane8 and self.tp is None) else None
        accs = SEM_TILED | SEM_ACCUMULATE

        def mats(names, l):
            return [(t[n][l], t[n + "_s"][l]) for n in names]

        for l in range(cfg.layers):
            if planes is not None:
                rms_norm_i8_planes(x, t["in_norm"][l], t["in_norm_s"][l], ng, eps, qh, qs, planes)
                linear_planes_batched(planes, qs, mats(("wq", "wk", "wv"), l), [pf["q"][:T], pf["k"][:T], pf["v"][:T]],
                                      T, H)
            else:
                rms_norm_i8(x, t["in_norm"][l], t["in_norm_s"][l], ng, eps, q=qh, q_scales=qs, quant_group=H)
                prod(qh, qs, ("wq", "wk", "wv"), l, [pf["q"][:T], pf["k"][:T], pf["v"][:T]], ws)
            qknorm_rope_kv_append(pf["q"][:T], pf["k"][:T], pf["v"][:T], self.kv[l], sq, ps, self.rope_cos,
                                  self.rope_sin, t["q_norm"][l], t["q_norm_s"][l], t["k_norm"][l],
                                  t["k_norm_s"][l], ng, eps)
            attn(pf["q"][:T], self.kv[l], sq, ps, self.max_ctx, out=pf["att"][:T], workspace=ws)
            if planes is not None:
                quantize_rows_planes(pf["att"][:T], qh, qs, planes)
                linear_planes_batched(planes, qs, mats(("wo",), l), [x], T, H, semantics=accs)
                rms_norm_i8_planes(x, t["post_norm"][l], t["post_norm_s"][l], ng, eps, qh, qs, planes)
                linear_planes_batched(planes, qs, mats(("wg", "wu"), l), [pf["gate"][:T], pf["up"][:T]], T, H)
                swiglu_(pf["gate"][:T], pf["up"][:T])
                quantize_rows_planes(pf["gate"][:T], q16, qs, planes)
                linear_planes_batched(planes, qs, mats(("wd",), l), [x], T, I, semantics=accs)
            else:
                _quantize_into(pf["att"][:T], qh, qs)
                prod(qh, qs, ("wo",), l, [x], ws, acc=True)
                rms_norm_i8(x, t["post_norm"][l], t["post_norm_s"][l], ng, eps, q=qh, q_scales=qs, quant_group=H)
                prod(qh, qs, ("wg", "wu"), l, [pf["gate"][:T], pf["up"][:T]], ws, swiglu=True,
                     up_scratch=pf["up"][:T])
                _quantize_into(pf["gate"][:T], q16, qs)
                prod(q16, qs, ("wd",), l, [x], ws, acc=True)
            if img_mask is not None and l < deepstack.shape[0]:
                # add_vector(x, deep-stack row): fp32 x + the fp16 value, image rows only
                x.copy_(torch.where(img_mask, x + deepstack[l].to(torch.float32)[img_idx], x))
        last = x[T - 1:T]
        rms_norm_i8(last, t["final_norm"], t["final_norm_s"], ng, eps, out=last, q=qh[:1], q_scales=qs[:1],
                    quant_group=H, inplace_form=True)
        if self.tp is None:
            linear_q16(qh[:1], qs[:1], t["embed"], t["embed_s"], H, C=pf["logits"], semantics=SEM_LANE8)
            greedy_decode(pf["logits"], out=self.tokens[seq:seq + 1])
        else:
            # LM head split by vocabulary rows; the greedy token from an
            # 8-byte (value, index) exchange per rank, the logits gathered
            from . import parallel as par
            a, b = par.shard_rows(cfg.vocab, self._tp_world, self._tp_rank)
            loc = self._tp_buf(("lm", b - a), (1, b - a))
            linear_q16(qh[:1], qs[:1], t["embed"][a:b], t["embed_s"][a:b], H, C=loc, semantics=SEM_LANE8)
            self.tokens[seq:seq + 1].copy_(par.split_greedy(loc, a, self.tp).to(torch.int32))
            pf["logits"].copy_(par.gather_columns(loc, cfg.vocab, self.tp))
        self.logits[seq].copy_(pf["logits"][0])
        self.positions[seq:seq + 1].fill_(start + T)

    @property
    def _tp_world(self):
        import torch.distributed as dist
        return dist.get_world_size(self.tp)

    @property
    def _tp_rank(self):
        import torch.distributed as dist
        return dist.get_rank(self.tp)

    def _tp_buf(self, key, shape, dtype=torch.float32):
        bufs = self.__dict__.setdefault("_tp_bufs", {})
        b = bufs.get(key)
        if b is None or b.numel() < int(np.prod(shape)):
            b = bufs[key] = torch.empty(int(np.prod(shape)), dtype=dtype, device=self.device)
        return b[:int(np.prod(shape))].view(shape)

    def _prefill_product_lane8(self, q, qs, names, l, outs, ws, acc=False, swiglu=False, up_scratch=None):
        """The products of the prompt rows in the reference's M=1 order (each
        row as its own GEMV), then swiglu(gate, up) into gate."""
        t = self.w.t
        K = q.shape[1]
        for n, out in zip(names, outs):
            linear_q16(q, qs, t[n][l], t[n + "_s"][l], K, C=out,
                       semantics=SEM_LANE8 | (SEM_ACCUMULATE if acc else 0))
        if swiglu:
            swiglu_(outs[0], outs[1])

    def _prefill_product(self, q, qs, names, l, outs, ws, acc=False, swiglu=False, up_scratch=None):
        """outs[i] (+)= q . dequant(W_names[i])^T for the prompt rows, one
        tensor-core product per matrix in the reference's M>1 order; with a
        tp group, split by output column and all-gathered (bit-identical)."""
        t = self.w.t
        mats = [(t[n][l], t[n + "_s"][l]) for n in names]
        if self.tp is None:
            linear_batched(q, qs, mats, outs, ws, semantics=SEM_TILED | (SEM_ACCUMULATE if acc else 0),
                           swiglu_pair=swiglu, up_scratch=up_scratch)
            return
        import torch.distributed as dist
        from . import parallel as par
        G, r = self._tp_world, self._tp_rank
        M = q.shape[0]
        local, spans = [], []
        for i, (W, S) in enumerate(mats):
            a, b = par.shard_rows(W.shape[0], G, r)
            spans.append((a, b))
            local.append(self._tp_buf(("out", i), (M, b - a)))
        up_loc = local[1] if swiglu else None
        linear_batched(q, qs, [(W[a:b], S[a:b]) for (W, S), (a, b) in zip(mats, spans)], local, ws,
                       semantics=SEM_TILED, swiglu_pair=swiglu, up_scratch=up_loc)
        outs = outs[:1] if swiglu else outs        # SwiGLU: only h (in gate's slot) is needed
        local = local[:len(outs)]
        if all(o.shape[1] % G == 0 for o in outs):
            # one all-gather for all the products of this input: rank slices
            # packed side by side, [G, M, sum of slice widths]
            widths = [l_.shape[1] for l_ in local]
            wsum = sum(widths)
            pack = self._tp_buf(("pack",), (M, wsum))
            c0 = 0
            for l_ in local:
                pack[:, c0:c0 + l_.shape[1]].copy_(l_)
                c0 += l_.shape[1]
            buf = self._tp_buf(("gather",), (G, M, wsum))
            dist.all_gather_into_tensor(buf, pack, group=self.tp)
            c0 = 0
            fulls = []
            for out, w in zip(outs, widths):
                fulls.append(buf[:, :, c0:c0 + w].permute(1, 0, 2).reshape(M, out.shape[1]))
                c0 += w
        else:
            fulls = [par.gather_columns(l_, o.shape[1], self.tp) for l_, o in zip(local, outs)]
        for out, full in zip(outs, fulls):
            if acc:
                out.add_(full)          # the reference's add_vector after the product
            else:
                out.copy_(full)

    # launches of our kernels per step (attention = 3 kernels)
    def kernels_per_step(self):
        if self.persistent:
            return 1
        if self.use_tc:
            # norm, q/k/v, rope + attention (reference order: 2 launches, the rope inside
            # the score pass; else rope, attention), quantise, o, norm, gate/up, swiglu,
            # quantise, down; embedding, final norm, LM head, argmax
            return 1 + self.cfg.layers * 12 + 3
        return 1 + self.cfg.layers * (1 + 1 + 1 + 3 + 1 + 1 + 1 + 1 + 1 + 1) + 1 + 1 + 1


def _quantize_into(x, q, qs):
    from . import _check, _ptr, _stream
    M, K = x.shape
    _check(load_library().qvl_quantize_rows(_ptr(x), _ptr(q), _ptr(qs), M, K, K, _stream(None)), "quantize_rows")


def fill_kv_random(dec: TextDecoder, ctx: int, seed: int = 0):
    """Synthetic prompt state: positions [0, ctx) of every request's cache
    hold fp16 N(0,1) keys/values (stands in for a prefilled prompt)."""
    g = torch.Generator(device=dec.device).manual_seed(seed)
    P = dec.kv[0].page_size
    npages = (ctx + P - 1) // P
    for kv in dec.kv:
        for b in range(dec.B):
            pages = kv.page_table[b, :npages].long()
            kv.k[pages] = torch.randn(kv.k[pages].shape, generator=g, device=dec.device).half()
            kv.v[pages] = torch.randn(kv.v[pages].shape, generator=g, device=dec.device).half()
    dec.positions.fill_(ctx)
