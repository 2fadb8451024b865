"""Test infrastructure only: one text-decoder token on the CPU, composed from
the reference engine's own compiled operators (backend "ref",
oracle/_ref/libqwen_ref.so) or from the C restatement (backend "orc"), in
the order of forward_text (model/src/forward.cpp:458-720).

Used by the GPU decoder parity test and as bench.py's CPU baseline.  The KV
cache is held as fp32 with fp16-rounded values, mirroring the GPU's FP16 cache
so that the comparison isolates the kernels (the reference itself caches FP32).
"""
from __future__ import annotations

import numpy as np

from . import (TILED, argmax, attention, embedding_i8, linear_i8, ref_attention, ref_embedding_i8,
               ref_i8_kernel, ref_rms_norm_i8, ref_rope, ref_swiglu, rms_norm_i8, rope_inplace,
               swiglu)


def _f16(a):
    return a.astype(np.float16).astype(np.float32)


class CpuDecoder:
    def __init__(self, cfg, w: dict, max_ctx: int, cos: np.ndarray, sin: np.ndarray, backend="ref",
                 order="lane8"):
        """order: "lane8" = the reference's M=1 decode GEMV order (what it
        runs per token); "tiled" = its M>1 kernel order (restatement only),
        for checking a batch computed as one M=B product."""
        self.cfg, self.w, self.S = cfg, w, max_ctx
        self.cos, self.sin = cos, sin
        self.backend = backend if order == "lane8" else "orc"
        self.order = order
        L, NKV, D = cfg.layers, cfg.kv_heads, cfg.head_dim
        self.kc = np.zeros((L, NKV, max_ctx, D), np.float32)
        self.vc = np.zeros((L, NKV, max_ctx, D), np.float32)

    # backend-specific operators (same arithmetic, pinned against each other)
    def _lin(self, x, W, S):
        x = x.reshape(1, -1)
        K = x.shape[1]
        if self.order == "tiled":
            return linear_i8(x, W, S, K, TILED)[0]
        if self.backend == "ref":
            return ref_i8_kernel(x, W, S, K)[0]
        return linear_i8(x, W, S, K)[0]

    def _rms(self, x, wq, ws, inplace):
        x = x.reshape(-1, wq.shape[0])
        g = self.cfg.norm_group
        if self.backend == "ref":
            return ref_rms_norm_i8(x, wq, ws, g, self.cfg.eps, inplace)
        return rms_norm_i8(x, wq, ws, g, self.cfg.eps, inplace)

    def _rope(self, x, pos):
        if self.backend == "ref":
            return ref_rope(x, self.cos, self.sin, pos)
        return rope_inplace(x.copy(), self.cos[pos], self.sin[pos])

    def step(self, token: int, pos: int):
        """Returns (logits, greedy token) for `token` at position `pos`."""
        cfg, w = self.cfg, self.w
        H, D = cfg.hidden, cfg.head_dim
        if self.backend == "ref":
            x = ref_embedding_i8(w["embed"], w["embed_s"], token)
        else:
            x = embedding_i8(w["embed"], w["embed_s"], token)
        for l in range(cfg.layers):
            t = self._rms(x, w["in_norm"][l], w["in_norm_s"][l], False)[0]
            q = self._lin(t, w["wq"][l], w["wq_s"][l])
            k = self._lin(t, w["wk"][l], w["wk_s"][l])
            v = self._lin(t, w["wv"][l], w["wv_s"][l])
            q = self._rms(q, w["q_norm"][l], w["q_norm_s"][l], True)
            k = self._rms(k, w["k_norm"][l], w["k_norm_s"][l], True)
            q = self._rope(q, pos)
            k = self._rope(k, pos)
            self.kc[l, :, pos] = _f16(k)
            self.vc[l, :, pos] = _f16(v.reshape(cfg.kv_heads, D))
            att_fn = ref_attention if self.backend == "ref" else attention
            a = att_fn(self.kc[l], self.vc[l], np.ascontiguousarray(q), pos).reshape(-1)
            x = (x + self._lin(a, w["wo"][l], w["wo_s"][l])).astype(np.float32)
            t = self._rms(x, w["post_norm"][l], w["post_norm_s"][l], False)[0]
            gate = self._lin(t, w["wg"][l], w["wg_s"][l])
            up = self._lin(t, w["wu"][l], w["wu_s"][l])
            h = ref_swiglu(gate, up) if self.backend == "ref" else swiglu(gate, up)
            x = (x + self._lin(h, w["wd"][l], w["wd_s"][l])).astype(np.float32)
        x = self._rms(x, w["final_norm"], w["final_norm_s"], True)[0]
        logits = self._lin(x, w["embed"], w["embed_s"])
        return logits, argmax(logits)
