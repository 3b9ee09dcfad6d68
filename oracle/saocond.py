"""Numpy restatement of the Stable Audio Open 1.0 conditioner (TEST ORACLE -- checker only).

Reference (audio.cpp):
* t5_base_relative_position_buckets (bidirectional, 32 buckets, max distance 128)
                                     src/framework/modules/text_encoders/t5_base_encoder.cpp:180-211
* T5BaseEncoderModule: embedding, per layer RMSNorm -> self-attention (no 1/sqrt(d) scale, + relative bias
  + additive padding mask -1e9) -> residual, RMSNorm -> ReLU FFN -> residual; final RMSNorm      :68-178, 222-245
* make_additive_attention_mask, number_embedding (x, sin / cos of 2 pi x f_i, projection)
                                     src/models/stable_audio/foundation/conditioner.cpp:126-200
* encode_one: cross tokens = T5 states of the kept tokens (zeros elsewhere) + the seconds_start and
  seconds_total embeddings; global = [seconds_start | seconds_total]; seconds_start = 0     :411-471
"""
from __future__ import annotations

import math
from typing import Dict

import numpy as np

from . import bundle as B
from .synth import SaoCondConfig

f32 = np.float32


def relative_buckets(n: int, num_buckets: int = 32, max_distance: int = 128) -> np.ndarray:
    out = np.zeros((n, n), np.int64)
    half = num_buckets // 2
    max_exact = half // 2
    for q in range(n):
        for k in range(n):
            rel = k - q
            b = half if rel > 0 else 0
            rel = abs(rel)
            if rel >= max_exact:
                lr = math.log(rel / max_exact) / math.log(max_distance / max_exact)
                bucket = min(max_exact + int(lr * (half - max_exact)), half - 1)
            else:
                bucket = rel
            out[q, k] = b + bucket
    return out


def rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    return (x / np.sqrt(ms + f32(eps)) * w).astype(np.float32)


def _softmax(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    e = np.exp((s - m).astype(np.float32)).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


class Conditioner:
    def __init__(self, w: Dict[str, B.Tensor], cfg: SaoCondConfig):
        self.cfg = cfg
        self.w = {k: v.array().astype(np.float32) for k, v in w.items()}

    def t5(self, ids: np.ndarray, mask: np.ndarray) -> np.ndarray:
        """ids / mask [B, P] -> encoder states [B, P, d]."""
        cfg, w = self.cfg, self.w
        Bn, P = ids.shape
        H, hd = cfg.heads, cfg.head_dim
        h = w["shared.weight"][ids]  # [B, P, d]
        bias = w["encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"][relative_buckets(P)]  # [P,P,H]
        bias = bias.transpose(2, 0, 1)[None]  # [1, H, P, P]
        add_mask = np.where(mask[:, None, None, :] != 0, f32(0.0), f32(-1e9)).astype(np.float32)
        for l in range(cfg.layers):
            p = "encoder.block.%d.layer." % l
            x = rms(h, w[p + "0.layer_norm.weight"], cfg.eps)
            q = (x @ w[p + "0.SelfAttention.q.weight"].T).reshape(Bn, P, H, hd).transpose(0, 2, 1, 3)
            k = (x @ w[p + "0.SelfAttention.k.weight"].T).reshape(Bn, P, H, hd).transpose(0, 2, 1, 3)
            v = (x @ w[p + "0.SelfAttention.v.weight"].T).reshape(Bn, P, H, hd).transpose(0, 2, 1, 3)
            s = (q @ k.transpose(0, 1, 3, 2) + bias + add_mask).astype(np.float32)
            ctx = (_softmax(s) @ v).transpose(0, 2, 1, 3).reshape(Bn, P, H * hd)
            h = (h + ctx @ w[p + "0.SelfAttention.o.weight"].T).astype(np.float32)
            x = rms(h, w[p + "1.layer_norm.weight"], cfg.eps)
            f = np.maximum(x @ w[p + "1.DenseReluDense.wi.weight"].T, 0).astype(np.float32)
            h = (h + f @ w[p + "1.DenseReluDense.wo.weight"].T).astype(np.float32)
        return rms(h, w["encoder.final_layer_norm.weight"], cfg.eps)

    def number(self, name: str, x: float) -> np.ndarray:
        p = "conditioner.conditioners.%s.embedder.embedding." % name
        fr = self.w[p + "0.weights"]
        arg = (f32(x) * fr * f32(2.0) * f32(math.pi)).astype(np.float32)
        feat = np.concatenate([[f32(x)], np.sin(arg), np.cos(arg)]).astype(np.float32)
        return (self.w[p + "1.weight"] @ feat + self.w[p + "1.bias"]).astype(np.float32)

    def encode_one(self, ids: np.ndarray, mask: np.ndarray, seconds: np.ndarray):
        """-> cross [B, P + 2, d], cross mask [B, P + 2], global [B, 2d]."""
        Bn, P = ids.shape
        d = self.cfg.hidden
        states = self.t5(ids, mask)
        cross = np.zeros((Bn, P + 2, d), np.float32)
        cmask = np.zeros((Bn, P + 2), np.float32)
        glob = np.zeros((Bn, 2 * d), np.float32)
        for b in range(Bn):
            keep = mask[b] != 0
            cross[b, :P][keep] = states[b][keep]
            cmask[b, :P] = keep
            start, total = self.number("seconds_start", 0.0), self.number("seconds_total", float(seconds[b]))
            cross[b, P], cross[b, P + 1] = start, total
            cmask[b, P:] = 1
            glob[b] = np.concatenate([start, total])
        return cross, cmask, glob
