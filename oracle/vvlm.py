"""Numpy restatement of the VibeVoice language model (Qwen2.5 decoder) prefill and cached steps
(TEST ORACLE -- checker only).

Reference (audio.cpp, src/models/vibevoice/decoder.cpp and the framework modules it builds):
* load_layer_weights / load_decoder_weights: q / k / v with bias, o without, SwiGLU MLP, tied lm_head   :186-365
* layer: RMSNorm -> attention (GQA, NEOX RoPE over the full head_dim with base rope_theta, causal,
  scale 1 / sqrt(head_dim)) -> residual; RMSNorm -> down(silu(gate) * up) -> residual; final RMSNorm;
  logits = norm(h) E^T                                                                            :1790-2060
* prefill returns the last position's logits and hidden state; each cached step appends one position.
"""
from __future__ import annotations

from typing import Dict

import numpy as np

from . import bundle as B
from .dit import apply_rope, rope_tables
from .synth import VVLmConfig
from .vibevoice import _silu, rms_norm

f32 = np.float32
P = "model.language_model."


class LanguageModel:
    def __init__(self, w: Dict[str, B.Tensor], cfg: VVLmConfig):
        self.cfg = cfg
        self.w = {k: v.array().astype(np.float32) for k, v in w.items()}
        self.cos, self.sin = rope_tables(cfg.max_positions, cfg.head_dim, cfg.rope_theta)

    def forward(self, ids) -> tuple:
        """Runs all positions of `ids` causally; returns logits [n, vocab] and hidden [n, d] (after the final norm)."""
        cfg, w = self.cfg, self.w
        n = len(ids)
        H, KV, hd = cfg.heads, cfg.kv_heads, cfg.head_dim
        h = w[P + "embed_tokens.weight"][np.asarray(ids)]
        cos, sin = self.cos[:n], self.sin[:n]
        causal = np.triu(np.full((n, n), -np.inf), 1)
        for l in range(cfg.layers):
            p = P + "layers.%d." % l
            x = rms_norm(h, cfg.eps, w[p + "input_layernorm.weight"])
            q = (x @ w[p + "self_attn.q_proj.weight"].T + w[p + "self_attn.q_proj.bias"]).reshape(n, H, hd)
            k = (x @ w[p + "self_attn.k_proj.weight"].T + w[p + "self_attn.k_proj.bias"]).reshape(n, KV, hd)
            v = (x @ w[p + "self_attn.v_proj.weight"].T + w[p + "self_attn.v_proj.bias"]).reshape(n, KV, hd)
            q = apply_rope(q.astype(np.float32), cos, sin, n_dims=hd)
            k = apply_rope(k.astype(np.float32), cos, sin, n_dims=hd)
            rep = H // KV
            kk = np.repeat(k, rep, axis=1).transpose(1, 0, 2).astype(np.float64)
            vv = np.repeat(v, rep, axis=1).transpose(1, 0, 2).astype(np.float64)
            s = q.transpose(1, 0, 2).astype(np.float64) @ kk.transpose(0, 2, 1) / np.sqrt(hd) + causal
            s -= s.max(axis=-1, keepdims=True)
            pr = np.exp(s)
            pr /= pr.sum(axis=-1, keepdims=True)
            ctx = (pr @ vv).transpose(1, 0, 2).reshape(n, H * hd).astype(np.float32)
            h = (h + ctx @ w[p + "self_attn.o_proj.weight"].T).astype(np.float32)
            x = rms_norm(h, cfg.eps, w[p + "post_attention_layernorm.weight"])
            m = (_silu((x @ w[p + "mlp.gate_proj.weight"].T).astype(np.float32)) *
                 (x @ w[p + "mlp.up_proj.weight"].T)).astype(np.float32)
            h = (h + m @ w[p + "mlp.down_proj.weight"].T).astype(np.float32)
        hn = rms_norm(h, cfg.eps, w[P + "norm.weight"])
        return (hn @ w[P + "embed_tokens.weight"].T).astype(np.float32), hn

    def run(self, prefill_ids, step_ids):
        """Logits / hidden of the prefill's last position, then of each cached step (as the reference's order)."""
        ids = list(prefill_ids) + list(step_ids)
        logits, hidden = self.forward(ids)
        sel = [len(prefill_ids) - 1 + i for i in range(len(step_ids) + 1)]
        return logits[sel], hidden[sel]
