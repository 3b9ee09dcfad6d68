"""Numpy restatement of the Stable Audio 3 rectified-flow DiT and its pingpong / euler
samplers with APG-CFG (TEST ORACLE -- checker only).

Reference (audio.cpp, src/models/stable_audio/rf_dit.cpp):
* constants, rms_norm (RMSNormModule with weight), one_plus, sigmoid_one_minus   :26-34, :109-125
* Fourier timestep frequencies / features, timestep MLP                          :158-182, :753-770
* rf_attention (flash attention, scale 1/sqrt(head_dim)), V x padding mask       :184-215
* self_attention: qkv (5d when differential), per-head qk-RMSNorm (eps 1e-6),
  NEOX RoPE on max(head_dim / 2, 32) dims, context - diff_context                 :217-262
* cross_attention (no RoPE, no mask; q 2d / kv 3d when differential)             :264-310
* swiglu_ff (value = first 4d, gate = last 4d)                                   :312-325
* build_local_embedding (zeros on the memory tokens)                             :327-341
* build_rf_layer: 6-way adaLN = global_six + to_scale_shift_gate, gates sigmoid(1 - g) :343-387
* build_graph_output (pre/post conv, memory tokens, cond / global embedders)     :772-832
* build_cfg_model_output (APG-CFG on x0 = x - sigma v)                           :834-873
* make_*_conditioning, make_padding_mask, write_latent_input                     :891-981
* sample: pingpong (TensorIterator Philox noise every step) / euler              :586-694
"""
from __future__ import annotations

import math
from typing import Dict

import numpy as np

from . import bundle as B
from . import philox
from .dit import apply_rope, attention, rope_tables
from .synth import SP, Sa3Config
from .vibevoice import Linear, _silu, rms_norm

f32 = np.float32
NORM_EPS = 1e-5
QK_EPS = 1e-6


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return (f32(1.0) / (f32(1.0) + np.exp(-x))).astype(np.float32)


def fourier_freqs() -> np.ndarray:
    """make_fourier_freqs: exp(ramp (ln 1e4 - ln 0.5) + ln 0.5) * 2 pi over 128 ramps (fp32)."""
    half = 128
    lmin, lmax = f32(math.log(f32(0.5))), f32(math.log(f32(10000.0)))
    out = np.zeros(half, np.float32)
    for i in range(half):
        ramp = f32(f32(i) / f32(half - 1))
        out[i] = f32(f32(np.exp(f32(ramp * f32(lmax - lmin)) + lmin)) * f32(2.0) * f32(math.pi))
    return out


class Sa3Dit:
    def __init__(self, w: Dict[str, B.Tensor], cfg: Sa3Config, act: str = "ggml"):
        self.cfg = cfg

        def lin(name, bias=False, conv=False):
            t = w[SP + name + ".weight"]
            if conv:
                t = B.Tensor(t.dtype, t.dims[:2], t.data)
            b = w[SP + name + ".bias"].data.astype(np.float32) if bias else None
            return Linear(t, b, act=act)

        def vec(name):
            return w[SP + name].data.astype(np.float32)

        self.freqs = fourier_freqs()
        self.cond0, self.cond2 = lin("to_cond_embed.0"), lin("to_cond_embed.2")
        self.glob0, self.glob2 = lin("to_global_embed.0"), lin("to_global_embed.2")
        self.t0, self.t2 = lin("to_timestep_embed.0", True), lin("to_timestep_embed.2", True)
        self.pre, self.post = lin("preprocess_conv", conv=True), lin("postprocess_conv", conv=True)
        self.pin, self.pout = lin("transformer.project_in"), lin("transformer.project_out")
        self.memory = vec("transformer.memory_tokens").reshape(cfg.num_memory_tokens, cfg.embed_dim)
        self.ge0 = lin("transformer.global_cond_embedder.0", True)
        self.ge2 = lin("transformer.global_cond_embedder.2", True)
        self.layers = []
        for i in range(cfg.depth):
            p = "transformer.layers.%d." % i
            self.layers.append(dict(
                pre=vec(p + "pre_norm.gamma"), cross_n=vec(p + "cross_attend_norm.gamma"), ff_n=vec(p + "ff_norm.gamma"),
                qkv=lin(p + "self_attn.to_qkv"), out=lin(p + "self_attn.to_out"),
                sq=vec(p + "self_attn.q_norm.gamma"), sk=vec(p + "self_attn.k_norm.gamma"),
                q=lin(p + "cross_attn.to_q"), kv=lin(p + "cross_attn.to_kv"), cout=lin(p + "cross_attn.to_out"),
                cq=vec(p + "cross_attn.q_norm.gamma"), ck=vec(p + "cross_attn.k_norm.gamma"),
                ff0=lin(p + "ff.ff.0.proj", True), ff2=lin(p + "ff.ff.2", True),
                lo0=lin(p + "to_local_embed.0", True), lo2=lin(p + "to_local_embed.2", True),
                ssg=vec(p + "to_scale_shift_gate")))
        n_tok = cfg.num_memory_tokens + cfg.latent_tokens
        self.rope = rope_tables(n_tok, max(cfg.head_dim // 2, 32))

    def _heads(self, x: np.ndarray) -> np.ndarray:
        return x.reshape(x.shape[0], self.cfg.num_heads, self.cfg.head_dim)

    def _self_attention(self, L, h: np.ndarray, vmask: np.ndarray) -> np.ndarray:
        d = self.cfg.embed_dim
        nd = max(self.cfg.head_dim // 2, 32)
        qkv = L["qkv"](h)
        q, k, v = self._heads(qkv[:, :d]), self._heads(qkv[:, d:2 * d]), self._heads(qkv[:, 2 * d:3 * d])
        q = apply_rope(rms_norm(q, QK_EPS, L["sq"]), *self.rope, n_dims=nd)
        k = apply_rope(rms_norm(k, QK_EPS, L["sk"]), *self.rope, n_dims=nd)
        v = (v * vmask[:, None, None]).astype(np.float32)
        ctx = attention(q, k, v)
        if self.cfg.differential:
            qd, kd = self._heads(qkv[:, 3 * d:4 * d]), self._heads(qkv[:, 4 * d:5 * d])
            qd = apply_rope(rms_norm(qd, QK_EPS, L["sq"]), *self.rope, n_dims=nd)
            kd = apply_rope(rms_norm(kd, QK_EPS, L["sk"]), *self.rope, n_dims=nd)
            ctx = (ctx - attention(qd, kd, v)).astype(np.float32)
        return L["out"](ctx.reshape(ctx.shape[0], d))

    def _cross_attention(self, L, h: np.ndarray, ctx_in: np.ndarray) -> np.ndarray:
        d = self.cfg.embed_dim
        qa, kv = L["q"](h), L["kv"](ctx_in)
        q = rms_norm(self._heads(qa[:, :d]), QK_EPS, L["cq"])
        k = rms_norm(self._heads(kv[:, :d]), QK_EPS, L["ck"])
        if self.cfg.differential:
            qd = rms_norm(self._heads(qa[:, d:2 * d]), QK_EPS, L["cq"])
            kd = rms_norm(self._heads(kv[:, d:2 * d]), QK_EPS, L["ck"])
            v = self._heads(kv[:, 2 * d:3 * d])
            ctx = (attention(q, k, v) - attention(qd, kd, v)).astype(np.float32)
        else:
            v = self._heads(kv[:, d:2 * d])
            ctx = attention(q, k, v)
        return L["cout"](ctx.reshape(ctx.shape[0], d))

    def forward(self, x: np.ndarray, sigma: float, cross: np.ndarray, glob: np.ndarray, local: np.ndarray,
                pad: np.ndarray) -> np.ndarray:
        """One graph-batch row: x [T, 64] (BTC), cross [P + 1, cond_dim], glob [global_cond_dim],
        local [T, local_add_cond_dim], pad [M + T] -> raw model output [T, 64]."""
        cfg = self.cfg
        d, M = cfg.embed_dim, cfg.num_memory_tokens
        hx = (x + self.pre(x)).astype(np.float32)
        h = np.concatenate([self.memory, self.pin(hx)]).astype(np.float32)
        ctx = self.cond2(_silu(self.cond0(cross)))
        arg = (f32(sigma) * self.freqs).astype(np.float32)
        feat = np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)[None, :]
        temb = self.t2(_silu(self.t0(feat)))
        g = (self.glob2(_silu(self.glob0(glob[None, :]))) + temb).astype(np.float32)
        six = self.ge2(_silu(self.ge0(g)))[0]
        for L in self.layers:
            ada = (six + L["ssg"]).astype(np.float32)
            sc_s, sh_s, g_s, sc_f, sh_f, g_f = (ada[i * d:(i + 1) * d] for i in range(6))
            hn = (rms_norm(h, NORM_EPS, L["pre"]) * (f32(1.0) + sc_s) + sh_s).astype(np.float32)
            att = (self._self_attention(L, hn, pad) * _sigmoid(f32(1.0) - g_s)).astype(np.float32)
            h = (h + att).astype(np.float32)
            h = (h + self._cross_attention(L, rms_norm(h, NORM_EPS, L["cross_n"]), ctx)).astype(np.float32)
            loc = L["lo2"](_silu(L["lo0"](local)))
            h = (h + np.concatenate([np.zeros((M, d), np.float32), loc])).astype(np.float32)
            fn = (rms_norm(h, NORM_EPS, L["ff_n"]) * (f32(1.0) + sc_f) + sh_f).astype(np.float32)
            p = L["ff0"](fn)
            ff = L["ff2"]((p[:, :4 * d] * _silu(p[:, 4 * d:])).astype(np.float32))
            h = (h + ff * _sigmoid(f32(1.0) - g_f)).astype(np.float32)
        y = self.pout(h[M:])
        return (y + self.post(y)).astype(np.float32)


def apg_cfg(raw: np.ndarray, x_cond: np.ndarray, sigma: np.ndarray, B_: int, mask: np.ndarray, cfg_scale: float,
            apg: float) -> np.ndarray:
    """build_cfg_model_output: raw [2B, T, 64], x_cond [B, T, 64], sigma [B], mask [B, T] -> guided v [B, T, 64]."""
    out = np.zeros_like(x_cond)
    for b in range(B_):
        s = f32(sigma[b])
        cx0 = (x_cond[b] - raw[b] * s).astype(np.float32)
        ux0 = (x_cond[b] - raw[B_ + b] * s).astype(np.float32)
        diff = (cx0 - ux0).astype(np.float32)
        m = mask[b][:, None]
        cm = (cx0 * m).astype(np.float32)
        norm = f32(np.sqrt(f32(np.sum((cm * cm).astype(np.float64)) + 1e-16)))
        v1 = (cm / norm).astype(np.float32)
        dot = f32(np.sum((diff * v1).astype(np.float64)))
        orth = ((diff - dot * v1) * m).astype(np.float32)
        cdiff = (f32(apg) * orth + f32(1.0 - apg) * diff).astype(np.float32)
        den = (cx0 + f32(cfg_scale - 1.0) * cdiff).astype(np.float32)
        out[b] = ((x_cond[b] - den) / s).astype(np.float32)
    return out


def sample(dit: Sa3Dit, cfg: Sa3Config, inp: Dict[str, B.Tensor]) -> np.ndarray:
    """StableAudioRfDitRuntime::sample: latents [B, 64, T] after len(schedule) - 1 steps."""
    Bn, T, C = cfg.batch, cfg.latent_tokens, cfg.io_channels
    M = cfg.num_memory_tokens
    use_cfg = cfg.cfg != 1.0
    Bg = 2 * Bn if use_cfg else Bn
    latent = inp["noise"].array().astype(np.float32).copy()
    sched = inp["schedule"].array()
    pos, neg = inp["cross_positive"].array(), inp["cross_negative"].array()
    nmask = inp["negative_mask"].array()
    glob, local, pmask = inp["global"].array(), inp["local_add"].array(), inp["padding_mask"].array()
    # cond || uncond (the negative prompt's masked-out tokens stay zero; global and local duplicated)
    cross = [pos[b] for b in range(Bn)]
    if use_cfg:
        cross += [(neg[b] * (nmask[b][:, None] != 0)).astype(np.float32) if int(inp["has_negative"].data[0])
                  else np.zeros_like(pos[b]) for b in range(Bn)]
    pads = [np.concatenate([np.ones(M, np.float32), pmask[bb % Bn]]) for bb in range(Bg)]
    seed, sms, mt = cfg.seed, cfg.rng_sms, cfg.rng_max_threads
    offset = int(inp["rng_offset"].data[0])
    for step in range(sched.shape[1] - 1):
        sig, nxt = sched[:, step], sched[:, step + 1]
        xg = latent.transpose(0, 2, 1)  # BTC
        raw = np.stack([dit.forward(xg[bb % Bn], float(sig[bb % Bn]), cross[bb], glob[bb % Bn],
                                    local[bb % Bn], pads[bb]) for bb in range(Bg)])
        v = apg_cfg(raw, xg, sig, Bn, pmask, cfg.cfg, cfg.apg) if use_cfg else raw
        v = v.transpose(0, 2, 1)  # BCT
        if cfg.sampler == "pingpong":
            noise = philox.tensor_iterator_randn(latent.size, seed, offset, sms, mt).reshape(latent.shape)
            offset += philox.offset_blocks(latent.size, sms, mt)
            for b in range(Bn):
                den = (latent[b] - f32(sig[b]) * v[b]).astype(np.float32)
                latent[b] = ((f32(1.0) - f32(nxt[b])) * den + f32(nxt[b]) * noise[b]).astype(np.float32)
        else:
            for b in range(Bn):
                latent[b] = (latent[b] + f32(nxt[b] - sig[b]) * v[b]).astype(np.float32)
    return latent
