"""Numpy restatement of the Stable Audio Open 1.0 ("foundation") DiT denoiser and
its DPM++ 2M sampler with CFG/APG (TEST ORACLE -- checker only).

Reference (audio.cpp, src/models/stable_audio/foundation/rf_dit.cpp):
* timestep features / embedding   :163-173, :939-950 (write_timestep_features)
* layer_norm / rf_layer            :132-139, :288-305
* self-attention (+ partial NEOX RoPE, V x padding mask)  :200-237
* cross-attention (KV heads repeated)                     :113-130, :239-271
* SwiGLU feed-forward               :273-286
* graph body (pre/post conv, project in/out, global token) :952-986
* CFG + APG in-graph combine        :988-1028
* polyexponential sigmas / DPM++ 2M :606-626, :798-883
RoPE follows ggml's rope_f32 NEOX path (external/ggml/src/ggml-cpu/ops.cpp:5761-5775,5849-5866,5923):
theta_i = pos * theta_scale^i by repeated fp32 multiplication, theta_scale = powf(1e4, -2/n_dims).
"""
from __future__ import annotations

import math
from typing import Dict

import numpy as np

from . import bundle as B
from .synth import DP, DitConfig
from .vibevoice import Linear, _silu

f32 = np.float32
PI = f32(3.14159265358979323846)
EPS = 1e-5


def layer_norm(x: np.ndarray, g: np.ndarray, b: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    mean = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mean) ** 2).mean(axis=-1, keepdims=True)
    scale = (f32(1.0) / np.sqrt((var + EPS).astype(np.float32))).astype(np.float32)
    y = ((x - mean.astype(np.float32)) * scale).astype(np.float32)
    return (y * g + b).astype(np.float32)


def rope_tables(n_pos: int, n_dims: int = 32, base: float = 10000.0):
    theta_scale = f32(np.power(f32(base), f32(-2.0) / f32(n_dims)))
    cos = np.zeros((n_pos, n_dims // 2), np.float32)
    sin = np.zeros((n_pos, n_dims // 2), np.float32)
    for p in range(n_pos):
        th = f32(p)
        for i in range(n_dims // 2):
            cos[p, i] = np.cos(th)
            sin[p, i] = np.sin(th)
            th = f32(th * theta_scale)
    return cos, sin


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, n_dims: int = 32) -> np.ndarray:
    """x [..., T, heads, 64]; NEOX rotation of dims (i, i + n_dims/2) for i < n_dims/2."""
    h = n_dims // 2
    out = x.copy()
    c = cos[:, None, :]
    s = sin[:, None, :]
    x0, x1 = x[..., :h], x[..., h:n_dims]
    out[..., :h] = (x0 * c - x1 * s).astype(np.float32)
    out[..., h:n_dims] = (x0 * s + x1 * c).astype(np.float32)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """q [Lq, H, 64], k/v [Lk, H, 64] -> [Lq, H, 64], scale 1/8, fp64 softmax."""
    qh = q.transpose(1, 0, 2).astype(np.float64)
    kh = k.transpose(1, 0, 2).astype(np.float64)
    vh = v.transpose(1, 0, 2).astype(np.float64)
    s = qh @ kh.transpose(0, 2, 1) / math.sqrt(q.shape[-1])
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return (p @ vh).transpose(1, 0, 2).astype(np.float32)


class Dit:
    def __init__(self, w: Dict[str, B.Tensor], cfg: DitConfig, act: str = "ggml"):
        self.cfg = cfg
        self.act = act

        def lin(name, bias=False, conv=False):
            t = w[DP + name + ".weight"]
            if conv:
                t = B.Tensor(t.dtype, t.dims[:2], t.data)
            b = w[DP + name + ".bias"].data.astype(np.float32) if bias else None
            return Linear(t, b, act=act)

        self.freqs = w[DP + "timestep_features.weight"].data.astype(np.float32)
        self.cond0, self.cond2 = lin("to_cond_embed.0"), lin("to_cond_embed.2")
        self.glob0, self.glob2 = lin("to_global_embed.0"), lin("to_global_embed.2")
        self.t0, self.t2 = lin("to_timestep_embed.0", True), lin("to_timestep_embed.2", True)
        self.pre, self.post = lin("preprocess_conv", conv=True), lin("postprocess_conv", conv=True)
        self.pin, self.pout = lin("transformer.project_in"), lin("transformer.project_out")
        self.layers = []
        for i in range(cfg.depth):
            p = "transformer.layers.%d." % i
            g = lambda n: w[DP + p + n].data.astype(np.float32)
            self.layers.append(dict(
                ln=[(g(n + ".gamma"), g(n + ".beta")) for n in ("pre_norm", "cross_attend_norm", "ff_norm")],
                qkv=lin(p + "self_attn.to_qkv"), out=lin(p + "self_attn.to_out"), q=lin(p + "cross_attn.to_q"),
                kv=lin(p + "cross_attn.to_kv"), cout=lin(p + "cross_attn.to_out"),
                ff0=lin(p + "ff.ff.0.proj", True), ff2=lin(p + "ff.ff.2", True)))

    def timestep_features(self, t: float, rows: int) -> np.ndarray:
        arg = ((f32(t) * self.freqs.reshape(-1)) * f32(2.0) * PI).astype(np.float32)
        row = np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)
        return np.tile(row, (rows, 1))

    def forward(self, x: np.ndarray, t: float, cross: np.ndarray, glob: np.ndarray, pad: np.ndarray) -> np.ndarray:
        """x [Bg, T, 64] (BTC), cross [Bg, P+2, c], glob [Bg, gd], pad [Bg, T+1] -> raw [Bg, T, 64]."""
        cfg = self.cfg
        Bg, T, C = x.shape
        d, nh, hd = cfg.embed_dim, cfg.num_heads, cfg.head_dim
        kvh = cfg.cond_token_dim // hd
        h = (self.pre(x.reshape(-1, C)) + x.reshape(-1, C)).astype(np.float32)
        h = self.pin(h).reshape(Bg, T, d)
        cr = self.cond2(_silu(self.cond0(cross.reshape(-1, cross.shape[-1])))).reshape(Bg, -1, cfg.cond_token_dim)
        g = self.glob2(_silu(self.glob0(glob)))
        g = (g + self.t2(_silu(self.t0(self.timestep_features(t, Bg))))).astype(np.float32)
        h = np.concatenate([g[:, None, :], h], axis=1)
        cos, sin = rope_tables(T + 1, max(hd // 2, 32))
        for L in self.layers:
            out = np.empty_like(h)
            for b in range(Bg):
                hb = h[b]
                a = layer_norm(hb, *L["ln"][0])
                qkv = L["qkv"](a)
                q = apply_rope(qkv[:, :d].reshape(T + 1, nh, hd), cos, sin)
                k = apply_rope(qkv[:, d:2 * d].reshape(T + 1, nh, hd), cos, sin)
                v = (qkv[:, 2 * d:].reshape(T + 1, nh, hd) * pad[b][:, None, None]).astype(np.float32)
                hb = (hb + L["out"](attention(q, k, v).reshape(T + 1, d))).astype(np.float32)
                a = layer_norm(hb, *L["ln"][1])
                q = L["q"](a).reshape(T + 1, nh, hd)
                kv = L["kv"](cr[b])
                kk = np.repeat(kv[:, :cfg.cond_token_dim].reshape(-1, kvh, hd), nh // kvh, axis=1)
                vv = np.repeat(kv[:, cfg.cond_token_dim:].reshape(-1, kvh, hd), nh // kvh, axis=1)
                hb = (hb + L["cout"](attention(q, kk, vv).reshape(T + 1, d))).astype(np.float32)
                a = layer_norm(hb, *L["ln"][2])
                p = L["ff0"](a)
                inner = 4 * d
                hb = (hb + L["ff2"]((p[:, :inner] * _silu(p[:, inner:])).astype(np.float32))).astype(np.float32)
                out[b] = hb
            h = out
        y = self.pout(h.reshape(-1, d)).reshape(Bg, T + 1, C)[:, 1:]
        y2 = y.reshape(-1, C)
        return (y2 + self.post(y2)).reshape(Bg, T, C).astype(np.float32)


def cfg_apg(raw: np.ndarray, x_in: np.ndarray, t: float, B_: int, mask: np.ndarray, cfg_scale: float,
            apg: float) -> np.ndarray:
    """build_cfg_model_output (rf_dit.cpp:988-1028): raw [2B, T, C], x_in [B, T, C], mask [B, T] -> [B, T, C]."""
    sigma = f32(math.sin(float(f32(t) * PI * f32(0.5))))
    alpha = f32(math.cos(float(f32(t) * PI * f32(0.5))))
    cond, uncond = raw[:B_], raw[B_:]
    xa = (x_in * alpha).astype(np.float32)
    cx0 = (xa - cond * sigma).astype(np.float32)
    ux0 = (xa - uncond * sigma).astype(np.float32)
    diff = (cx0 - ux0).astype(np.float32)
    m = mask[:, :, None].astype(np.float32)
    cm = (cx0 * m).astype(np.float32)
    n = np.sqrt((np.sum(cm.astype(np.float64) ** 2, axis=(1, 2)) + 1e-16).astype(np.float32))[:, None, None]
    v1 = (cm / n).astype(np.float32)
    dot = np.sum((diff * v1).astype(np.float64), axis=(1, 2)).astype(np.float32)[:, None, None]
    orth = ((diff - dot * v1) * m).astype(np.float32)
    cd = (f32(apg) * orth + (f32(1.0) - f32(apg)) * diff).astype(np.float32)
    den = (cx0 + (f32(cfg_scale) - f32(1.0)) * cd).astype(np.float32)
    return ((xa - den) / sigma).astype(np.float32)


def polyexponential_sigmas(steps: int, smin: float, smax: float, rho: float):
    sig = [f32(0.0)] * (steps + 1)
    for i in range(steps):
        ramp = f32(1.0) if steps == 1 else f32(np.power(f32(1.0) - f32(i) / f32(steps - 1), f32(rho)))
        sig[i] = f32(np.exp(f32(ramp * f32(f32(np.log(f32(smax))) - f32(np.log(f32(smin))))) + f32(np.log(f32(smin)))))
    return sig


def _graph_inputs(cfg: DitConfig, inp: Dict[str, B.Tensor]):
    Bn, T = cfg.batch, cfg.latent_tokens
    use_cfg = cfg.cfg != 1.0
    pos, neg = inp["cross_positive"].array(), inp["cross_negative"].array()
    glob = inp["global"].array()
    pmask = inp["padding_mask"].array()
    cross = np.concatenate([pos, neg if int(inp["has_negative"].data[0]) else np.zeros_like(pos)]) if use_cfg else pos
    globg = np.concatenate([glob, glob]) if use_cfg else glob
    pad = np.ones((2 * Bn if use_cfg else Bn, T + 1), np.float32)
    pad[:, 1:] = np.concatenate([pmask, pmask]) if use_cfg else pmask
    return use_cfg, cross, globg, pad, pmask


def _model(dit: Dit, cfg: DitConfig, xin: np.ndarray, t_per_b: np.ndarray, cross, globg, pad, pmask, use_cfg):
    """run_dit_model with per-prompt timesteps: xin [B, C, T] -> model output [B, C, T]."""
    Bn = cfg.batch
    xbtc = xin.transpose(0, 2, 1)
    xg = np.concatenate([xbtc, xbtc]) if use_cfg else xbtc
    tg = np.concatenate([t_per_b, t_per_b]) if use_cfg else t_per_b
    if np.all(tg == tg[0]):
        raw = dit.forward(np.ascontiguousarray(xg), float(tg[0]), cross, globg, pad)
    else:  # per-row timestep features: run the graph row by row
        raw = np.concatenate([dit.forward(np.ascontiguousarray(xg[i:i + 1]), float(tg[i]), cross[i:i + 1],
                                          globg[i:i + 1], pad[i:i + 1]) for i in range(len(tg))])
    if not use_cfg:
        return raw.transpose(0, 2, 1)
    outs = [cfg_apg(raw[[b, Bn + b]], xbtc[b:b + 1], float(t_per_b[b]), 1, pmask[b:b + 1], cfg.cfg, cfg.apg)
            for b in range(Bn)]
    return np.concatenate(outs).transpose(0, 2, 1)


def sample_v_ddim(dit: Dit, cfg: DitConfig, inp: Dict[str, B.Tensor]) -> np.ndarray:
    """Graph::sample_v_ddim (rf_dit.cpp:514-604) on sampling.schedule [B, steps + 1]."""
    use_cfg, cross, globg, pad, pmask = _graph_inputs(cfg, inp)
    sched = inp["schedule"].array().reshape(cfg.batch, cfg.steps + 1)
    x = inp["noise"].array().astype(np.float32).copy()
    for step in range(cfg.steps):
        t = sched[:, step].astype(np.float32)
        tn = sched[:, step + 1].astype(np.float32)
        al = np.array([f32(math.cos(float(f32(v) * PI * f32(0.5)))) for v in t], np.float32)[:, None, None]
        sg = np.array([f32(math.sin(float(f32(v) * PI * f32(0.5)))) for v in t], np.float32)[:, None, None]
        aln = np.array([f32(math.cos(float(f32(v) * PI * f32(0.5)))) for v in tn], np.float32)[:, None, None]
        sgn = np.array([f32(math.sin(float(f32(v) * PI * f32(0.5)))) for v in tn], np.float32)[:, None, None]
        mo = _model(dit, cfg, x, t, cross, globg, pad, pmask, use_cfg)
        pred = (x * al - mo * sg).astype(np.float32)
        if step + 1 < cfg.steps:
            eps = (x * sg + mo * al).astype(np.float32)
            x = (pred * aln + eps * sgn).astype(np.float32)
        else:
            x = pred
    return x


def sample_dpmpp_3m_sde(dit: Dit, cfg: DitConfig, inp: Dict[str, B.Tensor]) -> np.ndarray:
    """Graph::sample_dpmpp_3m_sde (rf_dit.cpp:680-796); noise from the torch-CUDA TensorIterator Philox stream."""
    from . import philox
    use_cfg, cross, globg, pad, pmask = _graph_inputs(cfg, inp)
    seed = int(inp["seed"].data[0])
    sms, mt = int(inp["rng_sms"].data[0]), int(inp["rng_max_threads"].data[0])
    offset = int(inp["rng_offset"].data[0]) if "rng_offset" in inp else 0
    sig = polyexponential_sigmas(cfg.steps, cfg.sigma_min, cfg.sigma_max, cfg.rho)
    x = (inp["noise"].array() * sig[0]).astype(np.float32)
    d1 = d2 = None
    h1 = h2 = f32(0.0)
    for step in range(cfg.steps):
        s, sn = sig[step], sig[step + 1]
        c_in = f32(f32(1.0) / f32(math.sqrt(float(f32(s * s + f32(1.0))))))
        c_skip = f32(f32(1.0) / f32(s * s + f32(1.0)))
        c_out = f32(-s / f32(math.sqrt(float(f32(s * s + f32(1.0))))))
        t = f32(f32(math.atan(float(s))) * f32(2.0) / PI)
        mo = _model(dit, cfg, (x * c_in).astype(np.float32), np.full(cfg.batch, t, np.float32), cross, globg, pad,
                    pmask, use_cfg)
        den = (mo * c_out + x * c_skip).astype(np.float32)
        if sn == 0.0:
            x = den
            break
        h = f32(-f32(np.log(sn)) + f32(np.log(s)))
        he = f32(h * f32(2.0))
        x = (f32(np.exp(-he)) * x + f32(-np.expm1(-he)) * den).astype(np.float32)
        if d2 is not None:
            r0, r1 = f32(h1 / h), f32(h2 / h)
            phi2 = f32(f32(np.expm1(-he)) / he + f32(1.0))
            phi3 = f32(phi2 / he - f32(0.5))
            a = ((den - d1) / r0).astype(np.float32)
            b = ((d1 - d2) / r1).astype(np.float32)
            dd1 = (a + (a - b) * r0 / f32(r0 + r1)).astype(np.float32)
            dd2 = ((a - b) / f32(r0 + r1)).astype(np.float32)
            x = (x + phi2 * dd1 - phi3 * dd2).astype(np.float32)
        elif d1 is not None:
            r = f32(h1 / h)
            phi2 = f32(f32(np.expm1(-he)) / he + f32(1.0))
            x = (x + phi2 * ((den - d1) / r)).astype(np.float32)
        noise = philox.tensor_iterator_randn(x.size, seed, offset, sms, mt).reshape(x.shape)
        offset += philox.offset_blocks(x.size, sms, mt)
        x = (x + noise * f32(sn * f32(math.sqrt(float(f32(-np.expm1(f32(-2.0) * h))))))).astype(np.float32)
        d2, d1 = d1, den
        h2, h1 = h1, h
    return x


def sample(dit: Dit, cfg: DitConfig, inp: Dict[str, B.Tensor]) -> np.ndarray:
    return {"dpmpp-2m": sample_dpmpp_2m, "dpmpp-3m-sde": sample_dpmpp_3m_sde, "": sample_v_ddim}[cfg.sampler](
        dit, cfg, inp)


def sample_dpmpp_2m(dit: Dit, cfg: DitConfig, inp: Dict[str, B.Tensor]) -> np.ndarray:
    """Graph::sample_dpmpp_2m (rf_dit.cpp:798-883) with the graph's CFG/APG. Returns latents [B, 64, T]."""
    Bn, T, C = cfg.batch, cfg.latent_tokens, cfg.io_channels
    use_cfg = cfg.cfg != 1.0
    Bg = 2 * Bn if use_cfg else Bn
    noise = inp["noise"].array()
    pos, neg = inp["cross_positive"].array(), inp["cross_negative"].array()
    glob = inp["global"].array()
    pmask = inp["padding_mask"].array()
    cross = np.concatenate([pos, neg if int(inp["has_negative"].data[0]) else np.zeros_like(pos)]) if use_cfg else pos
    globg = np.concatenate([glob, glob]) if use_cfg else glob
    pad = np.ones((Bg, T + 1), np.float32)
    pad[:, 1:] = np.concatenate([pmask, pmask]) if use_cfg else pmask
    sig = polyexponential_sigmas(cfg.steps, cfg.sigma_min, cfg.sigma_max, cfg.rho)
    x = (noise * sig[0]).astype(np.float32)
    old = None
    for step in range(cfg.steps):
        s, sn = sig[step], sig[step + 1]
        c_in = f32(f32(1.0) / f32(math.sqrt(float(f32(s * s + f32(1.0))))))
        c_skip = f32(f32(1.0) / f32(s * s + f32(1.0)))
        c_out = f32(-s / f32(math.sqrt(float(f32(s * s + f32(1.0))))))
        t = f32(f32(math.atan(float(s))) * f32(2.0) / PI)
        xin = (x * c_in).astype(np.float32)                      # [B, C, T]
        xbtc = xin.transpose(0, 2, 1)
        xg = np.concatenate([xbtc, xbtc]) if use_cfg else xbtc
        raw = dit.forward(np.ascontiguousarray(xg), float(t), cross, globg, pad)
        out = cfg_apg(raw, xbtc, float(t), Bn, pmask, cfg.cfg, cfg.apg) if use_cfg else raw
        mo = out.transpose(0, 2, 1)
        den = (mo * c_out + x * c_skip).astype(np.float32)
        if sn == 0.0:
            x = den
            break
        h = f32(-f32(np.log(sn)) + f32(np.log(s)))
        xs = f32(sn / s)
        ds = f32(-np.expm1(f32(-h)))
        if old is None:
            x = (xs * x + ds * den).astype(np.float32)
        else:
            hl = f32(f32(np.log(sig[step - 1])) - f32(np.log(s)))
            r = f32(hl / h)
            dc = f32(f32(1.0) + f32(1.0) / f32(f32(2.0) * r))
            oc = f32(-f32(1.0) / f32(f32(2.0) * r))
            x = (xs * x + ds * (dc * den + oc * old)).astype(np.float32)
        old = den
    return x
