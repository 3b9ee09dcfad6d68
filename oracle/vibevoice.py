"""Numpy restatement of the VibeVoice diffusion head, DPM-Solver++ scheduler and
CFG sampler (TEST ORACLE -- checker only, never the product path).

Reference (audio.cpp):
* head forward        src/models/vibevoice/diffusion_head.cpp:130-220, 495-523
* timestep freqs      src/models/vibevoice/diffusion_head.cpp:59-66
* scheduler           src/models/vibevoice/scheduler.cpp:15-274
* sampler loop + CFG  src/models/vibevoice/diffusion_sampler.cpp:19-121

The matmuls reproduce ggml's CPU numerics: activations are rounded to the
weight's dot type before the product (F16 -> fp16, BF16 -> bf16, Q8_0 -> Q8_0
blocks; external/ggml/src/ggml-cpu/ggml-cpu.c:218-223,262-270,385-390) and the
product is accumulated in float64 here (fp32 in ggml), so the port tracks the
reference to ~1e-6 relative per op.  Norms reduce in float64 like ggml_rms_norm.
"""
from __future__ import annotations

import math
from typing import Dict, List

import numpy as np

from . import bundle as B
from . import q8
from .synth import HP, HeadConfig, decode_weight

f32 = np.float32


def _silu(x: np.ndarray) -> np.ndarray:
    return (x / (f32(1.0) + np.exp(-x))).astype(np.float32)


def round_activations(x: np.ndarray, wdtype: int) -> np.ndarray:
    if wdtype == B.F16:
        return x.astype(np.float16).astype(np.float32)
    if wdtype == B.BF16:
        return q8.from_bf16_bits(q8.to_bf16_bits(x)).reshape(x.shape)
    if wdtype == B.Q8_0:
        return q8.quantize_q8_0_activations(x)
    return x


class Linear:
    """y = x W^T (LinearModule::build, src/framework/modules/linear_module.cpp:73-108).

    act="ggml" rounds activations like ggml's CPU matmul; act="exact" keeps them
    fp32, which is the arithmetic the reference graph specifies and the GPU path
    approximates (fp16/bf16 operands, fp32 accumulation)."""

    def __init__(self, t: B.Tensor, bias: np.ndarray | None = None, act: str = "ggml"):
        self.dtype = t.dtype
        self.w = decode_weight(t).astype(np.float64)
        self.b = bias
        self.act = act

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        xr = round_activations(x, self.dtype) if self.act == "ggml" else x
        y = (xr.astype(np.float64) @ self.w.T).astype(np.float32)
        if self.b is not None:
            y = (y + self.b).astype(np.float32)
        return y


def rms_norm(x: np.ndarray, eps: float, weight: np.ndarray | None) -> np.ndarray:
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    scale = (f32(1.0) / np.sqrt((ms + eps).astype(np.float32))).astype(np.float32)
    y = (x * scale).astype(np.float32)
    if weight is not None:
        y = (y * weight).astype(np.float32)
    return y


def timestep_freqs() -> np.ndarray:
    half = 128
    i = np.arange(half, dtype=np.float32)
    return np.exp(f32(-math.log(10000.0)) * i / f32(half)).astype(np.float32)


class Head:
    """VibeVoiceDiffusionHeadWeightsRuntime::predict restated (diffusion_head.cpp:474-493)."""

    def __init__(self, weights: Dict[str, B.Tensor], cfg: HeadConfig, act: str = "ggml"):
        self.cfg = cfg
        def lin(name):
            return Linear(weights[HP + name + ".weight"], act=act)

        self.noisy = lin("noisy_images_proj")
        self.cond = lin("cond_proj")
        self.t1 = lin("t_embedder.mlp.0")
        self.t2 = lin("t_embedder.mlp.2")
        self.layers = []
        for i in range(cfg.layers):
            p = "layers.%d." % i
            self.layers.append(dict(
                gate=lin(p + "ffn.gate_proj"), up=lin(p + "ffn.up_proj"), down=lin(p + "ffn.down_proj"),
                norm=weights[HP + p + "norm.weight"].data.astype(np.float32), ada=lin(p + "adaLN_modulation.1")))
        self.fada = lin("final_layer.adaLN_modulation.1")
        self.flin = lin("final_layer.linear")
        self.freqs = timestep_freqs()

    def t_embedding(self, t: float, rows: int) -> np.ndarray:
        args = (np.full((rows, 1), t, np.float32) * self.freqs[None, :]).astype(np.float32)
        emb = np.concatenate([np.cos(args), np.sin(args)], axis=1).astype(np.float32)
        return self.t2(_silu(self.t1(emb)))

    def predict(self, noisy: np.ndarray, t: float, condition: np.ndarray) -> np.ndarray:
        H = self.cfg.hidden
        rows = noisy.shape[0]
        x = self.noisy(noisy)
        c = (self.cond(condition) + self.t_embedding(t, rows)).astype(np.float32)
        sc = _silu(c)
        for L in self.layers:
            mod = L["ada"](sc)
            shift, scale, gate = mod[:, :H], mod[:, H:2 * H], mod[:, 2 * H:]
            h = rms_norm(x, self.cfg.eps, L["norm"])
            h = (h * (f32(1.0) + scale) + shift).astype(np.float32)
            y = L["down"]((_silu(L["gate"](h)) * L["up"](h)).astype(np.float32))
            x = (x + gate * y).astype(np.float32)
        mod = self.fada(sc)
        shift, scale = mod[:, :H], mod[:, H:2 * H]
        h = rms_norm(x, self.cfg.eps, None)
        h = (h * (f32(1.0) + scale) + shift).astype(np.float32)
        return self.flin(h)


class Scheduler:
    """VibeVoiceDPMSolverScheduler restated (scheduler.cpp); fp32 scalar math as in C++."""

    def __init__(self, num_train_steps: int = 1000):
        pi = f32(3.14159265358979323846)

        def abar(t):
            v = f32(math.cos(float((f32(t) + f32(0.008)) / f32(1.008) * pi * f32(0.5))))
            return f32(v * v)

        cum = f32(1.0)
        ac = []
        for i in range(num_train_steps):
            t1 = f32(i) / f32(num_train_steps)
            t2 = f32(i + 1) / f32(num_train_steps)
            beta = min(f32(f32(1.0) - abar(t2) / abar(t1)), f32(0.999))
            cum = f32(cum * (f32(1.0) - beta))
            ac.append(cum)
        self.alphas_cumprod = np.array(ac, np.float32)
        self.num_train_steps = num_train_steps

    def set_timesteps(self, n: int) -> None:
        last = self.num_train_steps
        fwd = [int(np.rint(0.0 + (float(last - 1) - 0.0) * float(i) / float(n))) for i in range(n + 1)]
        self.timesteps = [fwd[i] for i in range(n, 0, -1)]
        base = np.sqrt(((f32(1.0) - self.alphas_cumprod) / self.alphas_cumprod).astype(np.float32)).astype(np.float32)
        self.sigmas = [f32(base[t]) for t in self.timesteps] + [f32(0.0)]

    @staticmethod
    def alpha_sigma(sigma):
        a = f32(f32(1.0) / f32(math.sqrt(float(f32(sigma * sigma + f32(1.0))))))
        return a, f32(sigma * a)

    @staticmethod
    def _lam(a, s):
        with np.errstate(divide="ignore"):
            return f32(np.log(np.float32(a)) - np.log(np.float32(s)))

    def coefficients(self, idx: int, order: int):
        """(sample_coeff, d0_coeff, second_order_d1_scale) for step idx, as scalar fp32."""
        a_t, s_t = self.alpha_sigma(self.sigmas[idx + 1])
        a_s0, s_s0 = self.alpha_sigma(self.sigmas[idx])
        lt, ls0 = self._lam(a_t, s_t), self._lam(a_s0, s_s0)
        h = f32(lt - ls0)
        with np.errstate(over="ignore"):
            e = f32(np.exp(np.float32(-h)))
        sample_coeff = f32(s_t / s_s0)
        d0 = f32(-a_t * f32(e - f32(1.0)))
        inv_r0 = f32(0.0)
        if order == 2:
            a_s1, s_s1 = self.alpha_sigma(self.sigmas[idx - 1])
            h0 = f32(ls0 - self._lam(a_s1, s_s1))
            r0 = f32(h0 / h)
            inv_r0 = f32(f32(1.0) / r0)
        return sample_coeff, d0, inv_r0

    def run(self, model_outputs: List[np.ndarray], sample: np.ndarray) -> List[np.ndarray]:
        """Apply step() for every timestep to the given per-step model outputs (vvsched KAT)."""
        hist: List[np.ndarray | None] = [None, None]
        trace = []
        lower = 0
        n = len(self.timesteps)
        for idx in range(n):
            a, s = self.alpha_sigma(self.sigmas[idx])
            conv = (a * sample - s * model_outputs[idx]).astype(np.float32)
            hist = [hist[1], conv]
            final = idx == n - 1
            if lower < 1 or final:
                sc, d0c, _ = self.coefficients(idx, 1)
                sample = (sc * sample + d0c * conv).astype(np.float32)
            else:
                sc, d0c, inv_r0 = self.coefficients(idx, 2)
                d1 = (inv_r0 * (hist[1] - hist[0])).astype(np.float32)
                sample = (sc * sample + d0c * hist[1] + f32(0.5) * d0c * d1).astype(np.float32)
            lower = min(lower + 1, 2)
            trace.append(sample.copy())
        return trace


def sample_speech_latents(head: Head, cfg: HeadConfig, pos: np.ndarray, neg: np.ndarray,
                          init: np.ndarray) -> np.ndarray:
    """sample_vibevoice_speech_latents restated (diffusion_sampler.cpp:79-121). Returns [B, latent]."""
    Bn = pos.shape[0]
    sched = Scheduler(cfg.ddpm_num_steps)
    sched.set_timesteps(cfg.steps)
    condition = np.concatenate([pos, neg], axis=0).astype(np.float32)
    speech = init.astype(np.float32).copy()
    hist: List[np.ndarray | None] = [None, None]
    lower = 0
    n = len(sched.timesteps)
    for idx, t in enumerate(sched.timesteps):
        combined = np.concatenate([speech[:Bn], speech[:Bn]], axis=0)
        pred = head.predict(combined, float(t), condition)
        c, u = pred[:Bn], pred[Bn:]
        g = (u + f32(cfg.cfg) * (c - u)).astype(np.float32)
        eps = np.concatenate([g, g], axis=0)
        a, s = sched.alpha_sigma(sched.sigmas[idx])
        conv = (a * speech - s * eps).astype(np.float32)
        hist = [hist[1], conv]
        if lower < 1 or idx == n - 1:
            sc, d0c, _ = sched.coefficients(idx, 1)
            speech = (sc * speech + d0c * conv).astype(np.float32)
        else:
            sc, d0c, inv_r0 = sched.coefficients(idx, 2)
            d1 = (inv_r0 * (hist[1] - hist[0])).astype(np.float32)
            speech = (sc * speech + d0c * hist[1] + f32(0.5) * d0c * d1).astype(np.float32)
        lower = min(lower + 1, 2)
    return speech[:Bn].copy()
