"""Seeded synthetic weights and inputs for the hot-path configurations (test oracle).

There are no real checkpoints or prompts in this environment; every config
uses random-init weights of the reference architecture and random inputs with
the shapes and distributions the configurations specify:

* weights ~ N(0, 0.02) (seed ``wseed``), stored as F16 / BF16 / Q8_0 exactly as
  the reference's weight store would encode them (RNE fp16, ggml's bf16
  rounding, ``quantize_row_q8_0_ref``); RMSNorm weights / LayerNorm gamma =
  1 + N(0, 0.02), LayerNorm beta = N(0, 0.02), kept in f32;
* head conditions ~ N(0, 1) (seed 1), null condition = zeros, x_T ~ N(0, 1) (seed 2);
* DiT: noise ~ N(0, 1), T5 states ~ N(0, 1), global ~ N(0, 1), per-prompt seeds.

Tensor names and shapes follow the reference's loaders:
``load_vibevoice_diffusion_head_weights`` (src/models/vibevoice/diffusion_head.cpp:335-399)
and ``load_foundation_rf_dit_weights`` (src/models/stable_audio/foundation/rf_dit.cpp:379-416).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict

import numpy as np

from . import bundle as B
from . import q8

F16, BF16, Q8_0, F32 = "f16", "bf16", "q8_0", "f32"


def _normal(rng: np.random.Generator, shape, std=1.0) -> np.ndarray:
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def encode_weight(w: np.ndarray, wtype: str) -> B.Tensor:
    """Encode an fp32 [out, in(, 1)] weight in the stored type."""
    dims = w.shape
    flat2d = w.reshape(-1, dims[-1]) if len(dims) == 2 else w.reshape(dims[0], -1)
    if wtype == F32:
        return B.Tensor(B.F32, dims, w.reshape(-1))
    if wtype == F16:
        return B.Tensor(B.F16, dims, w.astype(np.float16).reshape(-1))
    if wtype == BF16:
        return B.Tensor(B.BF16, dims, q8.to_bf16_bits(w).reshape(-1))
    if wtype == Q8_0:
        return B.Tensor(B.Q8_0, dims, q8.quantize_q8_0(flat2d).reshape(-1))
    raise ValueError(wtype)


def decode_weight(t: B.Tensor) -> np.ndarray:
    """Stored weight -> fp32 [out, in] (the values the reference computes with)."""
    dims = t.dims
    k = dims[1] if len(dims) >= 2 else dims[0]
    rows = dims[0]
    if t.dtype == B.F32:
        return t.data.reshape(rows, -1).astype(np.float32)
    if t.dtype == B.F16:
        return t.data.reshape(rows, -1).astype(np.float32)
    if t.dtype == B.BF16:
        return q8.from_bf16_bits(t.data).reshape(rows, -1)
    if t.dtype == B.Q8_0:
        return q8.dequantize_q8_0(t.data, int(np.prod(dims[1:])))
    raise ValueError(t.dtype)


# --------------------------------------------------------------- VibeVoice head
@dataclass
class HeadConfig:
    hidden: int = 1536
    latent: int = 64
    layers: int = 4
    ffn_ratio: float = 3.0
    eps: float = 1e-5
    ddpm_num_steps: int = 1000
    wtype: str = F16
    frames: int = 64
    steps: int = 10
    cfg: float = 1.3
    wseed: int = 0
    cseed: int = 1
    xseed: int = 2

    @property
    def ffn(self) -> int:
        return int(float(self.hidden) * self.ffn_ratio)

    def scalars(self) -> Dict[str, B.Tensor]:
        return {
            "hidden_size": B.i64(self.hidden), "latent_size": B.i64(self.latent),
            "head_layers": B.i64(self.layers), "head_ffn_ratio": B.f32(self.ffn_ratio),
            "rms_norm_eps": B.f32(self.eps), "ddpm_num_steps": B.i64(self.ddpm_num_steps),
            "inference_steps": B.i64(self.steps), "guidance_scale": B.f32(self.cfg),
        }


HEAD_CONFIGS = {
    # the benchmarked head configurations (C1, C2, C5)
    "vv15_f16_64": HeadConfig(wtype=F16, frames=64),
    "vv15_q8_1024": HeadConfig(wtype=Q8_0, frames=1024),
    "vv7_q8_8192": HeadConfig(hidden=3584, wtype=Q8_0, frames=8192),
    # C5's 7B width (hidden 3584, F = 10752, adaLN N = 50176) at 32 frames and 3 steps: parity at that shape
    # C5's per-rank share at 8 GPUs (1024 of the 8192 frames, 7B width, all 10 steps): full-length parity
    "vv7_q8_1024": HeadConfig(hidden=3584, wtype=Q8_0, frames=1024),
    "vv7_q8_32_3steps": HeadConfig(hidden=3584, wtype=Q8_0, frames=32, steps=3, wseed=7, cseed=8, xseed=9),
    # small parity configs
    "tiny_f16": HeadConfig(hidden=256, wtype=F16, frames=8),
    "tiny_q8": HeadConfig(hidden=256, wtype=Q8_0, frames=8),
    "tiny_bf16": HeadConfig(hidden=256, wtype=BF16, frames=5),
    "small_q8_ragged": HeadConfig(hidden=512, wtype=Q8_0, frames=100, steps=5),
    "one_frame_f16": HeadConfig(hidden=256, wtype=F16, frames=1, steps=3),
    "one_step_q8": HeadConfig(hidden=256, wtype=Q8_0, frames=4, steps=1, cfg=1.0),
}

HP = "model.prediction_head."


def head_weights(cfg: HeadConfig) -> Dict[str, B.Tensor]:
    rng = np.random.default_rng(cfg.wseed)
    H, F, L = cfg.hidden, cfg.ffn, cfg.latent
    w: Dict[str, B.Tensor] = {}

    def lin(name, out, inp):
        w[HP + name + ".weight"] = encode_weight(_normal(rng, (out, inp), 0.02), cfg.wtype)

    lin("noisy_images_proj", H, L)
    lin("cond_proj", H, H)
    lin("t_embedder.mlp.0", H, 256)
    lin("t_embedder.mlp.2", H, H)
    for i in range(cfg.layers):
        p = "layers.%d." % i
        lin(p + "ffn.gate_proj", F, H)
        lin(p + "ffn.up_proj", F, H)
        lin(p + "ffn.down_proj", H, F)
        w[HP + p + "norm.weight"] = B.f32(1.0 + _normal(rng, (H,), 0.02))
        lin(p + "adaLN_modulation.1", 3 * H, H)
    lin("final_layer.adaLN_modulation.1", 2 * H, H)
    lin("final_layer.linear", L, H)
    return w


def head_inputs(cfg: HeadConfig) -> Dict[str, B.Tensor]:
    cond = _normal(np.random.default_rng(cfg.cseed), (cfg.frames, cfg.hidden))
    x0 = _normal(np.random.default_rng(cfg.xseed), (2 * cfg.frames, cfg.latent))
    d = cfg.scalars()
    d["positive_condition"] = B.f32(cond)
    d["negative_condition"] = B.f32(np.zeros_like(cond))
    d["initial_speech"] = B.f32(x0)
    return d


# ----------------------------------------------------------- Stable Audio DiT
@dataclass
class DitConfig:
    embed_dim: int = 1536
    depth: int = 24
    num_heads: int = 24
    cond_token_dim: int = 768
    global_cond_dim: int = 1536
    io_channels: int = 64
    prompt_max_length: int = 128
    latent_tokens: int = 1024
    batch: int = 1
    steps: int = 100
    cfg: float = 7.0
    apg: float = 1.0
    sigma_min: float = 0.01
    sigma_max: float = 100.0
    rho: float = 1.0
    wtype: str = BF16
    wseed: int = 0
    prompt_seeds: tuple = field(default_factory=lambda: (0,))
    sampler: str = "dpmpp-2m"     # "dpmpp-2m", "dpmpp-3m-sde" or "" (v-DDIM on a given schedule)
    seed: int = 42                # Philox seed of the SDE noise
    rng_sms: int = 148            # TorchCudaSamplingPolicy of the reference caller
    rng_max_threads: int = 2048
    ragged_mask: bool = False

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    def scalars(self) -> Dict[str, B.Tensor]:
        return {k: B.i64(getattr(self, k)) for k in (
            "io_channels", "embed_dim", "depth", "num_heads", "cond_token_dim", "global_cond_dim",
            "prompt_max_length", "latent_tokens", "batch", "steps")} | {
            k + "": B.f32(getattr(self, a)) for k, a in (
                ("cfg_scale", "cfg"), ("apg_scale", "apg"), ("sigma_min", "sigma_min"),
                ("sigma_max", "sigma_max"), ("rho", "rho"))}


DIT_CONFIGS = {
    "sao_bf16_1x1024": DitConfig(),
    "sao_q8_16x1024": DitConfig(wtype=Q8_0, batch=16, prompt_seeds=tuple(range(16))),
    # full-size parity cases (the C3 / C4 shapes, 2 DPM++ steps so the CPU reference finishes in about a minute)
    "sao_bf16_1x1024_2steps": DitConfig(steps=2),
    # C3 at 10 DPM++ 2M steps: the multistep (second-order) update at full size, with the reference's latents
    # (BF16 and F32 weights) and the fp32-activation restatement
    "sao_bf16_1x1024_10steps": DitConfig(steps=10),
    # C3 in full (100 DPM++ 2M steps), with APG (the reference default) and as plain CFG
    "sao_bf16_1x1024_noapg": DitConfig(apg=0.0),
    # C4 at its full latent length: 16 prompts + CFG = 32 sequences x 1025 tokens, Q8_0, 2 steps
    "sao_q8_16x1024_2steps": DitConfig(wtype=Q8_0, batch=16, prompt_seeds=tuple(range(16)), steps=2),
    "sao_q8_1x1024_2steps": DitConfig(wtype=Q8_0, steps=2, prompt_seeds=(5,)),
    # C4's batch (16 prompts + CFG = 32 sequences, Q8_0, full width and depth) at 64 latent frames, 2 steps
    "sao_q8_16x64_2steps": DitConfig(wtype=Q8_0, batch=16, prompt_seeds=tuple(range(16)), latent_tokens=64, steps=2),
    "tiny_bf16": DitConfig(embed_dim=256, depth=2, num_heads=4, cond_token_dim=128, global_cond_dim=256,
                           prompt_max_length=14, latent_tokens=64, steps=6),
    "tiny_q8_b2_noapg": DitConfig(embed_dim=256, depth=2, num_heads=4, cond_token_dim=128, global_cond_dim=256,
                                  prompt_max_length=14, latent_tokens=48, steps=5, batch=2, apg=0.0,
                                  wtype=Q8_0, prompt_seeds=(3, 4)),
    "tiny_bf16_vddim": DitConfig(embed_dim=256, depth=2, num_heads=4, cond_token_dim=128, global_cond_dim=256,
                                 prompt_max_length=14, latent_tokens=40, steps=5, batch=2, sampler="",
                                 prompt_seeds=(6, 7), ragged_mask=True),
    "tiny_f16_3msde": DitConfig(embed_dim=256, depth=2, num_heads=4, cond_token_dim=128, global_cond_dim=256,
                                prompt_max_length=14, latent_tokens=40, steps=6, batch=2, sampler="dpmpp-3m-sde",
                                wtype=F16, prompt_seeds=(8, 9)),
    "tiny_f16_ragged": DitConfig(embed_dim=256, depth=1, num_heads=4, cond_token_dim=128, global_cond_dim=256,
                                 prompt_max_length=14, latent_tokens=37, steps=4, wtype=F16),
}

DP = "model.model."


def dit_weights(cfg: DitConfig) -> Dict[str, B.Tensor]:
    rng = np.random.default_rng(cfg.wseed)
    d, C, c = cfg.embed_dim, cfg.io_channels, cfg.cond_token_dim
    w: Dict[str, B.Tensor] = {}

    def lin(name, out, inp, bias=False, conv=False):
        shape = (out, inp, 1) if conv else (out, inp)
        # a [out, in, 1] conv weight has last dim 1, which GGUF cannot store as Q8_0 blocks;
        # the reference's weight store keeps such tensors in F32 (backend_weight_store.h:237-255)
        wtype = F32 if (conv and cfg.wtype == Q8_0) else cfg.wtype
        w[DP + name + ".weight"] = encode_weight(_normal(rng, shape, 0.02), wtype)
        if bias:
            w[DP + name + ".bias"] = B.f32(_normal(rng, (out,), 0.02))

    w[DP + "timestep_features.weight"] = B.f32(_normal(rng, (128, 1)))
    lin("to_cond_embed.0", c, c)
    lin("to_cond_embed.2", c, c)
    lin("to_global_embed.0", d, cfg.global_cond_dim)
    lin("to_global_embed.2", d, d)
    lin("to_timestep_embed.0", d, 256, bias=True)
    lin("to_timestep_embed.2", d, d, bias=True)
    lin("preprocess_conv", C, C, conv=True)
    lin("postprocess_conv", C, C, conv=True)
    lin("transformer.project_in", d, C)
    lin("transformer.project_out", C, d)
    for i in range(cfg.depth):
        p = "transformer.layers.%d." % i
        for n in ("pre_norm", "cross_attend_norm", "ff_norm"):
            w[DP + p + n + ".gamma"] = B.f32(1.0 + _normal(rng, (d,), 0.02))
            w[DP + p + n + ".beta"] = B.f32(_normal(rng, (d,), 0.02))
        lin(p + "self_attn.to_qkv", 3 * d, d)
        lin(p + "self_attn.to_out", d, d)
        lin(p + "cross_attn.to_q", d, d)
        lin(p + "cross_attn.to_kv", 2 * c, c)
        lin(p + "cross_attn.to_out", d, d)
        lin(p + "ff.ff.0.proj", 8 * d, d, bias=True)
        lin(p + "ff.ff.2", d, 4 * d, bias=True)
    return w


def dit_inputs(cfg: DitConfig) -> Dict[str, B.Tensor]:
    """Per prompt b (seed s_b): noise [64, T], T5 states [P, c] + the two c-halves of a
    global vector as the 2 number tokens, global [global_cond_dim]; negative cross = zeros."""
    Bn, T, C, c = cfg.batch, cfg.latent_tokens, cfg.io_channels, cfg.cond_token_dim
    P = cfg.prompt_max_length
    noise = np.zeros((Bn, C, T), np.float32)
    cross = np.zeros((Bn, P + 2, c), np.float32)
    glob = np.zeros((Bn, cfg.global_cond_dim), np.float32)
    for b, s in enumerate(cfg.prompt_seeds[:Bn]):
        rng = np.random.default_rng(1000 + s)
        noise[b] = _normal(rng, (C, T))
        cross[b, :P] = _normal(rng, (P, c))
        g = _normal(rng, (cfg.global_cond_dim,))
        glob[b] = g
        cross[b, P] = g[:c]
        cross[b, P + 1] = g[c:2 * c] if cfg.global_cond_dim >= 2 * c else g[:c]
    d = cfg.scalars()
    d["noise"] = B.f32(noise)
    d["cross_positive"] = B.f32(cross)
    d["cross_negative"] = B.f32(np.zeros_like(cross))
    d["global"] = B.f32(glob)
    mask = np.ones((Bn, T), np.float32)
    if cfg.ragged_mask:  # prompt b keeps its first T - 7 (b + 1) latent frames, as a shorter duration would
        for b in range(Bn):
            mask[b, T - 7 * (b + 1):] = 0.0
    d["padding_mask"] = B.f32(mask)
    d["has_negative"] = B.i64(1)
    d["sampler"] = B.i64({"dpmpp-2m": 0, "dpmpp-3m-sde": 1, "": 2}[cfg.sampler])
    d["seed"] = B.i64(cfg.seed)
    d["rng_sms"] = B.i64(cfg.rng_sms)
    d["rng_max_threads"] = B.i64(cfg.rng_max_threads)
    d["rng_offset"] = B.i64(0)
    # v-DDIM schedule [B, steps + 1]: 1 -> 0 with a per-prompt warp (make_schedule, stable_audio/sampler.cpp:131-154)
    lin = np.linspace(1.0, 0.0, cfg.steps + 1, dtype=np.float64)
    sched = np.stack([lin ** (1.0 + 0.25 * b) for b in range(Bn)]).astype(np.float32)
    sched[:, 0], sched[:, -1] = 1.0, 0.0
    d["schedule"] = B.f32(sched)
    return d


# ------------------------------------------------------------------ Stable Audio 3 DiT
@dataclass
class Sa3Config:
    """StableAudioConfig fields of the SA3 rectified-flow DiT (include/engine/models/stable_audio/assets.h:14-84)
    plus the sampling request (StableAudioRfDitRuntime::sample, src/models/stable_audio/rf_dit.cpp:586-694)."""
    embed_dim: int = 256
    depth: int = 2
    num_heads: int = 4
    cond_dim: int = 128
    global_cond_dim: int = 64
    local_add_cond_dim: int = 32
    num_memory_tokens: int = 4
    differential: bool = False
    io_channels: int = 64
    prompt_max_length: int = 14       # cross tokens = prompt_max_length + 1
    latent_tokens: int = 40
    batch: int = 1
    steps: int = 4
    cfg: float = 7.0
    apg: float = 1.0
    sampler: str = "pingpong"         # "pingpong" (Philox noise each step) or "euler"
    wtype: str = F32
    wseed: int = 3
    prompt_seeds: tuple = field(default_factory=lambda: (0,))
    seed: int = 7
    rng_sms: int = 148
    rng_max_threads: int = 2048
    ragged_mask: bool = False

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    def scalars(self) -> Dict[str, B.Tensor]:
        d = {k: B.i64(getattr(self, k)) for k in (
            "io_channels", "embed_dim", "depth", "num_heads", "cond_dim", "global_cond_dim", "local_add_cond_dim",
            "num_memory_tokens", "prompt_max_length", "latent_tokens", "batch", "steps", "seed", "rng_sms",
            "rng_max_threads")}
        d["differential"] = B.i64(int(self.differential))
        d["sampler"] = B.i64({"pingpong": 0, "euler": 1}[self.sampler])
        d["cfg_scale"] = B.f32(self.cfg)
        d["apg_scale"] = B.f32(self.apg)
        d["rng_offset"] = B.i64(0)
        return d


SA3_CONFIGS = {
    "sa3_tiny_f32": Sa3Config(),
    "sa3_tiny_f32_diff_b2": Sa3Config(differential=True, batch=2, prompt_seeds=(1, 2), ragged_mask=True),
    "sa3_tiny_f32_euler_nocfg": Sa3Config(sampler="euler", cfg=1.0, prompt_seeds=(3,)),
    "sa3_tiny_bf16_diff": Sa3Config(differential=True, wtype=BF16, prompt_seeds=(4,), steps=5),
    # several attention / GEMM tiles per sequence, a local-add width that is not a multiple of 64
    "sa3_mid_bf16_diff_b2": Sa3Config(embed_dim=512, num_heads=8, cond_dim=256, global_cond_dim=128,
                                      local_add_cond_dim=40, num_memory_tokens=8, prompt_max_length=30,
                                      latent_tokens=300, batch=2, differential=True, wtype=BF16, prompt_seeds=(5, 6),
                                      ragged_mask=True),
    # bench workload: the reference tree does not publish the SA3 transformer dimensions (they come from
    # the model package's JSON); this uses the SAO 1.0 transformer size with SA3's conditioning layout,
    # 120 s of latents at the SAO latent rate, the documented defaults (8 pingpong steps, CFG 7, APG 1)
    "sa3_bench_bf16": Sa3Config(embed_dim=1536, depth=24, num_heads=24, cond_dim=768, global_cond_dim=768,
                                local_add_cond_dim=64, num_memory_tokens=64, prompt_max_length=128,
                                latent_tokens=2584, steps=8, wtype=BF16, prompt_seeds=(0,)),
    # 128-wide GEMM tiles (3d, d not multiples of 256), Q8_0 weights, euler with partial APG
    "sa3_mid_q8_euler": Sa3Config(embed_dim=384, num_heads=6, cond_dim=192, global_cond_dim=64,
                                  local_add_cond_dim=32, num_memory_tokens=16, prompt_max_length=20,
                                  latent_tokens=200, cfg=4.5, apg=0.5, sampler="euler", wtype=Q8_0,
                                  prompt_seeds=(7,)),
}

SP = "model.model."


def sa3_weights(cfg: Sa3Config) -> Dict[str, B.Tensor]:
    """Tensor names and shapes of load_stable_audio_rf_dit_weights (rf_dit.cpp:386-585)."""
    rng = np.random.default_rng(cfg.wseed)
    d, C, hd = cfg.embed_dim, cfg.io_channels, cfg.head_dim
    w: Dict[str, B.Tensor] = {}

    def lin(name, out, inp, bias=False, conv=False, std=0.02):
        shape = (out, inp, 1) if conv else (out, inp)
        wtype = F32 if (conv and cfg.wtype == Q8_0) else cfg.wtype
        w[SP + name + ".weight"] = encode_weight(_normal(rng, shape, std), wtype)
        if bias:
            w[SP + name + ".bias"] = B.f32(_normal(rng, (out,), 0.02))

    def vec(name, n, base=0.0, std=0.02):
        w[SP + name] = B.f32(base + _normal(rng, (n,), std))

    lin("to_cond_embed.0", d, cfg.cond_dim)
    lin("to_cond_embed.2", d, d)
    lin("to_global_embed.0", d, cfg.global_cond_dim)
    lin("to_global_embed.2", d, d)
    lin("to_timestep_embed.0", d, 256, bias=True)
    lin("to_timestep_embed.2", d, d, bias=True)
    lin("preprocess_conv", C, C, conv=True)
    lin("postprocess_conv", C, C, conv=True)
    lin("transformer.project_in", d, C)
    lin("transformer.project_out", C, d)
    w[SP + "transformer.memory_tokens"] = B.f32(_normal(rng, (cfg.num_memory_tokens, d)))
    lin("transformer.global_cond_embedder.0", d, d, bias=True)
    lin("transformer.global_cond_embedder.2", 6 * d, d, bias=True)
    for i in range(cfg.depth):
        p = "transformer.layers.%d." % i
        for n in ("pre_norm", "cross_attend_norm", "ff_norm"):
            vec(p + n + ".gamma", d, 1.0)
        lin(p + "self_attn.to_qkv", d * (5 if cfg.differential else 3), d)
        lin(p + "self_attn.to_out", d, d)
        lin(p + "cross_attn.to_q", d * (2 if cfg.differential else 1), d)
        lin(p + "cross_attn.to_kv", d * (3 if cfg.differential else 2), d)
        lin(p + "cross_attn.to_out", d, d)
        for a in ("self_attn", "cross_attn"):
            vec(p + a + ".q_norm.gamma", hd, 1.0, 0.1)
            vec(p + a + ".k_norm.gamma", hd, 1.0, 0.1)
        lin(p + "ff.ff.0.proj", 8 * d, d, bias=True)
        lin(p + "ff.ff.2", d, 4 * d, bias=True)
        lin(p + "to_local_embed.0", d, cfg.local_add_cond_dim, bias=True)
        lin(p + "to_local_embed.2", d, d, bias=True)
        vec(p + "to_scale_shift_gate", 6 * d, 0.0, 0.1)
    return w


def sa3_inputs(cfg: Sa3Config) -> Dict[str, B.Tensor]:
    """Per prompt: noise [64, T], T5-like states [P + 1, cond_dim], global [global_cond_dim], local-add
    features [T, local_add_cond_dim]; the negative prompt keeps every other token (its mask) and zeros the rest;
    the rectified-flow schedule runs 1 -> 0 with a per-prompt warp."""
    Bn, T, C = cfg.batch, cfg.latent_tokens, cfg.io_channels
    P1 = cfg.prompt_max_length + 1
    noise = np.zeros((Bn, C, T), np.float32)
    cross = np.zeros((Bn, P1, cfg.cond_dim), np.float32)
    cneg = np.zeros_like(cross)
    glob = np.zeros((Bn, cfg.global_cond_dim), np.float32)
    local = np.zeros((Bn, T, cfg.local_add_cond_dim), np.float32)
    for b, s in enumerate(cfg.prompt_seeds[:Bn]):
        rng = np.random.default_rng(2000 + s)
        noise[b] = _normal(rng, (C, T))
        cross[b] = _normal(rng, (P1, cfg.cond_dim))
        cneg[b] = _normal(rng, (P1, cfg.cond_dim))
        glob[b] = _normal(rng, (cfg.global_cond_dim,))
        local[b] = _normal(rng, (T, cfg.local_add_cond_dim))
    nmask = np.zeros((Bn, P1), np.float32)
    nmask[:, ::2] = 1.0
    d = cfg.scalars()
    d["noise"] = B.f32(noise)
    d["cross_positive"] = B.f32(cross)
    d["cross_negative"] = B.f32(cneg)
    d["negative_mask"] = B.f32(nmask)
    d["has_negative"] = B.i64(1)
    d["global"] = B.f32(glob)
    d["local_add"] = B.f32(local)
    mask = np.ones((Bn, T), np.float32)
    if cfg.ragged_mask:
        for b in range(Bn):
            mask[b, T - 5 * (b + 1):] = 0.0
    d["padding_mask"] = B.f32(mask)
    lin = np.linspace(1.0, 0.0, cfg.steps + 1, dtype=np.float64)
    sched = np.stack([lin ** (1.0 + 0.3 * b) for b in range(Bn)]).astype(np.float32)
    sched[:, 0], sched[:, -1] = 1.0, 0.0
    d["schedule"] = B.f32(sched)
    return d


@dataclass
class OobleckConfig:
    """StableAudioConfig fields of the Oobleck VAE decoder (include/engine/models/stable_audio/assets.h:14-84:
    latent_dim, same_channels, same_c_mults, same_strides, audio_channels) and the decode request."""
    latent_dim: int = 64
    channels: int = 64
    c_mults: tuple = (1, 2, 4)
    strides: tuple = (2, 4, 2)
    audio_channels: int = 2
    batch: int = 1
    latent_tokens: int = 32
    wseed: int = 11
    seed: int = 12

    def decoder_channels(self):
        return [self.channels * m for m in (1,) + tuple(self.c_mults)]

    def scalars(self) -> Dict[str, B.Tensor]:
        d = {k: B.i64(getattr(self, k)) for k in ("latent_dim", "channels", "audio_channels", "batch",
                                                    "latent_tokens")}
        d["c_mults"] = B.i64(np.array(self.c_mults, np.int64))
        d["strides"] = B.i64(np.array(self.strides, np.int64))
        return d


OOBLECK_CONFIGS = {
    "oobleck_tiny": OobleckConfig(),
    "oobleck_tiny_b2_odd": OobleckConfig(c_mults=(1, 2), strides=(3, 5), batch=2, latent_tokens=21, wseed=13,
                                         seed=14),
    # bench: the Stable Audio Open 1.0 VAE shape (channels 128, c_mults 1 2 4 8 16, strides 2 4 4 8 8 -> 2048x
    # upsampling), one 1024-latent generation (47.5 s of 44.1 kHz stereo)
    "oobleck_bench_sao_1x1024": OobleckConfig(channels=128, c_mults=(1, 2, 4, 8, 16), strides=(2, 4, 4, 8, 8),
                                              latent_tokens=1024, wseed=15, seed=16),
    # parity at the bench's channel / stride shape on a short latent (16 latents -> 32768 frames)
    "oobleck_sao_shape_1x16": OobleckConfig(channels=128, c_mults=(1, 2, 4, 8, 16), strides=(2, 4, 4, 8, 8),
                                            latent_tokens=16, wseed=15, seed=17),
}

OP = "pretransform.model.decoder.layers."


def oobleck_weights(cfg: OobleckConfig) -> Dict[str, B.Tensor]:
    """Tensor names and shapes of load_oobleck_autoencoder_weights' decoder half
    (src/models/stable_audio/foundation/oobleck_autoencoder.cpp:334-420): weight-normalised convs stored as
    weight_v / weight_g (+ bias), snake alpha / beta stored as logarithms."""
    rng = np.random.default_rng(cfg.wseed)
    ch = cfg.decoder_channels()
    w: Dict[str, B.Tensor] = {}

    def conv(prefix, shape, gain, bias=True):
        w[prefix + ".weight_v"] = B.f32(_normal(rng, shape))
        w[prefix + ".weight_g"] = B.f32((gain * (0.75 + 0.5 * rng.random((shape[0], 1, 1)))).astype(np.float32))
        if bias:
            w[prefix + ".bias"] = B.f32(_normal(rng, (shape[0],), 0.02))

    def snake(prefix, c):
        w[prefix + ".alpha"] = B.f32(_normal(rng, (c,), 0.2))
        w[prefix + ".beta"] = B.f32(_normal(rng, (c,), 0.2))

    conv(OP + "0", (ch[-1], cfg.latent_dim, 7), 1.0)
    n = len(cfg.strides)
    for block in range(n, 0, -1):
        p = OP + str(n - block + 1) + ".layers."
        cin, cout, s = ch[block], ch[block - 1], cfg.strides[block - 1]
        snake(p + "0", cin)
        # ConvTranspose1d weight [in, out, 2 s], weight_g per input channel, bias per output channel
        w[p + "1.weight_v"] = B.f32(_normal(rng, (cin, cout, 2 * s)))
        w[p + "1.weight_g"] = B.f32((0.75 + 0.5 * rng.random((cin, 1, 1))).astype(np.float32))
        w[p + "1.bias"] = B.f32(_normal(rng, (cout,), 0.02))
        for r in (2, 3, 4):
            q = p + str(r) + ".layers."
            snake(q + "0", cout)
            conv(q + "1", (cout, cout, 7), 0.4)
            snake(q + "2", cout)
            conv(q + "3", (cout, cout, 1), 0.4)
    snake(OP + str(n + 1), ch[0])
    conv(OP + str(n + 2), (cfg.audio_channels, ch[0], 7), 1.0, bias=False)
    # the encoder half, which the reference's loader also requires (decode does not use it)
    E = "pretransform.model.encoder.layers."
    conv(E + "0", (ch[0], cfg.audio_channels, 7), 1.0)
    for block in range(n):
        p = E + str(block + 1) + ".layers."
        for r in range(3):
            q = p + str(r) + ".layers."
            snake(q + "0", ch[block])
            conv(q + "1", (ch[block], ch[block], 7), 0.4)
            snake(q + "2", ch[block])
            conv(q + "3", (ch[block], ch[block], 1), 0.4)
        snake(p + "3", ch[block])
        conv(p + "4", (ch[block + 1], ch[block], 2 * cfg.strides[block]), 1.0)
    snake(E + str(n + 1), ch[-1])
    conv(E + str(n + 2), (2 * cfg.latent_dim, ch[-1], 3), 1.0)
    return w


def oobleck_inputs(cfg: OobleckConfig) -> Dict[str, B.Tensor]:
    """Latents [B, latent_dim, T] ~ N(0, 1)."""
    d = cfg.scalars()
    d["latents"] = B.f32(_normal(np.random.default_rng(cfg.seed), (cfg.batch, cfg.latent_dim, cfg.latent_tokens)))
    return d


@dataclass
class VVDecConfig:
    """VibeVoiceTokenizerConfig fields of the acoustic sigma-VAE (include/engine/models/vibevoice/assets.h:15-37):
    decoder channels n_filters << (D - 1 - stage), decoder depths = reversed encoder depths, decoder ratios =
    encoder ratios; plus the small semantic encoder the tokenizer loader also reads."""
    vae_dim: int = 64
    n_filters: int = 64
    ratios: tuple = (2, 3)
    depths: tuple = (1, 1, 2)          # encoder depths; the decoder runs them reversed
    disable_last_norm: bool = True
    eps: float = 1e-5
    frames: int = 24
    semantic_vae_dim: int = 32
    wseed: int = 21
    seed: int = 22

    def scalars(self) -> Dict[str, B.Tensor]:
        d = {}
        for p, vd, nf, ratios, depths, dln in (("acoustic_", self.vae_dim, self.n_filters, self.ratios, self.depths,
                                                 self.disable_last_norm),
                                                ("semantic_", self.semantic_vae_dim, 32, (2,), (1, 1), True)):
            d[p + "vae_dim"] = B.i64(vd)
            d[p + "n_filters"] = B.i64(nf)
            d[p + "ratios"] = B.i64(np.array(ratios, np.int64))
            d[p + "depths"] = B.i64(np.array(depths, np.int64))
            d[p + "disable_last_norm"] = B.i64(int(dln))
            d[p + "eps"] = B.f32(self.eps)
        return d


VVDEC_CONFIGS = {
    "vvdec_tiny": VVDecConfig(),
    "vvdec_tiny_norm": VVDecConfig(ratios=(4, 2), depths=(2, 1, 1), disable_last_norm=False, frames=17, wseed=23,
                                   seed=24),
    # the released decoders' channel plan: 32 filters, so the last stage has 32 channels (zero-padded on the GPU)
    "vvdec_tiny_c32": VVDecConfig(n_filters=32, ratios=(2, 2), depths=(1, 1, 1), disable_last_norm=False, frames=20,
                                  wseed=25, seed=26),
}


def _tok_block(w, rng, p, c):
    w[p + ".norm.weight"] = B.f32(1.0 + _normal(rng, (c,), 0.1))
    w[p + ".mixer.conv.conv.conv.weight"] = B.f32(_normal(rng, (c, 1, 7), 0.3))
    w[p + ".mixer.conv.conv.conv.bias"] = B.f32(_normal(rng, (c,), 0.02))
    w[p + ".gamma"] = B.f32(_normal(rng, (c,), 0.3))
    w[p + ".ffn_norm.weight"] = B.f32(1.0 + _normal(rng, (c,), 0.1))
    w[p + ".ffn.linear1.weight"] = B.f32(_normal(rng, (4 * c, c), 1.0 / np.sqrt(c)))
    w[p + ".ffn.linear1.bias"] = B.f32(_normal(rng, (4 * c,), 0.02))
    w[p + ".ffn.linear2.weight"] = B.f32(_normal(rng, (c, 4 * c), 1.0 / np.sqrt(4 * c)))
    w[p + ".ffn.linear2.bias"] = B.f32(_normal(rng, (c,), 0.02))
    w[p + ".ffn_gamma"] = B.f32(_normal(rng, (c,), 0.3))


def _tok_conv(w, rng, p, shape):
    w[p + ".weight"] = B.f32(_normal(rng, shape, 1.0 / np.sqrt(shape[1] * shape[2]) if shape[1] > 1 else 0.3))
    w[p + ".bias"] = B.f32(_normal(rng, (shape[0],), 0.02))


def _tok_encoder(w, rng, prefix, vae_dim, nf, ratios, depths, last_norm):
    rr = list(reversed(ratios))
    _tok_conv(w, rng, prefix + ".downsample_layers.0.0.conv.conv", (nf, 1, 7))
    for i, r in enumerate(rr):
        _tok_conv(w, rng, prefix + ".downsample_layers.%d.0.conv.conv" % (i + 1), (nf << (i + 1), nf << i, 2 * r))
    for s, dep in enumerate(depths):
        for b in range(dep):
            _tok_block(w, rng, prefix + ".stages.%d.%d" % (s, b), nf << s)
    if last_norm:
        w[prefix + ".norm.weight"] = B.f32(1.0 + _normal(rng, (nf << (len(depths) - 1),), 0.1))
    _tok_conv(w, rng, prefix + ".head.conv.conv", (vae_dim, nf << (len(depths) - 1), 7))


def vvdec_weights(cfg: VVDecConfig) -> Dict[str, B.Tensor]:
    """Tensor names and shapes of load_vibevoice_tokenizer_weights (src/models/vibevoice/tokenizer_audio.cpp:
    214-388, 1507-1542): acoustic encoder + decoder and semantic encoder, f32."""
    rng = np.random.default_rng(cfg.wseed)
    w: Dict[str, B.Tensor] = {}
    D = len(cfg.depths)
    dd = list(reversed(cfg.depths))
    P = "model.acoustic_tokenizer.decoder"
    _tok_conv(w, rng, P + ".upsample_layers.0.0.conv.conv", (cfg.n_filters << (D - 1), cfg.vae_dim, 7))
    for i, r in enumerate(cfg.ratios):
        cin, cout = cfg.n_filters << (D - 1 - i), cfg.n_filters << (D - 2 - i)
        w[P + ".upsample_layers.%d.0.convtr.convtr.weight" % (i + 1)] = B.f32(
            _normal(rng, (cin, cout, 2 * r), 1.0 / np.sqrt(cin * 2)))
        w[P + ".upsample_layers.%d.0.convtr.convtr.bias" % (i + 1)] = B.f32(_normal(rng, (cout,), 0.02))
    for s, dep in enumerate(dd):
        for b in range(dep):
            _tok_block(w, rng, P + ".stages.%d.%d" % (s, b), cfg.n_filters << (D - 1 - s))
    if not cfg.disable_last_norm:
        w[P + ".norm.weight"] = B.f32(1.0 + _normal(rng, (cfg.n_filters,), 0.1))
    _tok_conv(w, rng, P + ".head.conv.conv", (1, cfg.n_filters, 7))
    _tok_encoder(w, rng, "model.acoustic_tokenizer.encoder", cfg.vae_dim, cfg.n_filters, cfg.ratios, cfg.depths,
                 not cfg.disable_last_norm)
    _tok_encoder(w, rng, "model.semantic_tokenizer.encoder", cfg.semantic_vae_dim, 32, (2,), (1, 1), False)
    return w


def vvdec_inputs(cfg: VVDecConfig) -> Dict[str, B.Tensor]:
    """Acoustic latents [frames, vae_dim] ~ N(0, 1) (VibeVoiceTokenizerLatents.values, time-major)."""
    d = cfg.scalars()
    d["latents"] = B.f32(_normal(np.random.default_rng(cfg.seed), (cfg.frames, cfg.vae_dim)))
    return d


@dataclass
class SaoCondConfig:
    """StableAudioConfig T5 fields (include/engine/models/stable_audio/assets.h:14-84) of the SAO 1.0
    conditioner, and one seeded token batch (ids, padding masks, normalized seconds_total)."""
    hidden: int = 128
    layers: int = 2
    heads: int = 2
    head_dim: int = 64
    intermediate: int = 256
    vocab: int = 200
    eps: float = 1e-6
    prompt_max_length: int = 12
    batch: int = 2
    has_negative: bool = True
    wseed: int = 31
    seed: int = 32

    def scalars(self) -> Dict[str, B.Tensor]:
        d = {"t5_" + k: B.i64(getattr(self, a)) for k, a in (
            ("hidden_size", "hidden"), ("layers", "layers"), ("heads", "heads"), ("head_dim", "head_dim"),
            ("intermediate", "intermediate"), ("vocab", "vocab"))}
        d["t5_eps"] = B.f32(self.eps)
        d["prompt_max_length"] = B.i64(self.prompt_max_length)
        d["batch"] = B.i64(self.batch)
        d["has_negative"] = B.i64(int(self.has_negative))
        return d


SAOCOND_CONFIGS = {
    "saocond_tiny": SaoCondConfig(),
    "saocond_tiny_b1_noneg": SaoCondConfig(layers=1, heads=4, head_dim=32, prompt_max_length=40, batch=1,
                                           has_negative=False, wseed=33, seed=34),
}


def saocond_weights(cfg: SaoCondConfig) -> Dict[str, B.Tensor]:
    """T5-base encoder tensors (load_t5_base_runtime_weights, conditioner.cpp:52-112, 202-233) and the two number
    conditioners (load_number_conditioner :165-175), f32."""
    rng = np.random.default_rng(cfg.wseed)
    d, I, H = cfg.hidden, cfg.intermediate, cfg.heads * cfg.head_dim
    w: Dict[str, B.Tensor] = {"shared.weight": B.f32(_normal(rng, (cfg.vocab, d)))}
    w["encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"] = B.f32(_normal(rng, (32, cfg.heads)))
    for l in range(cfg.layers):
        p = "encoder.block.%d.layer." % l
        w[p + "0.layer_norm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
        w[p + "1.layer_norm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
        for n in "qkv":
            w[p + "0.SelfAttention.%s.weight" % n] = B.f32(_normal(rng, (H, d), 1.0 / np.sqrt(d)))
        w[p + "0.SelfAttention.o.weight"] = B.f32(_normal(rng, (d, H), 1.0 / np.sqrt(H)))
        w[p + "1.DenseReluDense.wi.weight"] = B.f32(_normal(rng, (I, d), 1.0 / np.sqrt(d)))
        w[p + "1.DenseReluDense.wo.weight"] = B.f32(_normal(rng, (d, I), 1.0 / np.sqrt(I)))
    w["encoder.final_layer_norm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
    for n in ("seconds_start", "seconds_total"):
        p = "conditioner.conditioners.%s.embedder.embedding." % n
        w[p + "0.weights"] = B.f32(_normal(rng, (128,)))
        w[p + "1.weight"] = B.f32(_normal(rng, (d, 257), 1.0 / np.sqrt(257)))
        w[p + "1.bias"] = B.f32(_normal(rng, (d,), 0.02))
    return w


def saocond_inputs(cfg: SaoCondConfig) -> Dict[str, B.Tensor]:
    """Token ids in [1, vocab), padding after a per-prompt length, normalized seconds_total in (0, 1)."""
    rng = np.random.default_rng(cfg.seed)
    P = cfg.prompt_max_length
    d = cfg.scalars()
    for ids, mask in (("input_ids", "attention_mask"), ("negative_ids", "negative_mask")):
        lens = rng.integers(1, P + 1, cfg.batch)
        ids_a = rng.integers(1, cfg.vocab, (cfg.batch, P))
        m = (np.arange(P)[None, :] < lens[:, None]).astype(np.int64)
        d[ids] = B.i64(ids_a * m)
        d[mask] = B.i64(m)
    d["normalized_seconds"] = B.f32(rng.random(cfg.batch).astype(np.float32))
    return d


@dataclass
class VVLmConfig:
    """VibeVoiceDecoderConfig fields (include/engine/models/vibevoice/assets.h:39-54) of the Qwen2.5 LM that
    produces the diffusion head's conditions, and one prefill + cached-step request."""
    hidden: int = 128
    intermediate: int = 256
    heads: int = 4
    kv_heads: int = 2
    head_dim: int = 32
    layers: int = 2
    vocab: int = 300
    max_positions: int = 256
    eps: float = 1e-6
    rope_theta: float = 1e6
    prefill: int = 9
    steps: int = 3
    wseed: int = 41
    seed: int = 42

    def scalars(self) -> Dict[str, B.Tensor]:
        d = {k: B.i64(getattr(self, a)) for k, a in (
            ("hidden_size", "hidden"), ("intermediate_size", "intermediate"), ("num_heads", "heads"),
            ("num_kv_heads", "kv_heads"), ("num_layers", "layers"), ("vocab_size", "vocab"), ("head_dim", "head_dim"),
            ("max_positions", "max_positions"), ("prefill", "prefill"))}
        d["rms_norm_eps"] = B.f32(self.eps)
        d["rope_theta"] = B.f32(self.rope_theta)
        return d


VVLM_CONFIGS = {
    "vvlm_tiny": VVLmConfig(),
    "vvlm_tiny_mha_long": VVLmConfig(heads=2, kv_heads=2, head_dim=64, layers=1, prefill=70, steps=2, wseed=43,
                                     seed=44),
}


def vvlm_weights(cfg: VVLmConfig) -> Dict[str, B.Tensor]:
    """load_decoder_weights tensors (src/models/vibevoice/decoder.cpp:186-365), tied embeddings, f32."""
    rng = np.random.default_rng(cfg.wseed)
    d, I = cfg.hidden, cfg.intermediate
    q, kv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    P = "model.language_model."
    w: Dict[str, B.Tensor] = {P + "embed_tokens.weight": B.f32(_normal(rng, (cfg.vocab, d)))}
    for l in range(cfg.layers):
        p = P + "layers.%d." % l
        w[p + "input_layernorm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
        w[p + "post_attention_layernorm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
        for n, rows in (("q", q), ("k", kv), ("v", kv)):
            w[p + "self_attn.%s_proj.weight" % n] = B.f32(_normal(rng, (rows, d), 1.0 / np.sqrt(d)))
            w[p + "self_attn.%s_proj.bias" % n] = B.f32(_normal(rng, (rows,), 0.1))
        w[p + "self_attn.o_proj.weight"] = B.f32(_normal(rng, (d, q), 1.0 / np.sqrt(q)))
        w[p + "mlp.gate_proj.weight"] = B.f32(_normal(rng, (I, d), 1.0 / np.sqrt(d)))
        w[p + "mlp.up_proj.weight"] = B.f32(_normal(rng, (I, d), 1.0 / np.sqrt(d)))
        w[p + "mlp.down_proj.weight"] = B.f32(_normal(rng, (d, I), 1.0 / np.sqrt(I)))
    w[P + "norm.weight"] = B.f32(1.0 + _normal(rng, (d,), 0.1))
    return w


def vvlm_inputs(cfg: VVLmConfig) -> Dict[str, B.Tensor]:
    rng = np.random.default_rng(cfg.seed)
    d = cfg.scalars()
    d["prefill_ids"] = B.i64(rng.integers(0, cfg.vocab, cfg.prefill))
    d["step_ids"] = B.i64(rng.integers(0, cfg.vocab, cfg.steps))
    return d
