"""Numpy restatement of the Stable Audio Oobleck VAE decoder (TEST ORACLE -- checker only).

Reference (audio.cpp, src/models/stable_audio/foundation/oobleck_autoencoder.cpp):
* decoder_channels: same_channels x (1, c_mults...)                                   :38-47
* effective_weight_norm_conv: w = v * g / sqrt(max(sum v^2 (fp64 sum), 1e-24)) per dim-0 row   :60-84
* snake_beta: x + sin(exp(alpha) x)^2 / (exp(beta) + 1e-9)                            :209-224
* residual_unit: snake -> conv k7 (dilation d, padding 3d) -> snake -> conv k1 -> + x  :226-239
* decoder_block: snake -> ConvTranspose1d(k 2s, stride s) -> crop [ceil(s/2), +L s) -> residual units d = 1, 3, 9  :241-264
* DecodeGraph::build_graph_output: in-conv k7 -> blocks (deepest first) -> snake -> out-conv k7 (no bias)  :675-692
* decode: latents [B, latent_dim, T] -> audio per prompt, interleaved [frames, channels]  :600-640
"""
from __future__ import annotations

import math
from typing import Dict

import numpy as np

from . import bundle as B
from .synth import OP, OobleckConfig

f32 = np.float32


def weight_norm(v: np.ndarray, g: np.ndarray) -> np.ndarray:
    outer = v.shape[0]
    flat = v.reshape(outer, -1).astype(np.float32)
    out = np.empty_like(flat)
    for o in range(outer):
        nsq = float(np.sum(flat[o].astype(np.float64) ** 2))
        scale = f32(f32(g.reshape(-1)[o]) / f32(math.sqrt(f32(max(nsq, 1e-24)))))
        out[o] = (flat[o] * scale).astype(np.float32)
    return out.reshape(v.shape)


def snake(x: np.ndarray, alpha_log: np.ndarray, beta_log: np.ndarray) -> np.ndarray:
    """x [C, L]."""
    a = np.exp(alpha_log.astype(np.float32)).astype(np.float32)[:, None]
    b = np.exp(beta_log.astype(np.float32)).astype(np.float32)[:, None]
    s = np.sin((x * a).astype(np.float32)).astype(np.float32)
    return (x + (s * s).astype(np.float32) / (b + f32(1e-9))).astype(np.float32)


def conv1d(x: np.ndarray, w: np.ndarray, b, pad: int, dil: int) -> np.ndarray:
    """Stride-1 conv: x [Cin, L], w [Cout, Cin, K] -> [Cout, L + 2 pad - dil (K - 1)]."""
    cin, L = x.shape
    cout, _, K = w.shape
    xp = np.zeros((cin, L + 2 * pad), np.float32)
    xp[:, pad:pad + L] = x
    Lo = L + 2 * pad - dil * (K - 1)
    cols = np.stack([xp[:, k * dil:k * dil + Lo] for k in range(K)], axis=1)  # [Cin, K, Lo]
    y = (w.reshape(cout, cin * K) @ cols.reshape(cin * K, Lo)).astype(np.float32)
    if b is not None:
        y = (y + b[:, None]).astype(np.float32)
    return y


def conv_transpose1d(x: np.ndarray, w: np.ndarray, b: np.ndarray, stride: int) -> np.ndarray:
    """x [Cin, L], w [Cin, Cout, K] -> [Cout, (L - 1) stride + K] (padding 0, dilation 1)."""
    cin, L = x.shape
    _, cout, K = w.shape
    y = np.zeros((cout, (L - 1) * stride + K), np.float32)
    contrib = np.einsum("ct,cok->okt", x, w).astype(np.float32)  # [Cout, K, L]
    for k in range(K):
        y[:, k:k + (L - 1) * stride + 1:stride] += contrib[:, k, :]
    return (y + b[:, None]).astype(np.float32)


class OobleckDecoder:
    def __init__(self, w: Dict[str, B.Tensor], cfg: OobleckConfig):
        self.cfg = cfg

        def arr(name):
            return w[name].array().astype(np.float32)

        def wn(prefix):
            return weight_norm(arr(prefix + ".weight_v"), arr(prefix + ".weight_g"))

        def sn(prefix):
            return arr(prefix + ".alpha"), arr(prefix + ".beta")

        n = len(cfg.strides)
        self.in_w, self.in_b = wn(OP + "0"), arr(OP + "0.bias")
        self.blocks = []
        for i in range(1, n + 1):
            p = OP + str(i) + ".layers."
            res = []
            for r, dil in ((2, 1), (3, 3), (4, 9)):
                q = p + str(r) + ".layers."
                res.append((dil, sn(q + "0"), wn(q + "1"), arr(q + "1.bias"), sn(q + "2"), wn(q + "3"),
                            arr(q + "3.bias")))
            self.blocks.append((cfg.strides[n - i], sn(p + "0"), wn(p + "1"), arr(p + "1.bias"), res))
        self.final_snake = sn(OP + str(n + 1))
        self.out_w = wn(OP + str(n + 2))

    def decode_one(self, z: np.ndarray) -> np.ndarray:
        """z [latent_dim, T] -> audio [channels, T x prod(strides)]."""
        h = conv1d(z, self.in_w, self.in_b, 3, 1)
        for stride, s0, wt, bt, res in self.blocks:
            L = h.shape[1]
            h = conv_transpose1d(snake(h, *s0), wt, bt, stride)
            crop = int(math.ceil(stride / 2.0))
            h = h[:, crop:crop + L * stride]
            for dil, sa, w1, b1, sb, w3, b3 in res:
                y = conv1d(snake(h, *sa), w1, b1, 3 * dil, dil)
                y = conv1d(snake(y, *sb), w3, b3, 0, 1)
                h = (h + y).astype(np.float32)
        h = snake(h, *self.final_snake)
        return conv1d(h, self.out_w, None, 3, 1)

    def decode(self, latents: np.ndarray) -> np.ndarray:
        """latents [B, latent_dim, T] -> audio [B, frames, channels] (interleaved as AudioBuffer.samples)."""
        return np.stack([self.decode_one(latents[b]).T for b in range(latents.shape[0])]).astype(np.float32)
