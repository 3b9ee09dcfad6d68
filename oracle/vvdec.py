"""Numpy restatement of the VibeVoice acoustic sigma-VAE decoder (TEST ORACLE -- checker only).

Reference (audio.cpp, src/models/vibevoice/tokenizer_audio.cpp):
* load_decoder: stem, upsample_layers, stages (decoder depths = reversed encoder depths), norm, head  :322-388
* sconv1d: causal left padding (K - 1) dil - (stride - 1) plus the extra right padding, then Conv1d  :390-475
* sconv_depthwise1d: the same padding around a depthwise Conv1d (+ bias)                               :477-511
* sconv_transpose1d: ConvTranspose1d (k 2r, stride r) then trim K - r frames on the right               :513-544
* channel_rms_norm: RMSNorm over channels with weight (eps layernorm_eps)                             :679-689
* tokenizer_block: x + gamma * dwconv(rms(x)); then + ffn_gamma * linear2(gelu_erf(linear1(rms(x))))   :719-740
* build_decoder                                                                                         :814-838
* VibeVoiceTokenizerDecoderGraph::run: latents [frames, vae_dim] -> channel-major -> mono samples      :1013-1133
"""
from __future__ import annotations

import math
from typing import Dict

import numpy as np

from . import bundle as B
from .synth import VVDecConfig

f32 = np.float32
P = "model.acoustic_tokenizer.decoder"


def _erf(x: np.ndarray) -> np.ndarray:
    return np.vectorize(math.erf, otypes=[np.float64])(x.astype(np.float64)).astype(np.float32)


def gelu_erf(x: np.ndarray) -> np.ndarray:
    return (f32(0.5) * x * (f32(1.0) + _erf((x / f32(math.sqrt(2.0))).astype(np.float32)))).astype(np.float32)


def causal_conv1d(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Stride-1 sconv1d: x [Cin, L], w [Cout, Cin, K] -> [Cout, L] with K - 1 zeros on the left."""
    cin, L = x.shape
    cout, _, K = w.shape
    xp = np.concatenate([np.zeros((cin, K - 1), np.float32), x], axis=1)
    cols = np.stack([xp[:, k:k + L] for k in range(K)], axis=1)  # [Cin, K, L]
    return (w.reshape(cout, cin * K) @ cols.reshape(cin * K, L) + b[:, None]).astype(np.float32)


def causal_depthwise(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """x [C, L], w [C, 1, K]."""
    C, L = x.shape
    K = w.shape[2]
    xp = np.concatenate([np.zeros((C, K - 1), np.float32), x], axis=1)
    y = np.zeros((C, L), np.float32)
    for k in range(K):
        y += (w[:, 0, k:k + 1] * xp[:, k:k + L]).astype(np.float32)
    return (y + b[:, None]).astype(np.float32)


def conv_transpose_trim(x: np.ndarray, w: np.ndarray, b: np.ndarray, r: int) -> np.ndarray:
    """x [Cin, L], w [Cin, Cout, 2r] -> the first L r frames of the full transposed conv (+ bias)."""
    cin, L = x.shape
    _, cout, K = w.shape
    y = np.zeros((cout, (L - 1) * r + K), np.float32)
    contrib = np.einsum("ct,cok->okt", x, w).astype(np.float32)
    for k in range(K):
        y[:, k:k + (L - 1) * r + 1:r] += contrib[:, k, :]
    return (y[:, :L * r] + b[:, None]).astype(np.float32)


def rms_channels(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    ms = np.mean((x.astype(np.float64) ** 2), axis=0).astype(np.float32)
    return (x / np.sqrt(ms + f32(eps))[None, :] * w[:, None]).astype(np.float32)


class AcousticDecoder:
    def __init__(self, w: Dict[str, B.Tensor], cfg: VVDecConfig):
        self.cfg = cfg
        self.w = {k: v.array().astype(np.float32) for k, v in w.items() if k.startswith(P)}

    def _block(self, x: np.ndarray, p: str) -> np.ndarray:
        w, eps = self.w, self.cfg.eps
        h = rms_channels(x, w[p + ".norm.weight"], eps)
        h = causal_depthwise(h, w[p + ".mixer.conv.conv.conv.weight"], w[p + ".mixer.conv.conv.conv.bias"])
        x = (x + h * w[p + ".gamma"][:, None]).astype(np.float32)
        h = rms_channels(x, w[p + ".ffn_norm.weight"], eps).T  # [L, C]
        h = (h @ w[p + ".ffn.linear1.weight"].T + w[p + ".ffn.linear1.bias"]).astype(np.float32)
        h = gelu_erf(h)
        h = (h @ w[p + ".ffn.linear2.weight"].T + w[p + ".ffn.linear2.bias"]).astype(np.float32).T
        return (x + h * w[p + ".ffn_gamma"][:, None]).astype(np.float32)

    def decode(self, latents: np.ndarray) -> np.ndarray:
        """latents [frames, vae_dim] -> mono samples [frames x prod(ratios)]."""
        w, cfg = self.w, self.cfg
        h = latents.T.astype(np.float32)
        dd = list(reversed(cfg.depths))
        for s, dep in enumerate(dd):
            if s == 0:
                h = causal_conv1d(h, w[P + ".upsample_layers.0.0.conv.conv.weight"],
                                  w[P + ".upsample_layers.0.0.conv.conv.bias"])
            else:
                q = P + ".upsample_layers.%d.0.convtr.convtr" % s
                h = conv_transpose_trim(h, w[q + ".weight"], w[q + ".bias"], cfg.ratios[s - 1])
            for b in range(dep):
                h = self._block(h, P + ".stages.%d.%d" % (s, b))
        if not cfg.disable_last_norm:
            h = rms_channels(h, w[P + ".norm.weight"], cfg.eps)
        return causal_conv1d(h, w[P + ".head.conv.conv.weight"], w[P + ".head.conv.conv.bias"])[0]
