"""Q8_0 / F16 / BF16 weight encodings, restated from vendored ggml (test oracle).

* ``quantize_q8_0``   follows ``quantize_row_q8_0_ref``  (external/ggml/src/ggml-quants.c:234-257):
  per 32-element block, d = amax/127 (fp32), id = 1/d (0 when d == 0),
  q = roundf(x*id) (half away from zero), d stored as fp16 (round to nearest even).
* ``dequantize_q8_0`` follows ``dequantize_row_q8_0`` (ggml-quants.c:491-505): x = q * fp32(d).
* ``to_bf16_bits``    follows ``ggml_compute_fp32_to_bf16`` (external/ggml/src/ggml-impl.h:611-624).
* ``quantize_q8_0_activations`` follows the x86 activation quantizer ggml's CPU
  matmul applies to activations before a Q8_0 dot product
  (external/ggml/src/ggml-cpu/arch/x86/quants.c ``quantize_row_q8_0``: id = 127/amax,
  round to nearest even) -- used only to reproduce the reference's numerics.

A Q8_0 block is 34 bytes: fp16 d (little endian) followed by 32 int8 quants
(external/ggml/src/ggml-common.h:241-246).
"""
from __future__ import annotations

import numpy as np

QK = 32
BLOCK_BYTES = 34


def _round_half_away(v: np.ndarray) -> np.ndarray:
    v64 = v.astype(np.float64)
    return np.sign(v64) * np.floor(np.abs(v64) + 0.5)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """[rows, K] float32 -> [rows, K/32*34] uint8 GGUF Q8_0 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    if k % QK:
        raise ValueError("Q8_0 row length must be a multiple of 32")
    blocks = x.reshape(rows, k // QK, QK)
    amax = np.max(np.abs(blocks), axis=2)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, np.float32(1)), np.float32(0)).astype(np.float32)
    scaled = (blocks * idv[:, :, None]).astype(np.float32)
    q = _round_half_away(scaled).astype(np.int8)
    out = np.empty((rows, k // QK, BLOCK_BYTES), dtype=np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, k // QK, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, (k // QK) * BLOCK_BYTES)


def split_q8_0(qbytes: np.ndarray, k: int):
    """GGUF Q8_0 bytes [rows, K/32*34] -> (int8 quants [rows, K], fp16 scales [rows, K/32])."""
    rows = qbytes.size // ((k // QK) * BLOCK_BYTES)
    b = np.ascontiguousarray(qbytes, dtype=np.uint8).reshape(rows, k // QK, BLOCK_BYTES)
    d = b[:, :, 0:2].copy().view(np.float16).reshape(rows, k // QK)
    q = b[:, :, 2:].copy().view(np.int8).reshape(rows, k)
    return q, d


def dequantize_q8_0(qbytes: np.ndarray, k: int) -> np.ndarray:
    q, d = split_q8_0(qbytes, k)
    rows = q.shape[0]
    return (q.reshape(rows, k // QK, QK).astype(np.float32) * d.astype(np.float32)[:, :, None]).reshape(rows, k)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    rounded = ((u.astype(np.uint64) + 0x7FFF + ((u >> np.uint32(16)) & np.uint32(1))) >> 16).astype(np.uint16)
    quiet = ((u >> np.uint32(16)) | np.uint32(64)).astype(np.uint16)
    return np.where(nan, quiet, rounded).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def quantize_q8_0_activations(x: np.ndarray) -> np.ndarray:
    """Round activation rows the way ggml's CPU Q8_0 matmul does; returns the dequantized fp32 values."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    blocks = x.reshape(rows, k // QK, QK)
    amax = np.max(np.abs(blocks), axis=2).astype(np.float32)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(amax != 0, np.float32(127.0) / np.where(amax != 0, amax, np.float32(1)), np.float32(0)).astype(np.float32)
    q = np.rint((blocks * idv[:, :, None]).astype(np.float32))
    d16 = d.astype(np.float16).astype(np.float32)
    return (q * d16[:, :, None]).reshape(rows, k).astype(np.float32)
