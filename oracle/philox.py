"""Numpy restatement of audio.cpp's torch-CUDA-compatible normal generator (TEST ORACLE).

Reference: src/framework/sampling/torch_random.cpp:17-99 (Philox4x32-10, Box-Muller,
per-index form) and :131-143, :186-246, :379-399 (TensorIterator layout: element
i = loop * 4 * stride + c * stride + seq takes component c of Philox(counter =
(offset_blocks + loop, seq)), stride = 256 * min(ceil(n / 256), SMs * max_threads / 256),
and each call advances offset_blocks by ceil(n / (4 * stride))).
Known-answer vectors: tests/unittests/test_torch_random.cpp:33-100.
"""
from __future__ import annotations

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint64(0x9E3779B9), np.uint64(0xBB67AE85)
MASK = np.uint64(0xFFFFFFFF)
INV_2_32 = np.float32(2.3283064365386963e-10)
INV_2_32_2PI = np.float32(1.4629180792671596e-09)


def philox4x32_10(c0, c1, c2, c3, seed: int):
    """Vectorised over counter arrays (uint64 holding 32-bit values)."""
    x, y, z, w = (np.asarray(v, np.uint64) & MASK for v in (c0, c1, c2, c3))
    k0 = np.uint64(seed & 0xFFFFFFFF)
    k1 = np.uint64((seed >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0 = M0 * x
        p1 = M1 * z
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        x, y, z, w = (hi1 ^ y ^ k0) & MASK, lo1, (hi0 ^ w ^ k1) & MASK, lo0
        k0 = (k0 + W0) & MASK
        k1 = (k1 + W1) & MASK
    return x, y, z, w


def box_muller(u0, u1):
    r_in = (u0.astype(np.float32) * INV_2_32 + INV_2_32 * np.float32(0.5)).astype(np.float32)
    ang = (u1.astype(np.float32) * INV_2_32_2PI + INV_2_32_2PI * np.float32(0.5)).astype(np.float32)
    r = np.sqrt(np.float32(-2.0) * np.log(r_in)).astype(np.float32)
    return (r * np.sin(ang)).astype(np.float32), (r * np.cos(ang)).astype(np.float32)


def round_bf16(v: np.ndarray) -> np.ndarray:
    b = v.astype(np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def torch_cuda_randn(count: int, seed: int, bf16: bool = False, start: int = 0) -> np.ndarray:
    """generate_torch_cuda_randn: element i = normal0 of Philox(counter = (0, 0, i_lo, i_hi))."""
    idx = np.arange(start, start + count, dtype=np.uint64)
    x, y, _, _ = philox4x32_10(0, 0, idx & MASK, idx >> np.uint64(32), seed)
    n0, _ = box_muller(x, y)
    return round_bf16(n0) if bf16 else n0


def iterator_stride(total: int, sms: int, max_threads: int) -> int:
    grid = (total + 255) // 256
    per_sm = max(1, max_threads // 256)
    return 256 * max(1, min(sms * per_sm, grid))


def offset_blocks(total: int, sms: int, max_threads: int) -> int:
    return (total - 1) // (iterator_stride(total, sms, max_threads) * 4) + 1


def tensor_iterator_randn(count: int, seed: int, offset: int, sms: int = 1, max_threads: int = 256,
                          bf16: bool = False) -> np.ndarray:
    stride = iterator_stride(count, sms, max_threads)
    i = np.arange(count, dtype=np.uint64)
    q = i // np.uint64(stride)
    loop = q // np.uint64(4)
    comp = (q % np.uint64(4)).astype(np.int64)
    seq = i % np.uint64(stride)
    ctr = np.uint64(offset) + loop
    x, y, z, w = philox4x32_10(ctr & MASK, ctr >> np.uint64(32), seq & MASK, seq >> np.uint64(32), seed)
    a0, a1 = box_muller(x, y)
    a2, a3 = box_muller(z, w)
    out = np.choose(comp, [a0, a1, a2, a3]).astype(np.float32)
    return round_bf16(out) if bf16 else out
