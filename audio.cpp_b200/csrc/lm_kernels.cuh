// Kernels of the VibeVoice language model (Qwen2.5 decoder, src/models/vibevoice/decoder.cpp) that are not GEMMs:
// NEOX RoPE over the full head dimension with the new rows' K / V appended to the per-layer cache, causal GQA
// attention of the new rows against the cache, and silu(gate) * up.
#pragma once

#include "kernels.cuh"

namespace b2d {

// qkv fp32 [n, (H + 2 KV) hd] ([q | k | v] per row, biases already added): rotate q and k of row r at position
// pos0 + r with tables cos / sin [max_pos][hd / 2] (NEOX pairs i, i + hd / 2), write q back in place and k, v
// into the layer's cache [max_pos][KV hd] (fp32).  One thread per (row, head slot, pair).
__global__ void lm_rope_append_kernel(float* __restrict__ qkv, int n, int H, int KV, int hd, int pos0,
                                      const float* __restrict__ cs, const float* __restrict__ sn,
                                      float* __restrict__ kcache, float* __restrict__ vcache) {
    const int half = hd / 2;
    const int slots = H + 2 * KV;
    const int64_t total = int64_t(n) * slots * half;
    const int ld = slots * hd;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int j = int(i % half);
        const int slot = int((i / half) % slots);
        const int r = int(i / (int64_t(half) * slots));
        const int pos = pos0 + r;
        float* row = qkv + int64_t(r) * ld + slot * hd;
        if (slot < H + KV) {
            const float c = cs[int64_t(pos) * half + j], s = sn[int64_t(pos) * half + j];
            const float x0 = row[j], x1 = row[j + half];
            const float y0 = x0 * c - x1 * s, y1 = x0 * s + x1 * c;
            if (slot < H) {
                row[j] = y0;
                row[j + half] = y1;
            } else {
                float* kr = kcache + int64_t(pos) * KV * hd + (slot - H) * hd;
                kr[j] = y0;
                kr[j + half] = y1;
            }
        } else {
            float* vr = vcache + int64_t(pos) * KV * hd + (slot - H - KV) * hd;
            vr[j] = row[j];
            vr[j + half] = row[j + half];
        }
    }
}

// Causal attention of the n new rows (positions pos0 ..) against the cache: head h reads KV head h / (H / KV),
// scores scaled by 1 / sqrt(hd), keys 0 .. pos; one warp per (row, head), lanes over the keys with an online
// softmax, then the context reduced across lanes.  Output ct [n, H hd].
template <typename CT, int HD>
__global__ void __launch_bounds__(256) lm_attention_kernel(const float* __restrict__ qkv, int n, int H, int KV,
                                                           int pos0, const float* __restrict__ kcache,
                                                           const float* __restrict__ vcache, CT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t unit = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (unit >= int64_t(n) * H) return;
    const int r = int(unit / H), h = int(unit % H);
    const int kvh = h / (H / KV);
    const int ld = (H + 2 * KV) * HD;
    const float* q = qkv + int64_t(r) * ld + h * HD;
    float qv[HD];
#pragma unroll
    for (int j = 0; j < HD; ++j) qv[j] = q[j];
    const float scale = 1.0f / sqrtf(float(HD));
    const int last = pos0 + r;
    float m = -INFINITY, l = 0.f, o[HD];
#pragma unroll
    for (int j = 0; j < HD; ++j) o[j] = 0.f;
    for (int k = lane; k <= last; k += 32) {
        const float* kr = kcache + int64_t(k) * KV * HD + kvh * HD;
        const float* vr = vcache + int64_t(k) * KV * HD + kvh * HD;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < HD; ++j) s += qv[j] * kr[j];
        s *= scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), p = expf(s - mn);
        l = l * corr + p;
#pragma unroll
        for (int j = 0; j < HD; ++j) o[j] = o[j] * corr + p * vr[j];
        m = mn;
    }
    // merge the 32 lanes' partial softmax states
    float mall = m;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mall = fmaxf(mall, __shfl_xor_sync(0xffffffffu, mall, off));
    const float f = (m == -INFINITY) ? 0.f : expf(m - mall);
    l *= f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    CT* orow = out + int64_t(r) * H * HD + h * HD;
#pragma unroll
    for (int j = 0; j < HD; ++j) {
        float v = o[j] * f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) orow[j] = from_f32<CT>(v / l);
    }
}

// gu fp32 [n, 2 I] ([gate | up] per row) -> ct [n, I] = silu(gate) * up.
template <typename CT>
__global__ void lm_swiglu_kernel(const float* __restrict__ gu, int64_t n, int I, CT* __restrict__ out) {
    const int64_t total = n * I;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / I;
        const int c = int(i % I);
        const float g = gu[r * 2 * I + c], u = gu[r * 2 * I + I + c];
        out[i] = from_f32<CT>(g / (1.0f + expf(-g)) * u);
    }
}

}  // namespace b2d
