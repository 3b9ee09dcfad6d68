// torch-CUDA-compatible normal generator on the device: Philox4x32-10 + Box-Muller, in the
// per-index form (generate_torch_cuda_randn) and the TensorIterator layout used for sampler
// noise (generate_torch_cuda_tensor_iterator_randn), restated from
// src/framework/sampling/torch_random.cpp:17-99, 131-143, 186-246, 379-399.
#pragma once

#include <cstdint>

namespace b2d {

struct Philox4 {
    uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ Philox4 philox4x32_10(Philox4 c, uint64_t seed) {
    uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = uint64_t(0xD2511F53u) * c.x;
        const uint64_t p1 = uint64_t(0xCD9E8D57u) * c.z;
        c = Philox4{uint32_t(p1 >> 32) ^ c.y ^ k0, uint32_t(p1), uint32_t(p0 >> 32) ^ c.w ^ k1, uint32_t(p0)};
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

// Box-Muller on two 32-bit uniforms: u in (0, 1) as torch maps them; returns (r sin a, r cos a).
__device__ __forceinline__ void box_muller(uint32_t u0, uint32_t u1, float& n0, float& n1) {
    const float inv = 2.3283064365386963e-10f, inv2pi = 1.4629180792671596e-09f;
    const float rin = float(u0) * inv + inv * 0.5f;
    const float ang = float(u1) * inv2pi + inv2pi * 0.5f;
    const float r = sqrtf(-2.0f * logf(rin));
    n0 = r * sinf(ang);
    n1 = r * cosf(ang);
}

__device__ __forceinline__ float round_to_bf16_value(float v) {
    uint32_t b = __float_as_uint(v);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return __uint_as_float(b & 0xFFFF0000u);
}

// Element `index` of generate_torch_cuda_randn(seed).
__device__ __forceinline__ float torch_randn_at(uint64_t seed, uint64_t index) {
    const Philox4 r = philox4x32_10(Philox4{0u, 0u, uint32_t(index), uint32_t(index >> 32)}, seed);
    float n0, n1;
    box_muller(r.x, r.y, n0, n1);
    return n0;
}

// Element `i` of generate_torch_cuda_tensor_iterator_randn(count, seed, offset_blocks, policy),
// stride = 256 * min(ceil(count / 256), SMs * max_threads / 256).
__device__ __forceinline__ float torch_iterator_randn_at(uint64_t seed, uint64_t offset_blocks, uint64_t stride,
                                                         uint64_t i) {
    const uint64_t q = i / stride;
    const uint64_t loop = q >> 2;
    const int comp = int(q & 3u);
    const uint64_t seq = i % stride;
    const uint64_t ctr = offset_blocks + loop;
    const Philox4 r = philox4x32_10(Philox4{uint32_t(ctr), uint32_t(ctr >> 32), uint32_t(seq), uint32_t(seq >> 32)},
                                    seed);
    float a, b;
    if (comp < 2)
        box_muller(r.x, r.y, a, b);
    else
        box_muller(r.z, r.w, a, b);
    return (comp & 1) ? b : a;
}

__host__ __device__ inline uint64_t torch_iterator_stride(uint64_t total, int64_t sms, int64_t max_threads) {
    uint64_t grid = (total + 255) / 256;
    uint64_t per_sm = uint64_t(max_threads) / 256;
    if (per_sm == 0) per_sm = 1;
    const uint64_t cap = uint64_t(sms) * per_sm;
    grid = grid < cap ? grid : cap;
    if (grid < 1) grid = 1;
    return 256 * grid;
}

__host__ __device__ inline uint64_t torch_iterator_offset_blocks(uint64_t total, int64_t sms, int64_t max_threads) {
    return (total - 1) / (torch_iterator_stride(total, sms, max_threads) * 4) + 1;
}

__global__ void torch_randn_kernel(int layout, uint64_t seed, uint64_t offset, uint64_t stride, int64_t count,
                                   int bf16, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x) {
        float v = layout == 0 ? torch_randn_at(seed, offset + uint64_t(i))
                              : torch_iterator_randn_at(seed, offset, stride, uint64_t(i));
        out[i] = bf16 ? round_to_bf16_value(v) : v;
    }
}

}  // namespace b2d
