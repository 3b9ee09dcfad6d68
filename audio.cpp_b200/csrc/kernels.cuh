// Memory-bound kernels of the diffusion hot path: weight dequantisation,
// fused RMSNorm + adaLN modulate, SiLU conditioning, the timestep-embedding
// MLP, and the fused CFG + DPM-Solver++ update.  All use 128-bit accesses
// along rows and warp-shuffle reductions; grids are sized to fill the SMs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "gemm.cuh"

namespace b2d {

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ weights
// Source encodings (ggml type ids): 0 = F32, 1 = F16, 8 = Q8_0, 30 = BF16.
// Row r of the source lands in destination row
//   dst_row(r) = (r / blk) * blk_stride + (r % blk) + row_offset
// which expresses plain copies (blk = rows) and the block interleaving used to
// pair SwiGLU halves inside one GEMM tile.
struct RowMap {
    int64_t blk;
    int64_t blk_stride;
    int64_t row_offset;
    __device__ __forceinline__ int64_t operator()(int64_t r) const { return (r / blk) * blk_stride + (r % blk) + row_offset; }
};

// Q8_0 block = fp16 scale d + 32 int8 quants (external/ggml/src/ggml-common.h:241-246).
// value = q * fp32(d) exactly as dequantize_row_q8_0 (ggml-quants.c:491-505), then one
// rounding to the GEMM operand type.
template <typename OutT>
__global__ void dequant_q8_0_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t k, OutT* __restrict__ dst,
                                    int64_t ldd, RowMap map) {
    const int64_t nblk_row = k / 32;
    const int64_t total = rows * nblk_row;
    for (int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; b < total; b += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = b / nblk_row, kb = b % nblk_row;
        const uint8_t* blk = src + b * 34;
        const uint16_t dbits = uint16_t(blk[0]) | (uint16_t(blk[1]) << 8);
        const float d = __half2float(__ushort_as_half(dbits));
        OutT* o = dst + map(r) * ldd + kb * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = from_f32<OutT>(float(int8_t(blk[2 + j])) * d);
    }
}

// Q8_0 blocks of a [rows, k] weight -> the k-block-major planar form the weight-streaming GEMM reads:
// quants q[k/64][n_total][64] (int8) and scales d[k/64][n_total][2] (the fp16 scale bits of the two 32-blocks),
// destination row map(r).  A lossless rearrangement of the checkpoint's bytes.
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t k, int8_t* __restrict__ q,
                                   __half* __restrict__ d, int64_t n_total, RowMap map) {
    const int64_t nblk_row = k / 32;
    const int64_t total = rows * nblk_row;
    for (int64_t b = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; b < total; b += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = b / nblk_row, kb = b % nblk_row;
        const uint8_t* blk = src + b * 34;
        const int64_t n = map(r), k64 = kb / 2, half = kb % 2;
        d[(k64 * n_total + n) * 2 + half] = __ushort_as_half(uint16_t(blk[0]) | (uint16_t(blk[1]) << 8));
        int8_t* o = q + (k64 * n_total + n) * 64 + half * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = int8_t(blk[2 + j]);
    }
}

template <typename InT, typename OutT>
__global__ void convert_rows_kernel(const InT* __restrict__ src, int64_t rows, int64_t k, OutT* __restrict__ dst,
                                    int64_t ldd, RowMap map) {
    const int64_t total = rows * k;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / k, c = i % k;
        dst[map(r) * ldd + c] = from_f32<OutT>(to_f32(src[i]));
    }
}

__global__ void bf16_bits_to_f32_kernel(const uint16_t* __restrict__ src, int64_t n, float* __restrict__ dst) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = __uint_as_float(uint32_t(src[i]) << 16);
}

// ------------------------------------------------- RMSNorm + adaLN modulate
// h = ct( (x / sqrt(mean(x^2) + eps)) * w * (1 + scale) + shift )   per row
// (RMSNormModule + modulate: src/models/vibevoice/diffusion_head.cpp:130-139,183-220)
// One CTA per row; x, shift, scale are fp32 rows read with float4.
template <typename CT, int THREADS>
__global__ void __launch_bounds__(THREADS) rms_modulate_kernel(const float* __restrict__ x, int64_t ldx,
                                                               const float* __restrict__ w, const float* __restrict__ shift,
                                                               const float* __restrict__ scale, int64_t ldm, float eps,
                                                               int H, CT* __restrict__ out, int64_t ldo) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x + row * ldx);
    const int n4 = H / 4;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n4; i += THREADS) {
        const float4 v = x4[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    __shared__ float red[THREADS / 32];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < THREADS / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / float(H) + eps);
    const float4* s4 = reinterpret_cast<const float4*>(shift + row * ldm);
    const float4* c4 = reinterpret_cast<const float4*>(scale + row * ldm);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int i = threadIdx.x; i < n4; i += THREADS) {
        float4 v = x4[i];
        const float4 sh = s4[i], sc = c4[i];
        const float4 ww = w ? w4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        const float a = v.x * inv * ww.x * (1.f + sc.x) + sh.x;
        const float b = v.y * inv * ww.y * (1.f + sc.y) + sh.y;
        const float c = v.z * inv * ww.z * (1.f + sc.z) + sh.z;
        const float d = v.w * inv * ww.w * (1.f + sc.w) + sh.w;
        uint2 p = make_uint2(CtTraits<CT>::pack2(a, b), CtTraits<CT>::pack2(c, d));
        reinterpret_cast<uint2*>(out + row * ldo)[i] = p;
    }
}

// Block-wide sum over blockDim.x (a multiple of 32, at most 1024) threads; every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();  // red may still be read by a previous reduction
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = (threadIdx.x & 31) < nw ? red[threadIdx.x & 31] : 0.f;
    return warp_sum(t);
}

// Same computation, one CTA per row with 8 values per thread (blockDim = H / 8): every operand of the row --
// x, shift, scale and the norm weight -- is requested before the reduction, so a row costs one memory
// latency, and a few thousand rows keep every SM busy.
template <typename CT>
__global__ void __launch_bounds__(1024) rms_modulate_row_kernel(const float* __restrict__ x, int64_t ldx,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ shift,
                                                                const float* __restrict__ scale, int64_t ldm,
                                                                float eps, int H, CT* __restrict__ out, int64_t ldo) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int i0 = threadIdx.x * 2;  // float4 index
    const float4* x4 = reinterpret_cast<const float4*>(x + row * ldx) + i0;
    const float4* s4 = reinterpret_cast<const float4*>(shift + row * ldm) + i0;
    const float4* c4 = reinterpret_cast<const float4*>(scale + row * ldm) + i0;
    const float4 v0 = x4[0], v1 = x4[1];
    const float4 sh0 = s4[0], sh1 = s4[1], sc0 = c4[0], sc1 = c4[1];
    float4 w0 = make_float4(1.f, 1.f, 1.f, 1.f), w1 = w0;
    if (w) {
        w0 = __ldg(reinterpret_cast<const float4*>(w) + i0);
        w1 = __ldg(reinterpret_cast<const float4*>(w) + i0 + 1);
    }
    const float ss = v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w + v1.x * v1.x + v1.y * v1.y +
                     v1.z * v1.z + v1.w * v1.w;
    const float inv = 1.0f / sqrtf(block_sum(ss, red) / float(H) + eps);
    uint4 o;
    o.x = CtTraits<CT>::pack2(v0.x * inv * w0.x * (1.f + sc0.x) + sh0.x, v0.y * inv * w0.y * (1.f + sc0.y) + sh0.y);
    o.y = CtTraits<CT>::pack2(v0.z * inv * w0.z * (1.f + sc0.z) + sh0.z, v0.w * inv * w0.w * (1.f + sc0.w) + sh0.w);
    o.z = CtTraits<CT>::pack2(v1.x * inv * w1.x * (1.f + sc1.x) + sh1.x, v1.y * inv * w1.y * (1.f + sc1.y) + sh1.y);
    o.w = CtTraits<CT>::pack2(v1.z * inv * w1.z * (1.f + sc1.z) + sh1.z, v1.w * inv * w1.w * (1.f + sc1.w) + sh1.w);
    reinterpret_cast<uint4*>(out + row * ldo)[threadIdx.x] = o;
}

// Same computation, one warp per row with the row held in registers (x read once, reductions by
// shuffles only): rows of H <= 128 * MAXV floats; 8 rows per 256-thread CTA.
template <typename CT, int MAXV>
__global__ void __launch_bounds__(256) rms_modulate_warp_kernel(const float* __restrict__ x, int64_t ldx,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ shift,
                                                                const float* __restrict__ scale, int64_t ldm, float eps,
                                                                int H, int64_t rows, CT* __restrict__ out, int64_t ldo) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int n4 = H / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x + row * ldx);
    float4 v[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        v[i] = idx < n4 ? x4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    const float inv = 1.0f / sqrtf(warp_sum(ss) / float(H) + eps);
    const float4* s4 = reinterpret_cast<const float4*>(shift + row * ldm);
    const float4* c4 = reinterpret_cast<const float4*>(scale + row * ldm);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    uint2* o2 = reinterpret_cast<uint2*>(out + row * ldo);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        if (idx < n4) {
            const float4 sh = s4[idx], sc = c4[idx];
            const float4 ww = w ? __ldg(w4 + idx) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float a = v[i].x * inv * ww.x * (1.f + sc.x) + sh.x;
            const float b = v[i].y * inv * ww.y * (1.f + sc.y) + sh.y;
            const float c = v[i].z * inv * ww.z * (1.f + sc.z) + sh.z;
            const float d = v[i].w * inv * ww.w * (1.f + sc.w) + sh.w;
            o2[idx] = make_uint2(CtTraits<CT>::pack2(a, b), CtTraits<CT>::pack2(c, d));
        }
    }
}

// sc[r, :] = ct(silu(cp[r, :] + temb[:]))   (SiluModule on c = cond_proj + t_emb)
template <typename CT>
__global__ void silu_cond_kernel(const float* __restrict__ cp, const float* __restrict__ temb, int64_t rows, int H,
                                 CT* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t n4 = rows * H / 4;
    const int h4 = H / 4;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        const float4 c = reinterpret_cast<const float4*>(cp)[i];
        const float4 t = reinterpret_cast<const float4*>(temb)[i % h4];
        const float a = c.x + t.x, b = c.y + t.y, d = c.z + t.z, e = c.w + t.w;
        reinterpret_cast<uint2*>(out)[i] =
            make_uint2(CtTraits<CT>::pack2(silu_f(a), silu_f(b)), CtTraits<CT>::pack2(silu_f(d), silu_f(e)));
    }
}

// ------------------------------------------------ timestep embedding input
// feat_s = [cos(t_s f_i) | sin(t_s f_i)], f_i = exp(-ln(1e4) i / 128), i < 128
// (make_timestep_freqs + build_timestep_embedding, diffusion_head.cpp:59-66,141-163).
// One block of 128 threads per timestep row; the MLP runs on the tensor-core GEMM.
constexpr int kMaxTembSteps = 32;

template <typename CT>
__global__ void temb_feat_kernel(const float* __restrict__ tsteps, CT* __restrict__ feat) {
    const int s = blockIdx.x, j = threadIdx.x;
    const float f = expf(-logf(10000.0f) * float(j) / 128.0f);
    const float a = tsteps[s] * f;
    feat[s * 256 + j] = from_f32<CT>(cosf(a));
    feat[s * 256 + 128 + j] = from_f32<CT>(sinf(a));
}

template <typename CT>
__global__ void silu_to_ct_kernel(const float* __restrict__ src, int64_t n, CT* __restrict__ dst) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = from_f32<CT>(silu_f(src[i]));
}

// out[i] = sum over split-K partials part[s * n + i] (fixed order: deterministic).
__global__ void sum_partials_kernel(const float* __restrict__ part, int splits, int64_t n, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < splits; ++s) v += part[s * n + i];
        out[i] = v;
    }
}

// --------------------------------------------- CFG + DPM-Solver++(2M) step
// Per-step scalars, computed on the host in fp32 exactly as
// VibeVoiceDPMSolverScheduler::step (src/models/vibevoice/scheduler.cpp:165-274).
struct VvStepCoef {
    float alpha_s;       // convert_model_output: x0 = alpha_s * x - sigma_s * eps
    float sigma_s;
    float sample_coeff;  // sigma_t / sigma_s0
    float d0_coeff;      // -alpha_t * (exp(-h) - 1)
    float inv_r0;        // 1 / r0 (second order only)
    int order;           // 1 or 2
    int last;            // 1 on the final step (write latents out)
    int pad;
};

// v: head output [2B, 64] (cond rows then uncond rows) as `splits` split-K partials
// spaced `split_stride` apart, summed here in a fixed order.  x: sampler state [B, 64].
// hist_prev / hist_cur: converted outputs of the previous / this step [B, 64].
// noisy: next head input [2B, 64] in ct, both halves = x (duplicate_positive_half).
template <typename CT>
__global__ void vv_cfg_dpm_kernel(const float* __restrict__ v, int splits, int64_t split_stride, float* __restrict__ x, const float* __restrict__ hist_prev,
                                  float* __restrict__ hist_cur, CT* __restrict__ noisy, float* __restrict__ out_latents,
                                  int64_t n_half, const VvStepCoef* __restrict__ coefs, int step, float cfg,
                                  int* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const VvStepCoef c = coefs[step];
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n_half; i += int64_t(gridDim.x) * blockDim.x) {
        float vc = 0.f, vu = 0.f;
        for (int s = 0; s < splits; ++s) {
            vc += v[s * split_stride + i];
            vu += v[s * split_stride + n_half + i];
        }
        const float g = vu + cfg * (vc - vu);            // apply_cfg, diffusion_sampler.cpp:35-56
        const float xs = x[i];
        const float conv = c.alpha_s * xs - c.sigma_s * g;  // convert_model_output
        float nx;
        if (c.order == 1) {
            nx = c.sample_coeff * xs + c.d0_coeff * conv;  // first_order_update
        } else {
            const float d1 = c.inv_r0 * (conv - hist_prev[i]);  // second_order_update
            nx = c.sample_coeff * xs + c.d0_coeff * conv + 0.5f * c.d0_coeff * d1;
        }
        hist_cur[i] = conv;
        x[i] = nx;
        if (!isfinite(nx)) atomicCAS(status, 0, kErrNonFinite);
        if (c.last) {
            out_latents[i] = nx;
        } else {
            const CT h = from_f32<CT>(nx);
            noisy[i] = h;
            noisy[n_half + i] = h;
        }
    }
}

// Step 0 set-up: x = initial_speech[:B]; noisy = [x; x] in ct.
template <typename CT>
__global__ void vv_init_kernel(const float* __restrict__ init, float* __restrict__ x, CT* __restrict__ noisy, int64_t n_half) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n_half; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = init[i];
        x[i] = v;
        const CT h = from_f32<CT>(v);
        noisy[i] = h;
        noisy[n_half + i] = h;
    }
}

template <typename CT>
__global__ void f32_to_ct_kernel(const float* __restrict__ src, int64_t n, CT* __restrict__ dst) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        dst[i] = from_f32<CT>(src[i]);
}

}  // namespace b2d
