// Memory-bound kernels of the Stable Audio 3 rectified-flow DiT step
// (src/models/stable_audio/rf_dit.cpp): per-head q/k RMSNorm + partial NEOX RoPE, the 6-way
// adaLN table, RMSNorm + modulation (with the local-add residual folded in), memory-token rows,
// differential-attention subtraction, and the fused APG-CFG + pingpong / euler update.
#pragma once

#include "dit_kernels.cuh"

namespace b2d {

constexpr int kSa3Io = 64;

// Fourier timestep features: arg = sigma * freq_i (freq_i already carries the 2 pi factor),
// feat = [cos(arg) | sin(arg)]   (make_fourier_freqs / timestep features, rf_dit.cpp:158-182).
template <typename CT>
__global__ void sa3_tfeat_kernel(const float* __restrict__ sig, const float* __restrict__ freqs, CT* __restrict__ feat) {
    const int s = blockIdx.x, i = threadIdx.x;  // 128 threads
    const float arg = sig[s] * freqs[i];
    feat[s * 256 + i] = from_f32<CT>(cosf(arg));
    feat[s * 256 + 128 + i] = from_f32<CT>(sinf(arg));
}

// g[s, bb] = global_embed[bb] + timestep_embed[s, bb % B]   (rf_dit.cpp:800-806), for every step.
template <typename CT>
__global__ void sa3_gsum_kernel(const float* __restrict__ gpre, const float* __restrict__ temb, int S, int B, int Bg,
                                int d, CT* __restrict__ out) {
    const int64_t total = int64_t(S) * Bg * d;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int j = int(i % d);
        const int64_t sb = i / d;
        const int s = int(sb / Bg), bb = int(sb % Bg);
        out[i] = from_f32<CT>(gpre[int64_t(bb) * d + j] + temb[(int64_t(s) * B + bb % B) * d + j]);
    }
}

// adaLN table of one step for every layer: ada = global_six + to_scale_shift_gate, stored as
// mod[l][bb][slot][d] with slots (1 + scale_self, shift_self, sigmoid(1 - gate_self),
// 1 + scale_ff, shift_ff, sigmoid(1 - gate_ff))   (build_rf_layer, rf_dit.cpp:343-387).
__global__ void sa3_ada_kernel(const float* __restrict__ six, const float* __restrict__ ssg, int depth, int Bg, int d,
                               float* __restrict__ mod) {
    const int64_t per_layer = int64_t(Bg) * 6 * d;
    const int64_t total = int64_t(depth) * per_layer;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int l = int(i / per_layer);
        const int64_t r = i % per_layer;  // bb * 6d + slot * d + j
        const int slot = int((r / d) % 6);
        const float a = six[r] + ssg[int64_t(l) * 6 * d + r % (6 * int64_t(d))];
        float v;
        if (slot == 0 || slot == 3)
            v = 1.0f + a;
        else if (slot == 2 || slot == 5)
            v = 1.0f / (1.0f + expf(-(1.0f - a)));
        else
            v = a;
        mod[i] = v;
    }
}

// Memory-token rows of every sequence: h[bb * L1 + m] = memory_tokens[m]   (rf_dit.cpp:779-781).
__global__ void sa3_memrows_kernel(float* __restrict__ h, const float* __restrict__ mem, int Bg, int L1, int M, int d) {
    const int64_t total = int64_t(Bg) * M * d;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int j = int(i % d);
        const int m = int((i / d) % M);
        const int bb = int(i / (int64_t(M) * d));
        h[(int64_t(bb) * L1 + m) * d + j] = mem[int64_t(m) * d + j];
    }
}

// RMSNorm over d (multiple of 128, <= 32 * 4 * NV4) with gamma, then optional modulation:
//   y = ct(x / sqrt(mean(x^2) + eps) * gamma * mod[0:d] + mod[d:2d])   (mod per sequence: row / L1)
// When loc is given, the token rows (row % L1 >= M) first take h += loc[(bb % B) * T + t - M] and write
// h back (the local-add residual, build_local_embedding rf_dit.cpp:327-341).  One warp per row.
template <typename CT, int NV4>
__global__ void __launch_bounds__(256) sa3_rms_mod_kernel(float* __restrict__ h, int d, int64_t rows, int L1, int M,
                                                          const float* __restrict__ loc, int T, int B,
                                                          const float* __restrict__ gamma, const float* __restrict__ mod,
                                                          int64_t mod_seq_stride, float eps, CT* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * 8 + warp;
    if (row >= rows) return;
    const int nv = d >> 7;  // float4 per lane
    float4* hr = reinterpret_cast<float4*>(h + row * d);
    const int bb = int(row / L1), t = int(row % L1);
    const float4* lr = (loc && t >= M) ? reinterpret_cast<const float4*>(loc + (int64_t(bb % B) * T + t - M) * d) : nullptr;
    float4 v[NV4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        if (i < nv) {
            float4 a = hr[i * 32 + lane];
            if (lr) {
                const float4 b = lr[i * 32 + lane];
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
                hr[i * 32 + lane] = a;
            }
            v[i] = a;
            ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float sc = 1.0f / sqrtf(ss / float(d) + eps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* m4 = mod ? reinterpret_cast<const float4*>(mod + int64_t(bb) * mod_seq_stride) : nullptr;
    CT* o = out + row * d;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
        if (i < nv) {
            const int q = i * 32 + lane;
            const float4 g = __ldg(g4 + q);
            float y0 = v[i].x * sc * g.x, y1 = v[i].y * sc * g.y, y2 = v[i].z * sc * g.z, y3 = v[i].w * sc * g.w;
            if (m4) {
                const float4 s = __ldg(m4 + q), b = __ldg(m4 + (d >> 2) + q);
                y0 = y0 * s.x + b.x;
                y1 = y1 * s.y + b.y;
                y2 = y2 * s.z + b.z;
                y3 = y3 * s.w + b.w;
            }
            *reinterpret_cast<uint2*>(o + 4 * q) =
                make_uint2(CtTraits<CT>::pack2(y0, y1), CtTraits<CT>::pack2(y2, y3));
        }
    }
}

// Column slots of a fused projection (each d = heads x 64 wide): kind 0 = copy (x vmask[row] when
// given), 1 = per-head RMSNorm with gamma_q, 2 = per-head RMSNorm with gamma_k.
struct Sa3Slots {
    int n;
    int kind[5];
};

// fp32 projection [rows, n * d] -> ct [rows, n * d]: per-head RMSNorm (eps 1e-6) over the 64 head
// dims, then NEOX RoPE on dims [0, 32) (pairs j, j + 16; position = row % L1) when tables are given
// (self_attention rf_dit.cpp:217-262, cross_attention :264-310 without RoPE).  One warp per head.
template <typename CT>
__global__ void __launch_bounds__(256) sa3_qknorm_kernel(const float* __restrict__ in, CT* __restrict__ out,
                                                         int64_t rows, int heads, Sa3Slots slots,
                                                         const float* __restrict__ gq, const float* __restrict__ gk,
                                                         const float* __restrict__ rope_cos,
                                                         const float* __restrict__ rope_sin, int L1,
                                                         const float* __restrict__ vmask) {
    const int lane = threadIdx.x & 31;
    const int64_t units = rows * slots.n * heads;
    const int64_t ld = int64_t(slots.n) * heads * 64;
    for (int64_t u = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < units;
         u += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        const int hd = int(u % heads);
        const int slot = int((u / heads) % slots.n);
        const int64_t row = u / (int64_t(heads) * slots.n);
        const int64_t base = row * ld + int64_t(slot) * heads * 64 + hd * 64;
        float a = in[base + lane], b = in[base + 32 + lane];
        const int kind = slots.kind[slot];
        if (kind == 0) {
            if (vmask) {
                const float m = __ldg(vmask + row);
                a *= m;
                b *= m;
            }
        } else {
            float ss = a * a + b * b;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float sc = 1.0f / sqrtf(ss / 64.0f + 1e-6f);
            const float* g = kind == 1 ? gq : gk;
            a = a * sc * __ldg(g + lane);
            b = b * sc * __ldg(g + 32 + lane);
            if (rope_cos) {
                const int pos = int(row % L1), j = lane & 15;
                const float c = __ldg(rope_cos + pos * 16 + j), s = __ldg(rope_sin + pos * 16 + j);
                const float p = __shfl_xor_sync(0xffffffffu, a, 16);
                a = lane < 16 ? a * c - p * s : p * s + a * c;
            }
        }
        out[base + lane] = from_f32<CT>(a);
        out[base + 32 + lane] = from_f32<CT>(b);
    }
}

// Per hidden row V factor: 1 on the memory tokens, the latent mask on the token rows
// (make_padding_mask, rf_dit.cpp:948-963).
__global__ void dit_padrow_mem_kernel(const float* __restrict__ mask, int B, int Bg, int T, int M,
                                      float* __restrict__ padrow) {
    const int L1 = M + T;
    const int64_t total = int64_t(Bg) * L1;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int bb = int(i / L1), t = int(i % L1);
        padrow[i] = t < M ? 1.0f : mask[int64_t(bb % B) * T + t - M];
    }
}

// Differential attention: a = ct(a - b)   (context - diff_context, rf_dit.cpp:246-262, 277-300).
template <typename CT>
__global__ void sa3_sub_kernel(CT* __restrict__ a, const CT* __restrict__ b, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        a[i] = from_f32<CT>(to_f32(a[i]) - to_f32(b[i]));
}

// Local-add features [B * T, la] fp32 -> ct [B * T, kp] zero-padded to the GEMM K granule.
template <typename CT>
__global__ void sa3_pad_cols_kernel(const float* __restrict__ src, int64_t rows, int la, int kp, CT* __restrict__ dst) {
    const int64_t total = rows * kp;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % kp);
        const int64_t r = i / kp;
        dst[i] = from_f32<CT>(c < la ? src[r * la + c] : 0.0f);
    }
}

// Unconditional prompt rows: keep the negative prompt's masked-in tokens, zero the rest
// (make_cross_conditioning, rf_dit.cpp:891-914).  rows = B * tokens.
__global__ void sa3_neg_mask_kernel(float* __restrict__ cross_neg, const float* __restrict__ nmask, int64_t rows,
                                    int cd) {
    const int64_t total = rows * cd;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x)
        if (nmask[i / cd] == 0.0f) cross_neg[i] = 0.0f;
}

// Latent [B, 64, T] (BCT) -> graph input [Bg * T, 64] (write_latent_input, rf_dit.cpp:967-978).
template <typename CT>
__global__ void sa3_step_input_kernel(const float* __restrict__ x, int B, int Bg, int T, CT* __restrict__ X) {
    const int64_t total = int64_t(Bg) * T * kSa3Io;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % kSa3Io);
        const int t = int((i / kSa3Io) % T);
        const int bb = int(i / (int64_t(T) * kSa3Io));
        X[i] = from_f32<CT>(x[(int64_t(bb % B) * kSa3Io + c) * T + t]);
    }
}

// Per-step sampler scalars (StableAudioRfDitRuntime::sample, rf_dit.cpp:586-694).
struct Sa3StepCoef {
    float cfg_scale, apg_scale;
    int sampler;     // 0 pingpong, 1 euler
    int final_step;
    unsigned long long seed, rng_offset, rng_stride;  // pingpong noise: TensorIterator Philox stream
    unsigned long long rng_elem0;                      // first element of this request within the batched draw
};
struct Sa3BatchCoef {
    float sigma, next_sigma, dt;  // next_sigma = sigma + dt, dt = schedule[s + 1] - schedule[s] (fp32)
    float pad;
};

// Raw model output of sequence bb, latent token t, channel c (rows bb * L1 + M + t; split-K partials summed).
__device__ __forceinline__ float sa3_raw(const float* __restrict__ part, int splits, int64_t split_stride, int bb,
                                         int L1, int M, int t, int c) {
    const int64_t idx = (int64_t(bb) * L1 + M + t) * kSa3Io + c;
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += part[s * split_stride + idx];
    return v;
}

// APG reductions per prompt b on x0 = x - sigma v: s1 = sum (x0_c m)^2, s2 = sum (x0_c - x0_u)(x0_c m)
// (build_cfg_model_output, rf_dit.cpp:834-873); finished by dit_apg_finish_kernel.
__global__ void __launch_bounds__(256) sa3_apg_partial_kernel(const float* __restrict__ part, int splits,
                                                              int64_t split_stride, const float* __restrict__ x,
                                                              const float* __restrict__ mask, int B, int T, int L1,
                                                              int M, const Sa3BatchCoef* __restrict__ bcoefs, int step,
                                                              double* __restrict__ partials) {
    const int b = blockIdx.y, chunk = blockIdx.x;
    const float sg = bcoefs[int64_t(step) * B + b].sigma;
    const int n = T * kSa3Io;
    const int per = (n + kApgChunks - 1) / kApgChunks;
    const int i0 = chunk * per, i1 = min(n, i0 + per);
    double s1 = 0.0, s2 = 0.0;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const int t = i / kSa3Io, c = i % kSa3Io;
        const float xv = x[(int64_t(b) * kSa3Io + c) * T + t];
        const float cx0 = xv - sa3_raw(part, splits, split_stride, b, L1, M, t, c) * sg;
        const float ux0 = xv - sa3_raw(part, splits, split_stride, b + B, L1, M, t, c) * sg;
        const float cm = cx0 * mask[int64_t(b) * T + t];
        s1 += double(cm) * cm;
        s2 += double(cx0 - ux0) * cm;
    }
    __shared__ double r1[8], r2[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if ((threadIdx.x & 31) == 0) {
        r1[threadIdx.x >> 5] = s1;
        r2[threadIdx.x >> 5] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0.0, c = 0.0;
        for (int w = 0; w < 8; ++w) {
            a += r1[w];
            c += r2[w];
        }
        partials[(int64_t(b) * kApgChunks + chunk) * 2] = a;
        partials[(int64_t(b) * kApgChunks + chunk) * 2 + 1] = c;
    }
}

// Fused APG-CFG combine (or the raw output) and the sampler update of latent [B, 64, T]:
//   pingpong: x = (1 - next) (x - sigma v) + next * randn (TensorIterator Philox, this step's offset)
//   euler:    x = x + dt v
// then the next step's graph input, or the result on the final step; non-finite outputs set status.
template <typename CT>
__global__ void sa3_update_kernel(const float* __restrict__ part, int splits, int64_t split_stride,
                                  float* __restrict__ x, const float* __restrict__ mask, const float* __restrict__ sums,
                                  int B, int Bg, int T, int L1, int M, int use_cfg,
                                  const Sa3StepCoef* __restrict__ coefs, const Sa3BatchCoef* __restrict__ bcoefs,
                                  int step, CT* __restrict__ Xnext, float* __restrict__ out, int* __restrict__ status) {
    const Sa3StepCoef k = coefs[step];
    const int64_t total = int64_t(B) * kSa3Io * T;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int t = int(i % T);
        const int c = int((i / T) % kSa3Io);
        const int b = int(i / (int64_t(T) * kSa3Io));
        const Sa3BatchCoef kb = bcoefs[int64_t(step) * B + b];
        const float xv = x[i];
        float v;
        if (use_cfg) {
            const float cx0 = xv - sa3_raw(part, splits, split_stride, b, L1, M, t, c) * kb.sigma;
            const float ux0 = xv - sa3_raw(part, splits, split_stride, b + B, L1, M, t, c) * kb.sigma;
            const float diff = cx0 - ux0;
            const float m = mask[int64_t(b) * T + t];
            const float n = sums[2 * b], dot = sums[2 * b + 1];
            const float v1 = (cx0 * m) / n;
            const float orth = (diff - dot * v1) * m;
            const float cd = k.apg_scale * orth + (1.0f - k.apg_scale) * diff;
            const float den = cx0 + (k.cfg_scale - 1.0f) * cd;
            v = (xv - den) / kb.sigma;
        } else {
            v = sa3_raw(part, splits, split_stride, b, L1, M, t, c);
        }
        float nx;
        if (k.sampler == 0) {
            const float den = xv - kb.sigma * v;
            nx = (1.0f - kb.next_sigma) * den +
                 kb.next_sigma * torch_iterator_randn_at(k.seed, k.rng_offset, k.rng_stride, uint64_t(i) + k.rng_elem0);
        } else {
            nx = xv + kb.dt * v;
        }
        if (!isfinite(v) || !isfinite(nx)) atomicCAS(status, 0, kErrNonFinite);
        x[i] = nx;
        if (k.final_step) {
            out[i] = nx;
        } else {
            const CT hv = from_f32<CT>(nx);
            for (int bb = b; bb < Bg; bb += B) Xnext[(int64_t(bb) * T + t) * kSa3Io + c] = hv;
        }
    }
}

}  // namespace b2d
