// Memory-bound kernels of the Stable Audio Open 1.0 DiT step
// (src/models/stable_audio/foundation/rf_dit.cpp): LayerNorm, partial NEOX RoPE
// with the V padding mask, the global-token row, the sampler's input transpose,
// and the fused CFG/APG + DPM++ 2M update with its per-sequence reductions.
#pragma once

#include "kernels.cuh"
#include "philox.cuh"

namespace b2d {

// LayerNorm over d (<= 4096): y = ct((x - mean) / sqrt(var + eps) * gamma + beta)
// (ggml_norm + affine, src/framework/modules/norm_modules.cpp:200-228).  One CTA (128 thr) per row.
template <typename CT>
__global__ void __launch_bounds__(128) layernorm_kernel(const float* __restrict__ x, int d, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps, CT* __restrict__ out) {
    constexpr int MAXV = 8;
    const int64_t row = blockIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x + row * d);
    const int n4 = d / 4;
    float4 v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = threadIdx.x + i * 128;
        v[i] = idx < n4 ? x4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    __shared__ float red[4];
    __shared__ float bc;
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) bc = (red[0] + red[1] + red[2] + red[3]) / float(d);
    __syncthreads();
    const float mean = bc;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = threadIdx.x + i * 128;
        if (idx < n4) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
            q += a * a + b * b + c * c + e * e;
        }
    }
    q = warp_sum(q);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = q;
    __syncthreads();
    if (threadIdx.x == 0) bc = (red[0] + red[1] + red[2] + red[3]) / float(d);
    __syncthreads();
    const float rstd = 1.0f / sqrtf(bc + eps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = threadIdx.x + i * 128;
        if (idx < n4) {
            const float4 gg = g4[idx], bb = b4[idx];
            const float a = (v[i].x - mean) * rstd * gg.x + bb.x;
            const float b = (v[i].y - mean) * rstd * gg.y + bb.y;
            const float c = (v[i].z - mean) * rstd * gg.z + bb.z;
            const float e = (v[i].w - mean) * rstd * gg.w + bb.w;
            reinterpret_cast<uint2*>(out + row * d)[idx] =
                make_uint2(CtTraits<CT>::pack2(a, b), CtTraits<CT>::pack2(c, e));
        }
    }
}

// Same LayerNorm, one warp per row with the row in registers and shuffle-only reductions
// (d <= 128 * MAXV); 8 rows per 256-thread CTA.
template <typename CT, int MAXV>
__global__ void __launch_bounds__(256) layernorm_warp_kernel(const float* __restrict__ x, int d, int64_t rows,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ beta, float eps,
                                                             CT* __restrict__ out) {
    const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int n4 = d / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x + row * d);
    float4 v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        v[i] = idx < n4 ? x4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    const float mean = warp_sum(s) / float(d);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        if (lane + 32 * i < n4) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
            q += a * a + b * b + c * c + e * e;
        }
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / float(d) + eps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
    uint2* o2 = reinterpret_cast<uint2*>(out + row * d);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + 32 * i;
        if (idx < n4) {
            const float4 gg = __ldg(g4 + idx), bb = __ldg(b4 + idx);
            const float a = (v[i].x - mean) * rstd * gg.x + bb.x;
            const float b = (v[i].y - mean) * rstd * gg.y + bb.y;
            const float c = (v[i].z - mean) * rstd * gg.z + bb.z;
            const float e = (v[i].w - mean) * rstd * gg.w + bb.w;
            o2[idx] = make_uint2(CtTraits<CT>::pack2(a, b), CtTraits<CT>::pack2(c, e));
        }
    }
}

// Global-token rows: h[seq, 0, :] = gpre[seq, :] + temb[step, seq % B, :]   (rf_dit.cpp:545-552);
// temb holds one row per (step, prompt) since v-DDIM gives every prompt its own timestep.
__global__ void dit_global_row_kernel(float* __restrict__ h, int64_t seq_rows, const float* __restrict__ gpre,
                                      const float* __restrict__ temb_step, int B, int d, int nseq) {
    const int64_t total = int64_t(nseq) * d;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t s = i / d, c = i % d;
        h[s * seq_rows * d + c] = gpre[i] + temb_step[(s % B) * d + c];
    }
}

// Timestep features for every sampler step: [cos(2 pi t w_i) | sin(2 pi t w_i)], learned w (rf_dit.cpp:939-950).
template <typename CT>
__global__ void dit_tfeat_kernel(const float* __restrict__ tvals, const float* __restrict__ w, CT* __restrict__ feat) {
    const int s = blockIdx.x, i = threadIdx.x;  // 128 threads
    const float arg = tvals[s] * w[i] * 2.0f * 3.14159265358979323846f;
    feat[s * 256 + i] = from_f32<CT>(cosf(arg));
    feat[s * 256 + 128 + i] = from_f32<CT>(sinf(arg));
}

// Per-step sampler scalars, computed on the host in fp32 exactly as the reference's samplers
// (Graph::sample_dpmpp_2m :798-883, sample_dpmpp_3m_sde :680-796, sample_v_ddim :514-604 of
// src/models/stable_audio/foundation/rf_dit.cpp).
enum DitSamplerMode : int { kDpmpp2m = 0, kDpmpp3mSde = 1, kVDdim = 2 };

struct DitStepCoef {
    float c_in, c_skip, c_out;   // denoiser scalings (v-DDIM: c_in = 1, c_skip/c_out unused)
    float x_scale, d_scale;      // 2M: sigma_next/sigma, -expm1(-h); 3M: exp(-2h), -expm1(-2h)
    float d_coeff, old_coeff;    // 2M second-order blend
    float c_in_next;             // next step's input scale
    float cfg_scale, apg_scale;
    float sig;                   // sigma of this step (sigma_0 scales the initial noise; v-DDIM: 1)
    float phi2, phi3, r0, r1;    // 3M history corrections
    float noise_scale;           // 3M: sigma_next * sqrt(-expm1(-2h))
    int mode;                    // DitSamplerMode
    int final_step;              // last step: x = denoised (2M/3M) or pred (v-DDIM)
    int first_step;
    int hist;                    // 3M: previous denoised outputs available (0, 1, 2)
    unsigned long long seed, rng_offset, rng_stride;  // 3M noise: TensorIterator Philox stream of this step
    unsigned long long rng_elem0;                      // first element of this request within the batched draw
};

// Per (step, prompt): alpha / sigma = cos / sin(t pi / 2) of this and the next timestep.
struct DitBatchCoef {
    float alpha, sigma, alpha_next, sigma_next;
};

// Step input: X[bb, t, c] = ct(x[b, c, t] * c_in), bb over the (CFG-doubled) graph batch.
template <typename CT>
__global__ void dit_step_input_kernel(const float* __restrict__ x, int B, int Bg, int T,
                                      const DitStepCoef* __restrict__ coefs, CT* __restrict__ X) {
    const float c_in = coefs[0].c_in;
    const int64_t total = int64_t(Bg) * T * 64;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % 64);
        const int64_t r = i / 64;
        const int t = int(r % T);
        const int bb = int(r / T);
        X[i] = from_f32<CT>(x[(int64_t(bb % B) * 64 + c) * T + t] * c_in);
    }
}

// raw model output y[bb, t, c] = sum of split-K partials at hidden row bb*(T+1) + t + 1.
__device__ __forceinline__ float dit_raw(const float* part, int splits, int64_t split_stride, int bb, int T, int t,
                                         int c) {
    const int64_t idx = (int64_t(bb) * (T + 1) + t + 1) * 64 + c;
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += part[s * split_stride + idx];
    return v;
}

// APG reductions per prompt b: s1 = sum (x0_c * m)^2, s2 = sum (x0_c - x0_u) * (x0_c * m).
// Stage 1: kApgChunks CTAs per prompt each reduce a contiguous slice in double; stage 2 folds the
// chunk partials in a fixed order (deterministic) and writes n = sqrt(s1 + 1e-16), dot = s2 / n.
constexpr int kApgChunks = 64;

__global__ void __launch_bounds__(256) dit_apg_partial_kernel(const float* __restrict__ part, int splits,
                                                              int64_t split_stride, const float* __restrict__ x,
                                                              const float* __restrict__ mask, int B, int T,
                                                              const DitStepCoef* __restrict__ coefs,
                                                              const DitBatchCoef* __restrict__ bcoefs, int step,
                                                              double* __restrict__ partials) {
    const DitStepCoef k = coefs[step];
    const int b = blockIdx.y, chunk = blockIdx.x;
    const DitBatchCoef kb = bcoefs[int64_t(step) * B + b];
    const int n = T * 64;
    const int per = (n + kApgChunks - 1) / kApgChunks;
    const int i0 = chunk * per, i1 = min(n, i0 + per);
    double s1 = 0.0, s2 = 0.0;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const int t = i / 64, c = i % 64;
        const float xin = x[(int64_t(b) * 64 + c) * T + t] * k.c_in;
        const float xa = xin * kb.alpha;
        const float cx0 = xa - dit_raw(part, splits, split_stride, b, T, t, c) * kb.sigma;
        const float ux0 = xa - dit_raw(part, splits, split_stride, b + B, T, t, c) * kb.sigma;
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

__global__ void dit_apg_finish_kernel(const double* __restrict__ partials, float* __restrict__ sums) {
    const int b = blockIdx.x;
    if (threadIdx.x == 0) {
        double a = 0.0, c = 0.0;
        for (int i = 0; i < kApgChunks; ++i) {
            a += partials[(int64_t(b) * kApgChunks + i) * 2];
            c += partials[(int64_t(b) * kApgChunks + i) * 2 + 1];
        }
        const float nrm = sqrtf(float(a) + 1e-16f);
        sums[2 * b] = nrm;
        sums[2 * b + 1] = float(c) / nrm;
    }
}

// Fused: CFG/APG combine (or the raw output without CFG), then the sampler update of
// x [B, 64, T] (BCT): DPM++ 2M, DPM++ 3M SDE (history ring + inline Philox noise) or v-DDIM;
// writes this step's denoised output to hist_cur and the next step's input; non-finite check.
template <typename CT>
__global__ void dit_update_kernel(const float* __restrict__ part, int splits, int64_t split_stride,
                                  float* __restrict__ x, float* __restrict__ hist_cur,
                                  const float* __restrict__ hist_p1, const float* __restrict__ hist_p2,
                                  const float* __restrict__ mask, const float* __restrict__ sums, int B, int Bg, int T,
                                  int use_cfg, const DitStepCoef* __restrict__ coefs,
                                  const DitBatchCoef* __restrict__ bcoefs, int step, CT* __restrict__ Xnext,
                                  float* __restrict__ out, int* __restrict__ status) {
    const DitStepCoef k = coefs[step];
    const int64_t total = int64_t(B) * 64 * T;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int t = int(i % T);
        const int c = int((i / T) % 64);
        const int b = int(i / (int64_t(T) * 64));
        const DitBatchCoef kb = bcoefs[int64_t(step) * B + b];
        const float xv = x[i];
        float mo;
        if (use_cfg) {  // build_cfg_model_output, rf_dit.cpp:988-1028
            const float xa = (xv * k.c_in) * kb.alpha;
            const float cx0 = xa - dit_raw(part, splits, split_stride, b, T, t, c) * kb.sigma;
            const float ux0 = xa - dit_raw(part, splits, split_stride, b + B, T, t, c) * kb.sigma;
            const float diff = cx0 - ux0;
            const float m = mask[int64_t(b) * T + t];
            const float n = sums[2 * b], dot = sums[2 * b + 1];
            const float v1 = (cx0 * m) / n;
            const float orth = (diff - dot * v1) * m;
            const float cd = k.apg_scale * orth + (1.0f - k.apg_scale) * diff;
            const float den = cx0 + (k.cfg_scale - 1.0f) * cd;
            mo = (xa - den) / kb.sigma;
        } else {
            mo = dit_raw(part, splits, split_stride, b, T, t, c);
        }
        float nx;
        bool bad = !isfinite(mo);
        if (k.mode == kVDdim) {
            const float pred = xv * kb.alpha - mo * kb.sigma;
            if (k.final_step) {
                nx = pred;
            } else {
                const float eps = xv * kb.sigma + mo * kb.alpha;
                nx = pred * kb.alpha_next + eps * kb.sigma_next;
            }
        } else {
            const float denoised = mo * k.c_out + xv * k.c_skip;
            bad = bad || !isfinite(denoised);
            if (k.final_step) {
                nx = denoised;
            } else if (k.mode == kDpmpp2m) {
                const float dd = k.first_step ? denoised : k.d_coeff * denoised + k.old_coeff * hist_p1[i];
                nx = k.x_scale * xv + k.d_scale * dd;
            } else {  // DPM++ 3M SDE
                nx = k.x_scale * xv + k.d_scale * denoised;
                if (k.hist >= 2) {
                    const float d1_0 = (denoised - hist_p1[i]) / k.r0;
                    const float d1_1 = (hist_p1[i] - hist_p2[i]) / k.r1;
                    const float d1 = d1_0 + (d1_0 - d1_1) * k.r0 / (k.r0 + k.r1);
                    const float d2 = (d1_0 - d1_1) / (k.r0 + k.r1);
                    nx += k.phi2 * d1 - k.phi3 * d2;
                } else if (k.hist == 1) {
                    nx += k.phi2 * ((denoised - hist_p1[i]) / k.r0);
                }
                nx += torch_iterator_randn_at(k.seed, k.rng_offset, k.rng_stride, uint64_t(i) + k.rng_elem0) * k.noise_scale;
            }
            hist_cur[i] = denoised;
        }
        bad = bad || !isfinite(nx);
        if (bad) atomicCAS(status, 0, kErrNonFinite);
        x[i] = nx;
        if (k.final_step) {
            out[i] = nx;
        } else {
            const CT h = from_f32<CT>(nx * k.c_in_next);
            for (int bb = b; bb < Bg; bb += B) Xnext[(int64_t(bb) * T + t) * 64 + c] = h;
        }
    }
}

// x = noise * sigma_0   (rf_dit.cpp:810-813)
__global__ void dit_init_kernel(const float* __restrict__ noise, int64_t n, const DitStepCoef* __restrict__ coefs,
                                float* __restrict__ x) {
    const float s0 = coefs[0].sig;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        x[i] = noise[i] * s0;
}

// Per hidden row padding factor: 1 for the global token, the latent mask for token rows
// (make_padding_mask, rf_dit.cpp:1085-1095).
__global__ void dit_padrow_kernel(const float* __restrict__ mask, int B, int Bg, int T, float* __restrict__ padrow) {
    const int64_t total = int64_t(Bg) * (T + 1);
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int bb = int(i / (T + 1)), t = int(i % (T + 1));
        padrow[i] = t == 0 ? 1.0f : mask[int64_t(bb % B) * T + t - 1];
    }
}

}  // namespace b2d
