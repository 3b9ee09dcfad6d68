// Implicit-GEMM 1-D convolution on tcgen05 for the Oobleck VAE decoder
// (src/models/stable_audio/foundation/oobleck_autoencoder.cpp): activations are time-major
// [sequence][time][channel] fp16/bf16, so tap j of a conv is the activation tile shifted by
// j * dil - pad rows.  The producer loads that shifted tile straight from global memory with a 3-D
// TMA box (rows before 0 or past the sequence end read zeros = the conv's zero padding), so no
// im2col buffer exists.  K = taps x Cin walks (tap, 64-channel block); the weights are pre-laid
// out as [N][taps * Cin].  A transposed conv (kernel 2s, stride s) is the same GEMM with two taps
// (offsets -1, 0) and N = s x Cout phases; its epilogue scatters phase p of input row q to output
// time q s + p - crop, which also applies the reference's crop.
//
// Roles per CTA (192 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue (one
// TMEM lane quarter each, thread = output row).  Persistent grid over (sequence, 128-row tile,
// BN-column tile); double-buffered TMEM accumulator; every wait bounded (status word on expiry).
#pragma once

#include "gemm.cuh"
#include "ptx.cuh"

namespace b2d {

enum ConvMode : int {
    kConvStoreF32 = 0,  // out_f32[row, n] = acc + bias[n]
    kConvSnakeCt = 1,   // out_ct[row, n] = ct(snake(acc + bias[n]))
    kConvResid = 2,     // v = acc + bias[n] (+ out_f32 when accumulate); out_f32 = v; out_ct = ct(snake(v)) if given
    kConvUpsample = 3,  // transposed conv: column n = (phase, o); row q -> time q s + phase - crop; then as kConvResid
    kConvGeluCt = 4,    // out_ct[row, n] = ct(gelu_erf(acc + bias[n]))
};

struct ConvParams {
    int mseq;          // GEMM rows (output rows) per sequence (upsample: input rows + 1)
    int nseq;
    int cinb;          // Cin / 64
    int dil, pad;      // tap j reads activation row r + j * dil - pad
    int mode;
    int accumulate;    // kConvResid: add the existing out_f32
    const float* bias;
    float* out_f32;
    int64_t ld_f32;    // row stride of out_f32 (elements)
    void* out_ct;
    int64_t ld_ct;
    const float* snake_a;      // exp(alpha) per column (or per o for upsample)
    const float* snake_ib;     // 1 / (exp(beta) + 1e-9)
    int stride, crop, cout;    // kConvUpsample
    int64_t out_rows_seq;      // kConvUpsample: output rows per sequence (input rows x stride)
    const float* scale;        // kConvResid: per-column factor on (acc + bias) before the accumulate (or null)
    int* status;
};

// The sine goes to the SFU (__sinf): the epilogues evaluate one per output element (about 3 G per
// SAO-shape decode), and the full-range sinf made them the critical path; the SFU result's absolute
// error (a few 1e-6 for the |alpha x| of a decoder) is far below the fp16 rounding of the operands.
__device__ __forceinline__ float snake_f(float x, float a, float ib) {
    const float s = __sinf(x * a);
    return x + s * s * ib;
}

template <int BN, typename CT>
__global__ void __launch_bounds__(192, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int N, int K,
                   ConvParams cp) {
    using S = GemmShape<BN>;
    constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * S::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int mt_seq = (cp.mseq + BM - 1) / BM;
    const int m_tiles = mt_seq * cp.nseq;
    const int num_tiles = m_tiles * (N / BN);
    const int k_blocks = K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int mt = tile % m_tiles;
                const int seq = mt / mt_seq;
                const int m0 = (mt % mt_seq) * BM;
                const int n0 = (tile / m_tiles) * BN;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, cp.status, kErrTimeoutProducer)) goto done;
                    const int tap = kb / cp.cinb;
                    const int c0 = (kb - tap * cp.cinb) * BK;
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], S::STAGE_BYTES);
                    tma_load_3d(sa, &tmA, &full[stage], c0, m0 + tap * cp.dil - cp.pad, seq);
                    tma_load_2d(sa + S::A_BYTES, &tmB, &full[stage], kb * BK, n0);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(CtTraits<CT>::kFmt, BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, cp.status, kErrTimeoutMma)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, cp.status, kErrTimeoutMma)) goto done;
                    tc_fence_after();
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    const uint64_t adesc = smem_desc_sw128(sa);
                    const uint64_t bdesc = smem_desc_sw128(sa + S::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16_ss(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                   (kb | k) != 0 ? 1u : 0u);
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                mma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    } else {
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int mt = tile % m_tiles;
            const int seq = mt / mt_seq;
            const int m0 = (mt % mt_seq) * BM;
            const int n0 = (tile / m_tiles) * BN;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, cp.status, kErrTimeoutEpilogue)) goto done;
            tc_fence_after();
            const int r = m0 + quarter * 32 + lane;  // output row within the sequence (upsample: input row q)
            const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(tbase + uint32_t(c * 32), v);
                tmem_ld_wait();
                if (r >= cp.mseq) continue;
                const int col0 = n0 + c * 32;
                int64_t orow;
                int ocol0;
                if (cp.mode == kConvUpsample) {
                    const int ph = col0 / cp.cout;
                    ocol0 = col0 - ph * cp.cout;
                    const int64_t t = int64_t(r) * cp.stride + ph - cp.crop;
                    if (t < 0 || t >= cp.out_rows_seq) continue;
                    orow = int64_t(seq) * cp.out_rows_seq + t;
                } else {
                    ocol0 = col0;
                    orow = int64_t(seq) * cp.mseq + r;
                }
                if (cp.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += __ldg(cp.bias + ocol0 + j);
                }
                if (cp.mode == kConvResid && cp.scale) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] *= __ldg(cp.scale + ocol0 + j);
                }
                if (cp.mode == kConvGeluCt) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.0f + erff(v[j] * 0.70710678118654752f));
                }
                if (cp.mode != kConvSnakeCt && cp.mode != kConvGeluCt) {
                    float4* o4 = reinterpret_cast<float4*>(cp.out_f32 + orow * cp.ld_f32 + ocol0);
                    if (cp.mode == kConvResid && cp.accumulate) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 h = o4[q];
                            v[4 * q] += h.x;
                            v[4 * q + 1] += h.y;
                            v[4 * q + 2] += h.z;
                            v[4 * q + 3] += h.w;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                }
                if (cp.mode != kConvStoreF32 && cp.out_ct) {
                    if (cp.snake_a) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            v[j] = snake_f(v[j], __ldg(cp.snake_a + ocol0 + j), __ldg(cp.snake_ib + ocol0 + j));
                    }
                    uint32_t packed[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) packed[j] = CtTraits<CT>::pack2(v[2 * j], v[2 * j + 1]);
                    uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<CT*>(cp.out_ct) + orow * cp.ld_ct + ocol0);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, S::TMEM_COLS);
    }
}

// Latents [B, C, T] (BCT, fp32) -> time-major operand [B][T][C].
template <typename CT>
__global__ void bct_to_btc_kernel(const float* __restrict__ x, int B, int C, int T, CT* __restrict__ out) {
    const int64_t total = int64_t(B) * C * T;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % C);
        const int t = int((i / C) % T);
        const int b = int(i / (int64_t(C) * T));
        out[i] = from_f32<CT>(x[(int64_t(b) * C + c) * T + t]);
    }
}

// First `ch` columns of the padded out-conv result [B * F, ld] -> audio [B, F, ch] (interleaved frames).
__global__ void take_channels_kernel(const float* __restrict__ y, int64_t ld, int64_t rows, int ch,
                                     float* __restrict__ audio, int* __restrict__ status) {
    const int64_t total = rows * ch;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = y[(i / ch) * ld + i % ch];
        if (!isfinite(v)) atomicCAS(status, 0, kErrNonFinite);
        audio[i] = v;
    }
}

// VibeVoice tokenizer blocks (src/models/vibevoice/tokenizer_audio.cpp:679-740), time-major rows of C channels.
// Per-row RMS scale 1 / sqrt(mean(x^2) + eps); with `out` also ct(x * scale * w).  One warp per row.
// C is the row stride; cmean the channels the mean runs over (the rest are zero padding with zero weights).
template <typename CT>
__global__ void __launch_bounds__(256) tok_rms_kernel(const float* __restrict__ x, int C, int cmean, int64_t rows,
                                                      const float* __restrict__ w, float eps,
                                                      float* __restrict__ scale, CT* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* xr = x + row * C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) ss += xr[c] * xr[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float sc = 1.0f / sqrtf(ss / float(cmean) + eps);
    if (scale && lane == 0) scale[row] = sc;
    if (out)
        for (int c = lane; c < C; c += 32) out[row * C + c] = from_f32<CT>(xr[c] * sc * __ldg(w + c));
}

// Block mixer: y[t, c] = x[t, c] + gamma[c] (b[c] + sum_k dw[c, k] rms(x)[t - K + 1 + k, c]), rms(x) = x * scale[t]
// * nw[c], zeros before t = 0 (the causal depthwise conv).  Rows of one sequence; y must not alias x.
__global__ void tok_mixer_kernel(const float* __restrict__ x, const float* __restrict__ scale, int C, int64_t rows,
                                 const float* __restrict__ nw, const float* __restrict__ dw, int K,
                                 const float* __restrict__ db, const float* __restrict__ gamma, float* __restrict__ y) {
    const int64_t total = rows * C;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % C);
        const int64_t t = i / C;
        float acc = 0.f;
        for (int k = 0; k < K; ++k) {
            const int64_t tt = t - (K - 1) + k;
            if (tt >= 0) acc += dw[c * K + k] * (x[tt * C + c] * scale[tt] * nw[c]);
        }
        y[i] = x[i] + gamma[c] * (acc + db[c]);
    }
}

}  // namespace b2d
