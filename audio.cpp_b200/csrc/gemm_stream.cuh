// Weight-streaming tcgen05 GEMM for few activation rows:  C = A * W^T with M <= 128.
//
// With a hundred-odd rows a projection does only 2 M FLOP per weight it reads (M = 128 rows of an fp16
// weight: 128 FLOP per byte, against a ridge of about 260), so it is bound by the HBM weight stream and every
// SM must pull weights at once, whatever N is.  The grid is n_tiles x S CTAs: each column tile of BN weight
// rows is split over the K dimension into S contiguous ranges, computed by the S CTAs of one thread-block
// cluster.  Each CTA accumulates its K range in TMEM, copies the 128 x BN fp32 partial into its own shared
// memory, and after a cluster barrier CTA r sums rows [r 128 / S, (r + 1) 128 / S) of all S partials in rank
// order through distributed shared memory (fixed order: results do not depend on timing), applies the
// epilogue and writes the output with row-contiguous 16-byte stores.  No partial sum leaves the chip.
//
// Weights come either as 16-bit [N, K] matrices (TMA, 128-byte swizzle) or as Q8_0 blocks
// (ggml-common.h block_q8_0: 32 int8 quants + an fp16 scale d, value = q * d), stored k-block-major:
// quants [K/64][N][64] int8 and scales [K/64][N][2] fp16, so one 64-deep k-block of BN rows is two
// contiguous bulk copies (BN * 64 + BN * 4 bytes: 1.06 bytes per weight from HBM).  Four dequantising
// warps expand them in shared memory to fp16(q * fp32(d)) -- the value dequantize_row_q8_0
// (ggml-quants.c) produces, rounded once to fp16 -- in the swizzled K-major layout the MMA reads.
//
// CTA: warp 0 issues the weight loads (and, for 16-bit weights, the activation loads), warp 1 owns TMEM and
// issues tcgen05.mma (M = 128, N = BN, K = 16) from one lane, warps 2-5 move the accumulator to shared
// memory, warps 6-9 (Q8_0 only) dequantise and load the activations; all warps take part in the reduction.
#pragma once

#include "gemm.cuh"

namespace b2d {

enum WeightFmt : int { WF_16 = 0, WF_Q8 = 1 };

template <int BN, int WF>
struct StreamShape {
    static constexpr int BK = 64;
    static constexpr uint32_t A_BYTES = 128 * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t Q_BYTES = BN * 64;  // int8 quants of one k-block
    static constexpr uint32_t D_BYTES = BN * 4;   // two fp16 scales per row
    static constexpr uint32_t RAW_BYTES = Q_BYTES + D_BYTES;
    static constexpr int LDS = BN + 4;            // fp32 row stride of the accumulator copy (bank spread)
    static constexpr uint32_t ACC_BYTES = 128 * LDS * 4;
    // 16-bit weights: a deep operand ring (the weight stream needs ~64 KB in flight per SM); Q8_0: a short
    // operand ring fed by the dequantisers and a deep ring of raw blocks.
    static constexpr int STAGES = WF == WF_Q8 ? 3 : (BN == 64 ? 8 : BN == 128 ? 6 : BN == 192 ? 5 : 4);
    static constexpr size_t OPER_BYTES = size_t(STAGES) * STAGE_BYTES > ACC_BYTES ? size_t(STAGES) * STAGE_BYTES
                                                                                    : ACC_BYTES;
    static constexpr size_t BUDGET = 232448 - 1024 - 512;
    static constexpr int RAW_FIT = WF == WF_Q8 ? int((BUDGET - OPER_BYTES) / RAW_BYTES) : 0;
    static constexpr int RAW_STAGES = RAW_FIT > 8 ? 8 : RAW_FIT;
    static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static_assert(BN % 64 == 0 && BN <= 256, "tile width");
    static constexpr size_t SMEM_BYTES = OPER_BYTES + size_t(RAW_STAGES) * RAW_BYTES + 512 + 1024;
    static constexpr int THREADS = WF == WF_Q8 ? 320 : 192;
    static_assert(WF != WF_Q8 || RAW_STAGES >= 2, "raw ring");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

struct StreamArgs {
    int M = 0, N = 0, K = 0;
    int k_blocks = 0;
    const int8_t* q8 = nullptr;   // WF_Q8: quants [K/64][N][64]
    const __half* q8d = nullptr;  // WF_Q8: scales [K/64][N][2]
    // Up to two ranges the NEXT projection streams (its weights; Q8_0: quants and scales), hinted into L2 once
    // this kernel has issued all of its own loads: HBM keeps streaming through this kernel's tail (TMEM drain,
    // cluster reduction, epilogue) and the next kernel's launch and pipeline fill.  Each CTA takes an equal
    // 16-byte-aligned share.  Values are unaffected: a prefetch only warms L2.
    const uint8_t* pf[2] = {nullptr, nullptr};
    uint64_t pf_bytes[2] = {0, 0};
};

// This CTA's share of the L2 prefetch ranges, in pieces of at most 64 KB.
__device__ __forceinline__ void stream_prefetch_next(const StreamArgs& sa) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        if (sa.pf[r] == nullptr || sa.pf_bytes[r] < 16) continue;
        const uint64_t units = sa.pf_bytes[r] >> 4;  // whole 16-byte units (a tail below 16 bytes is left out)
        const uint64_t u0 = units * blockIdx.x / gridDim.x, u1 = units * (blockIdx.x + 1) / gridDim.x;
        for (uint64_t u = u0; u < u1; u += 4096) {
            const uint64_t n = u1 - u < 4096 ? u1 - u : 4096;
            bulk_prefetch_l2(sa.pf[r] + (u << 4), uint32_t(n << 4));
        }
    }
}

// Epilogue of 4 consecutive output columns [col, col + 4) of one row (col within the weight rows, n0 = the
// tile's first).  EPI_SWIGLU: v = gate sums, u = the matching linear-half sums (128 columns further);
// EPI_RESID: x, g = the residual and gate values there.
template <int EPI, typename CT>
__device__ __forceinline__ void stream_apply4(float4 v, float4 u, float4 x, float4 g, int64_t row, int col, int n0,
                                              const EpiParams& ep) {
    if constexpr (EPI == EPI_SWIGLU) {
        if (ep.bias) {
            const float4 bg = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
            const float4 bu = __ldg(reinterpret_cast<const float4*>(ep.bias + col + 128));
            v = make_float4(v.x + bg.x, v.y + bg.y, v.z + bg.z, v.w + bg.w);
            u = make_float4(u.x + bu.x, u.y + bu.y, u.z + bu.z, u.w + bu.w);
        }
        const uint2 o = make_uint2(CtTraits<CT>::pack2(silu_f(v.x) * u.x, silu_f(v.y) * u.y),
                                   CtTraits<CT>::pack2(silu_f(v.z) * u.z, silu_f(v.w) * u.w));
        *reinterpret_cast<uint2*>(reinterpret_cast<CT*>(ep.out) + row * ep.ldo + (n0 / 2 + (col - n0))) = o;
    } else {
        if (ep.bias) {
            const float4 b = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
            v = make_float4(v.x + b.x, v.y + b.y, v.z + b.z, v.w + b.w);
        }
        if constexpr (EPI == EPI_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(ep.out) + row * ep.ldo + col) = v;
        } else if constexpr (EPI == EPI_CT) {
            *reinterpret_cast<uint2*>(reinterpret_cast<CT*>(ep.out) + row * ep.ldo + col) =
                make_uint2(CtTraits<CT>::pack2(v.x, v.y), CtTraits<CT>::pack2(v.z, v.w));
        } else {  // EPI_RESID: x += g * v (x, g loaded by the caller; g = 1 without a gate)
            *reinterpret_cast<float4*>(ep.resid + row * ep.ldr + col) =
                make_float4(x.x + g.x * v.x, x.y + g.y * v.y, x.z + g.z * v.z, x.w + g.w * v.w);
        }
    }
}

template <int BN, int WF, int EPI, typename CT>
__global__ void __launch_bounds__(StreamShape<BN, WF>::THREADS, 1)
    gemm_stream_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       StreamArgs sa, EpiParams ep) {
    using S = StreamShape<BN, WF>;
    constexpr int STAGES = S::STAGES, RAW = WF == WF_Q8 ? S::RAW_STAGES : 1;
    constexpr int C = BN / 32;
    static_assert(EPI != EPI_SWIGLU || BN == 256, "SwiGLU tiles pair 128 + 128 columns");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* raw = smem + S::OPER_BYTES;
    float* accs = reinterpret_cast<float*>(smem);  // the accumulator copy reuses the operand ring at the end
    uint64_t* full = reinterpret_cast<uint64_t*>(raw + size_t(WF == WF_Q8 ? S::RAW_STAGES : 0) * S::RAW_BYTES);
    uint64_t* bfull = full + STAGES;
    uint64_t* empty = bfull + STAGES;
    uint64_t* rfull = empty + STAGES;
    uint64_t* rempty = rfull + RAW;
    uint64_t* tfull = rempty + RAW;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nsplit = int(cluster_nctarank());
    const int rank = int(cluster_ctarank());
    const int tile = int(blockIdx.x) / nsplit;
    const int n0 = tile * BN;
    const int kb = sa.k_blocks;
    const int kb0 = rank * kb / nsplit, nk = (rank + 1) * kb / nsplit - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&bfull[s], 4);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < RAW; ++r) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], 4);
        }
        mbar_init(tfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        if (WF == WF_16) tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // The weights are constant: the first ring's worth of weight tiles is requested before waiting for
            // the previous kernel (programmatic dependent launch); activations only after it.
            const int pre = WF == WF_16 ? (nk < STAGES ? nk : STAGES) : 0;
            for (int i = 0; i < pre; ++i) {
                uint8_t* st = smem + size_t(i) * S::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[i], S::STAGE_BYTES);
                tma_load_2d(st + S::A_BYTES, &tmB, &full[i], (kb0 + i) * 64, n0);
            }
            if (WF == WF_16) pdl_wait();
            for (int i = 0; i < pre; ++i) tma_load_2d(smem + size_t(i) * S::STAGE_BYTES, &tmA, &full[i], (kb0 + i) * 64, 0);
            for (int i = pre; i < nk; ++i) {
                const int k = kb0 + i;
                if constexpr (WF == WF_16) {
                    const int s = i % STAGES;
                    const uint32_t ph = uint32_t(i / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, ep.status, kErrTimeoutProducer)) break;
                    uint8_t* st = smem + size_t(s) * S::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
                    tma_load_2d(st, &tmA, &full[s], k * 64, 0);
                    tma_load_2d(st + S::A_BYTES, &tmB, &full[s], k * 64, n0);
                } else {
                    const int r = i % RAW;
                    const uint32_t ph = uint32_t(i / RAW) & 1u;
                    if (!mbar_wait(&rempty[r], ph ^ 1u, abort_flag, ep.status, kErrTimeoutProducer)) break;
                    uint8_t* rb = raw + size_t(r) * S::RAW_BYTES;
                    mbar_arrive_expect_tx(&rfull[r], S::RAW_BYTES);
                    const int64_t blk = int64_t(k) * sa.N + n0;
                    bulk_load(rb, sa.q8 + blk * 64, S::Q_BYTES, &rfull[r]);
                    bulk_load(rb + S::Q_BYTES, sa.q8d + blk * 2, S::D_BYTES, &rfull[r]);
                }
            }
            stream_prefetch_next(sa);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(CtTraits<CT>::kFmt, 128, BN);
            bool ok = true;
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = uint32_t(i / STAGES) & 1u;
                ok = mbar_wait(&full[s], ph, abort_flag, ep.status, kErrTimeoutMma);
                if (ok && WF == WF_Q8) ok = mbar_wait(&bfull[s], ph, abort_flag, ep.status, kErrTimeoutMma);
                if (!ok) break;
                tc_fence_after();
                uint8_t* st = smem + size_t(s) * S::STAGE_BYTES;
                const uint64_t adesc = smem_desc_sw128(st);
                const uint64_t bdesc = smem_desc_sw128(st + S::A_BYTES);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16_ss(tmem_base, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                               (i | k) != 0 ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(tfull);
        }
    } else if (warp >= 6) {
        // Q8_0 dequantisation (+ activation loads): 128 threads, BN / 128 weight rows each (BN 64: half the
        // threads)
        const int t = threadIdx.x - 192;
        if (t == 0) pdl_wait();  // before the first activation load
        for (int i = 0; i < nk; ++i) {
            const int s = i % STAGES, r = i % RAW;
            const int k = kb0 + i;
            if (!mbar_wait(&rfull[r], uint32_t(i / RAW) & 1u, abort_flag, ep.status, kErrTimeoutProducer)) break;
            if (!mbar_wait(&empty[s], (uint32_t(i / STAGES) & 1u) ^ 1u, abort_flag, ep.status, kErrTimeoutProducer))
                break;
            uint8_t* st = smem + size_t(s) * S::STAGE_BYTES;
            if (t == 0) {
                mbar_arrive_expect_tx(&full[s], S::A_BYTES);
                tma_load_2d(st, &tmA, &full[s], k * 64, 0);
            }
            const uint8_t* rb = raw + size_t(r) * S::RAW_BYTES;
            const __half* dsc = reinterpret_cast<const __half*>(rb + S::Q_BYTES);
            uint8_t* bt = st + S::A_BYTES;
#pragma unroll
            for (int rr = 0; rr < (BN + 127) / 128; ++rr) {
                const int n = t + 128 * rr;
                if (n >= BN) break;
                const float d0 = __half2float(dsc[2 * n]), d1 = __half2float(dsc[2 * n + 1]);
                const int4* q4 = reinterpret_cast<const int4*>(rb + n * 64);
#pragma unroll
                for (int c = 0; c < 4; ++c) {  // 16 quants -> two 16-byte chunks of 8 halves
                    const int4 qv = q4[c];
                    const int8_t* q = reinterpret_cast<const int8_t*>(&qv);
                    const float d = c < 2 ? d0 : d1;
                    uint32_t h[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const __half2 p = __floats2half2_rn(float(q[2 * j]) * d, float(q[2 * j + 1]) * d);
                        h[j] = *reinterpret_cast<const uint32_t*>(&p);
                    }
                    const int j0 = 2 * c, j1 = 2 * c + 1;  // 16-byte chunk index along K
                    *reinterpret_cast<uint4*>(bt + n * 128 + ((j0 ^ (n & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<uint4*>(bt + n * 128 + ((j1 ^ (n & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bfull[s]);
                mbar_arrive(&rempty[r]);
            }
        }
    } else {
        // warps 2-5: TMEM lanes [32 q, 32 q + 32) -> accumulator copy rows (stride LDS floats)
        const int quarter = warp & 3;
        if (mbar_wait(tfull, 0, abort_flag, ep.status, kErrTimeoutEpilogue)) {
            tc_fence_after();
            const uint32_t tb = tmem_base + (uint32_t(quarter * 32) << 16);
            float* arow = accs + size_t(quarter * 32 + lane) * S::LDS;
#pragma unroll 1
            for (int c = 0; c < C; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(tb + uint32_t(c * 32), v);
                tmem_ld_wait();
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<float4*>(arow + c * 32 + 4 * q) =
                        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
    }
    // Every thread of every CTA of the cluster reaches both cluster barriers, also after a wait gave up (the
    // status word then reports it and the output is not used).
    tc_fence_before();
    __syncthreads();
    if (nsplit > 1) cluster_sync();
    pdl_wait();  // outputs / residual / gate belong to the previous kernels until they completed
    {
        const int r0 = rank * 128 / nsplit;
        int r1 = (rank + 1) * 128 / nsplit;
        if (r1 > sa.M) r1 = sa.M;
        constexpr int GC = EPI == EPI_SWIGLU ? 128 / 4 : BN / 4;  // 4-column groups per row
        constexpr int U = 4;                                     // groups in flight per thread
        const uint32_t base = smem_u32(accs);
        const int total = (r1 - r0) * GC;
        for (int e0 = threadIdx.x; e0 < total; e0 += U * int(blockDim.x)) {
            // issue every load of U groups (peer partials; residual and gate) before using any of them
            float4 v[U], u[U], x[U], g[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                v[k] = u[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                x[k] = g[k] = make_float4(1.f, 1.f, 1.f, 1.f);
                const int e = e0 + k * int(blockDim.x);
                if (EPI == EPI_RESID && e < total) {
                    const int64_t row = r0 + e / GC;
                    const int col = n0 + (e % GC) * 4;
                    x[k] = *reinterpret_cast<const float4*>(ep.resid + row * ep.ldr + col);
                    if (ep.gate)
                        g[k] = *reinterpret_cast<const float4*>(
                            ep.gate + (ep.gate_rows ? row / ep.gate_rows : row) * ep.ldg + col);
                }
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (q >= nsplit) break;
                float4 p[U], pu[U];
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    const int e = e0 + k * int(blockDim.x);
                    if (e < total) {
                        const uint32_t off = uint32_t(((r0 + e / GC) * S::LDS + (e % GC) * 4) * 4);
                        const uint32_t a = map_to_cta(base + off, uint32_t(q));
                        p[k] = ld_dsmem_f4(a);
                        if (EPI == EPI_SWIGLU) pu[k] = ld_dsmem_f4(a + 128 * 4);
                    }
                }
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    v[k] = make_float4(v[k].x + p[k].x, v[k].y + p[k].y, v[k].z + p[k].z, v[k].w + p[k].w);
                    if (EPI == EPI_SWIGLU)
                        u[k] = make_float4(u[k].x + pu[k].x, u[k].y + pu[k].y, u[k].z + pu[k].z, u[k].w + pu[k].w);
                }
            }
            if (*abort_flag) continue;
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int e = e0 + k * int(blockDim.x);
                if (e < total)
                    stream_apply4<EPI, CT>(v[k], u[k], x[k], g[k], r0 + e / GC, n0 + (e % GC) * 4, n0, ep);
            }
        }
    }
    if (nsplit > 1) cluster_sync();  // no CTA leaves while a partner still reads its shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, S::TMEM_COLS);
    }
}

}  // namespace b2d
