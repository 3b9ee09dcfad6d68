// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 64:
// O = softmax(Q K^T / 8) V for every (sequence, head, 128-query tile).  Same contract as
// flash_attn_kernel (attention.cuh), which it replaces on the DiT path: ggml_flash_attn_ext
// as rf_attention uses it (src/models/stable_audio/foundation/rf_dit.cpp:175-198), both the
// self-attention (L = 1025) and the T5 cross-attention (130 keys, KV head = h / kv_rep).
//
// CTA (352 threads, one CTA per SM) = two 128-query tiles of one (sequence, head) sharing the
// K/V stream:
//   warp 0      TMA producer: Q tiles once, then 128-key K and V blocks through a 2-deep ring
//               (3-D tensor maps [sequence][row][column]: rows past a sequence's end read 0)
//   warps 1, 2  MMA issuers of tile 0 / tile 1 (warp 1 also owns TMEM), so the two tiles never
//               wait on each other.  S_t = Q_t K_j^T is issued as two 64-key halves
//               (M 128, N 64, K 64) with their own full / free barriers, so the first half of the
//               next block is computed while the softmax still works on the second half of this
//               one; O_t += P_t V_j  (M 128, N 64, K 128; P K-major from smem, V MN-major).  A K
//               or V stage is released when the MMAs of every active tile that read it completed.
//   warps 3-6   softmax of tile 0, warps 7-10 softmax of tile 1 (thread = query row = TMEM lane).
//               Per 32-key chunk: S -> registers, p = 2^(s*scale*log2e - m) -> fp16/bf16 P (SW128
//               K-major, double-buffered so the next P never waits for the previous P V), row sum.
//               m is a lazily raised running max: only when a score exceeds it by more than 2^8
//               (p > 256, still exact in fp32 / fp16 / bf16 range) is m raised to the chunk max and
//               the row's sum, its P chunks already written for this block, and O (in TMEM) scaled
//               down.  The epilogue applies 1/l, stages O through the dead Q tile and writes it
//               with one TMA store (rows past the sequence are clipped).
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,320), O_1 [320,384).
// Keys past lk get p = 0; V rows there are zero-filled by TMA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "gemm.cuh"
#include "ptx.cuh"

namespace b2d {

constexpr int kFaStages = 2;
constexpr int kFaThreads = 352;
constexpr uint32_t kFaTile = 128 * 64 * 2;              // one 128 x 64 fp16/bf16 tile, 16 KB
constexpr uint32_t kFaQ = 0;                            // two Q tiles (reused as O staging)
constexpr uint32_t kFaK = 2 * kFaTile;                  // K ring
constexpr uint32_t kFaV = kFaK + kFaStages * kFaTile;   // V ring
constexpr uint32_t kFaP = kFaV + kFaStages * kFaTile;   // P[tile][buffer], 128 x 128 = two 16 KB panels
constexpr uint32_t kFaBar = kFaP + 8 * kFaTile;
constexpr uint32_t kFaSmemBytes = kFaBar + 256 + 1024;  // + barriers + alignment slack
constexpr float kFaRescaleLog2 = 8.0f;                  // lazy-rescale bound (log2 units)

// Optional phase trace of CTA (0,0,0) for profiling builds (-DB2D_FA_TRACE): clock64 stamps
// at trace[event * 64 + block].
#ifdef B2D_FA_TRACE
__device__ unsigned long long g_fa_trace[32 * 64];
#define FA_STAMP(ev, j)                                                                      \
    do {                                                                                     \
        if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (j) < 64)               \
            g_fa_trace[(ev) * 64 + (j)] = clock64();                                         \
    } while (0)
#else
#define FA_STAMP(ev, j) \
    do {                \
    } while (0)
#endif

struct FaArgs {
    int lq, lk, kv_rep, nseq;
    float scale_log2;
    int* status;
};

// Scales the 8 packed fp16/bf16 values of one 16-byte P chunk by f.
template <typename CT>
__device__ __forceinline__ void fa_scale_chunk(uint8_t* p, float f) {
    uint4 v = *reinterpret_cast<uint4*>(p);
    uint32_t* w = &v.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        CT h[2];
        *reinterpret_cast<uint32_t*>(h) = w[i];
        w[i] = CtTraits<CT>::pack2(float(h[0]) * f, float(h[1]) * f);
    }
    *reinterpret_cast<uint4*>(p) = v;
}

template <typename CT>
__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, FaArgs a) {
    extern __shared__ uint8_t fa_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFaBar);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;               // [stage]
    uint64_t* k_empty = k_full + kFaStages;    // [stage]
    uint64_t* v_full = k_empty + kFaStages;    // [stage]
    uint64_t* v_empty = v_full + kFaStages;    // [stage]
    uint64_t* s_full = v_empty + kFaStages;    // [tile][half]
    uint64_t* s_free = s_full + 4;             // [tile][half]
    uint64_t* p_full = s_free + 4;             // [tile]
    uint64_t* pv_done = p_full + 2;            // [tile][P buffer]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.y, seq = blockIdx.z;
    const int kvh = head / a.kv_rep;
    const int q0[2] = {int(blockIdx.x) * 256, int(blockIdx.x) * 256 + 128};
    const bool active[2] = {q0[0] < a.lq, q0[1] < a.lq};
    const int nb = (a.lk + 127) / 128;

    if (threadIdx.x == 0) {
        const uint32_t readers = uint32_t(active[0]) + uint32_t(active[1]);
        mbar_init(q_full, 1);
        for (int s = 0; s < kFaStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], readers);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], readers);
        }
        // softmax arrivals come only from warps that own a valid query row (a warp without one
        // would run ahead and complete the next phase early)
        for (int t = 0; t < 2; ++t) {
            const uint32_t warps = active[t] ? uint32_t(min(4, (a.lq - q0[t] + 31) >> 5)) : 1u;
            for (int h = 0; h < 2; ++h) {
                mbar_init(&s_full[t * 2 + h], 1);
                mbar_init(&s_free[t * 2 + h], warps);
                mbar_init(&pv_done[t * 2 + h], 1);
            }
            mbar_init(&p_full[t], warps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmO);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, (active[0] + active[1]) * kFaTile);
            for (int t = 0; t < 2; ++t)
                if (active[t]) tma_load_3d(smem + kFaQ + t * kFaTile, &tmQ, q_full, head * 64, q0[t], seq);
            for (int j = 0; j < nb; ++j) {
                const int s = j % kFaStages;
                const uint32_t ph = uint32_t(j / kFaStages) & 1u;
                if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag, a.status, kErrTimeoutProducer)) break;
                FA_STAMP(0, j);
                mbar_arrive_expect_tx(&k_full[s], kFaTile);
                tma_load_3d(smem + kFaK + s * kFaTile, &tmK, &k_full[s], kvh * 64, j * 128, seq);
                if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag, a.status, kErrTimeoutProducer)) break;
                FA_STAMP(1, j);
                mbar_arrive_expect_tx(&v_full[s], kFaTile);
                tma_load_3d(smem + kFaV + s * kFaTile, &tmV, &v_full[s], kvh * 64, j * 128, seq);
            }
        }
    } else if (warp <= 2) {
        const int t = warp - 1;
        if (lane == 0 && active[t]) {
            constexpr uint32_t idS = idesc_f16(CtTraits<CT>::kFmt, 128, 64);
            constexpr uint32_t idPV = idesc_f16(CtTraits<CT>::kFmt, 128, 64) | (1u << 16);  // B (V) MN-major
            const uint32_t dS = tmem_base + uint32_t(t * 128), dO = tmem_base + 256u + uint32_t(t * 64);
            const uint64_t qd = smem_desc_sw128(smem + kFaQ + t * kFaTile);
            bool ok = mbar_wait(q_full, 0, abort_flag, a.status, kErrTimeoutMma);
            // S halves of block j are issued before P V of block j - 1
            for (int j = 0; ok && j <= nb; ++j) {
                if (j < nb) {
                    const int s = j % kFaStages;
                    if (!(ok = mbar_wait(&k_full[s], uint32_t(j / kFaStages) & 1u, abort_flag, a.status,
                                         kErrTimeoutMma)))
                        break;
                    const uint64_t kd = smem_desc_sw128(smem + kFaK + s * kFaTile);
                    for (int h = 0; h < 2; ++h) {
                        if (j > 0 && !(ok = mbar_wait(&s_free[t * 2 + h], uint32_t(j - 1) & 1u, abort_flag,
                                                      a.status, kErrTimeoutMma)))
                            break;
                        tc_fence_after();
                        if (h == 0) FA_STAMP(2 + t, j);
                        // keys 64h.. of the K tile start 64 rows = 8 KB in (8 x 1024 B swizzle atoms)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            mma_f16_ss(dS + uint32_t(h * 64), qd + uint64_t(2 * k),
                                       kd + uint64_t(h * (8192 >> 4) + 2 * k), idS, k > 0 ? 1u : 0u);
                        mma_commit(&s_full[t * 2 + h]);
                    }
                    if (!ok) break;
                    mma_commit(&k_empty[s]);
                }
                if (j > 0) {
                    const int jj = j - 1, s = jj % kFaStages;
                    if (!(ok = mbar_wait(&v_full[s], uint32_t(jj / kFaStages) & 1u, abort_flag, a.status,
                                         kErrTimeoutMma)))
                        break;
                    if (!(ok = mbar_wait(&p_full[t], uint32_t(jj) & 1u, abort_flag, a.status, kErrTimeoutMma)))
                        break;
                    tc_fence_after();
                    FA_STAMP(4 + t, jj);
                    const uint8_t* pt = smem + kFaP + (t * 2 + (jj & 1)) * 2 * kFaTile;
                    const uint64_t vd = smem_desc_sw128(smem + kFaV + s * kFaTile);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        // P: K-major, two 64-key panels; V: MN-major, 16 keys = 2 x 1024 B groups
                        const uint64_t pd = smem_desc_sw128(pt + (k >> 2) * kFaTile) + uint64_t(2 * (k & 3));
                        mma_f16_ss(dO, pd, vd + uint64_t(128 * k), idPV, (jj | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(&pv_done[t * 2 + (jj & 1)]);
                    mma_commit(&v_empty[s]);
                }
            }
        }
    } else {
        const int t = (warp - 3) >> 2;  // query tile of this softmax group
        const int wq = warp & 3;        // TMEM lane quarter this warp may access
        const int row = wq * 32 + lane;
        const bool warp_rows = q0[t] + wq * 32 < a.lq;  // warp-uniform: any valid query row
        if (active[t] && warp_rows) {
            const uint32_t lane_off = uint32_t(wq * 32) << 16;
            const uint32_t tS = tmem_base + lane_off + uint32_t(t * 128);
            const uint32_t tO = tmem_base + lane_off + 256u + uint32_t(t * 64);
            const uint32_t sw = uint32_t(row & 7);
            const float sl = a.scale_log2;
            float m_used = 0.f, l = 0.f;  // m_used is set by the first chunk of block 0
            bool ok = true;
            for (int j = 0; j < nb && ok; ++j) {
                const int nvalid = min(128, a.lk - j * 128);
                const int nchunk = (nvalid + 31) >> 5;
                uint8_t* prow = smem + kFaP + (t * 2 + (j & 1)) * 2 * kFaTile + row * 128;
                // this P buffer was last read by P V of block j - 2
                if (j >= 2) {
                    ok = mbar_wait(&pv_done[t * 2 + (j & 1)], uint32_t((j >> 1) - 1) & 1u, abort_flag, a.status,
                                   kErrTimeoutEpilogue);
                    if (!ok) break;
                }
                float alpha_o = 1.f;  // factor this block applies to O (product of the chunk rescales)
                bool need_o = false;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    ok = mbar_wait(&s_full[t * 2 + h], uint32_t(j) & 1u, abort_flag, a.status, kErrTimeoutEpilogue);
                    if (!ok) break;
                    tc_fence_after();
                    if (h == 0 && wq == 0 && lane == 0) FA_STAMP(6 + t, j);
                    float x[2][32];
                    if (warp_rows) {
                        if (2 * h < nchunk) tmem_ld_32x32b_x32(tS + uint32_t(64 * h), x[0]);
                        if (2 * h + 1 < nchunk) tmem_ld_32x32b_x32(tS + uint32_t(64 * h + 32), x[1]);
                        tmem_ld_wait();
                    }
                    // the half is in registers: the next block's scores may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_free[t * 2 + h]);
                    if (!warp_rows) continue;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int c = 2 * h + cc;
                        float (&v)[32] = x[cc];
                        if (c < nchunk) {
                            if (j == 0 && c == 0) {
                                // first chunk of the row: m = its max (chunk 0 of block 0 has a valid key)
                                float amax = -INFINITY;
#pragma unroll
                                for (int i = 0; i < 32; ++i) {
                                    v[i] = i < nvalid ? v[i] * sl : -INFINITY;
                                    amax = fmaxf(amax, v[i]);
                                }
                                m_used = amax;
#pragma unroll
                                for (int i = 0; i < 32; ++i) v[i] -= amax;
                            } else {
                                // arguments of 2^(.) with the current running max; masked keys -> -inf
                                float amax = -INFINITY;
                                const float neg_m = -m_used;
                                if (nvalid == 128) {
#pragma unroll
                                    for (int i = 0; i < 32; ++i) {
                                        v[i] = fmaf(v[i], sl, neg_m);
                                        amax = fmaxf(amax, v[i]);
                                    }
                                } else {
#pragma unroll
                                    for (int i = 0; i < 32; ++i) {
                                        v[i] = c * 32 + i < nvalid ? fmaf(v[i], sl, neg_m) : -INFINITY;
                                        amax = fmaxf(amax, v[i]);
                                    }
                                }
                                const bool exceed = amax > kFaRescaleLog2;
                                if (__any_sync(0xffffffffu, exceed)) {
                                    // raise m to this chunk's max: shift the arguments, scale the row's sum,
                                    // the P chunks already written for this block and (later) O
                                    const float shift = exceed ? amax : 0.f;
                                    const float f = ex2_approx(-shift);
                                    m_used += shift;
                                    l *= f;
                                    alpha_o *= f;
#pragma unroll
                                    for (int i = 0; i < 32; ++i) v[i] -= shift;
                                    if (exceed) {
#pragma unroll
                                        for (int cp = 0; cp < c; ++cp)
#pragma unroll
                                            for (int q = 0; q < 4; ++q) {
                                                const uint32_t ch = uint32_t(cp * 4 + q);
                                                fa_scale_chunk<CT>(prow + (ch >> 3) * kFaTile + (((ch & 7u) ^ sw) << 4), f);
                                            }
                                    }
                                    need_o = true;
                                }
                            }
                            float s8[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) s8[e] = 0.f;
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                v[i] = ex2_approx(v[i]);
                                s8[i & 7] += v[i];
                            }
                            l += ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] = 0.f;
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint4 pk;
                            pk.x = CtTraits<CT>::pack2(v[8 * q + 0], v[8 * q + 1]);
                            pk.y = CtTraits<CT>::pack2(v[8 * q + 2], v[8 * q + 3]);
                            pk.z = CtTraits<CT>::pack2(v[8 * q + 4], v[8 * q + 5]);
                            pk.w = CtTraits<CT>::pack2(v[8 * q + 6], v[8 * q + 7]);
                            const uint32_t ch = uint32_t(c * 4 + q);  // 16-byte chunk of the 256-byte P row
                            *reinterpret_cast<uint4*>(prow + (ch >> 3) * kFaTile + (((ch & 7u) ^ sw) << 4)) = pk;
                        }
                    }
                    if (h == 0 && wq == 0 && lane == 0) FA_STAMP(8 + t, j);
                }
                if (!ok) break;
                if (warp_rows) fence_proxy_async_smem();
                if (wq == 0 && lane == 0) FA_STAMP(10 + t, j);
                // O holds the P V sums of blocks < j at the old max: scale it once P V of block j - 1 is in
                if (j > 0 && warp_rows && __any_sync(0xffffffffu, need_o)) {
                    ok = mbar_wait(&pv_done[t * 2 + ((j - 1) & 1)], uint32_t((j - 1) >> 1) & 1u, abort_flag, a.status,
                                   kErrTimeoutEpilogue);
                    if (!ok) break;
                    tc_fence_after();
                    float o[32];
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        tmem_ld_32x32b_x32(tO + uint32_t(c * 32), o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha_o;
                        tmem_st_32x32b_x32(tO + uint32_t(c * 32), o);
                    }
                    tmem_st_wait();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[t]);
                if (wq == 0 && lane == 0) FA_STAMP(12 + t, j);
            }
            // every warp of the group reaches the named barrier below exactly once, aborted or not
            if (ok)
                ok = mbar_wait(&pv_done[t * 2 + ((nb - 1) & 1)], uint32_t((nb - 1) >> 1) & 1u, abort_flag, a.status,
                               kErrTimeoutEpilogue);
            if (ok) {
                tc_fence_after();
                uint8_t* orow = smem + kFaQ + t * kFaTile + row * 128;  // Q tile is dead: stage O there
                if (warp_rows) {
                    const float inv = 1.f / l;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float o[32];
                        tmem_ld_32x32b_x32(tO + uint32_t(c * 32), o);
                        tmem_ld_wait();
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint4 v;
                            v.x = CtTraits<CT>::pack2(o[8 * q + 0] * inv, o[8 * q + 1] * inv);
                            v.y = CtTraits<CT>::pack2(o[8 * q + 2] * inv, o[8 * q + 3] * inv);
                            v.z = CtTraits<CT>::pack2(o[8 * q + 4] * inv, o[8 * q + 5] * inv);
                            v.w = CtTraits<CT>::pack2(o[8 * q + 6] * inv, o[8 * q + 7] * inv);
                            *reinterpret_cast<uint4*>(orow + ((uint32_t(c * 4 + q) ^ sw) << 4)) = v;
                        }
                    }
                    fence_proxy_async_smem();
                }
            }
            named_bar_sync(1 + t, 32u * uint32_t(min(4, (a.lq - q0[t] + 31) >> 5)));
            if (wq == 0 && lane == 0 && *abort_flag == 0) {
                tma_store_3d(&tmO, smem + kFaQ + t * kFaTile, head * 64, q0[t], seq);
                bulk_commit_group();
                bulk_wait_read_all();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

}  // namespace b2d
