// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 64:
// O = softmax(Q K^T / 8) V for every (sequence, head, 128-query tile).  Same contract as
// flash_attn_kernel (attention.cuh), which it replaces on the DiT path: ggml_flash_attn_ext
// as rf_attention uses it (src/models/stable_audio/foundation/rf_dit.cpp:175-198), both the
// self-attention (L = 1025) and the T5 cross-attention (130 keys, KV head = h / kv_rep).
//
// CTA (608 threads, one CTA per SM) = two 128-query tiles of one (sequence, head) sharing the
// K/V stream.  Keys come in 128-key blocks; each block is split into two 64-key halves, and
// half h of every block belongs to its own softmax warp set with its own running max, row sum
// and O accumulator (flash-decoding style split of the key range, merged in the epilogue):
//   warp 0        TMA producer: Q tiles once, then K and V blocks through a 2-deep ring
//                 (3-D tensor maps [sequence][row][column]: rows past a sequence's end read 0)
//   warps 1, 2    MMA issuers of tile 0 / tile 1 (warp 1 also owns TMEM):
//                 S_{t,h} = Q_t K_{j,h}^T   (M 128, N 64, K 64) into TMEM,
//                 O_{t,h} += P_{t,h} V_{j,h} (M 128, N 64, K 64; P K-major from smem, V MN-major);
//                 a K / V stage is released when the MMAs of every active tile that read it completed
//   warps 3-18    softmax, 4 warps per (tile, half); thread = query row = TMEM lane.  Per block:
//                 S half -> registers, p = 2^(s*scale*log2e - m) -> fp16/bf16 P (SW128 K-major,
//                 double-buffered so the next P never waits for the previous P V), row sum.  m is a
//                 lazily raised running max: only when a score exceeds it by more than 2^8 (p > 256,
//                 still exact in fp32 / fp16 / bf16 range) is it raised to the half's max and the
//                 row's sum and O (in TMEM) scaled down.  Four softmax warps share each SM
//                 sub-partition, so one warp's exponentials overlap another's bookkeeping.
// Epilogue: m = max(m_0, m_1), O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)),
// staged through the dead Q tile and written with one TMA store (rows past the sequence clipped).
// TMEM (512 columns): S_t at [128 t, 128 t + 128) (half h at +64 h), O_{t,h} at 256 + 128 t + 64 h.
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
constexpr int kFaThreads = 608;
constexpr uint32_t kFaTile = 128 * 64 * 2;              // one 128 x 64 fp16/bf16 tile, 16 KB
constexpr uint32_t kFaQ = 0;                            // two Q tiles (reused as O staging)
constexpr uint32_t kFaK = 2 * kFaTile;                  // K ring
constexpr uint32_t kFaV = kFaK + kFaStages * kFaTile;   // V ring
constexpr uint32_t kFaP = kFaV + kFaStages * kFaTile;   // P[tile][buffer][half]: 128 rows x 64 keys each
constexpr uint32_t kFaBar = kFaP + 8 * kFaTile;
constexpr uint32_t kFaSmemBytes = kFaBar + 256 + 1024;  // + barriers + alignment slack
constexpr float kFaRescaleLog2 = 8.0f;                  // lazy-rescale bound (log2 units)


struct FaArgs {
    int lq, lk, kv_rep, nseq;
    float scale_log2;
    int* status;
};

__device__ __forceinline__ float fa_max8(const float (&m)[8]) {
    return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
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
    uint64_t* p_full = s_free + 4;             // [tile][half]
    uint64_t* pv_done = p_full + 4;            // [tile][half][P buffer]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.y, seq = blockIdx.z;
    const int kvh = head / a.kv_rep;
    const int q0[2] = {int(blockIdx.x) * 256, int(blockIdx.x) * 256 + 128};
    const bool active[2] = {q0[0] < a.lq, q0[1] < a.lq};
    // softmax warps per (tile, half) that own a valid query row; only they arrive on the
    // softmax barriers (a warp without rows would run ahead and complete the next phase early)
    const int vw[2] = {active[0] ? min(4, (a.lq - q0[0] + 31) >> 5) : 0,
                       active[1] ? min(4, (a.lq - q0[1] + 31) >> 5) : 0};
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
        for (int t = 0; t < 2; ++t)
            for (int h = 0; h < 2; ++h) {
                const uint32_t w = vw[t] > 0 ? uint32_t(vw[t]) : 1u;
                mbar_init(&s_full[t * 2 + h], 1);
                mbar_init(&s_free[t * 2 + h], w);
                mbar_init(&p_full[t * 2 + h], w);
                mbar_init(&pv_done[(t * 2 + h) * 2 + 0], 1);
                mbar_init(&pv_done[(t * 2 + h) * 2 + 1], 1);
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
                mbar_arrive_expect_tx(&k_full[s], kFaTile);
                tma_load_3d(smem + kFaK + s * kFaTile, &tmK, &k_full[s], kvh * 64, j * 128, seq);
                if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag, a.status, kErrTimeoutProducer)) break;
                mbar_arrive_expect_tx(&v_full[s], kFaTile);
                tma_load_3d(smem + kFaV + s * kFaTile, &tmV, &v_full[s], kvh * 64, j * 128, seq);
            }
        }
    } else if (warp <= 2) {
        const int t = warp - 1;
        if (lane == 0 && active[t]) {
            constexpr uint32_t idS = idesc_f16(CtTraits<CT>::kFmt, 128, 64);
            constexpr uint32_t idPV = idesc_f16(CtTraits<CT>::kFmt, 128, 64) | (1u << 16);  // B (V) MN-major
            const uint32_t dS = tmem_base + uint32_t(t * 128), dO = tmem_base + 256u + uint32_t(t * 128);
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
                    const uint64_t vd = smem_desc_sw128(smem + kFaV + s * kFaTile);
                    for (int h = 0; h < 2; ++h) {
                        if (!(ok = mbar_wait(&p_full[t * 2 + h], uint32_t(jj) & 1u, abort_flag, a.status,
                                             kErrTimeoutMma)))
                            break;
                        tc_fence_after();
                        const uint64_t pd = smem_desc_sw128(smem + kFaP + ((t * 2 + (jj & 1)) * 2 + h) * kFaTile);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            // P: K-major 64-key panel (+32 B per 16 keys); V: MN-major, keys 64h + 16k
                            // start (64h + 16k) rows x 128 B in
                            mma_f16_ss(dO + uint32_t(h * 64), pd + uint64_t(2 * k),
                                       vd + uint64_t(h * (8192 >> 4) + 128 * k), idPV, (jj | k) != 0 ? 1u : 0u);
                        mma_commit(&pv_done[(t * 2 + h) * 2 + (jj & 1)]);
                    }
                    if (!ok) break;
                    mma_commit(&v_empty[s]);
                }
            }
        }
    } else {
        const int u = warp - 3;
        const int t = u >> 3;        // query tile
        const int h = (u >> 2) & 1;  // key half of every block owned by this warp set
        const int wq = warp & 3;     // TMEM lane quarter this warp may access
        const int row = wq * 32 + lane;
        if (active[t] && wq < vw[t]) {
            const uint32_t lane_off = uint32_t(wq * 32) << 16;
            const uint32_t tS = tmem_base + lane_off + uint32_t(t * 128 + h * 64);
            const uint32_t tO = tmem_base + lane_off + 256u + uint32_t(t * 128 + h * 64);
            const uint32_t sw = uint32_t(row & 7);
            const float sl = a.scale_log2;
            uint64_t* my_s_full = &s_full[t * 2 + h];
            uint64_t* my_s_free = &s_free[t * 2 + h];
            uint64_t* my_p_full = &p_full[t * 2 + h];
            uint64_t* my_pv = &pv_done[(t * 2 + h) * 2];
            float m_used = -INFINITY, l = 0.f;
            bool first = true;  // warp-uniform: no valid key seen yet
            bool ok = true;
            for (int j = 0; j < nb && ok; ++j) {
                const int kv = min(64, a.lk - j * 128 - h * 64);  // valid keys of this half (may be <= 0)
                uint8_t* prow = smem + kFaP + ((t * 2 + (j & 1)) * 2 + h) * kFaTile + row * 128;
                // this P buffer was last read by P V of block j - 2
                if (j >= 2) {
                    ok = mbar_wait(&my_pv[j & 1], uint32_t((j >> 1) - 1) & 1u, abort_flag, a.status,
                                   kErrTimeoutEpilogue);
                    if (!ok) break;
                }
                ok = mbar_wait(my_s_full, uint32_t(j) & 1u, abort_flag, a.status, kErrTimeoutEpilogue);
                if (!ok) break;
                tc_fence_after();
                // max over this half's valid keys, scaled to log2 units (S reloaded from TMEM)
                auto half_max = [&]() -> float {
                    float mx[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        if (c * 32 >= kv) break;
                        float x[32];
                        tmem_ld_32x32b_x32(tS + uint32_t(c * 32), x);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) mx[i & 7] = fmaxf(mx[i & 7], c * 32 + i < kv ? x[i] : -INFINITY);
                    }
                    return fa_max8(mx) * sl;
                };
                // p = 2^(s * scale - m) for the 64 keys, stored as this row's P (8 x 16 B chunks,
                // 128-byte swizzle); returns the row sum, and the largest p in pmax
                auto exp_pass = [&](float m, float& pmax) -> float {
                    float s8[8], p8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) s8[e] = p8[e] = 0.f;
                    const float neg_m = -m;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float x[32];
                        if (c * 32 < kv) {
                            tmem_ld_32x32b_x32(tS + uint32_t(c * 32), x);
                            tmem_ld_wait();
                            if (kv == 64) {
#pragma unroll
                                for (int i = 0; i < 32; ++i) x[i] = ex2_approx(fmaf(x[i], sl, neg_m));
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    x[i] = c * 32 + i < kv ? ex2_approx(fmaf(x[i], sl, neg_m)) : 0.f;
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) x[i] = 0.f;
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            s8[i & 7] += x[i];
                            p8[i & 7] = fmaxf(p8[i & 7], x[i]);
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint4 pk;
                            pk.x = CtTraits<CT>::pack2(x[8 * q + 0], x[8 * q + 1]);
                            pk.y = CtTraits<CT>::pack2(x[8 * q + 2], x[8 * q + 3]);
                            pk.z = CtTraits<CT>::pack2(x[8 * q + 4], x[8 * q + 5]);
                            pk.w = CtTraits<CT>::pack2(x[8 * q + 6], x[8 * q + 7]);
                            *reinterpret_cast<uint4*>(prow + ((uint32_t(c * 4 + q) ^ sw) << 4)) = pk;
                        }
                    }
                    pmax = fa_max8(p8);
                    return ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
                };
                float f_o = 1.f;  // factor O needs before this block's P V (lazy max raised)
                bool need_o = false;
                if (kv > 0) {
                    if (first) {  // first keys of the row: m = their max
                        m_used = half_max();
                        first = false;
                    }
                    float pmax;
                    float sum = exp_pass(m_used, pmax);
                    // a p above 2^8 (argument above 8, or +inf) flags a row whose max grew
                    const bool exceed = pmax > 256.f;
                    if (__any_sync(0xffffffffu, exceed)) {
                        // raise m to this half's max, redo p (overwriting P), scale the row's sum
                        // now and O before this block's P V
                        const float hm = half_max();
                        const float m_new = exceed ? hm : m_used;
                        f_o = ex2_approx(m_used - m_new);
                        m_used = m_new;
                        l *= f_o;
                        need_o = true;
                        sum = exp_pass(m_used, pmax);
                    }
                    l += sum;
                } else {
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch)
                        *reinterpret_cast<uint4*>(prow + ((uint32_t(ch) ^ sw) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                }
                // S half consumed: the next block's scores may overwrite it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(my_s_free);
                fence_proxy_async_smem();
                // P V of block j - 1 must be complete before P of block j is announced: it proves the
                // MMA warp consumed the previous announcement (an mbarrier phase must not be
                // completed twice before its waiter looks), and O is only rescaled after it
                if (j > 0) {
                    ok = mbar_wait(&my_pv[(j - 1) & 1], uint32_t((j - 1) >> 1) & 1u, abort_flag, a.status,
                                   kErrTimeoutEpilogue);
                    if (!ok) break;
                }
                // O holds this half's P V sums of blocks < j at the old max
                if (j > 0 && __any_sync(0xffffffffu, need_o)) {
                    tc_fence_after();
                    float o[32];
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        tmem_ld_32x32b_x32(tO + uint32_t(c * 32), o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= f_o;
                        tmem_st_32x32b_x32(tO + uint32_t(c * 32), o);
                    }
                    tmem_st_wait();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(my_p_full);
            }
            // every warp of the tile reaches both named barriers below exactly once, aborted or not
            if (ok)
                ok = mbar_wait(&my_pv[(nb - 1) & 1], uint32_t((nb - 1) >> 1) & 1u, abort_flag, a.status,
                               kErrTimeoutEpilogue);
            // (m, l) of half 1 go through its own P panel of the last block, dead once its P V is done
            float2* ml = reinterpret_cast<float2*>(smem + kFaP + ((t * 2 + ((nb - 1) & 1)) * 2 + 1) * kFaTile) + row;
            if (h == 1) *ml = make_float2(m_used, l);
            const uint32_t tile_threads = 64u * uint32_t(vw[t]);
            named_bar_sync(1 + t, tile_threads);
            if (ok && h == 0) {
                tc_fence_after();
                const float2 o1 = *ml;
                const float m = fmaxf(m_used, o1.x);
                const float f0 = ex2_approx(m_used - m), f1 = ex2_approx(o1.x - m);
                const float inv = 1.f / (l * f0 + o1.y * f1);
                const float g0 = f0 * inv, g1 = f1 * inv;
                uint8_t* orow = smem + kFaQ + t * kFaTile + row * 128;  // Q tile is dead: stage O there
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float o0[32], o1v[32];
                    tmem_ld_32x32b_x32(tO + uint32_t(c * 32), o0);
                    tmem_ld_32x32b_x32(tO + 64u + uint32_t(c * 32), o1v);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float r[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) r[e] = o0[8 * q + e] * g0 + o1v[8 * q + e] * g1;
                        uint4 v;
                        v.x = CtTraits<CT>::pack2(r[0], r[1]);
                        v.y = CtTraits<CT>::pack2(r[2], r[3]);
                        v.z = CtTraits<CT>::pack2(r[4], r[5]);
                        v.w = CtTraits<CT>::pack2(r[6], r[7]);
                        *reinterpret_cast<uint4*>(orow + ((uint32_t(c * 4 + q) ^ sw) << 4)) = v;
                    }
                }
                fence_proxy_async_smem();
            }
            named_bar_sync(1 + t, tile_threads);
            if (h == 0 && wq == 0 && lane == 0 && *abort_flag == 0) {
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
