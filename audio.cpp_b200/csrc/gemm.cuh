// Persistent warp-specialised tcgen05 GEMM for sm_100a:  C = A * B^T
//   A: activations [M, K], K contiguous (fp16 or bf16)
//   B: weights     [N, K], K contiguous (the ggml [out, in] layout), same type as A
// with fp32 accumulation in TMEM and a fused epilogue.  This is the dense
// contraction behind every ggml_mul_mat(W, X) on the diffusion hot path
// (LinearModule::build, src/framework/modules/linear_module.cpp:73-108).
//
// CTA = 6 warps: warp 0 issues TMA loads (128B-swizzled K-major tiles) into a
// STAGES-deep shared-memory ring; warp 1 owns TMEM and issues tcgen05.mma
// (M=128, N=BN, K=16 per instruction) from one lane; warps 2-5 drain the
// double-buffered TMEM accumulator (2 x BN fp32 columns) and run the epilogue
// while the next tile's MMAs proceed.  One CTA per SM, grid = min(tiles, SMs),
// tiles walk M fastest so CTAs running together share a weight slice in L2.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <type_traits>

#include "ptx.cuh"

namespace b2d {



enum EpiKind : int {
    EPI_F32 = 0,     // out_f32[r, n] = acc + bias[n]
    EPI_CT = 1,      // out_ct[r, n]  = ct(acc + bias[n])
    EPI_SWIGLU = 2,  // BN=256 tile = [128 "activated" | 128 "linear"] cols -> out_ct[r, n0/2 + j] = silu(a+ba) * (l+bl)
    EPI_RESID = 3,   // resid[r, n] += gate[r, n] * (acc + bias[n])   (gate == nullptr -> 1)
};

struct EpiParams {
    void* out = nullptr;
    int64_t ldo = 0;
    const float* bias = nullptr;
    float* resid = nullptr;
    int64_t ldr = 0;
    const float* gate = nullptr;
    int64_t ldg = 0;
    int gate_rows = 0;          // EPI_RESID: gate row = r / gate_rows (one gate row per sequence); 0: row r
    int* status = nullptr;
    int splits = 1;             // split-K factor (EPI_F32 only): split s writes out + s * split_stride
    int64_t split_stride = 0;
    int seg_rows = 0;           // EPI_F32 row remap: output row = r + (r / seg_rows + 1) * seg_pad
    int seg_pad = 0;
    // EPI_CT on a fused [q | k | v] projection: NEOX RoPE on dims [0, 32) of every 64-wide head in
    // columns < rope_cols (pairs j, j + 16), position = row % rope_L, tables [rope_L, 16];
    // columns >= rope_cols (V) are scaled by vmask[row].
    const float* rope_cos = nullptr;
    const float* rope_sin = nullptr;
    int rope_L = 0;
    int rope_cols = 0;
    const float* vmask = nullptr;
    // EPI_F32 through TMA stores (the kernel's tmO map: fp32 [M rows][N cols], box 32 x 32, 128B
    // swizzle); set by the launcher when there is no split-K and no row remap.
    int tma_out = 0;
    // EPI_RESID through TMA: the residual (tmO) and, when gate != nullptr, the gate (tmG) are loaded as
    // 32 x 32 fp32 boxes into a per-warp ring while the accumulator is still being computed, updated in
    // shared memory and written back by TMA stores; set by the launcher (no per-sequence gate rows,
    // 16-byte aligned bases and strides).
    int tma_resid = 0;
};

template <typename CT>
struct CtTraits;
template <>
struct CtTraits<__half> {
    static constexpr uint32_t kFmt = 0;
    __device__ static __forceinline__ __half cvt(float a) { return __float2half_rn(a); }
    __device__ static __forceinline__ uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <>
struct CtTraits<__nv_bfloat16> {
    static constexpr uint32_t kFmt = 1;
    __device__ static __forceinline__ __nv_bfloat16 cvt(float a) { return __float2bfloat16_rn(a); }
    __device__ static __forceinline__ uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// SiLU with the hardware exp2 and fast reciprocal-division intrinsics (a few ulp; the result is
// rounded to fp16/bf16 or consumed by an fp32 accumulation downstream).
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Residual epilogue staging: per epilogue warp four 4 KB boxes (a ring of 4 residual boxes, or of 2
// residual + gate pairs) and, after all warps' boxes, 4 mbarriers per warp.
constexpr uint32_t kResidBoxBytes = 4096;
constexpr uint32_t kResidWarpBytes = 4 * kResidBoxBytes;
constexpr size_t kResidStageBytes = 4 * kResidWarpBytes + 4 * 4 * 8;

template <int BN, int EPI = -1>
struct GemmShape {
    static constexpr int BM = 128;
    static constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr bool RESID_TMA = EPI == EPI_RESID;
    // operand ring depth: as deep as fits next to the epilogue staging, at most 8
    static constexpr int STAGES_FIT = int((232448 - 1024 - 256 - (RESID_TMA ? kResidStageBytes : 0)) /
                                          STAGE_BYTES);
    static constexpr int STAGES_DEF = BN >= 192 ? (BN == 192 ? 5 : 4) : (BN >= 128 ? 6 : 8);
    static constexpr int STAGES = RESID_TMA ? (STAGES_FIT < 6 ? STAGES_FIT : 6) : STAGES_DEF;
    static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;  // power of two
    // Epilogue staging right after the operand ring (1024-aligned): per warp either a 32 x 33 fp32
    // transpose buffer or, for the TMA-store fp32 path, two 128B-swizzled 32 x 32 fp32 boxes; for the
    // residual epilogue the TMA box ring (which also holds the fallback path's transpose buffers).
    static constexpr bool TMA_F32_OUT = BN != 192;  // the two 4 KB boxes per warp fit next to the ring
    static constexpr size_t EPI_STAGE_BYTES = RESID_TMA ? kResidStageBytes
                                                        : (TMA_F32_OUT ? 4 * 2 * 4096 : 4 * 32 * 33 * 4);
    static constexpr size_t SMEM_BYTES = size_t(STAGES) * STAGE_BYTES + EPI_STAGE_BYTES + 256 + 1024;
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// Residual epilogue over all of this warp's units: x[r, n] += g[r, n] * (acc + bias[n]) on the fp32
// residual stream, 32 x 32 boxes through TMA.  The warp keeps up to 4 (2 with a gate) box loads in flight
// ahead of the chunk it is updating, including the next unit's first chunks, so the residual / gate reads
// overlap the MMA main loop instead of following it.  Returns false when a wait gave up.
// Units: u = first, first + stride, ... < num_units; unit u covers rows (t % m_tiles) * m_step + row_off and
// columns (t / m_tiles) * BN, t = u % num_tiles (1-SM tiles: m_step 128, row_off 0; 2-SM pair tiles: m_step
// 256, row_off = 128 x the CTA's rank).  The accumulator goes back to the MMA warp on tempty[acc], or on the
// leader CTA's barrier tempty_remote[acc] (a cluster address) for pair tiles.
template <int BN>
__device__ __forceinline__ bool resid_tma_epilogue(uint32_t tmem_base, int quarter, int lane, uint8_t* boxes,
                                                   uint64_t* bars, const CUtensorMap* tmR, const CUtensorMap* tmG,
                                                   const EpiParams& ep, int m_tiles, int num_tiles, int num_units,
                                                   uint64_t* tfull, uint64_t* tempty, volatile int* abort_flag,
                                                   int first, int stride, int m_step, int row_off,
                                                   const uint32_t* tempty_remote) {
    constexpr int C = BN / 32;
    const bool has_gate = ep.gate != nullptr;
    const uint32_t nb = has_gate ? 2u : 4u;
    const uint32_t slot_bytes = has_gate ? 2 * kResidBoxBytes : kResidBoxBytes;
    int lu = first, lc = 0;  // next box load: unit, chunk
    uint32_t ld_seq = 0, cs_seq = 0;
    auto issue_next = [&]() {
        if (lu >= num_units) return;
        const int tile = lu % num_tiles;
        const int m0 = (tile % m_tiles) * m_step + row_off, n0 = (tile / m_tiles) * BN;
        const uint32_t slot = ld_seq % nb;
        uint8_t* box = boxes + slot * slot_bytes;
        mbar_arrive_expect_tx(&bars[slot], slot_bytes);
        tma_load_2d(box, tmR, &bars[slot], n0 + lc * 32, m0 + quarter * 32);
        if (has_gate) tma_load_2d(box + kResidBoxBytes, tmG, &bars[slot], n0 + lc * 32, m0 + quarter * 32);
        ++ld_seq;
        if (++lc == C) {
            lc = 0;
            lu += stride;
        }
    };
    if (lane == 0)
        for (uint32_t i = 0; i < nb; ++i) issue_next();
    const uint32_t sw = uint32_t(lane & 7);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = first; u < num_units; u += stride) {
        const int tile = u % num_tiles;
        const int m0 = (tile % m_tiles) * m_step + row_off, n0 = (tile / m_tiles) * BN;
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ep.status, kErrTimeoutEpilogue)) return false;
        tc_fence_after();
        const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
        for (int c = 0; c < C; ++c) {
            float v[32];
            tmem_ld_32x32b_x32(tbase + uint32_t(c * 32), v);
            tmem_ld_wait();
            if (c == C - 1) {  // the accumulator is in registers: hand TMEM back to the MMA warp
                tc_fence_before();
                if (tempty_remote)
                    mbar_arrive_cluster(tempty_remote[acc]);
                else
                    mbar_arrive(&tempty[acc]);
            }
            if (ep.bias) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __ldg(ep.bias + n0 + c * 32 + j);
            }
            const uint32_t slot = cs_seq % nb;
            if (!mbar_wait(&bars[slot], (cs_seq / nb) & 1u, abort_flag, ep.status, kErrTimeoutEpilogue)) return false;
            uint8_t* rrow = boxes + slot * slot_bytes + lane * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4* rp = reinterpret_cast<float4*>(rrow + ((uint32_t(q) ^ sw) << 4));
                float4 r = *rp;
                if (has_gate) {
                    const float4 g = *reinterpret_cast<const float4*>(rrow + kResidBoxBytes + ((uint32_t(q) ^ sw) << 4));
                    r.x += g.x * v[4 * q];
                    r.y += g.y * v[4 * q + 1];
                    r.z += g.z * v[4 * q + 2];
                    r.w += g.w * v[4 * q + 3];
                } else {
                    r.x += v[4 * q];
                    r.y += v[4 * q + 1];
                    r.z += v[4 * q + 2];
                    r.w += v[4 * q + 3];
                }
                *rp = r;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(tmR, boxes + slot * slot_bytes, n0 + c * 32, m0 + quarter * 32);
                bulk_commit_group();
                bulk_wait_read_all();  // the store has read the box: its slot takes the next load
                issue_next();
            }
            __syncwarp();
            ++cs_seq;
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    return true;
}

// Drains one 128-row accumulator tile (this warp's 32 TMEM lanes at `tbase`) through the epilogue.
template <int BN, int EPI, typename CT>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, int rbase, int rows_live, int n0, float* out_f32,
                                              const EpiParams& ep, float* stg, int lane,
                                              const CUtensorMap* tmO = nullptr) {
    constexpr int CHUNKS = EPI == EPI_SWIGLU ? 4 : BN / 32;
    if constexpr (EPI == EPI_F32 && GemmShape<BN>::TMA_F32_OUT) {
        if (ep.tma_out) {
            // thread = row: its 32 columns go into a 128B-swizzled 32 x 32 box (conflict-free
            // 16 B stores), one lane writes the box with a single TMA store (rows >= M clipped);
            // two boxes per warp so the next chunk fills one while the other drains.
            uint8_t* box0 = reinterpret_cast<uint8_t*>(stg);
            const uint32_t sw = uint32_t(lane & 7);
#pragma unroll 1
            for (int c = 0; c < CHUNKS; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(tbase + uint32_t(c * 32), v);
                tmem_ld_wait();
                if (ep.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += __ldg(ep.bias + n0 + c * 32 + j);
                }
                uint8_t* box = box0 + (c & 1) * 4096;
                // the store issued two chunks ago read this box
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<float4*>(box + lane * 128 + ((uint32_t(q) ^ sw) << 4)) =
                        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                                     reinterpret_cast<uint64_t>(tmO)),
                                 "r"(smem_u32(box)), "r"(n0 + c * 32), "r"(rbase)
                                 : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
            return;
        }
    }
#pragma unroll 1
        for (int c = 0; c < CHUNKS; ++c) {
            float v[32];
            __syncwarp();
            if constexpr (EPI == EPI_SWIGLU) {
                float l[32];
                tmem_ld_32x32b_x32(tbase + uint32_t(c * 32), v);
                tmem_ld_32x32b_x32(tbase + uint32_t(128 + c * 32), l);
                tmem_ld_wait();
                const float* ba = ep.bias ? ep.bias + n0 + c * 32 : nullptr;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float av = ba ? v[j] + __ldg(ba + j) : v[j];
                    const float lv = ba ? l[j] + __ldg(ba + 128 + j) : l[j];
                    v[j] = silu_f(av) * lv;
                }
            } else {
                tmem_ld_32x32b_x32(tbase + uint32_t(c * 32), v);
                tmem_ld_wait();
            }
            if constexpr (EPI == EPI_SWIGLU || EPI == EPI_CT) {
                // 16-bit outputs: each thread stores its row's 32 values as 4 x 16 B (no smem
                // traffic, which would compete with the next tile's tcgen05 operand reads).
                const int row = rbase + lane;
                if (lane < rows_live) {
                    const int col0 = (EPI == EPI_SWIGLU ? n0 / 2 : n0) + c * 32;
                    if (EPI == EPI_CT && ep.rope_cos) {
                        if (col0 < ep.rope_cols) {
                            if ((col0 & 63) == 0) {
                                const int pos = row % ep.rope_L;
                                const float* cs = ep.rope_cos + pos * 16;
                                const float* sn = ep.rope_sin + pos * 16;
#pragma unroll
                                for (int j = 0; j < 16; ++j) {
                                    const float x0 = v[j], x1 = v[j + 16], cj = __ldg(cs + j), sj = __ldg(sn + j);
                                    v[j] = x0 * cj - x1 * sj;
                                    v[j + 16] = x0 * sj + x1 * cj;
                                }
                            }
                        } else if (ep.vmask) {
                            const float mv = __ldg(ep.vmask + row);
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] *= mv;
                        }
                    }
                    if (EPI == EPI_CT && ep.bias) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] += __ldg(ep.bias + col0 + j);
                    }
                    uint32_t packed[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) packed[j] = CtTraits<CT>::pack2(v[2 * j], v[2 * j + 1]);
                    uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<CT*>(ep.out) + int64_t(row) * ep.ldo + col0);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
                }
                continue;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = v[j];
            __syncwarp();
            const int col = (EPI == EPI_SWIGLU ? n0 / 2 : n0) + c * 32 + lane;
            const float bcol = (EPI != EPI_SWIGLU && ep.bias) ? __ldg(ep.bias + col) : 0.f;
            if constexpr (EPI == EPI_RESID) {
                float* __restrict__ R = ep.resid;
                const float* __restrict__ G = ep.gate;
#pragma unroll 1
                for (int r0 = 0; r0 < rows_live; r0 += 32) {
                    float rv[32], gv[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int64_t row = rbase + r0 + i;
                        const bool ok = r0 + i < rows_live;
                        rv[i] = ok ? R[row * ep.ldr + col] : 0.f;
                        gv[i] = (ok && G) ? G[(ep.gate_rows ? row / ep.gate_rows : row) * ep.ldg + col] : 1.f;
                    }
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (r0 + i < rows_live)
                            R[int64_t(rbase + r0 + i) * ep.ldr + col] = rv[i] + gv[i] * (stg[(r0 + i) * 33 + lane] + bcol);
                    }
                }
            } else {
#pragma unroll 4
                for (int r = 0; r < 32; ++r) {
                    if (r < rows_live) {
                        const float x = stg[r * 33 + lane] + bcol;
                        int64_t row = rbase + r;
                        if constexpr (EPI == EPI_F32) {
                            if (ep.seg_rows) row += (row / ep.seg_rows + 1) * ep.seg_pad;
                            out_f32[row * ep.ldo + col] = x;
                        } else {
                            reinterpret_cast<CT*>(ep.out)[row * ep.ldo + col] = CtTraits<CT>::cvt(x);
                        }
                    }
                }
            }
        }
}

template <int BN, int EPI, typename CT>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmG, int M, int N,
                   int K, EpiParams ep) {
    using S = GemmShape<BN, EPI>;
    constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES;
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert(EPI != EPI_SWIGLU || BN == 256, "SwiGLU tiles pair 128 + 128 columns");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * S::STAGE_BYTES + S::EPI_STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM;
    const int num_tiles = m_tiles * (N / BN);
    // Work unit u = (tile, split): split-K partitions the K blocks into `splits` equal ranges.
    const int splits = ep.splits > 1 ? ep.splits : 1;
    const int num_units = num_tiles * splits;
    const int k_blocks = K / BK / splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
        }
        if constexpr (S::RESID_TMA) {
            uint64_t* rb = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * S::STAGE_BYTES + 4 * kResidWarpBytes);
            for (int i = 0; i < 16; ++i) mbar_init(&rb[i], 1);
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
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            int stage = 0;
            uint32_t phase = 0;
            for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
                const int tile = u % num_tiles;
                const int kb0 = (u / num_tiles) * k_blocks;
                const int m0 = (tile % m_tiles) * BM;
                const int n0 = (tile / m_tiles) * BN;
                // Each tile starts its K walk at its own offset: CTAs that share an A row block
                // or a B column block then fetch different K slices at any moment instead of all
                // hitting the same L2 lines (the accumulation order is fixed per tile).
                const int rot = ((tile % m_tiles) * 5 + (tile / m_tiles) * 3) % k_blocks;
                for (int i = 0; i < k_blocks; ++i) {
                    const int kb = kb0 + (rot + i < k_blocks ? rot + i : rot + i - k_blocks);
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, ep.status, kErrTimeoutProducer)) goto done;
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], S::STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
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
            for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, ep.status, kErrTimeoutMma)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, ep.status, kErrTimeoutMma)) goto done;
                    tc_fence_after();
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    const uint64_t adesc = smem_desc_sw128(sa);
                    const uint64_t bdesc = smem_desc_sw128(sa + S::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        // +32 bytes along K inside the 128-byte swizzle row == +2 in the >>4 address field
                        mma_f16_ss(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                   (kb | k) != 0 ? 1u : 0u);  // kb counts within this unit's K range
                    }
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
        // Epilogue: TMEM -> registers (thread = row).  fp32 and residual outputs then go
        // through a padded shared-memory transpose (32 x 33 floats per warp) so each warp
        // instruction reads/writes one contiguous 32-column row segment (coalesced, and the
        // residual read-modify-write issues all 32 rows' loads before any store instead of serialising).
        const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32) belong to this warp
        pdl_wait();
        if constexpr (S::RESID_TMA) {
            if (ep.tma_resid) {
                uint8_t* epi = smem + size_t(STAGES) * S::STAGE_BYTES;
                resid_tma_epilogue<BN>(tmem_base, quarter, lane, epi + quarter * kResidWarpBytes,
                                       reinterpret_cast<uint64_t*>(epi + 4 * kResidWarpBytes) + quarter * 4, &tmO,
                                       &tmG, ep, m_tiles, num_tiles, num_units, tfull, tempty, abort_flag,
                                       int(blockIdx.x), int(gridDim.x), BM, 0, nullptr);
                goto done;
            }
        }
        float* stg = reinterpret_cast<float*>(smem + size_t(STAGES) * S::STAGE_BYTES +
                                              quarter * (S::RESID_TMA ? kResidWarpBytes : S::EPI_STAGE_BYTES / 4));
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
            const int tile = u % num_tiles;
            float* out_f32 = reinterpret_cast<float*>(ep.out) + int64_t(u / num_tiles) * ep.split_stride;
            const int m0 = (tile % m_tiles) * BM;
            const int n0 = (tile / m_tiles) * BN;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ep.status, kErrTimeoutEpilogue)) goto done;
            tc_fence_after();
            const int rbase = m0 + quarter * 32;
            const int rows_live = M - rbase < 32 ? M - rbase : 32;
            const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
            epilogue_tile<BN, EPI, CT>(tbase, rbase, rows_live, n0, out_f32, ep, stg, lane, &tmO);
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

// 2-SM variant: a cluster of 2 CTAs computes a 256 x BN tile (BN = 256 or 192) with
// tcgen05.mma.cta_group::2 (M = 256 split across the pair's TMEM).  Each CTA loads its own 128
// rows of A and its own BN / 2 rows (half) of B, so per SM the operand traffic per FLOP is 2/3
// (BN 256) or 0.73 (BN 192) of the single-CTA 128 x BN tile -- these GEMMs are bounded by the
// L2 -> SM operand stream, not by the tensor pipe.  The leader CTA (rank 0) issues the MMAs; TMA completion of
// both halves is counted on the leader's full barrier; commits multicast to both CTAs'
// empty / tmem-full barriers; both epilogues release the accumulator on the leader's
// tmem-empty barrier.  No TMA multicast is used.
template <int BN_, int EPI = -1>
struct GemmPairShape {
    static constexpr int BM = 128;  // rows per CTA (256 per pair)
    static constexpr int BN = BN_;  // columns per pair tile (BN / 2 rows of B per CTA): 192 or 256
    static constexpr int BK = 64;
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    // residual epilogue: the TMA box ring (1024-aligned, after the barrier block) next to a shorter operand ring
    static constexpr bool RESID_TMA = EPI == EPI_RESID;
    static constexpr int STAGES_FIT = int((232448 - 2048 - kResidStageBytes) / STAGE_BYTES);
    static constexpr int STAGES = RESID_TMA ? (STAGES_FIT < 6 ? STAGES_FIT : 6) : (BN == 256 ? 6 : 7);
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr size_t EPI_BYTES = RESID_TMA ? 1024 + kResidStageBytes : 256 + 4 * 32 * 33 * 4;
    static constexpr size_t SMEM_BYTES = size_t(STAGES) * STAGE_BYTES + 1024 + EPI_BYTES;
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <int BN_, int EPI, typename CT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmG, int M, int N,
                    int K, EpiParams ep) {
    using S = GemmPairShape<BN_, EPI>;
    constexpr int BM = S::BM, BN = S::BN, BK = S::BK, STAGES = S::STAGES;

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
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pm = (M + 2 * BM - 1) / (2 * BM);  // 256-row pair tiles
    const int num_units = pm * (N / BN);
    const int k_blocks = K / BK;
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 256);
        }
        if constexpr (S::RESID_TMA) {
            uint64_t* rb = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * S::STAGE_BYTES + 1024 +
                                                       4 * kResidWarpBytes);
            for (int i = 0; i < 16; ++i) mbar_init(&rb[i], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            int stage = 0;
            uint32_t phase = 0;
            for (int u = cluster; u < num_units; u += nclusters) {
                const int m0 = (u % pm) * 2 * BM + int(rank) * BM;
                const int n0 = (u / pm) * BN + int(rank) * (BN / 2);
                const int rot = ((u % pm) * 5 + (u / pm) * 3) % k_blocks;  // staggered K walk (see above)
                for (int i = 0; i < k_blocks; ++i) {
                    const int kb = rot + i < k_blocks ? rot + i : rot + i - k_blocks;
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, ep.status, kErrTimeoutProducer)) goto done;
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::STAGE_BYTES);
                    const uint32_t bar = map_to_cta(smem_u32(&full[stage]), 0);
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    tma_load_2d_pair(sa, &tmA, bar, kb * BK, m0);
                    tma_load_2d_pair(sa + S::A_BYTES, &tmB, bar, kb * BK, n0);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_f16(CtTraits<CT>::kFmt, 2 * BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int u = cluster; u < num_units; u += nclusters) {
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, ep.status, kErrTimeoutMma)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, ep.status, kErrTimeoutMma)) goto done;
                    tc_fence_after();
                    uint8_t* sa = smem + size_t(stage) * S::STAGE_BYTES;
                    const uint64_t adesc = smem_desc_sw128(sa);
                    const uint64_t bdesc = smem_desc_sw128(sa + S::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16_pair(d_tmem, adesc + uint64_t(2 * k), bdesc + uint64_t(2 * k), idesc,
                                     (kb | k) != 0 ? 1u : 0u);
                    mma_commit_pair(&empty[stage], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                mma_commit_pair(&tfull[acc], 0x3);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    } else {
        const int quarter = warp & 3;
        uint8_t* epi = smem + size_t(STAGES) * S::STAGE_BYTES + (S::RESID_TMA ? 1024 : 256);
        float* stg = reinterpret_cast<float*>(epi) + quarter * (S::RESID_TMA ? kResidWarpBytes / 4 : 32 * 33);
        const uint32_t tempty_leader[2] = {map_to_cta(smem_u32(&tempty[0]), 0), map_to_cta(smem_u32(&tempty[1]), 0)};
        pdl_wait();
        if constexpr (S::RESID_TMA) {
            if (ep.tma_resid) {
                resid_tma_epilogue<BN>(tmem_base, quarter, lane, epi + quarter * kResidWarpBytes,
                                       reinterpret_cast<uint64_t*>(epi + 4 * kResidWarpBytes) + quarter * 4, &tmO,
                                       &tmG, ep, pm, num_units, num_units, tfull, tempty, abort_flag, cluster,
                                       nclusters, 2 * BM, int(rank) * BM, tempty_leader);
                goto done;
            }
        }
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int u = cluster; u < num_units; u += nclusters) {
            const int n0 = (u / pm) * BN;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ep.status, kErrTimeoutEpilogue)) goto done;
            tc_fence_after();
            const int rbase = (u % pm) * 2 * BM + int(rank) * BM + quarter * 32;
            const int rows_live = M - rbase < 32 ? M - rbase : 32;
            const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
            epilogue_tile<BN, EPI, CT>(tbase, rbase, rows_live, n0, reinterpret_cast<float*>(ep.out), ep, stg, lane);
            tc_fence_before();
            mbar_arrive_cluster(tempty_leader[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
    }
}

}  // namespace b2d
