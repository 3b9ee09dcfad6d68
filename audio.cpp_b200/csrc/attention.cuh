// Flash attention for head_dim 64: O = softmax(Q K^T / 8) V per (sequence, head),
// online softmax in fp32, Q/K/V/O in the GEMM operand type (fp16 or bf16).
// Replaces ggml_flash_attn_ext as used by rf_attention
// (src/models/stable_audio/foundation/rf_dit.cpp:175-198) for both the DiT
// self-attention (L = 1025) and the T5 cross-attention (L_k = 130, KV heads
// repeated: query head h reads KV head h / kv_rep, rf_dit.cpp:113-130).
//
// CTA = 4 warps x MT x 16 queries (MT = 1 or 2; two tiles per warp share each K/V fragment); K/V streamed in 64-key blocks through a
// cp.async double buffer; S = Q K^T and O += P V on mma.sync m16n8k16 with
// fp32 accumulators (operands fetched with ldmatrix; V with .trans).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace b2d {

constexpr int kAttnD = 64;        // head dim
constexpr int kAttnWarps = 4;     // warps per CTA; each owns MT x 16 query rows
constexpr int kAttnKeys = 64;     // keys per block
constexpr int kAttnPitch = 72;    // smem row pitch in elements (144 B: ldmatrix conflict-free)

template <typename CT>
struct MmaOp;
template <>
struct MmaOp<__half> {
    __device__ static __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    __device__ static __forceinline__ uint32_t pack(float x, float y) {
        __half2 h = __floats2half2_rn(x, y);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <>
struct MmaOp<__nv_bfloat16> {
    __device__ static __forceinline__ void run(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    __device__ static __forceinline__ uint32_t pack(float x, float y) {
        __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

// 16-byte async copy; src_bytes = 0 zero-fills (rows past the end).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Loads a [64 rows x 64] tile (rows >= valid are zero) into smem with pitch kAttnPitch.
template <typename CT>
__device__ __forceinline__ void load_tile(CT* dst, const CT* src, int64_t row_stride, int valid, int rows = 64) {
    for (int i = threadIdx.x; i < rows * 8; i += blockDim.x) {
        const int r = i >> 3, c = (i & 7) * 8;
        const bool ok = r < valid;
        cp_async16(dst + r * kAttnPitch + c, ok ? src + int64_t(r) * row_stride + c : src, ok ? 16 : 0);
    }
}

struct AttnArgs {
    const void* q;
    int64_t q_row, q_seq;    // element strides: token row, sequence
    const void* k;
    const void* v;
    int64_t kv_row, kv_seq;
    void* o;
    int64_t o_row, o_seq;
    int lq, lk;
    int kv_rep;              // query head h reads KV head h / kv_rep
    float scale_log2;        // softmax scale * log2(e)
};

constexpr size_t attn_smem_bytes(int mt) { return size_t(kAttnWarps * 16 * mt + 4 * kAttnKeys) * kAttnPitch * 2; }

template <typename CT, int MT>
__global__ void __launch_bounds__(128) flash_attn_kernel(AttnArgs a) {
    constexpr int ROWS = kAttnWarps * 16 * MT;  // queries per CTA
    extern __shared__ __align__(128) uint8_t attn_smem[];  // attn_smem_bytes(MT)
    CT* sq = reinterpret_cast<CT*>(attn_smem);
    CT* sk[2] = {sq + ROWS * kAttnPitch, sq + (ROWS + kAttnKeys) * kAttnPitch};
    CT* sv[2] = {sq + (ROWS + 2 * kAttnKeys) * kAttnPitch, sq + (ROWS + 3 * kAttnKeys) * kAttnPitch};

    const int q0 = blockIdx.x * ROWS;
    const int head = blockIdx.y;
    const int seq = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;

    const CT* qb = static_cast<const CT*>(a.q) + seq * a.q_seq + int64_t(q0) * a.q_row + head * kAttnD;
    const int kvh = head / a.kv_rep;
    const CT* kb = static_cast<const CT*>(a.k) + seq * a.kv_seq + kvh * kAttnD;
    const CT* vb = static_cast<const CT*>(a.v) + seq * a.kv_seq + kvh * kAttnD;

    load_tile(sq, qb, a.q_row, a.lq - q0, ROWS);
    load_tile(sk[0], kb, a.kv_row, a.lk);
    load_tile(sv[0], vb, a.kv_row, a.lk);
    cp_async_commit();

    uint32_t qf[MT][4][4];  // A fragments of this warp's MT x 16 query rows, 4 chunks of 16 dims
    float o[MT][8][4];
    float mrow[MT][2], lrow[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[mt][i][0] = o[mt][i][1] = o[mt][i][2] = o[mt][i][3] = 0.f;
        mrow[mt][0] = mrow[mt][1] = -INFINITY;
        lrow[mt][0] = lrow[mt][1] = 0.f;
    }

    const int nblk = (a.lk + kAttnKeys - 1) / kAttnKeys;
    for (int j = 0; j < nblk; ++j) {
        const int buf = j & 1;
        if (j + 1 < nblk) {
            const int k1 = (j + 1) * kAttnKeys;
            load_tile(sk[buf ^ 1], kb + int64_t(k1) * a.kv_row, a.kv_row, a.lk - k1);
            load_tile(sv[buf ^ 1], vb + int64_t(k1) * a.kv_row, a.kv_row, a.lk - k1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (j == 0) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int kc = 0; kc < 4; ++kc) {
                    const int r = (warp * MT + mt) * 16 + (lane & 15);
                    const int c = kc * 16 + (lane >> 4) * 8;
                    ldsm_x4(qf[mt][kc], sq + r * kAttnPitch + c);
                }
        }
        // S = Q K^T for 64 keys: 8 blocks of 8 keys
        float s[MT][8][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int i = 0; i < 8; ++i) s[mt][i][0] = s[mt][i][1] = s[mt][i][2] = s[mt][i][3] = 0.f;
        const CT* skb = sk[buf];
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
            for (int nb = 0; nb < 8; nb += 2) {
                uint32_t b[4];
                const int r = nb * 8 + (lane >> 4) * 8 + (lane & 7);
                const int c = kc * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(b, skb + r * kAttnPitch + c);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    MmaOp<CT>::run(s[mt][nb], qf[mt][kc], b[0], b[1]);
                    MmaOp<CT>::run(s[mt][nb + 1], qf[mt][kc], b[2], b[3]);
                }
            }
        }
        // mask keys past the end, online softmax (rows g and g + 8 of each 16-row tile)
        const int kbase = j * kAttnKeys;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            float mx0 = mrow[mt][0], mx1 = mrow[mt][1];
#pragma unroll
            for (int nb = 0; nb < 8; ++nb) {
                const int key = kbase + nb * 8 + 2 * t;
                if (key >= a.lk) s[mt][nb][0] = s[mt][nb][2] = -INFINITY;
                if (key + 1 >= a.lk) s[mt][nb][1] = s[mt][nb][3] = -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(s[mt][nb][0], s[mt][nb][1]));
                mx1 = fmaxf(mx1, fmaxf(s[mt][nb][2], s[mt][nb][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float al0 = exp2f((mrow[mt][0] - mx0) * a.scale_log2);
            const float al1 = exp2f((mrow[mt][1] - mx1) * a.scale_log2);
            mrow[mt][0] = mx0;
            mrow[mt][1] = mx1;
            const float ms0 = mx0 * a.scale_log2, ms1 = mx1 * a.scale_log2;
            float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
            for (int nb = 0; nb < 8; ++nb) {
                s[mt][nb][0] = exp2f(s[mt][nb][0] * a.scale_log2 - ms0);
                s[mt][nb][1] = exp2f(s[mt][nb][1] * a.scale_log2 - ms0);
                s[mt][nb][2] = exp2f(s[mt][nb][2] * a.scale_log2 - ms1);
                s[mt][nb][3] = exp2f(s[mt][nb][3] * a.scale_log2 - ms1);
                rs0 += s[mt][nb][0] + s[mt][nb][1];
                rs1 += s[mt][nb][2] + s[mt][nb][3];
            }
            lrow[mt][0] = lrow[mt][0] * al0 + rs0;
            lrow[mt][1] = lrow[mt][1] * al1 + rs1;
#pragma unroll
            for (int db = 0; db < 8; ++db) {
                o[mt][db][0] *= al0;
                o[mt][db][1] *= al0;
                o[mt][db][2] *= al1;
                o[mt][db][3] *= al1;
            }
        }
        // O += P V: 4 chunks of 16 keys
        const CT* svb = sv[buf];
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
            uint32_t pa[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                pa[mt][0] = MmaOp<CT>::pack(s[mt][2 * kc][0], s[mt][2 * kc][1]);
                pa[mt][1] = MmaOp<CT>::pack(s[mt][2 * kc][2], s[mt][2 * kc][3]);
                pa[mt][2] = MmaOp<CT>::pack(s[mt][2 * kc + 1][0], s[mt][2 * kc + 1][1]);
                pa[mt][3] = MmaOp<CT>::pack(s[mt][2 * kc + 1][2], s[mt][2 * kc + 1][3]);
            }
#pragma unroll
            for (int db = 0; db < 8; db += 2) {
                uint32_t b[4];
                const int r = kc * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
                const int c = db * 8 + (lane >> 4) * 8;
                ldsm_x4_t(b, svb + r * kAttnPitch + c);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    MmaOp<CT>::run(o[mt][db], pa[mt], b[0], b[1]);
                    MmaOp<CT>::run(o[mt][db + 1], pa[mt], b[2], b[3]);
                }
            }
        }
        __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
    }
    // row sums across the quad, normalise, store
    CT* ob = static_cast<CT*>(a.o) + seq * a.o_seq + head * kAttnD;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        float l0 = lrow[mt][0], l1 = lrow[mt][1];
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        const float inv0 = 1.f / l0, inv1 = 1.f / l1;
        const int r0 = q0 + (warp * MT + mt) * 16 + g, r1 = r0 + 8;
#pragma unroll
        for (int db = 0; db < 8; ++db) {
            const int c = db * 8 + 2 * t;
            if (r0 < a.lq)
                *reinterpret_cast<uint32_t*>(ob + int64_t(r0) * a.o_row + c) =
                    MmaOp<CT>::pack(o[mt][db][0] * inv0, o[mt][db][1] * inv0);
            if (r1 < a.lq)
                *reinterpret_cast<uint32_t*>(ob + int64_t(r1) * a.o_row + c) =
                    MmaOp<CT>::pack(o[mt][db][2] * inv1, o[mt][db][3] * inv1);
        }
    }
}

}  // namespace b2d
