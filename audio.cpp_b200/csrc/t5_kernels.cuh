// Kernels of the Stable Audio Open 1.0 conditioner (src/models/stable_audio/foundation/conditioner.cpp and
// src/framework/modules/text_encoders/t5_base_encoder.cpp) that are not GEMMs: the token-embedding gather,
// T5 self-attention over one prompt (no 1/sqrt(d) scale, bucketed relative-position bias, additive padding
// mask), ReLU on the FFN activation, the seconds number embeddings and the cross / global assembly.
#pragma once

#include "kernels.cuh"

namespace b2d {

// h[r, :] = E[ids[r], :]   (EmbeddingModule, lookup_modules.cpp:88-112)
__global__ void t5_embed_kernel(const int* __restrict__ ids, int64_t rows, int d, const float* __restrict__ table,
                                int vocab, float* __restrict__ h, int* __restrict__ status) {
    const int64_t total = rows * d;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / d;
        const int id = ids[r];
        if (id < 0 || id >= vocab) {
            atomicCAS(status, 0, kErrNonFinite);
            h[i] = 0.f;
            continue;
        }
        h[i] = table[int64_t(id) * d + i % d];
    }
}

// One (sequence, head): scores = q k^T + bias[head] + (mask[k] ? 0 : -1e9), softmax, context = P v.
// qkv fp32 [rows, 3 * H * hd] ([q | k | v] per row); K / V of the sequence staged in shared memory; one thread per
// query with an online (running max) softmax over the keys.  Output ct [rows, H * hd].
template <typename CT, int HD>
__global__ void __launch_bounds__(128) t5_attention_kernel(const float* __restrict__ qkv, int P, int H,
                                                           const float* __restrict__ bias,
                                                           const float* __restrict__ mask, CT* __restrict__ out) {
    extern __shared__ float kv_s[];  // [P][HD] keys then [P][HD] values
    const int head = blockIdx.x, seq = blockIdx.y;
    const int D = H * HD;
    const float* base = qkv + int64_t(seq) * P * 3 * D;
    float* ks = kv_s;
    float* vs = kv_s + P * HD;
    for (int i = threadIdx.x; i < P * HD; i += blockDim.x) {
        const int t = i / HD, j = i % HD;
        ks[i] = base[int64_t(t) * 3 * D + D + head * HD + j];
        vs[i] = base[int64_t(t) * 3 * D + 2 * D + head * HD + j];
    }
    __syncthreads();
    const float* mk = mask + int64_t(seq) * P;
    for (int q = threadIdx.x; q < P; q += blockDim.x) {
        float qv[HD], o[HD];
#pragma unroll
        for (int j = 0; j < HD; ++j) {
            qv[j] = base[int64_t(q) * 3 * D + head * HD + j];
            o[j] = 0.f;
        }
        const float* brow = bias + (int64_t(head) * P + q) * P;
        float m = -INFINITY, l = 0.f;
        for (int k = 0; k < P; ++k) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < HD; ++j) s += qv[j] * ks[k * HD + j];
            s += brow[k] + (mk[k] != 0.f ? 0.f : -1.0e9f);
            const float mn = fmaxf(m, s);
            const float corr = expf(m - mn), p = expf(s - mn);
            l = l * corr + p;
#pragma unroll
            for (int j = 0; j < HD; ++j) o[j] = o[j] * corr + p * vs[k * HD + j];
            m = mn;
        }
        const float inv = 1.f / l;
        CT* orow = out + (int64_t(seq) * P + q) * D + head * HD;
#pragma unroll
        for (int j = 0; j < HD; ++j) orow[j] = from_f32<CT>(o[j] * inv);
    }
}

template <typename CT>
__global__ void relu_ct_kernel(CT* __restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = to_f32(x[i]);
        x[i] = from_f32<CT>(v > 0.f ? v : 0.f);
    }
}

// number_embedding (conditioner.cpp:177-200) of seconds_start (which = 0, value 0) and seconds_total (which = 1)
// for prompt b: features [x, sin(2 pi x f_i), cos(2 pi x f_i)] (257), out = W features + bias, written into the
// prompt's cross row P + which and global half `which`.  One block per (which, prompt).
__global__ void t5_number_kernel(const float* __restrict__ seconds, const float* __restrict__ freqs,
                                 const float* __restrict__ w, const float* __restrict__ bvec, int d, int P,
                                 float* __restrict__ cross, float* __restrict__ global) {
    __shared__ float feat[257];
    const int which = blockIdx.x, b = blockIdx.y;
    const float x = which == 0 ? 0.f : seconds[b];
    const float* fr = freqs + which * 128;
    for (int i = threadIdx.x; i < 128; i += blockDim.x) {
        const float arg = x * fr[i] * 2.0f * 3.14159265358979323846f;
        feat[1 + i] = sinf(arg);
        feat[1 + 128 + i] = cosf(arg);
    }
    if (threadIdx.x == 0) feat[0] = x;
    __syncthreads();
    const float* W = w + int64_t(which) * d * 257;
    for (int o = threadIdx.x; o < d; o += blockDim.x) {
        float sum = bvec[which * d + o];
        for (int i = 0; i < 257; ++i) sum += W[int64_t(o) * 257 + i] * feat[i];
        cross[(int64_t(b) * (P + 2) + P + which) * d + o] = sum;
        global[int64_t(b) * 2 * d + which * d + o] = sum;
    }
}

// Cross tokens [B, P + 2, d]: the encoder states of kept tokens, zeros for padding (rows P, P + 1 written by
// t5_number_kernel); cross mask [B, P + 2] as 0 / 1 floats.
__global__ void t5_assemble_kernel(const float* __restrict__ states, const float* __restrict__ mask, int B, int P,
                                   int d, float* __restrict__ cross, float* __restrict__ cmask) {
    const int64_t total = int64_t(B) * P * d;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int o = int(i % d);
        const int64_t bt = i / d;
        const int b = int(bt / P), t = int(bt % P);
        const bool keep = mask[bt] != 0.f;
        cross[(int64_t(b) * (P + 2) + t) * d + o] = keep ? states[i] : 0.f;
        if (o == 0) {
            cmask[int64_t(b) * (P + 2) + t] = keep ? 1.f : 0.f;
            if (t == 0) {
                cmask[int64_t(b) * (P + 2) + P] = 1.f;
                cmask[int64_t(b) * (P + 2) + P + 1] = 1.f;
            }
        }
    }
}

}  // namespace b2d
