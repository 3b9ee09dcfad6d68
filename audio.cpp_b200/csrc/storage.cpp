// Weight storage-type selection and conversion on the host, at load time: the part of audio.cpp's weight
// store that decides in which ggml type a checkpoint tensor is kept and converts it (quantize-on-load).
//
//  * Resolution (BackendWeightStore::type_for_storable_loaded_tensor / backend_safe_loaded_storage_type,
//    include/engine/framework/core/backend_weight_store.h:237-290): Native keeps the checkpoint's own type;
//    any other request is taken as given, except that a quantized target falls back to F32 for tensors of
//    rank < 2 or whose last dimension is not a multiple of the 32-element block.
//  * Conversion (src/framework/assets/tensor_source.cpp:150-200): the stored values are decoded to fp32
//    and re-encoded -- F16 with round-to-nearest-even (ggml_fp32_to_fp16_row), BF16 with ggml's rounding
//    (round-to-nearest-even, NaNs kept quiet), Q8_0 as quantize_row_q8_0_ref (ggml-quants.c): per 32-block
//    d = amax / 127, q = roundf(x / d) (half away from zero), d stored as fp16.
// The arithmetic is restated here in this library's own code; tests pin it to the reference's bytes.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/b200diff.h"

namespace {

float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            exp = 127 - 15 + 1;
            while (!(man & 0x400u)) {
                man <<= 1;
                --exp;
            }
            man &= 0x3ffu;
            bits = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// fp32 -> fp16, round to nearest even; overflow to infinity; NaN stays NaN.
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint16_t sign = uint16_t((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return uint16_t(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0));
    if (ax >= 0x477ff000u) return uint16_t(sign | 0x7c00u);  // rounds to >= 65520: infinity
    if (ax < 0x38800000u) {                                  // below the smallest normal half: subnormal or zero
        if (ax < 0x33000000u) return sign;                   // < 2^-25 rounds to zero (2^-25 itself ties to 0)
        const uint32_t e = ax >> 23;                         // 102 .. 112
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;                      // 14 .. 24: value = m * 2^(e - 150)
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return uint16_t(sign | h);
    }
    uint32_t h = ((ax >> 13) - ((127u - 15u) << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return uint16_t(sign | h);
}

uint16_t f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 64u);  // quiet NaN
    return uint16_t((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

int64_t elements(const int64_t* dims, int32_t ndim) {
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= dims[i];
    return n;
}

bool decode(const b2d_tensor_view* t, std::vector<float>& out) {
    const int64_t n = elements(t->dims, t->ndim);
    out.resize(size_t(n));
    const uint8_t* p = static_cast<const uint8_t*>(t->data);
    switch (t->ggml_type) {
        case B2D_TYPE_F32:
            if (t->nbytes != size_t(n) * 4) return false;
            std::memcpy(out.data(), p, size_t(n) * 4);
            return true;
        case B2D_TYPE_F16:
            if (t->nbytes != size_t(n) * 2) return false;
            for (int64_t i = 0; i < n; ++i) out[size_t(i)] = f16_to_f32(uint16_t(p[2 * i] | (p[2 * i + 1] << 8)));
            return true;
        case B2D_TYPE_BF16:
            if (t->nbytes != size_t(n) * 2) return false;
            for (int64_t i = 0; i < n; ++i) {
                const uint32_t bits = uint32_t(p[2 * i] | (p[2 * i + 1] << 8)) << 16;
                std::memcpy(&out[size_t(i)], &bits, 4);
            }
            return true;
        case B2D_TYPE_Q8_0: {
            if (n % 32 || t->nbytes != size_t(n / 32) * 34) return false;
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * 34;
                const float d = f16_to_f32(uint16_t(blk[0] | (blk[1] << 8)));
                for (int j = 0; j < 32; ++j) out[size_t(b * 32 + j)] = float(int8_t(blk[2 + j])) * d;
            }
            return true;
        }
        default:
            return false;
    }
}

}  // namespace

extern "C" {

B2D_API int32_t b2d_storage_resolve(int32_t storage_type, const b2d_tensor_view* t) {
    if (!t) return -1;
    int32_t type;
    switch (storage_type) {
        case B2D_STORAGE_NATIVE: return t->ggml_type;
        case B2D_STORAGE_F32: type = B2D_TYPE_F32; break;
        case B2D_STORAGE_F16: type = B2D_TYPE_F16; break;
        case B2D_STORAGE_BF16: type = B2D_TYPE_BF16; break;
        case B2D_STORAGE_Q8_0: type = B2D_TYPE_Q8_0; break;
        default: return -1;  // the K-quant / Q4 / Q5 storage types are not on this path
    }
    if (type == B2D_TYPE_Q8_0 && (t->ndim < 2 || t->dims[t->ndim - 1] % 32 != 0)) return B2D_TYPE_F32;
    return type;
}

B2D_API size_t b2d_tensor_bytes(int32_t ggml_type, const int64_t* dims, int32_t ndim) {
    if (!dims || ndim < 1 || ndim > 4) return 0;
    const int64_t n = elements(dims, ndim);
    switch (ggml_type) {
        case B2D_TYPE_F32: return size_t(n) * 4;
        case B2D_TYPE_F16:
        case B2D_TYPE_BF16: return size_t(n) * 2;
        case B2D_TYPE_Q8_0: return n % 32 ? 0 : size_t(n / 32) * 34;
        default: return 0;
    }
}

B2D_API b2d_status b2d_tensor_convert(const b2d_tensor_view* t, int32_t ggml_type, void* out, size_t out_bytes) {
    if (!t || !t->data || !out || t->ndim < 1 || t->ndim > 4) return B2D_EINVAL;
    const size_t need = b2d_tensor_bytes(ggml_type, t->dims, t->ndim);
    if (need == 0 || out_bytes != need) return B2D_EINVAL;
    if (ggml_type == B2D_TYPE_Q8_0 && (t->ndim < 2 || t->dims[t->ndim - 1] % 32 != 0)) return B2D_EINVAL;
    if (ggml_type == t->ggml_type) {  // same encoding: bytes unchanged
        if (t->nbytes != need) return B2D_EINVAL;
        std::memcpy(out, t->data, need);
        return B2D_OK;
    }
    std::vector<float> v;
    if (!decode(t, v)) return B2D_EINVAL;
    uint8_t* o = static_cast<uint8_t*>(out);
    const size_t n = v.size();
    switch (ggml_type) {
        case B2D_TYPE_F32:
            std::memcpy(o, v.data(), n * 4);
            break;
        case B2D_TYPE_F16:
            for (size_t i = 0; i < n; ++i) {
                const uint16_t h = f32_to_f16(v[i]);
                o[2 * i] = uint8_t(h & 0xff);
                o[2 * i + 1] = uint8_t(h >> 8);
            }
            break;
        case B2D_TYPE_BF16:
            for (size_t i = 0; i < n; ++i) {
                const uint16_t h = f32_to_bf16(v[i]);
                o[2 * i] = uint8_t(h & 0xff);
                o[2 * i + 1] = uint8_t(h >> 8);
            }
            break;
        case B2D_TYPE_Q8_0:
            for (size_t b = 0; b < n / 32; ++b) {
                const float* x = v.data() + b * 32;
                float amax = 0.0F;
                for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(x[j]));
                const float d = amax / 127.0F;
                const float id = d != 0.0F ? 1.0F / d : 0.0F;
                uint8_t* blk = o + b * 34;
                const uint16_t dh = f32_to_f16(d);
                blk[0] = uint8_t(dh & 0xff);
                blk[1] = uint8_t(dh >> 8);
                for (int j = 0; j < 32; ++j) blk[2 + j] = uint8_t(int8_t(std::roundf(x[j] * id)));
            }
            break;
        default:
            return B2D_EINVAL;
    }
    return B2D_OK;
}

}  // extern "C"
