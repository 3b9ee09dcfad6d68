// Allocation-free split-K GEMM: the same tcgen05 kernel as b2d_gemm's fp32
// epilogue, with its split-K partial sums kept in a fixed, file-scope device
// array instead of memory the library or the caller allocates.
//
// Who needs it: code that runs where it may not (or cannot) call cudaMalloc --
// e.g. a host that hands the library only pre-allocated input/output buffers
// from its own pool or arena, or a process whose allocator is locked while it
// serves requests.  Every GPU that loads this library holds the array
// (kNoAllocScratchFloats floats = 32 MiB) until the process exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/b200diff.h"
#include "gemm.cuh"

using namespace b2d;

namespace {

constexpr int64_t kNoAllocScratchFloats = B2D_NOALLOC_SCRATCH_FLOATS;
constexpr int kMaxDevices = 64;

// Split-K partials [splits, m, n] live here.  In host code this name is only a
// host-side stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress (see device_setup).
static __device__ __align__(256) float g_scratch[kNoAllocScratchFloats];
// Status word for the kernel's bounded waits (cleared at the start of each call).
static __device__ __align__(256) int g_status[64];

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceSetup {
    bool done = false;
    float* scratch = nullptr;
    int* status = nullptr;
    int num_sms = 0;
    EncodeFn encode = nullptr;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mutex;

void put_err(char* buf, size_t len, const char* msg) {
    if (buf && len) std::snprintf(buf, len, "%s", msg);
}

// Once per device, with that device current: resolve the arrays' device addresses.
b2d_status device_setup(int dev, DeviceSetup*& out, char* err, size_t err_len) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSetup& s = g_setup[dev];
    if (!s.done) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess) {
            cudaGetLastError();
            put_err(err, err_len, "cudaGetSymbolAddress(scratch) failed");
            return B2D_ECUDA;
        }
        s.scratch = static_cast<float*>(p);
        if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) {
            cudaGetLastError();
            put_err(err, err_len, "cudaGetSymbolAddress(status) failed");
            return B2D_ECUDA;
        }
        s.status = static_cast<int*>(p);
        if (cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            put_err(err, err_len, "cudaDeviceGetAttribute failed");
            return B2D_ECUDA;
        }
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !p) {
            cudaGetLastError();
            put_err(err, err_len, "cuTensorMapEncodeTiled entry point not found");
            return B2D_ECUDA;
        }
        s.encode = reinterpret_cast<EncodeFn>(p);
        s.done = true;
    }
    out = &s;
    return B2D_OK;
}

bool encode(EncodeFn fn, CUtensorMap* m, const void* base, bool bf16, uint64_t rows, uint64_t k, uint32_t box_rows) {
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// out[r, c] = bias[c] + sum_s part[s, r, c]  (fixed order: deterministic).  When the GEMM gave up on a bounded
// wait (status word non-zero) its partials are incomplete: the output is set to NaN instead of a plausible sum.
static __global__ void noalloc_reduce_kernel(const float* __restrict__ part, int splits, int64_t m, int64_t n,
                                             const float* __restrict__ bias, float* __restrict__ out, int64_t ldo,
                                             const int* __restrict__ status) {
    const bool failed = *reinterpret_cast<const volatile int*>(status) != 0;
    const int64_t total = m * n;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        float v = bias ? bias[i % n] : 0.f;
        for (int s = 0; s < splits; ++s) v += part[s * total + i];
        out[(i / n) * ldo + (i % n)] = failed ? __int_as_float(0x7fc00000) : v;
    }
}

// The bounded wait every kernel of the library uses, on an mbarrier nothing arrives on: it gives up after
// `polls` polls and records a timeout code in the status word.  No fault is involved.
static __global__ void noalloc_selftest_wait_kernel(uint32_t polls, int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, status, kErrTimeoutMma, polls);
}

template <int BN, typename CT>
b2d_status launch(const CUtensorMap& ta, const CUtensorMap& tb, int64_t m, int64_t n, int64_t k, int splits,
                  float* scratch, int* status, int num_sms, cudaStream_t st) {
    using S = GemmShape<BN>;
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_F32, CT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(S::SMEM_BYTES)) != cudaSuccess)
        return B2D_ECUDA;
    EpiParams ep;
    ep.out = scratch;
    ep.ldo = n;
    ep.status = status;
    ep.splits = splits;
    ep.split_stride = m * n;
    const int64_t units = ((m + 127) / 128) * (n / BN) * splits;
    const int grid = int(units < num_sms ? units : num_sms);
    const CUtensorMap no_out{};  // split-K partials take the plain fp32 store path
    gemm_tc_kernel<BN, EPI_F32, CT><<<grid, 192, S::SMEM_BYTES, st>>>(ta, tb, no_out, no_out, int(m), int(n), int(k),
                                                                       ep);
    return cudaGetLastError() == cudaSuccess ? B2D_OK : B2D_ECUDA;
}

}  // namespace

extern "C" B2D_API b2d_status b2d_gemm_splitk_noalloc(int32_t bf16, const void* a_dev, const void* b_dev, int64_t m,
                                                       int64_t n, int64_t k, int32_t splits, int32_t bn,
                                                       const float* bias_dev, float* out_dev, int64_t ldo,
                                                       void* stream, char* err, size_t err_len) {
    if (!a_dev || !b_dev || !out_dev || m <= 0 || n <= 0 || k <= 0 || ldo < n) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: null pointer or non-positive size");
        return B2D_EINVAL;
    }
    if (k % 64 || (bn != 64 && bn != 128 && bn != 256) || n % bn) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: need k % 64 == 0, bn in {64,128,256}, n % bn == 0");
        return B2D_EINVAL;
    }
    if (splits < 1 || (k / 64) % splits) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: splits must divide k / 64");
        return B2D_EINVAL;
    }
    if (int64_t(splits) * m * n > kNoAllocScratchFloats) {
        char msg[200];
        std::snprintf(msg, sizeof(msg),
                      "b2d_gemm_splitk_noalloc: splits * m * n = %lld exceeds the fixed scratch of %lld floats",
                      (long long)(int64_t(splits) * m * n), (long long)kNoAllocScratchFloats);
        put_err(err, err_len, msg);
        return B2D_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(a_dev) | reinterpret_cast<uintptr_t>(b_dev)) % 16) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: operands must be 16-byte aligned");
        return B2D_EINVAL;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: no current CUDA device");
        return B2D_ENODEV;
    }
    DeviceSetup* ds = nullptr;
    b2d_status rc = device_setup(dev, ds, err, err_len);
    if (rc != B2D_OK) return rc;
    CUtensorMap ta, tb;
    if (!encode(ds->encode, &ta, a_dev, bf16 != 0, uint64_t(m), uint64_t(k), 128) ||
        !encode(ds->encode, &tb, b_dev, bf16 != 0, uint64_t(n), uint64_t(k), uint32_t(bn))) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: cuTensorMapEncodeTiled failed");
        return B2D_ECUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(ds->status, 0, sizeof(int), st) != cudaSuccess) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: status clear failed");
        return B2D_ECUDA;
    }
    // No zeroing of the partials is needed: every split writes its full [m, n] slice.
    if (bf16) {
        if (bn == 256) rc = launch<256, __nv_bfloat16>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
        else if (bn == 128) rc = launch<128, __nv_bfloat16>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
        else rc = launch<64, __nv_bfloat16>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
    } else {
        if (bn == 256) rc = launch<256, __half>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
        else if (bn == 128) rc = launch<128, __half>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
        else rc = launch<64, __half>(ta, tb, m, n, k, splits, ds->scratch, ds->status, ds->num_sms, st);
    }
    if (rc != B2D_OK) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: kernel launch failed");
        return rc;
    }
    int64_t blocks = (m * n + 255) / 256;
    if (blocks > int64_t(ds->num_sms) * 8) blocks = int64_t(ds->num_sms) * 8;
    noalloc_reduce_kernel<<<unsigned(blocks), 256, 0, st>>>(ds->scratch, splits, m, n, bias_dev, out_dev, ldo,
                                                            ds->status);
    if (cudaGetLastError() != cudaSuccess) {
        put_err(err, err_len, "b2d_gemm_splitk_noalloc: reduce launch failed");
        return B2D_ECUDA;
    }
    return B2D_OK;
}

extern "C" B2D_API b2d_status b2d_gemm_splitk_noalloc_status(void* stream, char* err, size_t err_len) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc_status: no current CUDA device");
        return B2D_ENODEV;
    }
    DeviceSetup* ds = nullptr;
    b2d_status rc = device_setup(dev, ds, err, err_len);
    if (rc != B2D_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int code = 0;
    if (cudaMemcpyAsync(&code, ds->status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc_status: status read failed");
        return B2D_ECUDA;
    }
    if (code == 0) return B2D_OK;
    if (cudaMemsetAsync(ds->status, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
        cudaGetLastError();
        put_err(err, err_len, "b2d_gemm_splitk_noalloc_status: status clear failed");
        return B2D_ECUDA;
    }
    char msg[160];
    std::snprintf(msg, sizeof(msg),
                  "b2d_gemm_splitk_noalloc: device-side wait expired (code %d); the output was set to NaN", code);
    put_err(err, err_len, msg);
    return B2D_ETIMEOUT;
}

extern "C" B2D_API b2d_status b2d_gemm_splitk_noalloc_selftest_timeout(uint32_t polls, void* stream, char* err,
                                                                        size_t err_len) {
    if (polls == 0 || polls > (1u << 24)) {
        put_err(err, err_len, "polls must be in [1, 2^24]");
        return B2D_EINVAL;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        put_err(err, err_len, "no current CUDA device");
        return B2D_ENODEV;
    }
    DeviceSetup* ds = nullptr;
    b2d_status rc = device_setup(dev, ds, err, err_len);
    if (rc != B2D_OK) return rc;
    noalloc_selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, ds->status);
    if (cudaGetLastError() != cudaSuccess) {
        put_err(err, err_len, "self-test launch failed");
        return B2D_ECUDA;
    }
    return B2D_OK;
}
