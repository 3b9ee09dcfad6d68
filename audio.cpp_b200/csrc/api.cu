// C ABI implementation (include/b200diff.h): device context, weight upload,
// the VibeVoice diffusion-head runtime and its graph-captured sampling loop,
// plus kernel-level entry points used by the parity tests.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/b200diff.h"
#include "attention_tc.cuh"
#include "dit_kernels.cuh"
#include "sa3_kernels.cuh"
#include "conv_tc.cuh"
#include "t5_kernels.cuh"
#include "lm_kernels.cuh"
#include "gemm.cuh"
#include "gemm_stream.cuh"
#include "kernels.cuh"

using namespace b2d;

namespace {

// ------------------------------------------------------------ error plumbing
struct Fail {
    b2d_status code;
    std::string msg;
};

[[noreturn]] void fail(b2d_status code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    throw Fail{code, buf};
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) fail(B2D_ECUDA, "%s failed: %s", #call, cudaGetErrorString(e_));    \
    } while (0)

// ----------------------------------------------------------- device buffers
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    explicit DevBuf(size_t n) { alloc(n); }
    void alloc(size_t n) {
        release();
        if (n == 0) return;
        cudaError_t e = cudaMalloc(&p, n);
        if (e != cudaSuccess) {
            p = nullptr;
            cudaGetLastError();
            fail(B2D_ENOMEM, "device allocation of %zu bytes failed: %s", n, cudaGetErrorString(e));
        }
        bytes = n;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    ~DevBuf() { release(); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) {
        o.p = nullptr;
        o.bytes = 0;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

// ------------------------------------------------------ kernel launches
// Launches inside a PdlScope carry the programmatic-stream-serialization attribute: the next kernel may start
// its prologue (and its constant-weight loads) while this one finishes; every kernel launched this way calls
// pdl_wait before touching data of its predecessors.  Per host thread, so concurrent contexts do not interact.
thread_local bool tl_pdl = false;

struct PdlScope {
    bool prev;
    PdlScope() : prev(tl_pdl) { tl_pdl = true; }
    ~PdlScope() { tl_pdl = prev; }
};

template <typename... KArgs, typename... Args>
void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
              Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    int n = 0;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = unsigned(cluster_x);
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    if (tl_pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = unsigned(n);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) fail(B2D_ECUDA, "kernel launch failed: %s", cudaGetErrorString(e));
}

// ---------------------------------------------------------- TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_host_mutex;  // guards the process-wide lookups below

EncodeTiledFn encode_fn() {
    static std::atomic<EncodeTiledFn> fn{nullptr};
    EncodeTiledFn f = fn.load(std::memory_order_acquire);
    if (!f) {
        std::lock_guard<std::mutex> lock(g_host_mutex);
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) fail(B2D_ECUDA, "cuTensorMapEncodeTiled unavailable");
        f = reinterpret_cast<EncodeTiledFn>(p);
        fn.store(f, std::memory_order_release);
    }
    return f;
}

// A kernel's dynamic shared-memory limit is an attribute of the function in the CURRENT device's context, so it
// is set once per (kernel, device): a second context on another device in the same process sets its own.
template <typename K>
void set_smem_limit(K* kernel, int bytes) {
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
    std::lock_guard<std::mutex> lock(g_host_mutex);
    if (done.count(key)) return;
    CK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.insert(key);
}

// 2-D K-major operand [rows, k] of 16-bit elements, boxes of 64 (K) x box_rows, 128B swizzle.
CUtensorMap make_tmap(const void* base, bool bf16, uint64_t rows, uint64_t k, uint32_t box_rows) {
    if (reinterpret_cast<uintptr_t>(base) % 16) fail(B2D_EINVAL, "GEMM operand is not 16-byte aligned");
    if (k % 64) fail(B2D_EINVAL, "GEMM K (%llu) must be a multiple of 64", (unsigned long long)k);
    CUtensorMap m;
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {k * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(B2D_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return m;
}

// ------------------------------------------------------------ GEMM launcher
// fp32 [rows][cols] matrix with row stride ld (elements) as 32 x 32 boxes, 128B swizzle (TMA epilogues).
CUtensorMap make_tmap_f32_box32(const void* base, int64_t rows, int64_t cols, int64_t ld) {
    CUtensorMap m{};
    const cuuint64_t dims[2] = {uint64_t(cols), uint64_t(rows)};
    const cuuint64_t strides[1] = {uint64_t(ld) * 4};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(B2D_ECUDA, "cuTensorMapEncodeTiled (fp32 box) failed (%d)", int(r));
    return m;
}

// The residual (and gate) of EPI_RESID can go through TMA boxes: plain 16-byte aligned fp32 matrices.
bool resid_tma_ok(const EpiParams& ep, int64_t N) {
    return !ep.gate_rows && reinterpret_cast<uintptr_t>(ep.resid) % 16 == 0 && ep.ldr % 4 == 0 && ep.ldr >= N &&
           (!ep.gate || (reinterpret_cast<uintptr_t>(ep.gate) % 16 == 0 && ep.ldg % 4 == 0 && ep.ldg >= N));
}

template <int BN, int EPI, typename CT>
void launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, int64_t M, int64_t N, int64_t K, const EpiParams& ep,
                   int num_sms, cudaStream_t st) {
    using S = GemmShape<BN, EPI>;
    set_smem_limit(gemm_tc_kernel<BN, EPI, CT>, int(S::SMEM_BYTES));
    const int splits = ep.splits > 1 ? ep.splits : 1;
    if ((K / 64) % splits) fail(B2D_EINVAL, "split-K %d does not divide the %lld K blocks", splits, (long long)(K / 64));
    if (splits > 1 && EPI != EPI_F32) fail(B2D_EINVAL, "split-K needs the fp32 partial-output epilogue");
    const int64_t tiles = ((M + 127) / 128) * (N / BN) * splits;
    if (tiles == 0) return;
    const int grid = int(tiles < num_sms ? tiles : num_sms);
    CUtensorMap to{}, tg{};
    EpiParams e = ep;
    // fp32 output through TMA stores when the output is a plain [M, ldo] fp32 matrix
    if (EPI == EPI_F32 && S::TMA_F32_OUT && splits == 1 && !ep.seg_rows && ep.out &&
        reinterpret_cast<uintptr_t>(ep.out) % 16 == 0 && ep.ldo % 4 == 0 && ep.ldo >= N) {
        to = make_tmap_f32_box32(ep.out, M, N, ep.ldo);
        e.tma_out = 1;
    }
    // residual (and gate) through TMA boxes when both are plain 16-byte aligned fp32 matrices
    if (EPI == EPI_RESID && resid_tma_ok(ep, N)) {
        to = make_tmap_f32_box32(ep.resid, M, N, ep.ldr);
        if (ep.gate) tg = make_tmap_f32_box32(ep.gate, M, N, ep.ldg);
        e.tma_resid = 1;
    }
    launch_k(gemm_tc_kernel<BN, EPI, CT>, dim3(unsigned(grid)), dim3(192), S::SMEM_BYTES, st, 1, ta, tb, to, tg, int(M),
             int(N), int(K), e);
}

// 2-SM (cta_group::2) 256 x 256 pair tiles; B operands need a 128-row TMA box.

template <int BN, int EPI, typename CT>
void launch_gemm_pair_t(const CUtensorMap& ta, const CUtensorMap& tb_half, int64_t M, int64_t N, int64_t K,
                        const EpiParams& ep, int num_sms, cudaStream_t st) {
    using S = GemmPairShape<BN, EPI>;
    set_smem_limit(gemm_tc2_kernel<BN, EPI, CT>, int(S::SMEM_BYTES));
    const int64_t units = ((M + 255) / 256) * (N / BN);
    if (units == 0) return;
    const int64_t pairs = units < num_sms / 2 ? units : num_sms / 2;
    CUtensorMap to{}, tg{};
    EpiParams e = ep;
    if (EPI == EPI_RESID && resid_tma_ok(ep, N)) {
        to = make_tmap_f32_box32(ep.resid, M, N, ep.ldr);
        if (ep.gate) tg = make_tmap_f32_box32(ep.gate, M, N, ep.ldg);
        e.tma_resid = 1;
    }
    launch_k(gemm_tc2_kernel<BN, EPI, CT>, dim3(unsigned(2 * pairs)), dim3(192), S::SMEM_BYTES, st, 1, ta, tb_half,
             to, tg, int(M), int(N), int(K), e);
}

// 2-SM pair tiles of 256 x bn (bn = 256 or 192); tb_half is B's tensor map with a bn / 2-row box.
template <typename CT>
void launch_gemm_pair(int epi, const CUtensorMap& ta, const CUtensorMap& tb_half, int64_t M, int64_t N, int64_t K,
                      const EpiParams& ep, int num_sms, cudaStream_t st, int bn = 256) {
    if (bn != 256 && bn != 192) fail(B2D_EINVAL, "pair GEMM tile width %d (256 or 192)", bn);
    if (N % bn) fail(B2D_EINVAL, "pair GEMM N (%lld) must be a multiple of %d", (long long)N, bn);
    if (ep.splits > 1) fail(B2D_EINVAL, "pair GEMM has no split-K");
    if (bn == 192 && epi == EPI_SWIGLU) fail(B2D_EINVAL, "SwiGLU pair tiles are 256 wide");
#define B2D_P(BNv, EPIv)                                                              \
    if (bn == BNv && epi == EPIv) {                                                   \
        launch_gemm_pair_t<BNv, EPIv, CT>(ta, tb_half, M, N, K, ep, num_sms, st);     \
        return;                                                                       \
    }
    B2D_P(256, EPI_F32) B2D_P(256, EPI_CT) B2D_P(256, EPI_SWIGLU) B2D_P(256, EPI_RESID)
    B2D_P(192, EPI_F32) B2D_P(192, EPI_CT) B2D_P(192, EPI_RESID)
#undef B2D_P
    fail(B2D_EINVAL, "unsupported pair GEMM epilogue %d", epi);
}

template <typename CT>
void launch_gemm(int bn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, int64_t M, int64_t N, int64_t K,
                 const EpiParams& ep, int num_sms, cudaStream_t st) {
    if (N % bn) fail(B2D_EINVAL, "GEMM N (%lld) must be a multiple of the tile width %d", (long long)N, bn);
#define B2D_G(BNv, EPIv)                                                  \
    if (bn == BNv && epi == EPIv) {                                      \
        launch_gemm_t<BNv, EPIv, CT>(ta, tb, M, N, K, ep, num_sms, st); \
        return;                                                          \
    }
    B2D_G(256, EPI_F32) B2D_G(256, EPI_CT) B2D_G(256, EPI_SWIGLU) B2D_G(256, EPI_RESID)
    B2D_G(192, EPI_F32) B2D_G(192, EPI_CT) B2D_G(192, EPI_RESID)
    B2D_G(128, EPI_F32) B2D_G(128, EPI_CT) B2D_G(128, EPI_RESID)
    B2D_G(64, EPI_F32) B2D_G(64, EPI_CT) B2D_G(64, EPI_RESID)
#undef B2D_G
    fail(B2D_EINVAL, "unsupported GEMM tile %d / epilogue %d", bn, epi);
}

// Fraction of the SM-slots a tile count keeps busy over its waves.
double waves_eff(int64_t tiles, int sms) {
    const int64_t waves = (tiles + sms - 1) / sms;
    return waves == 0 ? 0.0 : double(tiles) / double(waves * sms);
}

int grid_for(int64_t n, int threads, int num_sms) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = int64_t(num_sms) * 8;
    if (g > cap) g = cap;
    return int(g < 1 ? 1 : g);
}

// ------------------------------------------------------------------ weights
struct HostTensor {
    const b2d_tensor_view* v = nullptr;
};

const b2d_tensor_view* find_tensor(const b2d_tensor_view* ts, int n, const std::string& name) {
    for (int i = 0; i < n; ++i)
        if (ts[i].name && name == ts[i].name) return &ts[i];
    return nullptr;
}

size_t type_row_bytes(int type, int64_t k) {
    switch (type) {
        case B2D_TYPE_F32: return size_t(k) * 4;
        case B2D_TYPE_F16:
        case B2D_TYPE_BF16: return size_t(k) * 2;
        case B2D_TYPE_Q8_0: return size_t(k / 32) * 34;
        default: return 0;
    }
}

// Uploads a [rows, k] weight (any supported encoding) into `dst` (ct, leading dim k) with a row map.
template <typename CT>
void upload_weight(const b2d_tensor_view* t, int64_t rows, int64_t k, CT* dst, RowMap map, int num_sms,
                   cudaStream_t st) {
    int64_t elems = 1;
    for (int i = 0; i < t->ndim; ++i) elems *= t->dims[i];
    if (t->dims[0] != rows || elems != rows * k) fail(B2D_EINVAL, "tensor shape mismatch for %s", t->name);
    if (t->ggml_type == B2D_TYPE_Q8_0 && k % 32) fail(B2D_EINVAL, "Q8_0 row not divisible by 32: %s", t->name);
    const size_t need = type_row_bytes(t->ggml_type, k) * size_t(rows);
    if (need == 0) fail(B2D_EINVAL, "unsupported tensor type %d for %s", t->ggml_type, t->name);
    if (t->nbytes != need) fail(B2D_EINVAL, "tensor byte size mismatch for %s", t->name);
    DevBuf staging(need);
    CK(cudaMemcpyAsync(staging.p, t->data, need, cudaMemcpyHostToDevice, st));
    const int grid = grid_for(rows * k, 256, num_sms);
    switch (t->ggml_type) {
        case B2D_TYPE_Q8_0:
            dequant_q8_0_kernel<CT><<<grid_for(rows * k / 32, 256, num_sms), 256, 0, st>>>(staging.as<uint8_t>(), rows,
                                                                                          k, dst, k, map);
            break;
        case B2D_TYPE_F16:
            convert_rows_kernel<__half, CT><<<grid, 256, 0, st>>>(staging.as<__half>(), rows, k, dst, k, map);
            break;
        case B2D_TYPE_BF16:
            convert_rows_kernel<__nv_bfloat16, CT><<<grid, 256, 0, st>>>(staging.as<__nv_bfloat16>(), rows, k, dst, k,
                                                                         map);
            break;
        default:
            convert_rows_kernel<float, CT><<<grid, 256, 0, st>>>(staging.as<float>(), rows, k, dst, k, map);
            break;
    }
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(st));
}

std::vector<float> host_f32(const b2d_tensor_view* t, int64_t n) {
    if (!t) fail(B2D_EINVAL, "missing f32 tensor");
    std::vector<float> v(static_cast<size_t>(n));
    if (t->ggml_type == B2D_TYPE_F32 && t->nbytes == size_t(n) * 4) {
        std::memcpy(v.data(), t->data, size_t(n) * 4);
    } else if (t->ggml_type == B2D_TYPE_F16 && t->nbytes == size_t(n) * 2) {
        const uint16_t* h = static_cast<const uint16_t*>(t->data);
        for (int64_t i = 0; i < n; ++i) {
            __half_raw r;
            r.x = h[i];
            v[size_t(i)] = __half2float(__half(r));
        }
    } else if (t->ggml_type == B2D_TYPE_BF16 && t->nbytes == size_t(n) * 2) {
        const uint16_t* h = static_cast<const uint16_t*>(t->data);
        for (int64_t i = 0; i < n; ++i) {
            uint32_t u = uint32_t(h[i]) << 16;
            std::memcpy(&v[size_t(i)], &u, 4);
        }
    } else {
        fail(B2D_EINVAL, "tensor byte size mismatch for %s", t->name);
    }
    return v;
}

// ------------------------------------------------------------- VibeVoice head
constexpr int kHeadLatent = 64;

// Launch plan of the weight-streaming GEMM for one shape: column-tile width and the K split (= cluster size).
struct StreamPlan {
    int bn = 0, split = 1;
};

struct HeadWorkspace {
    int64_t batch = 0;  // B; GEMM rows = 2B
    // rows <= 128: weight-streaming plans of the per-step projections and weight maps with their tile widths
    StreamPlan plan_ada, plan_gu, plan_down;
    CUtensorMap tm_ada_s{};
    std::vector<CUtensorMap> tm_gu_s, tm_down_s;
    DevBuf x, cp, sc, ada, h, ffn, v, noisy, cond, cond_ct, init, xstate, hist0, hist1, out, temb, h1, tsteps, coefs, ptstep, vpart, feat_ct, h1pre, h1_ct;
    int final_splits = 1;
    CUtensorMap tm_noisy, tm_cond, tm_sc, tm_h, tm_ffn, tm_feat, tm_h1;
    std::map<std::tuple<int64_t, uint32_t>, cudaGraphExec_t> graphs;  // (steps, cfg bits) -> graph
    ~HeadWorkspace() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    }
};

struct DitModel;
struct Sa3Model;
struct OobModel;
struct VdModel;
struct T5Model;
struct LmModel;

struct HeadModel {
    b2d_vv_head_config cfg{};
    int64_t H = 0, F = 0, NADA = 0;
    bool bf16 = false;
    DevBuf w_in, w_cond, w_t1, w_t2, w_ada, w_final, norms;
    std::vector<DevBuf> w_gu, w_down;
    CUtensorMap tm_in, tm_cond, tm_ada, tm_final, tm_t1, tm_t2;
    std::vector<CUtensorMap> tm_gu, tm_gu128, tm_down256, tm_down192, tm_down128;
    // Q8_0 checkpoints: the same projections kept as k-block-major Q8_0 planes for the weight-streaming GEMM
    // (few rows), next to the fp16 copies the tensor-bound GEMMs read.
    bool q8 = false;
    DevBuf q_ada, d_ada;
    std::vector<DevBuf> q_gu, d_gu, q_down, d_down;
    std::unique_ptr<HeadWorkspace> ws;
};

}  // namespace

struct b2d_ctx {
    int device = 0;
    int num_sms = 148;
    std::string err;
    DevBuf status;  // int device-side status word
    cudaStream_t load_stream = nullptr;
    std::unique_ptr<HeadModel> head;
    std::unique_ptr<DitModel> dit;
    std::unique_ptr<Sa3Model> sa3;
    std::unique_ptr<OobModel> oob;
    std::unique_ptr<VdModel> vvdec;
    std::unique_ptr<T5Model> t5;
    std::unique_ptr<LmModel> lm;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

template <typename F>
b2d_status guarded(b2d_ctx* ctx, F&& f) {
    if (!ctx) return B2D_EINVAL;
    try {
        DeviceGuard g(ctx->device);
        f();
        ctx->err.clear();
        return B2D_OK;
    } catch (const Fail& e) {
        ctx->err = e.msg;
        return e.code;
    } catch (const std::exception& e) {
        ctx->err = e.what();
        return B2D_EINVAL;
    }
}

void check_status_word(b2d_ctx* ctx, cudaStream_t st) {
    int s = 0;
    CK(cudaMemcpyAsync(&s, ctx->status.p, sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (s != 0) {
        CK(cudaMemsetAsync(ctx->status.p, 0, sizeof(int), st));
        CK(cudaStreamSynchronize(st));
        if (s == kErrNonFinite) fail(B2D_ENONFINITE, "VibeVoice diffusion sampler produced non-finite latent");
        fail(B2D_ETIMEOUT, "a device-side wait expired (code %d); the kernel unwound", s);
    }
}

// Q8_0 [rows, k] weight -> k-block-major planes (q [k/64][n_total][64], d [k/64][n_total][2]) at rows map(r).
void upload_q8_planar(const b2d_tensor_view* t, int64_t rows, int64_t k, int8_t* q, __half* d, int64_t n_total,
                      RowMap map, int num_sms, cudaStream_t st) {
    if (t->ggml_type != B2D_TYPE_Q8_0) fail(B2D_EINVAL, "%s is not Q8_0", t->name);
    if (t->dims[0] != rows || k % 64) fail(B2D_EINVAL, "Q8_0 plane shape for %s", t->name);
    const size_t need = type_row_bytes(B2D_TYPE_Q8_0, k) * size_t(rows);
    if (t->nbytes != need) fail(B2D_EINVAL, "tensor byte size mismatch for %s", t->name);
    DevBuf staging(need);
    CK(cudaMemcpyAsync(staging.p, t->data, need, cudaMemcpyHostToDevice, st));
    repack_q8_0_kernel<<<grid_for(rows * k / 32, 256, num_sms), 256, 0, st>>>(staging.as<uint8_t>(), rows, k, q, d,
                                                                               n_total, map);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(st));
}

template <int BN, int WF, int EPI, typename CT>
int stream_max_clusters(int split) {
    using S = StreamShape<BN, WF>;
    set_smem_limit(gemm_stream_kernel<BN, WF, EPI, CT>, int(S::SMEM_BYTES));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(unsigned(split), 1, 1);
    cfg.blockDim = dim3(S::THREADS, 1, 1);
    cfg.dynamicSmemBytes = S::SMEM_BYTES;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(split);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_stream_kernel<BN, WF, EPI, CT>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

template <int WF, int EPI, typename CT>
int stream_max_clusters_bn(int bn, int split) {
    switch (bn) {
        case 64: if constexpr (EPI != EPI_SWIGLU) return stream_max_clusters<64, WF, EPI, CT>(split); break;
        case 128: if constexpr (EPI != EPI_SWIGLU) return stream_max_clusters<128, WF, EPI, CT>(split); break;
        case 192: if constexpr (EPI != EPI_SWIGLU) return stream_max_clusters<192, WF, EPI, CT>(split); break;
        default: return stream_max_clusters<256, WF, EPI, CT>(split);
    }
    return 0;
}

// Picks (bn, split) so that the n_tiles x split CTAs run in one wave (every cluster co-resident) and keep as many
// SMs streaming as possible; ties go to the smaller split (less reduction traffic), then the wider tile.
template <int WF, int EPI, typename CT>
StreamPlan stream_plan_t(int num_sms, int64_t N, int64_t K) {
    StreamPlan best;
    int64_t best_ctas = -1;
    const int64_t kb = K / 64;
    const int bns[4] = {256, 192, 128, 64};
    for (int bn : bns) {
        if (EPI == EPI_SWIGLU && bn != 256) continue;
        if (N % bn) continue;
        const int64_t tiles = N / bn;
        for (int split : {1, 2, 3, 4, 6, 8}) {
            if (split > kb) break;
            const int64_t ctas = tiles * split;
            if (ctas > num_sms) break;
            const int maxc = stream_max_clusters_bn<WF, EPI, CT>(bn, split);
            if (maxc < tiles) continue;
            if (ctas > best_ctas || (ctas == best_ctas && split < best.split)) {
                best_ctas = ctas;
                best.bn = bn;
                best.split = split;
            }
        }
    }
    if (best.bn == 0) {  // nothing fits one wave: the widest tile without a split
        for (int bn : bns)
            if (N % bn == 0 && (EPI != EPI_SWIGLU || bn == 256)) {
                best.bn = bn;
                break;
            }
    }
    return best;
}

template <typename CT>
StreamPlan stream_plan(b2d_ctx* ctx, bool q8, int epi, int64_t N, int64_t K) {
    switch (epi * 2 + (q8 ? 1 : 0)) {
        case EPI_F32 * 2: return stream_plan_t<WF_16, EPI_F32, CT>(ctx->num_sms, N, K);
        case EPI_F32 * 2 + 1: return stream_plan_t<WF_Q8, EPI_F32, CT>(ctx->num_sms, N, K);
        case EPI_CT * 2: return stream_plan_t<WF_16, EPI_CT, CT>(ctx->num_sms, N, K);
        case EPI_CT * 2 + 1: return stream_plan_t<WF_Q8, EPI_CT, CT>(ctx->num_sms, N, K);
        case EPI_SWIGLU * 2: return stream_plan_t<WF_16, EPI_SWIGLU, CT>(ctx->num_sms, N, K);
        case EPI_SWIGLU * 2 + 1: return stream_plan_t<WF_Q8, EPI_SWIGLU, CT>(ctx->num_sms, N, K);
        case EPI_RESID * 2: return stream_plan_t<WF_16, EPI_RESID, CT>(ctx->num_sms, N, K);
        default: return stream_plan_t<WF_Q8, EPI_RESID, CT>(ctx->num_sms, N, K);
    }
}

template <int BN, int WF, int EPI, typename CT>
void launch_stream_t(const CUtensorMap& ta, const CUtensorMap& tb, const int8_t* q, const __half* d, int64_t M,
                     int64_t N, int64_t K, int split, const EpiParams& ep, cudaStream_t st, const DevBuf* pf0,
                     const DevBuf* pf1) {
    using S = StreamShape<BN, WF>;
    set_smem_limit(gemm_stream_kernel<BN, WF, EPI, CT>, int(S::SMEM_BYTES));
    StreamArgs a;
    a.M = int(M);
    a.N = int(N);
    a.K = int(K);
    a.k_blocks = int(K / 64);
    a.q8 = q;
    a.q8d = d;
    const DevBuf* pf[2] = {pf0, pf1};
    for (int r = 0; r < 2; ++r)
        if (pf[r] && pf[r]->p) {
            a.pf[r] = static_cast<const uint8_t*>(pf[r]->p);  // cudaMalloc base: 256-byte aligned
            a.pf_bytes[r] = pf[r]->bytes;
        }
    launch_k(gemm_stream_kernel<BN, WF, EPI, CT>, dim3(unsigned((N / BN) * split)), dim3(S::THREADS), S::SMEM_BYTES, st,
             split, ta, tb, a, ep);
}

// C = A W^T for M <= 128 rows with the weight-streaming kernel and a plan from stream_plan; W either 16-bit
// through `tb` (box rows = plan.bn) or Q8_0 planes (q, d).  Outputs need 16-byte aligned rows.
template <typename CT>
void launch_stream(StreamPlan plan, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const int8_t* q,
                   const __half* d, int64_t M, int64_t N, int64_t K, const EpiParams& ep, cudaStream_t st,
                   const DevBuf* pf0 = nullptr, const DevBuf* pf1 = nullptr) {
    if (M > 128 || M <= 0) fail(B2D_EINVAL, "weight-streaming GEMM takes 1..128 rows (got %lld)", (long long)M);
    const int bn = plan.bn;
    if (bn == 0 || N % bn || K % 64 || plan.split < 1 || plan.split > K / 64)
        fail(B2D_EINVAL, "weight-streaming GEMM shape %lld x %lld (tile %d, split %d)", (long long)N, (long long)K, bn,
             plan.split);
    if (ep.splits > 1 || ep.seg_rows || ep.rope_cos) fail(B2D_EINVAL, "weight-streaming GEMM epilogue options");
    const bool wq = q != nullptr;
#define B2D_S(BNv, EPIv)                                                                                     \
    if (bn == BNv && epi == EPIv) {                                                                          \
        if (wq) launch_stream_t<BNv, WF_Q8, EPIv, CT>(ta, tb, q, d, M, N, K, plan.split, ep, st, pf0, pf1);  \
        else launch_stream_t<BNv, WF_16, EPIv, CT>(ta, tb, q, d, M, N, K, plan.split, ep, st, pf0, pf1);     \
        return;                                                                                              \
    }
    B2D_S(256, EPI_F32) B2D_S(256, EPI_SWIGLU) B2D_S(256, EPI_RESID) B2D_S(256, EPI_CT)
    B2D_S(192, EPI_F32) B2D_S(192, EPI_RESID) B2D_S(192, EPI_CT)
    B2D_S(128, EPI_F32) B2D_S(128, EPI_RESID) B2D_S(128, EPI_CT)
    B2D_S(64, EPI_F32) B2D_S(64, EPI_RESID) B2D_S(64, EPI_CT)
#undef B2D_S
    fail(B2D_EINVAL, "unsupported weight-streaming GEMM tile %d / epilogue %d", bn, epi);
}

// ------------------------------------------------------------ head: load
template <typename CT>
void head_load_t(b2d_ctx* ctx, HeadModel& m, const b2d_tensor_view* ts, int n) {
    const int64_t H = m.H, F = m.F, L = m.cfg.head_layers;
    const std::string P = "model.prediction_head.";
    cudaStream_t st = ctx->load_stream;
    auto need = [&](const std::string& name) {
        const b2d_tensor_view* t = find_tensor(ts, n, P + name);
        if (!t) fail(B2D_EINVAL, "missing tensor %s%s", P.c_str(), name.c_str());
        return t;
    };
    auto plain = [](int64_t rows) { return RowMap{rows, 0, 0}; };
    const size_t e = sizeof(CT);
    m.w_in.alloc(size_t(H) * kHeadLatent * e);
    upload_weight<CT>(need("noisy_images_proj.weight"), H, kHeadLatent, m.w_in.as<CT>(), plain(H), ctx->num_sms, st);
    m.w_cond.alloc(size_t(H) * H * e);
    upload_weight<CT>(need("cond_proj.weight"), H, H, m.w_cond.as<CT>(), plain(H), ctx->num_sms, st);
    m.w_t1.alloc(size_t(H) * 256 * e);
    upload_weight<CT>(need("t_embedder.mlp.0.weight"), H, 256, m.w_t1.as<CT>(), plain(H), ctx->num_sms, st);
    m.w_t2.alloc(size_t(H) * H * e);
    upload_weight<CT>(need("t_embedder.mlp.2.weight"), H, H, m.w_t2.as<CT>(), plain(H), ctx->num_sms, st);
    // All adaLN projections in one [NADA, H] matrix: layer l at rows [3H l, 3H (l+1)), final at [3H L, 3H L + 2H).
    m.w_ada.alloc(size_t(m.NADA) * H * e);
    std::vector<float> norms(static_cast<size_t>(L * H));
    m.w_gu.resize(size_t(L));
    m.w_down.resize(size_t(L));
    for (int64_t l = 0; l < L; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        upload_weight<CT>(need(p + "adaLN_modulation.1.weight"), 3 * H, H, m.w_ada.as<CT>(),
                          RowMap{3 * H, 0, 3 * H * l}, ctx->num_sms, st);
        // gate_proj / up_proj interleaved in 128-row blocks: [g0..g127 | u0..u127 | g128.. ] so one
        // 256-column GEMM tile holds matching gate and up columns for the SwiGLU epilogue.
        m.w_gu[size_t(l)].alloc(size_t(2 * F) * H * e);
        upload_weight<CT>(need(p + "ffn.gate_proj.weight"), F, H, m.w_gu[size_t(l)].as<CT>(), RowMap{128, 256, 0},
                          ctx->num_sms, st);
        upload_weight<CT>(need(p + "ffn.up_proj.weight"), F, H, m.w_gu[size_t(l)].as<CT>(), RowMap{128, 256, 128},
                          ctx->num_sms, st);
        m.w_down[size_t(l)].alloc(size_t(H) * F * e);
        upload_weight<CT>(need(p + "ffn.down_proj.weight"), H, F, m.w_down[size_t(l)].as<CT>(), plain(H),
                          ctx->num_sms, st);
        const auto nw = host_f32(need(p + "norm.weight"), H);
        std::memcpy(norms.data() + l * H, nw.data(), size_t(H) * 4);
    }
    upload_weight<CT>(need("final_layer.adaLN_modulation.1.weight"), 2 * H, H, m.w_ada.as<CT>(),
                      RowMap{2 * H, 0, 3 * H * L}, ctx->num_sms, st);
    // Q8_0 checkpoints also keep the per-step projections as Q8_0 planes (same row order as the fp16 copies)
    m.q8 = need("layers.0.ffn.gate_proj.weight")->ggml_type == B2D_TYPE_Q8_0 && H % 64 == 0 && F % 64 == 0;
    for (int64_t l = 0; m.q8 && l < L; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        for (const char* nm : {"adaLN_modulation.1.weight", "ffn.gate_proj.weight", "ffn.up_proj.weight",
                               "ffn.down_proj.weight"})
            if (need(p + nm)->ggml_type != B2D_TYPE_Q8_0) m.q8 = false;
    }
    if (need("final_layer.adaLN_modulation.1.weight")->ggml_type != B2D_TYPE_Q8_0) m.q8 = false;
    if (m.q8) {
        m.q_ada.alloc(size_t(m.NADA) * H);
        m.d_ada.alloc(size_t(m.NADA) * (H / 32) * 2);
        m.q_gu.resize(size_t(L));
        m.d_gu.resize(size_t(L));
        m.q_down.resize(size_t(L));
        m.d_down.resize(size_t(L));
        for (int64_t l = 0; l < L; ++l) {
            const std::string p = "layers." + std::to_string(l) + ".";
            const size_t li = size_t(l);
            upload_q8_planar(need(p + "adaLN_modulation.1.weight"), 3 * H, H, m.q_ada.as<int8_t>(),
                             m.d_ada.as<__half>(), m.NADA, RowMap{3 * H, 0, 3 * H * l}, ctx->num_sms, st);
            m.q_gu[li].alloc(size_t(2 * F) * H);
            m.d_gu[li].alloc(size_t(2 * F) * (H / 32) * 2);
            upload_q8_planar(need(p + "ffn.gate_proj.weight"), F, H, m.q_gu[li].as<int8_t>(), m.d_gu[li].as<__half>(),
                             2 * F, RowMap{128, 256, 0}, ctx->num_sms, st);
            upload_q8_planar(need(p + "ffn.up_proj.weight"), F, H, m.q_gu[li].as<int8_t>(), m.d_gu[li].as<__half>(),
                             2 * F, RowMap{128, 256, 128}, ctx->num_sms, st);
            m.q_down[li].alloc(size_t(H) * F);
            m.d_down[li].alloc(size_t(H) * (F / 32) * 2);
            upload_q8_planar(need(p + "ffn.down_proj.weight"), H, F, m.q_down[li].as<int8_t>(),
                             m.d_down[li].as<__half>(), H, RowMap{H, 0, 0}, ctx->num_sms, st);
        }
        upload_q8_planar(need("final_layer.adaLN_modulation.1.weight"), 2 * H, H, m.q_ada.as<int8_t>(),
                         m.d_ada.as<__half>(), m.NADA, RowMap{2 * H, 0, 3 * H * L}, ctx->num_sms, st);
    }
    m.w_final.alloc(size_t(kHeadLatent) * H * e);
    upload_weight<CT>(need("final_layer.linear.weight"), kHeadLatent, H, m.w_final.as<CT>(), plain(kHeadLatent),
                      ctx->num_sms, st);
    m.norms.alloc(norms.size() * 4);
    CK(cudaMemcpy(m.norms.p, norms.data(), norms.size() * 4, cudaMemcpyHostToDevice));

    const bool bf = m.bf16;
    m.tm_in = make_tmap(m.w_in.p, bf, H, kHeadLatent, 256);
    m.tm_cond = make_tmap(m.w_cond.p, bf, H, H, 256);
    m.tm_ada = make_tmap(m.w_ada.p, bf, m.NADA, H, 256);
    m.tm_final = make_tmap(m.w_final.p, bf, kHeadLatent, H, 64);
    m.tm_t1 = make_tmap(m.w_t1.p, bf, H, 256, 256);
    m.tm_t2 = make_tmap(m.w_t2.p, bf, H, H, 256);
    m.tm_gu.clear();
    m.tm_gu128.clear();
    m.tm_down256.clear();
    m.tm_down192.clear();
    m.tm_down128.clear();
    for (int64_t l = 0; l < L; ++l) {
        m.tm_gu.push_back(make_tmap(m.w_gu[size_t(l)].p, bf, 2 * F, H, 256));
        m.tm_gu128.push_back(make_tmap(m.w_gu[size_t(l)].p, bf, 2 * F, H, 128));  // 2-SM pair tiles
        m.tm_down256.push_back(make_tmap(m.w_down[size_t(l)].p, bf, H, F, 256));
        if (H % 192 == 0) m.tm_down192.push_back(make_tmap(m.w_down[size_t(l)].p, bf, H, F, 192));
        if (H % 256 == 0) m.tm_down128.push_back(make_tmap(m.w_down[size_t(l)].p, bf, H, F, 128));  // pair tiles
    }
}

// --------------------------------------------------------- head: workspace
template <typename CT>
HeadWorkspace& head_workspace(b2d_ctx* ctx, HeadModel& m, int64_t batch) {
    if (m.ws && m.ws->batch == batch) return *m.ws;
    m.ws.reset();
    auto ws = std::make_unique<HeadWorkspace>();
    ws->batch = batch;
    const int64_t R = 2 * batch, H = m.H, F = m.F;
    if (R <= 128) {  // weight-streaming plans of the per-step projections (planned outside any capture)
        ws->plan_ada = stream_plan<CT>(ctx, m.q8, EPI_F32, m.NADA, H);
        ws->plan_gu = stream_plan<CT>(ctx, m.q8, EPI_SWIGLU, 2 * F, H);
        ws->plan_down = stream_plan<CT>(ctx, m.q8, EPI_RESID, H, F);
        if (!m.q8) {
            ws->tm_ada_s = make_tmap(m.w_ada.p, m.bf16, m.NADA, H, uint32_t(ws->plan_ada.bn));
            for (size_t l = 0; l < m.w_gu.size(); ++l) {
                ws->tm_gu_s.push_back(make_tmap(m.w_gu[l].p, m.bf16, 2 * F, H, uint32_t(ws->plan_gu.bn)));
                ws->tm_down_s.push_back(make_tmap(m.w_down[l].p, m.bf16, H, F, uint32_t(ws->plan_down.bn)));
            }
        }
    }
    const size_t e = sizeof(CT);
    ws->x.alloc(size_t(R) * H * 4);
    ws->cp.alloc(size_t(R) * H * 4);
    ws->sc.alloc(size_t(R) * H * e);
    ws->ada.alloc(size_t(R) * m.NADA * 4);
    ws->h.alloc(size_t(R) * H * e);
    ws->ffn.alloc(size_t(R) * F * e);
    ws->v.alloc(size_t(R) * kHeadLatent * 4);
    ws->noisy.alloc(size_t(R) * kHeadLatent * e);
    ws->cond.alloc(size_t(R) * H * 4);
    ws->cond_ct.alloc(size_t(R) * H * e);
    ws->init.alloc(size_t(R) * kHeadLatent * 4);
    ws->xstate.alloc(size_t(batch) * kHeadLatent * 4);
    ws->hist0.alloc(size_t(batch) * kHeadLatent * 4);
    ws->hist1.alloc(size_t(batch) * kHeadLatent * 4);
    ws->out.alloc(size_t(batch) * kHeadLatent * 4);
    ws->temb.alloc(size_t(kMaxTembSteps) * H * 4);
    ws->h1.alloc(size_t(kMaxTembSteps) * H * 4);
    ws->tsteps.alloc(size_t(kMaxTembSteps) * 4);
    ws->coefs.alloc(size_t(kMaxTembSteps) * sizeof(VvStepCoef));
    ws->ptstep.alloc(256);
    // final projection (N = 64) runs split-K: as many K ranges as keep the SMs busy
    {
        const int64_t tiles = (R + 127) / 128, kb = H / 64;
        int sp = 1;
        for (int c = 8; c >= 1; --c)
            if (kb % c == 0 && tiles * c <= ctx->num_sms) {
                sp = c;
                break;
            }
        ws->final_splits = sp;
    }
    ws->vpart.alloc(size_t(ws->final_splits) * R * kHeadLatent * 4);
    ws->feat_ct.alloc(size_t(kMaxTembSteps) * 256 * e);
    ws->h1pre.alloc(size_t(kMaxTembSteps) * H * 4);
    ws->h1_ct.alloc(size_t(kMaxTembSteps) * H * e);
    const bool bf = m.bf16;
    ws->tm_feat = make_tmap(ws->feat_ct.p, bf, kMaxTembSteps, 256, 128);
    ws->tm_h1 = make_tmap(ws->h1_ct.p, bf, kMaxTembSteps, H, 128);
    ws->tm_noisy = make_tmap(ws->noisy.p, bf, R, kHeadLatent, 128);
    ws->tm_cond = make_tmap(ws->cond_ct.p, bf, R, H, 128);
    ws->tm_sc = make_tmap(ws->sc.p, bf, R, H, 128);
    ws->tm_h = make_tmap(ws->h.p, bf, R, H, 128);
    ws->tm_ffn = make_tmap(ws->ffn.p, bf, R, F, 128);
    m.ws = std::move(ws);
    return *m.ws;
}

// One evaluation of the head on ws.noisy / ws.cp (cond_proj already applied) with
// the time embedding row temb_row -> ws.v.  diffusion_head.cpp:495-523.
// RMSNorm + modulate of R rows: one CTA per row (H a multiple of 256, up to 8192), else the warp-per-row kernel up
// to H = 4096 and the looping CTA-per-row one above.
template <typename CT>
void launch_rms_modulate(const float* x, int64_t ldx, const float* w, const float* shift, const float* scale,
                         int64_t ldm, float eps, int64_t H, int64_t R, CT* out, int64_t ldo, cudaStream_t st) {
    const unsigned grid = unsigned((R + 7) / 8);
    if (H % 256 == 0 && H <= 8192 && ldx % 4 == 0 && ldm % 4 == 0 && ldo % 8 == 0)  // CTA per row, 8 values per thread
        launch_k(rms_modulate_row_kernel<CT>, dim3(unsigned(R)), dim3(unsigned(H / 8)), 0, st, 1, x, ldx, w, shift,
                 scale, ldm, eps, int(H), out, ldo);
    else if (H <= 2048)
        launch_k(rms_modulate_warp_kernel<CT, 16>, dim3(grid), dim3(256), 0, st, 1, x, ldx, w, shift, scale, ldm, eps,
                 int(H), R, out, ldo);
    else if (H <= 4096)
        launch_k(rms_modulate_warp_kernel<CT, 32>, dim3(grid), dim3(256), 0, st, 1, x, ldx, w, shift, scale, ldm, eps,
                 int(H), R, out, ldo);
    else
        launch_k(rms_modulate_kernel<CT, 256>, dim3(unsigned(R)), dim3(256), 0, st, 1, x, ldx, w, shift, scale, ldm,
                 eps, int(H), out, ldo);
}

template <typename CT>
void head_forward(b2d_ctx* ctx, HeadModel& m, HeadWorkspace& ws, int temb_row, cudaStream_t st) {
    const int64_t R = 2 * ws.batch, H = m.H, F = m.F, L = m.cfg.head_layers;
    const int sms = ctx->num_sms;
    int* status = ctx->status.as<int>();
    EpiParams ep;
    ep.status = status;
    // x = noisy * W_in^T
    ep.out = ws.x.p;
    ep.ldo = H;
    launch_gemm<CT>(256, EPI_F32, ws.tm_noisy, m.tm_in, R, H, kHeadLatent, ep, sms, st);
    // sc = silu(cond_proj + t_emb)
    launch_k(silu_cond_kernel<CT>, dim3(unsigned(grid_for(R * H / 4, 256, sms))), dim3(256), 0, st, 1,
             (const float*)ws.cp.as<float>(), (const float*)(ws.temb.as<float>() + int64_t(temb_row) * H), R, int(H),
             ws.sc.as<CT>());
    // every adaLN modulation of every layer in one GEMM: ada = sc * W_ada^T  [R, NADA]
    ep = EpiParams{};
    ep.status = status;
    ep.out = ws.ada.p;
    ep.ldo = m.NADA;
    // Up to 128 rows the per-step projections stream their weights (HBM-bound); above, tensor-bound tiles.
    const bool stream = R <= 128 && m.NADA % 256 == 0 && H % 256 == 0 && (2 * F) % 256 == 0 && m.NADA % 4 == 0;
    const bool q8s = stream && m.q8;
    // Each streamed projection hints the next one's weights into L2 (gate/up of layer l after adaLN or the
    // down projection of layer l - 1; down of layer l after gate/up of layer l).
    const auto gu_pf = [&](int64_t l, int r) -> const DevBuf* {
        if (l >= L) return nullptr;
        return q8s ? (r == 0 ? &m.q_gu[size_t(l)] : &m.d_gu[size_t(l)]) : (r == 0 ? &m.w_gu[size_t(l)] : nullptr);
    };
    const auto down_pf = [&](int64_t l, int r) -> const DevBuf* {
        return q8s ? (r == 0 ? &m.q_down[size_t(l)] : &m.d_down[size_t(l)]) : (r == 0 ? &m.w_down[size_t(l)] : nullptr);
    };
    if (stream)
        launch_stream<CT>(ws.plan_ada, EPI_F32, ws.tm_sc, ws.tm_ada_s, q8s ? m.q_ada.as<int8_t>() : nullptr,
                          q8s ? m.d_ada.as<__half>() : nullptr, R, m.NADA, H, ep, st, gu_pf(0, 0), gu_pf(0, 1));
    else
        launch_gemm<CT>(256, EPI_F32, ws.tm_sc, m.tm_ada, R, m.NADA, H, ep, sms, st);
    const float* ada = ws.ada.as<float>();
    for (int64_t l = 0; l < L; ++l) {
        const float* shift = ada + 3 * H * l;
        launch_rms_modulate<CT>(ws.x.as<float>(), H, m.norms.as<float>() + l * H, shift, shift + H, m.NADA,
                                m.cfg.rms_norm_eps, H, R, ws.h.as<CT>(), H, st);
        ep = EpiParams{};
        ep.status = status;
        ep.out = ws.ffn.p;
        ep.ldo = F;
        // SwiGLU GEMMs run on 2-SM 256 x 256 pair tiles (measured faster at every tensor-bound head shape)
        if (stream)
            launch_stream<CT>(ws.plan_gu, EPI_SWIGLU, ws.tm_h, q8s ? ws.tm_ada_s : ws.tm_gu_s[size_t(l)],
                              q8s ? m.q_gu[size_t(l)].as<int8_t>() : nullptr,
                              q8s ? m.d_gu[size_t(l)].as<__half>() : nullptr, R, 2 * F, H, ep, st, down_pf(l, 0),
                              down_pf(l, 1));
        else
            launch_gemm_pair<CT>(EPI_SWIGLU, ws.tm_h, m.tm_gu128[size_t(l)], R, 2 * F, H, ep, sms, st);
        ep = EpiParams{};
        ep.status = status;
        ep.resid = ws.x.as<float>();
        ep.ldr = H;
        ep.gate = shift + 2 * H;
        ep.ldg = m.NADA;
        // 192-wide tiles when they fill the SMs better (H = 1536: 8 x 16 = 128 tiles vs 96); 2-SM 256 x 256 pair
        // tiles for wide or many-row projections, which cut the operand stream per SM by a third (measured with
        // the gate: 7B width 2048 / 8192 / 16384 rows 175 / 580 / 1121 us against 216 / 738 / 1254 us for 1-SM
        // 256-wide tiles; H = 1536 x 16384 rows 232 against 275 us; at H = 1536 x 2048 rows the 1-SM 192-wide
        // tiles stay ahead, 34.9 against 36.9 us)
        const int64_t mt = (R + 127) / 128;
        const int64_t pair_units = ((R + 255) / 256) * (H / 256);
        const bool use_pair = !m.tm_down128.empty() && F >= 4096 && (pair_units >= sms || H >= 3072);
        const bool use192 = !m.tm_down192.empty() && waves_eff(mt * (H / 192), sms) > waves_eff(mt * (H / 256), sms);
        if (stream)
            launch_stream<CT>(ws.plan_down, EPI_RESID, ws.tm_ffn, q8s ? ws.tm_ada_s : ws.tm_down_s[size_t(l)],
                              q8s ? m.q_down[size_t(l)].as<int8_t>() : nullptr,
                              q8s ? m.d_down[size_t(l)].as<__half>() : nullptr, R, H, F, ep, st, gu_pf(l + 1, 0),
                              gu_pf(l + 1, 1));
        else if (use_pair)
            launch_gemm_pair<CT>(EPI_RESID, ws.tm_ffn, m.tm_down128[size_t(l)], R, H, F, ep, sms, st, 256);
        else if (use192)
            launch_gemm<CT>(192, EPI_RESID, ws.tm_ffn, m.tm_down192[size_t(l)], R, H, F, ep, sms, st);
        else
            launch_gemm<CT>(256, EPI_RESID, ws.tm_ffn, m.tm_down256[size_t(l)], R, H, F, ep, sms, st);
    }
    const float* fshift = ada + 3 * H * L;
    launch_rms_modulate<CT>(ws.x.as<float>(), H, nullptr, fshift, fshift + H, m.NADA, m.cfg.rms_norm_eps, H, R,
                            ws.h.as<CT>(), H, st);
    ep = EpiParams{};
    ep.status = status;
    ep.out = ws.vpart.p;
    ep.ldo = kHeadLatent;
    ep.splits = ws.final_splits;
    ep.split_stride = R * kHeadLatent;
    launch_gemm<CT>(64, EPI_F32, ws.tm_h, m.tm_final, R, kHeadLatent, H, ep, sms, st);
}

// cond_ct = ct(cond); cp = cond * W_cond^T (step-invariant, hoisted out of the loop)
template <typename CT>
void head_cond_proj(b2d_ctx* ctx, HeadModel& m, HeadWorkspace& ws, cudaStream_t st) {
    const int64_t R = 2 * ws.batch, H = m.H;
    f32_to_ct_kernel<CT><<<grid_for(R * H, 256, ctx->num_sms), 256, 0, st>>>(ws.cond.as<float>(), R * H,
                                                                              ws.cond_ct.as<CT>());
    CK(cudaGetLastError());
    EpiParams ep;
    ep.status = ctx->status.as<int>();
    ep.out = ws.cp.p;
    ep.ldo = H;
    launch_gemm<CT>(256, EPI_F32, ws.tm_cond, m.tm_cond, R, H, H, ep, ctx->num_sms, st);
}

// t_emb rows for S timesteps: feat = [cos | sin](t f) -> Linear(256->H) -> SiLU -> Linear(H->H),
// both linears on the tensor-core GEMM (rows = S, masked inside 128-row tiles).
template <typename CT>
void head_temb(b2d_ctx* ctx, HeadModel& m, HeadWorkspace& ws, const float* tsteps, int S, cudaStream_t st) {
    const int64_t H = m.H;
    temb_feat_kernel<CT><<<S, 128, 0, st>>>(tsteps, ws.feat_ct.as<CT>());
    CK(cudaGetLastError());
    EpiParams ep;
    ep.status = ctx->status.as<int>();
    ep.out = ws.h1pre.p;
    ep.ldo = H;
    launch_gemm<CT>(256, EPI_F32, ws.tm_feat, m.tm_t1, S, H, 256, ep, ctx->num_sms, st);
    silu_to_ct_kernel<CT><<<grid_for(int64_t(S) * H, 256, ctx->num_sms), 256, 0, st>>>(ws.h1pre.as<float>(),
                                                                                         int64_t(S) * H, ws.h1_ct.as<CT>());
    CK(cudaGetLastError());
    ep.out = ws.temb.p;
    launch_gemm<CT>(256, EPI_F32, ws.tm_h1, m.tm_t2, S, H, H, ep, ctx->num_sms, st);
}

// The full sampling loop on workspace buffers (ws.cond, ws.init filled; coefs/tsteps uploaded).
template <typename CT>
void head_sample_body(b2d_ctx* ctx, HeadModel& m, HeadWorkspace& ws, int S, float cfg, cudaStream_t st) {
    const int64_t n_half = ws.batch * kHeadLatent;
    const int sms = ctx->num_sms;
    head_cond_proj<CT>(ctx, m, ws, st);
    head_temb<CT>(ctx, m, ws, ws.tsteps.as<float>(), S, st);
    vv_init_kernel<CT><<<grid_for(n_half, 256, sms), 256, 0, st>>>(ws.init.as<float>(), ws.xstate.as<float>(),
                                                                     ws.noisy.as<CT>(), n_half);
    CK(cudaGetLastError());
    PdlScope pdl;  // the step loop's kernels overlap each other's launch and prologue
    for (int s = 0; s < S; ++s) {
        head_forward<CT>(ctx, m, ws, s, st);
        float* hp = (s & 1) ? ws.hist0.as<float>() : ws.hist1.as<float>();
        float* hc = (s & 1) ? ws.hist1.as<float>() : ws.hist0.as<float>();
        launch_k(vv_cfg_dpm_kernel<CT>, dim3(unsigned(grid_for(n_half, 256, sms))), dim3(256), 0, st, 1,
                 (const float*)ws.vpart.as<float>(), ws.final_splits, 2 * n_half, ws.xstate.as<float>(),
                 (const float*)hp, hc, ws.noisy.as<CT>(), ws.out.as<float>(), n_half,
                 (const VvStepCoef*)ws.coefs.as<VvStepCoef>(), s, cfg, ctx->status.as<int>());
    }
}

template <typename CT>
void head_sample(b2d_ctx* ctx, const float* pos, const float* neg, const float* init, int64_t batch, int64_t steps,
                 float cfg, float* out, cudaStream_t st, bool host) {
    HeadModel& m = *ctx->head;
    if (steps > kMaxTembSteps) fail(B2D_EINVAL, "at most %d inference steps per call are supported", kMaxTembSteps);
    HeadWorkspace& ws = head_workspace<CT>(ctx, m, batch);
    const int64_t H = m.H;
    const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const size_t half = size_t(batch) * H * 4;
    CK(cudaMemcpyAsync(ws.cond.p, pos, half, kind, st));
    CK(cudaMemcpyAsync(ws.cond.as<char>() + half, neg, half, kind, st));
    CK(cudaMemcpyAsync(ws.init.p, init, size_t(2 * batch) * kHeadLatent * 4, kind, st));

    std::vector<b2d_vv_step> sched(static_cast<size_t>(steps));
    if (b2d_vv_schedule(m.cfg.ddpm_num_steps, steps, sched.data()) != B2D_OK)
        fail(B2D_EINVAL, "VibeVoice scheduler requires positive timestep counts");
    uint32_t cfg_bits;
    std::memcpy(&cfg_bits, &cfg, 4);
    const auto key = std::make_tuple(steps, cfg_bits);
    auto it = ws.graphs.find(key);
    if (it == ws.graphs.end()) {
        // Step tables are constant for a given (ddpm steps, steps): upload once, then capture.
        std::vector<VvStepCoef> coefs(static_cast<size_t>(steps));
        std::vector<float> ts(static_cast<size_t>(steps));
        for (int64_t i = 0; i < steps; ++i) {
            const b2d_vv_step& s = sched[size_t(i)];
            coefs[size_t(i)] = VvStepCoef{s.alpha_s, s.sigma_s, s.sample_coeff, s.d0_coeff, s.inv_r0, s.order,
                                          i == steps - 1 ? 1 : 0, 0};
            ts[size_t(i)] = float(s.timestep);
        }
        CK(cudaMemcpyAsync(ws.coefs.p, coefs.data(), coefs.size() * sizeof(VvStepCoef), cudaMemcpyHostToDevice, st));
        CK(cudaMemcpyAsync(ws.tsteps.p, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice, st));
        CK(cudaStreamSynchronize(st));
        cudaStream_t cap;
        CK(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
        try {
            head_sample_body<CT>(ctx, m, ws, int(steps), cfg, cap);
        } catch (...) {
            cudaStreamEndCapture(cap, &g);
            if (g) cudaGraphDestroy(g);
            cudaStreamDestroy(cap);
            throw;
        }
        CK(cudaStreamEndCapture(cap, &g));
        cudaGraphExec_t exec = nullptr;
        CK(cudaGraphInstantiate(&exec, g, 0));
        cudaGraphDestroy(g);
        cudaStreamDestroy(cap);
        // The tables in ws.coefs/ws.tsteps belong to the most recently captured key; keep one
        // schedule resident by dropping graphs of other step counts.
        for (auto& kv : ws.graphs) cudaGraphExecDestroy(kv.second);
        ws.graphs.clear();
        it = ws.graphs.emplace(key, exec).first;
    }
    CK(cudaGraphLaunch(it->second, st));
    CK(cudaMemcpyAsync(out, ws.out.p, size_t(batch) * kHeadLatent * 4,
                       host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, st));
    if (host) check_status_word(ctx, st);
}

template <typename CT>
void head_predict(b2d_ctx* ctx, const float* noisy, int64_t frames, float timestep, const float* cond, float* out,
                  cudaStream_t st) {
    HeadModel& m = *ctx->head;
    // predict() evaluates `frames` rows; the workspace holds 2*batch rows, so use ceil(frames/2).
    const int64_t batch = (frames + 1) / 2;
    HeadWorkspace& ws = head_workspace<CT>(ctx, m, batch);
    const int64_t R = 2 * batch, H = m.H;
    CK(cudaMemsetAsync(ws.cond.p, 0, size_t(R) * H * 4, st));
    CK(cudaMemcpyAsync(ws.cond.p, cond, size_t(frames) * H * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemsetAsync(ws.init.p, 0, size_t(R) * kHeadLatent * 4, st));
    CK(cudaMemcpyAsync(ws.init.p, noisy, size_t(frames) * kHeadLatent * 4, cudaMemcpyHostToDevice, st));
    f32_to_ct_kernel<CT><<<grid_for(R * kHeadLatent, 256, ctx->num_sms), 256, 0, st>>>(
        ws.init.as<float>(), R * kHeadLatent, ws.noisy.as<CT>());
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(ws.ptstep.p, &timestep, 4, cudaMemcpyHostToDevice, st));
    head_cond_proj<CT>(ctx, m, ws, st);
    head_temb<CT>(ctx, m, ws, ws.ptstep.as<float>(), 1, st);
    head_forward<CT>(ctx, m, ws, 0, st);
    sum_partials_kernel<<<grid_for(R * kHeadLatent, 256, ctx->num_sms), 256, 0, st>>>(
        ws.vpart.as<float>(), ws.final_splits, R * kHeadLatent, ws.v.as<float>());
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(out, ws.v.p, size_t(frames) * kHeadLatent * 4, cudaMemcpyDeviceToHost, st));
    check_status_word(ctx, st);
}

#include "dit_runtime.inc"
#include "sa3_runtime.inc"
#include "oobleck_runtime.inc"
#include "vvdec_runtime.inc"
#include "t5_runtime.inc"
#include "lm_runtime.inc"

// Forgets the decoder's cached positions (after a device-side failure of an asynchronous forward).
void lm_invalidate(b2d_ctx* ctx) {
    if (ctx && ctx->lm) ctx->lm->pos = 0;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

const char* b2d_version(void) { return "b200diff 0.1 (sm_100a)"; }

b2d_status b2d_create(int device, b2d_ctx** out) {
    if (!out) return B2D_EINVAL;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        cudaGetLastError();
        return B2D_ENODEV;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return B2D_ENODEV;
    auto ctx = std::make_unique<b2d_ctx>();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    b2d_status s = guarded(ctx.get(), [&] {
        ctx->status.alloc(256);
        CK(cudaMemset(ctx->status.p, 0, 256));
        CK(cudaStreamCreateWithFlags(&ctx->load_stream, cudaStreamNonBlocking));
        encode_fn();
    });
    if (s != B2D_OK) return s;
    *out = ctx.release();
    return B2D_OK;
}

void b2d_destroy(b2d_ctx* ctx) {
    if (!ctx) return;
    {
        DeviceGuard g(ctx->device);
        cudaDeviceSynchronize();
        ctx->head.reset();
        ctx->dit.reset();
        ctx->sa3.reset();
        ctx->oob.reset();
        ctx->vvdec.reset();
        ctx->t5.reset();
        ctx->lm.reset();
        ctx->status.release();
        if (ctx->load_stream) cudaStreamDestroy(ctx->load_stream);
    }
    delete ctx;
}

const char* b2d_last_error(const b2d_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

namespace {
// One thread waits on an mbarrier that nothing ever arrives on, through the same bounded wait the
// kernels use (with `polls` as its limit instead of kSpinLimit): the wait gives up, records the
// timeout code in the status word and the kernel returns.
__global__ void selftest_wait_kernel(uint32_t polls, int* status) {
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
}  // namespace

b2d_status b2d_selftest_wait_timeout(b2d_ctx* ctx, uint32_t polls, void* stream) {
    return guarded(ctx, [&] {
        if (polls == 0 || polls > (1u << 24)) fail(B2D_EINVAL, "polls must be in [1, 2^24]");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        selftest_wait_kernel<<<1, 32, 0, st>>>(polls, ctx->status.as<int>());
        CK(cudaGetLastError());
        check_status_word(ctx, st);
    });
}

b2d_status b2d_sync(b2d_ctx* ctx, void* stream) {
    return guarded(ctx, [&] {
        try {
            check_status_word(ctx, static_cast<cudaStream_t>(stream));
        } catch (...) {
            // an asynchronous decoder forward may have written garbage cache rows: the next call must prefill
            lm_invalidate(ctx);
            throw;
        }
    });
}

b2d_status b2d_vv_head_load(b2d_ctx* ctx, const b2d_vv_head_config* config, const b2d_tensor_view* tensors,
                            int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0)) fail(B2D_EINVAL, "VibeVoice diffusion head requires model weights");
        const b2d_vv_head_config& c = *config;
        if (c.hidden_size <= 0 || c.latent_size <= 0 || c.head_layers <= 0)
            fail(B2D_EINVAL, "VibeVoice diffusion head dimensions must be positive");
        if (!(c.head_ffn_ratio > 0.0F)) fail(B2D_EINVAL, "VibeVoice diffusion head FFN ratio must be positive");
        if (!(c.rms_norm_eps > 0.0F)) fail(B2D_EINVAL, "VibeVoice diffusion head RMS epsilon must be positive");
        if (c.latent_size != kHeadLatent) fail(B2D_EINVAL, "latent_size must be 64 on this path");
        auto m = std::make_unique<HeadModel>();
        m->cfg = c;
        m->H = c.hidden_size;
        m->F = int64_t(double(c.hidden_size) * double(c.head_ffn_ratio));
        if (m->F <= 0) fail(B2D_EINVAL, "VibeVoice diffusion head FFN dimension is invalid");
        if (m->H % 256 || m->F % 128)
            fail(B2D_EINVAL, "hidden_size must be a multiple of 256 and the FFN width a multiple of 128");
        m->NADA = 3 * m->H * c.head_layers + 2 * m->H;
        // fp16 operands for F16 / Q8_0 / F32 weights; bf16 when the weights are BF16.
        const b2d_tensor_view* probe = find_tensor(tensors, n_tensors, "model.prediction_head.cond_proj.weight");
        m->bf16 = probe && probe->ggml_type == B2D_TYPE_BF16;
        ctx->head.reset();
        if (m->bf16)
            head_load_t<__nv_bfloat16>(ctx, *m, tensors, n_tensors);
        else
            head_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->head = std::move(m);
    });
}

b2d_status b2d_vv_predict(b2d_ctx* ctx, const float* noisy, int64_t frames, int64_t latent_size, float timestep,
                          const float* condition, int64_t condition_hidden_size, float* out, void* stream) {
    return guarded(ctx, [&] {
        if (!ctx->head) fail(B2D_ESTATE, "VibeVoice diffusion head weights are not loaded");
        const HeadModel& m = *ctx->head;
        if (frames <= 0 || latent_size != m.cfg.latent_size || condition_hidden_size != m.H)
            fail(B2D_EINVAL, "VibeVoice diffusion head received invalid input shape");
        if (!noisy || !condition || !out) fail(B2D_EINVAL, "VibeVoice diffusion head received invalid input shape");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (m.bf16)
            head_predict<__nv_bfloat16>(ctx, noisy, frames, timestep, condition, out, st);
        else
            head_predict<__half>(ctx, noisy, frames, timestep, condition, out, st);
    });
}

static b2d_status vv_sample_common(b2d_ctx* ctx, const float* pos, const float* neg, const float* init, int64_t batch,
                                   int64_t steps, float cfg, float* out, void* stream, bool host) {
    return guarded(ctx, [&] {
        if (!ctx->head) fail(B2D_ESTATE, "VibeVoice diffusion head weights are not loaded");
        if (batch <= 0) fail(B2D_EINVAL, "VibeVoice diffusion sampler requires positive dimensions");
        if (steps <= 0) fail(B2D_EINVAL, "VibeVoice diffusion sampler requires positive inference steps");
        if (!pos) fail(B2D_EINVAL, "VibeVoice diffusion sampler payload size mismatch for positive_condition");
        if (!neg) fail(B2D_EINVAL, "VibeVoice diffusion sampler payload size mismatch for negative_condition");
        if (!init) fail(B2D_EINVAL, "VibeVoice diffusion sampler payload size mismatch for initial_speech");
        if (!out) fail(B2D_EINVAL, "output buffer is null");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (ctx->head->bf16)
            head_sample<__nv_bfloat16>(ctx, pos, neg, init, batch, steps, cfg, out, st, host);
        else
            head_sample<__half>(ctx, pos, neg, init, batch, steps, cfg, out, st, host);
    });
}

b2d_status b2d_vv_sample(b2d_ctx* ctx, const float* positive_condition, const float* negative_condition,
                         const float* initial_speech, int64_t batch, int64_t steps, float cfg, float* out_latents,
                         void* stream) {
    return vv_sample_common(ctx, positive_condition, negative_condition, initial_speech, batch, steps, cfg,
                            out_latents, stream, true);
}

b2d_status b2d_vv_sample_device(b2d_ctx* ctx, const float* positive_condition, const float* negative_condition,
                                const float* initial_speech, int64_t batch, int64_t steps, float cfg,
                                float* out_latents, void* stream) {
    return vv_sample_common(ctx, positive_condition, negative_condition, initial_speech, batch, steps, cfg,
                            out_latents, stream, false);
}

b2d_status b2d_q8_0_dequantize(b2d_ctx* ctx, const void* q8_dev, int64_t rows, int64_t k, float* out_dev,
                               void* stream) {
    return guarded(ctx, [&] {
        if (!q8_dev || !out_dev || rows <= 0 || k <= 0 || k % 32) fail(B2D_EINVAL, "invalid Q8_0 shape");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        dequant_q8_0_kernel<float><<<grid_for(rows * k / 32, 256, ctx->num_sms), 256, 0, st>>>(
            static_cast<const uint8_t*>(q8_dev), rows, k, out_dev, k, RowMap{rows, 0, 0});
        CK(cudaGetLastError());
    });
}

b2d_status b2d_gemm(b2d_ctx* ctx, int32_t bf16, const void* a_dev, const void* b_dev, int64_t m, int64_t n,
                    int64_t k, int32_t epilogue, int32_t bn, const float* bias_dev, void* out_dev, int64_t ldo,
                    float* resid_dev, int64_t ldr, const float* gate_dev, int64_t ldg, void* stream) {
    return guarded(ctx, [&] {
        if (m <= 0 || n <= 0 || k <= 0) fail(B2D_EINVAL, "GEMM dimensions must be positive");
        if (epilogue == EPI_SWIGLU && bn != 256 && bn != 512) fail(B2D_EINVAL, "SwiGLU epilogue needs 256-column tiles");
        if (epilogue == EPI_RESID ? !resid_dev : !out_dev) fail(B2D_EINVAL, "GEMM output is null");
        // 512 / 384 select the 2-SM pair-tile kernel with 256 x 256 / 256 x 192 tiles
        const bool pair = bn == 512 || bn == 384;
        const int pair_bn = bn / 2;
        const CUtensorMap ta = make_tmap(a_dev, bf16 != 0, uint64_t(m), uint64_t(k), 128);
        const CUtensorMap tb =
            make_tmap(b_dev, bf16 != 0, uint64_t(n), uint64_t(k), pair ? uint32_t(pair_bn / 2) : uint32_t(bn));
        EpiParams ep;
        ep.out = out_dev;
        ep.ldo = ldo;
        ep.bias = bias_dev;
        ep.resid = resid_dev;
        ep.ldr = ldr;
        ep.gate = gate_dev;
        ep.ldg = ldg;
        ep.status = ctx->status.as<int>();
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (pair) {
            if (bf16)
                launch_gemm_pair<__nv_bfloat16>(epilogue, ta, tb, m, n, k, ep, ctx->num_sms, st, pair_bn);
            else
                launch_gemm_pair<__half>(epilogue, ta, tb, m, n, k, ep, ctx->num_sms, st, pair_bn);
        } else if (bf16) {
            launch_gemm<__nv_bfloat16>(bn, epilogue, ta, tb, m, n, k, ep, ctx->num_sms, st);
        } else {
            launch_gemm<__half>(bn, epilogue, ta, tb, m, n, k, ep, ctx->num_sms, st);
        }
    });
}

b2d_status b2d_gemm_stream(b2d_ctx* ctx, int32_t bf16, const void* a_dev, const void* w_dev, int32_t w_type,
                           int64_t m, int64_t n, int64_t k, int32_t epilogue, int32_t bn, int32_t split,
                           const float* bias_dev,
                           void* out_dev, int64_t ldo, float* resid_dev, int64_t ldr, const float* gate_dev,
                           int64_t ldg, void* stream) {
    return guarded(ctx, [&] {
        if (m <= 0 || n <= 0 || k <= 0 || !a_dev || !w_dev) fail(B2D_EINVAL, "GEMM dimensions must be positive");
        if (epilogue == EPI_RESID ? !resid_dev : !out_dev) fail(B2D_EINVAL, "GEMM output is null");
        const bool q8 = w_type == B2D_TYPE_Q8_0;
        if (!q8 && w_type != (bf16 ? B2D_TYPE_BF16 : B2D_TYPE_F16)) fail(B2D_EINVAL, "weight type");
        if (q8 && bf16) fail(B2D_EINVAL, "Q8_0 weights stream as fp16 operands");
        const bool f32out = epilogue == EPI_F32 || epilogue == EPI_RESID;
        if ((f32out && epilogue == EPI_F32 && (ldo % 4 || reinterpret_cast<uintptr_t>(out_dev) % 16)) ||
            (epilogue == EPI_RESID && (ldr % 4 || reinterpret_cast<uintptr_t>(resid_dev) % 16 ||
                                       (gate_dev && (ldg % 4 || reinterpret_cast<uintptr_t>(gate_dev) % 16)))) ||
            ((epilogue == EPI_CT || epilogue == EPI_SWIGLU) && (ldo % 8 || reinterpret_cast<uintptr_t>(out_dev) % 16)))
            fail(B2D_EINVAL, "weight-streaming GEMM outputs need 16-byte aligned rows");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        StreamPlan plan;
        if (bn == 0) {
            plan = bf16 ? stream_plan<__nv_bfloat16>(ctx, q8, epilogue, n, k) : stream_plan<__half>(ctx, q8, epilogue, n, k);
        } else {
            plan.bn = bn;
            plan.split = split < 1 ? 1 : split;
        }
        const CUtensorMap ta = make_tmap(a_dev, bf16 != 0, uint64_t(m), uint64_t(k), 128);
        CUtensorMap tb{};
        DevBuf qbuf, dbuf;
        if (q8) {
            if (k % 64) fail(B2D_EINVAL, "K %% 64");
            qbuf.alloc(size_t(n) * k);
            dbuf.alloc(size_t(n) * (k / 32) * 2);
            repack_q8_0_kernel<<<grid_for(n * k / 32, 256, ctx->num_sms), 256, 0, st>>>(
                static_cast<const uint8_t*>(w_dev), n, k, qbuf.as<int8_t>(), dbuf.as<__half>(), n, RowMap{n, 0, 0});
            CK(cudaGetLastError());
        } else {
            tb = make_tmap(w_dev, bf16 != 0, uint64_t(n), uint64_t(k), uint32_t(plan.bn));
        }
        EpiParams ep;
        ep.out = out_dev;
        ep.ldo = ldo;
        ep.bias = bias_dev;
        ep.resid = resid_dev;
        ep.ldr = ldr;
        ep.gate = gate_dev;
        ep.ldg = ldg;
        ep.status = ctx->status.as<int>();
        if (bf16)
            launch_stream<__nv_bfloat16>(plan, epilogue, ta, tb, nullptr, nullptr, m, n, k, ep, st);
        else
            launch_stream<__half>(plan, epilogue, ta, tb, q8 ? qbuf.as<int8_t>() : nullptr,
                                  q8 ? dbuf.as<__half>() : nullptr, m, n, k, ep, st);
        if (q8) CK(cudaStreamSynchronize(st));  // the planes are freed on return
    });
}

b2d_status b2d_torch_randn(b2d_ctx* ctx, int32_t layout, uint64_t seed, uint64_t offset, int64_t count,
                           int64_t multiprocessor_count, int64_t max_threads_per_multiprocessor, int32_t bf16,
                           float* out_dev, void* stream) {
    return guarded(ctx, [&] {
        if (count <= 0 || !out_dev || (layout != 0 && layout != 1)) fail(B2D_EINVAL, "invalid randn request");
        if (layout == 1 && (multiprocessor_count <= 0 || max_threads_per_multiprocessor <= 0))
            fail(B2D_EINVAL, "torch CUDA TensorIterator randn requires CUDA device properties");
        const uint64_t stride =
            layout == 1 ? torch_iterator_stride(uint64_t(count), multiprocessor_count, max_threads_per_multiprocessor) : 0;
        torch_randn_kernel<<<grid_for(count, 256, ctx->num_sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            layout, seed, offset, stride, count, bf16, out_dev);
        CK(cudaGetLastError());
    });
}

b2d_status b2d_attention(b2d_ctx* ctx, int32_t bf16, const void* q, int64_t q_row, int64_t q_seq, const void* k,
                         const void* v, int64_t kv_row, int64_t kv_seq, void* o, int64_t o_row, int64_t o_seq,
                         int32_t lq, int32_t lk, int32_t heads, int32_t kv_rep, int32_t nseq, void* stream) {
    return guarded(ctx, [&] {
        if (!q || !k || !v || !o || lq <= 0 || lk <= 0 || heads <= 0 || kv_rep <= 0 || nseq <= 0 ||
            heads % kv_rep)
            fail(B2D_EINVAL, "invalid attention shape");
        if ((q_row | kv_row | q_seq | kv_seq | o_row | o_seq) % 8 ||
            (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
             reinterpret_cast<uintptr_t>(o)) % 16)
            fail(B2D_EINVAL, "attention operands need 16-byte aligned rows");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (bf16)
            dit_attention<__nv_bfloat16>(q, q_row, q_seq, k, v, kv_row, kv_seq, o, o_row, o_seq, lq, lk, kv_rep,
                                         heads, nseq, ctx->status.as<int>(), st);
        else
            dit_attention<__half>(q, q_row, q_seq, k, v, kv_row, kv_seq, o, o_row, o_seq, lq, lk, kv_rep, heads,
                                  nseq, ctx->status.as<int>(), st);
    });
}

b2d_status b2d_dit_load(b2d_ctx* ctx, const b2d_dit_config* config, const b2d_tensor_view* tensors,
                        int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0))
            fail(B2D_EINVAL, "Stable Audio Foundation RF DiT runtime requires assets");
        const b2d_dit_config& c = *config;
        if (c.num_heads <= 0 || c.embed_dim % c.num_heads != 0)
            fail(B2D_EINVAL, "Stable Audio Foundation RF DiT head dimensions are invalid");
        if (c.embed_dim / c.num_heads != 64) fail(B2D_EINVAL, "head_dim must be 64 on this path");
        if (c.cond_token_dim <= 0 || c.cond_token_dim % 64 != 0)
            fail(B2D_EINVAL, "Stable Audio Foundation RF DiT context head dimensions are invalid");
        if (c.num_heads % (c.cond_token_dim / 64) != 0)
            fail(B2D_EINVAL, "Stable Audio Foundation cross-attention head repeat mismatch");
        if (c.io_channels != 64) fail(B2D_EINVAL, "io_channels must be 64 on this path");
        if (c.embed_dim % 256 || c.cond_token_dim % 128 || c.global_cond_dim % 64 || c.depth <= 0)
            fail(B2D_EINVAL, "embed_dim must be a multiple of 256 and cond_token_dim of 128");
        auto m = std::make_unique<DitModel>();
        m->cfg = c;
        m->d = c.embed_dim;
        m->heads = c.num_heads;
        m->c = c.cond_token_dim;
        m->gd = c.global_cond_dim;
        m->P2 = c.prompt_max_length + 2;
        m->ffi = 4 * c.embed_dim;
        m->kvh = c.cond_token_dim / 64;
        const b2d_tensor_view* probe =
            find_tensor(tensors, n_tensors, "model.model.transformer.layers.0.self_attn.to_qkv.weight");
        m->bf16 = probe && probe->ggml_type == B2D_TYPE_BF16;
        ctx->dit.reset();
        if (m->bf16)
            dit_load_t<__nv_bfloat16>(ctx, *m, tensors, n_tensors);
        else
            dit_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->dit = std::move(m);
    });
}

static b2d_status dit_sample_common(b2d_ctx* ctx, const b2d_dit_request* rq, float* out, void* stream, bool host) {
    return guarded(ctx, [&] {
        if (!ctx->dit) fail(B2D_ESTATE, "Stable Audio Foundation RF DiT weights are not loaded");
        if (!rq || !out) fail(B2D_EINVAL, "Stable Audio Foundation RF DiT request is null");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (ctx->dit->bf16)
            dit_sample<__nv_bfloat16>(ctx, *rq, out, st, host);
        else
            dit_sample<__half>(ctx, *rq, out, st, host);
    });
}

b2d_status b2d_dit_sample(b2d_ctx* ctx, const b2d_dit_request* request, float* out_latents, void* stream) {
    return dit_sample_common(ctx, request, out_latents, stream, true);
}

b2d_status b2d_dit_sample_device(b2d_ctx* ctx, const b2d_dit_request* request, float* out_latents, void* stream) {
    return dit_sample_common(ctx, request, out_latents, stream, false);
}

b2d_status b2d_sa3_load(b2d_ctx* ctx, const b2d_sa3_config* config, const b2d_tensor_view* tensors,
                        int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0)) fail(B2D_EINVAL, "Stable Audio RF DiT runtime requires assets");
        const b2d_sa3_config& c = *config;
        if (c.num_heads <= 0 || c.embed_dim % c.num_heads != 0)
            fail(B2D_EINVAL, "Stable Audio RF DiT head dimensions are invalid");
        if (c.embed_dim / c.num_heads != 64) fail(B2D_EINVAL, "head_dim must be 64 on this path");
        if (c.io_channels != 64) fail(B2D_EINVAL, "io_channels must be 64 on this path");
        if (c.embed_dim % 128 || c.embed_dim > 4096 || c.cond_dim <= 0 || c.cond_dim % 64 || c.global_cond_dim <= 0 ||
            c.global_cond_dim % 64 || c.local_add_cond_dim <= 0 || c.num_memory_tokens <= 0 || c.depth <= 0 ||
            c.prompt_max_length < 0)
            fail(B2D_EINVAL, "embed_dim must be a multiple of 128 (<= 4096), cond_dim and global_cond_dim of 64");
        auto m = std::make_unique<Sa3Model>();
        m->cfg = c;
        m->d = c.embed_dim;
        m->heads = c.num_heads;
        m->cd = c.cond_dim;
        m->gd = c.global_cond_dim;
        m->la = c.local_add_cond_dim;
        m->lak = (c.local_add_cond_dim + 63) / 64 * 64;
        m->M = c.num_memory_tokens;
        m->P1 = c.prompt_max_length + 1;
        m->F = 4 * c.embed_dim;
        m->nq = c.differential_attention ? 5 : 3;
        m->nqc = c.differential_attention ? 2 : 1;
        m->nkv = c.differential_attention ? 3 : 2;
        const b2d_tensor_view* probe =
            find_tensor(tensors, n_tensors, "model.model.transformer.layers.0.self_attn.to_qkv.weight");
        m->bf16 = probe && probe->ggml_type == B2D_TYPE_BF16;
        ctx->sa3.reset();
        if (m->bf16)
            sa3_load_t<__nv_bfloat16>(ctx, *m, tensors, n_tensors);
        else
            sa3_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->sa3 = std::move(m);
    });
}

static b2d_status sa3_sample_common(b2d_ctx* ctx, const b2d_sa3_request* rq, float* out, void* stream, bool host) {
    return guarded(ctx, [&] {
        if (!ctx->sa3) fail(B2D_ESTATE, "Stable Audio RF DiT weights are not loaded");
        if (!rq || !out) fail(B2D_EINVAL, "Stable Audio RF DiT request is null");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (ctx->sa3->bf16)
            sa3_sample<__nv_bfloat16>(ctx, *rq, out, st, host);
        else
            sa3_sample<__half>(ctx, *rq, out, st, host);
    });
}

b2d_status b2d_sa3_sample(b2d_ctx* ctx, const b2d_sa3_request* request, float* out_latents, void* stream) {
    return sa3_sample_common(ctx, request, out_latents, stream, true);
}

b2d_status b2d_sa3_sample_device(b2d_ctx* ctx, const b2d_sa3_request* request, float* out_latents, void* stream) {
    return sa3_sample_common(ctx, request, out_latents, stream, false);
}

b2d_status b2d_oobleck_load(b2d_ctx* ctx, const b2d_oobleck_config* config, const b2d_tensor_view* tensors,
                            int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0))
            fail(B2D_EINVAL, "Stable Audio Foundation Oobleck runtime requires assets");
        const b2d_oobleck_config& c = *config;
        if (c.n_blocks <= 0 || c.n_blocks > 8 || c.channels <= 0 || c.latent_dim <= 0 || c.latent_dim % 64 ||
            c.audio_channels <= 0 || c.audio_channels > 64)
            fail(B2D_EINVAL, "Oobleck config: latent_dim must be a multiple of 64, 1..8 blocks, 1..64 audio channels");
        for (int i = 0; i < c.n_blocks; ++i)
            if (c.c_mults[i] <= 0 || c.strides[i] <= 0) fail(B2D_EINVAL, "Oobleck config: c_mults / strides must be positive");
        auto m = std::make_unique<OobModel>();
        m->cfg = c;
        ctx->oob.reset();
        oob_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->oob = std::move(m);
    });
}

static b2d_status oob_decode_common(b2d_ctx* ctx, const float* latents, int64_t batch, int64_t latent_tokens,
                                    float* audio, void* stream, bool host) {
    return guarded(ctx, [&] {
        if (!ctx->oob) fail(B2D_ESTATE, "Stable Audio Foundation Oobleck weights are not loaded");
        oob_decode<__half>(ctx, latents, batch, latent_tokens, audio, static_cast<cudaStream_t>(stream), host);
    });
}

b2d_status b2d_oobleck_decode(b2d_ctx* ctx, const float* latents, int64_t batch, int64_t latent_tokens, float* audio,
                              void* stream) {
    return oob_decode_common(ctx, latents, batch, latent_tokens, audio, stream, true);
}

b2d_status b2d_oobleck_decode_device(b2d_ctx* ctx, const float* latents, int64_t batch, int64_t latent_tokens,
                                     float* audio, void* stream) {
    return oob_decode_common(ctx, latents, batch, latent_tokens, audio, stream, false);
}

b2d_status b2d_vvdec_load(b2d_ctx* ctx, const b2d_vvdec_config* config, const b2d_tensor_view* tensors,
                          int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0)) fail(B2D_EINVAL, "VibeVoice tokenizer weights runtime requires assets");
        const b2d_vvdec_config& c = *config;
        // stages narrower than 64 channels (the released decoders' 32-channel last stage) run zero-padded to 64
        if (c.n_stages < 1 || c.n_stages > 8 || c.vae_dim <= 0 || c.vae_dim % 64 || c.n_filters <= 0 ||
            c.n_filters % 32)
            fail(B2D_EINVAL, "tokenizer decoder config: 1..8 stages, vae_dim a multiple of 64, n_filters of 32");
        for (int i = 0; i < c.n_stages; ++i)
            if (c.depths[i] <= 0 || (i + 1 < c.n_stages && c.ratios[i] <= 0))
                fail(B2D_EINVAL, "tokenizer decoder config: depths / ratios must be positive");
        auto m = std::make_unique<VdModel>();
        m->cfg = c;
        ctx->vvdec.reset();
        vd_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->vvdec = std::move(m);
    });
}

static b2d_status vd_decode_common(b2d_ctx* ctx, const float* latents, int64_t frames, float* samples, void* stream,
                                   bool host) {
    return guarded(ctx, [&] {
        if (!ctx->vvdec) fail(B2D_ESTATE, "VibeVoice acoustic decoder weights are not loaded");
        vd_decode<__half>(ctx, latents, frames, samples, static_cast<cudaStream_t>(stream), host);
    });
}

b2d_status b2d_vvdec_decode(b2d_ctx* ctx, const float* latents, int64_t frames, float* samples, void* stream) {
    return vd_decode_common(ctx, latents, frames, samples, stream, true);
}

b2d_status b2d_vvdec_decode_device(b2d_ctx* ctx, const float* latents, int64_t frames, float* samples,
                                   void* stream) {
    return vd_decode_common(ctx, latents, frames, samples, stream, false);
}

b2d_status b2d_saocond_load(b2d_ctx* ctx, const b2d_saocond_config* config, const b2d_tensor_view* tensors,
                            int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0)) fail(B2D_EINVAL, "Stable Audio Foundation conditioner requires assets");
        const b2d_saocond_config& c = *config;
        if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.vocab <= 0 || c.intermediate <= 0 ||
            c.prompt_max_length <= 0 || (c.head_dim != 64 && c.head_dim != 32))
            fail(B2D_EINVAL, "T5BaseEncoderConfig dimensions must be positive (head_dim 32 or 64 on this path)");
        if (c.hidden % 64 || (c.heads * c.head_dim) % 64 || c.intermediate % 64)
            fail(B2D_EINVAL, "T5 hidden, heads x head_dim and intermediate sizes must be multiples of 64");
        auto m = std::make_unique<T5Model>();
        m->cfg = c;
        ctx->t5.reset();
        t5_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->t5 = std::move(m);
    });
}

static b2d_status t5_encode_common(b2d_ctx* ctx, const int32_t* ids, const float* mask, const float* seconds,
                                   int64_t batch, float* cross, float* cross_mask, float* global, void* stream,
                                   bool host) {
    return guarded(ctx, [&] {
        if (!ctx->t5) fail(B2D_ESTATE, "Stable Audio Foundation conditioner weights are not loaded");
        t5_encode<__half>(ctx, ids, mask, seconds, batch, cross, cross_mask, global, static_cast<cudaStream_t>(stream),
                          host);
    });
}

b2d_status b2d_saocond_encode(b2d_ctx* ctx, const int32_t* input_ids, const float* attention_mask,
                              const float* normalized_seconds, int64_t batch, float* cross, float* cross_mask,
                              float* global_cond, void* stream) {
    return t5_encode_common(ctx, input_ids, attention_mask, normalized_seconds, batch, cross, cross_mask, global_cond,
                            stream, true);
}

b2d_status b2d_saocond_encode_device(b2d_ctx* ctx, const int32_t* input_ids, const float* attention_mask,
                                     const float* normalized_seconds, int64_t batch, float* cross, float* cross_mask,
                                     float* global_cond, void* stream) {
    return t5_encode_common(ctx, input_ids, attention_mask, normalized_seconds, batch, cross, cross_mask, global_cond,
                            stream, false);
}

b2d_status b2d_vvlm_load(b2d_ctx* ctx, const b2d_vvlm_config* config, const b2d_tensor_view* tensors,
                         int32_t n_tensors) {
    return guarded(ctx, [&] {
        if (!config || (!tensors && n_tensors > 0)) fail(B2D_EINVAL, "VibeVoice decoder weights require model weights");
        const b2d_vvlm_config& c = *config;
        if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
            c.vocab <= 0 || c.max_positions <= 0 || (c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128))
            fail(B2D_EINVAL, "VibeVoice decoder config: positive sizes, heads a multiple of kv_heads, head_dim 32/64/128");
        if (c.hidden % 64 || c.intermediate % 64 || (c.heads * c.head_dim) % 64)
            fail(B2D_EINVAL, "VibeVoice decoder hidden, intermediate and heads x head_dim must be multiples of 64");
        auto m = std::make_unique<LmModel>();
        m->cfg = c;
        ctx->lm.reset();
        lm_load_t<__half>(ctx, *m, tensors, n_tensors);
        ctx->lm = std::move(m);
    });
}

b2d_status b2d_vvlm_prefill(b2d_ctx* ctx, const float* embeddings, int64_t steps, float* logits, float* last_hidden,
                            void* stream) {
    return guarded(ctx, [&] {
        if (!ctx->lm) fail(B2D_ESTATE, "VibeVoice decoder weights are not loaded");
        ctx->lm->pos = 0;
        lm_forward<__half>(ctx, embeddings, steps, logits, last_hidden, static_cast<cudaStream_t>(stream));
    });
}

b2d_status b2d_vvlm_step(b2d_ctx* ctx, const float* embedding, float* logits, float* last_hidden, void* stream) {
    return guarded(ctx, [&] {
        if (!ctx->lm) fail(B2D_ESTATE, "VibeVoice decoder weights are not loaded");
        if (ctx->lm->pos == 0) fail(B2D_ESTATE, "VibeVoice decoder cached step before prefill");
        lm_forward<__half>(ctx, embedding, 1, logits, last_hidden, static_cast<cudaStream_t>(stream));
    });
}

b2d_status b2d_vvlm_prefill_device(b2d_ctx* ctx, const float* embeddings, int64_t steps, float* logits,
                                   float* last_hidden, void* stream) {
    return guarded(ctx, [&] {
        if (!ctx->lm) fail(B2D_ESTATE, "VibeVoice decoder weights are not loaded");
        ctx->lm->pos = 0;
        lm_forward<__half>(ctx, embeddings, steps, logits, last_hidden, static_cast<cudaStream_t>(stream), true);
    });
}

b2d_status b2d_vvlm_step_device(b2d_ctx* ctx, const float* embedding, float* logits, float* last_hidden,
                                void* stream) {
    return guarded(ctx, [&] {
        if (!ctx->lm) fail(B2D_ESTATE, "VibeVoice decoder weights are not loaded");
        if (ctx->lm->pos == 0) fail(B2D_ESTATE, "VibeVoice decoder cached step before prefill");
        lm_forward<__half>(ctx, embedding, 1, logits, last_hidden, static_cast<cudaStream_t>(stream), true);
    });
}

}  // extern "C"
