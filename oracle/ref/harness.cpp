// Test-infrastructure harness around the reference's own CPU implementation of
// the diffusion hot path.  It links the unmodified audio.cpp translation units
// (VibeVoice diffusion head / DPM-Solver++ scheduler / sampler, Stable Audio
// Open 1.0 foundation DiT) and vendored ggml's CPU backend, feeds them weights
// and inputs from a "B2DB" bundle file written by oracle/bundle.py, and writes
// the reference's outputs (and wall-clock timings) back as a bundle.
//
// Commands (all inputs/outputs are bundles):
//   q8     <in> <out>                      ggml_quantize_chunk(Q8_0) + dequantize of rows "x"
//   vvsched <in> <out>                     VibeVoiceDPMSolverScheduler::step over given model outputs
//   vvpredict <weights> <in> <out> <thr>   one VibeVoiceDiffusionHeadWeightsRuntime::predict
//   vv <weights> <in> <out> <thr> <reps>   sample_vibevoice_speech_latents (whole step loop)
//   dit <weights> <in> <out> <thr> <reps> FoundationRfDitRuntime::sample
//   dit_fresh <weights> <in> <out> <thr> <reps>  the same DPM++ 2M trajectory with a fresh FoundationRfDitRuntime
//                                         for every model evaluation (see cmd_dit)
//   sa3 <weights> <in> <out> <thr> <reps> StableAudioRfDitRuntime::sample (Stable Audio 3 DiT)
//
// Reference entry points exercised (paths inside audio.cpp):
//   include/engine/models/vibevoice/diffusion_sampler.h:23  sample_vibevoice_speech_latents
//   include/engine/models/vibevoice/diffusion_head.h:58-97  VibeVoiceDiffusionHeadWeightsRuntime
//   include/engine/models/vibevoice/scheduler.h:14-47       VibeVoiceDPMSolverScheduler
//   include/engine/models/stable_audio/foundation/rf_dit.h:73-106 FoundationRfDitRuntime
//   external/ggml/src/ggml-quants.c:234-257,491-505         Q8_0 quantize / dequantize

#include "engine/framework/assets/tensor_source.h"
#include "engine/framework/core/execution_context.h"
#include "engine/framework/sampling/torch_random.h"
#include "engine/models/stable_audio/foundation/conditioner.h"
#include "engine/models/stable_audio/foundation/oobleck_autoencoder.h"
#include "engine/models/stable_audio/foundation/rf_dit.h"
#include "engine/models/stable_audio/rf_dit.h"
#include "engine/models/vibevoice/decoder.h"
#include "engine/models/vibevoice/diffusion_head.h"
#include "engine/models/vibevoice/diffusion_sampler.h"
#include "engine/models/vibevoice/scheduler.h"
#include "engine/models/vibevoice/tokenizer_audio.h"

#include "engine/framework/io/yaml.h"

#include <ggml.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

// Backend the reference runtimes are created on: CPU unless B2D_REF_BACKEND=cuda (a build with VARIANT=cuda, which
// links the vendored ggml-cuda backend; device 0).  The CUDA backend is a timing comparison point only.
engine::core::BackendType ref_backend() {
    const char * b = std::getenv("B2D_REF_BACKEND");
    if (b != nullptr && std::strcmp(b, "cuda") == 0) return engine::core::BackendType::Cuda;
    return engine::core::BackendType::Cpu;
}

// ---------------------------------------------------------------- bundle I/O
// Layout: "B2DB" u32 version u32 count, then per entry
//   u16 name_len, name, u8 dtype, u8 ndim, i64 dims[ndim], u64 nbytes, bytes.
enum Dtype : uint8_t { F32 = 0, F16 = 1, BF16 = 2, Q8_0 = 3, I64 = 4, I32 = 5, U8 = 6 };

struct Entry {
    uint8_t dtype = F32;
    std::vector<int64_t> dims;
    std::vector<std::byte> bytes;
};

using Bundle = std::map<std::string, Entry>;

template <typename T>
void read_pod(std::ifstream & in, T & v) {
    in.read(reinterpret_cast<char *>(&v), sizeof(T));
    if (!in) throw std::runtime_error("bundle truncated");
}

Bundle read_bundle(const std::string & path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot open bundle " + path);
    char magic[4];
    in.read(magic, 4);
    if (std::memcmp(magic, "B2DB", 4) != 0) throw std::runtime_error("bad bundle magic: " + path);
    uint32_t version = 0, count = 0;
    read_pod(in, version);
    read_pod(in, count);
    Bundle out;
    for (uint32_t i = 0; i < count; ++i) {
        uint16_t nlen = 0;
        read_pod(in, nlen);
        std::string name(nlen, '\0');
        in.read(name.data(), nlen);
        Entry e;
        uint8_t ndim = 0;
        read_pod(in, e.dtype);
        read_pod(in, ndim);
        e.dims.resize(ndim);
        for (auto & d : e.dims) read_pod(in, d);
        uint64_t nbytes = 0;
        read_pod(in, nbytes);
        e.bytes.resize(nbytes);
        in.read(reinterpret_cast<char *>(e.bytes.data()), static_cast<std::streamsize>(nbytes));
        if (!in) throw std::runtime_error("bundle truncated in " + name);
        out.emplace(std::move(name), std::move(e));
    }
    return out;
}

void write_bundle(const std::string & path, const Bundle & b) {
    std::ofstream out(path, std::ios::binary);
    out.write("B2DB", 4);
    const uint32_t version = 1, count = static_cast<uint32_t>(b.size());
    out.write(reinterpret_cast<const char *>(&version), 4);
    out.write(reinterpret_cast<const char *>(&count), 4);
    for (const auto & [name, e] : b) {
        const uint16_t nlen = static_cast<uint16_t>(name.size());
        out.write(reinterpret_cast<const char *>(&nlen), 2);
        out.write(name.data(), nlen);
        out.write(reinterpret_cast<const char *>(&e.dtype), 1);
        const uint8_t ndim = static_cast<uint8_t>(e.dims.size());
        out.write(reinterpret_cast<const char *>(&ndim), 1);
        for (int64_t d : e.dims) out.write(reinterpret_cast<const char *>(&d), 8);
        const uint64_t nbytes = e.bytes.size();
        out.write(reinterpret_cast<const char *>(&nbytes), 8);
        out.write(reinterpret_cast<const char *>(e.bytes.data()), static_cast<std::streamsize>(nbytes));
    }
    if (!out) throw std::runtime_error("cannot write bundle " + path);
}

const Entry & need(const Bundle & b, const std::string & name) {
    auto it = b.find(name);
    if (it == b.end()) throw std::runtime_error("bundle lacks entry " + name);
    return it->second;
}

std::vector<float> f32s(const Bundle & b, const std::string & name) {
    const auto & e = need(b, name);
    if (e.dtype != F32) throw std::runtime_error("entry is not f32: " + name);
    std::vector<float> v(e.bytes.size() / 4);
    std::memcpy(v.data(), e.bytes.data(), e.bytes.size());
    return v;
}

std::vector<int64_t> i64s(const Bundle & b, const std::string & name) {
    const auto & e = need(b, name);
    if (e.dtype != I64) throw std::runtime_error("entry is not i64: " + name);
    std::vector<int64_t> v(e.bytes.size() / 8);
    std::memcpy(v.data(), e.bytes.data(), e.bytes.size());
    return v;
}

float f32_scalar(const Bundle & b, const std::string & name) { return f32s(b, name).at(0); }
int64_t i64_scalar(const Bundle & b, const std::string & name) { return i64s(b, name).at(0); }

Entry f32_entry(const std::vector<float> & v, std::vector<int64_t> dims) {
    Entry e;
    e.dtype = F32;
    e.dims = std::move(dims);
    e.bytes.resize(v.size() * 4);
    std::memcpy(e.bytes.data(), v.data(), e.bytes.size());
    return e;
}

Entry raw_entry(uint8_t dtype, const void * p, size_t n, std::vector<int64_t> dims) {
    Entry e;
    e.dtype = dtype;
    e.dims = std::move(dims);
    e.bytes.resize(n);
    std::memcpy(e.bytes.data(), p, n);
    return e;
}

const char * dtype_name(uint8_t d) {
    switch (d) {
        case F32: return "f32";
        case F16: return "f16";
        case BF16: return "bf16";
        case Q8_0: return "q8_0";
        case I64: return "i64";
        case I32: return "i32";
        default: return "u8";
    }
}

// ------------------------------------------------- in-memory tensor source
// Serves a bundle's entries through the reference's TensorSource interface
// (include/engine/framework/assets/tensor_source.h:59-120) so the reference's
// own weight loaders and BackendWeightStore upload path run unchanged.
class BundleTensorSource final : public engine::assets::TensorSource {
public:
    explicit BundleTensorSource(Bundle b) : bundle_(std::move(b)) {}

    const std::filesystem::path & source_path() const noexcept override { return path_; }
    bool has_tensor(std::string_view name) const noexcept override {
        return bundle_.count(std::string(name)) != 0;
    }
    engine::assets::TensorMetadata require_metadata(std::string_view name) const override {
        const auto & e = need(bundle_, std::string(name));
        return {std::string(name), dtype_name(e.dtype), e.dims};
    }
    std::vector<engine::assets::TensorMetadata> tensors() const override {
        std::vector<engine::assets::TensorMetadata> out;
        for (const auto & [n, e] : bundle_) out.push_back({n, dtype_name(e.dtype), e.dims});
        return out;
    }
    engine::assets::RawTensorData require_tensor_data(std::string_view name) const override {
        const auto & e = need(bundle_, std::string(name));
        return {{std::string(name), dtype_name(e.dtype), e.dims}, e.bytes};
    }
    std::vector<float> require_f32(
        std::string_view name,
        const std::optional<std::vector<int64_t>> & expected_shape) const override {
        const auto & e = need(bundle_, std::string(name));
        if (expected_shape && *expected_shape != e.dims) {
            throw std::runtime_error("tensor shape mismatch for " + std::string(name));
        }
        return f32s(bundle_, std::string(name));
    }
    std::optional<std::vector<float>> optional_f32(
        std::string_view name,
        const std::optional<std::vector<int64_t>> & expected_shape) const override {
        if (!has_tensor(name)) return std::nullopt;
        return require_f32(name, expected_shape);
    }
    int64_t require_i64_scalar(std::string_view name) const override {
        return i64_scalar(bundle_, std::string(name));
    }

private:
    Bundle bundle_;
    std::filesystem::path path_ = "bundle";
};

double now_ms() {
    using namespace std::chrono;
    return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

// ----------------------------------------------------------- VibeVoice
engine::models::vibevoice::VibeVoiceDiffusionHeadConfig head_config(const Bundle & in) {
    engine::models::vibevoice::VibeVoiceDiffusionHeadConfig c;
    c.hidden_size = i64_scalar(in, "hidden_size");
    c.latent_size = i64_scalar(in, "latent_size");
    c.head_layers = i64_scalar(in, "head_layers");
    c.head_ffn_ratio = f32_scalar(in, "head_ffn_ratio");
    c.rms_norm_eps = f32_scalar(in, "rms_norm_eps");
    c.ddpm_num_steps = i64_scalar(in, "ddpm_num_steps");
    c.ddpm_num_inference_steps = i64_scalar(in, "inference_steps");
    c.ddpm_beta_schedule = "cosine";
    c.diffusion_type = "ddpm";
    c.prediction_type = "v_prediction";
    return c;
}

std::shared_ptr<const engine::models::vibevoice::VibeVoiceAssets> head_assets(
    const std::string & weights_path, const Bundle & in) {
    auto assets = std::make_shared<engine::models::vibevoice::VibeVoiceAssets>();
    assets->config.diffusion_head = head_config(in);
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(weights_path));
    return assets;
}

int cmd_vvsched(const std::string & in_path, const std::string & out_path) {
    const Bundle in = read_bundle(in_path);
    auto cfg = head_config(in);
    const int64_t steps = i64_scalar(in, "inference_steps");
    auto sample = f32s(in, "sample");
    const auto outputs = f32s(in, "model_outputs");
    const size_t n = sample.size();
    engine::models::vibevoice::VibeVoiceDPMSolverScheduler sched(cfg);
    sched.set_timesteps(steps);
    std::vector<float> trace;
    std::vector<float> ts;
    for (size_t s = 0; s < sched.timesteps().size(); ++s) {
        std::vector<float> mo(outputs.begin() + static_cast<std::ptrdiff_t>(s * n),
                              outputs.begin() + static_cast<std::ptrdiff_t>((s + 1) * n));
        sample = sched.step(mo, sched.timesteps()[s], sample).prev_sample;
        trace.insert(trace.end(), sample.begin(), sample.end());
        ts.push_back(static_cast<float>(sched.timesteps()[s]));
    }
    Bundle out;
    out["trace"] = f32_entry(trace, {steps, static_cast<int64_t>(n)});
    out["timesteps"] = f32_entry(ts, {steps});
    write_bundle(out_path, out);
    return 0;
}

int cmd_vvpredict(const std::string & w, const std::string & in_path, const std::string & out_path, int threads) {
    const Bundle in = read_bundle(in_path);
    auto assets = head_assets(w, in);
    engine::models::vibevoice::VibeVoiceDiffusionHeadWeightsRuntime head(
        assets, ref_backend(), 0, threads);
    const auto noisy = f32s(in, "noisy");
    const auto cond = f32s(in, "condition");
    const int64_t latent = assets->config.diffusion_head.latent_size;
    const int64_t hidden = assets->config.diffusion_head.hidden_size;
    const int64_t frames = static_cast<int64_t>(noisy.size()) / latent;
    auto pred = head.predict(noisy, frames, latent, f32_scalar(in, "timestep"), cond, hidden);
    Bundle out;
    out["prediction"] = f32_entry(pred.values, {frames, latent});
    write_bundle(out_path, out);
    return 0;
}

int cmd_vv(const std::string & w, const std::string & in_path, const std::string & out_path, int threads, int reps) {
    const Bundle in = read_bundle(in_path);
    auto assets = head_assets(w, in);
    const auto & cfg = assets->config.diffusion_head;
    // optional "storage_type": assets::TensorStorageType value for the weight store (quantize-on-load)
    const auto storage = in.count("storage_type")
                             ? static_cast<engine::assets::TensorStorageType>(i64_scalar(in, "storage_type"))
                             : engine::assets::TensorStorageType::Native;
    engine::models::vibevoice::VibeVoiceDiffusionHeadWeightsRuntime head(
        assets, ref_backend(), 0, threads, 64ull * 1024ull * 1024ull, 64ull * 1024ull * 1024ull,
        storage);
    engine::models::vibevoice::VibeVoiceDPMSolverScheduler sched(cfg);
    engine::models::vibevoice::VibeVoiceSpeechDiffusionInput input;
    input.positive_condition = f32s(in, "positive_condition");
    input.negative_condition = f32s(in, "negative_condition");
    input.initial_speech = f32s(in, "initial_speech");
    input.hidden_size = cfg.hidden_size;
    input.latent_size = cfg.latent_size;
    input.batch_size = static_cast<int64_t>(input.positive_condition.size()) / cfg.hidden_size;
    input.inference_steps = i64_scalar(in, "inference_steps");
    input.guidance_scale = f32_scalar(in, "guidance_scale");
    sched.set_timesteps(input.inference_steps);
    std::vector<float> times;
    std::vector<float> latents;
    for (int r = 0; r < std::max(reps, 1); ++r) {
        const double t0 = now_ms();
        auto result = engine::models::vibevoice::sample_vibevoice_speech_latents(head, sched, input);
        times.push_back(static_cast<float>(now_ms() - t0));
        latents.clear();
        for (const auto & l : result) latents.insert(latents.end(), l.values.begin(), l.values.end());
    }
    Bundle out;
    out["latents"] = f32_entry(latents, {input.batch_size, input.latent_size});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ---------------------------------------------------------- Stable Audio DiT
int cmd_dit(const std::string & w, const std::string & in_path, const std::string & out_path, int threads, int reps,
            bool fresh_graph_per_step = false) {
    namespace sa = engine::models::stable_audio;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<sa::StableAudioAssets>();
    auto & c = assets->config;
    c.io_channels = i64_scalar(in, "io_channels");
    c.embed_dim = i64_scalar(in, "embed_dim");
    c.depth = i64_scalar(in, "depth");
    c.num_heads = i64_scalar(in, "num_heads");
    c.cond_token_dim = i64_scalar(in, "cond_token_dim");
    c.global_cond_dim = i64_scalar(in, "global_cond_dim");
    c.prompt_max_length = i64_scalar(in, "prompt_max_length");
    c.stable_audio_open_v1 = true;
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(w));

    const int64_t batch = i64_scalar(in, "batch");
    const int64_t tokens = i64_scalar(in, "latent_tokens");
    const int64_t steps = i64_scalar(in, "steps");
    sa::StableAudioSamplingState sampling;
    sampling.batch = batch;
    sampling.latent_sample_size = tokens;
    sampling.channels = c.io_channels;
    sampling.schedule_points = steps + 1;
    sampling.schedule.assign(static_cast<size_t>(batch * (steps + 1)), 0.0F);
    sampling.padding_mask = f32s(in, "padding_mask");
    sampling.noise = f32s(in, "noise");

    sa::StableAudioConditioningInputs cond;
    const int64_t cross_tokens = c.prompt_max_length + 2;
    cond.positive.batch = batch;
    cond.positive.cross_tokens = cross_tokens;
    cond.positive.cond_dim = c.cond_token_dim;
    cond.positive.cross_attention = f32s(in, "cross_positive");
    cond.positive.global = f32s(in, "global");
    cond.has_negative = i64_scalar(in, "has_negative") != 0;
    if (cond.has_negative) {
        cond.negative = cond.positive;
        cond.negative.cross_attention = f32s(in, "cross_negative");
    }
    const float cfg_scale = f32_scalar(in, "cfg_scale");
    const float apg_scale = f32_scalar(in, "apg_scale");
    // sampler: 0 "dpmpp-2m", 1 "dpmpp-3m-sde", 2 "" (v-DDIM on sampling.schedule)
    const int64_t sampler = in.count("sampler") ? i64_scalar(in, "sampler") : 0;
    const uint64_t seed = in.count("seed") ? static_cast<uint64_t>(i64_scalar(in, "seed")) : 0;
    if (in.count("schedule")) sampling.schedule = f32s(in, "schedule");
    const char * sampler_name = sampler == 1 ? "dpmpp-3m-sde" : (sampler == 2 ? "" : "dpmpp-2m");
    const float sigma_min = f32_scalar(in, "sigma_min");
    const float sigma_max = f32_scalar(in, "sigma_max");
    const float rho = f32_scalar(in, "rho");

    engine::core::ExecutionContext exec({ref_backend(), 0, threads});
    const auto storage = in.count("storage_type")
                             ? static_cast<engine::assets::TensorStorageType>(i64_scalar(in, "storage_type"))
                             : engine::assets::TensorStorageType::Native;
    sa::foundation::FoundationRfDitRuntime dit(exec, assets, storage);
    engine::sampling::TorchCudaSamplingPolicy policy;
    if (in.count("rng_sms")) policy.multiprocessor_count = i64_scalar(in, "rng_sms");
    if (in.count("rng_max_threads")) policy.max_threads_per_multiprocessor = i64_scalar(in, "rng_max_threads");
    std::vector<float> times;
    uint64_t final_offset = 0;
    std::vector<float> result;
    if (fresh_graph_per_step) {
        // FoundationRfDitRuntime computes correctly only on the first compute of its graph: its RoPE positions
        // input is written once, when the graph is built (src/models/stable_audio/foundation/rf_dit.cpp:928-932),
        // and ggml's graph allocator hands an input's memory to later nodes once its last consumer has run
        // (external/ggml/src/ggml-alloc.c:692, 803-815), so every later compute reads stale positions.  Here each
        // model evaluation runs on a fresh runtime (a one-step sample from sigma_i, which returns the denoised
        // latent), and the DPM++ 2M update of sample_dpmpp_2m (rf_dit.cpp:814-872) is restated around it.
        if (sampler != 0) throw std::runtime_error("dit_fresh supports the dpmpp-2m sampler only");
        const double t0 = now_ms();
        std::vector<float> sig(static_cast<size_t>(steps + 1), 0.0F);
        for (int64_t i = 0; i < steps; ++i) {
            const float ramp = steps == 1 ? 1.0F
                                          : std::pow(1.0F - static_cast<float>(i) / static_cast<float>(steps - 1), rho);
            sig[static_cast<size_t>(i)] = std::exp(ramp * (std::log(sigma_max) - std::log(sigma_min)) + std::log(sigma_min));
        }
        std::vector<float> x = sampling.noise;
        for (float & v : x) v *= sig[0];
        std::vector<float> old;
        sa::StableAudioSamplingState one = sampling;
        one.schedule_points = 2;
        one.schedule.assign(static_cast<size_t>(batch * 2), 0.0F);
        for (int64_t step = 0; step < steps; ++step) {
            const float s = sig[static_cast<size_t>(step)], sn = sig[static_cast<size_t>(step + 1)];
            for (size_t i = 0; i < x.size(); ++i) one.noise[i] = x[i] / s;
            sa::foundation::FoundationRfDitRuntime fresh(exec, assets, storage);
            fresh.prepare(one, cfg_scale);
            uint64_t offset = 0;
            std::vector<float> den = fresh.sample(one, cond, seed, offset, policy, sampler_name, 0.5F * s, s, rho,
                                                  cfg_scale, apg_scale);
            std::fprintf(stderr, "dit_fresh step %lld / %lld sigma %g\n", static_cast<long long>(step + 1),
                         static_cast<long long>(steps), static_cast<double>(s));
            if (sn == 0.0F) {
                x = std::move(den);
                break;
            }
            const float h = -std::log(sn) + std::log(s);
            const float x_scale = sn / s;
            const float den_scale = -std::expm1(-h);
            if (old.empty()) {
                for (size_t i = 0; i < x.size(); ++i) x[i] = x_scale * x[i] + den_scale * den[i];
            } else {
                const float h_last = std::log(sig[static_cast<size_t>(step - 1)]) - std::log(s);
                const float r = h_last / h;
                const float dc = 1.0F + 1.0F / (2.0F * r), oc = -1.0F / (2.0F * r);
                for (size_t i = 0; i < x.size(); ++i) x[i] = x_scale * x[i] + den_scale * (dc * den[i] + oc * old[i]);
            }
            old = std::move(den);
        }
        result = std::move(x);
        times.push_back(static_cast<float>(now_ms() - t0));
        reps = 0;
    } else {
        dit.prepare(sampling, cfg_scale);
        reps = std::max(reps, 1);
    }
    for (int r = 0; r < reps; ++r) {
        uint64_t offset = in.count("rng_offset") ? static_cast<uint64_t>(i64_scalar(in, "rng_offset")) : 0;
        const double t0 = now_ms();
        result = dit.sample(sampling, cond, seed, offset, policy, sampler_name, sigma_min, sigma_max, rho, cfg_scale,
                            apg_scale);
        times.push_back(static_cast<float>(now_ms() - t0));
        final_offset = offset;
    }
    Bundle out;
    const int64_t fo = static_cast<int64_t>(final_offset);
    out["rng_offset_out"] = raw_entry(I64, &fo, 8, {1});
    out["latents"] = f32_entry(result, {batch, c.io_channels, tokens});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ------------------------------------------------------ Stable Audio 3 DiT
// StableAudioRfDitRuntime::sample (src/models/stable_audio/rf_dit.cpp:586-694): rectified-flow DiT with
// memory tokens, local-add conditioning, qk-RMSNorm, optional differential attention, 6-way adaLN,
// APG-CFG when cfg_scale != 1, and the pingpong (Philox noise) or euler sampler on sampling.schedule.
int cmd_sa3(const std::string & w, const std::string & in_path, const std::string & out_path, int threads, int reps) {
    namespace sa = engine::models::stable_audio;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<sa::StableAudioAssets>();
    auto & c = assets->config;
    c.io_channels = i64_scalar(in, "io_channels");
    c.embed_dim = i64_scalar(in, "embed_dim");
    c.depth = i64_scalar(in, "depth");
    c.num_heads = i64_scalar(in, "num_heads");
    c.cond_dim = i64_scalar(in, "cond_dim");
    c.cond_token_dim = c.cond_dim;
    c.global_cond_dim = i64_scalar(in, "global_cond_dim");
    c.local_add_cond_dim = i64_scalar(in, "local_add_cond_dim");
    c.num_memory_tokens = i64_scalar(in, "num_memory_tokens");
    c.differential_attention = i64_scalar(in, "differential") != 0;
    c.prompt_max_length = i64_scalar(in, "prompt_max_length");
    c.stable_audio_open_v1 = false;
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(w));

    const int64_t batch = i64_scalar(in, "batch");
    const int64_t tokens = i64_scalar(in, "latent_tokens");
    const int64_t steps = i64_scalar(in, "steps");
    sa::StableAudioSamplingState sampling;
    sampling.batch = batch;
    sampling.latent_sample_size = tokens;
    sampling.channels = c.io_channels;
    sampling.schedule_points = steps + 1;
    sampling.schedule = f32s(in, "schedule");
    sampling.padding_mask = f32s(in, "padding_mask");
    sampling.noise = f32s(in, "noise");
    sampling.local_add_conditioning = f32s(in, "local_add");

    sa::StableAudioConditioningInputs cond;
    const int64_t cross_tokens = c.prompt_max_length + 1;
    cond.positive.batch = batch;
    cond.positive.cross_tokens = cross_tokens;
    cond.positive.cond_dim = c.cond_dim;
    cond.positive.cross_attention = f32s(in, "cross_positive");
    cond.positive.global = f32s(in, "global");
    cond.has_negative = i64_scalar(in, "has_negative") != 0;
    if (cond.has_negative) {
        cond.negative = cond.positive;
        cond.negative.cross_attention = f32s(in, "cross_negative");
        const auto m = f32s(in, "negative_mask");
        cond.negative.cross_attention_mask.assign(m.size(), 0);
        for (size_t i = 0; i < m.size(); ++i) cond.negative.cross_attention_mask[i] = m[i] != 0.0F ? 1 : 0;
    }
    const float cfg_scale = f32_scalar(in, "cfg_scale");
    const float apg_scale = f32_scalar(in, "apg_scale");
    // sampler: 0 "pingpong", 1 "euler"
    const char * sampler_name = i64_scalar(in, "sampler") == 1 ? "euler" : "pingpong";
    const uint64_t seed = static_cast<uint64_t>(i64_scalar(in, "seed"));

    engine::core::ExecutionContext exec({ref_backend(), 0, threads});
    sa::StableAudioRfDitRuntime dit(exec, assets, engine::assets::TensorStorageType::Native);
    engine::sampling::TorchCudaSamplingPolicy policy;
    policy.multiprocessor_count = i64_scalar(in, "rng_sms");
    policy.max_threads_per_multiprocessor = i64_scalar(in, "rng_max_threads");
    std::vector<float> times, result;
    uint64_t final_offset = 0;
    dit.prepare(sampling, cfg_scale);
    for (int r = 0; r < std::max(reps, 1); ++r) {
        uint64_t offset = static_cast<uint64_t>(i64_scalar(in, "rng_offset"));
        const double t0 = now_ms();
        result = dit.sample(sampling, cond, seed, offset, policy, sampler_name, cfg_scale, apg_scale);
        times.push_back(static_cast<float>(now_ms() - t0));
        final_offset = offset;
    }
    Bundle out;
    const int64_t fo = static_cast<int64_t>(final_offset);
    out["rng_offset_out"] = raw_entry(I64, &fo, 8, {1});
    out["latents"] = f32_entry(result, {batch, c.io_channels, tokens});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ------------------------------------------------------ Oobleck VAE decode
// OobleckAutoencoderRuntime::decode (src/models/stable_audio/foundation/oobleck_autoencoder.cpp:600-705):
// weight-normalised in-conv, decoder blocks (snake, transposed-conv upsampling, crop, three dilated
// residual units), final snake and out-conv; latents [B, latent_dim, T] -> audio [B, frames, channels].
int cmd_oobleck(const std::string & w, const std::string & in_path, const std::string & out_path, int threads,
                int reps) {
    namespace sf = engine::models::stable_audio::foundation;
    namespace sa = engine::models::stable_audio;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<sa::StableAudioAssets>();
    auto & c = assets->config;
    c.latent_dim = i64_scalar(in, "latent_dim");
    c.audio_channels = static_cast<int>(i64_scalar(in, "audio_channels"));
    c.sample_rate = 44100;
    c.same_channels = i64_scalar(in, "channels");
    c.same_c_mults = i64s(in, "c_mults");
    c.same_strides = i64s(in, "strides");
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(w));
    const int64_t batch = i64_scalar(in, "batch");
    const int64_t tokens = i64_scalar(in, "latent_tokens");
    const auto latents = f32s(in, "latents");
    engine::core::ExecutionContext exec({ref_backend(), 0, threads});
    sf::OobleckAutoencoderRuntime vae(exec, assets, engine::assets::TensorStorageType::Native);
    vae.prepare_decode(batch, tokens);
    std::vector<float> times, audio;
    int64_t frames = 0;
    for (int r = 0; r < std::max(reps, 1); ++r) {
        const double t0 = now_ms();
        const auto out = vae.decode(latents, batch, tokens);
        times.push_back(static_cast<float>(now_ms() - t0));
        audio.clear();
        for (const auto & a : out) audio.insert(audio.end(), a.samples.begin(), a.samples.end());
        frames = static_cast<int64_t>(out.front().samples.size()) / c.audio_channels;
    }
    Bundle out;
    out["audio"] = f32_entry(audio, {batch, frames, static_cast<int64_t>(c.audio_channels)});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ----------------------------------------------- VibeVoice acoustic decode
// VibeVoiceTokenizerWeightsRuntime::decode_acoustic (src/models/vibevoice/tokenizer_audio.cpp:1855-1878): the
// causal sigma-VAE decoder (stem conv, transposed-conv upsampling, ConvNeXt-style blocks with depthwise mixer and
// GELU FFN, head conv); latents [frames, vae_dim] -> mono samples.  The loader also reads the acoustic and
// semantic encoders, which the synthetic bundle carries.
std::string yaml_free_depths(const std::vector<int64_t> & d) {
    std::string out;
    for (size_t i = 0; i < d.size(); ++i) out += (i ? "-" : "") + std::to_string(d[i]);
    return out;
}

engine::models::vibevoice::VibeVoiceTokenizerConfig tok_config(const Bundle & in, const std::string & p) {
    engine::models::vibevoice::VibeVoiceTokenizerConfig c;
    c.channels = 1;
    c.causal = true;
    c.vae_dim = i64_scalar(in, p + "vae_dim");
    c.mixer_layer = "depthwise_conv";
    c.conv_norm = "none";
    c.pad_mode = "constant";
    c.disable_last_norm = i64_scalar(in, p + "disable_last_norm") != 0;
    c.layernorm = "RMSNorm";
    c.layernorm_eps = f32_scalar(in, p + "eps");
    c.layernorm_elementwise_affine = true;
    c.conv_bias = true;
    c.layer_scale_init_value = 1.0e-6F;
    c.encoder_n_filters = i64_scalar(in, p + "n_filters");
    c.encoder_ratios = i64s(in, p + "ratios");
    c.encoder_depths = yaml_free_depths(i64s(in, p + "depths"));
    c.decoder_n_filters = c.encoder_n_filters;
    c.decoder_ratios = c.encoder_ratios;
    return c;
}

int cmd_vvdec(const std::string & w, const std::string & in_path, const std::string & out_path, int threads, int reps) {
    namespace vv = engine::models::vibevoice;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<vv::VibeVoiceAssets>();
    assets->config.acoustic_tokenizer = tok_config(in, "acoustic_");
    assets->config.semantic_tokenizer = tok_config(in, "semantic_");
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(w));
    vv::VibeVoiceTokenizerWeightsRuntime rt(assets, ref_backend(), 0, threads);
    vv::VibeVoiceTokenizerLatents lat;
    lat.values = f32s(in, "latents");
    lat.dim = assets->config.acoustic_tokenizer.vae_dim;
    lat.frames = static_cast<int64_t>(lat.values.size()) / lat.dim;
    std::vector<float> times, samples;
    for (int r = 0; r < std::max(reps, 1); ++r) {
        const double t0 = now_ms();
        samples = rt.decode_acoustic(lat).samples;
        times.push_back(static_cast<float>(now_ms() - t0));
    }
    Bundle out;
    out["samples"] = f32_entry(samples, {static_cast<int64_t>(samples.size())});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ------------------------------------------------ SAO 1.0 conditioner (T5)
// FoundationConditionerRuntime::encode (src/models/stable_audio/foundation/conditioner.cpp:411-471): T5-base
// encoder over the prompt tokens (relative position buckets, additive padding mask, ReLU FFN), cross tokens =
// T5 states of the kept tokens + the seconds_start / seconds_total number embeddings, global = both embeddings.
// The T5 and the number-conditioner tensors come from one bundle.
int cmd_saocond(const std::string & w, const std::string & in_path, const std::string & out_path, int threads,
                int reps) {
    namespace sa = engine::models::stable_audio;
    namespace sf = engine::models::stable_audio::foundation;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<sa::StableAudioAssets>();
    auto & c = assets->config;
    c.t5_hidden_size = i64_scalar(in, "t5_hidden_size");
    c.t5_layers = i64_scalar(in, "t5_layers");
    c.t5_attention_heads = i64_scalar(in, "t5_heads");
    c.t5_head_dim = i64_scalar(in, "t5_head_dim");
    c.t5_intermediate_size = i64_scalar(in, "t5_intermediate");
    c.t5_vocab_size = i64_scalar(in, "t5_vocab");
    c.t5_rms_norm_eps = f32_scalar(in, "t5_eps");
    c.t5_pad_token_id = 0;
    c.prompt_max_length = i64_scalar(in, "prompt_max_length");
    c.cond_dim = c.t5_hidden_size;
    c.cond_token_dim = c.cond_dim;
    c.global_cond_dim = 2 * c.cond_dim;
    auto src = std::make_shared<BundleTensorSource>(read_bundle(w));
    assets->model_weights = src;
    assets->t5_weights = src;
    const int64_t batch = i64_scalar(in, "batch");
    auto tokens = [&](const std::string & ids, const std::string & mask) {
        sa::StableAudioTokenBatch t;
        t.batch = batch;
        t.tokens = c.prompt_max_length;
        for (const int64_t v : i64s(in, ids)) t.input_ids.push_back(static_cast<int32_t>(v));
        for (const int64_t v : i64s(in, mask)) t.attention_mask.push_back(static_cast<uint8_t>(v != 0));
        return t;
    };
    const bool neg = i64_scalar(in, "has_negative") != 0;
    const auto seconds = f32s(in, "normalized_seconds");
    // On the CPU backend a FoundationConditionerRuntime computes its T5 graph correctly only once: a second
    // encode on the same runtime trips ggml-cpu's get_rows bounds assert (the relative-bucket input is not
    // rewritten between runs).  So every encode here runs on its own runtime; for the negative prompt that is
    // exactly encode_one on the negative tokens (conditioner.cpp:414-418).
    auto encode_fresh = [&](const std::string & ids, const std::string & mask, double & ms) {
        sa::StableAudioConditioningBatch b;
        b.prompt_tokens = tokens(ids, mask);
        b.normalized_seconds = seconds;
        engine::core::ExecutionContext exec({ref_backend(), 0, threads});
        sf::FoundationConditionerRuntime rt(exec, assets, engine::assets::TensorStorageType::Native, batch);
        rt.prepare();
        const double t0 = now_ms();
        auto r = rt.encode(b);
        ms = now_ms() - t0;
        return r.positive;
    };
    std::vector<float> times;
    sa::StableAudioConditioningInputs res;
    for (int r = 0; r < std::max(reps, 1); ++r) {
        double ms = 0.0;
        res.positive = encode_fresh("input_ids", "attention_mask", ms);
        times.push_back(static_cast<float>(ms));
    }
    if (neg) {
        double ms = 0.0;
        res.negative = encode_fresh("negative_ids", "negative_mask", ms);
        res.has_negative = true;
    }
    Bundle out;
    const int64_t P2 = c.prompt_max_length + 2;
    out["cross_positive"] = f32_entry(res.positive.cross_attention, {batch, P2, c.cond_dim});
    out["global"] = f32_entry(res.positive.global, {batch, c.global_cond_dim});
    std::vector<float> mk(res.positive.cross_attention_mask.begin(), res.positive.cross_attention_mask.end());
    out["cross_mask"] = f32_entry(mk, {batch, P2});
    if (res.has_negative) out["cross_negative"] = f32_entry(res.negative.cross_attention, {batch, P2, c.cond_dim});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ------------------------------------------------- VibeVoice LM (Qwen2.5)
// VibeVoiceDecoderWeightsRuntime (src/models/vibevoice/decoder.cpp): prefill of `prefill` input embeddings, then
// `steps` cached single-token steps (each fed the embedding of a given token id); logits and last hidden of the
// prefill's final position and of every step.
int cmd_vvlm(const std::string & w, const std::string & in_path, const std::string & out_path, int threads, int reps) {
    namespace vv = engine::models::vibevoice;
    const Bundle in = read_bundle(in_path);
    auto assets = std::make_shared<vv::VibeVoiceAssets>();
    auto & c = assets->config.decoder;
    c.hidden_size = i64_scalar(in, "hidden_size");
    c.intermediate_size = i64_scalar(in, "intermediate_size");
    c.num_attention_heads = i64_scalar(in, "num_heads");
    c.num_key_value_heads = i64_scalar(in, "num_kv_heads");
    c.num_hidden_layers = i64_scalar(in, "num_layers");
    c.vocab_size = i64_scalar(in, "vocab_size");
    c.head_dim = i64_scalar(in, "head_dim");
    c.max_position_embeddings = i64_scalar(in, "max_positions");
    c.rms_norm_eps = f32_scalar(in, "rms_norm_eps");
    c.rope_theta = f32_scalar(in, "rope_theta");
    c.tie_word_embeddings = true;
    assets->model_weights = std::make_shared<BundleTensorSource>(read_bundle(w));
    vv::VibeVoiceDecoderWeightsRuntime lm(assets, ref_backend(), 0, threads);
    const int64_t prefill = i64_scalar(in, "prefill");
    std::vector<int32_t> ids;
    for (const int64_t v : i64s(in, "prefill_ids")) ids.push_back(static_cast<int32_t>(v));
    std::vector<int32_t> step_ids;
    for (const int64_t v : i64s(in, "step_ids")) step_ids.push_back(static_cast<int32_t>(v));
    std::vector<float> logits, hidden, times;
    const double t0 = now_ms();
    const auto emb = lm.embed_tokens(ids);
    auto pre = lm.prefill_embeddings(emb.values, prefill);
    times.push_back(static_cast<float>(now_ms() - t0));
    logits = pre.result.logits.values;
    hidden = pre.result.last_hidden.values;
    vv::VibeVoiceDecoderCachedState state;
    lm.reset_cached_state(state, std::move(pre.state));
    for (const int32_t id : step_ids) {
        const auto e = lm.embed_tokens({id});
        const double t1 = now_ms();
        const auto r = lm.cached_step(e.values, state, prefill + static_cast<int64_t>(step_ids.size()));
        times.push_back(static_cast<float>(now_ms() - t1));
        logits.insert(logits.end(), r.logits.values.begin(), r.logits.values.end());
        hidden.insert(hidden.end(), r.last_hidden.values.begin(), r.last_hidden.values.end());
    }
    (void)reps;
    const int64_t n = 1 + static_cast<int64_t>(step_ids.size());
    Bundle out;
    out["logits"] = f32_entry(logits, {n, c.vocab_size});
    out["last_hidden"] = f32_entry(hidden, {n, c.hidden_size});
    out["wall_ms"] = f32_entry(times, {static_cast<int64_t>(times.size())});
    write_bundle(out_path, out);
    return 0;
}

// ------------------------------------------------------------- Philox randn
// torch-CUDA compatible normals (src/framework/sampling/torch_random.cpp)
int cmd_randn(const std::string & in_path, const std::string & out_path) {
    const Bundle in = read_bundle(in_path);
    const int64_t count = i64_scalar(in, "count");
    const uint64_t seed = static_cast<uint64_t>(i64_scalar(in, "seed"));
    const uint64_t offset = static_cast<uint64_t>(i64_scalar(in, "offset"));
    engine::sampling::TorchCudaSamplingPolicy policy;
    policy.multiprocessor_count = i64_scalar(in, "sms");
    policy.max_threads_per_multiprocessor = i64_scalar(in, "max_threads");
    const auto a = engine::sampling::generate_torch_cuda_randn(size_t(count), seed,
                                                               engine::sampling::TorchRandnPrecision::Float32);
    const auto b = engine::sampling::generate_torch_cuda_randn(size_t(count), seed,
                                                               engine::sampling::TorchRandnPrecision::BFloat16);
    const auto c = engine::sampling::generate_torch_cuda_tensor_iterator_randn(
        size_t(count), seed, offset, policy, engine::sampling::TorchRandnPrecision::Float32);
    const int64_t next = static_cast<int64_t>(offset + engine::sampling::torch_cuda_tensor_iterator_offset_blocks(
                                                          uint64_t(count), policy));
    Bundle out;
    out["randn_f32"] = f32_entry(a, {count});
    out["randn_bf16"] = f32_entry(b, {count});
    out["iterator_f32"] = f32_entry(c, {count});
    out["next_offset"] = raw_entry(I64, &next, 8, {1});
    write_bundle(out_path, out);
    return 0;
}

// ---------------------------------------------------------------- Q8_0 KAT
int cmd_q8(const std::string & in_path, const std::string & out_path) {
    const Bundle in = read_bundle(in_path);
    const auto & e = need(in, "x");
    const auto x = f32s(in, "x");
    const int64_t cols = e.dims.back();
    const int64_t rows = static_cast<int64_t>(x.size()) / cols;
    std::vector<std::byte> q(static_cast<size_t>(rows) * ggml_row_size(GGML_TYPE_Q8_0, cols));
    ggml_quantize_chunk(GGML_TYPE_Q8_0, x.data(), q.data(), 0, rows, cols, nullptr);
    std::vector<float> deq(x.size());
    const auto * traits = ggml_get_type_traits(GGML_TYPE_Q8_0);
    for (int64_t r = 0; r < rows; ++r) {
        traits->to_float(q.data() + r * ggml_row_size(GGML_TYPE_Q8_0, cols), deq.data() + r * cols, cols);
    }
    Bundle out;
    out["q8"] = raw_entry(Q8_0, q.data(), q.size(), {rows, cols});
    out["dequant"] = f32_entry(deq, {rows, cols});
    write_bundle(out_path, out);
    return 0;
}

}  // namespace

// ResourceBundle (linked in through the asset structs) references the YAML
// parser; the harness never reads YAML, so libyaml is not linked and this
// definition stands in for it.
namespace engine::io::yaml {
FlattenedDocument parse_flattened_document(std::string_view) {
    throw std::runtime_error("YAML parsing is not available in the oracle harness");
}
}  // namespace engine::io::yaml

int main(int argc, char ** argv) {
    try {
        if (argc < 2) {
            std::fprintf(stderr, "usage: %s q8|vvsched|vvpredict|vv|dit ...\n", argv[0]);
            return 2;
        }
        const std::string cmd = argv[1];
        auto arg = [&](int i) -> std::string {
            if (i >= argc) throw std::runtime_error("missing argument " + std::to_string(i));
            return argv[i];
        };
        if (cmd == "q8") return cmd_q8(arg(2), arg(3));
        if (cmd == "randn") return cmd_randn(arg(2), arg(3));
        if (cmd == "vvsched") return cmd_vvsched(arg(2), arg(3));
        if (cmd == "vvpredict") return cmd_vvpredict(arg(2), arg(3), arg(4), std::stoi(arg(5)));
        if (cmd == "vv") return cmd_vv(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "dit") return cmd_dit(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "dit_fresh") return cmd_dit(arg(2), arg(3), arg(4), std::stoi(arg(5)), 1, true);
        if (cmd == "sa3") return cmd_sa3(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "vvlm") return cmd_vvlm(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "saocond") return cmd_saocond(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "vvdec") return cmd_vvdec(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        if (cmd == "oobleck") return cmd_oobleck(arg(2), arg(3), arg(4), std::stoi(arg(5)), std::stoi(arg(6)));
        std::fprintf(stderr, "unknown command %s\n", cmd.c_str());
        return 2;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "b2d_ref error: %s\n", e.what());
        return 1;
    }
}
