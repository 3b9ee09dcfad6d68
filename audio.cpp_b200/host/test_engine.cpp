// C++ tests of the audio.cpp-facing classes (engine_b200.h), written like audio.cpp's own
// unit tests (a main() per check group, require_close helpers, non-zero exit on failure).
//
//   test_engine sched <golden dir>                          scheduler vs reference vectors (no GPU)
//   test_engine head  <weights> <inputs> <golden>           sample_vibevoice_speech_latents on the GPU
//   test_engine dit   <weights> <inputs> <golden>           FoundationRfDitRuntime::sample on the GPU
//   test_engine sa3   <weights> <inputs> <golden>           StableAudioRfDitRuntime::sample on the GPU
// Bundles are B2DB files (see oracle/bundle.py): weights by tensor name, inputs and goldens by key.
#include "engine_b200.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct Entry {
    uint8_t dtype = 0;
    std::vector<int64_t> dims;
    std::vector<uint8_t> bytes;
};
using Bundle = std::map<std::string, Entry>;

template <typename T>
void rd(std::ifstream & in, T & v) {
    in.read(reinterpret_cast<char *>(&v), sizeof(T));
    if (!in) throw std::runtime_error("bundle truncated");
}

Bundle read_bundle(const std::string & path) {
    std::ifstream in(path, std::ios::binary);
    char magic[4];
    in.read(magic, 4);
    if (!in || std::memcmp(magic, "B2DB", 4) != 0) throw std::runtime_error("bad bundle " + path);
    uint32_t version = 0, count = 0;
    rd(in, version);
    rd(in, count);
    Bundle b;
    for (uint32_t i = 0; i < count; ++i) {
        uint16_t n = 0;
        rd(in, n);
        std::string name(n, '\0');
        in.read(name.data(), n);
        Entry e;
        uint8_t nd = 0;
        rd(in, e.dtype);
        rd(in, nd);
        e.dims.resize(nd);
        for (auto & d : e.dims) rd(in, d);
        uint64_t nb = 0;
        rd(in, nb);
        e.bytes.resize(nb);
        in.read(reinterpret_cast<char *>(e.bytes.data()), static_cast<std::streamsize>(nb));
        b.emplace(name, std::move(e));
    }
    return b;
}

std::vector<float> f32(const Bundle & b, const std::string & k) {
    const auto & e = b.at(k);
    std::vector<float> v(e.bytes.size() / 4);
    std::memcpy(v.data(), e.bytes.data(), e.bytes.size());
    return v;
}

int64_t i64(const Bundle & b, const std::string & k) {
    int64_t v = 0;
    std::memcpy(&v, b.at(k).bytes.data(), 8);
    return v;
}

float f1(const Bundle & b, const std::string & k) { return f32(b, k).at(0); }

// B2DB dtype codes -> ggml type ids
int ggml_type(uint8_t code) {
    switch (code) {
        case 0: return B2D_TYPE_F32;
        case 1: return B2D_TYPE_F16;
        case 2: return B2D_TYPE_BF16;
        default: return B2D_TYPE_Q8_0;
    }
}

std::vector<engine::b200::RawTensor> tensors_of(const Bundle & b) {
    std::vector<engine::b200::RawTensor> out;
    for (const auto & [name, e] : b) out.push_back({name, ggml_type(e.dtype), e.dims, e.bytes});
    return out;
}

int failures = 0;

void require(bool ok, const std::string & what) {
    if (!ok) {
        std::fprintf(stderr, "FAILED: %s\n", what.c_str());
        ++failures;
    }
}

void require_close(const std::vector<float> & a, const std::vector<float> & b, double rtol, double atol,
                   const std::string & what) {
    if (a.size() != b.size()) return require(false, what + " (size)");
    for (size_t i = 0; i < a.size(); ++i)
        if (std::fabs(double(a[i]) - b[i]) > atol + rtol * std::fabs(double(b[i])))
            return require(false, what + " at " + std::to_string(i));
}

double rel_l2(const std::vector<float> & a, const std::vector<float> & b) {
    double n = 0, d = 0;
    for (size_t i = 0; i < a.size(); ++i) {
        n += (double(a[i]) - b[i]) * (double(a[i]) - b[i]);
        d += double(b[i]) * b[i];
    }
    return std::sqrt(n / (d > 0 ? d : 1e-30));
}

template <typename F>
void require_throws(F && f, const std::string & message) {
    try {
        f();
    } catch (const std::runtime_error & e) {
        require(std::string(e.what()).find(message) != std::string::npos,
                "message '" + std::string(e.what()) + "' lacks '" + message + "'");
        return;
    }
    require(false, "expected exception: " + message);
}

int test_sched(const std::string & dir) {
    using namespace engine::models::vibevoice;
    for (int steps : {1, 2, 10, 20}) {
        const Bundle g = read_bundle(dir + "/sched_" + std::to_string(steps) + ".b2db");
        VibeVoiceDiffusionHeadConfig cfg;
        VibeVoiceDPMSolverScheduler s(cfg);
        s.set_timesteps(steps);
        const auto ts = f32(g, "timesteps");
        for (int i = 0; i < steps; ++i) require(float(s.timesteps()[size_t(i)]) == ts[size_t(i)], "timestep");
        auto sample = f32(g, "sample");
        const auto outs = f32(g, "model_outputs");
        const auto trace = f32(g, "trace");
        const size_t n = sample.size();
        for (int i = 0; i < steps; ++i) {
            std::vector<float> mo(outs.begin() + i * n, outs.begin() + (i + 1) * n);
            sample = s.step(mo, s.timesteps()[size_t(i)], sample).prev_sample;
            require_close(sample, std::vector<float>(trace.begin() + i * n, trace.begin() + (i + 1) * n), 1e-6, 1e-6,
                          "scheduler step " + std::to_string(i) + " of " + std::to_string(steps));
        }
    }
    VibeVoiceDiffusionHeadConfig bad;
    bad.ddpm_beta_schedule = "linear";
    require_throws([&] { VibeVoiceDPMSolverScheduler s(bad); }, "only supports cosine beta schedule");
    VibeVoiceDiffusionHeadConfig cfg;
    VibeVoiceDPMSolverScheduler s(cfg);
    require_throws([&] { s.set_timesteps(0); }, "inference steps must be positive");
    require_throws([&] { s.step({1.f}, 0, {1.f}); }, "set_timesteps must be called before step");
    return failures;
}

int test_head(const std::string & wpath, const std::string & ipath, const std::string & gpath) {
    using namespace engine::models::vibevoice;
    const Bundle in = read_bundle(ipath), g = read_bundle(gpath);
    VibeVoiceDiffusionHeadConfig cfg;
    cfg.hidden_size = i64(in, "hidden_size");
    cfg.latent_size = i64(in, "latent_size");
    cfg.head_layers = i64(in, "head_layers");
    cfg.head_ffn_ratio = f1(in, "head_ffn_ratio");
    cfg.rms_norm_eps = f1(in, "rms_norm_eps");
    VibeVoiceDiffusionHeadWeightsRuntime head(cfg, tensors_of(read_bundle(wpath)), 0);
    VibeVoiceDPMSolverScheduler sched(cfg);
    VibeVoiceSpeechDiffusionInput input;
    input.positive_condition = f32(in, "positive_condition");
    input.negative_condition = f32(in, "negative_condition");
    input.initial_speech = f32(in, "initial_speech");
    input.hidden_size = cfg.hidden_size;
    input.latent_size = cfg.latent_size;
    input.batch_size = int64_t(input.positive_condition.size()) / cfg.hidden_size;
    input.inference_steps = i64(in, "inference_steps");
    input.guidance_scale = f1(in, "guidance_scale");
    require_throws([&] { sample_vibevoice_speech_latents(head, sched, input); },
                   "timesteps do not match request inference steps");
    sched.set_timesteps(input.inference_steps);
    const auto result = sample_vibevoice_speech_latents(head, sched, input);
    std::vector<float> got;
    for (const auto & l : result) got.insert(got.end(), l.values.begin(), l.values.end());
    const double err = rel_l2(got, f32(g, "exact_latents"));
    std::printf("head rel-L2 vs fp32-activation oracle %.3g\n", err);
    require(err < 3e-3, "head latents vs oracle");
    auto bad = input;
    bad.initial_speech.pop_back();
    require_throws([&] { sample_vibevoice_speech_latents(head, sched, bad); },
                   "payload size mismatch for initial_speech");
    require_throws([&] { head.predict({0.f}, 1, 3, 1.0f, {0.f}, cfg.hidden_size); }, "received invalid input shape");
    return failures;
}

int test_dit(const std::string & wpath, const std::string & ipath, const std::string & gpath) {
    namespace sa = engine::models::stable_audio;
    const Bundle in = read_bundle(ipath), g = read_bundle(gpath);
    sa::StableAudioConfig cfg;
    cfg.embed_dim = i64(in, "embed_dim");
    cfg.depth = i64(in, "depth");
    cfg.num_heads = i64(in, "num_heads");
    cfg.cond_token_dim = i64(in, "cond_token_dim");
    cfg.global_cond_dim = i64(in, "global_cond_dim");
    cfg.prompt_max_length = i64(in, "prompt_max_length");
    sa::foundation::FoundationRfDitRuntime dit(cfg, tensors_of(read_bundle(wpath)), 0);
    sa::StableAudioSamplingState st;
    st.batch = i64(in, "batch");
    st.latent_sample_size = i64(in, "latent_tokens");
    st.channels = 64;
    st.schedule_points = i64(in, "steps") + 1;
    st.noise = f32(in, "noise");
    st.padding_mask = f32(in, "padding_mask");
    sa::StableAudioConditioningInputs c;
    c.positive = {st.batch, cfg.prompt_max_length + 2, cfg.cond_token_dim, f32(in, "cross_positive"), {}, f32(in, "global")};
    c.negative = c.positive;
    c.negative.cross_attention = f32(in, "cross_negative");
    c.has_negative = true;
    uint64_t off = 0;
    engine::sampling::TorchCudaSamplingPolicy pol;
    const auto out = dit.sample(st, c, 0, off, pol, "dpmpp-2m", f1(in, "sigma_min"), f1(in, "sigma_max"), f1(in, "rho"),
                                f1(in, "cfg_scale"), f1(in, "apg_scale"));
    const double err = rel_l2(out, f32(g, "exact_latents"));
    std::printf("dit rel-L2 vs fp32-activation oracle %.3g\n", err);
    require(err < 2e-2, "DiT latents vs oracle");
    require_throws([&] { dit.sample(st, c, 0, off, pol, "bogus", 0.01f, 100.f, 1.f, 7.f, 1.f); },
                   "sampler_type is not supported");
    auto bad = c;
    bad.positive.cond_dim = 7;
    require_throws([&] { dit.sample(st, bad, 0, off, pol, "dpmpp-2m", 0.01f, 100.f, 1.f, 7.f, 1.f); },
                   "positive conditioning shape mismatch");
    return failures;
}

int test_sa3(const std::string & wpath, const std::string & ipath, const std::string & gpath) {
    namespace sa = engine::models::stable_audio;
    const Bundle in = read_bundle(ipath), g = read_bundle(gpath);
    sa::StableAudioConfig cfg;
    cfg.embed_dim = i64(in, "embed_dim");
    cfg.depth = i64(in, "depth");
    cfg.num_heads = i64(in, "num_heads");
    cfg.cond_dim = i64(in, "cond_dim");
    cfg.global_cond_dim = i64(in, "global_cond_dim");
    cfg.local_add_cond_dim = i64(in, "local_add_cond_dim");
    cfg.num_memory_tokens = i64(in, "num_memory_tokens");
    cfg.prompt_max_length = i64(in, "prompt_max_length");
    cfg.differential_attention = i64(in, "differential") != 0;
    sa::StableAudioRfDitRuntime dit(cfg, tensors_of(read_bundle(wpath)), 0);
    sa::StableAudioSamplingState st;
    st.batch = i64(in, "batch");
    st.latent_sample_size = i64(in, "latent_tokens");
    st.channels = 64;
    st.schedule_points = i64(in, "steps") + 1;
    st.schedule = f32(in, "schedule");
    st.noise = f32(in, "noise");
    st.padding_mask = f32(in, "padding_mask");
    st.local_add_conditioning = f32(in, "local_add");
    const int64_t P1 = cfg.prompt_max_length + 1;
    sa::StableAudioConditioningInputs c;
    c.positive = {st.batch, P1, cfg.cond_dim, f32(in, "cross_positive"), {}, f32(in, "global")};
    c.negative = c.positive;
    c.negative.cross_attention = f32(in, "cross_negative");
    for (const float m : f32(in, "negative_mask")) c.negative.cross_attention_mask.push_back(m != 0.0F ? 1 : 0);
    c.has_negative = true;
    uint64_t off = 0;
    engine::sampling::TorchCudaSamplingPolicy pol;
    pol.multiprocessor_count = i64(in, "rng_sms");
    pol.max_threads_per_multiprocessor = i64(in, "rng_max_threads");
    const auto out = dit.sample(st, c, uint64_t(i64(in, "seed")), off, pol, i64(in, "sampler") == 0 ? "pingpong" : "euler",
                                f1(in, "cfg_scale"), f1(in, "apg_scale"));
    const double err = rel_l2(out, f32(g, "latents"));
    std::printf("sa3 rel-L2 vs the reference %.3g\n", err);
    require(err < 2e-2, "SA3 latents vs reference");
    require(int64_t(off) == i64(g, "rng_offset_out"), "rng_offset_blocks out-parameter");
    require_throws([&] { dit.sample(st, c, 0, off, pol, "dpmpp-2m", 7.f, 1.f); },
                   "sampler_type must be pingpong or euler");
    auto bad = st;
    bad.local_add_conditioning.pop_back();
    require_throws([&] { dit.sample(bad, c, 0, off, pol, "pingpong", 7.f, 1.f); }, "local conditioning shape mismatch");
    auto badc = c;
    badc.positive.cond_dim = 7;
    require_throws([&] { dit.sample(st, badc, 0, off, pol, "pingpong", 7.f, 1.f); },
                   "positive conditioning shape mismatch");
    return failures;
}

}  // namespace

int main(int argc, char ** argv) {
    try {
        if (argc >= 3 && std::string(argv[1]) == "sched") return test_sched(argv[2]) ? 1 : 0;
        if (argc >= 5 && std::string(argv[1]) == "head") return test_head(argv[2], argv[3], argv[4]) ? 1 : 0;
        if (argc >= 5 && std::string(argv[1]) == "dit") return test_dit(argv[2], argv[3], argv[4]) ? 1 : 0;
        if (argc >= 5 && std::string(argv[1]) == "sa3") return test_sa3(argv[2], argv[3], argv[4]) ? 1 : 0;
        std::fprintf(stderr, "usage: %s sched <dir> | head|dit|sa3 <weights> <inputs> <golden>\n", argv[0]);
        return 2;
    } catch (const std::exception & e) {
        std::fprintf(stderr, "FAILED with exception: %s\n", e.what());
        return 1;
    }
}
