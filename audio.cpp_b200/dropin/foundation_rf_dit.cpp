// Drop-in replacement for the FoundationRfDitRuntime class of audio.cpp's
// src/models/stable_audio/foundation/rf_dit.cpp, compiled against audio.cpp's own unmodified header
// (include/engine/models/stable_audio/foundation/rf_dit.h:73-106) and linked in place of that translation unit.
// FoundationSession's calls (prepare, sample) do not change; the sampler runs on a B200 through libb200diff
// (include/b200diff.h) as one captured CUDA graph instead of a ggml graph per step.
//
// The ExecutionContext's device ordinal selects the B200 whatever its backend type says.  Weights load on the
// first prepare(), as the reference's require_rf_weights does, with the storage type given at construction.
#include "engine/models/stable_audio/foundation/rf_dit.h"

#include <stdexcept>
#include <string>
#include <vector>

#include "b200diff.h"

namespace engine::models::stable_audio::foundation {

// The device context of one runtime (the reference keeps its ggml graph here).
class FoundationRfDitRuntime::Graph {
public:
    explicit Graph(int device) {
        if (b2d_create(device, &ctx) != B2D_OK)
            throw std::runtime_error("Stable Audio Foundation RF DiT: no usable B200 device " + std::to_string(device));
    }
    ~Graph() { b2d_destroy(ctx); }
    void check(b2d_status s) const {
        if (s != B2D_OK) throw std::runtime_error(b2d_last_error(ctx));
    }
    b2d_ctx* ctx = nullptr;
};

FoundationRfDitRuntime::FoundationRfDitRuntime(core::ExecutionContext& execution,
                                               std::shared_ptr<const StableAudioAssets> assets,
                                               assets::TensorStorageType weight_storage_type)
    : execution_(&execution), assets_(std::move(assets)), weight_storage_type_(weight_storage_type) {
    if (execution_ == nullptr)
        throw std::runtime_error("Stable Audio Foundation RF DiT runtime requires execution context");
    if (assets_ == nullptr) throw std::runtime_error("Stable Audio Foundation RF DiT runtime requires assets");
}

FoundationRfDitRuntime::~FoundationRfDitRuntime() = default;

namespace {

struct LoadedTensor {
    std::string name;
    b2d_tensor_view view{};
    std::vector<std::byte> raw;
    std::vector<unsigned char> converted;
};

// The reference's weight store converts the linear matrices to the requested storage type and keeps 1-D
// tensors (norm gamma / beta, biases) and the timestep feature table as f32-readable values.
void load_tensor(const assets::TensorSource& src, const std::string& name, assets::TensorStorageType storage,
                 LoadedTensor& t) {
    auto data = src.require_tensor_data(name);
    t.name = name;
    t.raw = std::move(data.bytes);
    const auto& shape = data.metadata.shape;
    if (shape.empty() || shape.size() > 4) throw std::runtime_error("tensor rank is unsupported: " + name);
    t.view.ggml_type = static_cast<int32_t>(assets::ggml_type_for_tensor_dtype(data.metadata.dtype));
    t.view.ndim = static_cast<int32_t>(shape.size());
    for (size_t i = 0; i < shape.size(); ++i) t.view.dims[i] = shape[i];
    t.view.data = t.raw.data();
    t.view.nbytes = t.raw.size();
    if (shape.size() < 2 || name.find("timestep_features") != std::string::npos) return;
    const int32_t target = b2d_storage_resolve(static_cast<int32_t>(storage), &t.view);
    if (target < 0) throw std::runtime_error("unsupported weight storage type for " + name);
    if (target == t.view.ggml_type) return;
    t.converted.resize(b2d_tensor_bytes(target, t.view.dims, t.view.ndim));
    if (t.converted.empty() ||
        b2d_tensor_convert(&t.view, target, t.converted.data(), t.converted.size()) != B2D_OK)
        throw std::runtime_error("weight conversion failed for " + name);
    t.view.ggml_type = target;
    t.view.data = t.converted.data();
    t.view.nbytes = t.converted.size();
}

}  // namespace

void FoundationRfDitRuntime::prepare(const StableAudioSamplingState& sampling, float /*cfg_scale*/) const {
    if (sampling.batch <= 0 || sampling.latent_sample_size <= 0)
        throw std::runtime_error("Stable Audio Foundation RF DiT graph requires positive batch and latent length");
    if (graph_) return;
    const auto& c = assets_->config;
    if (assets_->model_weights == nullptr) throw std::runtime_error("Stable Audio Foundation RF DiT requires weights");
    auto g = std::make_unique<Graph>(execution_->config().device);
    std::vector<LoadedTensor> tensors;
    for (const auto& meta : assets_->model_weights->tensors()) {
        if (meta.name.rfind("model.model.", 0) != 0) continue;
        tensors.emplace_back();
        load_tensor(*assets_->model_weights, meta.name, weight_storage_type_, tensors.back());
    }
    std::vector<b2d_tensor_view> views;
    for (auto& t : tensors) {
        t.view.name = t.name.c_str();
        views.push_back(t.view);
    }
    const b2d_dit_config dc{c.embed_dim, c.depth, c.num_heads, c.cond_token_dim, c.global_cond_dim, c.io_channels,
                            c.prompt_max_length};
    g->check(b2d_dit_load(g->ctx, &dc, views.data(), static_cast<int32_t>(views.size())));
    graph_ = std::move(g);
}

std::vector<float> FoundationRfDitRuntime::sample(const StableAudioSamplingState& sampling,
                                                  const StableAudioConditioningInputs& conditioning, uint64_t seed,
                                                  uint64_t& rng_offset_blocks,
                                                  const engine::sampling::TorchCudaSamplingPolicy& rng_policy,
                                                  std::string_view sampler_type, float sigma_min, float sigma_max,
                                                  float rho, float cfg_scale, float apg_scale) const {
    prepare(sampling, cfg_scale);
    const auto& c = assets_->config;
    if (!sampler_type.empty() && sampler_type != "euler" && sampler_type != "pingpong" && sampler_type != "dpmpp-2m" &&
        sampler_type != "dpmpp-3m-sde")
        throw std::runtime_error("Stable Audio Foundation sampler_type is not supported for the v sampler");
    // "dpmpp-2m" and "dpmpp-3m-sde" by name; every other accepted name runs the v-DDIM sampler (rf_dit.cpp:461-511)
    const int32_t sampler = sampler_type == "dpmpp-2m"       ? B2D_SAMPLER_DPMPP_2M
                            : sampler_type == "dpmpp-3m-sde" ? B2D_SAMPLER_DPMPP_3M_SDE
                                                             : B2D_SAMPLER_V_DDIM;
    const int64_t B = sampling.batch, T = sampling.latent_sample_size, P2 = c.prompt_max_length + 2;
    if (sampling.channels != c.io_channels) throw std::runtime_error("Stable Audio Foundation RF DiT channel mismatch");
    if (conditioning.positive.batch != B || conditioning.positive.cross_tokens != P2 ||
        conditioning.positive.cond_dim != c.cond_token_dim ||
        static_cast<int64_t>(conditioning.positive.cross_attention.size()) != B * P2 * c.cond_token_dim ||
        static_cast<int64_t>(conditioning.positive.global.size()) != B * c.global_cond_dim)
        throw std::runtime_error("Stable Audio Foundation RF DiT positive conditioning shape mismatch");
    if (conditioning.has_negative &&
        (conditioning.negative.batch != B || conditioning.negative.cross_tokens != P2 ||
         conditioning.negative.cond_dim != c.cond_token_dim ||
         static_cast<int64_t>(conditioning.negative.cross_attention.size()) != B * P2 * c.cond_token_dim))
        throw std::runtime_error("Stable Audio Foundation RF DiT negative conditioning shape mismatch");
    if (static_cast<int64_t>(sampling.noise.size()) != B * c.io_channels * T ||
        static_cast<int64_t>(sampling.padding_mask.size()) != B * T)
        throw std::runtime_error("Stable Audio Foundation RF DiT graph shape mismatch");
    if (sampling.schedule_points <= 1 ||
        (sampler == B2D_SAMPLER_V_DDIM && static_cast<int64_t>(sampling.schedule.size()) != B * sampling.schedule_points))
        throw std::runtime_error("Stable Audio Foundation RF DiT schedule shape mismatch");
    b2d_dit_request rq{};
    rq.batch = B;
    rq.latent_tokens = T;
    rq.steps = sampling.schedule_points - 1;
    rq.noise = sampling.noise.data();
    rq.padding_mask = sampling.padding_mask.data();
    rq.cross_positive = conditioning.positive.cross_attention.data();
    rq.cross_negative = conditioning.has_negative ? conditioning.negative.cross_attention.data() : nullptr;
    rq.global_cond = conditioning.positive.global.data();
    rq.sigma_min = sigma_min;
    rq.sigma_max = sigma_max;
    rq.rho = rho;
    rq.cfg_scale = cfg_scale;
    rq.apg_scale = apg_scale;
    rq.sampler = sampler;
    rq.schedule = sampling.schedule.empty() ? nullptr : sampling.schedule.data();
    rq.seed = seed;
    rq.rng_offset_blocks = &rng_offset_blocks;
    rq.rng_multiprocessor_count = rng_policy.multiprocessor_count;
    rq.rng_max_threads_per_multiprocessor = rng_policy.max_threads_per_multiprocessor;
    std::vector<float> out(sampling.noise.size());
    graph_->check(b2d_dit_sample(graph_->ctx, &rq, out.data(), nullptr));
    return out;
}

}  // namespace engine::models::stable_audio::foundation
