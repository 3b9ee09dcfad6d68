// Drop-in replacement for audio.cpp's src/models/vibevoice/diffusion_head.cpp (the runtime class) and
// src/models/vibevoice/diffusion_sampler.cpp, compiled against audio.cpp's own unmodified headers
// (include/engine/models/vibevoice/diffusion_head.h:58-97, diffusion_sampler.h:12-26) and linked in place of
// those two translation units.  Callers (VibeVoiceSession, generate_vibevoice) do not change: the same
// constructor, predict() and sample_vibevoice_speech_latents(), the same exceptions; the work runs on a B200
// through libb200diff (include/b200diff.h) instead of a ggml graph.
//
// Differences a caller can observe: `device` is the CUDA ordinal of the B200 that runs the head whatever
// `backend_type` says (there is no ggml backend: backend() is null, weights() holds no ggml tensors and
// constants() must not be called); weight_context_bytes / constant_context_bytes are not needed.
#include "engine/models/vibevoice/diffusion_head.h"
#include "engine/models/vibevoice/diffusion_sampler.h"
#include "engine/framework/core/constant_tensor_cache.h"

#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "b200diff.h"

namespace engine::models::vibevoice {

// Holds the device context of one runtime (the reference keeps its ggml graph cache here).
class VibeVoiceDiffusionHeadGraph {
public:
    explicit VibeVoiceDiffusionHeadGraph(int device) {
        if (b2d_create(device, &ctx) != B2D_OK)
            throw std::runtime_error("VibeVoice diffusion head: no usable B200 device " + std::to_string(device));
    }
    ~VibeVoiceDiffusionHeadGraph() { b2d_destroy(ctx); }
    void check(b2d_status s) const {
        if (s != B2D_OK) throw std::runtime_error(b2d_last_error(ctx));
    }
    b2d_ctx* ctx = nullptr;
};

namespace {

// sample_vibevoice_speech_latents is a free function: it finds the runtime's device context here.
std::mutex g_registry_mutex;
std::unordered_map<const VibeVoiceDiffusionHeadWeightsRuntime*, const VibeVoiceDiffusionHeadGraph*> g_registry;

const VibeVoiceDiffusionHeadGraph& device_of(const VibeVoiceDiffusionHeadWeightsRuntime& rt) {
    std::lock_guard<std::mutex> lock(g_registry_mutex);
    auto it = g_registry.find(&rt);
    if (it == g_registry.end()) throw std::runtime_error("VibeVoice diffusion head runtime is not initialized");
    return *it->second;
}

// A checkpoint tensor as the C ABI takes it, converted to the requested storage type the way the reference's
// weight store does (matrices only: the reference reads 1-D tensors such as the RMSNorm weights as f32
// whatever the storage type).
struct LoadedTensor {
    std::string name;
    b2d_tensor_view view{};
    std::vector<std::byte> raw;
    std::vector<unsigned char> converted;
};

void load_tensor(const assets::TensorSource& src, const std::string& name, assets::TensorStorageType storage,
                 LoadedTensor& t) {
    auto data = src.require_tensor_data(name);
    t.name = name;
    t.raw = std::move(data.bytes);
    const auto& shape = data.metadata.shape;
    if (shape.empty() || shape.size() > 4) throw std::runtime_error("tensor rank is unsupported: " + name);
    t.view.name = t.name.c_str();
    t.view.ggml_type = static_cast<int32_t>(assets::ggml_type_for_tensor_dtype(data.metadata.dtype));
    t.view.ndim = static_cast<int32_t>(shape.size());
    for (size_t i = 0; i < shape.size(); ++i) t.view.dims[i] = shape[i];
    t.view.data = t.raw.data();
    t.view.nbytes = t.raw.size();
    if (shape.size() < 2) return;
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

VibeVoiceDiffusionHeadWeightsRuntime::VibeVoiceDiffusionHeadWeightsRuntime(
    std::shared_ptr<const VibeVoiceAssets> assets, core::BackendType backend_type, int device, int threads,
    size_t /*weight_context_bytes*/, size_t /*constant_context_bytes*/, assets::TensorStorageType weight_storage_type)
    : assets_(std::move(assets)), backend_type_(backend_type), threads_(threads) {
    if (assets_ == nullptr) throw std::runtime_error("VibeVoice diffusion head weights runtime requires assets");
    if (threads_ <= 0)
        throw std::runtime_error("VibeVoice diffusion head weights runtime requires positive thread count");
    if (assets_->model_weights == nullptr) throw std::runtime_error("VibeVoice diffusion head requires model weights");
    const auto& cfg = assets_->config.diffusion_head;
    graph_ = std::make_unique<VibeVoiceDiffusionHeadGraph>(device);
    // every prediction_head tensor the reference's loader reads (diffusion_head.cpp:335-399)
    std::vector<LoadedTensor> tensors;
    for (const auto& meta : assets_->model_weights->tensors()) {
        if (meta.name.rfind("model.prediction_head.", 0) != 0) continue;
        tensors.emplace_back();
        load_tensor(*assets_->model_weights, meta.name, weight_storage_type, tensors.back());
    }
    std::vector<b2d_tensor_view> views;
    for (auto& t : tensors) {
        t.view.name = t.name.c_str();
        views.push_back(t.view);
    }
    const b2d_vv_head_config c{cfg.hidden_size, cfg.latent_size, cfg.head_layers, cfg.head_ffn_ratio,
                               cfg.rms_norm_eps, cfg.ddpm_num_steps};
    graph_->check(b2d_vv_head_load(graph_->ctx, &c, views.data(), static_cast<int32_t>(views.size())));
    weights_ = std::make_shared<VibeVoiceDiffusionHeadWeights>();
    std::lock_guard<std::mutex> lock(g_registry_mutex);
    g_registry[this] = graph_.get();
}

VibeVoiceDiffusionHeadWeightsRuntime::~VibeVoiceDiffusionHeadWeightsRuntime() {
    {
        std::lock_guard<std::mutex> lock(g_registry_mutex);
        g_registry.erase(this);
    }
    graph_.reset();
}

const VibeVoiceAssets& VibeVoiceDiffusionHeadWeightsRuntime::assets() const noexcept { return *assets_; }

const VibeVoiceDiffusionHeadWeights& VibeVoiceDiffusionHeadWeightsRuntime::weights() const noexcept {
    return *weights_;
}

ggml_backend_t VibeVoiceDiffusionHeadWeightsRuntime::backend() const noexcept { return backend_; }

core::BackendType VibeVoiceDiffusionHeadWeightsRuntime::backend_type() const noexcept { return backend_type_; }

core::ConstantTensorCache& VibeVoiceDiffusionHeadWeightsRuntime::constants() const noexcept { return *constants_; }

int VibeVoiceDiffusionHeadWeightsRuntime::threads() const noexcept { return threads_; }

VibeVoiceDiffusionPrediction VibeVoiceDiffusionHeadWeightsRuntime::predict(
    const std::vector<float>& noisy_images, int64_t frames, int64_t latent_size, float timestep,
    const std::vector<float>& condition, int64_t condition_hidden_size) const {
    const auto& config = assets_->config.diffusion_head;
    if (frames <= 0 || latent_size != config.latent_size || condition_hidden_size != config.hidden_size)
        throw std::runtime_error("VibeVoice diffusion head received invalid input shape");
    if (static_cast<int64_t>(noisy_images.size()) != frames * latent_size ||
        static_cast<int64_t>(condition.size()) != frames * condition_hidden_size)
        throw std::runtime_error("VibeVoice diffusion head received invalid input shape");
    VibeVoiceDiffusionPrediction out;
    out.frames = frames;
    out.latent_size = latent_size;
    out.values.resize(static_cast<size_t>(frames * latent_size));
    graph_->check(b2d_vv_predict(graph_->ctx, noisy_images.data(), frames, latent_size, timestep, condition.data(),
                                 condition_hidden_size, out.values.data(), nullptr));
    return out;
}

namespace {

void require_payload_size(const std::vector<float>& values, int64_t expected, const char* label) {
    if (static_cast<int64_t>(values.size()) != expected)
        throw std::runtime_error(std::string("VibeVoice diffusion sampler payload size mismatch for ") + label);
}

}  // namespace

// The whole DPM-Solver++ loop with CFG runs on the device as one captured graph (b2d_vv_sample); the scheduler
// object's timesteps are checked against the request as the reference does, and its step state is reset.
std::vector<VibeVoiceTokenizerLatents> sample_vibevoice_speech_latents(
    const VibeVoiceDiffusionHeadWeightsRuntime& prediction_head, VibeVoiceDPMSolverScheduler& scheduler,
    const VibeVoiceSpeechDiffusionInput& input) {
    if (input.batch_size <= 0 || input.hidden_size <= 0 || input.latent_size <= 0)
        throw std::runtime_error("VibeVoice diffusion sampler requires positive dimensions");
    if (input.inference_steps <= 0)
        throw std::runtime_error("VibeVoice diffusion sampler requires positive inference steps");
    require_payload_size(input.positive_condition, input.batch_size * input.hidden_size, "positive_condition");
    require_payload_size(input.negative_condition, input.batch_size * input.hidden_size, "negative_condition");
    require_payload_size(input.initial_speech, 2 * input.batch_size * input.latent_size, "initial_speech");
    if (static_cast<int64_t>(scheduler.timesteps().size()) != input.inference_steps)
        throw std::runtime_error("VibeVoice diffusion scheduler timesteps do not match request inference steps");
    const auto& config = prediction_head.assets().config.diffusion_head;
    if (input.hidden_size != config.hidden_size || input.latent_size != config.latent_size)
        throw std::runtime_error("VibeVoice diffusion head received invalid input shape");
    // the device computes the schedule of VibeVoiceDPMSolverScheduler(ddpm_num_steps).set_timesteps(steps)
    std::vector<b2d_vv_step> table(static_cast<size_t>(input.inference_steps));
    if (b2d_vv_schedule(config.ddpm_num_steps, input.inference_steps, table.data()) != B2D_OK)
        throw std::runtime_error("VibeVoice scheduler requires positive timestep counts");
    for (size_t i = 0; i < table.size(); ++i)
        if (table[i].timestep != scheduler.timesteps()[i])
            throw std::runtime_error("VibeVoice diffusion scheduler timesteps do not match the device schedule");
    scheduler.reset_step_state();
    const auto& dev = device_of(prediction_head);
    std::vector<float> latents(static_cast<size_t>(input.batch_size * input.latent_size));
    dev.check(b2d_vv_sample(dev.ctx, input.positive_condition.data(), input.negative_condition.data(),
                            input.initial_speech.data(), input.batch_size, input.inference_steps,
                            input.guidance_scale, latents.data(), nullptr));
    std::vector<VibeVoiceTokenizerLatents> out(static_cast<size_t>(input.batch_size));
    for (int64_t b = 0; b < input.batch_size; ++b) {
        auto& l = out[static_cast<size_t>(b)];
        l.frames = 1;
        l.dim = input.latent_size;
        l.values.assign(latents.begin() + b * input.latent_size, latents.begin() + (b + 1) * input.latent_size);
    }
    return out;
}

}  // namespace engine::models::vibevoice
