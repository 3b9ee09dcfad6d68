// Implementation of the audio.cpp-facing C++ classes (engine_b200.h) over the b200diff C ABI.
#include "engine_b200.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace engine::b200 {

Device::Device(int device) {
    const b2d_status s = b2d_create(device, &ctx_);
    if (s != B2D_OK) {
        throw std::runtime_error("b200diff: no usable sm_100 device " + std::to_string(device) + " (status " +
                                 std::to_string(s) + ")");
    }
}

Device::~Device() { b2d_destroy(ctx_); }

void Device::check(b2d_status status) const {
    if (status != B2D_OK) throw std::runtime_error(b2d_last_error(ctx_));
}

std::vector<b2d_tensor_view> views_of(const std::vector<RawTensor> & tensors) {
    std::vector<b2d_tensor_view> views;
    views.reserve(tensors.size());
    for (const auto & t : tensors) {
        b2d_tensor_view v{};
        v.name = t.name.c_str();
        v.ggml_type = t.ggml_type;
        v.ndim = static_cast<int32_t>(t.dims.size());
        for (size_t i = 0; i < t.dims.size() && i < 4; ++i) v.dims[i] = t.dims[i];
        v.data = t.bytes.data();
        v.nbytes = t.bytes.size();
        views.push_back(v);
    }
    return views;
}

}  // namespace engine::b200

namespace engine::models::vibevoice {

// ----------------------------------------------------------------- scheduler
// Validation and messages as VibeVoiceDPMSolverScheduler (src/models/vibevoice/scheduler.cpp:95-274).
VibeVoiceDPMSolverScheduler::VibeVoiceDPMSolverScheduler(const VibeVoiceDiffusionHeadConfig & config)
    : config_(config) {
    if (config_.diffusion_type != "ddpm") throw std::runtime_error("VibeVoice scheduler only supports ddpm diffusion_type");
    if (config_.ddpm_beta_schedule != "cosine")
        throw std::runtime_error("VibeVoice scheduler only supports cosine beta schedule");
    if (config_.prediction_type != "v_prediction")
        throw std::runtime_error("VibeVoice scheduler only supports v_prediction");
    if (config_.ddpm_num_steps <= 0 || config_.ddpm_num_inference_steps <= 0)
        throw std::runtime_error("VibeVoice scheduler requires positive DDPM step counts");
}

void VibeVoiceDPMSolverScheduler::set_timesteps(int64_t inference_steps) {
    if (inference_steps <= 0) throw std::runtime_error("VibeVoice scheduler inference steps must be positive");
    table_.assign(static_cast<size_t>(inference_steps), b2d_vv_step{});
    if (b2d_vv_schedule(config_.ddpm_num_steps, inference_steps, table_.data()) != B2D_OK)
        throw std::runtime_error("VibeVoice scheduler requires positive timestep counts");
    timesteps_.clear();
    for (const auto & s : table_) timesteps_.push_back(s.timestep);
    reset_step_state();
}

void VibeVoiceDPMSolverScheduler::reset_step_state() {
    previous_.clear();
    step_index_ = -1;
}

VibeVoiceSchedulerStepResult VibeVoiceDPMSolverScheduler::step(const std::vector<float> & model_output,
                                                               int64_t timestep, const std::vector<float> & sample) {
    if (table_.empty()) throw std::runtime_error("VibeVoice scheduler set_timesteps must be called before step");
    if (model_output.size() != sample.size())
        throw std::runtime_error("VibeVoice scheduler size mismatch for convert_model_output");
    if (step_index_ < 0) {
        step_index_ = static_cast<int64_t>(timesteps_.size()) - 1;
        for (size_t i = 0; i < timesteps_.size(); ++i)
            if (timesteps_[i] == timestep) {
                step_index_ = static_cast<int64_t>(i);
                break;
            }
    }
    if (step_index_ >= static_cast<int64_t>(table_.size()))
        throw std::runtime_error("VibeVoice scheduler step index is invalid");
    const b2d_vv_step & s = table_[static_cast<size_t>(step_index_)];
    std::vector<float> conv(sample.size()), out(sample.size());
    for (size_t i = 0; i < sample.size(); ++i) conv[i] = s.alpha_s * sample[i] - s.sigma_s * model_output[i];
    if (s.order == 1 || previous_.size() != sample.size()) {
        for (size_t i = 0; i < sample.size(); ++i) out[i] = s.sample_coeff * sample[i] + s.d0_coeff * conv[i];
    } else {
        for (size_t i = 0; i < sample.size(); ++i) {
            const float d1 = s.inv_r0 * (conv[i] - previous_[i]);
            out[i] = s.sample_coeff * sample[i] + s.d0_coeff * conv[i] + 0.5F * s.d0_coeff * d1;
        }
    }
    previous_ = std::move(conv);
    ++step_index_;
    return {std::move(out)};
}

// ------------------------------------------------------------ head runtime
VibeVoiceDiffusionHeadWeightsRuntime::VibeVoiceDiffusionHeadWeightsRuntime(
    const VibeVoiceDiffusionHeadConfig & config, const std::vector<engine::b200::RawTensor> & tensors, int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    const auto views = engine::b200::views_of(tensors);
    const b2d_vv_head_config c{config.hidden_size, config.latent_size, config.head_layers, config.head_ffn_ratio,
                               config.rms_norm_eps, config.ddpm_num_steps};
    device_->check(b2d_vv_head_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

VibeVoiceDiffusionPrediction VibeVoiceDiffusionHeadWeightsRuntime::predict(
    const std::vector<float> & noisy_images, int64_t frames, int64_t latent_size, float timestep,
    const std::vector<float> & condition, int64_t condition_hidden_size) const {
    if (frames <= 0 || latent_size != config_.latent_size || condition_hidden_size != config_.hidden_size)
        throw std::runtime_error("VibeVoice diffusion head received invalid input shape");
    if (static_cast<int64_t>(noisy_images.size()) != frames * latent_size)
        throw std::runtime_error("VibeVoice diffusion head noisy latent payload size mismatch");
    if (static_cast<int64_t>(condition.size()) != frames * condition_hidden_size)
        throw std::runtime_error("VibeVoice diffusion head condition payload size mismatch");
    VibeVoiceDiffusionPrediction out;
    out.frames = frames;
    out.latent_size = latent_size;
    out.values.resize(static_cast<size_t>(frames * latent_size));
    device_->check(b2d_vv_predict(device_->ctx(), noisy_images.data(), frames, latent_size, timestep,
                                  condition.data(), condition_hidden_size, out.values.data(), nullptr));
    return out;
}

// Validation and messages as sample_vibevoice_speech_latents (src/models/vibevoice/diffusion_sampler.cpp:79-121);
// the step loop itself runs on the GPU (b2d_vv_sample).
std::vector<VibeVoiceTokenizerLatents> sample_vibevoice_speech_latents(
    const VibeVoiceDiffusionHeadWeightsRuntime & prediction_head, VibeVoiceDPMSolverScheduler & scheduler,
    const VibeVoiceSpeechDiffusionInput & input) {
    if (input.batch_size <= 0 || input.hidden_size <= 0 || input.latent_size <= 0)
        throw std::runtime_error("VibeVoice diffusion sampler requires positive dimensions");
    if (input.inference_steps <= 0)
        throw std::runtime_error("VibeVoice diffusion sampler requires positive inference steps");
    auto require = [](const std::vector<float> & v, int64_t n, const char * label) {
        if (static_cast<int64_t>(v.size()) != n)
            throw std::runtime_error(std::string("VibeVoice diffusion sampler payload size mismatch for ") + label);
    };
    require(input.positive_condition, input.batch_size * input.hidden_size, "positive_condition");
    require(input.negative_condition, input.batch_size * input.hidden_size, "negative_condition");
    require(input.initial_speech, 2 * input.batch_size * input.latent_size, "initial_speech");
    if (static_cast<int64_t>(scheduler.timesteps().size()) != input.inference_steps)
        throw std::runtime_error("VibeVoice diffusion scheduler timesteps do not match request inference steps");
    if (input.hidden_size != prediction_head.config().hidden_size ||
        input.latent_size != prediction_head.config().latent_size)
        throw std::runtime_error("VibeVoice diffusion head received invalid input shape");
    scheduler.reset_step_state();
    std::vector<float> latents(static_cast<size_t>(input.batch_size * input.latent_size));
    prediction_head.check(b2d_vv_sample(prediction_head.ctx(), input.positive_condition.data(),
                                        input.negative_condition.data(), input.initial_speech.data(),
                                        input.batch_size, input.inference_steps, input.guidance_scale,
                                        latents.data(), nullptr));
    std::vector<VibeVoiceTokenizerLatents> out(static_cast<size_t>(input.batch_size));
    for (int64_t b = 0; b < input.batch_size; ++b) {
        auto & l = out[static_cast<size_t>(b)];
        l.frames = 1;
        l.dim = input.latent_size;
        l.values.assign(latents.begin() + b * input.latent_size, latents.begin() + (b + 1) * input.latent_size);
    }
    return out;
}

}  // namespace engine::models::vibevoice

namespace engine::models::stable_audio {

StableAudioRfDitRuntime::StableAudioRfDitRuntime(const StableAudioConfig & config,
                                                 const std::vector<engine::b200::RawTensor> & tensors, int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    const auto views = engine::b200::views_of(tensors);
    const b2d_sa3_config c{config.embed_dim,          config.depth,
                           config.num_heads,          config.cond_dim,
                           config.global_cond_dim,    config.local_add_cond_dim,
                           config.num_memory_tokens,  config.io_channels,
                           config.prompt_max_length,  config.differential_attention ? 1 : 0};
    device_->check(b2d_sa3_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

void StableAudioRfDitRuntime::prepare(const StableAudioSamplingState & sampling, float) const {
    if (sampling.batch <= 0 || sampling.latent_sample_size <= 0)
        throw std::runtime_error("Stable Audio RF DiT graph requires positive batch and latent length");
}

// Validation and messages as Graph::sample / validate_inputs / make_*_conditioning
// (src/models/stable_audio/rf_dit.cpp:586-622, 868-946); the whole sampler runs on the GPU (b2d_sa3_sample).
std::vector<float> StableAudioRfDitRuntime::sample(const StableAudioSamplingState & sampling,
                                                   const StableAudioConditioningInputs & conditioning, uint64_t seed,
                                                   uint64_t & rng_offset_blocks,
                                                   const engine::sampling::TorchCudaSamplingPolicy & rng_policy,
                                                   std::string_view sampler_type, float cfg_scale,
                                                   float apg_scale) const {
    prepare(sampling, cfg_scale);
    const int64_t B = sampling.batch, T = sampling.latent_sample_size, P1 = config_.prompt_max_length + 1;
    if (static_cast<int64_t>(sampling.noise.size()) != B * config_.io_channels * T ||
        static_cast<int64_t>(sampling.padding_mask.size()) != B * T)
        throw std::runtime_error("Stable Audio RF DiT graph shape mismatch");
    if (sampling.channels != config_.io_channels) throw std::runtime_error("Stable Audio RF DiT channel count mismatch");
    if (conditioning.positive.batch != B || conditioning.positive.cross_tokens != P1 ||
        conditioning.positive.cond_dim != config_.cond_dim ||
        static_cast<int64_t>(conditioning.positive.global.size()) != B * config_.global_cond_dim)
        throw std::runtime_error("Stable Audio RF DiT positive conditioning shape mismatch");
    if (conditioning.has_negative &&
        (conditioning.negative.batch != B || conditioning.negative.cross_tokens != P1 ||
         conditioning.negative.cond_dim != config_.cond_dim))
        throw std::runtime_error("Stable Audio RF DiT negative conditioning shape mismatch");
    const bool pingpong = sampler_type.empty() || sampler_type == "pingpong";
    if (!pingpong && sampler_type != "euler")
        throw std::runtime_error("Stable Audio sampler_type must be pingpong or euler");
    if (static_cast<int64_t>(sampling.local_add_conditioning.size()) != B * T * config_.local_add_cond_dim)
        throw std::runtime_error("Stable Audio RF DiT local conditioning shape mismatch");
    if (sampling.schedule_points <= 1 || static_cast<int64_t>(sampling.schedule.size()) != B * sampling.schedule_points)
        throw std::runtime_error("Stable Audio RF DiT schedule shape mismatch");
    // the negative prompt's token mask as the C ABI's float mask (make_cross_conditioning keeps tokens with mask != 0)
    std::vector<float> nmask;
    if (conditioning.has_negative) {
        nmask.assign(static_cast<size_t>(B * P1), 1.0F);
        for (size_t i = 0; i < nmask.size() && i < conditioning.negative.cross_attention_mask.size(); ++i)
            nmask[i] = conditioning.negative.cross_attention_mask[i] != 0 ? 1.0F : 0.0F;
    }
    b2d_sa3_request rq{};
    rq.batch = B;
    rq.latent_tokens = T;
    rq.schedule_points = sampling.schedule_points;
    rq.noise = sampling.noise.data();
    rq.padding_mask = sampling.padding_mask.data();
    rq.schedule = sampling.schedule.data();
    rq.cross_positive = conditioning.positive.cross_attention.data();
    rq.cross_negative = conditioning.has_negative ? conditioning.negative.cross_attention.data() : nullptr;
    rq.negative_mask = conditioning.has_negative ? nmask.data() : nullptr;
    rq.global_cond = conditioning.positive.global.data();
    rq.local_add = sampling.local_add_conditioning.data();
    rq.cfg_scale = cfg_scale;
    rq.apg_scale = apg_scale;
    rq.sampler = pingpong ? B2D_SA3_PINGPONG : B2D_SA3_EULER;
    rq.seed = seed;
    rq.rng_offset_blocks = &rng_offset_blocks;
    rq.rng_multiprocessor_count = rng_policy.multiprocessor_count;
    rq.rng_max_threads_per_multiprocessor = rng_policy.max_threads_per_multiprocessor;
    std::vector<float> out(sampling.noise.size());
    device_->check(b2d_sa3_sample(device_->ctx(), &rq, out.data(), nullptr));
    return out;
}

}  // namespace engine::models::stable_audio

namespace engine::models::stable_audio::foundation {

FoundationRfDitRuntime::FoundationRfDitRuntime(const StableAudioConfig & config,
                                               const std::vector<engine::b200::RawTensor> & tensors, int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    const auto views = engine::b200::views_of(tensors);
    const b2d_dit_config c{config.embed_dim, config.depth, config.num_heads, config.cond_token_dim,
                           config.global_cond_dim, config.io_channels, config.prompt_max_length};
    device_->check(b2d_dit_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

void FoundationRfDitRuntime::prepare(const StableAudioSamplingState & sampling, float) const {
    if (sampling.batch <= 0 || sampling.latent_sample_size <= 0)
        throw std::runtime_error("Stable Audio Foundation RF DiT graph requires positive batch and latent length");
}

// Validation and messages as Graph::sample / validate_inputs (src/models/stable_audio/foundation/rf_dit.cpp:461-511,
// 1030-1047); the whole sampler runs on the GPU (b2d_dit_sample).
std::vector<float> FoundationRfDitRuntime::sample(const StableAudioSamplingState & sampling,
                                                  const StableAudioConditioningInputs & conditioning, uint64_t seed,
                                                  uint64_t & rng_offset_blocks,
                                                  const engine::sampling::TorchCudaSamplingPolicy & rng_policy,
                                                  std::string_view sampler_type, float sigma_min, float sigma_max,
                                                  float rho, float cfg_scale, float apg_scale) const {
    prepare(sampling, cfg_scale);
    if (!sampler_type.empty() && sampler_type != "euler" && sampler_type != "pingpong" && sampler_type != "dpmpp-2m" &&
        sampler_type != "dpmpp-3m-sde")
        throw std::runtime_error("Stable Audio Foundation sampler_type is not supported for the v sampler");
    // "dpmpp-2m" and "dpmpp-3m-sde" by name; everything else accepted above is the v-DDIM sampler
    const int32_t sampler = sampler_type == "dpmpp-2m"       ? B2D_SAMPLER_DPMPP_2M
                            : sampler_type == "dpmpp-3m-sde" ? B2D_SAMPLER_DPMPP_3M_SDE
                                                             : B2D_SAMPLER_V_DDIM;
    const int64_t B = sampling.batch, T = sampling.latent_sample_size, P2 = config_.prompt_max_length + 2;
    if (conditioning.positive.batch != B || conditioning.positive.cross_tokens != P2 ||
        conditioning.positive.cond_dim != config_.cond_token_dim ||
        static_cast<int64_t>(conditioning.positive.global.size()) != B * config_.global_cond_dim)
        throw std::runtime_error("Stable Audio Foundation RF DiT positive conditioning shape mismatch");
    if (conditioning.has_negative &&
        (conditioning.negative.batch != B || conditioning.negative.cross_tokens != P2 ||
         conditioning.negative.cond_dim != config_.cond_token_dim))
        throw std::runtime_error("Stable Audio Foundation RF DiT negative conditioning shape mismatch");
    if (static_cast<int64_t>(sampling.noise.size()) != B * config_.io_channels * T ||
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
    device_->check(b2d_dit_sample(device_->ctx(), &rq, out.data(), nullptr));
    return out;
}

}  // namespace engine::models::stable_audio::foundation

namespace engine::models::vibevoice {

VibeVoiceTokenizerWeightsRuntime::VibeVoiceTokenizerWeightsRuntime(const VibeVoiceTokenizerConfig & acoustic,
                                                                   const std::vector<engine::b200::RawTensor> & tensors,
                                                                   int device)
    : config_(acoustic), device_(std::make_unique<engine::b200::Device>(device)) {
    if (acoustic.encoder_depths.empty() || acoustic.encoder_depths.size() != acoustic.decoder_ratios.size() + 1 ||
        acoustic.encoder_depths.size() > 8)
        throw std::runtime_error("VibeVoice tokenizer decoder depths/ratios mismatch");
    b2d_vvdec_config c{};
    c.vae_dim = acoustic.vae_dim;
    c.n_filters = acoustic.decoder_n_filters;
    c.n_stages = static_cast<int32_t>(acoustic.encoder_depths.size());
    for (size_t i = 0; i < acoustic.decoder_ratios.size(); ++i) c.ratios[i] = acoustic.decoder_ratios[i];
    for (size_t i = 0; i < acoustic.encoder_depths.size(); ++i) c.depths[i] = acoustic.encoder_depths[i];
    c.disable_last_norm = acoustic.disable_last_norm ? 1 : 0;
    c.eps = acoustic.layernorm_eps;
    const auto views = engine::b200::views_of(tensors);
    device_->check(b2d_vvdec_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

// Validation and messages as decode_acoustic (src/models/vibevoice/tokenizer_audio.cpp:1855-1878).
AudioBuffer VibeVoiceTokenizerWeightsRuntime::decode_acoustic(const VibeVoiceTokenizerLatents & latents) const {
    if (latents.frames <= 0 || latents.dim != config_.vae_dim)
        throw std::runtime_error("VibeVoice acoustic decoder received invalid latent shape");
    if (static_cast<int64_t>(latents.values.size()) != latents.frames * latents.dim)
        throw std::runtime_error("VibeVoice acoustic decoder latent payload size mismatch");
    int64_t hop = 1;
    for (const int64_t r : config_.decoder_ratios) hop *= r;
    AudioBuffer out{24000, 1, std::vector<float>(static_cast<size_t>(latents.frames * hop))};
    device_->check(b2d_vvdec_decode(device_->ctx(), latents.values.data(), latents.frames, out.samples.data(), nullptr));
    return out;
}

}  // namespace engine::models::vibevoice

namespace engine::models::stable_audio::foundation {

OobleckAutoencoderRuntime::OobleckAutoencoderRuntime(const OobleckConfig & config,
                                                     const std::vector<engine::b200::RawTensor> & tensors, int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    if (config.same_strides.empty() || config.same_strides.size() > 8 ||
        config.same_c_mults.size() != config.same_strides.size())
        throw std::runtime_error("Stable Audio Foundation Oobleck c_mults / strides mismatch");
    b2d_oobleck_config c{};
    c.latent_dim = config.latent_dim;
    c.channels = config.same_channels;
    c.audio_channels = config.audio_channels;
    c.n_blocks = static_cast<int32_t>(config.same_strides.size());
    for (size_t i = 0; i < config.same_strides.size(); ++i) {
        c.c_mults[i] = config.same_c_mults[i];
        c.strides[i] = config.same_strides[i];
    }
    const auto views = engine::b200::views_of(tensors);
    device_->check(b2d_oobleck_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

// Validation and messages as DecodeGraph::decode (src/models/stable_audio/foundation/oobleck_autoencoder.cpp:600-640).
std::vector<engine::models::vibevoice::AudioBuffer> OobleckAutoencoderRuntime::decode(const std::vector<float> & latents,
                                                                                      int64_t batch,
                                                                                      int64_t latent_tokens) const {
    if (batch <= 0 || latent_tokens <= 0 ||
        static_cast<int64_t>(latents.size()) != batch * config_.latent_dim * latent_tokens)
        throw std::runtime_error("Stable Audio Foundation Oobleck latent shape mismatch");
    int64_t hop = 1;
    for (const int64_t s : config_.same_strides) hop *= s;
    const int64_t frames = latent_tokens * hop;
    std::vector<float> audio(static_cast<size_t>(batch * frames * config_.audio_channels));
    device_->check(b2d_oobleck_decode(device_->ctx(), latents.data(), batch, latent_tokens, audio.data(), nullptr));
    std::vector<engine::models::vibevoice::AudioBuffer> out;
    const size_t per = static_cast<size_t>(frames * config_.audio_channels);
    for (int64_t b = 0; b < batch; ++b)
        out.push_back({config_.sample_rate, config_.audio_channels,
                       std::vector<float>(audio.begin() + static_cast<std::ptrdiff_t>(b * per),
                                          audio.begin() + static_cast<std::ptrdiff_t>((b + 1) * per))});
    return out;
}

}  // namespace engine::models::stable_audio::foundation

namespace engine::models::vibevoice {

VibeVoiceDecoderWeightsRuntime::VibeVoiceDecoderWeightsRuntime(const VibeVoiceDecoderConfig & config,
                                                               const std::vector<engine::b200::RawTensor> & tensors,
                                                               int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    const b2d_vvlm_config c{config.hidden_size,         config.intermediate_size, config.num_attention_heads,
                            config.num_key_value_heads, config.head_dim,          config.num_hidden_layers,
                            config.vocab_size,          config.max_position_embeddings,
                            config.rms_norm_eps,        config.rope_theta};
    const auto views = engine::b200::views_of(tensors);
    device_->check(b2d_vvlm_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

VibeVoiceDecoderResult VibeVoiceDecoderWeightsRuntime::prefill_embeddings(const std::vector<float> & embeddings,
                                                                          int64_t steps) const {
    if (steps <= 0 || static_cast<int64_t>(embeddings.size()) != steps * config_.hidden_size)
        throw std::runtime_error("VibeVoice decoder prefill embedding payload size mismatch");
    VibeVoiceDecoderResult r{std::vector<float>(static_cast<size_t>(config_.vocab_size)),
                             std::vector<float>(static_cast<size_t>(config_.hidden_size))};
    device_->check(b2d_vvlm_prefill(device_->ctx(), embeddings.data(), steps, r.logits.data(), r.last_hidden.data(),
                                    nullptr));
    return r;
}

VibeVoiceDecoderResult VibeVoiceDecoderWeightsRuntime::cached_step(const std::vector<float> & embedding) const {
    if (static_cast<int64_t>(embedding.size()) != config_.hidden_size)
        throw std::runtime_error("VibeVoice decoder cached step embedding payload size mismatch");
    VibeVoiceDecoderResult r{std::vector<float>(static_cast<size_t>(config_.vocab_size)),
                             std::vector<float>(static_cast<size_t>(config_.hidden_size))};
    device_->check(b2d_vvlm_step(device_->ctx(), embedding.data(), r.logits.data(), r.last_hidden.data(), nullptr));
    return r;
}

}  // namespace engine::models::vibevoice

namespace engine::models::stable_audio::foundation {

FoundationConditionerRuntime::FoundationConditionerRuntime(const T5Config & config,
                                                           const std::vector<engine::b200::RawTensor> & tensors,
                                                           int device)
    : config_(config), device_(std::make_unique<engine::b200::Device>(device)) {
    const b2d_saocond_config c{config.t5_hidden_size,       config.t5_layers,     config.t5_attention_heads,
                               config.t5_head_dim,          config.t5_intermediate_size, config.t5_vocab_size,
                               config.prompt_max_length,    config.t5_rms_norm_eps};
    const auto views = engine::b200::views_of(tensors);
    device_->check(b2d_saocond_load(device_->ctx(), &c, views.data(), static_cast<int32_t>(views.size())));
}

// As FoundationConditionerRuntime::encode (src/models/stable_audio/foundation/conditioner.cpp:411-420).
StableAudioConditioningInputs FoundationConditionerRuntime::encode(const StableAudioConditioningBatch & inputs) const {
    StableAudioConditioningInputs out;
    const std::vector<float> start(static_cast<size_t>(std::max<int64_t>(inputs.prompt_tokens.batch, 0)), 0.0F);
    out.positive = encode_one(inputs.prompt_tokens, start, inputs.normalized_seconds);
    if (inputs.negative_prompt_tokens.batch > 0) {
        out.negative = encode_one(inputs.negative_prompt_tokens, start, inputs.normalized_seconds);
        out.has_negative = true;
    }
    return out;
}

// Validation and messages as encode_one (src/models/stable_audio/foundation/conditioner.cpp:156-163, 422-430).
StableAudioConditionedInput FoundationConditionerRuntime::encode_one(
    const StableAudioTokenBatch & tokens, const std::vector<float> & normalized_start_seconds,
    const std::vector<float> & normalized_total_seconds) const {
    for (const auto * seconds : {&normalized_start_seconds, &normalized_total_seconds}) {
        if (tokens.batch <= 0) throw std::runtime_error("Stable Audio Foundation conditioner requires a positive batch");
        if (static_cast<int64_t>(seconds->size()) != tokens.batch)
            throw std::runtime_error("Stable Audio Foundation conditioner seconds batch does not match prompt batch");
    }
    for (const float s : normalized_start_seconds)
        if (s != 0.0F) throw std::runtime_error("b200: conditioner evaluates seconds_start at 0 only");
    if (tokens.tokens != config_.prompt_max_length)
        throw std::runtime_error("Stable Audio Foundation conditioner token length mismatch");
    const int64_t B = tokens.batch, P = tokens.tokens, d = config_.t5_hidden_size;
    std::vector<float> mask(static_cast<size_t>(B * P));
    for (size_t i = 0; i < mask.size() && i < tokens.attention_mask.size(); ++i)
        mask[i] = tokens.attention_mask[i] != 0 ? 1.0F : 0.0F;
    StableAudioConditionedInput out;
    out.batch = B;
    out.cross_tokens = P + 2;
    out.cond_dim = d;
    out.cross_attention.resize(static_cast<size_t>(B * (P + 2) * d));
    out.global.resize(static_cast<size_t>(B * 2 * d));
    std::vector<float> cmask(static_cast<size_t>(B * (P + 2)));
    device_->check(b2d_saocond_encode(device_->ctx(), tokens.input_ids.data(), mask.data(),
                                      normalized_total_seconds.data(), B, out.cross_attention.data(), cmask.data(),
                                      out.global.data(), nullptr));
    out.cross_attention_mask.assign(cmask.size(), 0);
    for (size_t i = 0; i < cmask.size(); ++i) out.cross_attention_mask[i] = cmask[i] != 0.0F ? 1 : 0;
    return out;
}

}  // namespace engine::models::stable_audio::foundation
