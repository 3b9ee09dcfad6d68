// C++ host layer over the b200diff C ABI, mirroring audio.cpp's entry points for the
// diffusion hot path: same class / function names, same argument meaning, same
// std::runtime_error texts.  An audio.cpp build swaps its ggml-graph bodies for
// these (the weight tensors come from its TensorSource as raw GGUF bytes).
//
//   engine::models::vibevoice::VibeVoiceDPMSolverScheduler          include/engine/models/vibevoice/scheduler.h:14-47
//   engine::models::vibevoice::VibeVoiceDiffusionHeadWeightsRuntime include/engine/models/vibevoice/diffusion_head.h:58-97
//   engine::models::vibevoice::sample_vibevoice_speech_latents       include/engine/models/vibevoice/diffusion_sampler.h:23-26
//   engine::models::stable_audio::foundation::FoundationRfDitRuntime include/engine/models/stable_audio/foundation/rf_dit.h:73-106
//   engine::models::stable_audio::StableAudioRfDitRuntime            include/engine/models/stable_audio/rf_dit.h:78-100
//   engine::models::stable_audio::foundation::OobleckAutoencoderRuntime (decode) include/engine/models/stable_audio/foundation/oobleck_autoencoder.h:71-96
//   engine::models::vibevoice::VibeVoiceTokenizerWeightsRuntime (decode_acoustic) include/engine/models/vibevoice/tokenizer_audio.h:94-140
//   engine::models::vibevoice::VibeVoiceDecoderWeightsRuntime (prefill / cached step) include/engine/models/vibevoice/decoder.h:106-143
//   engine::models::stable_audio::foundation::FoundationConditionerRuntime (encode_one) include/engine/models/stable_audio/foundation/conditioner.h:43-66
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

#include "../../include/b200diff.h"

namespace engine::b200 {

// One weight tensor as stored in the checkpoint (ggml type id, [out, in] dims, raw bytes).
struct RawTensor {
    std::string name;
    int ggml_type = B2D_TYPE_F32;
    std::vector<int64_t> dims;
    std::vector<uint8_t> bytes;
};

// Owns one b2d_ctx (one device).
class Device {
public:
    explicit Device(int device);
    ~Device();
    Device(const Device &) = delete;
    Device & operator=(const Device &) = delete;
    b2d_ctx * ctx() const noexcept { return ctx_; }
    void check(b2d_status status) const;  // throws std::runtime_error(b2d_last_error)

private:
    b2d_ctx * ctx_ = nullptr;
};

std::vector<b2d_tensor_view> views_of(const std::vector<RawTensor> & tensors);

}  // namespace engine::b200

namespace engine::models::vibevoice {

struct VibeVoiceDiffusionHeadConfig {
    int64_t ddpm_num_inference_steps = 20;
    int64_t ddpm_num_steps = 1000;
    std::string ddpm_beta_schedule = "cosine";
    std::string diffusion_type = "ddpm";
    std::string prediction_type = "v_prediction";
    float head_ffn_ratio = 3.0F;
    int64_t head_layers = 4;
    int64_t hidden_size = 0;
    int64_t latent_size = 0;
    float rms_norm_eps = 1.0e-5F;
};

struct VibeVoiceDiffusionPrediction {
    std::vector<float> values;
    int64_t frames = 0;
    int64_t latent_size = 0;
};

struct VibeVoiceTokenizerLatents {
    std::vector<float> values;
    int64_t frames = 0;
    int64_t dim = 0;
};

struct VibeVoiceSchedulerStepResult {
    std::vector<float> prev_sample;
};

// Host scheduler: timesteps and per-step coefficients from b2d_vv_schedule; step() applies
// the DPM-Solver++(2M) update to host vectors exactly as the reference does.
class VibeVoiceDPMSolverScheduler final {
public:
    explicit VibeVoiceDPMSolverScheduler(const VibeVoiceDiffusionHeadConfig & config);
    void set_timesteps(int64_t inference_steps);
    void reset_step_state();
    const std::vector<int64_t> & timesteps() const noexcept { return timesteps_; }
    VibeVoiceSchedulerStepResult step(const std::vector<float> & model_output, int64_t timestep,
                                      const std::vector<float> & sample);
    const VibeVoiceDiffusionHeadConfig & config() const noexcept { return config_; }

private:
    VibeVoiceDiffusionHeadConfig config_;
    std::vector<b2d_vv_step> table_;
    std::vector<int64_t> timesteps_;
    std::vector<float> previous_;
    int64_t step_index_ = -1;
};

class VibeVoiceDiffusionHeadWeightsRuntime final {
public:
    VibeVoiceDiffusionHeadWeightsRuntime(const VibeVoiceDiffusionHeadConfig & config,
                                         const std::vector<engine::b200::RawTensor> & tensors, int device);
    VibeVoiceDiffusionPrediction predict(const std::vector<float> & noisy_images, int64_t frames, int64_t latent_size,
                                         float timestep, const std::vector<float> & condition,
                                         int64_t condition_hidden_size) const;
    const VibeVoiceDiffusionHeadConfig & config() const noexcept { return config_; }
    b2d_ctx * ctx() const noexcept { return device_->ctx(); }
    void check(b2d_status s) const { device_->check(s); }

private:
    VibeVoiceDiffusionHeadConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

struct VibeVoiceSpeechDiffusionInput {
    std::vector<float> positive_condition;
    std::vector<float> negative_condition;
    std::vector<float> initial_speech;
    int64_t batch_size = 0;
    int64_t hidden_size = 0;
    int64_t latent_size = 0;
    int64_t inference_steps = 0;
    float guidance_scale = 1.0F;
};

// VibeVoiceTokenizerConfig fields the acoustic decoder uses (include/engine/models/vibevoice/assets.h:15-37).
struct VibeVoiceTokenizerConfig {
    int64_t vae_dim = 64;
    int64_t decoder_n_filters = 32;
    std::vector<int64_t> decoder_ratios;
    std::vector<int64_t> encoder_depths;  // the decoder runs them reversed (decoder_depths unset)
    bool disable_last_norm = true;
    float layernorm_eps = 1.0e-5F;
};

struct AudioBuffer {
    int sample_rate = 0;
    int channels = 0;
    std::vector<float> samples;  // interleaved frames x channels
};

// The acoustic decode of VibeVoiceTokenizerWeightsRuntime on the GPU (b2d_vvdec_*).
class VibeVoiceTokenizerWeightsRuntime final {
public:
    VibeVoiceTokenizerWeightsRuntime(const VibeVoiceTokenizerConfig & acoustic,
                                     const std::vector<engine::b200::RawTensor> & tensors, int device);
    AudioBuffer decode_acoustic(const VibeVoiceTokenizerLatents & latents) const;

private:
    VibeVoiceTokenizerConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

// VibeVoiceDecoderConfig (include/engine/models/vibevoice/assets.h:39-54), tied embeddings.
struct VibeVoiceDecoderConfig {
    int64_t hidden_size = 0;
    int64_t intermediate_size = 0;
    int64_t max_position_embeddings = 0;
    int64_t num_attention_heads = 0;
    int64_t num_hidden_layers = 0;
    int64_t num_key_value_heads = 0;
    int64_t vocab_size = 0;
    int64_t head_dim = 0;
    float rms_norm_eps = 1.0e-6F;
    float rope_theta = 1000000.0F;
};

struct VibeVoiceDecoderResult {
    std::vector<float> logits;
    std::vector<float> last_hidden;
};

// The Qwen2.5 LM on the GPU (b2d_vvlm_*): one KV cache per runtime; prefill resets it, each step appends.
class VibeVoiceDecoderWeightsRuntime final {
public:
    VibeVoiceDecoderWeightsRuntime(const VibeVoiceDecoderConfig & config,
                                   const std::vector<engine::b200::RawTensor> & tensors, int device);
    VibeVoiceDecoderResult prefill_embeddings(const std::vector<float> & embeddings, int64_t steps) const;
    VibeVoiceDecoderResult cached_step(const std::vector<float> & embedding) const;

private:
    VibeVoiceDecoderConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

std::vector<VibeVoiceTokenizerLatents> sample_vibevoice_speech_latents(
    const VibeVoiceDiffusionHeadWeightsRuntime & prediction_head, VibeVoiceDPMSolverScheduler & scheduler,
    const VibeVoiceSpeechDiffusionInput & input);

}  // namespace engine::models::vibevoice

namespace engine::sampling {

// TorchCudaSamplingPolicy (include/engine/framework/sampling/torch_random.h:12-17)
struct TorchCudaSamplingPolicy {
    int64_t multiprocessor_count = 1;
    int64_t max_threads_per_multiprocessor = 256;
    bool cuda_fast_path = false;
    int cuda_device_index = 0;
};

}  // namespace engine::sampling

namespace engine::models::stable_audio {

struct StableAudioConfig {
    int64_t io_channels = 64;
    int64_t prompt_max_length = 128;
    int64_t embed_dim = 1536;
    int64_t depth = 24;
    int64_t num_heads = 24;
    int64_t cond_token_dim = 768;
    int64_t global_cond_dim = 1536;
    // Stable Audio 3 fields (include/engine/models/stable_audio/assets.h:14-84)
    int64_t cond_dim = 0;
    int64_t local_add_cond_dim = 0;
    int64_t num_memory_tokens = 0;
    bool differential_attention = false;
};

struct StableAudioSamplingState {
    int64_t audio_sample_size = 0;
    int64_t latent_sample_size = 0;
    int64_t batch = 0;
    int64_t channels = 0;
    int64_t schedule_points = 0;
    std::vector<float> schedule;
    std::vector<float> padding_mask;
    std::vector<float> noise;
    std::vector<float> local_add_conditioning;
};

// Token batches and the conditioning batch (include/engine/models/stable_audio/conditioner.h:14-26).
struct StableAudioTokenBatch {
    int64_t batch = 0;
    int64_t tokens = 0;
    std::vector<int32_t> input_ids;
    std::vector<uint8_t> attention_mask;
};

struct StableAudioConditioningBatch {
    StableAudioTokenBatch prompt_tokens;
    StableAudioTokenBatch negative_prompt_tokens;
    std::vector<float> normalized_seconds;
    std::vector<float> seconds_fourier_features;
};

struct StableAudioConditionedInput {
    int64_t batch = 0;
    int64_t cross_tokens = 0;
    int64_t cond_dim = 0;
    std::vector<float> cross_attention;
    std::vector<uint8_t> cross_attention_mask;
    std::vector<float> global;
};

struct StableAudioConditioningInputs {
    StableAudioConditionedInput positive;
    StableAudioConditionedInput negative;
    bool has_negative = false;
};

// Stable Audio 3 rectified-flow DiT: pingpong / euler samplers with APG-CFG, the whole loop on the GPU
// (b2d_sa3_sample).
class StableAudioRfDitRuntime {
public:
    StableAudioRfDitRuntime(const StableAudioConfig & config, const std::vector<engine::b200::RawTensor> & tensors,
                            int device);
    void prepare(const StableAudioSamplingState & sampling, float cfg_scale) const;
    std::vector<float> sample(const StableAudioSamplingState & sampling,
                              const StableAudioConditioningInputs & conditioning, uint64_t seed,
                              uint64_t & rng_offset_blocks, const engine::sampling::TorchCudaSamplingPolicy & rng_policy,
                              std::string_view sampler_type, float cfg_scale, float apg_scale) const;

private:
    StableAudioConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

namespace foundation {

// The Oobleck VAE fields of StableAudioConfig (include/engine/models/stable_audio/assets.h:14-84).
struct OobleckConfig {
    int64_t latent_dim = 64;
    int64_t same_channels = 128;
    std::vector<int64_t> same_c_mults;
    std::vector<int64_t> same_strides;
    int audio_channels = 2;
    int sample_rate = 44100;
};

// T5 fields of StableAudioConfig (include/engine/models/stable_audio/assets.h:14-84).
struct T5Config {
    int64_t t5_hidden_size = 768;
    int64_t t5_layers = 12;
    int64_t t5_attention_heads = 12;
    int64_t t5_head_dim = 64;
    int64_t t5_intermediate_size = 3072;
    int64_t t5_vocab_size = 32128;
    int64_t prompt_max_length = 128;
    float t5_rms_norm_eps = 1.0e-6F;
};

// FoundationConditionerRuntime on the GPU (b2d_saocond_*): encode runs the prompt batch and, when it has one, the
// negative prompt batch, with normalized start seconds 0 and the batch's normalized total seconds, as
// include/engine/models/stable_audio/foundation/conditioner.h:43-72 declares it (encode public, encode_one private).
class FoundationConditionerRuntime {
public:
    FoundationConditionerRuntime(const T5Config & config, const std::vector<engine::b200::RawTensor> & tensors,
                                 int device);
    StableAudioConditioningInputs encode(const StableAudioConditioningBatch & inputs) const;

private:
    // The device path evaluates seconds_start at 0 only (what encode passes); other start values are rejected.
    StableAudioConditionedInput encode_one(const StableAudioTokenBatch & tokens,
                                           const std::vector<float> & normalized_start_seconds,
                                           const std::vector<float> & normalized_total_seconds) const;

    T5Config config_;
    std::unique_ptr<engine::b200::Device> device_;
};

// OobleckAutoencoderRuntime's decode on the GPU (b2d_oobleck_*); audio per prompt as interleaved samples.
class OobleckAutoencoderRuntime {
public:
    OobleckAutoencoderRuntime(const OobleckConfig & config, const std::vector<engine::b200::RawTensor> & tensors,
                              int device);
    std::vector<engine::models::vibevoice::AudioBuffer> decode(const std::vector<float> & latents, int64_t batch,
                                                               int64_t latent_tokens) const;

private:
    OobleckConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

class FoundationRfDitRuntime {
public:
    FoundationRfDitRuntime(const StableAudioConfig & config, const std::vector<engine::b200::RawTensor> & tensors,
                           int device);
    void prepare(const StableAudioSamplingState & sampling, float cfg_scale) const;
    std::vector<float> sample(const StableAudioSamplingState & sampling,
                              const StableAudioConditioningInputs & conditioning, uint64_t seed,
                              uint64_t & rng_offset_blocks, const engine::sampling::TorchCudaSamplingPolicy & rng_policy,
                              std::string_view sampler_type, float sigma_min, float sigma_max, float rho,
                              float cfg_scale, float apg_scale) const;

private:
    StableAudioConfig config_;
    std::unique_ptr<engine::b200::Device> device_;
};

}  // namespace foundation
}  // namespace engine::models::stable_audio
