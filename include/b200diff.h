/*
 * b200diff.h -- C ABI of the B200 (sm_100a) diffusion denoising library.
 *
 * This library replaces, for audio.cpp's diffusion hot path, everything below
 * the model-family entry points: the ggml graphs, ggml-cuda kernels and the
 * host-side step loops.  The C++ classes of audio.cpp keep their signatures
 * and call these functions instead of building ggml graphs.  Each entry point
 * names the reference interface it replaces (paths inside audio.cpp).
 *
 * Conventions
 *   - Plain pointers and sizes only.  "host" pointers are ordinary (ideally
 *     pinned) CPU memory; "dev" pointers are device memory of the context's GPU.
 *   - All tensors are row-major with the innermost dimension last.  Weight
 *     tensors keep the ggml/GGUF [out, in] layout and encoding (F32, F16,
 *     BF16, Q8_0 34-byte blocks); the library converts them once at load.
 *   - Every function returns B2D_OK (0) or a negative status; the message of
 *     the last failure on a context is returned by b2d_last_error().  Messages
 *     reuse the reference's exception texts where one exists.
 *   - A context is bound to one device and is not thread-safe (the reference
 *     runtimes are not re-entrant either); independent contexts on different
 *     devices may be used concurrently from different threads or processes.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).
 */
#ifndef B200DIFF_H
#define B200DIFF_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2D_API __attribute__((visibility("default")))
#else
#define B2D_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2d_ctx b2d_ctx;
typedef int b2d_status;

enum {
    B2D_OK = 0,
    B2D_EINVAL = -1,      /* bad argument / shape (reference: std::runtime_error on validation) */
    B2D_ECUDA = -2,       /* CUDA runtime / driver error */
    B2D_ENOMEM = -3,      /* device allocation failed */
    B2D_ESTATE = -4,      /* call order violated (e.g. sample before load) */
    B2D_ENONFINITE = -5,  /* non-finite latent produced (reference: "... non-finite latent ...") */
    B2D_ETIMEOUT = -6,    /* a bounded device-side wait expired; the kernel unwound */
    B2D_ENODEV = -7       /* no usable sm_100 device */
};

/* ggml type ids accepted in tensor views (external/ggml/include/ggml.h enum ggml_type). */
enum { B2D_TYPE_F32 = 0, B2D_TYPE_F16 = 1, B2D_TYPE_Q8_0 = 8, B2D_TYPE_BF16 = 30 };

/* One named weight tensor as stored in GGUF / safetensors (raw bytes, host memory).
 * dims are in the reference's metadata order ([out, in] for linears).
 * Replaces TensorSource::require_tensor_data + BackendWeightStore::load_tensor
 * (include/engine/framework/assets/tensor_source.h:59-120,
 *  include/engine/framework/core/backend_weight_store.h:50-75). */
typedef struct {
    const char* name;
    int32_t ggml_type;
    int32_t ndim;
    int64_t dims[4];
    const void* data;
    size_t nbytes;
} b2d_tensor_view;

/* ------------------------------------------------- weight storage types */
/* audio.cpp's assets::TensorStorageType (include/engine/framework/assets/tensor_source.h:19-34), same values;
 * this path computes with the Native / F32 / F16 / BF16 / Q8_0 members. */
enum { B2D_STORAGE_NATIVE = 0, B2D_STORAGE_F32 = 1, B2D_STORAGE_F16 = 2, B2D_STORAGE_BF16 = 3, B2D_STORAGE_Q8_0 = 13 };

/* ggml type a checkpoint tensor is kept in under a storage request, as the reference's weight store
 * resolves it (include/engine/framework/core/backend_weight_store.h:237-290): Native keeps the stored type; a
 * Q8_0 request falls back to F32 for tensors of rank < 2 or whose last dimension is not a multiple of 32.
 * -1 for storage types this path does not support.  Host only. */
B2D_API int32_t b2d_storage_resolve(int32_t storage_type, const b2d_tensor_view* tensor);
/* Bytes of a tensor of `dims` in ggml type F32 / F16 / BF16 / Q8_0 (0 when not representable). */
B2D_API size_t b2d_tensor_bytes(int32_t ggml_type, const int64_t* dims, int32_t ndim);
/* Quantize-on-load / re-encoding (src/framework/assets/tensor_source.cpp:150-200): decodes `tensor` to fp32
 * and encodes it as `ggml_type` into `out` (exactly b2d_tensor_bytes bytes): F16 round-to-nearest-even,
 * BF16 with ggml's rounding, Q8_0 as quantize_row_q8_0_ref (d = amax / 127, q = roundf(x / d), d as fp16).
 * Host only; the same bytes the reference's weight store produces. */
B2D_API b2d_status b2d_tensor_convert(const b2d_tensor_view* tensor, int32_t ggml_type, void* out, size_t out_bytes);

/* ---------------------------------------------------------------- context */
/* Replaces core::init_backend for these graphs (src/framework/core/backend.cpp:94-144). */
B2D_API b2d_status b2d_create(int device, b2d_ctx** out);
B2D_API void b2d_destroy(b2d_ctx* ctx);
B2D_API const char* b2d_last_error(const b2d_ctx* ctx);
/* Waits for the context's outstanding work and reports any device-side status
 * (non-finite latent, expired wait) raised since the last check.  When it reports one, the context's VibeVoice
 * decoder cache position is also cleared (its next call must be a prefill). */
B2D_API b2d_status b2d_sync(b2d_ctx* ctx, void* stream);
/* Version string of the library build. */
B2D_API const char* b2d_version(void);

/* ------------------------------------------------- VibeVoice diffusion head */
/* Mirrors VibeVoiceDiffusionHeadConfig (include/engine/models/vibevoice/assets.h:56-69). */
typedef struct {
    int64_t hidden_size;
    int64_t latent_size;     /* must be 64 */
    int64_t head_layers;
    float head_ffn_ratio;
    float rms_norm_eps;
    int64_t ddpm_num_steps;  /* cosine schedule length, 1000 */
} b2d_vv_head_config;

/* Per-step scalars of VibeVoiceDPMSolverScheduler::step (src/models/vibevoice/scheduler.cpp:165-274). */
typedef struct {
    int64_t timestep;
    float sigma;         /* sigmas_[step] */
    float sigma_next;    /* sigmas_[step + 1] (0 after the last step) */
    float alpha_s;       /* convert_model_output: x0 = alpha_s * x - sigma_s * v */
    float sigma_s;
    float sample_coeff;  /* sigma_t / sigma_s0 */
    float d0_coeff;      /* -alpha_t * (exp(-h) - 1) */
    float inv_r0;        /* 1 / r0 (second-order steps) */
    int32_t order;       /* 1 or 2 */
} b2d_vv_step;

/* Host-only (no GPU needed).  Fills `steps` entries with the schedule
 * VibeVoiceDPMSolverScheduler(ddpm_num_steps).set_timesteps(steps) produces
 * and the coefficients its step() applies at each index (scheduler.cpp:15-274). */
B2D_API b2d_status b2d_vv_schedule(int64_t ddpm_num_steps, int64_t steps, b2d_vv_step* out);

/* Loads the prediction head from its GGUF/safetensors tensors
 * ("model.prediction_head.*", names as load_vibevoice_diffusion_head_weights,
 *  src/models/vibevoice/diffusion_head.cpp:335-399).
 * Replaces VibeVoiceDiffusionHeadWeightsRuntime's constructor
 * (include/engine/models/vibevoice/diffusion_head.h:60-67). */
B2D_API b2d_status b2d_vv_head_load(b2d_ctx* ctx, const b2d_vv_head_config* config, const b2d_tensor_view* tensors,
                            int32_t n_tensors);

/* One head evaluation: noisy [frames, latent], condition [frames, hidden] -> out [frames, latent].
 * Replaces VibeVoiceDiffusionHeadWeightsRuntime::predict (diffusion_head.h:81-87, diffusion_head.cpp:474-493).
 * Host buffers; synchronous. */
B2D_API b2d_status b2d_vv_predict(b2d_ctx* ctx, const float* noisy, int64_t frames, int64_t latent_size, float timestep,
                          const float* condition, int64_t condition_hidden_size, float* out, void* stream);

/* The whole sampling loop: for each of `steps` DPM-Solver++ steps, predict on
 * [cond || uncond] rows, apply CFG (scale cfg) and the scheduler update, as
 * sample_vibevoice_speech_latents (include/engine/models/vibevoice/diffusion_sampler.h:23-26,
 * src/models/vibevoice/diffusion_sampler.cpp:79-121).
 *   positive_condition, negative_condition: [batch, hidden]
 *   initial_speech: [2 * batch, latent]   out_latents: [batch, latent]
 * Host buffers (pinned memory gives asynchronous copies); returns after the
 * latents are in `out_latents`.  The step loop runs as one captured CUDA graph. */
B2D_API b2d_status b2d_vv_sample(b2d_ctx* ctx, const float* positive_condition, const float* negative_condition,
                         const float* initial_speech, int64_t batch, int64_t steps, float cfg, float* out_latents,
                         void* stream);

/* Same as b2d_vv_sample with device pointers; asynchronous on `stream`
 * (check b2d_sync for device-side status). */
B2D_API b2d_status b2d_vv_sample_device(b2d_ctx* ctx, const float* positive_condition, const float* negative_condition,
                                const float* initial_speech, int64_t batch, int64_t steps, float cfg,
                                float* out_latents, void* stream);

/* -------------------------------------- Stable Audio Open 1.0 ("foundation") DiT */
/* Mirrors the StableAudioConfig fields the foundation DiT uses
 * (include/engine/models/stable_audio/assets.h:14-84).  head_dim = embed_dim / num_heads must be 64. */
typedef struct {
    int64_t embed_dim;          /* 1536 */
    int64_t depth;              /* 24 */
    int64_t num_heads;          /* 24 */
    int64_t cond_token_dim;     /* 768: cross-attention KV heads = cond_token_dim / 64, repeated to num_heads */
    int64_t global_cond_dim;    /* 1536 */
    int64_t io_channels;        /* must be 64 */
    int64_t prompt_max_length;  /* 128: cross tokens = prompt_max_length + 2 */
} b2d_dit_config;

/* FoundationRfDitRuntime::sample sampler_type values: "dpmpp-2m", "dpmpp-3m-sde", and "" / "euler" /
 * "pingpong", which the reference routes to its v-DDIM sampler on sampling.schedule (rf_dit.cpp:461-604). */
enum { B2D_SAMPLER_DPMPP_2M = 0, B2D_SAMPLER_DPMPP_3M_SDE = 1, B2D_SAMPLER_V_DDIM = 2 };

/* One FoundationRfDitRuntime::sample request (include/engine/models/stable_audio/foundation/rf_dit.h:73-106)
 * with its StableAudioSamplingState / StableAudioConditioningInputs payloads (fp32, row-major):
 *   noise [batch, 64, latent_tokens] (BCT), padding_mask [batch, latent_tokens],
 *   cross_positive / cross_negative [batch, prompt_max_length + 2, cond_token_dim] (negative may be NULL: zeros),
 *   global_cond [batch, global_cond_dim].
 * CFG runs when cfg_scale != 1 (graph batch 2 * batch, APG with apg_scale), as the reference's graph cache key. */
typedef struct {
    int64_t batch;
    int64_t latent_tokens;
    int64_t steps;
    const float* noise;
    const float* padding_mask;
    const float* cross_positive;
    const float* cross_negative;
    const float* global_cond;
    float sigma_min, sigma_max, rho;
    float cfg_scale, apg_scale;
    int32_t sampler;            /* B2D_SAMPLER_* */
    const float* schedule;      /* v-DDIM: sampling.schedule [batch, steps + 1]; otherwise unused */
    uint64_t seed;              /* DPM++ 3M SDE noise seed */
    uint64_t* rng_offset_blocks;            /* in/out: TensorIterator Philox offset (may be NULL: starts at 0) */
    int64_t rng_multiprocessor_count;       /* TorchCudaSamplingPolicy (include/engine/framework/sampling/ */
    int64_t rng_max_threads_per_multiprocessor;  /* torch_random.h:12-17); <= 0 selects 1 / 256 */
    /* No counterpart in the reference (0, 0 = the request is the whole batch): this request holds prompts
     * [rng_batch_first, rng_batch_first + batch) of a batch of rng_batch_total prompts and draws its slice of
     * that batched call's noise, so data-parallel shards reproduce the single batched call. */
    int64_t rng_batch_total;
    int64_t rng_batch_first;
} b2d_dit_request;

/* Loads the DiT from its GGUF tensors ("model.model.*", names as load_foundation_rf_dit_weights,
 * src/models/stable_audio/foundation/rf_dit.cpp:379-416).  Replaces the weight load in
 * FoundationRfDitRuntime::prepare (rf_dit.cpp:1173-1180). */
B2D_API b2d_status b2d_dit_load(b2d_ctx* ctx, const b2d_dit_config* config, const b2d_tensor_view* tensors,
                                int32_t n_tensors);

/* The whole sampling loop as one captured CUDA graph: Graph::sample_dpmpp_2m (rf_dit.cpp:798-883),
 * sample_dpmpp_3m_sde (:680-796, Philox noise generated on the device in the TensorIterator layout,
 * *rng_offset_blocks advanced as the reference does) or sample_v_ddim (:514-604, on request->schedule),
 * each with the in-graph CFG/APG of build_cfg_model_output (:988-1028).  Host buffers; returns latents
 * [batch, 64, latent_tokens] (BCT) in out_latents.  Replaces FoundationRfDitRuntime::sample. */
B2D_API b2d_status b2d_dit_sample(b2d_ctx* ctx, const b2d_dit_request* request, float* out_latents, void* stream);

/* Same with every pointer of the request and out_latents in device memory; asynchronous. */
B2D_API b2d_status b2d_dit_sample_device(b2d_ctx* ctx, const b2d_dit_request* request, float* out_latents,
                                         void* stream);

/* ------------------------------------------ Stable Audio 3 rectified-flow DiT */
/* Mirrors the StableAudioConfig fields the SA3 DiT uses (include/engine/models/stable_audio/assets.h:14-84).
 * head_dim = embed_dim / num_heads must be 64, embed_dim a multiple of 128, cond_dim and
 * global_cond_dim multiples of 64. */
typedef struct {
    int64_t embed_dim;
    int64_t depth;
    int64_t num_heads;
    int64_t cond_dim;            /* T5 hidden width of the cross tokens */
    int64_t global_cond_dim;
    int64_t local_add_cond_dim;  /* local-add features per latent token (> 0) */
    int64_t num_memory_tokens;   /* > 0 */
    int64_t io_channels;         /* must be 64 */
    int64_t prompt_max_length;   /* cross tokens = prompt_max_length + 1 */
    int32_t differential_attention;
} b2d_sa3_config;

/* StableAudioRfDitRuntime::sample sampler_type values ("" selects pingpong, rf_dit.cpp:596-599). */
enum { B2D_SA3_PINGPONG = 0, B2D_SA3_EULER = 1 };

/* One StableAudioRfDitRuntime::sample request (include/engine/models/stable_audio/rf_dit.h:78-100) with
 * its StableAudioSamplingState / StableAudioConditioningInputs payloads (fp32, row-major):
 *   noise [batch, 64, latent_tokens] (BCT), padding_mask [batch, latent_tokens],
 *   schedule [batch, schedule_points] (sigma per step, 1 -> 0),
 *   cross_positive / cross_negative [batch, prompt_max_length + 1, cond_dim] (negative NULL: zeros),
 *   negative_mask [batch, prompt_max_length + 1] (NULL: keep every negative token),
 *   global_cond [batch, global_cond_dim], local_add [batch, latent_tokens, local_add_cond_dim].
 * CFG runs when cfg_scale != 1 (graph batch 2 * batch, APG-CFG with apg_scale). */
typedef struct {
    int64_t batch;
    int64_t latent_tokens;
    int64_t schedule_points;
    const float* noise;
    const float* padding_mask;
    const float* schedule;
    const float* cross_positive;
    const float* cross_negative;
    const float* negative_mask;
    const float* global_cond;
    const float* local_add;
    float cfg_scale, apg_scale;
    int32_t sampler;            /* B2D_SA3_* */
    uint64_t seed;              /* pingpong noise seed */
    uint64_t* rng_offset_blocks;            /* in/out: TensorIterator Philox offset (may be NULL: starts at 0) */
    int64_t rng_multiprocessor_count;       /* TorchCudaSamplingPolicy; <= 0 selects 1 */
    int64_t rng_max_threads_per_multiprocessor;  /* <= 0 selects 256 */
    int64_t rng_batch_total;    /* as in b2d_dit_request (0, 0 = the request is the whole batch) */
    int64_t rng_batch_first;
} b2d_sa3_request;

/* Loads the SA3 DiT from its GGUF tensors ("model.model.*", names as load_stable_audio_rf_dit_weights,
 * src/models/stable_audio/rf_dit.cpp:386-585).  Replaces the weight load of StableAudioRfDitRuntime's
 * constructor. */
B2D_API b2d_status b2d_sa3_load(b2d_ctx* ctx, const b2d_sa3_config* config, const b2d_tensor_view* tensors,
                                int32_t n_tensors);

/* The whole sampling loop as one captured CUDA graph: the pingpong sampler (Philox noise generated on the
 * device in the TensorIterator layout, *rng_offset_blocks advanced once per step as the reference does) or
 * euler, with the in-graph APG-CFG of build_cfg_model_output (rf_dit.cpp:834-873).  Host buffers; returns
 * latents [batch, 64, latent_tokens] (BCT).  Replaces StableAudioRfDitRuntime::sample (rf_dit.cpp:586-694). */
B2D_API b2d_status b2d_sa3_sample(b2d_ctx* ctx, const b2d_sa3_request* request, float* out_latents, void* stream);

/* Same with every pointer of the request (schedule included) and out_latents in device memory. */
B2D_API b2d_status b2d_sa3_sample_device(b2d_ctx* ctx, const b2d_sa3_request* request, float* out_latents,
                                         void* stream);

/* --------------------------------------------- Stable Audio Oobleck VAE decode */
/* The StableAudioConfig fields of the Oobleck decoder (include/engine/models/stable_audio/assets.h:14-84):
 * decoder channels = channels x (1, c_mults[0..n_blocks)), all multiples of 64; latent_dim a multiple of 64. */
typedef struct {
    int64_t latent_dim;      /* 64 */
    int64_t channels;        /* same_channels: 128 */
    int64_t audio_channels;  /* 2 */
    int32_t n_blocks;        /* len(same_strides) <= 8 */
    int64_t c_mults[8];      /* same_c_mults: 1, 2, 4, 8, 16 */
    int64_t strides[8];      /* same_strides: 2, 4, 4, 8, 8 */
} b2d_oobleck_config;

/* Loads the decoder half of load_oobleck_autoencoder_weights (src/models/stable_audio/foundation/
 * oobleck_autoencoder.cpp:334-420): "pretransform.model.decoder.layers.*" weight_v / weight_g / bias and snake
 * alpha / beta, weight norm folded on the host as the reference does. */
B2D_API b2d_status b2d_oobleck_load(b2d_ctx* ctx, const b2d_oobleck_config* config, const b2d_tensor_view* tensors,
                                    int32_t n_tensors);

/* OobleckAutoencoderRuntime::decode (oobleck_autoencoder.cpp:600-705, 764-770): latents [batch, latent_dim,
 * latent_tokens] (fp32, host) -> audio [batch, frames, audio_channels] (interleaved, as AudioBuffer::samples),
 * frames = latent_tokens x prod(strides).  Every conv runs as an implicit GEMM on the tensor cores. */
B2D_API b2d_status b2d_oobleck_decode(b2d_ctx* ctx, const float* latents, int64_t batch, int64_t latent_tokens,
                                      float* audio, void* stream);

/* Same with device pointers; asynchronous on `stream`. */
B2D_API b2d_status b2d_oobleck_decode_device(b2d_ctx* ctx, const float* latents, int64_t batch,
                                             int64_t latent_tokens, float* audio, void* stream);

/* ------------------------------------------ VibeVoice acoustic sigma-VAE decode */
/* VibeVoiceTokenizerConfig fields of the acoustic tokenizer's decoder (include/engine/models/vibevoice/assets.h:
 * 15-37): stage s has n_filters << (n_stages - 1 - s) channels (n_filters a multiple of 32; stages narrower than 64 channels run zero-padded to 64), the decoder runs
 * the encoder depths reversed, and stage s > 0 is entered by a transposed conv with ratio ratios[s - 1]. */
typedef struct {
    int64_t vae_dim;            /* 64 */
    int64_t n_filters;          /* decoder_n_filters */
    int32_t n_stages;           /* len(depths) = len(ratios) + 1 */
    int64_t ratios[8];          /* decoder_ratios */
    int64_t depths[8];          /* encoder_depths (the decoder uses them reversed) */
    int32_t disable_last_norm;
    float eps;                  /* layernorm_eps */
} b2d_vvdec_config;

/* Loads "model.acoustic_tokenizer.decoder.*" (load_decoder, src/models/vibevoice/tokenizer_audio.cpp:322-388). */
B2D_API b2d_status b2d_vvdec_load(b2d_ctx* ctx, const b2d_vvdec_config* config, const b2d_tensor_view* tensors,
                                  int32_t n_tensors);

/* VibeVoiceTokenizerWeightsRuntime::decode_acoustic (tokenizer_audio.cpp:1855-1878): latents [frames, vae_dim]
 * (time-major, host) -> mono samples [frames x prod(ratios)].  Convs and FFN linears on the tensor cores. */
B2D_API b2d_status b2d_vvdec_decode(b2d_ctx* ctx, const float* latents, int64_t frames, float* samples, void* stream);

/* Same with device pointers; asynchronous on `stream`. */
B2D_API b2d_status b2d_vvdec_decode_device(b2d_ctx* ctx, const float* latents, int64_t frames, float* samples,
                                           void* stream);

/* ------------------------------------- Stable Audio Open 1.0 conditioner (T5) */
/* StableAudioConfig T5 fields (include/engine/models/stable_audio/assets.h:14-84); cond_dim = hidden, global =
 * 2 x hidden.  head_dim 32 or 64; hidden, heads x head_dim and intermediate multiples of 64. */
typedef struct {
    int64_t hidden;             /* t5_hidden_size: 768 */
    int64_t layers;             /* 12 */
    int64_t heads;              /* 12 */
    int64_t head_dim;           /* 64 */
    int64_t intermediate;       /* 3072 */
    int64_t vocab;              /* t5_vocab_size */
    int64_t prompt_max_length;  /* 128 */
    float eps;                  /* t5_rms_norm_eps */
} b2d_saocond_config;

/* Loads the T5-base encoder ("shared.weight", "encoder.*", load_t5_base_runtime_weights, src/models/stable_audio/
 * foundation/conditioner.cpp:202-233) and the seconds_start / seconds_total number conditioners
 * ("conditioner.conditioners.*", :165-175). */
B2D_API b2d_status b2d_saocond_load(b2d_ctx* ctx, const b2d_saocond_config* config, const b2d_tensor_view* tensors,
                                    int32_t n_tensors);

/* FoundationConditionerRuntime::encode_one (conditioner.cpp:422-471) for one token batch: input_ids / attention_mask
 * (0 / 1) [batch, prompt_max_length], normalized seconds_total [batch] -> cross [batch, prompt_max_length + 2, hidden],
 * cross_mask [batch, prompt_max_length + 2] (may be NULL), global [batch, 2 hidden].  Host buffers.  A negative
 * prompt is a second call (as encode does). */
B2D_API b2d_status b2d_saocond_encode(b2d_ctx* ctx, const int32_t* input_ids, const float* attention_mask,
                                      const float* normalized_seconds, int64_t batch, float* cross, float* cross_mask,
                                      float* global_cond, void* stream);

/* Same with device pointers; asynchronous on `stream`. */
B2D_API b2d_status b2d_saocond_encode_device(b2d_ctx* ctx, const int32_t* input_ids, const float* attention_mask,
                                             const float* normalized_seconds, int64_t batch, float* cross,
                                             float* cross_mask, float* global_cond, void* stream);

/* --------------------------------------------- VibeVoice language model (Qwen2.5) */
/* VibeVoiceDecoderConfig fields (include/engine/models/vibevoice/assets.h:39-54); tied embeddings. */
typedef struct {
    int64_t hidden;          /* hidden_size */
    int64_t intermediate;    /* intermediate_size */
    int64_t heads;           /* num_attention_heads */
    int64_t kv_heads;        /* num_key_value_heads */
    int64_t head_dim;        /* 32, 64 or 128 */
    int64_t layers;          /* num_hidden_layers */
    int64_t vocab;           /* vocab_size */
    int64_t max_positions;   /* KV cache capacity (max_position_embeddings) */
    float eps;               /* rms_norm_eps */
    float rope_theta;
} b2d_vvlm_config;

/* Loads "model.language_model.*" (load_decoder_weights, src/models/vibevoice/decoder.cpp:186-365). */
B2D_API b2d_status b2d_vvlm_load(b2d_ctx* ctx, const b2d_vvlm_config* config, const b2d_tensor_view* tensors,
                                 int32_t n_tensors);

/* VibeVoiceDecoderWeightsRuntime::prefill_embeddings (include/engine/models/vibevoice/decoder.h:129): embeddings
 * [steps, hidden] (host) from position 0, resetting the context's KV cache; returns the last position's logits
 * [vocab] and final-norm hidden state [hidden] (host). */
B2D_API b2d_status b2d_vvlm_prefill(b2d_ctx* ctx, const float* embeddings, int64_t steps, float* logits,
                                    float* last_hidden, void* stream);

/* VibeVoiceDecoderWeightsRuntime::cached_step (decoder.h:134-137): one more position after the cached ones. */
B2D_API b2d_status b2d_vvlm_step(b2d_ctx* ctx, const float* embedding, float* logits, float* last_hidden,
                                 void* stream);

/* b2d_vvlm_prefill / b2d_vvlm_step with device buffers (embeddings in, logits and last_hidden out), asynchronous
 * on `stream`: the last hidden state can feed b2d_vv_sample_device as a condition without a host round trip (the
 * generator's per-token hand-off, src/models/vibevoice/generator.cpp:590-608).  Check b2d_sync for device-side
 * status; a failure reported there also clears the decoder's cache position (prefill again). */
B2D_API b2d_status b2d_vvlm_prefill_device(b2d_ctx* ctx, const float* embeddings, int64_t steps, float* logits,
                                           float* last_hidden, void* stream);
B2D_API b2d_status b2d_vvlm_step_device(b2d_ctx* ctx, const float* embedding, float* logits, float* last_hidden,
                                        void* stream);

/* ------------------------------------------------------ kernel-level entries */
/* Q8_0 rows (GGUF bytes, dev) -> fp32 (dev), bit-exact with dequantize_row_q8_0
 * (external/ggml/src/ggml-quants.c:491-505). */
B2D_API b2d_status b2d_q8_0_dequantize(b2d_ctx* ctx, const void* q8_dev, int64_t rows, int64_t k, float* out_dev,
                               void* stream);

/* Epilogue kinds of the tensor-core GEMM C = A * B^T (ggml_mul_mat(B, A),
 * src/framework/modules/linear_module.cpp:73-108). */
enum {
    B2D_EPI_F32 = 0,    /* out_f32 = acc + bias */
    B2D_EPI_CT = 1,     /* out_{f16|bf16} = acc + bias */
    B2D_EPI_SWIGLU = 2, /* 256-col tiles [128 a | 128 l] -> out_ct[:, n/2] = silu(a) * l */
    B2D_EPI_RESID = 3   /* resid += gate * (acc + bias) */
};

/* A [M, K] and B [N, K] are device fp16 (bf16 = 0) or bf16 (bf16 = 1) matrices.
 * K % 64 == 0.  bn in {64, 128, 192, 256} selects a single-SM 128 x bn tile (N % bn == 0);
 * bn = 512 / 384 select the 2-SM pair tile 256 x 256 / 256 x 192 (N % 256 / N % 192 == 0).
 * SwiGLU: bn 256 or 512.  bias/gate/resid may be NULL where unused. */
B2D_API b2d_status b2d_gemm(b2d_ctx* ctx, int32_t bf16, const void* a_dev, const void* b_dev, int64_t m, int64_t n,
                    int64_t k, int32_t epilogue, int32_t bn, const float* bias_dev, void* out_dev, int64_t ldo,
                    float* resid_dev, int64_t ldr, const float* gate_dev, int64_t ldg, void* stream);

/* The weight-streaming GEMM the VibeVoice head uses when a call has at most 128 rows (HBM-bound: every SM
 * streams weights; each column tile's K range is split over the CTAs of a thread-block cluster whose partial
 * sums are added on chip in a fixed order).  A [M <= 128, K] device fp16 / bf16 (bf16 != 0); W [N, K] on the device either
 * in the same 16-bit type (w_type B2D_TYPE_F16 / B2D_TYPE_BF16) or as ggml Q8_0 blocks (B2D_TYPE_Q8_0,
 * fp16 operands: each block is expanded in shared memory to fp16(q * d) inside the main loop).
 * bn = 0 picks the column-tile width and K split (the cluster size that sums the split partials on chip) for
 * the shape; else bn in {64, 128, 192, 256} (SwiGLU: 256) and split in 1..8 CTAs per column tile
 * (K / 64 >= split).  K % 64 == 0, N % bn == 0; outputs / residual / gate need 16-byte aligned rows.
 * Kernel-level entry for tests and benchmarks; no counterpart in the reference (it stands in for the
 * ggml-cuda GEMV paths behind ggml_mul_mat for few rows). */
B2D_API b2d_status b2d_gemm_stream(b2d_ctx* ctx, int32_t bf16, const void* a_dev, const void* w_dev, int32_t w_type,
                                   int64_t m, int64_t n, int64_t k, int32_t epilogue, int32_t bn, int32_t split,
                                   const float* bias_dev, void* out_dev, int64_t ldo, float* resid_dev, int64_t ldr,
                                   const float* gate_dev, int64_t ldg, void* stream);

/* torch-CUDA-compatible normals on the device (src/framework/sampling/torch_random.cpp):
 * layout 0 = generate_torch_cuda_randn(count, seed) starting at element `offset`;
 * layout 1 = generate_torch_cuda_tensor_iterator_randn(count, seed, offset_blocks = offset, policy).
 * bf16 != 0 rounds each value to bfloat16 like TorchRandnPrecision::BFloat16. */
B2D_API b2d_status b2d_torch_randn(b2d_ctx* ctx, int32_t layout, uint64_t seed, uint64_t offset, int64_t count,
                                   int64_t multiprocessor_count, int64_t max_threads_per_multiprocessor, int32_t bf16,
                                   float* out_dev, void* stream);

/* Flash attention, head_dim 64, scale 1/8: for each sequence s < nseq and head h < heads,
 * O[s, :, h] = softmax(Q[s, :, h] K[s, :, h / kv_rep]^T / 8) V[s, :, h / kv_rep]
 * (ggml_flash_attn_ext as rf_attention uses it, src/models/stable_audio/foundation/rf_dit.cpp:175-198).
 * Q/K/V/O are device fp16 (bf16 = 0) or bf16 matrices; element (s, i, h, j) of Q sits at
 * q + s * q_seq + i * q_row + h * 64 + j (strides in elements), likewise K, V (kv_*) and O (o_*). */
B2D_API b2d_status b2d_attention(b2d_ctx* ctx, int32_t bf16, const void* q, int64_t q_row, int64_t q_seq,
                                 const void* k, const void* v, int64_t kv_row, int64_t kv_seq, void* o,
                                 int64_t o_row, int64_t o_seq, int32_t lq, int32_t lk, int32_t heads, int32_t kv_rep,
                                 int32_t nseq, void* stream);

/* ------------------------------------------------------------- diagnostics */
/* Failure-path self-test: launches one kernel whose bounded device-side wait (the same wait every
 * kernel of the library uses, with `polls` in [1, 2^24] as its limit) can never succeed, so it gives up
 * and the call returns B2D_ETIMEOUT with its message.  No GPU fault is involved: the context, its
 * stream and its status word stay usable for the next call.  No counterpart in the reference. */
B2D_API b2d_status b2d_selftest_wait_timeout(b2d_ctx* ctx, uint32_t polls, void* stream);

/* ------------------------------------------------- allocation-free variant */
/* No counterpart in the reference: an addition for callers that cannot
 * allocate device memory -- hosts that only pass the library buffers they
 * carved from their own pool or arena, or that forbid cudaMalloc while serving.
 *
 * out[m, n] (fp32, leading dim ldo) = A * B^T (+ bias), A [m, k] and B [n, k]
 * fp16 (bf16 = 0) or bf16 (bf16 = 1) device matrices, computed by the same
 * tcgen05 kernel as b2d_gemm with `splits`-way split-K.  The split partials
 * live in a fixed file-scope device array of B2D_NOALLOC_SCRATCH_FLOATS floats
 * (32 MiB), which every GPU that loads this library keeps until the process
 * exits; the call itself allocates nothing.
 *   - Needs no b2d_ctx; runs on the current device.  The first call on a device
 *     looks up the array's device address (cudaGetSymbolAddress); make that
 *     first call before any stream capture.
 *   - Rejects splits * m * n > B2D_NOALLOC_SCRATCH_FLOATS (B2D_EINVAL).
 *   - All calls share the one array, so calls that overlap on the GPU (other
 *     streams, other threads) race; serialise them.  The partials need no
 *     clearing (each split writes its whole slice); the status word is cleared
 *     at the start of every call.
 *   - k % 64 == 0, bn in {64, 128, 256}, n % bn == 0, splits divides k / 64.
 *   - err / err_len (may be NULL / 0) receive a message when the call fails.
 *   - The call returns once its kernels are queued.  If the GEMM's bounded
 *     device-side wait expires, the kernel unwinds, records a code in the
 *     array's status word and the output is written as NaN; call
 *     b2d_gemm_splitk_noalloc_status after the stream to learn of it. */
#define B2D_NOALLOC_SCRATCH_FLOATS (8ll * 1024 * 1024)
B2D_API b2d_status b2d_gemm_splitk_noalloc(int32_t bf16, const void* a_dev, const void* b_dev, int64_t m, int64_t n,
                                           int64_t k, int32_t splits, int32_t bn, const float* bias_dev,
                                           float* out_dev, int64_t ldo, void* stream, char* err, size_t err_len);

/* Waits for `stream`, then reads the status word of b2d_gemm_splitk_noalloc on the current device:
 * B2D_OK, or B2D_ETIMEOUT with a message when a call's bounded wait expired (the word is then
 * cleared).  Allocates nothing.  No counterpart in the reference. */
B2D_API b2d_status b2d_gemm_splitk_noalloc_status(void* stream, char* err, size_t err_len);

/* Test hook for the above: runs the library's bounded wait on an mbarrier nothing arrives on, with
 * `polls` in [1, 2^24] as its limit, so that it gives up and records a timeout in the same status
 * word (no GPU fault).  No counterpart in the reference. */
B2D_API b2d_status b2d_gemm_splitk_noalloc_selftest_timeout(uint32_t polls, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* B200DIFF_H */
