#pragma once
// Public C++ API of the B200 denoising engine.
//
// Declaration-for-declaration this is the API of diffuse-cpp's include/diffuse.h
// (model load/free :71-73, context new/free :76-77, diffuse_forward :81-83,
// diffuse_generate :86-91, parameter structs :15-64) so that code written against
// diffuse-cpp recompiles and links against libdiffuse.so from this repository
// unchanged.  The implementation behind it is different: weights live in HBM, the
// forward pass and the remasking sampler run as sm_100a kernels, and the host loop
// only steers them (diffuse_b200.h is the C-ABI underneath).
//
// The autoregressive entry points (ar_generate, ar_speculative_generate) are
// declared so the header stays source-compatible; this library implements the
// denoising path only and those two return an empty vector after logging.

#include <cstdint>
#include <string>
#include <vector>
#include <functional>

struct diffuse_model;
struct diffuse_context;

// Model hyperparameters as read from GGUF metadata.
struct diffuse_hparams {
    uint32_t n_vocab      = 0;
    uint32_t n_embd       = 0;   // hidden size
    uint32_t n_head       = 0;
    uint32_t n_head_kv    = 0;   // < n_head for grouped-query attention
    uint32_t n_layer      = 0;
    uint32_t n_ff         = 0;   // SwiGLU intermediate size
    uint32_t n_ctx_max    = 0;
    float    rope_theta   = 500000.0f;
    float    rms_norm_eps = 1e-5f;
    uint32_t mask_token_id = 0;

    uint32_t n_embd_head() const { return n_head > 0 ? n_embd / n_head : 0; }
};

enum class diffuse_schedule {
    COSINE,
    LINEAR,
};

enum class diffuse_remasking {
    LOW_CONFIDENCE,
    RANDOM,
    ENTROPY_EXIT,   // commit every candidate whose entropy is under the threshold
    MASKGIT_PLUS,   // order by top-1 logit (same key as LOW_CONFIDENCE)
    TOPK_MARGIN,    // order by top-1 minus top-2 logit
};

struct diffuse_sampler_params {
    int      n_steps     = 32;
    float    temperature = 0.0f;  // 0 = argmax
    diffuse_schedule   schedule   = diffuse_schedule::COSINE;
    diffuse_remasking  remasking  = diffuse_remasking::LOW_CONFIDENCE;
    uint32_t seed       = 42;
    float    entropy_threshold = 1.5f;
    bool     use_cache   = true;        // inter-step K/V cache
    int      cache_refresh    = 0;      // full forward every N steps (0 = never)
    int      cache_keep_active = 0;     // keep recently changed positions active N more steps
};

struct diffuse_params {
    std::string model_path;
    std::string prompt;
    int         n_generate  = 128;
    int         n_threads   = 4;
    diffuse_sampler_params sampler;
};

using diffuse_step_callback = std::function<void(
    int step, int total_steps, const std::vector<int32_t>& tokens)>;

// Model: parses the GGUF file and uploads every tensor to the current CUDA device.
// Like diffuse-cpp, a file that cannot be opened or lacks a required key or tensor
// is fatal (message on stderr, exit(1)).
diffuse_model * diffuse_model_load(const std::string & path, int n_threads);
void            diffuse_model_free(diffuse_model * model);
const diffuse_hparams & diffuse_model_hparams(const diffuse_model * model);

// Context: owns the device activations, the K/V cache, the logits buffer and the
// CUDA stream of one generation.  n_ctx sizes the buffers (grown on demand).
diffuse_context * diffuse_context_new(const diffuse_model * model, int n_ctx, int n_threads);
void              diffuse_context_free(diffuse_context * ctx);

// One forward pass over n_tokens positions (no cache).
// logits_out is a host buffer of n_tokens * n_vocab floats, row-major [token][vocab].
bool diffuse_forward(diffuse_context * ctx,
                     const int32_t * tokens, int n_tokens,
                     float * logits_out);

// Full denoising loop; returns the n_generate generated ids.
std::vector<int32_t> diffuse_generate(
    diffuse_context * ctx,
    const std::vector<int32_t> & prompt_tokens,
    int n_generate,
    const diffuse_sampler_params & params,
    diffuse_step_callback callback = nullptr);

// ── Autoregressive API (declared for source compatibility; not implemented) ──
struct ar_sampler_params {
    float    temperature    = 0.0f;
    float    top_p          = 0.9f;
    int      top_k          = 40;
    float    repeat_penalty = 1.1f;
    int      repeat_last_n  = 64;
    uint32_t seed           = 42;
    int      layer_skip     = 0;
    int      sliding_window = 0;
};

using ar_token_callback = std::function<bool(int32_t token, int pos)>;

std::vector<int32_t> ar_generate(
    diffuse_context * ctx,
    const std::vector<int32_t> & prompt_tokens,
    int max_tokens,
    const ar_sampler_params & params,
    ar_token_callback callback = nullptr);

struct ar_spec_params {
    int K = 5;
    int layer_skip = 0;
    int sliding_window = 0;
};

struct ar_spec_stats {
    int total_draft_tokens  = 0;
    int total_accepted      = 0;
    int total_generated     = 0;
    int total_target_batches = 0;
    int total_target_decodes = 0;
    int total_fast_rejects   = 0;
    double prefill_ms = 0;
    double decode_ms  = 0;

    float acceptance_rate() const {
        return total_draft_tokens > 0
            ? (float)total_accepted / total_draft_tokens : 0.0f;
    }
    float tokens_per_target_call() const {
        int calls = total_target_batches + total_target_decodes;
        return calls > 0 ? (float)total_generated / calls : 1.0f;
    }
};

std::vector<int32_t> ar_speculative_generate(
    diffuse_context * target_ctx,
    diffuse_context * draft_ctx,
    const std::vector<int32_t> & prompt_tokens,
    int max_tokens,
    const ar_spec_params & params,
    ar_token_callback callback = nullptr,
    ar_spec_stats * stats_out = nullptr);
