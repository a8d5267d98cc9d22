/* extern "C" face of libdiffuse.so for FFI callers (ctypes, cgo, JNI ...).
 *
 * The C++ API of include/diffuse.h uses std::string / std::vector / std::function,
 * which no FFI can bind.  These wrappers expose the same operations with plain
 * pointers and sizes; each maps onto one diffuse.h call:
 *   dfc_model_load     -> diffuse_model_load     (diffuse-model.cpp:196; errors return NULL
 *                                                 instead of exiting)
 *   dfc_context_new    -> diffuse_context_new    (diffuse-graph.cpp:683)
 *   dfc_forward        -> diffuse_forward        (diffuse-graph.cpp:676)
 *   dfc_generate       -> diffuse_generate       (diffuse-sampler.cpp:373)
 *   dfc_quantize_file  -> tools/quantize.cpp (diffuse-quantize) type policy
 * plus a model synthesizer used to make seeded random-init fixtures.
 */
#ifndef DIFFUSE_C_H
#define DIFFUSE_C_H
#include <stdint.h>
#include "diffuse_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

const char *dfc_last_error(void);

void *dfc_model_load(const char *path, int n_threads);                /* diffuse_model* or NULL */
/* Tensor-parallel rank `rank` of `size` (no counterpart in the reference): the model's heads,
 * FFN features and vocabulary rows are split over the ranks, one process and GPU each
 * (DIFFUSE_DEVICE selects the device); every rank passes the same NCCL id (dfb_tp_unique_id on
 * one rank, shared by the caller) and loads at the same time.  Logits buffers then hold the
 * rank's vocabulary columns (dfb_model_tp_info). */
void *dfc_model_load_tp(const char *path, int rank, int size, const uint8_t *nccl_id, int id_bytes);
/* The loaded model's tensor-parallel place (dfb_model_tp_info). */
int dfc_model_tp_info(const void *model, int32_t *rank, int32_t *size, int32_t *v0, int32_t *n_vocab_local);
void  dfc_model_free(void *model);
/* ints: n_vocab n_embd n_head n_head_kv n_layer n_ff n_ctx_max mask_token_id is_dream
 * floats: rope_theta rms_norm_eps */
int   dfc_model_hparams(const void *model, int32_t *ints9, float *floats2);

void *dfc_context_new(void *model, int n_ctx, int n_threads);         /* diffuse_context* or NULL */
void  dfc_context_free(void *ctx);
/* The engine context (dfb_ctx*) behind a diffuse_context, for direct C-ABI calls. */
void *dfc_context_engine(void *ctx);
/* 1 on success, 0 on failure (like diffuse_forward's bool). */
int   dfc_forward(void *ctx, const int32_t *tokens, int n_tokens, float *logits_out);

/* Per-step record filled by dfc_generate (arrays caller-allocated, may be NULL). */
typedef struct {
    int32_t  max_steps;
    int32_t  steps_run;
    int32_t *n_active;     /* [max_steps] */
    int32_t *n_unmasked;   /* [max_steps] */
    int32_t *commit_pos;   /* [max_steps * n_generate] */
    int32_t *commit_tok;   /* [max_steps * n_generate] */
    float   *fwd_ms;       /* [max_steps] device time of the forward */
    float   *step_ms;      /* [max_steps] device time of forward + sampler */
    double   total_ms;     /* wall time of the whole generation */
} dfc_trace;

/* Runs the denoising loop; writes n_generate ids to out.  Returns the number of
 * steps run, or a negative DFB_ERR_* code. */
int   dfc_generate(void *ctx, const int32_t *prompt, int n_prompt, int n_generate,
                   const dfb_sampler_params *params, int32_t *out, dfc_trace *trace);

/* Per-step record of dfc_generate_batch (arrays caller-allocated, may be NULL). */
typedef struct {
    int32_t  max_steps;
    int32_t  steps_run;
    int32_t *n_active;     /* [max_steps * n_seq] rows each sequence's forward computed */
    int32_t *n_unmasked;   /* [max_steps * n_seq] */
    float   *fwd_ms;       /* [max_steps] device time of the step's forward (all sequences) */
    float   *step_ms;      /* [max_steps] device time of forward + sampler */
    double   total_ms;     /* wall time of the whole call */
} dfc_batch_trace;

/* Several independent sequences generated together (no counterpart in the reference,
 * which generates one sequence per call): each runs diffuse_generate's loop exactly as
 * alone (its own schedule, order, RNG stream seeded with params->seed, and end), while
 * every step runs one forward over all live sequences' active rows.  prompts are
 * concatenated; out receives n_seq x n_generate ids.  Returns the steps run. */
int   dfc_generate_batch(void *ctx, const int32_t *prompts, const int32_t *prompt_lens, int n_seq, int n_generate,
                         const dfb_sampler_params *params, int32_t *out, dfc_batch_trace *trace);

/* diffuse-quantize: type is "q8_0", "q4_k_m" (alias "q4_k"), "q6_k" or "f16". */
int   dfc_quantize_file(const char *in_path, const char *out_path, const char *type, int n_threads);

/* Seeded random-init GGUF with the converters' metadata and tensor names.
 * Weights ~ N(0, w_std) rounded through f16 (the converters' f16 output), norm
 * weights = 1, biases ~ N(0, w_std) when with_bias, then quantized per scheme. */
typedef struct {
    int32_t  is_dream;        /* model_type "dream" (else "llada") */
    int32_t  n_vocab, n_embd, n_head, n_head_kv, n_layer, n_ff, n_ctx, mask_token_id;
    float    rope_theta, rms_norm_eps;
    int32_t  scheme;          /* 0 f32, 1 f16, 2 q8_0, 3 q4_k_m */
    int32_t  with_bias;
    int32_t  tied_output;     /* omit output.weight (lm_head tied to token_embd) */
    uint64_t seed;
    float    w_std;
    int32_t  n_threads;
} dfc_synth_spec;
int   dfc_synth_model(const char *out_path, const dfc_synth_spec *spec);

/* Quantize / dequantize rows with this library's codecs (GGML block formats). */
int   dfc_quantize_rows(int32_t ggml_type, const float *src, int64_t n, void *dst);
int   dfc_dequantize_rows(int32_t ggml_type, const void *src, int64_t n, float *dst);

/* tokens_to_unmask of diffuse-sampler.cpp:12-31, as the host loop computes it. */
int   dfc_tokens_to_unmask(int step, int total_steps, int total_masked, int schedule);

#ifdef __cplusplus
}
#endif
#endif
