// CPU oracle for the denoising hot path — TEST INFRASTRUCTURE ONLY.
//
// This library is the checker that tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py compare the CUDA path against.
// It is never linked into, loaded by or called from the product library.
//
// It restates, op by op, the reference's CPU algorithm for one denoising run:
//   * GGUF model resolution         src/diffuse-model.cpp:83-185
//   * forward graph (full, cached)  src/diffuse-graph.cpp:11-160, 395-593
//   * inter-step K/V cache           src/diffuse-cache.h:14-147
//   * sampler loop + schedule        src/diffuse-sampler.cpp:12-370
// and the GGML arithmetic those call (GGML v0.9.8, not vendored in the reference
// checkout): block formats Q4_K / Q6_K / Q8_0 / F16 (pinned against gguf-py's
// dequantizers, tests/golden), RMSNorm, NEOX RoPE with GGML's iterative float
// angle recurrence, softmax, SiLU.
//
// Two arithmetic modes:
//   ORC_MODE_EXACT  f32 math on dequantized weights (the model's mathematics);
//   ORC_MODE_GGML   additionally quantizes matmul activations the way GGML's CPU
//                   mul_mat does before its vec_dot (Q8_K for K-quants, Q8_0 for
//                   Q8_0, F16 for F16).  This mode restates upstream GGML from its
//                   published design and is NOT pinned against a GGML build (the
//                   reference's ggml submodule is empty): parity with it is
//                   reported, not asserted.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_MODE_EXACT = 0, ORC_MODE_GGML = 1 };

typedef struct orc_model orc_model;

// Mirrors diffuse_sampler_params (include/diffuse.h) as a C struct.
typedef struct {
    int32_t  n_steps;
    float    temperature;
    int32_t  schedule;          // 0 COSINE, 1 LINEAR
    int32_t  remasking;         // 0 LOW_CONFIDENCE, 1 RANDOM, 2 ENTROPY_EXIT, 3 MASKGIT_PLUS, 4 TOPK_MARGIN
    uint32_t seed;
    float    entropy_threshold;
    int32_t  use_cache;
    int32_t  cache_refresh;
    int32_t  cache_keep_active;
} orc_sampler_params;

// Per-step record of one generation (all arrays caller-allocated).
typedef struct {
    int32_t  max_steps;         // capacity of the per-step arrays
    int32_t  n_gen;             // capacity per step of commit_pos / commit_tok
    int32_t  steps_run;         // out
    int32_t *n_active;          // [max_steps] rows the forward computed
    int32_t *n_unmask;          // [max_steps] positions committed
    int32_t *commit_pos;        // [max_steps * n_gen] in commit order
    int32_t *commit_tok;        // [max_steps * n_gen]
    float   *final_logits;      // optional [total_len * n_vocab]: logits buffer after the last forward
} orc_trace;

orc_model *orc_load(const char *path);
void       orc_free(orc_model *m);
// ints: n_vocab n_embd n_head n_head_kv n_layer n_ff n_ctx_max mask_token_id is_dream
// floats: rope_theta rms_norm_eps
int orc_hparams(const orc_model *m, int32_t *ints9, float *floats2);
// Raw view of a tensor of the loaded file: GGML type, ne0 (row length), ne1 (rows), data.
int orc_tensor(const orc_model *m, const char *name, int32_t *type, int64_t *ne0,
               int64_t *ne1, const void **data);

// Dequantize n elements (multiple of the block size) of a GGML-typed buffer.
int orc_dequantize(int32_t type, const void *src, int64_t n, float *dst);

// y[M x ne1] = x[M x ne0] . W^T for a named weight, in the given mode.
int orc_matmul(const orc_model *m, const char *name, const float *x, int32_t M, float *y,
               int32_t mode, int32_t n_threads);

// Full forward without cache (diffuse_forward): logits [n x n_vocab].
int orc_forward(const orc_model *m, const int32_t *tokens, int32_t n, float *logits,
                int32_t mode, int32_t n_threads);

// Same, through only the first n_layers transformer layers (then final norm + lm_head):
// a bounded sample of the full forward for CPU timing.
int orc_forward_layers(const orc_model *m, const int32_t *tokens, int32_t n, float *logits,
                       int32_t mode, int32_t n_threads, int32_t n_layers);

// The whole diffuse_sample loop. out_tokens: [n_gen]. trace may be NULL.
int orc_generate(const orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                 const orc_sampler_params *p, int32_t *out_tokens, orc_trace *trace,
                 int32_t mode, int32_t n_threads);

// Step-by-step form of the same loop (teacher-forced checks): a session holds the
// sequence, masks, persistent logits buffer, inter-step cache and mt19937 of one run.
typedef struct orc_session orc_session;
orc_session *orc_sess_new(const orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                          const orc_sampler_params *p, int32_t mode, int32_t n_threads);
void orc_sess_free(orc_session *s);
// The forward of `step` (full or cached by the reference's rules); returns the rows computed.
int orc_sess_forward(orc_session *s, int32_t step);
// The session's own sampler decision on its logits; returns the commit count.
int orc_sess_sample(orc_session *s, int32_t step, int32_t *commit_pos, int32_t *commit_tok);
// Apply commits decided elsewhere (teacher forcing); -1 if a position is not masked.
int orc_sess_commit(orc_session *s, const int32_t *pos, const int32_t *tok, int32_t n);
// Rows of the persistent logits buffer.
int orc_sess_logits(const orc_session *s, int32_t row0, int32_t nrows, float *out);
// Current sequence [n_prompt + n_gen]; returns the masked count.
int orc_sess_tokens(const orc_session *s, int32_t *seq_out);

// One sampler decision on a given logits buffer (teacher-forced checks):
// restates diffuse-sampler.cpp:222-323 for temperature <= 0.  is_masked [total_len]
// is updated in place, seq too.  Returns the number of committed positions and
// writes them (commit order) to commit_pos / commit_tok.  Also reports, per
// candidate in ascending position order, the entropy and confidence it used.
int orc_sampler_step(const float *logits_full, int32_t n_vocab, int32_t total_len,
                     int32_t *seq, uint8_t *is_masked, int32_t is_dream, int32_t step,
                     const orc_sampler_params *p, int32_t *commit_pos, int32_t *commit_tok,
                     float *cand_entropy, float *cand_conf);

// One temperature > 0 draw as the reference's sampling loop makes it
// (diffuse-sampler.cpp:256-269), with the uniform given: probabilities
// expf((l - max) / T) / sum (f32, serial sum), std::discrete_distribution's
// normalised cumulative sums (double), the first index reaching u.  Writes the drawn
// token's probability (the candidate's confidence) and the distance from u to the
// nearest cumulative sum bounding the draw.
int32_t orc_sample_row(const float *row, int32_t n_vocab, float temperature, double u, float *conf, double *margin);

// The uniforms std::discrete_distribution draws from std::mt19937(seed): n values of
// std::generate_canonical<double, 53>.
int orc_canonical(uint32_t seed, int32_t n, double *out);

// Schedule count (diffuse-sampler.cpp:12-31).
int orc_tokens_to_unmask(int32_t step, int32_t total_steps, int32_t total_masked, int32_t schedule);

// Entropy of one logits row (diffuse-sampler.cpp:34-57).
float orc_entropy(const float *row, int32_t n_vocab);

// Seeded random-init GGUF written with the oracle's own code (no product library):
// the converters' metadata and tensor names, weights ~ N(0, w_std) rounded through f16
// (the converters' f16 output; scheme f32 keeps f32), norms = 1, biases ~ N(0, w_std),
// blocks by the reference quantize tool's policy and quantizers.  Same bytes as the
// product's synthesizer for the same spec.
typedef struct {
    int32_t  is_dream;
    int32_t  n_vocab, n_embd, n_head, n_head_kv, n_layer, n_ff, n_ctx, mask_token_id;
    float    rope_theta, rms_norm_eps;
    int32_t  scheme;          // 0 f32, 1 f16, 2 q8_0, 3 q4_k_m
    int32_t  with_bias;
    int32_t  tied_output;
    uint64_t seed;
    float    w_std;
    int32_t  n_threads;
} orc_synth_spec;
int orc_synth_model(const char *path, const orc_synth_spec *spec);

// RoPE angle table of the reference (GGML NEOX): cos/sin[pos][i] for i < n_dims/2.
int orc_rope_table(int32_t n_pos, int32_t n_dims, float freq_base, float *cos_out, float *sin_out);

#ifdef __cplusplus
}
#endif
