/* C-ABI of the sm_100a denoising engine (libdfb_cuda.so).
 *
 * This is the seam the reference crosses between its sampler loop and its GGML
 * graph: diffuse_forward_full / diffuse_forward_cached (src/diffuse-graph.h:16-42,
 * called from src/diffuse-sampler.cpp:149,167,187) plus the per-step candidate
 * extraction / ordering / commit of src/diffuse-sampler.cpp:222-323.  Here one call
 * (dfb_gen_step) runs the active-set build, the whole forward and the sampler on the
 * device; tokens, masks, the K/V cache and the logits buffer stay in HBM.
 *
 * Conventions: plain C types only; every function returns 0 (DFB_OK) or a negative
 * DFB_ERR_* code and leaves a message for dfb_last_error() (thread-local).  The
 * library never exits the process.  Objects are single-threaded: one host thread
 * drives a dfb_ctx at a time; a dfb_model may be shared by several contexts on the
 * same device.  Calls that run the GEMM (dfb_forward, dfb_linear, dfb_gen_step,
 * dfb_linear_noalloc) hold a per-device lock until their work has finished: contexts of
 * one device driven from several host threads take turns, call by call (a GEMM launch
 * needs all of its CTAs resident at once, which two interleaved launches could deny).
 */
#ifndef DIFFUSE_B200_H
#define DIFFUSE_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFB_OK               0
#define DFB_ERR_ARG         -1   /* bad argument / shape / type */
#define DFB_ERR_CUDA        -2   /* CUDA runtime or driver error */
#define DFB_ERR_NOMEM       -3   /* device allocation failed */
#define DFB_ERR_STATE       -4   /* call out of order (e.g. step before begin) */
#define DFB_ERR_TIMEOUT     -5   /* a kernel gave up a bounded wait */
#define DFB_ERR_UNSUPPORTED -6   /* feature not available on this build */

typedef struct dfb_model dfb_model;
typedef struct dfb_ctx dfb_ctx;

/* Hyper-parameters, as resolved from GGUF metadata by the host loader
 * (diffuse-model.cpp:105-128). */
typedef struct {
    int32_t n_vocab, n_embd, n_head, n_head_kv, n_layer, n_ff, n_ctx_max, mask_token_id;
    float   rope_theta, rms_norm_eps;
    int32_t shift_logits; /* 1 for Dream: position i reads logits row max(i-1,0) (diffuse-sampler.cpp:74,235) */
} dfb_hparams;

/* Tensor roles (the tensors diffuse-model.cpp:146-178 resolves). */
enum {
    DFB_TOK_EMBD = 0, DFB_OUTPUT_NORM, DFB_OUTPUT,
    DFB_ATTN_NORM, DFB_WQ, DFB_WK, DFB_WV, DFB_WO, DFB_BQ, DFB_BK, DFB_BV,
    DFB_FFN_NORM, DFB_GATE, DFB_UP, DFB_DOWN,
    DFB_N_ROLES
};

/* GGML type ids accepted for tensors: F32 0, F16 1, Q8_0 8, Q4_K 12, Q6_K 14, BF16 30. */

/* Mirrors diffuse_sampler_params (include/diffuse.h) field by field. */
typedef struct {
    int32_t  n_steps;
    float    temperature;
    int32_t  schedule;          /* 0 COSINE, 1 LINEAR */
    int32_t  remasking;         /* 0 LOW_CONFIDENCE, 1 RANDOM, 2 ENTROPY_EXIT, 3 MASKGIT_PLUS, 4 TOPK_MARGIN */
    uint32_t seed;
    float    entropy_threshold;
    int32_t  use_cache;
    int32_t  cache_refresh;
    int32_t  cache_keep_active;
} dfb_sampler_params;

/* What one denoising step did (feeds the reference's per-step log line,
 * diffuse-sampler.cpp:328-335). */
typedef struct {
    int32_t n_active;    /* query rows the forward computed */
    int32_t n_unmasked;  /* positions committed this step */
    int32_t n_masked;    /* positions still masked after the step */
    int32_t used_cache;  /* 1 if the cached (active-set) forward ran */
    float   fwd_ms;      /* device time of the forward, CUDA events */
    float   step_ms;     /* device time of forward + sampler */
} dfb_step_stats;

const char *dfb_last_error(void);
int dfb_device_count(int *n);

/* ── model ── */
int  dfb_model_create(const dfb_hparams *hp, int device, dfb_model **out);
/* Upload one GGUF tensor (raw block bytes exactly as stored in the file; ne0 is the
 * row length, ne1 the row count).  Replaces diffuse-model.cpp:146-178's binding of
 * GGML tensors; weights are re-tiled for the GEMM on the way in. */
int  dfb_model_set_tensor(dfb_model *m, int role, int layer, int ggml_type, int64_t ne0, int64_t ne1,
                          const void *host_data, size_t nbytes);
int  dfb_model_finalize(dfb_model *m);
void dfb_model_free(dfb_model *m);
/* Device bytes held by the model's weights. */
int  dfb_model_bytes(const dfb_model *m, size_t *bytes);

/* ── context ── */
int  dfb_ctx_create(dfb_model *m, int n_ctx, dfb_ctx **out);
void dfb_ctx_free(dfb_ctx *c);

/* diffuse_forward (diffuse-graph.cpp:676-680): full forward over n host tokens, logits
 * copied to the host buffer [n * n_vocab]. */
int dfb_forward(dfb_ctx *c, const int32_t *tokens, int n, float *logits_host);

/* One linear layer through the production dequant-fused GEMM: y[M x ne1] = x[M x ne0] . W^T
 * for a model weight (host buffers).  Exposed for parity tests of the GEMM alone. */
int dfb_linear(dfb_ctx *c, int role, int layer, const float *x_host, int M, float *y_host);

/* Failure-detection test hook; no counterpart in the reference (its CPU loop has no
 * device waits).  Runs dfb_linear with one split-tile arrival counter preset so that the
 * tile's contributors wait for arrivals that never come, and with every wait of that
 * launch limited to timeout_ns (0 < timeout_ns <= 4 s).  The kernel gives up, raises its
 * error flag and returns; the call returns DFB_ERR_TIMEOUT and resets the counters, so the
 * context stays usable.  Nothing faults or hangs.  A weight and M whose tile 0 is split
 * across CTA pairs (many k-blocks, few output tiles) are needed for the wait to occur. */
int dfb_debug_stalled_linear(dfb_ctx *c, int role, int layer, const float *x_host, int M, float *y_host,
                             unsigned long long timeout_ns);

/* ── tensor parallelism (the north-star's optional TP mode; no counterpart in the reference) ──
 * Rank r of size holds heads [r H/size, (r+1) H/size) of Q/K/V/O (and their KV heads), FFN
 * features [r F/size, ...) of gate/up/down and vocabulary rows [v0, v0 + n_vocab_local) of the
 * lm_head.  O and down are row-parallel: an NCCL all-reduce of their outputs follows each (the
 * split of the residual adds, diffuse-graph.cpp:122-123, 140-142).  The sampler's per-candidate
 * statistics are combined with one all-gather and the entropy with one all-reduce, so every
 * rank makes the same decisions.  temperature > 0 and dfb_linear are not supported in this
 * mode.  NCCL is bound at run time (libnccl.so.2). */
/* A fresh NCCL unique id (nbytes >= 128) for one rank to share with the others. */
int dfb_tp_unique_id(uint8_t *id, int nbytes);
/* Before dfb_model_finalize; every rank calls it at the same time (NCCL communicator setup). */
int dfb_model_set_tp(dfb_model *m, int rank, int size, const uint8_t *id, int nbytes);
/* This rank's place: rank, size, first vocabulary row and vocabulary rows held. */
int dfb_model_tp_info(const dfb_model *m, int *rank, int *size, int *v0, int *n_vocab_local);

/* ── generation: the device side of diffuse_sample (diffuse-sampler.cpp:60-370) ── */
/* Set up seq = prompt ‖ MASK × n_gen, masks, cache and logits buffer on the device. */
int dfb_gen_begin(dfb_ctx *c, const int32_t *prompt, int n_prompt, int n_gen, const dfb_sampler_params *p);
/* One step: active set (or all positions when force_full), forward, sampler.
 * n_unmask_sched is tokens_to_unmask(step, ...) computed by the host exactly as the
 * reference does; for RANDOM remasking `order` holds the host-side shuffle of the
 * candidate indices (length n_masked), else NULL.  Blocks until the step is done and
 * fills *stats (may be NULL). */
int dfb_gen_step(dfb_ctx *c, int step, int n_unmask_sched, int force_full, const int32_t *order,
                 dfb_step_stats *stats);
/* temperature > 0: the uniforms of the next step's draws, one per masked position (batch:
 * per live sequence, concatenated in sequence order), each in ascending position order --
 * the values std::discrete_distribution draws from the loop's mt19937 in the reference's
 * sampling loop (diffuse-sampler.cpp:256-269: std::generate_canonical<double, 53>, taken
 * before any RANDOM shuffle of the same step).  Required before every step at
 * temperature > 0; the step draws token v with probability
 * expf((l_v - max) / T) / sum, and the candidate's confidence is that probability. */
int dfb_gen_set_uniforms(dfb_ctx *c, const double *u, int n);
/* Copy the whole current sequence (prompt ‖ generated) to the host (batch: all
 * sequences' positions, concatenated in order). */
int dfb_gen_tokens(dfb_ctx *c, int32_t *seq_host, int cap);
/* Positions / tokens committed by the last step, in commit order; returns the count. */
int dfb_gen_commits(dfb_ctx *c, int32_t *pos_host, int32_t *tok_host, int cap);

/* Several independent sequences stepped together (no counterpart in the reference,
 * whose API generates one sequence per call, README.md:303 "no batching"): each sequence
 * runs diffuse_sample's loop (diffuse-sampler.cpp:60-370) exactly as it would alone --
 * its own active set and cache fallback, schedule, remasking order and RNG -- while every
 * step's forward packs all sequences' active rows into one GEMM per weight.  Sequence s
 * occupies positions [off_s, off_s + prompt_lens[s] + n_gens[s]) of the concatenated
 * state (dfb_gen_tokens / dfb_gen_logits index it).  At most 256 sequences. */
int dfb_gen_begin_batch(dfb_ctx *c, int n_seq, const int32_t *prompts /* concatenated */,
                        const int32_t *prompt_lens, const int32_t *n_gens, const dfb_sampler_params *p);
/* One step of every sequence that still has masked positions: n_unmask_sched[s] is that
 * sequence's tokens_to_unmask; RANDOM: orders holds each live sequence's shuffle of its
 * candidate indices, concatenated in sequence order.  stats: [n_seq]. */
int dfb_gen_step_batch(dfb_ctx *c, int step, const int32_t *n_unmask_sched, int force_full, const int32_t *orders,
                       dfb_step_stats *stats);
/* Commits of the last step, concatenated in sequence order; counts[s] per sequence. */
int dfb_gen_commits_batch(dfb_ctx *c, int32_t *pos_host, int32_t *tok_host, int32_t *counts, int cap);
/* Rows [row0, row0+nrows) of the persistent logits buffer (parity checks). */
int dfb_gen_logits(dfb_ctx *c, int row0, int nrows, float *host);

/* Optional per-launch timing with CUDA events on the context's stream (off by
 * default; adds event records around each kernel).  Categories accumulate launches,
 * device ms, algorithmic FLOPs and algorithmic bytes (weights once + activations in
 * + outputs) of every forward / step run while enabled. */
enum { DFB_PROF_GEMM_ALL = 0, DFB_PROF_Q4K, DFB_PROF_Q6K, DFB_PROF_Q80, DFB_PROF_F16, DFB_PROF_LMHEAD,
       DFB_PROF_ATTN, DFB_PROF_N };
typedef struct {
    int32_t calls;
    double  ms;
    double  flops;
    double  bytes;
} dfb_prof_entry;
int dfb_ctx_profile(dfb_ctx *c, int enable);                            /* (re)start, zeroed */
int dfb_ctx_profile_read(dfb_ctx *c, dfb_prof_entry *out, int n);      /* n <= DFB_PROF_N */

/* Allocation-free linear layer.  No counterpart in the reference: it exists for callers
 * that cannot allocate device memory while they run (serving stacks whose caching
 * allocator owns all device memory, and code that cannot afford the device-wide
 * synchronization cudaMalloc / cudaFree can cause).  Computes
 * y[M x n_out] = x[M x K] . W^T through the dequant GEMM for an unfused weight
 * (DFB_WO, DFB_DOWN or DFB_OUTPUT); x_f16_dev is a device f16 matrix [M][K] (16-byte
 * aligned), y_dev a device f32 matrix [M][n_out], both owned by the caller.  The GEMM's scratch (split
 * partial sums and arrival counters) is a fixed 8 MiB + 8 KiB array compiled into the
 * library, held by every GPU that loads it until exit; M above 256 or a weight of more
 * than 2040 row tiles is rejected with DFB_ERR_ARG.  Nothing is allocated: no
 * cudaMalloc / cudaFree, no allocating library call.  The first call on a device looks
 * up the scratch address.  All calls share the
 * scratch, so calls that overlap on the GPU race; the call synchronizes `stream`
 * (cudaStream_t as void*, NULL = legacy default stream) before returning. */
int dfb_linear_noalloc(const dfb_model *m, int role, int layer, const void *x_f16_dev, int M, float *y_dev,
                       void *stream);

/* Device stream of a context (cudaStream_t as void*), for callers that time it. */
int dfb_ctx_stream(dfb_ctx *c, void **stream);

#ifdef __cplusplus
}
#endif
#endif
