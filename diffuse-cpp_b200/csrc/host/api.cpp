// libdiffuse: the reference's public API (include/diffuse.h) on top of the device
// engine (include/diffuse_b200.h), plus the extern "C" wrappers (include/diffuse_c.h).
//
//   diffuse_model_load   — GGUF parse + hparams with the reference's key fallback
//                          (src/diffuse-model.cpp:27-185), every tensor handed to
//                          dfb_model_set_tensor straight from the file mapping.
//   diffuse_generate     — the loop of src/diffuse-sampler.cpp:60-370: schedule,
//                          force-full rule, cache bookkeeping, per-step log line and
//                          callback, timing summary.  Each step is one dfb_gen_step.
//   diffuse_forward      — dfb_forward (src/diffuse-graph.cpp:676-680).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "../../../include/diffuse.h"
#include "../../../include/diffuse_b200.h"
#include "../../../include/diffuse_c.h"
#include "gguf.h"
#include "host_common.h"

namespace dfh {

static thread_local std::string g_err;
int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}
const char *last_error() { return g_err.c_str(); }
bool log_enabled() {
    static int lvl = [] { const char *e = getenv("DIFFUSE_LOG_LEVEL"); return e ? atoi(e) : 1; }();
    return lvl > 0;
}

// diffuse-model.cpp:27-57: diffuse.* then qwen2.* then llama.*
static bool get_u32_multi(const GgufReader &g, const char *suffix, uint32_t *out) {
    for (const char *pre : {"diffuse", "qwen2", "llama"}) {
        const GgufValue *v = g.find(std::string(pre) + "." + suffix);
        if (v) { *out = (uint32_t)v->u; return true; }
    }
    return false;
}
static float get_f32_multi(const GgufReader &g, const char *suffix, float def) {
    for (const char *pre : {"diffuse", "qwen2", "llama"}) {
        const GgufValue *v = g.find(std::string(pre) + "." + suffix);
        if (v) return (float)v->f;
    }
    return def;
}

}  // namespace dfh

using namespace dfh;

struct diffuse_model {
    diffuse_hparams hparams;
    std::string model_type;
    dfb_model *dm = nullptr;
};

struct diffuse_context {
    const diffuse_model *model = nullptr;
    dfb_ctx *dc = nullptr;
    int n_ctx = 0;
    int n_threads = 0;
};

// Loads a GGUF and uploads it; returns nullptr with the error recorded.
// tp: tensor-parallel rank / size and the NCCL id every rank of the group shares (size 1: whole model)
struct TpSpec {
    int rank = 0, size = 1;
    const uint8_t *id = nullptr;
    int id_bytes = 0;
};
static diffuse_model *load_model(const std::string &path, const TpSpec &tp = TpSpec{}) {
    DIFFUSE_LOG("loading model from %s", path.c_str());
    GgufReader g;
    std::string err;
    if (!g.open(path, &err)) { set_error(DFB_ERR_ARG, "failed to open GGUF file: %s", err.c_str()); return nullptr; }
    auto *m = new diffuse_model();
    diffuse_hparams &hp = m->hparams;
    std::string arch = "unknown";
    if (const GgufValue *a = g.find("general.architecture")) arch = a->s;
    else if (g.find("diffuse.block_count")) arch = "diffuse";
    else if (g.find("qwen2.block_count")) arch = "qwen2";
    else if (g.find("llama.block_count")) arch = "llama";
    DIFFUSE_LOG("  detected arch prefix: %s", arch.c_str());
    uint32_t u;
    const char *required[] = {"block_count", "attention.head_count", "attention.head_count_kv", "embedding_length",
                              "feed_forward_length"};
    uint32_t *slots[] = {&hp.n_layer, &hp.n_head, &hp.n_head_kv, &hp.n_embd, &hp.n_ff};
    for (int i = 0; i < 5; i++)
        if (!get_u32_multi(g, required[i], slots[i])) {
            set_error(DFB_ERR_ARG, "missing GGUF metadata key: *.%s (tried diffuse/qwen2/llama)", required[i]);
            delete m;
            return nullptr;
        }
    hp.n_ctx_max = get_u32_multi(g, "context_length", &u) ? u : 4096;
    hp.n_vocab = get_u32_multi(g, "vocab_size", &u) ? u : 0;
    hp.mask_token_id = get_u32_multi(g, "mask_token_id", &u) ? u : 0;
    hp.rope_theta = get_f32_multi(g, "rope.freq_base", 1000000.0f);
    hp.rms_norm_eps = get_f32_multi(g, "attention.layer_norm_rms_epsilon", 1e-6f);
    if (const GgufValue *t = g.find("diffuse.model_type")) m->model_type = t->s;
    else if (arch == "qwen2") m->model_type = "qwen2";
    else if (arch == "llama") m->model_type = "llama";
    else m->model_type = "llada";
    DIFFUSE_LOG("  arch: %s", m->model_type == "dream" ? "Dream (Qwen2.5 backbone, diffusion)"
                              : m->model_type == "llada" ? "LLaDA (Llama backbone, diffusion)" : m->model_type.c_str());
    const GgufTensor *emb = g.tensor("token_embd.weight");
    const GgufTensor *onorm = g.tensor("output_norm.weight");
    if (!emb) { set_error(DFB_ERR_ARG, "tensor not found: token_embd.weight"); delete m; return nullptr; }
    if (!onorm) { set_error(DFB_ERR_ARG, "tensor not found: output_norm.weight"); delete m; return nullptr; }
    if (hp.n_vocab == 0) hp.n_vocab = (uint32_t)emb->ne[1];
    DIFFUSE_LOG("  n_vocab=%u, n_embd=%u, n_head=%u/%u(kv), n_layer=%u, n_ff=%u", hp.n_vocab, hp.n_embd, hp.n_head,
                hp.n_head_kv, hp.n_layer, hp.n_ff);
    DIFFUSE_LOG("  rope_theta=%.0f, rms_norm_eps=%.1e, mask_token=%u", hp.rope_theta, hp.rms_norm_eps, hp.mask_token_id);

    // Every tensor the forward binds (diffuse-model.cpp:146-178) is present with its shape
    // before anything reaches the device: a missing or misshapen tensor is a host error.
    {
        const int64_t d = hp.n_embd, ff = hp.n_ff, V = hp.n_vocab;
        const int64_t kvd = hp.n_head ? (int64_t)hp.n_head_kv * (d / hp.n_head) : 0;
        auto check = [&](const std::string &n, int64_t ne0, int64_t ne1, bool optional) -> bool {
            const GgufTensor *t = g.tensor(n);
            if (!t) {
                if (optional) return true;
                set_error(DFB_ERR_ARG, "tensor not found: %s", n.c_str());
                return false;
            }
            if (t->ne[0] != ne0 || t->ne[1] != ne1) {
                set_error(DFB_ERR_ARG, "tensor %s has shape %lldx%lld, expected %lldx%lld", n.c_str(), (long long)t->ne[0],
                          (long long)t->ne[1], (long long)ne0, (long long)ne1);
                return false;
            }
            return true;
        };
        bool ok = check("token_embd.weight", d, V, false) && check("output_norm.weight", d, 1, false) &&
                  check("output.weight", d, V, true);
        const struct { const char *n; int64_t ne0, ne1; bool opt; } per_layer[] = {
            {"attn_norm.weight", d, 1, false}, {"attn_q.weight", d, d, false}, {"attn_k.weight", d, kvd, false},
            {"attn_v.weight", d, kvd, false}, {"attn_output.weight", d, d, false}, {"ffn_norm.weight", d, 1, false},
            {"ffn_gate.weight", d, ff, false}, {"ffn_up.weight", d, ff, false}, {"ffn_down.weight", ff, d, false},
            {"attn_q.bias", d, 1, true}, {"attn_k.bias", kvd, 1, true}, {"attn_v.bias", kvd, 1, true}};
        for (uint32_t l = 0; ok && l < hp.n_layer; l++)
            for (const auto &e : per_layer) {
                ok = check("blk." + std::to_string(l) + "." + e.n, e.ne0, e.ne1, e.opt);
                if (!ok) break;
            }
        if (!ok) {
            delete m;
            return nullptr;
        }
    }

    dfb_hparams dh{};
    dh.n_vocab = (int)hp.n_vocab; dh.n_embd = (int)hp.n_embd; dh.n_head = (int)hp.n_head;
    dh.n_head_kv = (int)hp.n_head_kv; dh.n_layer = (int)hp.n_layer; dh.n_ff = (int)hp.n_ff;
    dh.n_ctx_max = (int)hp.n_ctx_max; dh.mask_token_id = (int)hp.mask_token_id;
    dh.rope_theta = hp.rope_theta; dh.rms_norm_eps = hp.rms_norm_eps;
    dh.shift_logits = m->model_type == "dream" ? 1 : 0;
    int device = -1;
    if (const char *e = getenv("DIFFUSE_DEVICE")) device = atoi(e);
    if (dfb_model_create(&dh, device, &m->dm) != DFB_OK) {
        set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
        delete m;
        return nullptr;
    }
    if (tp.size > 1 && dfb_model_set_tp(m->dm, tp.rank, tp.size, tp.id, tp.id_bytes) != DFB_OK) {
        set_error(DFB_ERR_ARG, "%s", dfb_last_error());
        dfb_model_free(m->dm);
        delete m;
        return nullptr;
    }
    auto put = [&](int role, int layer, const GgufTensor *t) -> bool {
        if (dfb_model_set_tensor(m->dm, role, layer, t->type, t->ne[0], t->ne[1], t->data, t->nbytes) != DFB_OK) {
            set_error(DFB_ERR_ARG, "%s: %s", t->name.c_str(), dfb_last_error());
            return false;
        }
        return true;
    };
    bool ok = put(DFB_TOK_EMBD, 0, emb) && put(DFB_OUTPUT_NORM, 0, onorm);
    if (ok) {
        if (const GgufTensor *o = g.tensor("output.weight")) ok = put(DFB_OUTPUT, 0, o);  // else tied (model.cpp:157)
    }
    const char *names[] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                           "ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
    const int roles[] = {DFB_ATTN_NORM, DFB_WQ, DFB_WK, DFB_WV, DFB_WO, DFB_FFN_NORM, DFB_GATE, DFB_UP, DFB_DOWN};
    for (uint32_t l = 0; ok && l < hp.n_layer; l++) {
        for (int s = 0; ok && s < 9; s++) {
            const std::string n = "blk." + std::to_string(l) + "." + names[s];
            const GgufTensor *t = g.tensor(n);
            if (!t) { set_error(DFB_ERR_ARG, "tensor not found: %s", n.c_str()); ok = false; break; }
            ok = put(roles[s], (int)l, t);
        }
        const char *bn[] = {"attn_q.bias", "attn_k.bias", "attn_v.bias"};
        const int br[] = {DFB_BQ, DFB_BK, DFB_BV};
        for (int s = 0; ok && s < 3; s++)
            if (const GgufTensor *t = g.tensor("blk." + std::to_string(l) + "." + bn[s])) ok = put(br[s], (int)l, t);
    }
    if (ok && dfb_model_finalize(m->dm) != DFB_OK) {
        set_error(DFB_ERR_CUDA, "upload failed: %s", dfb_last_error());
        ok = false;
    }
    if (!ok) {
        dfb_model_free(m->dm);
        delete m;
        return nullptr;
    }
    size_t bytes = 0;
    dfb_model_bytes(m->dm, &bytes);
    DIFFUSE_LOG("model loaded: %zu tensors, %.2f GB on device", g.tensors().size(), bytes / 1e9);
    return m;
}

diffuse_model *diffuse_model_load(const std::string &path, int n_threads) {
    (void)n_threads;
    diffuse_model *m = load_model(path);
    if (!m) DIFFUSE_DIE("%s", last_error());
    return m;
}

void diffuse_model_free(diffuse_model *model) {
    if (!model) return;
    dfb_model_free(model->dm);
    delete model;
}

const diffuse_hparams &diffuse_model_hparams(const diffuse_model *model) { return model->hparams; }

diffuse_context *diffuse_context_new(const diffuse_model *model, int n_ctx, int n_threads) {
    auto *ctx = new diffuse_context();
    ctx->model = model;
    ctx->n_ctx = n_ctx;
    ctx->n_threads = n_threads;
    if (dfb_ctx_create(model->dm, n_ctx > 0 ? n_ctx : 0, &ctx->dc) != DFB_OK) {
        set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
        delete ctx;
        return nullptr;
    }
    return ctx;
}

void diffuse_context_free(diffuse_context *ctx) {
    if (!ctx) return;
    dfb_ctx_free(ctx->dc);
    delete ctx;
}

bool diffuse_forward(diffuse_context *ctx, const int32_t *tokens, int n_tokens, float *logits_out) {
    if (dfb_forward(ctx->dc, tokens, n_tokens, logits_out) != DFB_OK) {
        DIFFUSE_LOG("forward failed: %s", dfb_last_error());
        return false;
    }
    return true;
}

// diffuse-sampler.cpp:12-31 (same float expressions, same libm calls)
static int tokens_to_unmask(int step, int total_steps, int total_masked, diffuse_schedule schedule) {
    const float t0 = (float)step / total_steps;
    const float t1 = (float)(step + 1) / total_steps;
    float frac;
    if (schedule == diffuse_schedule::COSINE) {
        const float cos0 = cosf(t0 * M_PI * 0.5f);
        const float cos1 = cosf(t1 * M_PI * 0.5f);
        frac = (cos0 - cos1) / cos0;
    } else {
        frac = 1.0f / (total_steps - step);
    }
    int n = (int)roundf(frac * total_masked);
    if (n < 1 && total_masked > 0) n = 1;
    return std::min(n, total_masked);
}

static dfb_sampler_params to_c(const diffuse_sampler_params &p) {
    dfb_sampler_params c{};
    c.n_steps = p.n_steps;
    c.temperature = p.temperature;
    c.schedule = (int)p.schedule;
    c.remasking = (int)p.remasking;
    c.seed = p.seed;
    c.entropy_threshold = p.entropy_threshold;
    c.use_cache = p.use_cache ? 1 : 0;
    c.cache_refresh = p.cache_refresh;
    c.cache_keep_active = p.cache_keep_active;
    return c;
}

// The denoising loop of diffuse-sampler.cpp:60-370; returns steps run or a negative code.
static int generate_impl(diffuse_context *ctx, const std::vector<int32_t> &prompt, int n_generate,
                         const diffuse_sampler_params &params, const diffuse_step_callback &callback,
                         std::vector<int32_t> &out, dfc_trace *trace) {
    using clk = std::chrono::steady_clock;
    const int prompt_len = (int)prompt.size();
    const int total_len = prompt_len + n_generate;
    const dfb_sampler_params cp = to_c(params);
    if (dfb_gen_begin(ctx->dc, prompt.data(), prompt_len, n_generate, &cp) != DFB_OK)
        return set_error(DFB_ERR_ARG, "%s", dfb_last_error());
    const char *remasking_name = params.remasking == diffuse_remasking::ENTROPY_EXIT ? "entropy_exit"
                                 : params.remasking == diffuse_remasking::LOW_CONFIDENCE ? "low_confidence"
                                 : params.remasking == diffuse_remasking::MASKGIT_PLUS ? "maskgit_plus"
                                 : params.remasking == diffuse_remasking::TOPK_MARGIN ? "topk_margin" : "random";
    DIFFUSE_LOG("diffusion: %d steps, %d tokens to generate, scheduler=%s, cache=%s, refresh=%d, keep_active=%d",
                params.n_steps, n_generate, remasking_name, params.use_cache ? "ON" : "OFF", params.cache_refresh,
                params.cache_keep_active);
    std::mt19937 rng(params.seed);
    int n_masked = n_generate;
    bool cache_initialized = false;
    double total_forward_ms = 0, total_sample_ms = 0;
    int actual_steps = 0;
    std::vector<int32_t> seq(total_len), order;
    std::vector<double> unif;
    const auto gen_start = clk::now();
    for (int step = 0; step < params.n_steps && n_masked > 0; step++) {
        actual_steps++;
        const bool force_full = !params.use_cache || !cache_initialized ||
                                (params.cache_refresh > 0 && step > 0 && (step % params.cache_refresh == 0));
        const int n_unmask = tokens_to_unmask(step, params.n_steps, n_masked, params.schedule);
        const int32_t *ord = nullptr;
        if (params.temperature > 0.0f) {
            // the sampling loop's draws come first in the reference's step (sampler.cpp:256-269):
            // one generate_canonical per masked position, in position order
            unif.resize(n_masked);
            for (auto &x : unif) x = std::generate_canonical<double, std::numeric_limits<double>::digits>(rng);
            if (dfb_gen_set_uniforms(ctx->dc, unif.data(), n_masked) != DFB_OK)
                return set_error(DFB_ERR_ARG, "%s", dfb_last_error());
        }
        if (params.remasking == diffuse_remasking::RANDOM) {
            // std::shuffle of the ascending candidate list with the shared mt19937
            // (sampler.cpp:307): the permutation depends only on the count and the rng.
            order.resize(n_masked);
            std::iota(order.begin(), order.end(), 0);
            std::shuffle(order.begin(), order.end(), rng);
            ord = order.data();
        }
        dfb_step_stats st{};
        if (dfb_gen_step(ctx->dc, step, n_unmask, force_full ? 1 : 0, ord, &st) != DFB_OK)
            return set_error(DFB_ERR_CUDA, "forward pass failed at step %d: %s", step, dfb_last_error());
        if (params.use_cache) cache_initialized = true;
        n_masked = st.n_masked;
        total_forward_ms += st.fwd_ms;
        total_sample_ms += st.step_ms - st.fwd_ms;
        if (trace && step < trace->max_steps) {
            if (trace->n_active) trace->n_active[step] = st.n_active;
            if (trace->n_unmasked) trace->n_unmasked[step] = st.n_unmasked;
            if (trace->fwd_ms) trace->fwd_ms[step] = st.fwd_ms;
            if (trace->step_ms) trace->step_ms[step] = st.step_ms;
            if (trace->commit_pos && trace->commit_tok)
                dfb_gen_commits(ctx->dc, trace->commit_pos + (size_t)step * n_generate,
                                trace->commit_tok + (size_t)step * n_generate, n_generate);
        }
        DIFFUSE_LOG("  step %d/%d: unmasked %d tokens, %d remaining (fwd=%.1fms, active=%d/%d%s)", step + 1,
                    params.n_steps, st.n_unmasked, n_masked, st.fwd_ms, st.used_cache ? st.n_active : total_len,
                    total_len, st.used_cache ? " CACHED" : (force_full && step > 0) ? " REFRESH" : "");
        if (callback) {
            if (dfb_gen_tokens(ctx->dc, seq.data(), total_len) != DFB_OK)
                return set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
            callback(step + 1, params.n_steps, seq);
        }
    }
    const double gen_total_ms = std::chrono::duration<double, std::milli>(clk::now() - gen_start).count();
    const double overhead_ms = gen_total_ms - total_forward_ms - total_sample_ms;
    DIFFUSE_LOG("=== TIMING BREAKDOWN (%d steps, cache=%s) ===", actual_steps, params.use_cache ? "ON" : "OFF");
    DIFFUSE_LOG("  forward:   %8.1f ms  (%5.1f%%)  avg=%.1f ms/step", total_forward_ms,
                100.0 * total_forward_ms / gen_total_ms, total_forward_ms / std::max(actual_steps, 1));
    DIFFUSE_LOG("  sampling:  %8.1f ms  (%5.1f%%)  avg=%.1f ms/step", total_sample_ms,
                100.0 * total_sample_ms / gen_total_ms, total_sample_ms / std::max(actual_steps, 1));
    DIFFUSE_LOG("  sorting:   %8.1f ms  (%5.1f%%)", 0.0, 0.0);
    DIFFUSE_LOG("  unmask:    %8.1f ms  (%5.1f%%)", 0.0, 0.0);
    DIFFUSE_LOG("  overhead:  %8.1f ms  (%5.1f%%)", overhead_ms, 100.0 * overhead_ms / gen_total_ms);
    DIFFUSE_LOG("  TOTAL:     %8.1f ms  (%.2f tok/s)", gen_total_ms, 1000.0 * n_generate / gen_total_ms);
    if (dfb_gen_tokens(ctx->dc, seq.data(), total_len) != DFB_OK) return set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
    out.assign(seq.begin() + prompt_len, seq.end());
    if (trace) {
        trace->steps_run = actual_steps;
        trace->total_ms = gen_total_ms;
    }
    return actual_steps;
}

std::vector<int32_t> diffuse_generate(diffuse_context *ctx, const std::vector<int32_t> &prompt_tokens, int n_generate,
                                      const diffuse_sampler_params &params, diffuse_step_callback callback) {
    std::vector<int32_t> out;
    if (generate_impl(ctx, prompt_tokens, n_generate, params, callback, out, nullptr) < 0)
        DIFFUSE_DIE("%s", last_error());  // the reference dies on a failed forward (sampler.cpp:152)
    return out;
}

std::vector<int32_t> ar_generate(diffuse_context *, const std::vector<int32_t> &, int, const ar_sampler_params &,
                                 ar_token_callback) {
    DIFFUSE_LOG("ar_generate: the autoregressive path is not part of this library");
    return {};
}

std::vector<int32_t> ar_speculative_generate(diffuse_context *, diffuse_context *, const std::vector<int32_t> &, int,
                                             const ar_spec_params &, ar_token_callback, ar_spec_stats *) {
    DIFFUSE_LOG("ar_speculative_generate: the autoregressive path is not part of this library");
    return {};
}

// ───────────────────────── extern "C" wrappers ─────────────────────────
extern "C" {

const char *dfc_last_error(void) { return last_error(); }

void *dfc_model_load(const char *path, int n_threads) {
    (void)n_threads;
    if (!path) { set_error(DFB_ERR_ARG, "null path"); return nullptr; }
    return load_model(path);
}
void *dfc_model_load_tp(const char *path, int rank, int size, const uint8_t *nccl_id, int id_bytes) {
    if (!path) { set_error(DFB_ERR_ARG, "null path"); return nullptr; }
    TpSpec tp;
    tp.rank = rank; tp.size = size; tp.id = nccl_id; tp.id_bytes = id_bytes;
    return load_model(path, tp);
}
void dfc_model_free(void *model) { diffuse_model_free((diffuse_model *)model); }

int dfc_model_hparams(const void *model, int32_t *i9, float *f2) {
    if (!model || !i9 || !f2) return set_error(DFB_ERR_ARG, "null pointer");
    const auto *m = (const diffuse_model *)model;
    const diffuse_hparams &hp = m->hparams;
    i9[0] = hp.n_vocab; i9[1] = hp.n_embd; i9[2] = hp.n_head; i9[3] = hp.n_head_kv; i9[4] = hp.n_layer;
    i9[5] = hp.n_ff; i9[6] = hp.n_ctx_max; i9[7] = hp.mask_token_id; i9[8] = m->model_type == "dream";
    f2[0] = hp.rope_theta; f2[1] = hp.rms_norm_eps;
    return DFB_OK;
}

int dfc_model_tp_info(const void *model, int32_t *rank, int32_t *size, int32_t *v0, int32_t *n_vocab_local) {
    if (!model) return set_error(DFB_ERR_ARG, "null model");
    return dfb_model_tp_info(((const diffuse_model *)model)->dm, rank, size, v0, n_vocab_local);
}

void *dfc_context_new(void *model, int n_ctx, int n_threads) {
    if (!model) { set_error(DFB_ERR_ARG, "null model"); return nullptr; }
    return diffuse_context_new((const diffuse_model *)model, n_ctx, n_threads);
}
void dfc_context_free(void *ctx) { diffuse_context_free((diffuse_context *)ctx); }
void *dfc_context_engine(void *ctx) { return ctx ? (void *)((diffuse_context *)ctx)->dc : nullptr; }

int dfc_forward(void *ctx, const int32_t *tokens, int n_tokens, float *logits_out) {
    if (!ctx) return 0;
    if (dfb_forward(((diffuse_context *)ctx)->dc, tokens, n_tokens, logits_out) != DFB_OK) {
        set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
        return 0;
    }
    return 1;
}

int dfc_generate(void *ctx, const int32_t *prompt, int n_prompt, int n_generate, const dfb_sampler_params *p,
                 int32_t *out, dfc_trace *trace) {
    if (!ctx || !p || !out || n_generate <= 0 || n_prompt < 0) return set_error(DFB_ERR_ARG, "bad arguments");
    diffuse_sampler_params sp;
    sp.n_steps = p->n_steps;
    sp.temperature = p->temperature;
    sp.schedule = (diffuse_schedule)p->schedule;
    sp.remasking = (diffuse_remasking)p->remasking;
    sp.seed = p->seed;
    sp.entropy_threshold = p->entropy_threshold;
    sp.use_cache = p->use_cache != 0;
    sp.cache_refresh = p->cache_refresh;
    sp.cache_keep_active = p->cache_keep_active;
    std::vector<int32_t> pr(prompt, prompt + n_prompt), res;
    const int rc = generate_impl((diffuse_context *)ctx, pr, n_generate, sp, nullptr, res, trace);
    if (rc < 0) return rc;
    std::copy(res.begin(), res.end(), out);
    return rc;
}

// Several independent sequences, each running diffuse_sample's loop (diffuse-sampler.cpp:
// 60-370) as it would alone -- its own schedule counts, RNG stream (seeded with params.seed,
// as a separate diffuse_generate call would be) and end when nothing is left masked --
// while each step's forward runs all live sequences in one pass (dfb_gen_step_batch).
int dfc_generate_batch(void *ctx_, const int32_t *prompts, const int32_t *prompt_lens, int n_seq, int n_generate,
                       const dfb_sampler_params *p, int32_t *out, dfc_batch_trace *trace) {
    if (!ctx_ || !p || !out || !prompt_lens || n_generate <= 0 || n_seq <= 0) return set_error(DFB_ERR_ARG, "bad arguments");
    diffuse_context *ctx = (diffuse_context *)ctx_;
    using clk = std::chrono::steady_clock;
    const auto t_start = clk::now();
    std::vector<int32_t> gens(n_seq, n_generate);
    if (dfb_gen_begin_batch(ctx->dc, n_seq, prompts, prompt_lens, gens.data(), p) != DFB_OK)
        return set_error(DFB_ERR_ARG, "%s", dfb_last_error());
    std::vector<std::mt19937> rngs(n_seq, std::mt19937(p->seed));
    std::vector<int> n_masked(n_seq, n_generate);
    std::vector<int32_t> sched(n_seq), orders;
    std::vector<double> unif;
    std::vector<dfb_step_stats> st(n_seq);
    bool cache_initialized = false;
    int steps = 0;
    for (int step = 0; step < p->n_steps; step++) {
        int live = 0;
        for (int sg = 0; sg < n_seq; sg++) live += n_masked[sg] > 0;
        if (!live) break;
        const bool force_full = !p->use_cache || !cache_initialized ||
                                (p->cache_refresh > 0 && step > 0 && (step % p->cache_refresh == 0));
        orders.clear();
        unif.clear();
        for (int sg = 0; sg < n_seq; sg++) {
            if (!n_masked[sg]) { sched[sg] = -1; continue; }
            sched[sg] = tokens_to_unmask(step, p->n_steps, n_masked[sg], (diffuse_schedule)p->schedule);
            if (p->temperature > 0.0f)  // the sequence's sampling draws, before its shuffle (sampler.cpp:256-269)
                for (int i = 0; i < n_masked[sg]; i++)
                    unif.push_back(std::generate_canonical<double, std::numeric_limits<double>::digits>(rngs[sg]));
            if (p->remasking == (int)diffuse_remasking::RANDOM) {
                // the sequence's own std::shuffle of its ascending candidate list (sampler.cpp:307)
                std::vector<int32_t> o(n_masked[sg]);
                std::iota(o.begin(), o.end(), 0);
                std::shuffle(o.begin(), o.end(), rngs[sg]);
                orders.insert(orders.end(), o.begin(), o.end());
            }
        }
        if (p->temperature > 0.0f && dfb_gen_set_uniforms(ctx->dc, unif.data(), (int)unif.size()) != DFB_OK)
            return set_error(DFB_ERR_ARG, "%s", dfb_last_error());
        if (dfb_gen_step_batch(ctx->dc, step, sched.data(), force_full ? 1 : 0, orders.empty() ? nullptr : orders.data(),
                               st.data()) != DFB_OK)
            return set_error(DFB_ERR_CUDA, "forward pass failed at step %d: %s", step, dfb_last_error());
        if (p->use_cache) cache_initialized = true;
        int active = 0, unmasked = 0, remaining = 0;
        for (int sg = 0; sg < n_seq; sg++) {
            if (trace && step < trace->max_steps && trace->n_active) trace->n_active[(size_t)step * n_seq + sg] = st[sg].n_active;
            if (trace && step < trace->max_steps && trace->n_unmasked)
                trace->n_unmasked[(size_t)step * n_seq + sg] = sched[sg] < 0 ? 0 : st[sg].n_unmasked;
            if (sched[sg] >= 0) {
                active += st[sg].n_active;
                unmasked += st[sg].n_unmasked;
                n_masked[sg] = st[sg].n_masked;
            }
            remaining += n_masked[sg];
        }
        if (trace && step < trace->max_steps && trace->fwd_ms) trace->fwd_ms[step] = st[0].fwd_ms;
        if (trace && step < trace->max_steps && trace->step_ms) trace->step_ms[step] = st[0].step_ms;
        DIFFUSE_LOG("  step %d/%d: %d sequences, unmasked %d tokens, %d remaining (fwd=%.1fms, active rows=%d)",
                    step + 1, p->n_steps, live, unmasked, remaining, st[0].fwd_ms, active);
        steps++;
    }
    int total = 0;
    for (int sg = 0; sg < n_seq; sg++) total += prompt_lens[sg] + n_generate;
    std::vector<int32_t> seq(total);
    if (dfb_gen_tokens(ctx->dc, seq.data(), total) != DFB_OK) return set_error(DFB_ERR_CUDA, "%s", dfb_last_error());
    int off = 0;
    for (int sg = 0; sg < n_seq; sg++) {
        std::copy(seq.begin() + off + prompt_lens[sg], seq.begin() + off + prompt_lens[sg] + n_generate,
                  out + (size_t)sg * n_generate);
        off += prompt_lens[sg] + n_generate;
    }
    if (trace) {
        trace->steps_run = steps;
        trace->total_ms = std::chrono::duration<double, std::milli>(clk::now() - t_start).count();
    }
    return steps;
}

int dfc_tokens_to_unmask(int step, int total_steps, int total_masked, int schedule) {
    return tokens_to_unmask(step, total_steps, total_masked, (diffuse_schedule)schedule);
}

}  // extern "C"
