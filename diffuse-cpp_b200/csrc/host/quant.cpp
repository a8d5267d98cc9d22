// Host-side GGML block codecs, the reference's quantization type policy
// (tools/quantize.cpp:31-110), diffuse-quantize, and the random-init model
// synthesizer used for fixtures and benchmarks.
//
// The quantizers restate GGML's reference algorithms (ggml_quantize_chunk, called at
// tools/quantize.cpp:291; GGML v0.9.8 is not vendored in the reference checkout):
//   Q8_0  d = amax / 127, q = round(x / d)            (pinned bit-for-bit to gguf-py)
//   Q4_K  per 32-element sub-block a weighted least-squares search of scale and min
//         over 21 candidate grids (weights sqrt(mean x^2) + |x|), then 6-bit scale and
//         min codes relative to the block's largest, and a final rounding pass
//   Q6_K  per 16-element group a scale search over 19 candidate grids weighted by x^2,
//         then 8-bit signed scale codes relative to the block's largest |scale|
// so that a file re-quantized here carries the blocks diffuse-quantize would write.  The
// steps and constants must match GGML's for identical blocks; the code is this
// library's.  Sums are sequential float sums (the file is built with
// -ffp-contract=off), as written; an FMA-contracting GGML build can differ in the last
// bit of a sum, and with it, rarely, one rounding.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <cuda_fp16.h>

#include "../../../include/diffuse_c.h"
#include "gguf.h"
#include "host_common.h"

namespace dfh {

static uint16_t f2h(float f) {
    const __half h = __float2half_rn(f);
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}
static float h2f(uint16_t u) {
    __half_raw r;
    r.x = u;
    return __half2float(__half(r));
}

// ── block codecs ──
static void quant_q8_0(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / 32; b++) {
        float amax = 0.f;
        for (int j = 0; j < 32; j++) amax = std::max(amax, fabsf(x[32 * b + j]));
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        uint8_t *blk = out + 34 * b;
        const uint16_t dh = f2h(d);
        memcpy(blk, &dh, 2);
        for (int j = 0; j < 32; j++) blk[2 + j] = (uint8_t)(int8_t)roundf(x[32 * b + j] * id);
    }
}

// Round to nearest, ties to even (GGML's nearest_int for |v| < 2^22).
static inline int rne(float v) { return (int)lrintf(v); }

// Weighted search of (scale, min) for n values quantized to [0, nmax] as
// x ~ scale * q + min (min <= 0): the plain min/max grid first, then grids of
// (nmax + rmin + rdelta * i) steps over [min, max] for i = 0..nsteps, each refit by
// weighted least squares (min clamped to 0); the grid with the smallest weighted squared
// error wins.  Returns the scale; *neg_min = -min; q receives the codes.
static float search_scale_min(int n, int nmax, const float *x, const float *w, uint8_t *q, float *neg_min,
                              uint8_t *trial, float rmin, float rdelta, int nsteps) {
    float lo = x[0], hi = x[0], sw = w[0], sx = w[0] * x[0];
    for (int i = 1; i < n; i++) {
        lo = std::min(lo, x[i]);
        hi = std::max(hi, x[i]);
        sw += w[i];
        sx += w[i] * x[i];
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
        memset(q, 0, n);
        *neg_min = -lo;
        return 0.f;
    }
    float inv = nmax / (hi - lo);
    float scale = 1 / inv, mn = lo, best = 0;
    for (int i = 0; i < n; i++) {
        q[i] = (uint8_t)std::max(0, std::min(nmax, rne(inv * (x[i] - lo))));
        const float e = scale * q[i] + mn - x[i];
        best += w[i] * (e * e);
    }
    for (int k = 0; k <= nsteps; k++) {
        inv = (rmin + rdelta * k + nmax) / (hi - lo);
        float sl = 0, sl2 = 0, sxl = 0;
        for (int i = 0; i < n; i++) {
            const int l = std::max(0, std::min(nmax, rne(inv * (x[i] - lo))));
            trial[i] = (uint8_t)l;
            sl += w[i] * l;
            sl2 += w[i] * l * l;
            sxl += w[i] * l * x[i];
        }
        const float det = sw * sl2 - sl * sl;
        if (det <= 0) continue;
        float ts = (sw * sxl - sx * sl) / det, tm = (sl2 * sx - sl * sxl) / det;
        if (tm > 0) {
            tm = 0;
            ts = sxl / sl2;
        }
        float err = 0;
        for (int i = 0; i < n; i++) {
            const float e = ts * trial[i] + tm - x[i];
            err += w[i] * (e * e);
        }
        if (err < best) {
            memcpy(q, trial, n);
            best = err;
            scale = ts;
            mn = tm;
        }
    }
    *neg_min = -mn;
    return scale;
}

static void quant_q4_k(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const float *xb = x + 256 * b;
        uint8_t q[256], trial[32];
        float w[32], scale[8], mn[8], max_scale = 0.f, max_min = 0.f;
        for (int j = 0; j < 8; j++) {
            const float *xs = xb + 32 * j;
            float s2 = 0;
            for (int l = 0; l < 32; l++) s2 += xs[l] * xs[l];
            const float rms = sqrtf(s2 / 32);
            for (int l = 0; l < 32; l++) w[l] = rms + fabsf(xs[l]);
            scale[j] = search_scale_min(32, 15, xs, w, q + 32 * j, &mn[j], trial, -1.f, 0.1f, 20);
            max_scale = std::max(max_scale, scale[j]);
            max_min = std::max(max_min, mn[j]);
        }
        const float inv_s = max_scale > 0 ? 63.f / max_scale : 0.f, inv_m = max_min > 0 ? 63.f / max_min : 0.f;
        uint8_t *blk = out + 144 * b, *sc = blk + 4;
        memset(sc, 0, 12);
        uint8_t ls[8], lm[8];
        for (int j = 0; j < 8; j++) {
            ls[j] = (uint8_t)std::min(63, rne(inv_s * scale[j]));
            lm[j] = (uint8_t)std::min(63, rne(inv_m * mn[j]));
        }
        // 6-bit codes, GGML's packing (get_scale_min_k4 reads it back)
        for (int j = 0; j < 4; j++) {
            sc[j] = ls[j] | (uint8_t)((ls[j + 4] >> 4) << 6);
            sc[j + 4] = lm[j] | (uint8_t)((lm[j + 4] >> 4) << 6);
            sc[j + 8] = (uint8_t)((ls[j + 4] & 0xF) | ((lm[j + 4] & 0xF) << 4));
        }
        const uint16_t dh = f2h(max_scale / 63.f), mh = f2h(max_min / 63.f);
        memcpy(blk, &dh, 2);
        memcpy(blk + 2, &mh, 2);
        for (int j = 0; j < 8; j++) {
            const float dj = h2f(dh) * ls[j];
            if (dj == 0.f) continue;  // the search's codes stay (they decode to -dmin * m anyway)
            const float mj = h2f(mh) * lm[j];
            for (int l = 0; l < 32; l++) q[32 * j + l] = (uint8_t)std::max(0, std::min(15, rne((xb[32 * j + l] + mj) / dj)));
        }
        uint8_t *qs = blk + 16;
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

// Scale of n values quantized to [-nmax, nmax - 1], weighted by x^2: the grid
// -nmax / max (max = the value of largest magnitude) refit by least squares, then 18
// grids -(nmax + 0.1 k) / max, k = -9..9 (k != 0), kept when they improve
// (sum w x l)^2 / (sum w l^2).  q receives codes + nmax.
static float search_scale_sym(int n, int nmax, const float *x, uint8_t *q) {
    float mx = 0, amx = 0;
    for (int i = 0; i < n; i++)
        if (fabsf(x[i]) > amx) {
            amx = fabsf(x[i]);
            mx = x[i];
        }
    if (amx < 1e-15f) {
        memset(q, 0, n);
        return 0.f;
    }
    float inv = -nmax / mx, slx = 0, sl2 = 0;
    for (int i = 0; i < n; i++) {
        const int l = std::max(-nmax, std::min(nmax - 1, rne(inv * x[i])));
        q[i] = (uint8_t)(l + nmax);
        const float w = x[i] * x[i];
        slx += w * x[i] * l;
        sl2 += w * l * l;
    }
    float scale = sl2 ? slx / sl2 : 0.0f, best = scale * slx;
    for (int k = -9; k <= 9; k++) {
        if (k == 0) continue;
        inv = -(nmax + 0.1f * k) / mx;
        slx = sl2 = 0;
        for (int i = 0; i < n; i++) {
            const int l = std::max(-nmax, std::min(nmax - 1, rne(inv * x[i])));
            const float w = x[i] * x[i];
            slx += w * x[i] * l;
            sl2 += w * l * l;
        }
        if (sl2 > 0 && slx * slx > best * sl2) {
            for (int i = 0; i < n; i++) q[i] = (uint8_t)(std::max(-nmax, std::min(nmax - 1, rne(inv * x[i]))) + nmax);
            scale = slx / sl2;
            best = scale * slx;
        }
    }
    return scale;
}

static void quant_q6_k(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / 256; b++) {
        const float *xb = x + 256 * b;
        uint8_t q[256];
        float gs[16], max_scale = 0.f, max_abs = 0.f;
        for (int g = 0; g < 16; g++) {
            gs[g] = search_scale_sym(16, 32, xb + 16 * g, q + 16 * g);
            if (fabsf(gs[g]) > max_abs) {
                max_abs = fabsf(gs[g]);
                max_scale = gs[g];
            }
        }
        uint8_t *blk = out + 210 * b, *ql = blk, *qh = blk + 128;
        int8_t *sc = reinterpret_cast<int8_t *>(blk + 192);
        if (max_abs < 1e-15f) {
            memset(blk, 0, 210);
            continue;
        }
        const float inv = -128.f / max_scale;
        const uint16_t dh = f2h(1 / inv);
        memcpy(blk + 208, &dh, 2);
        for (int g = 0; g < 16; g++) sc[g] = (int8_t)std::min(127, rne(inv * gs[g]));
        for (int g = 0; g < 16; g++) {
            const float dg = h2f(dh) * sc[g];
            if (dg == 0.f) continue;
            for (int l = 0; l < 16; l++) q[16 * g + l] = (uint8_t)(std::max(-32, std::min(31, rne(xb[16 * g + l] / dg))) + 32);
        }
        // ql: low nibbles of elements l and l+64 (bytes 0-31), l+32 and l+96 (32-63) per
        // 128-element half; qh: the 2-bit high parts of elements l, l+32, l+64, l+96
        for (int h = 0; h < 2; h++) {
            const uint8_t *qq = q + 128 * h;
            for (int l = 0; l < 32; l++) {
                ql[64 * h + l] = (uint8_t)((qq[l] & 0xF) | ((qq[l + 64] & 0xF) << 4));
                ql[64 * h + 32 + l] = (uint8_t)((qq[l + 32] & 0xF) | ((qq[l + 96] & 0xF) << 4));
                qh[32 * h + l] = (uint8_t)((qq[l] >> 4) | ((qq[l + 32] >> 4) << 2) | ((qq[l + 64] >> 4) << 4) |
                                           ((qq[l + 96] >> 4) << 6));
            }
        }
    }
}

bool quantize_rows(int32_t type, const float *x, int64_t n, uint8_t *out) {
    if (n % ggml_block_size(type)) return false;
    switch (type) {
        case GT_F32: memcpy(out, x, n * 4); return true;
        case GT_F16: for (int64_t i = 0; i < n; i++) { uint16_t h = f2h(x[i]); memcpy(out + 2 * i, &h, 2); } return true;
        case GT_Q8_0: quant_q8_0(x, n, out); return true;
        case GT_Q4_K: quant_q4_k(x, n, out); return true;
        case GT_Q6_K: quant_q6_k(x, n, out); return true;
        default: return false;
    }
}

bool dequantize_rows(int32_t type, const uint8_t *src, int64_t n, float *dst) {
    if (n % ggml_block_size(type)) return false;
    switch (type) {
        case GT_F32: memcpy(dst, src, n * 4); return true;
        case GT_F16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = h2f(h); } return true;
        case GT_BF16: for (int64_t i = 0; i < n; i++) { uint32_t u = 0; memcpy((uint8_t *)&u + 2, src + 2 * i, 2); memcpy(&dst[i], &u, 4); } return true;
        case GT_Q8_0:
            for (int64_t b = 0; b < n / 32; b++) {
                uint16_t dh; memcpy(&dh, src + 34 * b, 2);
                const float d = h2f(dh);
                for (int l = 0; l < 32; l++) dst[32 * b + l] = d * (float)(int8_t)src[34 * b + 2 + l];
            }
            return true;
        case GT_Q4_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + 144 * b, *q = blk + 4, *qs = blk + 16;
                uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
                const float d = h2f(dh), dmin = h2f(mh);
                for (int j = 0; j < 8; j++) {
                    int sc, mn;
                    if (j < 4) { sc = q[j] & 63; mn = q[j + 4] & 63; }
                    else { sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
                    for (int l = 0; l < 32; l++) {
                        const int v = (j & 1) ? (qs[32 * (j >> 1) + l] >> 4) : (qs[32 * (j >> 1) + l] & 0xF);
                        dst[256 * b + 32 * j + l] = d * sc * v - dmin * mn;
                    }
                }
            }
            return true;
        case GT_Q6_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + 210 * b, *ql = blk, *qh = blk + 128;
                const int8_t *sc = (const int8_t *)(blk + 192);
                uint16_t dh; memcpy(&dh, blk + 208, 2);
                const float d = h2f(dh);
                for (int e = 0; e < 256; e++) {
                    const int h = e / 128, g = (e % 128) / 32, l = e % 32;
                    const uint8_t lb = ql[64 * h + (g & 1) * 32 + l];
                    const int nib = g >= 2 ? (lb >> 4) : (lb & 0xF);
                    const int qv = (nib | (((qh[32 * h + l] >> (2 * g)) & 3) << 4)) - 32;
                    dst[256 * b + e] = d * sc[e / 16] * qv;
                }
            }
            return true;
        default: return false;
    }
}

// ── type policy of diffuse-quantize (tools/quantize.cpp:31-110) ──
enum TClass { TC_NORM, TC_EMBED, TC_OUTPUT, TC_ATTN, TC_FFN, TC_FFN_EDGE };
static TClass classify(const std::string &name, int n_layers) {
    auto has = [&](const char *s) { return name.find(s) != std::string::npos; };
    if (has("_norm") || has("norm.")) return TC_NORM;
    if (has(".bias")) return TC_NORM;
    if (has("token_embd") || has("embed")) return TC_EMBED;
    int layer = -1;
    const size_t p = name.find("blk.");
    if (p != std::string::npos) layer = atoi(name.c_str() + p + 4);
    if (has("attn_q") || has("attn_k") || has("attn_v") || has("attn_output")) return TC_ATTN;
    if (has("ffn_gate") || has("ffn_up") || has("ffn_down")) return (layer == 0 || layer == n_layers - 1) ? TC_FFN_EDGE : TC_FFN;
    if (has("output.weight") || has("lm_head")) return TC_OUTPUT;
    return TC_ATTN;
}
// scheme -> target type per class; -1 for an unknown scheme
static int32_t target_type(const std::string &scheme, TClass tc) {
    if (scheme == "q8_0") return tc == TC_NORM ? GT_F32 : tc == TC_EMBED ? GT_F16 : GT_Q8_0;
    if (scheme == "q4_k_m" || scheme == "q4_k") {
        switch (tc) {
            case TC_NORM: return GT_F32;
            case TC_EMBED: return GT_F16;
            case TC_OUTPUT: case TC_FFN_EDGE: return GT_Q6_K;
            default: return GT_Q4_K;
        }
    }
    if (scheme == "q6_k") return tc == TC_NORM ? GT_F32 : tc == TC_EMBED ? GT_F16 : GT_Q6_K;
    if (scheme == "f16") return tc == TC_NORM ? GT_F32 : GT_F16;
    return -1;
}
static bool is_quantized(int32_t t) { return t == GT_Q8_0 || t == GT_Q4_K || t == GT_Q6_K; }

// Resolved type of one tensor: keeps the source type when the target is not smaller
// (quantize.cpp:197) or the row is not a whole number of target blocks (:142-150).
static int32_t resolve_type(int32_t src, int32_t dst, int64_t ne0) {
    if (dst == src || (!is_quantized(dst) && dst >= src)) return src;
    if (ne0 % ggml_block_size(dst)) return src;
    return dst;
}

// Converts rows [r0, r1) of a tensor to f32 then to dst type (rows of n_per_row).
static void convert_rows(int32_t src_type, const uint8_t *src, int32_t dst_type, uint8_t *dst, int64_t n_per_row,
                         int64_t r0, int64_t r1) {
    std::vector<float> row(n_per_row);
    const int64_t sb = ggml_row_size(src_type, n_per_row), db = ggml_row_size(dst_type, n_per_row);
    for (int64_t r = r0; r < r1; r++) {
        dequantize_rows(src_type, src + r * sb, n_per_row, row.data());
        quantize_rows(dst_type, row.data(), n_per_row, dst + r * db);
    }
}

static void parallel_rows(int64_t rows, int n_threads, const std::function<void(int64_t, int64_t)> &fn) {
    n_threads = std::max(1, std::min<int>(n_threads, (int)std::max<int64_t>(1, rows / 16)));
    std::vector<std::thread> th;
    for (int i = 0; i < n_threads; i++)
        th.emplace_back(fn, rows * i / n_threads, rows * (i + 1) / n_threads);
    for (auto &t : th) t.join();
}

int quantize_file(const char *in_path, const char *out_path, const char *type, int n_threads) {
    if (!in_path || !out_path || !type) return set_error(DFB_ERR_ARG, "null argument");
    std::string scheme(type);
    for (auto &ch : scheme) ch = (char)tolower(ch);
    if (target_type(scheme, TC_ATTN) < 0) return set_error(DFB_ERR_ARG, "unknown quantization type %s (q8_0, q4_k_m, q6_k, f16)", type);
    if (n_threads <= 0) n_threads = (int)std::thread::hardware_concurrency();
    GgufReader in;
    std::string err;
    if (!in.open(in_path, &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    uint32_t n_layers = 0;
    for (const char *pre : {"diffuse", "qwen2", "llama"}) {
        const GgufValue *v = in.find(std::string(pre) + ".block_count");
        if (v) { n_layers = (uint32_t)v->u; break; }
    }
    GgufWriter out;
    for (auto &kv : in.kv()) {
        const GgufValue &v = kv.second;
        if (kv.first == "general.alignment") continue;
        if (v.type == 8) out.add_str(kv.first, v.s);
        else if (v.type == 6 || v.type == 12) out.add_f32(kv.first, (float)v.f);
        else if (v.type == 9) continue;  // arrays (tokenizer tables) are not carried over
        else out.add_u32(kv.first, (uint32_t)v.u);
    }
    std::vector<int32_t> types;
    for (auto &t : in.tensors()) {
        const int32_t dst = resolve_type(t.type, target_type(scheme, classify(t.name, (int)n_layers)), t.ne[0]);
        types.push_back(dst);
        out.add_tensor_info(t.name, dst, t.n_dims, t.ne);
    }
    if (!out.begin(out_path, &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    for (size_t i = 0; i < in.tensors().size(); i++) {
        const GgufTensor &t = in.tensors()[i];
        const int64_t rows = t.ne[1] * t.ne[2] * t.ne[3];
        if (types[i] == t.type) {
            if (!out.write_tensor_data(t.data, t.nbytes, &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
            continue;
        }
        std::vector<uint8_t> buf((size_t)(ggml_row_size(types[i], t.ne[0]) * rows));
        parallel_rows(rows, n_threads, [&](int64_t r0, int64_t r1) { convert_rows(t.type, t.data, types[i], buf.data(), t.ne[0], r0, r1); });
        if (!out.write_tensor_data(buf.data(), buf.size(), &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    }
    if (!out.finish(&err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    return DFB_OK;
}

// ── random-init synthesizer ──
static inline uint64_t splitmix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
static uint64_t name_hash(const std::string &s, uint64_t seed) {
    uint64_t h = 1469598103934665603ull ^ seed;
    for (unsigned char ch : s) h = (h ^ ch) * 1099511628211ull;
    return splitmix(h);
}
// N(0, std) via Box-Muller on a counter-based stream: element i of a tensor depends
// only on (seed, tensor name, i), so rows can be generated in any order / thread.
// Elements 2j and 2j+1 share one (u1, u2) pair.
static void gauss_fill(float *out, int64_t i0, int64_t n, uint64_t key, float std_) {
    int64_t k = 0;
    while (k < n) {
        const int64_t i = i0 + k;
        const uint64_t r = splitmix(key ^ (uint64_t)(i >> 1) * 0xD1B54A32D192ED03ull);
        const float u1 = ((uint32_t)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
        const float u2 = (float)((uint32_t)r >> 8) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1)) * std_;
        float sn, cs;
        sincosf(6.2831853f * u2, &sn, &cs);
        if ((i & 1) == 0) {
            out[k++] = rad * cs;
            if (k < n) out[k++] = rad * sn;
        } else {
            out[k++] = rad * sn;
        }
    }
}

int synth_model(const char *path, const dfc_synth_spec *s) {
    if (!path || !s) return set_error(DFB_ERR_ARG, "null argument");
    if (s->n_layer <= 0 || s->n_embd <= 0 || s->n_head <= 0 || s->n_head_kv <= 0 || s->n_ff <= 0 || s->n_vocab <= 0 ||
        s->n_embd % s->n_head || s->n_head % s->n_head_kv)
        return set_error(DFB_ERR_ARG, "inconsistent synth dimensions");
    static const char *schemes[] = {"f32", "f16", "q8_0", "q4_k_m"};
    if (s->scheme < 0 || s->scheme > 3) return set_error(DFB_ERR_ARG, "bad scheme %d", s->scheme);
    const std::string scheme = schemes[s->scheme];
    const int nt = s->n_threads > 0 ? s->n_threads : (int)std::thread::hardware_concurrency();
    const int64_t d = s->n_embd, ff = s->n_ff, V = s->n_vocab, kvd = (int64_t)s->n_head_kv * (s->n_embd / s->n_head);
    struct T { std::string name; int64_t ne0, ne1; int kind; };  // kind 0 weight, 1 norm, 2 bias
    std::vector<T> ts;
    ts.push_back({"token_embd.weight", d, V, 0});
    ts.push_back({"output_norm.weight", d, 1, 1});
    if (!s->tied_output) ts.push_back({"output.weight", d, V, 0});
    for (int l = 0; l < s->n_layer; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        ts.push_back({p + "attn_norm.weight", d, 1, 1});
        ts.push_back({p + "attn_q.weight", d, d, 0});
        ts.push_back({p + "attn_k.weight", d, kvd, 0});
        ts.push_back({p + "attn_v.weight", d, kvd, 0});
        if (s->with_bias) {
            ts.push_back({p + "attn_q.bias", d, 1, 2});
            ts.push_back({p + "attn_k.bias", kvd, 1, 2});
            ts.push_back({p + "attn_v.bias", kvd, 1, 2});
        }
        ts.push_back({p + "attn_output.weight", d, d, 0});
        ts.push_back({p + "ffn_norm.weight", d, 1, 1});
        ts.push_back({p + "ffn_gate.weight", d, ff, 0});
        ts.push_back({p + "ffn_up.weight", d, ff, 0});
        ts.push_back({p + "ffn_down.weight", ff, d, 0});
    }
    GgufWriter w;
    w.add_str("general.architecture", "diffuse");
    w.add_str("general.name", s->is_dream ? "Dream-7B-random" : "LLaDA-8B-random");
    w.add_u32("diffuse.block_count", s->n_layer);
    w.add_u32("diffuse.attention.head_count", s->n_head);
    w.add_u32("diffuse.attention.head_count_kv", s->n_head_kv);
    w.add_u32("diffuse.embedding_length", s->n_embd);
    w.add_u32("diffuse.feed_forward_length", s->n_ff);
    w.add_u32("diffuse.context_length", s->n_ctx);
    w.add_u32("diffuse.vocab_size", s->n_vocab);
    w.add_f32("diffuse.rope.freq_base", s->rope_theta);
    w.add_f32("diffuse.attention.layer_norm_rms_epsilon", s->rms_norm_eps);
    w.add_u32("diffuse.mask_token_id", s->mask_token_id);
    w.add_str("diffuse.model_type", s->is_dream ? "dream" : "llada");
    std::vector<int32_t> types;
    // source tensors are what the converters emit: f32 (--type f32) or f16
    const int32_t src_type = s->scheme == 0 ? GT_F32 : GT_F16;
    for (auto &t : ts) {
        int32_t ty = src_type;
        if (s->scheme >= 2) ty = resolve_type(src_type, target_type(scheme, classify(t.name, s->n_layer)), t.ne0);
        else if (s->scheme == 1 && t.kind != 0) ty = GT_F16;
        types.push_back(ty);
        const int64_t ne[2] = {t.ne0, t.ne1};
        w.add_tensor_info(t.name, ty, t.ne1 > 1 ? 2 : 1, ne);
    }
    std::string err;
    if (!w.begin(path, &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    for (size_t i = 0; i < ts.size(); i++) {
        const T &t = ts[i];
        const int32_t ty = types[i];
        std::vector<uint8_t> buf((size_t)(ggml_row_size(ty, t.ne0) * t.ne1));
        const uint64_t key = name_hash(t.name, s->seed);
        parallel_rows(t.ne1, nt, [&](int64_t r0, int64_t r1) {
            std::vector<float> row(t.ne0);
            const int64_t rb = ggml_row_size(ty, t.ne0);
            for (int64_t r = r0; r < r1; r++) {
                if (t.kind == 1) std::fill(row.begin(), row.end(), 1.0f);
                else gauss_fill(row.data(), r * t.ne0, t.ne0, key, s->w_std);
                if (src_type == GT_F16)  // the converter's f16 rounding
                    for (auto &v : row) v = h2f(f2h(v));
                quantize_rows(ty, row.data(), t.ne0, buf.data() + r * rb);
            }
        });
        if (!w.write_tensor_data(buf.data(), buf.size(), &err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    }
    if (!w.finish(&err)) return set_error(DFB_ERR_ARG, "%s", err.c_str());
    return DFB_OK;
}

}  // namespace dfh

extern "C" int dfc_quantize_file(const char *in, const char *out, const char *type, int n_threads) {
    return dfh::quantize_file(in, out, type, n_threads);
}
extern "C" int dfc_synth_model(const char *path, const dfc_synth_spec *spec) { return dfh::synth_model(path, spec); }
extern "C" int dfc_quantize_rows(int32_t type, const float *src, int64_t n, void *dst) {
    return dfh::quantize_rows(type, src, n, (uint8_t *)dst) ? DFB_OK : dfh::set_error(DFB_ERR_ARG, "cannot quantize to type %d", type);
}
extern "C" int dfc_dequantize_rows(int32_t type, const void *src, int64_t n, float *dst) {
    return dfh::dequantize_rows(type, (const uint8_t *)src, n, dst) ? DFB_OK : dfh::set_error(DFB_ERR_ARG, "cannot dequantize type %d", type);
}
