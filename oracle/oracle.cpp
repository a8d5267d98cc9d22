// CPU oracle for the denoising hot path — TEST INFRASTRUCTURE ONLY (see oracle.h).
// Every function cites the reference lines it restates (paths relative to the
// diffuse-cpp checkout).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <random>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ───────────────────────── GGML scalar formats ─────────────────────────
enum : int32_t { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_BF16 = 30 };

float h2f(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) bits = s;
        else {  // subnormal: normalise
            e = 127 - 15 + 1;
            while (!(m & 0x400)) { m <<= 1; e--; }
            m &= 0x3ff;
            bits = s | (e << 23) | (m << 13);
        }
    } else if (e == 31) bits = s | 0x7f800000u | (m << 13);
    else bits = s | ((e + 127 - 15) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// round-to-nearest-even f32 -> f16 (GGML_FP32_TO_FP16 on IEEE hosts)
uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000;
    uint32_t ax = x & 0x7fffffff;
    if (ax >= 0x7f800000) return sign | 0x7c00 | (ax > 0x7f800000 ? 0x200 : 0);
    if (ax >= 0x477ff000) return sign | 0x7c00;  // rounds to inf
    if (ax < 0x38800000) {                        // subnormal half
        if (ax < 0x33000000) return sign;
        const uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
        const int shift = 126 - (int)e;           // 14..24
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1))) hm++;
        return sign | hm;
    }
    uint32_t hm = ((ax >> 13) & 0x3ff) | (((ax >> 23) - 112) << 10);
    const uint32_t rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (hm & 1))) hm++;
    return sign | hm;
}

float bf2f(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

int64_t blck_size(int32_t t) {
    switch (t) {
        case T_Q8_0: return 32;
        case T_Q4_K: case T_Q6_K: return 256;
        default: return 1;
    }
}
int64_t type_size(int32_t t) {
    switch (t) {
        case T_F32: return 4;
        case T_F16: case T_BF16: return 2;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        default: return 0;
    }
}

// 6-bit scale/min unpack of a Q4_K super-block (GGML get_scale_min_k4).
inline void q4k_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4);
    }
}

// Dequantize one row (n multiple of the block size).  Formats per GGML:
// Q4_K = {f16 d, f16 dmin, u8 scales[12], u8 qs[128]}; element 64j+l is the low
// nibble of qs[32j+l], element 64j+32+l its high nibble; value d*sc*q - dmin*m.
// Q6_K = {u8 ql[128], u8 qh[64], i8 scales[16], f16 d}.  Q8_0 = {f16 d, i8 qs[32]}.
void dequant_row(int32_t type, const uint8_t *src, int64_t n, float *dst) {
    switch (type) {
        case T_F32: memcpy(dst, src, n * 4); return;
        case T_F16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = h2f(h); } return;
        case T_BF16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = bf2f(h); } return;
        case T_Q8_0:
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t *blk = src + b * 34;
                uint16_t dh; memcpy(&dh, blk, 2);
                const float d = h2f(dh);
                for (int l = 0; l < 32; l++) dst[b * 32 + l] = d * (float)(int8_t)blk[2 + l];
            }
            return;
        case T_Q4_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + b * 144;
                uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
                const float d = h2f(dh), dmin = h2f(mh);
                const uint8_t *scales = blk + 4, *qs = blk + 16;
                float *y = dst + b * 256;
                for (int j = 0; j < 4; j++) {
                    uint8_t sc, mn;
                    q4k_scale_min(2 * j, scales, &sc, &mn);
                    const float d1 = d * sc, m1 = dmin * mn;
                    q4k_scale_min(2 * j + 1, scales, &sc, &mn);
                    const float d2 = d * sc, m2 = dmin * mn;
                    for (int l = 0; l < 32; l++) y[64 * j + l] = d1 * (qs[32 * j + l] & 0xF) - m1;
                    for (int l = 0; l < 32; l++) y[64 * j + 32 + l] = d2 * (qs[32 * j + l] >> 4) - m2;
                }
            }
            return;
        case T_Q6_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + b * 210;
                const uint8_t *ql = blk, *qh = blk + 128;
                const int8_t *sc = (const int8_t *)(blk + 192);
                uint16_t dh; memcpy(&dh, blk + 208, 2);
                const float d = h2f(dh);
                float *y = dst + b * 256;
                for (int h = 0; h < 2; h++) {
                    for (int l = 0; l < 32; l++) {
                        const int q1 = ((ql[64 * h + l] & 0xF) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32;
                        const int q2 = ((ql[64 * h + l + 32] & 0xF) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32;
                        const int q3 = ((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32;
                        const int q4 = ((ql[64 * h + l + 32] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32;
                        const int is = 8 * h + l / 16;
                        y[128 * h + l]      = d * sc[is + 0] * q1;
                        y[128 * h + l + 32] = d * sc[is + 2] * q2;
                        y[128 * h + l + 64] = d * sc[is + 4] * q3;
                        y[128 * h + l + 96] = d * sc[is + 6] * q4;
                    }
                }
            }
            return;
        default:
            fprintf(stderr, "[oracle] unsupported tensor type %d\n", type);
            abort();
    }
}

// ───────────────────────── GGUF reader ─────────────────────────
struct tensor_view {
    int32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int n_dims = 0;
    const uint8_t *data = nullptr;
    int64_t row_bytes() const { return ne[0] / blck_size(type) * type_size(type); }
};

struct kv_val {
    int32_t type = -1;
    uint64_t u = 0;
    double f = 0;
    std::string s;
};

struct gguf_file {
    void *map = MAP_FAILED;
    size_t size = 0;
    std::map<std::string, kv_val> kv;
    std::map<std::string, tensor_view> tensors;
    std::string arch;

    ~gguf_file() { if (map != MAP_FAILED) munmap(map, size); }

    bool open(const char *path) {
        int fd = ::open(path, O_RDONLY);
        if (fd < 0) return false;
        struct stat st;
        fstat(fd, &st);
        size = (size_t)st.st_size;
        map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (map == MAP_FAILED) return false;
        const uint8_t *p = (const uint8_t *)map, *end = p + size;
        auto rd = [&](void *dst, size_t n) -> bool {
            if (p + n > end) return false;
            memcpy(dst, p, n); p += n; return true;
        };
        auto rstr = [&](std::string &s) -> bool {
            uint64_t n; if (!rd(&n, 8) || p + n > end) return false;
            s.assign((const char *)p, n); p += n; return true;
        };
        uint32_t magic, version; uint64_t n_tensors, n_kv;
        if (!rd(&magic, 4) || magic != 0x46554747u) return false;  // "GGUF"
        if (!rd(&version, 4) || version < 2) return false;
        if (!rd(&n_tensors, 8) || !rd(&n_kv, 8)) return false;
        static const int scalar_size[] = {1, 1, 2, 2, 4, 4, 4, 1, -1, -1, 8, 8, 8};
        std::function<bool(int32_t, kv_val *)> rval;
        rval = [&](int32_t t, kv_val *v) -> bool {
            if (t == 8) { std::string s; if (!rstr(s)) return false; if (v) v->s = s; return true; }
            if (t == 9) {
                int32_t at; uint64_t n;
                if (!rd(&at, 4) || !rd(&n, 8)) return false;
                for (uint64_t i = 0; i < n; i++) if (!rval(at, nullptr)) return false;
                return true;
            }
            if (t < 0 || t > 12 || scalar_size[t] < 0) return false;
            uint8_t buf[8] = {0};
            if (!rd(buf, scalar_size[t])) return false;
            if (v) {
                switch (t) {
                    case 0: v->u = buf[0]; break;
                    case 1: v->u = (uint64_t)(int64_t)(int8_t)buf[0]; break;
                    case 2: { uint16_t x; memcpy(&x, buf, 2); v->u = x; } break;
                    case 3: { int16_t x; memcpy(&x, buf, 2); v->u = (uint64_t)(int64_t)x; } break;
                    case 4: { uint32_t x; memcpy(&x, buf, 4); v->u = x; } break;
                    case 5: { int32_t x; memcpy(&x, buf, 4); v->u = (uint64_t)(int64_t)x; } break;
                    case 6: { float x; memcpy(&x, buf, 4); v->f = x; } break;
                    case 7: v->u = buf[0]; break;
                    case 10: case 11: memcpy(&v->u, buf, 8); break;
                    case 12: memcpy(&v->f, buf, 8); break;
                }
            }
            return true;
        };
        for (uint64_t i = 0; i < n_kv; i++) {
            std::string key; int32_t t;
            if (!rstr(key) || !rd(&t, 4)) return false;
            kv_val v; v.type = t;
            if (!rval(t, &v)) return false;
            kv[key] = v;
        }
        struct tinfo { std::string name; tensor_view tv; uint64_t off; };
        std::vector<tinfo> infos(n_tensors);
        for (uint64_t i = 0; i < n_tensors; i++) {
            uint32_t nd;
            if (!rstr(infos[i].name) || !rd(&nd, 4) || nd > 4) return false;
            infos[i].tv.n_dims = (int)nd;
            for (uint32_t d = 0; d < nd; d++) if (!rd(&infos[i].tv.ne[d], 8)) return false;
            if (!rd(&infos[i].tv.type, 4) || !rd(&infos[i].off, 8)) return false;
        }
        uint64_t align = 32;
        auto it = kv.find("general.alignment");
        if (it != kv.end()) align = it->second.u;
        size_t data_off = (size_t)(p - (const uint8_t *)map);
        data_off = (data_off + align - 1) / align * align;
        for (auto &ti : infos) {
            // a type GGML's CPU path here does not decode, or data past the end of the file
            // (gguf_init_from_file fails on both, diffuse-model.cpp:92-95)
            if (blck_size(ti.tv.type) == 0 || type_size(ti.tv.type) == 0) {
                fprintf(stderr, "[oracle] tensor %s has unsupported type %d\n", ti.name.c_str(), ti.tv.type);
                return false;
            }
            uint64_t rows = 1;
            for (int d = 1; d < ti.tv.n_dims; d++) rows *= (uint64_t)ti.tv.ne[d];
            const uint64_t nbytes = (uint64_t)(ti.tv.ne[0] / blck_size(ti.tv.type) * type_size(ti.tv.type)) * rows;
            if (data_off + ti.off + nbytes > size) {
                fprintf(stderr, "[oracle] tensor %s data past the end of the file (truncated)\n", ti.name.c_str());
                return false;
            }
            ti.tv.data = (const uint8_t *)map + data_off + ti.off;
            tensors[ti.name] = ti.tv;
        }
        auto a = kv.find("general.architecture");
        if (a != kv.end()) arch = a->second.s;
        return true;
    }
};

// ───────────────────────── model ─────────────────────────
struct layer_w {
    const tensor_view *attn_norm, *wq, *wk, *wv, *wo, *ffn_norm, *gate, *up, *down;
    const tensor_view *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

struct hparams {
    int n_vocab, n_embd, n_head, n_head_kv, n_layer, n_ff, n_ctx_max, mask_id;
    float rope_theta, eps;
    int hd() const { return n_embd / n_head; }
};

}  // namespace

struct orc_model {
    gguf_file f;
    hparams hp;
    std::string model_type;
    const tensor_view *tok_embd, *output_norm, *output;
    std::vector<layer_w> layers;
};

namespace {

// Key lookup with the reference's prefix fallback (diffuse-model.cpp:27-57).
bool get_u32_multi(const gguf_file &f, const char *suffix, uint32_t *out) {
    static const char *prefixes[] = {"diffuse", "qwen2", "llama"};
    for (const char *pre : prefixes) {
        auto it = f.kv.find(std::string(pre) + "." + suffix);
        if (it != f.kv.end()) { *out = (uint32_t)it->second.u; return true; }
    }
    return false;
}
float get_f32_multi(const gguf_file &f, const char *suffix, float def) {
    static const char *prefixes[] = {"diffuse", "qwen2", "llama"};
    for (const char *pre : prefixes) {
        auto it = f.kv.find(std::string(pre) + "." + suffix);
        if (it != f.kv.end()) return (float)it->second.f;
    }
    return def;
}

const tensor_view *find_tensor(const orc_model &m, const std::string &name) {
    auto it = m.f.tensors.find(name);
    return it == m.f.tensors.end() ? nullptr : &it->second;
}

// Norm weights / biases may be F16 or F32; the reference casts them to f32
// (diffuse-graph.cpp:4-8, 53-56).
std::vector<float> vec_f32(const tensor_view *t) {
    std::vector<float> v(t->ne[0]);
    dequant_row(t->type, t->data, t->ne[0], v.data());
    return v;
}

int nthreads_or(int n) {
#ifdef _OPENMP
    return n > 0 ? n : omp_get_max_threads();
#else
    (void)n; return 1;
#endif
}

// ───────────────── GGML activation quantization (ORC_MODE_GGML) ─────────────────
inline int nearest_int(float fval) {
    float val = fval + 12582912.f;
    int i; memcpy(&i, &val, 4);
    return (i & 0x007fffff) - 0x00400000;
}

struct q8k_block { float d; int8_t qs[256]; int16_t bsums[16]; };

void quantize_q8k(const float *x, int64_t k, q8k_block *y) {
    for (int64_t b = 0; b < k / 256; b++) {
        const float *xb = x + b * 256;
        float max = 0, amax = 0;
        for (int j = 0; j < 256; j++) { float ax = fabsf(xb[j]); if (ax > amax) { amax = ax; max = xb[j]; } }
        if (amax == 0) { y[b].d = 0; memset(y[b].qs, 0, 256); memset(y[b].bsums, 0, 32); continue; }
        const float iscale = -128.f / max;
        for (int j = 0; j < 256; j++) { int v = nearest_int(iscale * xb[j]); y[b].qs[j] = (int8_t)std::min(127, v); }
        for (int j = 0; j < 16; j++) { int s = 0; for (int i = 0; i < 16; i++) s += y[b].qs[16 * j + i]; y[b].bsums[j] = (int16_t)s; }
        y[b].d = 1 / iscale;
    }
}

struct q80_block { float d; int8_t qs[32]; };
void quantize_q80(const float *x, int64_t k, q80_block *y) {
    for (int64_t b = 0; b < k / 32; b++) {
        float amax = 0;
        for (int j = 0; j < 32; j++) amax = std::max(amax, fabsf(x[b * 32 + j]));
        const float d = amax / 127.f, id = d ? 1.0f / d : 0.0f;
        y[b].d = h2f(f2h(d));
        for (int j = 0; j < 32; j++) y[b].qs[j] = (int8_t)roundf(x[b * 32 + j] * id);
    }
}

// Dot products of one weight row with one quantized activation row (GGML vec_dot semantics).
float dot_q4k_q8k(const uint8_t *w, const q8k_block *a, int64_t nb) {
    float sumf = 0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * 144;
        uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        int32_t isum = 0, msum = 0;
        for (int j = 0; j < 8; j++) {
            uint8_t sc, mn; q4k_scale_min(j, scales, &sc, &mn);
            const int half = j & 1, g = j >> 1;
            int32_t s = 0;
            for (int l = 0; l < 32; l++) {
                const int q = half ? (qs[32 * g + l] >> 4) : (qs[32 * g + l] & 0xF);
                s += q * a[b].qs[32 * j + l];
            }
            isum += sc * s;
            msum += mn * (a[b].bsums[2 * j] + a[b].bsums[2 * j + 1]);
        }
        sumf += h2f(dh) * a[b].d * isum - h2f(mh) * a[b].d * msum;
    }
    return sumf;
}

float dot_q6k_q8k(const uint8_t *w, const q8k_block *a, int64_t nb) {
    float sumf = 0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * 210;
        uint16_t dh; memcpy(&dh, blk + 208, 2);
        const int8_t *sc = (const int8_t *)(blk + 192);
        const uint8_t *ql = blk, *qh = blk + 128;
        int8_t qv[256];
        for (int h = 0; h < 2; h++)
            for (int l = 0; l < 32; l++) {
                qv[128 * h + l]      = (int8_t)(((ql[64 * h + l] & 0xF) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32);
                qv[128 * h + l + 32] = (int8_t)(((ql[64 * h + l + 32] & 0xF) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32);
                qv[128 * h + l + 64] = (int8_t)(((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32);
                qv[128 * h + l + 96] = (int8_t)(((ql[64 * h + l + 32] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32);
            }
        int32_t isum = 0;
        for (int g = 0; g < 16; g++) {
            int32_t s = 0;
            for (int l = 0; l < 16; l++) s += qv[16 * g + l] * a[b].qs[16 * g + l];
            isum += sc[g] * s;
        }
        sumf += h2f(dh) * a[b].d * isum;
    }
    return sumf;
}

float dot_q80_q80(const uint8_t *w, const q80_block *a, int64_t nb) {
    float sumf = 0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = w + b * 34;
        uint16_t dh; memcpy(&dh, blk, 2);
        int32_t s = 0;
        for (int l = 0; l < 32; l++) s += (int8_t)blk[2 + l] * a[b].qs[l];
        sumf += (float)s * (h2f(dh) * a[b].d);
    }
    return sumf;
}

inline float dot_f32(const float *a, const float *b, int64_t n) {
    float s = 0;
#pragma omp simd reduction(+ : s)
    for (int64_t i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

// y[M x N] = x[M x K] . W^T   (ggml_mul_mat(W, x) at diffuse-graph.cpp:61-63,122,136-140,154)
void matmul(const tensor_view *W, const float *x, int M, float *y, int mode, int nt) {
    const int64_t K = W->ne[0], N = W->ne[1];
    const int64_t rb = W->row_bytes();
    if (mode == ORC_MODE_GGML && (W->type == T_Q4_K || W->type == T_Q6_K)) {
        std::vector<q8k_block> q((size_t)M * (K / 256));
        for (int m = 0; m < M; m++) quantize_q8k(x + (size_t)m * K, K, q.data() + (size_t)m * (K / 256));
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int64_t n = 0; n < N; n++) {
            const uint8_t *w = W->data + n * rb;
            for (int m = 0; m < M; m++) {
                const q8k_block *a = q.data() + (size_t)m * (K / 256);
                y[(size_t)m * N + n] = W->type == T_Q4_K ? dot_q4k_q8k(w, a, K / 256) : dot_q6k_q8k(w, a, K / 256);
            }
        }
        return;
    }
    if (mode == ORC_MODE_GGML && W->type == T_Q8_0) {
        std::vector<q80_block> q((size_t)M * (K / 32));
        for (int m = 0; m < M; m++) quantize_q80(x + (size_t)m * K, K, q.data() + (size_t)m * (K / 32));
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int64_t n = 0; n < N; n++)
            for (int m = 0; m < M; m++)
                y[(size_t)m * N + n] = dot_q80_q80(W->data + n * rb, q.data() + (size_t)m * (K / 32), K / 32);
        return;
    }
    std::vector<float> xr;
    const float *xs = x;
    if (mode == ORC_MODE_GGML && (W->type == T_F16 || W->type == T_BF16)) {
        // F16 weights: GGML converts activations to f16 before the dot product
        xr.resize((size_t)M * K);
        for (size_t i = 0; i < xr.size(); i++) xr[i] = h2f(f2h(x[i]));
        xs = xr.data();
    }
#pragma omp parallel num_threads(nt)
    {
        std::vector<float> wrow(K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            dequant_row(W->type, W->data + n * rb, K, wrow.data());
            for (int m = 0; m < M; m++) y[(size_t)m * N + n] = dot_f32(wrow.data(), xs + (size_t)m * K, K);
        }
    }
}

// ggml_rms_norm (double accumulation of f32 squares) then ggml_mul by the weight
// (diffuse-graph.cpp:51-58).
void rmsnorm(const float *x, const float *w, float *y, int M, int K, float eps) {
    for (int m = 0; m < M; m++) {
        const float *xr = x + (size_t)m * K;
        double sum = 0.0;
        for (int i = 0; i < K; i++) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / K);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int i = 0; i < K; i++) y[(size_t)m * K + i] = (xr[i] * scale) * w[i];
    }
}

// GGML rope cache: theta = pos, multiplied by theta_scale = base^(-2/n_dims) once
// per rotated pair in float (ggml_rope_cache_init with freq_scale 1, ext_factor 0,
// attn_factor 1 as passed at diffuse-graph.cpp:76-79).
void rope_angles(int pos, int n_dims, float base, float *c, float *s) {
    const float theta_scale = powf(base, -2.0f / n_dims);
    float theta = (float)pos;
    for (int i = 0; i < n_dims / 2; i++) {
        c[i] = cosf(theta);
        s[i] = sinf(theta);
        theta *= theta_scale;
    }
}

// NEOX rotation of one head vector: pairs (i, i + n_dims/2).
void rope_neox(float *x, const float *c, const float *s, int n_dims) {
    const int h = n_dims / 2;
    for (int i = 0; i < h; i++) {
        const float x0 = x[i], x1 = x[i + h];
        x[i] = x0 * c[i] - x1 * s[i];
        x[i + h] = x0 * s[i] + x1 * c[i];
    }
}

// Inter-step cache (diffuse-cache.h:14-147).  K/V per layer [n_tokens][n_head_kv*hd]
// (the reference stores the GQA-expanded copy; the values are the same).
struct step_cache {
    bool initialized = false;
    int n_tokens = 0;
    std::vector<std::vector<float>> K, V;
    std::vector<int32_t> prev_seq;
    std::vector<int> last_changed_step;

    void init(int n_tok, int n_layer, int kv_dim) {   // cache.h:35-53
        n_tokens = n_tok;
        K.assign(n_layer, std::vector<float>((size_t)n_tok * kv_dim, 0.f));
        V.assign(n_layer, std::vector<float>((size_t)n_tok * kv_dim, 0.f));
        prev_seq.assign(n_tok, -1);
        last_changed_step.assign(n_tok, -1);
        initialized = false;
    }
    // cache.h:78-115
    void compute_active_set(const int32_t *seq, const std::vector<bool> &is_masked, int n_total,
                            int step, int extra, std::vector<int> &cached, std::vector<int> &active) {
        cached.clear(); active.clear();
        for (int i = 0; i < n_total; i++) {
            const bool changed = seq[i] != prev_seq[i];
            if (changed) last_changed_step[i] = step;
            const bool recent = extra > 0 && last_changed_step[i] >= 0 && (step - last_changed_step[i]) <= extra;
            if (changed || is_masked[i] || recent) active.push_back(i);
            else cached.push_back(i);
        }
    }
    void update_seq(const int32_t *seq, int n) {   // cache.h:142-145
        memcpy(prev_seq.data(), seq, n * sizeof(int32_t));
        initialized = true;
    }
};

// One forward over M query rows.  Full forward: active = all positions in order,
// cache may be null (diffuse-graph.cpp:11-160 / 165-306).  Cached forward: keys are
// [cached positions ‖ active positions] in that order, cached K/V read from the
// cache (diffuse-graph.cpp:395-593); fresh K/V of the active rows are written back
// afterwards (update_kv, cache.h:123-139 via graph.cpp:655-669).
void forward_rows(const orc_model &m, const int32_t *tokens, const int *pos, int M,
                  const std::vector<int> *cached_pos, step_cache *cache, float *logits,
                  int mode, int nt, int layer_limit = -1) {
    const hparams &hp = m.hp;
    const int d = hp.n_embd, H = hp.n_head, Hkv = hp.n_head_kv, hd = hp.hd(), ff = hp.n_ff;
    const int kvd = Hkv * hd, n_rep = H / Hkv;
    const int n_cached = cached_pos ? (int)cached_pos->size() : 0;
    const int N = n_cached + M;

    std::vector<float> x((size_t)M * d), h((size_t)M * d), q((size_t)M * d), k((size_t)M * kvd),
        v((size_t)M * kvd), att((size_t)M * d), o((size_t)M * d), g((size_t)M * ff), u((size_t)M * ff);
    // embedding rows (ggml_get_rows of F16/F32 token_embd, graph.cpp:43)
    for (int i = 0; i < M; i++)
        dequant_row(m.tok_embd->type, m.tok_embd->data + (int64_t)tokens[i] * m.tok_embd->row_bytes(), d,
                    x.data() + (size_t)i * d);
    std::vector<float> rc((size_t)M * (hd / 2)), rs((size_t)M * (hd / 2));
    for (int i = 0; i < M; i++) rope_angles(pos[i], hd, hp.rope_theta, &rc[(size_t)i * hd / 2], &rs[(size_t)i * hd / 2]);

    const float kq_scale = 1.0f / sqrtf((float)hd);
    std::vector<float> Kfull((size_t)N * kvd), Vfull((size_t)N * kvd);

    const int n_layers = layer_limit >= 0 ? std::min(layer_limit, hp.n_layer) : hp.n_layer;
    for (int il = 0; il < n_layers; il++) {
        const layer_w &L = m.layers[il];
        std::vector<float> wn = vec_f32(L.attn_norm);
        rmsnorm(x.data(), wn.data(), h.data(), M, d, hp.eps);
        matmul(L.wq, h.data(), M, q.data(), mode, nt);
        matmul(L.wk, h.data(), M, k.data(), mode, nt);
        matmul(L.wv, h.data(), M, v.data(), mode, nt);
        if (L.bq) { auto b = vec_f32(L.bq); for (int i = 0; i < M; i++) for (int j = 0; j < d; j++) q[(size_t)i * d + j] += b[j]; }
        if (L.bk) { auto b = vec_f32(L.bk); for (int i = 0; i < M; i++) for (int j = 0; j < kvd; j++) k[(size_t)i * kvd + j] += b[j]; }
        if (L.bv) { auto b = vec_f32(L.bv); for (int i = 0; i < M; i++) for (int j = 0; j < kvd; j++) v[(size_t)i * kvd + j] += b[j]; }
        for (int i = 0; i < M; i++) {
            for (int hh = 0; hh < H; hh++) rope_neox(&q[(size_t)i * d + hh * hd], &rc[(size_t)i * hd / 2], &rs[(size_t)i * hd / 2], hd);
            for (int hh = 0; hh < Hkv; hh++) rope_neox(&k[(size_t)i * kvd + hh * hd], &rc[(size_t)i * hd / 2], &rs[(size_t)i * hd / 2], hd);
        }
        // keys: [cached ‖ active]  (ggml_concat, graph.cpp:524-525)
        for (int c = 0; c < n_cached; c++) {
            const int p = (*cached_pos)[c];
            memcpy(&Kfull[(size_t)c * kvd], &cache->K[il][(size_t)p * kvd], kvd * 4);
            memcpy(&Vfull[(size_t)c * kvd], &cache->V[il][(size_t)p * kvd], kvd * 4);
        }
        memcpy(&Kfull[(size_t)n_cached * kvd], k.data(), (size_t)M * kvd * 4);
        memcpy(&Vfull[(size_t)n_cached * kvd], v.data(), (size_t)M * kvd * 4);
        // bidirectional attention, GQA grouped repeat (graph.cpp:84-119)
#pragma omp parallel num_threads(nt)
        {
            std::vector<float> sc(N);
#pragma omp for collapse(2) schedule(static)
            for (int hh = 0; hh < H; hh++)
                for (int i = 0; i < M; i++) {
                    const int kh = hh / n_rep;
                    const float *qi = &q[(size_t)i * d + hh * hd];
                    float mx = -INFINITY;
                    for (int j = 0; j < N; j++) {
                        sc[j] = dot_f32(&Kfull[(size_t)j * kvd + kh * hd], qi, hd) * kq_scale;
                        mx = std::max(mx, sc[j]);
                    }
                    double sum = 0.0;
                    for (int j = 0; j < N; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                    const float inv = (float)(1.0 / sum);
                    for (int j = 0; j < N; j++) sc[j] *= inv;
                    float *oi = &att[(size_t)i * d + hh * hd];
                    for (int e = 0; e < hd; e++) oi[e] = 0;
                    for (int j = 0; j < N; j++) {
                        const float *vj = &Vfull[(size_t)j * kvd + kh * hd];
                        for (int e = 0; e < hd; e++) oi[e] += sc[j] * vj[e];
                    }
                }
        }
        if (cache) {
            for (int i = 0; i < M; i++) {
                memcpy(&cache->K[il][(size_t)pos[i] * kvd], &k[(size_t)i * kvd], kvd * 4);
                memcpy(&cache->V[il][(size_t)pos[i] * kvd], &v[(size_t)i * kvd], kvd * 4);
            }
        }
        matmul(L.wo, att.data(), M, o.data(), mode, nt);
        for (size_t i = 0; i < x.size(); i++) x[i] = o[i] + x[i];
        // SwiGLU FFN (graph.cpp:126-142)
        wn = vec_f32(L.ffn_norm);
        rmsnorm(x.data(), wn.data(), h.data(), M, d, hp.eps);
        matmul(L.gate, h.data(), M, g.data(), mode, nt);
        matmul(L.up, h.data(), M, u.data(), mode, nt);
        for (size_t i = 0; i < g.size(); i++) { const float gv = g[i]; g[i] = (gv / (1.0f + expf(-gv))) * u[i]; }
        matmul(L.down, g.data(), M, o.data(), mode, nt);
        for (size_t i = 0; i < x.size(); i++) x[i] = o[i] + x[i];
    }
    std::vector<float> wn = vec_f32(m.output_norm);
    rmsnorm(x.data(), wn.data(), h.data(), M, d, hp.eps);
    matmul(m.output, h.data(), M, logits, mode, nt);
}

// ───────────────────────── sampler pieces ─────────────────────────
// diffuse-sampler.cpp:12-31
int tokens_to_unmask(int step, int total_steps, int total_masked, int schedule) {
    const float t0 = (float)step / total_steps;
    const float t1 = (float)(step + 1) / total_steps;
    float frac;
    if (schedule == 0) {
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

// diffuse-sampler.cpp:34-57 (serial f32 sums)
float compute_entropy(const float *logits, int n_vocab) {
    float max_val = logits[0];
    for (int v = 1; v < n_vocab; v++) if (logits[v] > max_val) max_val = logits[v];
    float sum_exp = 0.0f;
    for (int v = 0; v < n_vocab; v++) sum_exp += expf(logits[v] - max_val);
    const float log_sum = logf(sum_exp);
    float entropy = 0.0f;
    for (int v = 0; v < n_vocab; v++) {
        const float log_p = (logits[v] - max_val) - log_sum;
        const float p = expf(log_p);
        if (p > 1e-10f) entropy -= p * log_p;
    }
    return entropy;
}

struct candidate { int pos; int token; float confidence; float entropy; };

// candidate extraction + ordering + commit (diffuse-sampler.cpp:222-323).
int sampler_step(const float *logit_source, int n_vocab, int total_len, int32_t *seq,
                 std::vector<bool> &is_masked, int &n_masked, bool shift_logits, int step,
                 const orc_sampler_params &p, std::mt19937 &rng, int32_t *commit_pos,
                 int32_t *commit_tok, float *cand_entropy, float *cand_conf) {
    std::vector<candidate> candidates;
    candidates.reserve(n_masked);
    for (int i = 0; i < total_len; i++) {
        if (!is_masked[i]) continue;
        const int logit_pos = shift_logits ? std::max(i - 1, 0) : i;
        const float *row = logit_source + (size_t)logit_pos * n_vocab;
        const float ent = compute_entropy(row, n_vocab);
        if (p.temperature <= 0.0f) {
            int best = 0;
            float best_val = row[0], second_val = -1e30f;
            for (int v = 1; v < n_vocab; v++) {
                if (row[v] > best_val) { second_val = best_val; best_val = row[v]; best = v; }
                else if (row[v] > second_val) second_val = row[v];
            }
            const float conf = p.remasking == 4 ? (best_val - second_val) : best_val;
            candidates.push_back({i, best, conf, ent});
        } else {
            const float max_logit = *std::max_element(row, row + n_vocab);
            std::vector<float> probs(n_vocab);
            float sum = 0.0f;
            for (int v = 0; v < n_vocab; v++) { probs[v] = expf((row[v] - max_logit) / p.temperature); sum += probs[v]; }
            for (int v = 0; v < n_vocab; v++) probs[v] /= sum;
            std::discrete_distribution<int> dist(probs.begin(), probs.end());
            const int sampled = dist(rng);
            candidates.push_back({i, sampled, probs[sampled], ent});
        }
    }
    if (cand_entropy || cand_conf)
        for (size_t c = 0; c < candidates.size(); c++) {
            if (cand_entropy) cand_entropy[c] = candidates[c].entropy;
            if (cand_conf) cand_conf[c] = candidates[c].confidence;
        }
    int n_unmask = tokens_to_unmask(step, p.n_steps, n_masked, p.schedule);
    if (p.remasking == 2) {
        std::sort(candidates.begin(), candidates.end(),
                  [](const candidate &a, const candidate &b) { return a.entropy < b.entropy; });
        int n_easy = 0;
        for (const auto &c : candidates) { if (c.entropy < p.entropy_threshold) n_easy++; else break; }
        n_unmask = std::max(n_unmask, n_easy);
        n_unmask = std::min(n_unmask, (int)candidates.size());
    } else if (p.remasking == 0 || p.remasking == 3 || p.remasking == 4) {
        std::sort(candidates.begin(), candidates.end(),
                  [](const candidate &a, const candidate &b) { return a.confidence > b.confidence; });
    } else {
        std::shuffle(candidates.begin(), candidates.end(), rng);
    }
    int done = 0;
    for (int j = 0; j < n_unmask && j < (int)candidates.size(); j++) {
        const int pos = candidates[j].pos;
        seq[pos] = candidates[j].token;
        is_masked[pos] = false;
        n_masked--;
        if (commit_pos) commit_pos[done] = pos;
        if (commit_tok) commit_tok[done] = candidates[j].token;
        done++;
    }
    return done;
}

}  // namespace

// ───────────────────────── C API ─────────────────────────
extern "C" {

orc_model *orc_load(const char *path) {
    auto *m = new orc_model();
    if (!m->f.open(path)) { fprintf(stderr, "[oracle] cannot open GGUF %s\n", path); delete m; return nullptr; }
    hparams &hp = m->hp;
    uint32_t u;
    auto req = [&](const char *k, int *dst) -> bool {
        if (!get_u32_multi(m->f, k, &u)) { fprintf(stderr, "[oracle] missing key *.%s\n", k); return false; }
        *dst = (int)u; return true;
    };
    if (!req("block_count", &hp.n_layer) || !req("attention.head_count", &hp.n_head) ||
        !req("attention.head_count_kv", &hp.n_head_kv) || !req("embedding_length", &hp.n_embd) ||
        !req("feed_forward_length", &hp.n_ff)) { delete m; return nullptr; }
    hp.n_ctx_max = get_u32_multi(m->f, "context_length", &u) ? (int)u : 4096;
    hp.n_vocab = get_u32_multi(m->f, "vocab_size", &u) ? (int)u : 0;
    hp.mask_id = get_u32_multi(m->f, "mask_token_id", &u) ? (int)u : 0;
    hp.rope_theta = get_f32_multi(m->f, "rope.freq_base", 1000000.0f);
    hp.eps = get_f32_multi(m->f, "attention.layer_norm_rms_epsilon", 1e-6f);
    auto mt = m->f.kv.find("diffuse.model_type");
    if (mt != m->f.kv.end()) m->model_type = mt->second.s;
    else if (m->f.arch == "qwen2") m->model_type = "qwen2";
    else if (m->f.arch == "llama") m->model_type = "llama";
    else m->model_type = "llada";
    auto need = [&](const std::string &n) -> const tensor_view * {
        const tensor_view *t = find_tensor(*m, n);
        if (!t) fprintf(stderr, "[oracle] tensor not found: %s\n", n.c_str());
        return t;
    };
    m->tok_embd = need("token_embd.weight");
    m->output_norm = need("output_norm.weight");
    if (!m->tok_embd || !m->output_norm) { delete m; return nullptr; }
    if (hp.n_vocab == 0) hp.n_vocab = (int)m->tok_embd->ne[1];
    m->output = find_tensor(*m, "output.weight");
    if (!m->output) m->output = m->tok_embd;  // tied lm_head (model.cpp:157-158)
    m->layers.resize(hp.n_layer);
    char buf[128];
    for (int i = 0; i < hp.n_layer; i++) {
        layer_w &L = m->layers[i];
        const tensor_view **slots[] = {&L.attn_norm, &L.wq, &L.wk, &L.wv, &L.wo, &L.ffn_norm, &L.gate, &L.up, &L.down};
        const char *names[] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                               "ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};
        const int64_t d = hp.n_embd, kvd = (int64_t)hp.n_head_kv * (hp.n_embd / hp.n_head), ff = hp.n_ff;
        const int64_t shape[9][2] = {{d, 1}, {d, d}, {d, kvd}, {d, kvd}, {d, d}, {d, 1}, {d, ff}, {d, ff}, {ff, d}};
        for (int s = 0; s < 9; s++) {
            snprintf(buf, sizeof buf, "blk.%d.%s", i, names[s]);
            *slots[s] = need(buf);
            if (!*slots[s]) { delete m; return nullptr; }
            const int64_t n1 = (*slots[s])->n_dims > 1 ? (*slots[s])->ne[1] : 1;
            if ((*slots[s])->ne[0] != shape[s][0] || n1 != shape[s][1]) {
                fprintf(stderr, "[oracle] tensor %s has shape %lldx%lld, expected %lldx%lld\n", buf,
                        (long long)(*slots[s])->ne[0], (long long)n1, (long long)shape[s][0], (long long)shape[s][1]);
                delete m;
                return nullptr;
            }
        }
        snprintf(buf, sizeof buf, "blk.%d.attn_q.bias", i); L.bq = find_tensor(*m, buf);
        snprintf(buf, sizeof buf, "blk.%d.attn_k.bias", i); L.bk = find_tensor(*m, buf);
        snprintf(buf, sizeof buf, "blk.%d.attn_v.bias", i); L.bv = find_tensor(*m, buf);
    }
    return m;
}

void orc_free(orc_model *m) { delete m; }

int orc_hparams(const orc_model *m, int32_t *i9, float *f2) {
    const hparams &hp = m->hp;
    i9[0] = hp.n_vocab; i9[1] = hp.n_embd; i9[2] = hp.n_head; i9[3] = hp.n_head_kv; i9[4] = hp.n_layer;
    i9[5] = hp.n_ff; i9[6] = hp.n_ctx_max; i9[7] = hp.mask_id; i9[8] = m->model_type == "dream";
    f2[0] = hp.rope_theta; f2[1] = hp.eps;
    return 0;
}

int orc_tensor(const orc_model *m, const char *name, int32_t *type, int64_t *ne0, int64_t *ne1, const void **data) {
    const tensor_view *t = find_tensor(*m, name);
    if (!t) return -1;
    *type = t->type; *ne0 = t->ne[0]; *ne1 = t->ne[1]; *data = t->data;
    return 0;
}

int orc_dequantize(int32_t type, const void *src, int64_t n, float *dst) {
    if (type_size(type) == 0 || n % blck_size(type)) return -1;
    dequant_row(type, (const uint8_t *)src, n, dst);
    return 0;
}

int orc_matmul(const orc_model *m, const char *name, const float *x, int32_t M, float *y, int32_t mode, int32_t nt) {
    const tensor_view *t = find_tensor(*m, name);
    if (!t) return -1;
    matmul(t, x, M, y, mode, nthreads_or(nt));
    return 0;
}

int orc_forward(const orc_model *m, const int32_t *tokens, int32_t n, float *logits, int32_t mode, int32_t nt) {
    std::vector<int> pos(n);
    for (int i = 0; i < n; i++) pos[i] = i;
    forward_rows(*m, tokens, pos.data(), n, nullptr, nullptr, logits, mode, nthreads_or(nt));
    return 0;
}

int orc_forward_layers(const orc_model *m, const int32_t *tokens, int32_t n, float *logits, int32_t mode,
                       int32_t nt, int32_t n_layers) {
    std::vector<int> pos(n);
    for (int i = 0; i < n; i++) pos[i] = i;
    forward_rows(*m, tokens, pos.data(), n, nullptr, nullptr, logits, mode, nthreads_or(nt), n_layers);
    return 0;
}

// The state of one diffuse_sample run (diffuse-sampler.cpp:60-130): sequence, masks,
// the persistent logits buffer, the inter-step cache and the shared mt19937.
struct orc_session {
    const orc_model *m = nullptr;
    orc_sampler_params p{};
    int mode = 0, nt = 1;
    int n_prompt = 0, n_gen = 0, total_len = 0, n_masked = 0, last_n_active = 0;
    bool shift_logits = false;
    std::vector<int32_t> seq;
    std::vector<bool> is_masked;
    std::vector<float> logits_full;
    step_cache cache;
    std::vector<int> all_pos;
    std::mt19937 rng;
};

orc_session *orc_sess_new(const orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                          const orc_sampler_params *pp, int32_t mode, int32_t nt) {
    auto *s = new orc_session();
    s->m = m;
    s->p = *pp;
    s->mode = mode;
    s->nt = nthreads_or(nt);
    s->n_prompt = n_prompt;
    s->n_gen = n_gen;
    s->shift_logits = m->model_type == "dream";  // sampler.cpp:74
    s->seq.assign(prompt, prompt + n_prompt);     // sampler.cpp:77-87
    s->seq.resize(n_prompt + n_gen, m->hp.mask_id);
    s->total_len = n_prompt + n_gen;
    s->is_masked.assign(s->total_len, false);
    for (int i = n_prompt; i < s->total_len; i++) s->is_masked[i] = true;
    s->n_masked = n_gen;
    s->logits_full.assign((size_t)s->total_len * m->hp.n_vocab, 0.f);  // sampler.cpp:90
    s->rng.seed(pp->seed);
    if (pp->use_cache) s->cache.init(s->total_len, m->hp.n_layer, m->hp.n_head_kv * m->hp.hd());  // sampler.cpp:100
    s->all_pos.resize(s->total_len);
    for (int i = 0; i < s->total_len; i++) s->all_pos[i] = i;
    return s;
}

void orc_sess_free(orc_session *s) { delete s; }

// The forward of one step (diffuse-sampler.cpp:143-213): full or cached, the cache's
// sequence snapshot taken after it (update_seq), logits_full refreshed at the active rows.
// Returns the rows computed.
int orc_sess_forward(orc_session *s, int32_t step) {
    const orc_model &m = *s->m;
    const orc_sampler_params &p = s->p;
    const int total_len = s->total_len, n_vocab = m.hp.n_vocab;
    const bool use_cache = p.use_cache != 0;
    int n_active = total_len;
    const bool force_full = !use_cache || !s->cache.initialized ||
                            (p.cache_refresh > 0 && step > 0 && (step % p.cache_refresh == 0));
    if (force_full) {
        forward_rows(m, s->seq.data(), s->all_pos.data(), total_len, nullptr, use_cache ? &s->cache : nullptr,
                     s->logits_full.data(), s->mode, s->nt);
        if (use_cache) s->cache.update_seq(s->seq.data(), total_len);
    } else {
        std::vector<int> cached, active;
        s->cache.compute_active_set(s->seq.data(), s->is_masked, total_len, step, p.cache_keep_active, cached, active);
        n_active = (int)active.size();
        if (n_active >= total_len || n_active == 0) {
            forward_rows(m, s->seq.data(), s->all_pos.data(), total_len, nullptr, &s->cache, s->logits_full.data(),
                         s->mode, s->nt);
            s->cache.update_seq(s->seq.data(), total_len);
            n_active = total_len;
        } else {
            std::vector<int32_t> toks(n_active);
            for (int a = 0; a < n_active; a++) toks[a] = s->seq[active[a]];
            std::vector<float> la((size_t)n_active * n_vocab);
            forward_rows(m, toks.data(), active.data(), n_active, &cached, &s->cache, la.data(), s->mode, s->nt);
            s->cache.update_seq(s->seq.data(), total_len);
            for (int a = 0; a < n_active; a++)
                memcpy(&s->logits_full[(size_t)active[a] * n_vocab], &la[(size_t)a * n_vocab], n_vocab * 4);
        }
    }
    s->last_n_active = n_active;
    return n_active;
}

// The sampler decision of one step on the session's own logits (sampler.cpp:222-323).
int orc_sess_sample(orc_session *s, int32_t step, int32_t *commit_pos, int32_t *commit_tok) {
    return sampler_step(s->logits_full.data(), s->m->hp.n_vocab, s->total_len, s->seq.data(), s->is_masked,
                        s->n_masked, s->shift_logits, step, s->p, s->rng, commit_pos, commit_tok, nullptr, nullptr);
}

// Teacher forcing: apply commits decided elsewhere (sampler.cpp:316-323 with given picks).
int orc_sess_commit(orc_session *s, const int32_t *pos, const int32_t *tok, int32_t n) {
    for (int i = 0; i < n; i++) {
        if (pos[i] < 0 || pos[i] >= s->total_len || !s->is_masked[pos[i]]) return -1;
        s->seq[pos[i]] = tok[i];
        s->is_masked[pos[i]] = false;
        s->n_masked--;
    }
    return 0;
}

int orc_sess_logits(const orc_session *s, int32_t row0, int32_t nrows, float *out) {
    if (row0 < 0 || nrows < 0 || row0 + nrows > s->total_len) return -1;
    const size_t V = s->m->hp.n_vocab;
    memcpy(out, s->logits_full.data() + (size_t)row0 * V, (size_t)nrows * V * 4);
    return 0;
}

int orc_sess_tokens(const orc_session *s, int32_t *seq_out) {
    memcpy(seq_out, s->seq.data(), s->total_len * sizeof(int32_t));
    return s->n_masked;
}

// diffuse-sampler.cpp:256-269 with the draw's uniform given (the distribution's own draw
// is std::generate_canonical<double, 53> on the loop's rng, orc_canonical).
int32_t orc_sample_row(const float *row, int32_t n_vocab, float temperature, double u, float *conf, double *margin) {
    const float max_logit = *std::max_element(row, row + n_vocab);
    std::vector<float> probs(n_vocab);
    float sum = 0.0f;
    for (int v = 0; v < n_vocab; v++) {
        probs[v] = expf((row[v] - max_logit) / temperature);
        sum += probs[v];
    }
    for (int v = 0; v < n_vocab; v++) probs[v] /= sum;
    std::discrete_distribution<int>::param_type prm(probs.begin(), probs.end());
    const std::vector<double> w = prm.probabilities();  // normalised by their double sum
    std::vector<double> cp(w.size());
    std::partial_sum(w.begin(), w.end(), cp.begin());
    cp.back() = 1.0;
    const int k = (int)(std::lower_bound(cp.begin(), cp.end(), u) - cp.begin());
    if (conf) *conf = probs[k];
    if (margin) *margin = std::min(cp[k] - u, k ? u - cp[k - 1] : u);
    return k;
}

int orc_canonical(uint32_t seed, int32_t n, double *out) {
    std::mt19937 rng(seed);
    for (int i = 0; i < n; i++) out[i] = std::generate_canonical<double, std::numeric_limits<double>::digits>(rng);
    return 0;
}

// diffuse_sample, diffuse-sampler.cpp:60-370: forward + sampler per step until no mask is left.
int orc_generate(const orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                 const orc_sampler_params *pp, int32_t *out_tokens, orc_trace *trace, int32_t mode, int32_t nt_) {
    orc_session *s = orc_sess_new(m, prompt, n_prompt, n_gen, pp, mode, nt_);
    int steps_run = 0;
    for (int step = 0; step < pp->n_steps && s->n_masked > 0; step++) {
        const int n_active = orc_sess_forward(s, step);
        int32_t *cp = nullptr, *ct = nullptr;
        if (trace && step < trace->max_steps) {
            trace->n_active[step] = n_active;
            cp = trace->commit_pos + (size_t)step * trace->n_gen;
            ct = trace->commit_tok + (size_t)step * trace->n_gen;
        }
        const int done = orc_sess_sample(s, step, cp, ct);
        if (trace && step < trace->max_steps) trace->n_unmask[step] = done;
        steps_run++;
    }
    if (trace) {
        trace->steps_run = steps_run;
        if (trace->final_logits) memcpy(trace->final_logits, s->logits_full.data(), s->logits_full.size() * 4);
    }
    for (int i = 0; i < n_gen; i++) out_tokens[i] = s->seq[n_prompt + i];
    orc_sess_free(s);
    return steps_run;
}

int orc_sampler_step(const float *logits_full, int32_t n_vocab, int32_t total_len, int32_t *seq,
                     uint8_t *is_masked_u8, int32_t is_dream, int32_t step, const orc_sampler_params *p,
                     int32_t *commit_pos, int32_t *commit_tok, float *cand_entropy, float *cand_conf) {
    std::vector<bool> is_masked(total_len);
    int n_masked = 0;
    for (int i = 0; i < total_len; i++) { is_masked[i] = is_masked_u8[i] != 0; n_masked += is_masked[i]; }
    std::mt19937 rng(p->seed);
    const int done = sampler_step(logits_full, n_vocab, total_len, seq, is_masked, n_masked, is_dream != 0, step,
                                  *p, rng, commit_pos, commit_tok, cand_entropy, cand_conf);
    for (int i = 0; i < total_len; i++) is_masked_u8[i] = is_masked[i] ? 1 : 0;
    return done;
}

int orc_tokens_to_unmask(int32_t step, int32_t total_steps, int32_t total_masked, int32_t schedule) {
    return tokens_to_unmask(step, total_steps, total_masked, schedule);
}

float orc_entropy(const float *row, int32_t n_vocab) { return compute_entropy(row, n_vocab); }

int orc_rope_table(int32_t n_pos, int32_t n_dims, float base, float *c, float *s) {
    for (int p = 0; p < n_pos; p++) rope_angles(p, n_dims, base, c + (size_t)p * n_dims / 2, s + (size_t)p * n_dims / 2);
    return 0;
}

}  // extern "C"

// ───────────────────────── model synthesizer (CPU only) ─────────────────────────
// Writes the same seeded random-init GGUF as the product's synthesizer, from this
// file's own code, so that a CPU-only process (the benchmark's reference arm) can
// create its model without the product libraries; tests/test_host_cpu.py asserts the two
// files are byte-identical.  Quantization restates the reference's quantize tool
// (tools/quantize.cpp:31-98 type policy; blocks by GGML's reference quantizers, which
// ggml_quantize_chunk at tools/quantize.cpp:291 calls): Q8_0 amax / 127 rounding; Q4_K
// weighted least-squares (scale, min) search per 32-element sub-block over 21 grids then
// 6-bit codes; Q6_K x^2-weighted scale search per 16-element group over 19 grids then
// 8-bit signed codes.  Sums are sequential float sums without FMA contraction (this
// section is compiled with fp-contract off, like the product's quantizer).
#pragma GCC push_options
#pragma GCC optimize("fp-contract=off")
namespace {

inline int rne_i(float v) { return (int)lrintf(v); }

void q80_block(const float *x, uint8_t *out) {
    float amax = 0.f;
    for (int j = 0; j < 32; j++) amax = std::max(amax, fabsf(x[j]));
    const float d = amax / 127.f, id = d != 0.f ? 1.0f / d : 0.0f;
    const uint16_t dh = f2h(d);
    memcpy(out, &dh, 2);
    for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

// x ~ s * q + m over q in [0, nmax], m <= 0, weights w: returns s, *neg_m = -m.
float fit_affine(int n, int nmax, const float *x, const float *w, uint8_t *q, float *neg_m) {
    float lo = x[0], hi = x[0], sum_w = w[0], sum_wx = w[0] * x[0];
    for (int i = 1; i < n; i++) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
        sum_w += w[i];
        sum_wx += w[i] * x[i];
    }
    if (lo > 0) lo = 0;
    if (hi == lo) {
        for (int i = 0; i < n; i++) q[i] = 0;
        *neg_m = -lo;
        return 0.f;
    }
    float is = nmax / (hi - lo), s = 1 / is, m = lo, err_best = 0;
    for (int i = 0; i < n; i++) {
        int v = rne_i(is * (x[i] - lo));
        q[i] = (uint8_t)(v < 0 ? 0 : v > nmax ? nmax : v);
        const float e = s * q[i] + m - x[i];
        err_best += w[i] * (e * e);
    }
    uint8_t cand[32];
    for (int step = 0; step <= 20; step++) {
        is = (-1.f + 0.1f * step + nmax) / (hi - lo);
        float a = 0, b = 0, c = 0;  // sum w l, sum w l^2, sum w l x
        for (int i = 0; i < n; i++) {
            int v = rne_i(is * (x[i] - lo));
            v = v < 0 ? 0 : v > nmax ? nmax : v;
            cand[i] = (uint8_t)v;
            a += w[i] * v;
            b += w[i] * v * v;
            c += w[i] * v * x[i];
        }
        const float det = sum_w * b - a * a;
        if (!(det > 0)) continue;
        float s1 = (sum_w * c - sum_wx * a) / det, m1 = (b * sum_wx - a * c) / det;
        if (m1 > 0) {
            m1 = 0;
            s1 = c / b;
        }
        float err = 0;
        for (int i = 0; i < n; i++) {
            const float e = s1 * cand[i] + m1 - x[i];
            err += w[i] * (e * e);
        }
        if (err < err_best) {
            for (int i = 0; i < n; i++) q[i] = cand[i];
            err_best = err;
            s = s1;
            m = m1;
        }
    }
    *neg_m = -m;
    return s;
}

void q4k_block(const float *x, uint8_t *out) {
    uint8_t q[256];
    float w[32], s[8], mneg[8], smax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; j++) {
        float ss = 0;
        for (int l = 0; l < 32; l++) ss += x[32 * j + l] * x[32 * j + l];
        const float r = sqrtf(ss / 32);
        for (int l = 0; l < 32; l++) w[l] = r + fabsf(x[32 * j + l]);
        s[j] = fit_affine(32, 15, x + 32 * j, w, q + 32 * j, &mneg[j]);
        if (s[j] > smax) smax = s[j];
        if (mneg[j] > mmax) mmax = mneg[j];
    }
    const float is = smax > 0 ? 63.f / smax : 0.f, im = mmax > 0 ? 63.f / mmax : 0.f;
    int cs[8], cm[8];
    for (int j = 0; j < 8; j++) {
        cs[j] = std::min(63, rne_i(is * s[j]));
        cm[j] = std::min(63, rne_i(im * mneg[j]));
    }
    uint8_t *sc = out + 4;
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            sc[j] = (uint8_t)cs[j];
            sc[j + 4] = (uint8_t)cm[j];
        } else {
            sc[j + 4] = (uint8_t)((cs[j] & 0xF) | ((cm[j] & 0xF) << 4));
            sc[j - 4] |= (uint8_t)((cs[j] >> 4) << 6);
            sc[j] |= (uint8_t)((cm[j] >> 4) << 6);
        }
    }
    const uint16_t dh = f2h(smax / 63.f), mh = f2h(mmax / 63.f);
    memcpy(out, &dh, 2);
    memcpy(out + 2, &mh, 2);
    for (int j = 0; j < 8; j++) {
        uint8_t a, b;
        q4k_scale_min(j, sc, &a, &b);
        const float d = h2f(dh) * a;
        if (d == 0.f) continue;
        const float dm = h2f(mh) * b;
        for (int l = 0; l < 32; l++) {
            const int v = rne_i((x[32 * j + l] + dm) / d);
            q[32 * j + l] = (uint8_t)(v < 0 ? 0 : v > 15 ? 15 : v);
        }
    }
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) out[16 + 32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

// x ~ s * l over l in [-nmax, nmax - 1], weights x^2; codes l + nmax into q.
float fit_scale(int n, int nmax, const float *x, uint8_t *q) {
    float amax = 0, vmax = 0;
    for (int i = 0; i < n; i++)
        if (fabsf(x[i]) > amax) {
            amax = fabsf(x[i]);
            vmax = x[i];
        }
    if (amax < 1e-15f) {
        for (int i = 0; i < n; i++) q[i] = 0;
        return 0.f;
    }
    auto code = [&](float is, int i) {
        int v = rne_i(is * x[i]);
        return v < -nmax ? -nmax : v > nmax - 1 ? nmax - 1 : v;
    };
    float is = -nmax / vmax, a = 0, b = 0;  // sum w x l, sum w l^2
    for (int i = 0; i < n; i++) {
        const int l = code(is, i);
        q[i] = (uint8_t)(l + nmax);
        a += x[i] * x[i] * x[i] * l;
        b += x[i] * x[i] * l * l;
    }
    float s = b ? a / b : 0.0f, best = s * a;
    for (int k = -9; k <= 9; k++) {
        if (!k) continue;
        is = -(nmax + 0.1f * k) / vmax;
        a = b = 0;
        for (int i = 0; i < n; i++) {
            const int l = code(is, i);
            a += x[i] * x[i] * x[i] * l;
            b += x[i] * x[i] * l * l;
        }
        if (b > 0 && a * a > best * b) {
            for (int i = 0; i < n; i++) q[i] = (uint8_t)(code(is, i) + nmax);
            s = a / b;
            best = s * a;
        }
    }
    return s;
}

void q6k_block(const float *x, uint8_t *out) {
    uint8_t q[256];
    float s[16], smax = 0.f, amax = 0.f;
    for (int g = 0; g < 16; g++) {
        s[g] = fit_scale(16, 32, x + 16 * g, q + 16 * g);
        if (fabsf(s[g]) > amax) {
            amax = fabsf(s[g]);
            smax = s[g];
        }
    }
    memset(out, 0, 210);
    if (amax < 1e-15f) return;
    const float is = -128.f / smax;
    const uint16_t dh = f2h(1 / is);
    memcpy(out + 208, &dh, 2);
    int8_t *sc = reinterpret_cast<int8_t *>(out + 192);
    for (int g = 0; g < 16; g++) sc[g] = (int8_t)std::min(127, rne_i(is * s[g]));
    for (int g = 0; g < 16; g++) {
        const float d = h2f(dh) * sc[g];
        if (d == 0.f) continue;
        for (int l = 0; l < 16; l++) {
            const int v = rne_i(x[16 * g + l] / d);
            q[16 * g + l] = (uint8_t)((v < -32 ? -32 : v > 31 ? 31 : v) + 32);
        }
    }
    for (int h = 0; h < 2; h++) {
        const uint8_t *t = q + 128 * h;
        uint8_t *ql = out + 64 * h, *qh = out + 128 + 32 * h;
        for (int l = 0; l < 32; l++) {
            ql[l] = (uint8_t)((t[l] & 0xF) | ((t[l + 64] & 0xF) << 4));
            ql[l + 32] = (uint8_t)((t[l + 32] & 0xF) | ((t[l + 96] & 0xF) << 4));
            qh[l] = (uint8_t)((t[l] >> 4) | ((t[l + 32] >> 4) << 2) | ((t[l + 64] >> 4) << 4) | ((t[l + 96] >> 4) << 6));
        }
    }
}

// Counter-based N(0, std): element i of a tensor depends only on (seed, tensor name, i);
// elements 2k and 2k + 1 are the cosine and sine halves of one Box-Muller pair.
uint64_t mix64(uint64_t v) {
    v += 0x9E3779B97F4A7C15ull;
    v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
    v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
    return v ^ (v >> 31);
}
uint64_t tensor_key(const std::string &name, uint64_t seed) {
    uint64_t h = 1469598103934665603ull ^ seed;
    for (unsigned char ch : name) h = (h ^ ch) * 1099511628211ull;
    return mix64(h);
}
void normal_row(float *out, int64_t i0, int64_t n, uint64_t key, float sd) {
    for (int64_t k = 0; k < n;) {
        const int64_t i = i0 + k;
        const uint64_t r = mix64(key ^ (uint64_t)(i >> 1) * 0xD1B54A32D192ED03ull);
        const float u1 = ((uint32_t)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
        const float u2 = (float)((uint32_t)r >> 8) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1)) * sd;
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

// The quantize tool's type for a tensor under a scheme (tools/quantize.cpp:31-98):
// norms and biases f32, token_embd f16, Q4_K_M: output.weight and the FFN of the first
// and last layer Q6_K, the rest Q4_K; Q8_0: every linear Q8_0.
int32_t policy_type(const std::string &name, int scheme, int n_layer, int64_t ne0) {
    auto has = [&](const char *s) { return name.find(s) != std::string::npos; };
    if (scheme == 0) return T_F32;
    const bool norm = has("_norm") || has("norm.") || has(".bias");
    if (scheme == 1) return norm ? T_F32 : T_F16;
    if (norm) return T_F32;
    if (has("token_embd")) return T_F16;
    int32_t t;
    if (scheme == 2) t = T_Q8_0;
    else {
        int layer = -1;
        const size_t p = name.find("blk.");
        if (p != std::string::npos) layer = atoi(name.c_str() + p + 4);
        // attention weights first (attn_output.weight also contains "output.weight")
        const bool attn = has("attn_q") || has("attn_k") || has("attn_v") || has("attn_output");
        const bool ffn = has("ffn_gate") || has("ffn_up") || has("ffn_down");
        if (attn) t = T_Q4_K;
        else if (ffn) t = (layer == 0 || layer == n_layer - 1) ? T_Q6_K : T_Q4_K;
        else t = (has("output.weight") || has("lm_head")) ? T_Q6_K : T_Q4_K;
    }
    return ne0 % blck_size(t) ? T_F16 : t;  // rows that are not whole blocks keep the source type
}

// Minimal GGUF v3 writer: metadata and tensor infos, then 32-byte-aligned data.
struct gguf_out {
    std::vector<uint8_t> head;
    int n_kv = 0;
    struct ti { std::string name; int32_t type; int64_t ne0, ne1; uint64_t off, nbytes; };
    std::vector<ti> infos;
    uint64_t data_size = 0;
    void put(const void *p, size_t n) { head.insert(head.end(), (const uint8_t *)p, (const uint8_t *)p + n); }
    void put_str(const std::string &s) { const uint64_t n = s.size(); put(&n, 8); put(s.data(), n); }
    void kv_u32(const std::string &k, uint32_t v) { put_str(k); int32_t t = 4; put(&t, 4); put(&v, 4); n_kv++; }
    void kv_f32(const std::string &k, float v) { put_str(k); int32_t t = 6; put(&t, 4); put(&v, 4); n_kv++; }
    void kv_str(const std::string &k, const std::string &v) { put_str(k); int32_t t = 8; put(&t, 4); put_str(v); n_kv++; }
    void tensor(const std::string &name, int32_t type, int64_t ne0, int64_t ne1) {
        const uint64_t nb = (uint64_t)(ne0 / blck_size(type) * type_size(type)) * (uint64_t)ne1;
        infos.push_back({name, type, ne0, ne1, data_size, nb});
        data_size += (nb + 31) / 32 * 32;
    }
    std::vector<uint8_t> header() const {
        std::vector<uint8_t> h;
        auto p = [&](const void *d, size_t n) { h.insert(h.end(), (const uint8_t *)d, (const uint8_t *)d + n); };
        const uint32_t magic = 0x46554747u, version = 3;
        const uint64_t nt = infos.size(), nk = (uint64_t)n_kv;
        p(&magic, 4); p(&version, 4); p(&nt, 8); p(&nk, 8);
        h.insert(h.end(), head.begin(), head.end());
        for (const auto &t : infos) {
            const uint64_t n = t.name.size();
            p(&n, 8); p(t.name.data(), n);
            const uint32_t nd = t.ne1 > 1 ? 2 : 1;
            p(&nd, 4);
            p(&t.ne0, 8);
            if (nd == 2) p(&t.ne1, 8);
            p(&t.type, 4);
            p(&t.off, 8);
        }
        h.resize((h.size() + 31) / 32 * 32, 0);
        return h;
    }
};

}  // namespace

extern "C" int orc_synth_model(const char *path, const orc_synth_spec *s) {
    if (!path || !s || s->n_layer <= 0 || s->n_embd <= 0 || s->n_head <= 0 || s->n_head_kv <= 0 ||
        s->n_embd % s->n_head || s->n_head % s->n_head_kv || s->scheme < 0 || s->scheme > 3)
        return -1;
    const int64_t d = s->n_embd, ff = s->n_ff, V = s->n_vocab, kvd = (int64_t)s->n_head_kv * (s->n_embd / s->n_head);
    struct T { std::string name; int64_t ne0, ne1; int kind; };  // kind 0 weight, 1 norm (ones), 2 bias
    std::vector<T> ts = {{"token_embd.weight", d, V, 0}, {"output_norm.weight", d, 1, 1}};
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
    // converter metadata (tools/convert-llada.py:185-202, convert-dream.py:180-195)
    gguf_out g;
    g.kv_str("general.architecture", "diffuse");
    g.kv_str("general.name", s->is_dream ? "Dream-7B-random" : "LLaDA-8B-random");
    g.kv_u32("diffuse.block_count", s->n_layer);
    g.kv_u32("diffuse.attention.head_count", s->n_head);
    g.kv_u32("diffuse.attention.head_count_kv", s->n_head_kv);
    g.kv_u32("diffuse.embedding_length", s->n_embd);
    g.kv_u32("diffuse.feed_forward_length", s->n_ff);
    g.kv_u32("diffuse.context_length", s->n_ctx);
    g.kv_u32("diffuse.vocab_size", s->n_vocab);
    g.kv_f32("diffuse.rope.freq_base", s->rope_theta);
    g.kv_f32("diffuse.attention.layer_norm_rms_epsilon", s->rms_norm_eps);
    g.kv_u32("diffuse.mask_token_id", s->mask_token_id);
    g.kv_str("diffuse.model_type", s->is_dream ? "dream" : "llada");
    std::vector<int32_t> types;
    for (const auto &t : ts) {
        int32_t ty = policy_type(t.name, s->scheme, s->n_layer, t.ne0);
        if (s->scheme == 1 && t.kind != 0) ty = T_F16;  // the converter's --type f16 keeps norms f16
        types.push_back(ty);
        g.tensor(t.name, ty, t.ne0, t.ne1);
    }
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    const std::vector<uint8_t> h = g.header();
    fwrite(h.data(), 1, h.size(), f);
    const int nt = s->n_threads > 0 ? s->n_threads : omp_get_max_threads();
    const bool src_f16 = s->scheme != 0;  // the converter writes f16 sources for every quantized scheme
    for (size_t i = 0; i < ts.size(); i++) {
        const T &t = ts[i];
        const int32_t ty = types[i];
        const int64_t rb = t.ne0 / blck_size(ty) * type_size(ty);
        std::vector<uint8_t> buf((size_t)(rb * t.ne1));
        const uint64_t key = tensor_key(t.name, s->seed);
#pragma omp parallel for num_threads(nt) schedule(dynamic, 16)
        for (int64_t r = 0; r < t.ne1; r++) {
            std::vector<float> row(t.ne0);
            if (t.kind == 1) std::fill(row.begin(), row.end(), 1.0f);
            else normal_row(row.data(), r * t.ne0, t.ne0, key, s->w_std);
            if (src_f16)
                for (auto &v : row) v = h2f(f2h(v));
            uint8_t *o = buf.data() + r * rb;
            switch (ty) {
                case T_F32: memcpy(o, row.data(), t.ne0 * 4); break;
                case T_F16: for (int64_t k = 0; k < t.ne0; k++) { const uint16_t v = f2h(row[k]); memcpy(o + 2 * k, &v, 2); } break;
                case T_Q8_0: for (int64_t b = 0; b < t.ne0 / 32; b++) q80_block(row.data() + 32 * b, o + 34 * b); break;
                case T_Q4_K: for (int64_t b = 0; b < t.ne0 / 256; b++) q4k_block(row.data() + 256 * b, o + 144 * b); break;
                case T_Q6_K: for (int64_t b = 0; b < t.ne0 / 256; b++) q6k_block(row.data() + 256 * b, o + 210 * b); break;
            }
        }
        fwrite(buf.data(), 1, buf.size(), f);
        static const uint8_t zeros[32] = {0};
        if (buf.size() % 32) fwrite(zeros, 1, 32 - buf.size() % 32, f);
    }
    const bool ok = !ferror(f);
    fclose(f);
    return ok ? 0 : -1;
}
#pragma GCC pop_options
