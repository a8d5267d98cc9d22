// libdfb_cuda: implementation of the C-ABI in include/diffuse_b200.h.
//
// Owns the device-resident model (weights re-tiled for the dequant GEMM), the
// per-context activations / K/V cache / logits buffer / sequence state, and the
// launch order of one denoising step:
//   step_prepare -> embed -> L x [(residual +) rmsnorm, QKV(+bias,RoPE,cache write),
//   attention, O, residual + rmsnorm, gate|up(SwiGLU), down] -> residual + rmsnorm ->
//   lm_head (logits scattered to their positions) -> row statistics -> order + commit.
// The O and down projections write y; the next RMSNorm adds y into the residual stream x.
// This is the device side of src/diffuse-sampler.cpp:127-323 with the forward of
// src/diffuse-graph.cpp:11-160 / 395-593.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../../include/diffuse_b200.h"
#include "attention.cuh"
#include "gemm_dq.cuh"
#include "ops.cuh"

using namespace dfb;

// ───────────────────────── errors ─────────────────────────
static thread_local std::string g_err;
static int set_err(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}
#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return set_err(e_ == cudaErrorMemoryAllocation ? DFB_ERR_NOMEM : DFB_ERR_CUDA,         \
                           "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)
#define RET(x)                 \
    do {                       \
        int r_ = (x);          \
        if (r_ != DFB_OK) return r_; \
    } while (0)

extern "C" const char *dfb_last_error(void) { return g_err.c_str(); }


extern "C" int dfb_device_count(int *n) {
    if (!n) return set_err(DFB_ERR_ARG, "null pointer");
    cudaError_t e = cudaGetDeviceCount(n);
    if (e != cudaSuccess) {
        *n = 0;
        return set_err(DFB_ERR_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    return DFB_OK;
}

// ───────────────────────── tensor maps ─────────────────────────
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}
// 2-D f16 matrix [rows][cols], 128-byte swizzled boxes of box_rows x 64.
static int make_tmap(CUtensorMap *m, const void *ptr, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_err(DFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((cols * 2) % 16 != 0) return set_err(DFB_ERR_ARG, "row length %llu not a multiple of 8", (unsigned long long)cols);
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err(DFB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DFB_OK;
}

// The 3-D activation views the GEMM loads its B operand through (XMaps in gemm_dq.cuh):
// x is a row-major f16 matrix of rows of xs * K values (xs = 2: pair rows, xs = 1: plain),
// K a multiple of 64, x 16-byte aligned.
static int make_xmaps(XMaps *xm, const void *x, int K, int rows, int xs) {
    auto fn = encode_fn();
    if (!fn) return set_err(DFB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (K % 64) return set_err(DFB_ERR_UNSUPPORTED, "activation width %d not a multiple of 64", K);
    if (reinterpret_cast<uintptr_t>(x) % 16) return set_err(DFB_ERR_ARG, "activation matrix not 16-byte aligned");
    for (int i = 0; i < kXMaps; i++) {
        const int h = 16 * (i + 1);
        cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(xs * K / 64)};
        cuuint64_t strides[2] = {(cuuint64_t)xs * K * 2, 128};
        cuuint32_t box[3] = {64, (cuuint32_t)h, (cuuint32_t)(xs * x_slices(h))};
        cuuint32_t es[3] = {1, 1, 1};
        CUresult r = fn(&xm->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(x), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_err(DFB_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
    }
    return DFB_OK;
}

// ───────────────────────── host-side format helpers ─────────────────────────
enum { G_F32 = 0, G_F16 = 1, G_Q8_0 = 8, G_Q4_K = 12, G_Q6_K = 14, G_BF16 = 30 };

static int64_t ggml_row_bytes(int type, int64_t n) {
    switch (type) {
        case G_F32: return 4 * n;
        case G_F16: case G_BF16: return 2 * n;
        case G_Q8_0: return n / 32 * 34;
        case G_Q4_K: return n / 256 * 144;
        case G_Q6_K: return n / 256 * 210;
        default: return -1;
    }
}
static float h2f_host(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}
static uint16_t f2h_host(float f) {
    __half h = __float2half_rn(f);
    return reinterpret_cast<__half_raw &>(h).x;
}
static float bf2f_host(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
// Dequantize one row to f32 (host; used for norms, biases and non-F16 embeddings).
static void dequant_row_host(int type, const uint8_t *src, int64_t n, float *dst) {
    switch (type) {
        case G_F32: memcpy(dst, src, n * 4); return;
        case G_F16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = h2f_host(h); } return;
        case G_BF16: for (int64_t i = 0; i < n; i++) { uint16_t h; memcpy(&h, src + 2 * i, 2); dst[i] = bf2f_host(h); } return;
        case G_Q8_0:
            for (int64_t b = 0; b < n / 32; b++) {
                uint16_t dh; memcpy(&dh, src + 34 * b, 2);
                const float d = h2f_host(dh);
                for (int l = 0; l < 32; l++) dst[32 * b + l] = d * (float)(int8_t)src[34 * b + 2 + l];
            }
            return;
        case G_Q4_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + 144 * b;
                uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
                const float d = h2f_host(dh), dmin = h2f_host(mh);
                const uint8_t *q = blk + 4, *qs = blk + 16;
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
            return;
        case G_Q6_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t *blk = src + 210 * b, *ql = blk, *qh = blk + 128;
                const int8_t *sc = (const int8_t *)(blk + 192);
                uint16_t dh; memcpy(&dh, blk + 208, 2);
                const float d = h2f_host(dh);
                for (int e = 0; e < 256; e++) {
                    const int h = e / 128, g = (e % 128) / 32, l = e % 32;
                    const uint8_t lb = ql[64 * h + (g & 1) * 32 + l];
                    const int nib = (g >= 2) ? (lb >> 4) : (lb & 0xF);
                    const int q = (nib | (((qh[32 * h + l] >> (2 * g)) & 3) << 4)) - 32;
                    dst[256 * b + e] = d * sc[e / 16] * q;
                }
            }
            return;
    }
}

// ───────────────────────── device weights ─────────────────────────
struct WMat {
    int wt = -1;
    int n_rows = 0, n_tiles = 0, K = 0, kb = 0;
    int n_true = 0;     // output features the model defines (before padding / fusion slack)
    float wscale = 1.f; // power-of-two pre-scale of the dequantized weights (quantized types)
    int lo_row = 0, corr_row = 0;  // f16-tile weights: first row of the lo / correction matrix
    uint8_t *d = nullptr;
    CUtensorMap tm{};   // f16-tile weights: [hi | (lo, W_F32) | correction] matrices stacked by rows
    size_t bytes = 0;
};

static int wt_of(int ggml_type) {
    switch (ggml_type) {
        case G_Q4_K: return W_Q4K;
        case G_Q6_K: return W_Q6K;
        case G_Q8_0: return W_Q80;
        case G_F16: return W_F16;
        case G_F32: case G_BF16: return W_F32;
        default: return -1;
    }
}

// Re-tile rows (nullptr = zero row; rows.size() a multiple of 128) into the chunk
// layouts the dequant kernel reads (dequant.cuh), or into stacked [rows][K] matrices of
// f16-sized elements: W_F16 the weights and their correction matrix, W_F32 (F32 / BF16
// sources) hi, lo and correction.  A correction row holds, per 64-wide slice, 64 E4M3 of
// hi * 2^-10 then 64 E4M3 of lo (128 bytes: the width of 64 f16), the weight side of the
// GEMM's correction MMA (dequant.cuh).
static void retile_range(const std::vector<const uint8_t *> &rows, int type, int64_t K, int kb, int t0, int t1,
                         float ws, uint8_t *out) {
    const int wt = wt_of(type);
    const int RB = raw_chunk_bytes(wt);
    if (wt == W_F16 || wt == W_F32) {
        const size_t n_rows = rows.size();
        const int n_mats = wt == W_F32 ? 3 : 2;
        for (int r = t0 * 128; r < t1 * 128; r++) {
            uint16_t *dst = reinterpret_cast<uint16_t *>(out) + (size_t)r * K;
            uint16_t *dlo = reinterpret_cast<uint16_t *>(out) + (n_rows + r) * K;  // W_F32 only
            uint8_t *dcor = out + ((n_mats - 1) * n_rows + r) * K * 2;
            const uint8_t *src = rows[r];
            if (!src) {
                for (int mi = 0; mi < n_mats; mi++) memset(out + ((size_t)mi * n_rows + r) * K * 2, 0, K * 2);
                continue;
            }
            for (int64_t i = 0; i < K; i++) {
                float f;
                if (type == G_F16) { uint16_t h; memcpy(&h, src + 2 * i, 2); f = h2f_host(h); }
                else if (type == G_F32) memcpy(&f, src + 4 * i, 4);
                else { uint16_t b; memcpy(&b, src + 2 * i, 2); f = bf2f_host(b); }
                f *= ws;  // power of two: F16 values stay exact
                dst[i] = f2h_host(f);
                const float hi = h2f_host(dst[i]), lo = f - hi;
                if (wt == W_F32) dlo[i] = f2h_host(lo);
                const int64_t sl = i / 64, k = i % 64;
                dcor[128 * sl + k] = (uint8_t)(e4m3x2(hi * kCorrScale, 0.f) & 0xFF);
                dcor[128 * sl + 64 + k] = (uint8_t)(e4m3x2(lo, 0.f) & 0xFF);
            }
        }
        return;
    }
    static const uint8_t zeros[288] = {0};
    for (int t = t0; t < t1; t++)
        for (int b = 0; b < kb; b++) {
            uint8_t *C = out + ((size_t)t * kb + b) * RB;
            for (int r = 0; r < 128; r++) {
                const uint8_t *row = rows[(size_t)t * 128 + r];
                if (wt == W_Q4K) {
                    const uint8_t *blk = row ? row + (size_t)b * 144 : zeros;
                    memcpy(C + 4 * r, blk, 4);
                    memcpy(C + 512 + 12 * r, blk + 4, 12);
                    for (int c = 0; c < 8; c++) memcpy(C + 2048 + 128 * r + ((c ^ (r & 7)) << 4), blk + 16 + 16 * c, 16);
                } else if (wt == W_Q6K) {
                    const uint8_t *blk = row ? row + (size_t)b * 210 : zeros;
                    for (int c = 0; c < 8; c++) memcpy(C + 128 * r + ((c ^ (r & 7)) << 4), blk + 16 * c, 16);
                    for (int c = 0; c < 4; c++) memcpy(C + 16384 + 64 * r + ((c ^ ((r >> 1) & 3)) << 4), blk + 128 + 16 * c, 16);
                    memcpy(C + 24576 + 16 * r, blk + 192, 16);
                    memcpy(C + 26624 + 2 * r, blk + 208, 2);
                } else {  // Q8_0: 8 blocks of 32 per k-block; blocks past K are zero
                    for (int i = 0; i < 8; i++) {
                        const int64_t blk_idx = (int64_t)b * 8 + i;
                        const uint8_t *blk = (row && blk_idx * 32 < K) ? row + blk_idx * 34 : zeros;
                        memcpy(C + 16 * r + 2 * i, blk, 2);
                        for (int hlf = 0; hlf < 2; hlf++) {
                            const int c = 2 * i + hlf;
                            memcpy(C + 2048 + 256 * r + (((c & 8) | ((c & 7) ^ (r & 7))) << 4), blk + 2 + 16 * hlf, 16);
                        }
                    }
                }
            }
        }
}

// Upper bound of |w| over rows [r0, r1) of a matrix: quantized types from the block
// scales (Q4_K |d|*63*15 + |dmin|*63, Q6_K |d|*128*32, Q8_0 |d|*128), float types exactly.
static float weight_bound_range(const std::vector<const uint8_t *> &rows, int type, int64_t K, size_t r0, size_t r1) {
    float b = 0.f;
    for (size_t r = r0; r < r1; r++) {
        const uint8_t *row = rows[r];
        if (!row) continue;
        if (type == G_F16 || type == G_BF16 || type == G_F32) {
            for (int64_t i = 0; i < K; i++) {
                float f;
                if (type == G_F32) memcpy(&f, row + 4 * i, 4);
                else { uint16_t h; memcpy(&h, row + 2 * i, 2); f = type == G_F16 ? h2f_host(h) : bf2f_host(h); }
                if (std::isfinite(f)) b = std::max(b, fabsf(f));
            }
        } else if (type == G_Q4_K) {
            for (int64_t k = 0; k < K / 256; k++) {
                uint16_t dh, mh;
                memcpy(&dh, row + 144 * k, 2);
                memcpy(&mh, row + 144 * k + 2, 2);
                b = std::max(b, fabsf(h2f_host(dh)) * 945.f + fabsf(h2f_host(mh)) * 63.f);
            }
        } else if (type == G_Q6_K) {
            for (int64_t k = 0; k < K / 256; k++) {
                uint16_t dh;
                memcpy(&dh, row + 210 * k + 208, 2);
                b = std::max(b, fabsf(h2f_host(dh)) * 4096.f);
            }
        } else if (type == G_Q8_0) {
            for (int64_t k = 0; k < K / 32; k++) {
                uint16_t dh;
                memcpy(&dh, row + 34 * k, 2);
                b = std::max(b, fabsf(h2f_host(dh)) * 128.f);
            }
        }
    }
    return b;
}

// The pre-scale 2^e that puts the largest weight near 2^14: hi parts stay far below
// f16's maximum (65504) and the lo parts of all but negligible weights stay normal.
static float weight_prescale(float bound) {
    if (!(bound > 0.f) || !std::isfinite(bound)) return 1.f;
    const int e = std::max(-60, std::min(60, (int)floorf(log2f(16384.f / bound))));
    return ldexpf(1.f, e);
}

static int build_wmat(const std::vector<const uint8_t *> &rows_in, int type, int64_t K, WMat &w) {
    const int wt = wt_of(type);
    if (wt < 0) return set_err(DFB_ERR_UNSUPPORTED, "GGML type %d not supported for a linear weight", type);
    if (rows_in.size() % 128) return set_err(DFB_ERR_ARG, "internal: rows not padded");
    // the GEMM works on pair tiles of 256 rows: an odd last tile gets a zero partner
    std::vector<const uint8_t *> rows(rows_in);
    rows.resize((rows.size() + 255) / 256 * 256, nullptr);
    if ((wt == W_Q4K || wt == W_Q6K) && K % 256) return set_err(DFB_ERR_ARG, "K-quant row length %lld not a multiple of 256", (long long)K);
    if (wt == W_Q80 && K % 32) return set_err(DFB_ERR_ARG, "Q8_0 row length %lld not a multiple of 32", (long long)K);
    if (w_smem(wt) && K % 64) return set_err(DFB_ERR_ARG, "F16/F32 row length %lld not a multiple of 64", (long long)K);
    w.wt = wt;
    w.n_rows = (int)rows.size();
    w.n_tiles = w.n_rows / 128;
    w.K = (int)K;
    w.kb = (int)((K + 255) / 256);
    const int n_mats = wt == W_F16 ? 2 : wt == W_F32 ? 3 : 0;
    w.bytes = n_mats ? (size_t)n_mats * w.n_rows * K * 2 : (size_t)w.n_tiles * w.kb * raw_chunk_bytes(wt);
    w.lo_row = wt == W_F32 ? w.n_rows : 0;
    w.corr_row = n_mats ? (n_mats - 1) * w.n_rows : 0;
    std::vector<uint8_t> host(w.bytes);
    const int nthr = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    // the pre-scale first (f16 tiles are written scaled), then the re-tiling
    std::vector<float> bounds(nthr, 0.f);
    {
        std::vector<std::thread> th;
        for (int i = 0; i < nthr; i++) {
            const size_t r0 = (size_t)w.n_rows * i / nthr, r1 = (size_t)w.n_rows * (i + 1) / nthr;
            th.emplace_back([&, r0, r1, i] { bounds[i] = weight_bound_range(rows, type, K, r0, r1); });
        }
        for (auto &t : th) t.join();
    }
    w.wscale = weight_prescale(*std::max_element(bounds.begin(), bounds.end()));
    {
        std::vector<std::thread> th;
        for (int i = 0; i < nthr; i++) {
            const int t0 = (int)((int64_t)w.n_tiles * i / nthr), t1 = (int)((int64_t)w.n_tiles * (i + 1) / nthr);
            th.emplace_back([&, t0, t1] { retile_range(rows, type, K, w.kb, t0, t1, w.wscale, host.data()); });
        }
        for (auto &t : th) t.join();
    }
    CK(cudaMalloc(&w.d, w.bytes));
    CK(cudaMemcpy(w.d, host.data(), w.bytes, cudaMemcpyHostToDevice));
    if (w_smem(wt)) RET(make_tmap(&w.tm, w.d, (uint64_t)K, (uint64_t)n_mats * w.n_rows, 128));
    return DFB_OK;
}

// ───────────────────────── NCCL (tensor parallelism only) ─────────────────────────
// Bound at run time on first use, so the library loads and runs single-GPU without NCCL; in a
// process that already holds libnccl.so.2 (e.g. torch's) dlopen returns that copy.
struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};
static NcclApi &nccl_api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
        a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
        a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
        a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
        a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
        a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
        a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy && a.error_string;
    });
    return a;
}
#define NK(call)                                                                                      \
    do {                                                                                              \
        ncclResult_t _r = (call);                                                                     \
        if (_r != ncclSuccess) return set_err(DFB_ERR_CUDA, "%s: %s", #call, nccl_api().error_string(_r)); \
    } while (0)

struct LayerW {
    WMat qkv, o, gateup, down;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *bias_qkv = nullptr;
};

struct HostTensor {
    int type = -1;
    int64_t ne0 = 0, ne1 = 0;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

struct dfb_model {
    dfb_hparams hp{};
    int device = 0, n_sm = 0;
    // per-rank dimensions (the whole model's when tp_size == 1): query / KV features of the
    // rank's heads, its FFN features and its vocabulary rows [v0, v0 + n_vocab_l)
    int hd = 0, n_q = 0, n_kv = 0, nq_pad = 0, nk_pad = 0;
    int n_head_l = 0, n_ff_l = 0, v0 = 0, n_vocab_l = 0;
    // tensor parallelism (dfb_model_set_tp): this rank of tp_size, its NCCL communicator
    int tp_rank = 0, tp_size = 1;
    ncclComm_t comm = nullptr;
    std::vector<HostTensor> staged;  // [role + DFB_N_ROLES * layer]
    // device
    void *embd = nullptr;
    int embd_f16 = 1;
    float *output_norm = nullptr;
    WMat lm_head;
    std::vector<LayerW> layers;
    bool finalized = false;
    size_t bytes = 0;
    std::vector<void *> allocs;
};

static HostTensor &staged(dfb_model *m, int role, int layer) {
    return m->staged[(size_t)layer * DFB_N_ROLES + role];
}

extern "C" int dfb_model_create(const dfb_hparams *hp, int device, dfb_model **out) {
    if (!hp || !out) return set_err(DFB_ERR_ARG, "null pointer");
    *out = nullptr;
    if (hp->n_layer <= 0 || hp->n_embd <= 0 || hp->n_head <= 0 || hp->n_head_kv <= 0 || hp->n_ff <= 0 ||
        hp->n_vocab <= 0 || hp->n_head % hp->n_head_kv || hp->n_embd % hp->n_head)
        return set_err(DFB_ERR_ARG, "inconsistent hyper-parameters");
    const int hd = hp->n_embd / hp->n_head;
    if (hd != 16 && hd != 32 && hd != 64 && hd != 128)
        return set_err(DFB_ERR_UNSUPPORTED, "head_dim %d not supported (16/32/64/128)", hd);
    // GEMM activations are stored as pair rows of 64-wide slices
    if (hp->n_embd % 64 || hp->n_ff % 64)
        return set_err(DFB_ERR_UNSUPPORTED, "n_embd %d / n_ff %d not multiples of 64", hp->n_embd, hp->n_ff);
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0) CK(cudaGetDevice(&device));  // -1: the caller's current device
    if (device < 0 || device >= ndev) return set_err(DFB_ERR_ARG, "device %d out of range (%d devices)", device, ndev);
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return set_err(DFB_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device, prop.major, prop.minor);
    auto *m = new dfb_model();
    m->hp = *hp;
    m->device = device;
    m->n_sm = prop.multiProcessorCount;
    m->hd = hd;
    m->n_q = hp->n_embd;
    m->n_kv = hp->n_head_kv * hd;
    m->nq_pad = (m->n_q + 127) / 128 * 128;
    m->nk_pad = (m->n_kv + 127) / 128 * 128;
    m->n_head_l = hp->n_head;
    m->n_ff_l = hp->n_ff;
    m->n_vocab_l = hp->n_vocab;
    m->staged.resize((size_t)DFB_N_ROLES * hp->n_layer);
    m->layers.resize(hp->n_layer);
    *out = m;
    return DFB_OK;
}

extern "C" int dfb_model_set_tensor(dfb_model *m, int role, int layer, int type, int64_t ne0, int64_t ne1,
                                    const void *data, size_t nbytes) {
    if (!m || !data) return set_err(DFB_ERR_ARG, "null pointer");
    if (m->finalized) return set_err(DFB_ERR_STATE, "model already finalized");
    if (role < 0 || role >= DFB_N_ROLES) return set_err(DFB_ERR_ARG, "bad role %d", role);
    const bool global = role <= DFB_OUTPUT;
    if (global) layer = 0;
    else if (layer < 0 || layer >= m->hp.n_layer) return set_err(DFB_ERR_ARG, "bad layer %d", layer);
    const int64_t rb = ggml_row_bytes(type, ne0);
    if (rb < 0) return set_err(DFB_ERR_UNSUPPORTED, "GGML type %d not supported", type);
    if ((int64_t)nbytes < rb * std::max<int64_t>(ne1, 1)) return set_err(DFB_ERR_ARG, "tensor role %d: %zu bytes < %lld expected", role, nbytes, (long long)(rb * ne1));
    HostTensor &t = staged(m, role, layer);
    t.type = type; t.ne0 = ne0; t.ne1 = std::max<int64_t>(ne1, 1); t.data = (const uint8_t *)data; t.nbytes = nbytes;
    return DFB_OK;
}

static int upload_vec(dfb_model *m, const HostTensor &t, int64_t n, float **out) {
    if (t.ne0 * t.ne1 < n) return set_err(DFB_ERR_ARG, "vector has %lld elements, need %lld", (long long)(t.ne0 * t.ne1), (long long)n);
    std::vector<float> v(n);
    dequant_row_host(t.type, t.data, n, v.data());
    CK(cudaMalloc(out, n * 4));
    m->allocs.push_back(*out);
    CK(cudaMemcpy(*out, v.data(), n * 4, cudaMemcpyHostToDevice));
    m->bytes += n * 4;
    return DFB_OK;
}

static int check_mat(const HostTensor &t, const char *what, int64_t ne0, int64_t ne1) {
    if (!t.data) return set_err(DFB_ERR_STATE, "tensor %s missing", what);
    if (t.ne0 != ne0 || t.ne1 != ne1)
        return set_err(DFB_ERR_ARG, "tensor %s has shape %lldx%lld, expected %lldx%lld", what, (long long)t.ne0,
                       (long long)t.ne1, (long long)ne0, (long long)ne1);
    return DFB_OK;
}

extern "C" int dfb_model_finalize(dfb_model *m) {
    if (!m) return set_err(DFB_ERR_ARG, "null model");
    if (m->finalized) return DFB_OK;
    CK(cudaSetDevice(m->device));
    const dfb_hparams &hp = m->hp;
    const int d = hp.n_embd, ff = hp.n_ff, V = hp.n_vocab, hd = m->hd;
    // this rank's slices (everything when tp_size == 1): heads [h0, h0 + n_head_l) and their
    // KV heads, FFN features [f0, f0 + ffl), vocabulary rows [v0, v0 + n_vocab_l)
    const int gq = hp.n_embd, gkv = hp.n_head_kv * hd;             // whole-model Q / KV widths
    const int h0 = m->tp_rank * m->n_head_l, kvh0 = m->tp_rank * (m->n_kv / hd);
    const int ffl = m->n_ff_l, f0 = m->tp_rank * ffl;
    // a K-range [k0, k0 + n) of a GGUF row: its byte offset (k0 on a block boundary)
    auto k_offset = [&](int type, int64_t k0, const char *what) -> int64_t {
        const int64_t blk = type == G_Q4_K || type == G_Q6_K ? 256 : type == G_Q8_0 ? 32 : 1;
        if (k0 % blk) {
            set_err(DFB_ERR_UNSUPPORTED, "%s: the rank's K slice starts at %lld, inside a %lld-value block", what,
                    (long long)k0, (long long)blk);
            return -1;
        }
        return ggml_row_bytes(type, k0);
    };
    // embeddings: F16 kept, everything else dequantized to f32
    {
        const HostTensor &e = staged(m, DFB_TOK_EMBD, 0);
        RET(check_mat(e, "token_embd", d, V));
        const size_t n = (size_t)d * V;
        if (e.type == G_F16) {
            CK(cudaMalloc(&m->embd, n * 2));
            CK(cudaMemcpy(m->embd, e.data, n * 2, cudaMemcpyHostToDevice));
            m->embd_f16 = 1;
            m->bytes += n * 2;
        } else {
            std::vector<float> v(n);
            const int64_t rb = ggml_row_bytes(e.type, d);
            for (int64_t r = 0; r < V; r++) dequant_row_host(e.type, e.data + r * rb, d, v.data() + (size_t)r * d);
            CK(cudaMalloc(&m->embd, n * 4));
            CK(cudaMemcpy(m->embd, v.data(), n * 4, cudaMemcpyHostToDevice));
            m->embd_f16 = 0;
            m->bytes += n * 4;
        }
        m->allocs.push_back(m->embd);
    }
    RET(upload_vec(m, staged(m, DFB_OUTPUT_NORM, 0), d, &m->output_norm));
    // lm_head (tied to token_embd when output.weight is absent, diffuse-model.cpp:157-158)
    {
        HostTensor out = staged(m, DFB_OUTPUT, 0);
        if (!out.data) out = staged(m, DFB_TOK_EMBD, 0);
        RET(check_mat(out, "output", d, V));
        const int64_t rb = ggml_row_bytes(out.type, d);
        const int Vl = m->n_vocab_l;
        std::vector<const uint8_t *> rows((Vl + 127) / 128 * 128, nullptr);
        for (int r = 0; r < Vl; r++) rows[r] = out.data + (int64_t)(m->v0 + r) * rb;
        RET(build_wmat(rows, out.type, d, m->lm_head));
        m->lm_head.n_true = Vl;
        m->bytes += m->lm_head.bytes;
    }
    for (int l = 0; l < hp.n_layer; l++) {
        LayerW &L = m->layers[l];
        const HostTensor &wq = staged(m, DFB_WQ, l), &wk = staged(m, DFB_WK, l), &wv = staged(m, DFB_WV, l);
        RET(check_mat(wq, "attn_q", d, gq));
        RET(check_mat(wk, "attn_k", d, gkv));
        RET(check_mat(wv, "attn_v", d, gkv));
        if (wq.type != wk.type || wq.type != wv.type)
            return set_err(DFB_ERR_UNSUPPORTED, "layer %d: attn_q/k/v have different types (%d/%d/%d)", l, wq.type, wk.type, wv.type);
        // fused QKV rows: [Q | K | V], each section padded to 128 rows; Q and K rows
        // permuted inside each head so NEOX pairs (i, i+hd/2) sit in adjacent TMEM lanes
        {
            std::vector<const uint8_t *> rows(m->nq_pad + 2 * m->nk_pad, nullptr);
            const int64_t rb = ggml_row_bytes(wq.type, d);
            for (int r = 0; r < m->n_q; r++) {
                const int head = h0 + r / hd, rr = r % hd, i = rr >> 1, b = rr & 1;
                rows[r] = wq.data + (int64_t)(head * hd + i + b * (hd >> 1)) * rb;
            }
            for (int r = 0; r < m->n_kv; r++) {
                const int head = kvh0 + r / hd, rr = r % hd, i = rr >> 1, b = rr & 1;
                rows[m->nq_pad + r] = wk.data + (int64_t)(head * hd + i + b * (hd >> 1)) * rb;
                rows[m->nq_pad + m->nk_pad + r] = wv.data + (int64_t)(kvh0 * hd + r) * rb;
            }
            RET(build_wmat(rows, wq.type, d, L.qkv));
            L.qkv.n_true = m->n_q + 2 * m->n_kv;
        }
        const HostTensor &bq = staged(m, DFB_BQ, l), &bk = staged(m, DFB_BK, l), &bv = staged(m, DFB_BV, l);
        if (bq.data || bk.data || bv.data) {
            std::vector<float> b(m->nq_pad + 2 * m->nk_pad, 0.f), full(std::max(gq, gkv));
            auto slice = [&](const HostTensor &t, int n_all, int first, int n, float *dst) {
                dequant_row_host(t.type, t.data, n_all, full.data());
                std::copy(full.begin() + first, full.begin() + first + n, dst);
            };
            if (bq.data) slice(bq, gq, h0 * hd, m->n_q, b.data());
            if (bk.data) slice(bk, gkv, kvh0 * hd, m->n_kv, b.data() + m->nq_pad);
            if (bv.data) slice(bv, gkv, kvh0 * hd, m->n_kv, b.data() + m->nq_pad + m->nk_pad);
            CK(cudaMalloc(&L.bias_qkv, b.size() * 4));
            m->allocs.push_back(L.bias_qkv);
            CK(cudaMemcpy(L.bias_qkv, b.data(), b.size() * 4, cudaMemcpyHostToDevice));
        }
        const HostTensor &wo = staged(m, DFB_WO, l);
        RET(check_mat(wo, "attn_output", gq, d));
        {
            // the rank's heads' input columns of every output row (row-parallel: partial sums)
            std::vector<const uint8_t *> rows((d + 127) / 128 * 128, nullptr);
            const int64_t rb = ggml_row_bytes(wo.type, gq), off = k_offset(wo.type, (int64_t)h0 * hd, "attn_output");
            if (off < 0) return DFB_ERR_UNSUPPORTED;
            for (int r = 0; r < d; r++) rows[r] = wo.data + (int64_t)r * rb + off;
            RET(build_wmat(rows, wo.type, m->n_q, L.o));
            L.o.n_true = d;
        }
        const HostTensor &wg = staged(m, DFB_GATE, l), &wu = staged(m, DFB_UP, l), &wd = staged(m, DFB_DOWN, l);
        RET(check_mat(wg, "ffn_gate", d, ff));
        RET(check_mat(wu, "ffn_up", d, ff));
        RET(check_mat(wd, "ffn_down", ff, d));
        if (wg.type != wu.type) return set_err(DFB_ERR_UNSUPPORTED, "layer %d: ffn_gate/up types differ", l);
        {
            std::vector<const uint8_t *> rows((2 * ffl + 127) / 128 * 128, nullptr);
            const int64_t rb = ggml_row_bytes(wg.type, d);
            for (int i = 0; i < ffl; i++) {
                rows[2 * i] = wg.data + (int64_t)(f0 + i) * rb;
                rows[2 * i + 1] = wu.data + (int64_t)(f0 + i) * rb;
            }
            RET(build_wmat(rows, wg.type, d, L.gateup));
            L.gateup.n_true = 2 * ffl;
        }
        {
            // the rank's FFN features' input columns of every output row (row-parallel)
            std::vector<const uint8_t *> rows((d + 127) / 128 * 128, nullptr);
            const int64_t rb = ggml_row_bytes(wd.type, ff), off = k_offset(wd.type, f0, "ffn_down");
            if (off < 0) return DFB_ERR_UNSUPPORTED;
            for (int r = 0; r < d; r++) rows[r] = wd.data + (int64_t)r * rb + off;
            RET(build_wmat(rows, wd.type, ffl, L.down));
            L.down.n_true = d;
        }
        RET(upload_vec(m, staged(m, DFB_ATTN_NORM, l), d, &L.attn_norm));
        RET(upload_vec(m, staged(m, DFB_FFN_NORM, l), d, &L.ffn_norm));
        m->bytes += L.qkv.bytes + L.o.bytes + L.gateup.bytes + L.down.bytes;
    }
    m->staged.clear();
    m->staged.shrink_to_fit();
    m->finalized = true;
    return DFB_OK;
}

extern "C" int dfb_tp_unique_id(uint8_t *id, int nbytes) {
    if (!id || nbytes < (int)sizeof(ncclUniqueId)) return set_err(DFB_ERR_ARG, "need %d bytes", (int)sizeof(ncclUniqueId));
    if (!nccl_api().ok) return set_err(DFB_ERR_UNSUPPORTED, "libnccl.so.2 not found");
    ncclUniqueId u;
    NK(nccl_api().get_unique_id(&u));
    memcpy(id, &u, sizeof(u));
    return DFB_OK;
}

extern "C" int dfb_model_set_tp(dfb_model *m, int rank, int size, const uint8_t *id, int nbytes) {
    if (!m || size < 1 || rank < 0 || rank >= size) return set_err(DFB_ERR_ARG, "bad arguments");
    if (m->finalized) return set_err(DFB_ERR_STATE, "model already finalized");
    if (size == 1) return DFB_OK;
    if (!id || nbytes < (int)sizeof(ncclUniqueId)) return set_err(DFB_ERR_ARG, "need the %d-byte NCCL id", (int)sizeof(ncclUniqueId));
    const dfb_hparams &hp = m->hp;
    if (hp.n_head % size || hp.n_head_kv % size || hp.n_ff % (64 * size))
        return set_err(DFB_ERR_UNSUPPORTED, "%d-way tensor parallelism needs n_head %d, n_head_kv %d divisible and n_ff %d / %d a multiple of 64",
                       size, hp.n_head, hp.n_head_kv, hp.n_ff, size);
    if (!nccl_api().ok) return set_err(DFB_ERR_UNSUPPORTED, "libnccl.so.2 not found");
    m->tp_rank = rank;
    m->tp_size = size;
    m->n_head_l = hp.n_head / size;
    m->n_q = m->n_head_l * m->hd;
    m->n_kv = hp.n_head_kv / size * m->hd;
    m->nq_pad = (m->n_q + 127) / 128 * 128;
    m->nk_pad = (m->n_kv + 127) / 128 * 128;
    m->n_ff_l = hp.n_ff / size;
    const int vb = (hp.n_vocab + size - 1) / size;
    m->v0 = std::min(hp.n_vocab, rank * vb);
    m->n_vocab_l = std::min(hp.n_vocab, m->v0 + vb) - m->v0;
    CK(cudaSetDevice(m->device));
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    NK(nccl_api().comm_init_rank(&m->comm, size, u, rank));
    return DFB_OK;
}

extern "C" int dfb_model_tp_info(const dfb_model *m, int *rank, int *size, int *v0, int *n_vocab_local) {
    if (!m) return set_err(DFB_ERR_ARG, "null model");
    if (rank) *rank = m->tp_rank;
    if (size) *size = m->tp_size;
    if (v0) *v0 = m->v0;
    if (n_vocab_local) *n_vocab_local = m->n_vocab_l;
    return DFB_OK;
}

extern "C" void dfb_model_free(dfb_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->comm) nccl_api().comm_destroy(m->comm);
    for (void *p : m->allocs) cudaFree(p);
    cudaFree(m->lm_head.d);
    for (auto &L : m->layers) {
        cudaFree(L.qkv.d); cudaFree(L.o.d); cudaFree(L.gateup.d); cudaFree(L.down.d);
    }
    delete m;
}

extern "C" int dfb_model_bytes(const dfb_model *m, size_t *bytes) {
    if (!m || !bytes) return set_err(DFB_ERR_ARG, "null pointer");
    *bytes = m->bytes;
    return DFB_OK;
}

// ───────────────────────── context ─────────────────────────
struct dfb_ctx {
    dfb_model *m = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    int cap = 0;
    // activations
    float *x = nullptr, *y = nullptr, *logits = nullptr;  // residual stream, projection output, logits
    float *q = nullptr, *kc = nullptr, *vc = nullptr;      // Q rows, K/V cache [layer][position][n_kv] (f32)
    uint8_t *h = nullptr, *att = nullptr, *ffh = nullptr;  // GEMM inputs as pair rows (4 bytes per value)
    float2 *rope = nullptr;
    XMaps xm_h{}, xm_att{}, xm_ffh{};  // GEMM B-operand views of h, att, ffh
    // sequence state
    int32_t *seq = nullptr, *prev_seq = nullptr, *last_changed = nullptr, *cand_tok = nullptr, *commit_pos = nullptr,
            *commit_tok = nullptr, *order = nullptr;
    uint8_t *masked = nullptr;
    int *active_pos = nullptr, *masked_pos = nullptr, *cnt = nullptr;
    float *cand_conf = nullptr, *cand_ent = nullptr;
    double *unif = nullptr;  // temperature > 0: the host's uniforms of the next step, one per masked candidate
    float4 *tp_stats = nullptr, *tp_gath = nullptr;  // tensor parallelism: per-candidate statistics, all ranks'
    float2 *tp_g = nullptr;                          // their combination (max, log Z)
    int unif_n = -1;         // how many the host set for the next step (-1: none)
    // sequences (segments) stepping together: positions [seg_off[s], seg_off[s+1]) of the
    // concatenated state; per-segment counters, schedule counts, finished flags, work lists
    int *seg_off = nullptr, *seg_cnt = nullptr, *sched = nullptr, *tmp_active = nullptr, *tmp_masked = nullptr,
        *rope_pos = nullptr, *masked_row = nullptr;
    uint8_t *done = nullptr;
    int4 *tiles = nullptr;
    // GEMM scratch
    float *ws = nullptr;
    int *tile_cnt = nullptr, *err = nullptr;
    int n_tile_cnt = 0;
    // failure-detection test hook (dfb_debug_stalled_linear): the next GEMM launch starts
    // with tile counter 0 poisoned and every wait limited to stall_timeout_ns
    bool stall_next = false;
    unsigned long long stall_timeout_ns = 0;
    // optional per-launch timing (dfb_ctx_profile)
    struct ProfRec {
        cudaEvent_t a, b;
        int cat;
        double flops_per_row, bytes_fixed, bytes_per_row;
    };
    bool prof = false;
    std::vector<ProfRec> prof_pending;
    std::vector<cudaEvent_t> ev_pool;
    dfb_prof_entry prof_acc[DFB_PROF_N]{};
    // generation
    bool gen_active = false;
    int total = 0;                   // positions of all segments
    int n_seg = 0;
    std::vector<int> seg_off_h;      // [n_seg + 1]
    std::vector<int> seg_prompt, seg_gen, seg_masked;  // per segment, host copies
    dfb_sampler_params sp{};
};

static void ctx_free_buffers(dfb_ctx *c) {
    void *ps[] = {c->x, c->y, c->logits, c->h, c->att, c->q, c->ffh, c->kc, c->vc, c->rope, c->seq, c->prev_seq,
                  c->last_changed, c->cand_tok, c->commit_pos, c->commit_tok, c->order, c->masked, c->active_pos,
                  c->masked_pos, c->cnt, c->cand_conf, c->cand_ent, c->ws, c->tile_cnt, c->err, c->seg_off,
                  c->seg_cnt, c->sched, c->tmp_active, c->tmp_masked, c->rope_pos, c->masked_row, c->done, c->tiles,
                  c->unif, c->tp_stats, c->tp_gath, c->tp_g};
    for (void *p : ps) cudaFree(p);
    c->seg_off = c->seg_cnt = c->sched = c->tmp_active = c->tmp_masked = c->rope_pos = c->masked_row = nullptr;
    c->done = nullptr;
    c->tiles = nullptr;
    c->x = c->y = c->logits = c->q = c->kc = c->vc = nullptr; c->h = c->att = c->ffh = nullptr; c->rope = nullptr;
    c->unif = nullptr;
    c->tp_stats = c->tp_gath = nullptr;
    c->tp_g = nullptr;
    c->seq = c->prev_seq = c->last_changed = c->cand_tok = c->commit_pos = c->commit_tok = c->order = nullptr;
    c->masked = nullptr; c->active_pos = c->masked_pos = c->cnt = nullptr; c->cand_conf = c->cand_ent = nullptr;
    c->ws = nullptr; c->tile_cnt = c->err = nullptr;
    c->cap = 0;
}

// RoPE angles exactly as the reference's GGML NEOX path computes them: theta starts
// at the position and is multiplied by base^(-2/n_dims) once per pair, in float
// (ggml_rope_cache_init, with the arguments of diffuse-graph.cpp:76-79).
static void rope_table_host(int n_pos, int hd, float base, std::vector<float2> &out) {
    out.resize((size_t)n_pos * (hd / 2));
    const float theta_scale = powf(base, -2.0f / hd);
    for (int p = 0; p < n_pos; p++) {
        float theta = (float)p;
        for (int i = 0; i < hd / 2; i++) {
            out[(size_t)p * (hd / 2) + i] = make_float2(cosf(theta), sinf(theta));
            theta *= theta_scale;
        }
    }
}

static int ctx_reserve(dfb_ctx *c, int n) {
    if (n <= c->cap) return DFB_OK;
    const dfb_model *m = c->m;
    const dfb_hparams &hp = m->hp;
    const int cap = std::max(n, 64);
    ctx_free_buffers(c);
    // per-rank widths: FFN features and vocabulary rows of this rank (all of them at tp_size 1)
    const size_t d = hp.n_embd, ff = m->n_ff_l, V = m->n_vocab_l, L = hp.n_layer, kvd = m->n_kv, hd = m->hd;
#define AL(ptr, count) CK(cudaMalloc(&(ptr), sizeof(*(ptr)) * (size_t)(count)))
    AL(c->x, cap * d); AL(c->y, cap * d); AL(c->h, 4 * cap * d); AL(c->att, 4 * cap * d); AL(c->q, cap * d);
    AL(c->ffh, 4 * cap * ff);
    AL(c->kc, L * cap * kvd); AL(c->vc, L * cap * kvd); AL(c->logits, (size_t)cap * V); AL(c->rope, cap * hd / 2);
    AL(c->seq, cap); AL(c->prev_seq, cap); AL(c->last_changed, cap); AL(c->cand_tok, cap); AL(c->commit_pos, cap);
    AL(c->commit_tok, cap); AL(c->order, cap); AL(c->masked, cap); AL(c->active_pos, cap); AL(c->masked_pos, cap);
    AL(c->cnt, CNT_N); AL(c->cand_conf, cap); AL(c->cand_ent, cap); AL(c->unif, cap);
    if (m->tp_size > 1) { AL(c->tp_stats, cap); AL(c->tp_gath, (size_t)cap * m->tp_size); AL(c->tp_g, cap); }
    AL(c->seg_off, kMaxSeg + 1); AL(c->seg_cnt, kMaxSeg * SEG_N); AL(c->sched, kMaxSeg); AL(c->done, kMaxSeg);
    AL(c->tmp_active, cap); AL(c->tmp_masked, cap); AL(c->rope_pos, cap); AL(c->masked_row, cap);
    AL(c->tiles, cap / kAttnRows + kMaxSeg + 1);
    AL(c->ws, (size_t)m->n_sm * 2 * kWsTile); AL(c->err, 1);
    const int n_mg_max = (cap + kMaxTok - 1) / kMaxTok;
    int max_tiles = m->lm_head.n_tiles;
    for (auto &Lw : m->layers) max_tiles = std::max({max_tiles, Lw.qkv.n_tiles, Lw.gateup.n_tiles, Lw.o.n_tiles, Lw.down.n_tiles});
    c->n_tile_cnt = max_tiles * n_mg_max;
    AL(c->tile_cnt, c->n_tile_cnt);
#undef AL
    CK(cudaMemset(c->tile_cnt, 0, sizeof(int) * c->n_tile_cnt));
    CK(cudaMemset(c->err, 0, sizeof(int)));
    CK(cudaMemset(c->cnt, 0, sizeof(int) * CNT_N));
    CK(cudaMemset(c->seg_cnt, 0, sizeof(int) * kMaxSeg * SEG_N));
    CK(cudaMemset(c->x, 0, sizeof(float) * cap * d));
    CK(cudaMemset(c->y, 0, sizeof(float) * cap * d));
    CK(cudaMemset(c->h, 0, 4 * cap * d));
    CK(cudaMemset(c->att, 0, 4 * cap * d));
    CK(cudaMemset(c->ffh, 0, 4 * cap * ff));
    CK(cudaMemset(c->kc, 0, 4 * L * cap * kvd));
    CK(cudaMemset(c->vc, 0, 4 * L * cap * kvd));
    std::vector<float2> rope;
    rope_table_host(cap, (int)hd, hp.rope_theta, rope);
    CK(cudaMemcpy(c->rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));
    RET(make_xmaps(&c->xm_h, c->h, (int)d, cap, 2));
    RET(make_xmaps(&c->xm_att, c->att, m->n_q, cap, 2));
    RET(make_xmaps(&c->xm_ffh, c->ffh, (int)ff, cap, 2));
    c->cap = cap;
    return DFB_OK;
}

static cudaEvent_t prof_event(dfb_ctx *c) {
    if (c->ev_pool.empty()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        return e;
    }
    cudaEvent_t e = c->ev_pool.back();
    c->ev_pool.pop_back();
    return e;
}
static void prof_begin(dfb_ctx *c, cudaEvent_t *a) {
    if (!c->prof) return;
    *a = prof_event(c);
    cudaEventRecord(*a, c->st);
}
static void prof_end(dfb_ctx *c, cudaEvent_t a, int cat, double flops_per_row, double bytes_fixed, double bytes_per_row) {
    if (!c->prof) return;
    cudaEvent_t b = prof_event(c);
    cudaEventRecord(b, c->st);
    c->prof_pending.push_back({a, b, cat, flops_per_row, bytes_fixed, bytes_per_row});
}
// After the stream is synchronized: fold the pending launches of a pass over M rows.
static void prof_collect(dfb_ctx *c, int M) {
    for (auto &r : c->prof_pending) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, r.a, r.b);
        for (int cat : {r.cat, r.cat < DFB_PROF_ATTN ? (int)DFB_PROF_GEMM_ALL : -1}) {
            if (cat < 0) continue;
            dfb_prof_entry &e = c->prof_acc[cat];
            e.calls += 1;
            e.ms += ms;
            e.flops += r.flops_per_row * M;
            e.bytes += r.bytes_fixed + r.bytes_per_row * M;
        }
        c->ev_pool.push_back(r.a);
        c->ev_pool.push_back(r.b);
    }
    c->prof_pending.clear();
}

// Programmatic dependent launch: a kernel launched this way may start while the
// previous kernel of the stream is finishing; every such kernel executes
// griddepcontrol.wait before it touches memory the previous kernels write.
// DIFFUSE_PDL=0 turns it off (plain stream order).
static bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("DIFFUSE_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                            Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// CTA pairs of a GEMM instantiation that fit on the device at once (one CTA per SM).
template <int WT, int EPI, int XS>
static int gemm_max_pairs(int device, int n_sm) {
    static int cached[64] = {0};
    if (device < 0 || device >= 64) return n_sm / 2;
    if (!cached[device]) {
        constexpr int smem = gemm_smem_bytes(WT, XS);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(n_sm & ~1);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, dq_gemm_kernel<WT, EPI, XS>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = n_sm / 2;
        }
        cached[device] = std::min(n, n_sm / 2);
    }
    return cached[device];
}

// Parameters of one launch of the dequant GEMM on weight w (scratch supplied by the caller).
static GemmParams gemm_params(const WMat &w, const int *m_dev, float *ws, int *tile_cnt, int *err, const EpiArgs &epi) {
    GemmParams p;
    p.w = w.d;
    p.K = w.K;
    p.n_tiles = w.n_tiles;
    p.kb = w.kb;
    p.wscale = w.wscale;
    p.lo_row = w.lo_row;
    p.corr_row = w.corr_row;
    p.m_dev = m_dev;
    p.ws = ws;
    p.tile_cnt = tile_cnt;
    p.err = err;
    p.epi = epi;
    p.epi.out_scale = 1.0f / w.wscale;  // a power of two: exact
    return p;
}

template <int WT, int EPI>
static int launch_gemm_t(dfb_ctx *c, const WMat &w, const XMaps &xm, const EpiArgs &epi) {
    auto kern = dq_gemm_kernel<WT, EPI, 2>;
    constexpr int smem = gemm_smem_bytes(WT, 2);
    static bool attr_set[64] = {false};
    const int dev = c->m->device;
    if (!attr_set[dev]) {
        CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[dev] = true;
    }
    GemmParams p = gemm_params(w, c->cnt + CNT_M, c->ws, c->tile_cnt, c->err, epi);
    if (c->stall_next) {
        // a split tile's contributors wait for arrivals that cannot reach this count
        static const int kPoison = -(1 << 30);
        CK(cudaMemcpyAsync(c->tile_cnt, &kPoison, sizeof(int), cudaMemcpyHostToDevice, c->st));
        p.timeout_ns = c->stall_timeout_ns;
        c->stall_next = false;
    }
    cudaEvent_t ev0 = nullptr;
    prof_begin(c, &ev0);
    // A pair tile is split over at most n_pairs/n_ptiles + 2 pairs; keep that within kMaxContrib.
    const int n_pairs = std::min(gemm_max_pairs<WT, EPI, 2>(c->m->device, c->m->n_sm), (kMaxContrib - 2) * (w.n_tiles / 2));
    // the device schedule multiplies unit indices by the pair count in 32 bits
    if ((double)(w.n_tiles / 2) * ((c->cap + kMaxTok - 1) / kMaxTok) * w.kb * (n_pairs + 1) >= 4294967296.0)
        return set_err(DFB_ERR_UNSUPPORTED, "GEMM schedule too large for %d rows", c->cap);
    CK(launch_k(kern, dim3(2 * n_pairs), dim3(kThreads), smem, c->st, !c->prof, w.tm, xm, p));
    // algorithmic work: 2*K MACs per output, weights read once, X read (pair rows, 4 B per
    // value), Y written (f32, or pair rows for SwiGLU: 4 B per output feature either way)
    const int cat = WT == W_Q4K ? DFB_PROF_Q4K : WT == W_Q6K ? DFB_PROF_Q6K : WT == W_Q80 ? DFB_PROF_Q80 : DFB_PROF_F16;
    prof_end(c, ev0, EPI == EPI_LOGITS ? (int)DFB_PROF_LMHEAD : cat, 2.0 * w.K * (double)w.n_true, (double)w.bytes,
             4.0 * w.K + 4.0 * (EPI == EPI_SWIGLU ? w.n_true / 2 : w.n_true));
    return DFB_OK;
}

template <int EPI>
static int launch_gemm(dfb_ctx *c, const WMat &w, const XMaps &xm, const EpiArgs &epi) {
    switch (w.wt) {
        case W_Q4K: return launch_gemm_t<W_Q4K, EPI>(c, w, xm, epi);
        case W_Q6K: return launch_gemm_t<W_Q6K, EPI>(c, w, xm, epi);
        case W_Q80: return launch_gemm_t<W_Q80, EPI>(c, w, xm, epi);
        case W_F16: return launch_gemm_t<W_F16, EPI>(c, w, xm, epi);
        case W_F32: return launch_gemm_t<W_F32, EPI>(c, w, xm, epi);
    }
    return set_err(DFB_ERR_STATE, "weight not uploaded");
}

template <int HD>
// n_keys: keys per query row (the sequences' length; for the profile's accounting only).
static int launch_attn_t(dfb_ctx *c, const float *kc, const float *vc, int n_keys) {
    const dfb_model *m = c->m;
    constexpr int smem = attn_smem_bytes<HD>();
    static bool attr_set[64] = {false};
    if (!attr_set[m->device]) {
        CK(cudaFuncSetAttribute(attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[m->device] = true;
    }
    const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
    // work-list bound: tiles of <= 32 active rows of one sequence each
    dim3 grid(c->cap / kAttnRows + std::max(c->n_seg, 1) + 1, m->n_head_l);  // this rank's heads
    cudaEvent_t ev0 = nullptr;
    prof_begin(c, &ev0);
    CK(launch_k(attn_kernel<HD>, grid, dim3(kAttnThreads), smem, c->st, !c->prof, (const float *)c->q, m->n_q, kc, vc,
                m->n_kv, c->att, 4 * m->n_q, (const int4 *)c->tiles,
                (const int *)(c->cnt + CNT_NTILES),
                m->hp.n_head / m->hp.n_head_kv, scale_log2));
    // algorithmic bytes: K and V of every key once (f32), Q in (f32), O out (pair rows)
    prof_end(c, ev0, DFB_PROF_ATTN, 4.0 * n_keys * m->n_head_l * HD, 2.0 * 4.0 * n_keys * m->n_kv, 8.0 * m->n_q);
    return DFB_OK;
}

// Tensor parallelism: the O and down projections are row-parallel (each rank holds the input
// columns of its heads / FFN features), so y holds partial sums; an NCCL all-reduce over the
// context's rows makes it the whole projection on every rank before the RMSNorm that adds it
// into the (replicated) residual stream (the split of diffuse-graph.cpp:122-123, 140-142).
// All rows of the buffer are reduced: the active-row count lives on the device.
static int tp_sum_rows(dfb_ctx *c) {
    const dfb_model *m = c->m;
    if (m->tp_size == 1) return DFB_OK;
    NK(nccl_api().all_reduce(c->y, c->y, (size_t)c->cap * m->hp.n_embd, ncclFloat32, ncclSum, m->comm, c->st));
    return DFB_OK;
}

// The value checks of the forward and the sampler (cnt[CNT_ERR]): a token id outside the
// vocabulary reached the embedding (1), or a logits row had no finite maximum (2).  Reported
// once and cleared; the kernels read a valid row instead, so nothing faults.
static int check_values(dfb_ctx *c, int code) {
    if (!code) return DFB_OK;
    CK(cudaMemsetAsync(c->cnt + CNT_ERR, 0, sizeof(int), c->st));
    CK(cudaStreamSynchronize(c->st));
    return set_err(DFB_ERR_STATE, code == 1 ? "a token id outside the vocabulary reached the embedding"
                                            : "a logits row has no finite maximum (non-finite logits)");
}

// The forward of one step over the active rows listed by step_prepare.
static int run_forward(dfb_ctx *c, int n_total) {
    const dfb_model *m = c->m;
    const dfb_hparams &hp = m->hp;
    const int d = hp.n_embd, cap = c->cap;
    if (m->embd_f16)
        embed_kernel<__half><<<cap, 256, 0, c->st>>>((const __half *)m->embd, d, hp.n_vocab, c->seq, c->active_pos, c->cnt, c->x);
    else
        embed_kernel<float><<<cap, 256, 0, c->st>>>((const float *)m->embd, d, hp.n_vocab, c->seq, c->active_pos, c->cnt, c->x);
    CK(cudaGetLastError());
    for (int l = 0; l < hp.n_layer; l++) {
        const LayerW &L = m->layers[l];
        float *kc = c->kc + (size_t)l * cap * m->n_kv, *vc = c->vc + (size_t)l * cap * m->n_kv;
        // the previous layer's down projection is added to the residual stream here
        CK(launch_k(rmsnorm_kernel, dim3(cap), dim3(256), 0, c->st, true, c->x, (const float *)(l ? c->y : nullptr),
                    (const float *)L.attn_norm, d, hp.rms_norm_eps, (const int *)c->cnt, c->h));
        EpiArgs e;
        e.q_out = c->q; e.ld_q = m->n_q;
        e.k_cache = kc; e.v_cache = vc; e.ld_kv = m->n_kv;
        e.n_q_tiles = m->nq_pad / 128; e.n_k_tiles = m->nk_pad / 128;
        e.n_q = m->n_q; e.n_kv = m->n_kv; e.head_dim = m->hd;
        e.bias = L.bias_qkv; e.rope = c->rope; e.pos = c->active_pos; e.rope_pos = c->rope_pos;
        RET(launch_gemm<EPI_QKV>(c, L.qkv, c->xm_h, e));
        switch (m->hd) {
            case 16: RET(launch_attn_t<16>(c, kc, vc, n_total)); break;
            case 32: RET(launch_attn_t<32>(c, kc, vc, n_total)); break;
            case 64: RET(launch_attn_t<64>(c, kc, vc, n_total)); break;
            default: RET(launch_attn_t<128>(c, kc, vc, n_total)); break;
        }
        EpiArgs eo;  // attention output projection -> y, added to x by the next norm
        eo.out = c->y; eo.ld = d; eo.n_valid = d;
        RET(launch_gemm<EPI_F32>(c, L.o, c->xm_att, eo));
        RET(tp_sum_rows(c));  // row-parallel O: the ranks' partial sums
        CK(launch_k(rmsnorm_kernel, dim3(cap), dim3(256), 0, c->st, true, c->x, (const float *)c->y,
                    (const float *)L.ffn_norm, d, hp.rms_norm_eps, (const int *)c->cnt, c->h));
        EpiArgs eg;
        eg.out = c->ffh; eg.ld = 2 * m->n_ff_l; eg.n_valid = 2 * m->n_ff_l;  // pair rows
        RET(launch_gemm<EPI_SWIGLU>(c, L.gateup, c->xm_h, eg));
        EpiArgs ed;  // FFN down projection -> y, added to x by the next norm
        ed.out = c->y; ed.ld = d; ed.n_valid = d;
        RET(launch_gemm<EPI_F32>(c, L.down, c->xm_ffh, ed));
        RET(tp_sum_rows(c));  // row-parallel down
    }
    CK(launch_k(rmsnorm_kernel, dim3(cap), dim3(256), 0, c->st, true, c->x, (const float *)(hp.n_layer ? c->y : nullptr),
                (const float *)m->output_norm, d, hp.rms_norm_eps, (const int *)c->cnt, c->h));
    EpiArgs el;
    el.out = c->logits; el.ld = m->n_vocab_l; el.n_valid = m->n_vocab_l; el.pos = c->active_pos;
    RET(launch_gemm<EPI_LOGITS>(c, m->lm_head, c->xm_h, el));
    CK(cudaGetLastError());
    return DFB_OK;
}

// What a GEMM error code (the first code any CTA raised) means: which bounded wait gave up,
// or which consistency check failed.
static const char *gemm_err_str(int code) {
    switch (code - kErrTimeout) {
        case 1: return "weight producer waited for a free weight stage";
        case 2: return "activation producer waited for a free activation slot";
        case 3: return "MMA issuer waited for a drained accumulator";
        case 4: return "relay waited for activations to land";
        case 5: return "MMA issuer waited for a dequantized A stage";
        case 6: return "dequantizer waited for a weight chunk to land";
        case 7: return "dequantizer waited for a free A stage";
        case 8: return "epilogue waited for a finished accumulator";
        case 9: return "a split tile has more contributors than tracked";
        case 10: return "epilogue waited for staged partial sums";
        case 11: return "F16 weight producer waited for a free A stage";
        case 12: return "relay waited for an MMA to release its stage";
        case 13: return "split-tile contributor waited for the other contributors' partial sums";
        case 14: return "token count changed between the launch and the grid-dependency wait";
        default: return "unknown";
    }
}

// One entry point's GPU work at a time per device.  A dequant GEMM launch relies on all of
// its CTAs being resident together (split-tile contributors wait for each other), which
// holds when its launches follow each other in one stream, but not when two host threads
// interleave GEMM launches of two contexts on one device (both launches could end up
// partly resident and stall until their bounded waits fail).  Every entry point below that
// launches a GEMM synchronizes its stream before returning, so holding this lock for the
// call serializes the GEMMs of all contexts of the device.
static std::mutex g_device_mu[64];
static std::mutex &device_lock(int device) { return g_device_mu[device & 63]; }

static int check_err(dfb_ctx *c) {
    int e = 0;
    CK(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        cudaMemset(c->err, 0, sizeof(int));
        cudaMemset(c->tile_cnt, 0, sizeof(int) * c->n_tile_cnt);  // an aborted launch can leave counts behind
        return set_err(DFB_ERR_TIMEOUT, "a GEMM stopped (code 0x%x: %s); results of this call are invalid", e,
                       gemm_err_str(e));
    }
    return DFB_OK;
}

extern "C" int dfb_ctx_create(dfb_model *m, int n_ctx, dfb_ctx **out) {
    if (!m || !out) return set_err(DFB_ERR_ARG, "null pointer");
    if (!m->finalized) return set_err(DFB_ERR_STATE, "model not finalized");
    *out = nullptr;
    CK(cudaSetDevice(m->device));
    auto *c = new dfb_ctx();
    c->m = m;
    if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return set_err(DFB_ERR_CUDA, "cudaStreamCreate failed");
    }
    for (auto &e : c->ev) cudaEventCreate(&e);
    if (n_ctx > 0) {
        const int r = ctx_reserve(c, n_ctx);
        if (r != DFB_OK) { dfb_ctx_free(c); return r; }
    }
    *out = c;
    return DFB_OK;
}

extern "C" void dfb_ctx_free(dfb_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->m->device);
    if (c->st) cudaStreamSynchronize(c->st);
    ctx_free_buffers(c);
    for (auto &e : c->ev) if (e) cudaEventDestroy(e);
    for (auto &r : c->prof_pending) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    for (auto e : c->ev_pool) cudaEventDestroy(e);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

extern "C" int dfb_ctx_profile(dfb_ctx *c, int enable) {
    if (!c) return set_err(DFB_ERR_ARG, "null context");
    CK(cudaStreamSynchronize(c->st));
    prof_collect(c, 0);
    c->prof = enable != 0;
    for (auto &e : c->prof_acc) e = dfb_prof_entry{};
    return DFB_OK;
}

extern "C" int dfb_ctx_profile_read(dfb_ctx *c, dfb_prof_entry *out, int n) {
    if (!c || !out) return set_err(DFB_ERR_ARG, "null pointer");
    for (int i = 0; i < n && i < DFB_PROF_N; i++) out[i] = c->prof_acc[i];
    return DFB_OK;
}

extern "C" int dfb_ctx_stream(dfb_ctx *c, void **stream) {
    if (!c || !stream) return set_err(DFB_ERR_ARG, "null pointer");
    *stream = c->st;
    return DFB_OK;
}

// Segment layout of the context's state: offsets [n_seg + 1] and finished flags (all 0).
static int set_segments(dfb_ctx *c, const std::vector<int> &off) {
    const int n = (int)off.size() - 1;
    CK(cudaMemcpyAsync(c->seg_off, off.data(), sizeof(int) * off.size(), cudaMemcpyHostToDevice, c->st));
    CK(cudaMemsetAsync(c->done, 0, n, c->st));
    c->n_seg = n;
    c->seg_off_h = off;
    c->total = off.back();
    return DFB_OK;
}

// Active sets and work lists of one step over all segments (seg_prepare + seg_compact).
static int prepare_step(dfb_ctx *c, int full, int step, int keep_active) {
    seg_prepare_kernel<<<c->n_seg, 1024, 0, c->st>>>(full, step, keep_active, c->seg_off, c->done, c->seq, c->prev_seq,
                                                      c->last_changed, c->masked, c->tmp_active, c->tmp_masked,
                                                      c->seg_cnt);
    CK(cudaGetLastError());
    CK(launch_k(seg_compact_kernel, dim3(1), dim3(1024), 0, c->st, false, c->n_seg, (const int *)c->seg_off,
                (const int *)c->tmp_active, (const int *)c->tmp_masked, c->seg_cnt, c->m->hp.shift_logits, c->active_pos,
                c->rope_pos, c->masked_pos, c->masked_row, c->tiles, c->cnt));
    return DFB_OK;
}

extern "C" int dfb_forward(dfb_ctx *c, const int32_t *tokens, int n, float *logits_host) {
    if (!c || !tokens || !logits_host || n <= 0) return set_err(DFB_ERR_ARG, "bad arguments");
    std::lock_guard<std::mutex> lk(device_lock(c->m->device));
    CK(cudaSetDevice(c->m->device));
    const int V = c->m->hp.n_vocab;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= V) return set_err(DFB_ERR_ARG, "token %d at %d outside [0, %d)", tokens[i], i, V);
    RET(ctx_reserve(c, n));
    c->gen_active = false;
    RET(set_segments(c, {0, n}));
    CK(cudaMemcpyAsync(c->seq, tokens, n * sizeof(int32_t), cudaMemcpyHostToDevice, c->st));
    CK(cudaMemsetAsync(c->masked, 0, n, c->st));
    RET(prepare_step(c, 1, 0, 0));
    RET(run_forward(c, n));
    // (tensor parallelism: this rank's vocabulary columns, n x n_vocab_local)
    CK(cudaMemcpyAsync(logits_host, c->logits, (size_t)n * c->m->n_vocab_l * sizeof(float), cudaMemcpyDeviceToHost, c->st));
    int verr = 0;
    CK(cudaMemcpyAsync(&verr, c->cnt + CNT_ERR, sizeof(int), cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    RET(check_values(c, verr));
    prof_collect(c, n);
    return check_err(c);
}

extern "C" int dfb_linear(dfb_ctx *c, int role, int layer, const float *x_host, int M, float *y_host) {
    if (!c || !x_host || !y_host || M <= 0) return set_err(DFB_ERR_ARG, "bad arguments");
    const dfb_model *m = c->m;
    if (m->tp_size > 1) return set_err(DFB_ERR_UNSUPPORTED, "dfb_linear on a tensor-parallel model");
    std::lock_guard<std::mutex> lk(device_lock(m->device));
    CK(cudaSetDevice(m->device));
    const WMat *w = nullptr;
    int K = 0, n_out = 0;
    const int d = m->hp.n_embd, ff = m->hp.n_ff;
    if (role == DFB_OUTPUT) { w = &m->lm_head; K = d; n_out = m->hp.n_vocab; }
    else {
        if (layer < 0 || layer >= m->hp.n_layer) return set_err(DFB_ERR_ARG, "bad layer");
        const LayerW &L = m->layers[layer];
        switch (role) {
            case DFB_WQ: w = &L.qkv; K = d; n_out = m->n_q; break;
            case DFB_WK: w = &L.qkv; K = d; n_out = m->n_kv; break;
            case DFB_WV: w = &L.qkv; K = d; n_out = m->n_kv; break;
            case DFB_WO: w = &L.o; K = m->n_q; n_out = d; break;
            case DFB_GATE: case DFB_UP: w = &L.gateup; K = d; n_out = ff; break;
            case DFB_DOWN: w = &L.down; K = ff; n_out = d; break;
            default: return set_err(DFB_ERR_ARG, "role %d is not a linear weight", role);
        }
    }
    RET(ctx_reserve(c, M));
    uint8_t *xh = nullptr;
    float *xf = nullptr, *y = nullptr;
    CK(cudaMalloc(&xh, (size_t)M * K * 4));  // pair rows
    CK(cudaMalloc(&xf, (size_t)M * K * 4));
    CK(cudaMalloc(&y, (size_t)M * w->n_rows * 4));
    int rc = DFB_OK;
    XMaps xm;
    do {
        if ((rc = make_xmaps(&xm, xh, K, M, 2)) != DFB_OK) break;
        if (cudaMemcpyAsync(xf, x_host, (size_t)M * K * 4, cudaMemcpyHostToDevice, c->st) != cudaSuccess) { rc = set_err(DFB_ERR_CUDA, "H2D failed"); break; }
        f32_to_pair_kernel<<<256, 256, 0, c->st>>>(xf, xh, M, K);
        if (cudaMemcpyAsync(c->cnt + CNT_M, &M, sizeof(int), cudaMemcpyHostToDevice, c->st) != cudaSuccess) { rc = set_err(DFB_ERR_CUDA, "H2D failed"); break; }
        EpiArgs e;
        e.out = y; e.ld = w->n_rows; e.n_valid = w->n_rows;
        if ((rc = launch_gemm<EPI_F32>(c, *w, xm, e)) != DFB_OK) break;
        std::vector<float> full((size_t)M * w->n_rows);
        if (cudaMemcpyAsync(full.data(), y, full.size() * 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess ||
            cudaStreamSynchronize(c->st) != cudaSuccess) { rc = set_err(DFB_ERR_CUDA, "GEMM failed: %s", cudaGetErrorString(cudaGetLastError())); break; }
        if ((rc = check_err(c)) != DFB_OK) break;
        // undo the fused-row layout
        const int hd = m->hd;
        for (int t = 0; t < M; t++)
            for (int f = 0; f < n_out; f++) {
                int r;
                switch (role) {
                    case DFB_WQ: case DFB_WK: {
                        const int head = f / hd, rr = f % hd, i = rr < hd / 2 ? rr : rr - hd / 2, b = rr < hd / 2 ? 0 : 1;
                        r = (role == DFB_WK ? m->nq_pad : 0) + head * hd + 2 * i + b;
                    } break;
                    case DFB_WV: r = m->nq_pad + m->nk_pad + f; break;
                    case DFB_GATE: r = 2 * f; break;
                    case DFB_UP: r = 2 * f + 1; break;
                    default: r = f;
                }
                y_host[(size_t)t * n_out + f] = full[(size_t)t * w->n_rows + r];
            }
    } while (0);
    cudaFree(xh); cudaFree(xf); cudaFree(y);
    return rc;
}

extern "C" int dfb_debug_stalled_linear(dfb_ctx *c, int role, int layer, const float *x_host, int M, float *y_host,
                                        unsigned long long timeout_ns) {
    if (!c) return set_err(DFB_ERR_ARG, "null context");
    if (timeout_ns == 0 || timeout_ns > 4000000000ull) return set_err(DFB_ERR_ARG, "timeout_ns outside (0, 4 s]");
    c->stall_next = true;
    c->stall_timeout_ns = timeout_ns;
    const int rc = dfb_linear(c, role, layer, x_host, M, y_host);
    c->stall_next = false;
    return rc;
}

extern "C" int dfb_gen_begin_batch(dfb_ctx *c, int n_seq, const int32_t *prompts, const int32_t *prompt_lens,
                                   const int32_t *n_gens, const dfb_sampler_params *p) {
    if (!c || !p || !prompt_lens || !n_gens || n_seq <= 0) return set_err(DFB_ERR_ARG, "bad arguments");
    if (n_seq > kMaxSeg) return set_err(DFB_ERR_ARG, "%d sequences > %d per context", n_seq, kMaxSeg);
    if (!std::isfinite(p->temperature)) return set_err(DFB_ERR_ARG, "temperature must be finite");
    if (p->temperature > 0.0f && c->m->tp_size > 1)
        return set_err(DFB_ERR_UNSUPPORTED, "temperature > 0 sampling on a tensor-parallel model");
    if (p->remasking < 0 || p->remasking > 4) return set_err(DFB_ERR_ARG, "bad remasking %d", p->remasking);
    const dfb_model *m = c->m;
    CK(cudaSetDevice(m->device));
    if (m->hp.mask_token_id < 0 || m->hp.mask_token_id >= m->hp.n_vocab)
        return set_err(DFB_ERR_ARG, "mask token id %d outside the vocabulary", m->hp.mask_token_id);
    std::vector<int> off(n_seq + 1, 0);
    size_t n_prompt_all = 0;
    for (int sg = 0; sg < n_seq; sg++) {
        if (prompt_lens[sg] < 0 || n_gens[sg] <= 0 || n_gens[sg] > 65536)
            return set_err(DFB_ERR_ARG, "sequence %d: prompt %d / n_generate %d out of range", sg, prompt_lens[sg], n_gens[sg]);
        off[sg + 1] = off[sg] + prompt_lens[sg] + n_gens[sg];
        n_prompt_all += prompt_lens[sg];
    }
    if (n_prompt_all > 0 && !prompts) return set_err(DFB_ERR_ARG, "null prompts");
    for (size_t i = 0; i < n_prompt_all; i++)
        if (prompts[i] < 0 || prompts[i] >= m->hp.n_vocab) return set_err(DFB_ERR_ARG, "prompt token %d out of range", prompts[i]);
    const int total = off.back();
    RET(ctx_reserve(c, total));
    // seq = prompt ‖ MASK x n_gen per sequence (diffuse-sampler.cpp:77-87), concatenated
    std::vector<int32_t> seq(total, m->hp.mask_token_id), neg(total, -1);
    std::vector<uint8_t> msk(total, 0);
    size_t pi = 0;
    for (int sg = 0; sg < n_seq; sg++) {
        std::copy(prompts + pi, prompts + pi + prompt_lens[sg], seq.begin() + off[sg]);
        pi += prompt_lens[sg];
        std::fill(msk.begin() + off[sg] + prompt_lens[sg], msk.begin() + off[sg + 1], 1);
    }
    RET(set_segments(c, off));
    CK(cudaMemcpyAsync(c->seq, seq.data(), total * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->prev_seq, neg.data(), total * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->last_changed, neg.data(), total * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->masked, msk.data(), total, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemsetAsync(c->cnt, 0, sizeof(int) * CNT_N, c->st));
    CK(cudaMemsetAsync(c->seg_cnt, 0, sizeof(int) * kMaxSeg * SEG_N, c->st));
    CK(cudaStreamSynchronize(c->st));
    c->seg_prompt.assign(prompt_lens, prompt_lens + n_seq);
    c->seg_gen.assign(n_gens, n_gens + n_seq);
    c->seg_masked.assign(n_gens, n_gens + n_seq);
    c->sp = *p;
    c->unif_n = -1;
    c->gen_active = true;
    return DFB_OK;
}

extern "C" int dfb_gen_set_uniforms(dfb_ctx *c, const double *u, int n) {
    if (!c || n < 0 || (n > 0 && !u)) return set_err(DFB_ERR_ARG, "bad arguments");
    if (!c->gen_active) return set_err(DFB_ERR_STATE, "dfb_gen_begin not called");
    if (n > c->cap) return set_err(DFB_ERR_ARG, "%d uniforms > %d positions", n, c->cap);
    for (int i = 0; i < n; i++)
        if (!(u[i] >= 0.0 && u[i] < 1.0)) return set_err(DFB_ERR_ARG, "uniform %d outside [0, 1)", i);
    CK(cudaSetDevice(c->m->device));
    if (n) CK(cudaMemcpyAsync(c->unif, u, sizeof(double) * n, cudaMemcpyHostToDevice, c->st));
    c->unif_n = n;
    return DFB_OK;
}

extern "C" int dfb_gen_begin(dfb_ctx *c, const int32_t *prompt, int n_prompt, int n_gen, const dfb_sampler_params *p) {
    if (n_prompt < 0 || (n_prompt > 0 && !prompt)) return set_err(DFB_ERR_ARG, "bad arguments");
    return dfb_gen_begin_batch(c, 1, prompt, &n_prompt, &n_gen, p);
}

extern "C" int dfb_gen_step_batch(dfb_ctx *c, int step, const int32_t *n_unmask_sched, int force_full,
                                  const int32_t *orders, dfb_step_stats *stats) {
    if (!c || !n_unmask_sched) return set_err(DFB_ERR_ARG, "null argument");
    if (!c->gen_active) return set_err(DFB_ERR_STATE, "dfb_gen_begin not called");
    const dfb_model *m = c->m;
    std::lock_guard<std::mutex> lk(device_lock(m->device));
    CK(cudaSetDevice(m->device));
    const int S = c->n_seg;
    // a sequence whose loop has ended (no position left masked) takes no part in the step
    std::vector<int32_t> sched(n_unmask_sched, n_unmask_sched + S);
    std::vector<uint8_t> done(S);
    int max_masked = 0, n_live = 0, masked_all = 0;
    for (int sg = 0; sg < S; sg++) {
        done[sg] = c->seg_masked[sg] == 0;
        if (done[sg]) sched[sg] = -1;
        else n_live++;
        max_masked = std::max(max_masked, c->seg_masked[sg]);
        masked_all += c->seg_masked[sg];
    }
    if (n_live == 0) return set_err(DFB_ERR_STATE, "every sequence is complete");
    const bool sampled = c->sp.temperature > 0.0f;
    if (sampled && c->unif_n != masked_all)
        return set_err(DFB_ERR_ARG, "temperature > 0: the step needs %d uniforms (dfb_gen_set_uniforms), %d set", masked_all,
                       c->unif_n);
    if (c->sp.remasking == 1) {
        if (!orders) return set_err(DFB_ERR_ARG, "RANDOM remasking needs the host shuffle orders");
        CK(cudaMemcpyAsync(c->order, orders, sizeof(int32_t) * masked_all, cudaMemcpyHostToDevice, c->st));
    }
    CK(cudaMemcpyAsync(c->sched, sched.data(), sizeof(int32_t) * S, cudaMemcpyHostToDevice, c->st));
    CK(cudaMemcpyAsync(c->done, done.data(), S, cudaMemcpyHostToDevice, c->st));
    CK(cudaEventRecord(c->ev[0], c->st));
    RET(prepare_step(c, force_full ? 1 : 0, step, c->sp.cache_keep_active));
    RET(run_forward(c, c->total / S));
    CK(cudaEventRecord(c->ev[1], c->st));
    const int margin = c->sp.remasking == 4 ? 1 : 0;
    if (m->tp_size == 1) {
        row_stats_kernel<<<masked_all, 512, 0, c->st>>>(c->logits, m->hp.n_vocab, c->masked_row, c->cnt, margin, c->cand_tok,
                                                        c->cand_conf, c->cand_ent);
        CK(cudaGetLastError());
    } else {
        // vocabulary-parallel rows: local statistics, one all-gather, the combination, the
        // entropy terms over local columns, one all-reduce (every rank then decides the same)
        tp_stats_kernel<<<masked_all, 512, 0, c->st>>>(c->logits, m->n_vocab_l, m->v0, c->masked_row, c->cnt, c->tp_stats);
        CK(cudaGetLastError());
        NK(nccl_api().all_gather(c->tp_stats, c->tp_gath, (size_t)masked_all * 4, ncclFloat32, m->comm, c->st));
        tp_combine_kernel<<<(masked_all + 255) / 256, 256, 0, c->st>>>(c->tp_gath, m->tp_size, masked_all, c->cnt, margin,
                                                                      c->cand_tok, c->cand_conf, c->tp_g);
        tp_entropy_kernel<<<masked_all, 512, 0, c->st>>>(c->logits, m->n_vocab_l, c->masked_row, c->cnt, c->tp_g, c->cand_ent);
        CK(cudaGetLastError());
        NK(nccl_api().all_reduce(c->cand_ent, c->cand_ent, (size_t)masked_all, ncclFloat32, ncclSum, m->comm, c->st));
    }
    if (sampled) {  // draw the candidates' tokens; the entropy stays row_stats'
        sample_kernel<<<masked_all, kSampleThreads, 0, c->st>>>(c->logits, m->hp.n_vocab, c->masked_row, c->cnt,
                                                                 c->sp.temperature, c->unif, c->cand_tok, c->cand_conf);
        CK(cudaGetLastError());
        c->unif_n = -1;
    }
    int np = 1;
    while (np < max_masked) np <<= 1;
    const size_t sel_smem = sizeof(unsigned long long) * (size_t)np;
    if (sel_smem > 48 * 1024) CK(cudaFuncSetAttribute(select_commit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel_smem));
    select_commit_kernel<<<S, 1024, sel_smem, c->st>>>(c->sp.remasking, c->sched, c->sp.entropy_threshold, np, c->order,
                                                       c->masked_pos, c->cand_tok, c->cand_conf, c->cand_ent, c->seq,
                                                       c->masked, c->commit_pos, c->commit_tok, c->seg_cnt);
    CK(cudaGetLastError());
    CK(cudaEventRecord(c->ev[2], c->st));
    int h_cnt[CNT_N];
    std::vector<int> h_seg((size_t)S * SEG_N);
    CK(cudaMemcpyAsync(h_cnt, c->cnt, sizeof(h_cnt), cudaMemcpyDeviceToHost, c->st));
    CK(cudaMemcpyAsync(h_seg.data(), c->seg_cnt, sizeof(int) * h_seg.size(), cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    prof_collect(c, h_cnt[CNT_M]);
    RET(check_err(c));
    RET(check_values(c, h_cnt[CNT_ERR]));
    float fwd = 0, all = 0;
    cudaEventElapsedTime(&fwd, c->ev[0], c->ev[1]);
    cudaEventElapsedTime(&all, c->ev[0], c->ev[2]);
    for (int sg = 0; sg < S; sg++) {
        const int *hs = &h_seg[(size_t)sg * SEG_N];
        if (hs[SEG_ERR]) return set_err(DFB_ERR_STATE, "sequence %d: device and host disagree on the masked count", sg);
        if (!done[sg] && hs[SEG_NMASK] != c->seg_masked[sg] - hs[SEG_COMMITTED])
            return set_err(DFB_ERR_STATE, "sequence %d: masked count out of step", sg);
        c->seg_masked[sg] = done[sg] ? 0 : hs[SEG_NMASK];
        if (stats) {
            stats[sg].n_active = hs[SEG_NACT];
            stats[sg].n_unmasked = hs[SEG_COMMITTED];
            stats[sg].n_masked = c->seg_masked[sg];
            stats[sg].used_cache = hs[SEG_USED_CACHE];
            stats[sg].fwd_ms = fwd;
            stats[sg].step_ms = all;
        }
    }
    return DFB_OK;
}

extern "C" int dfb_gen_step(dfb_ctx *c, int step, int n_unmask_sched, int force_full, const int32_t *order,
                            dfb_step_stats *stats) {
    if (!c) return set_err(DFB_ERR_ARG, "null context");
    if (c->gen_active && c->n_seg != 1) return set_err(DFB_ERR_STATE, "batch generation: use dfb_gen_step_batch");
    return dfb_gen_step_batch(c, step, &n_unmask_sched, force_full, order, stats);
}

extern "C" int dfb_gen_tokens(dfb_ctx *c, int32_t *seq_host, int cap) {
    if (!c || !seq_host) return set_err(DFB_ERR_ARG, "null pointer");
    if (!c->gen_active) return set_err(DFB_ERR_STATE, "no generation");
    if (cap < c->total) return set_err(DFB_ERR_ARG, "buffer of %d < %d positions", cap, c->total);
    CK(cudaMemcpyAsync(seq_host, c->seq, c->total * 4, cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    return DFB_OK;
}

extern "C" int dfb_gen_commits_batch(dfb_ctx *c, int32_t *pos_host, int32_t *tok_host, int32_t *counts, int cap) {
    if (!c || !pos_host || !tok_host || !counts) return set_err(DFB_ERR_ARG, "null pointer");
    if (!c->gen_active) return set_err(DFB_ERR_STATE, "no generation");
    const int S = c->n_seg;
    std::vector<int> h_seg((size_t)S * SEG_N);
    CK(cudaMemcpyAsync(h_seg.data(), c->seg_cnt, sizeof(int) * h_seg.size(), cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    int w = 0;
    for (int sg = 0; sg < S; sg++) {
        const int n = h_seg[(size_t)sg * SEG_N + SEG_COMMITTED], off = h_seg[(size_t)sg * SEG_N + SEG_MOFF];
        if (w + n > cap) return set_err(DFB_ERR_ARG, "buffer of %d commits too small", cap);
        counts[sg] = n;
        if (n) {
            CK(cudaMemcpyAsync(pos_host + w, c->commit_pos + off, n * 4, cudaMemcpyDeviceToHost, c->st));
            CK(cudaMemcpyAsync(tok_host + w, c->commit_tok + off, n * 4, cudaMemcpyDeviceToHost, c->st));
        }
        w += n;
    }
    CK(cudaStreamSynchronize(c->st));
    return w;
}

extern "C" int dfb_gen_commits(dfb_ctx *c, int32_t *pos_host, int32_t *tok_host, int cap) {
    if (!c) return set_err(DFB_ERR_ARG, "null context");
    if (c->gen_active && c->n_seg != 1) return set_err(DFB_ERR_STATE, "batch generation: use dfb_gen_commits_batch");
    int32_t count = 0;
    return dfb_gen_commits_batch(c, pos_host, tok_host, &count, cap);
}

extern "C" int dfb_gen_logits(dfb_ctx *c, int row0, int nrows, float *host) {
    if (!c || !host || row0 < 0 || nrows <= 0 || row0 + nrows > c->cap) return set_err(DFB_ERR_ARG, "bad arguments");
    const size_t V = c->m->n_vocab_l;  // (tensor parallelism: this rank's vocabulary columns)
    CK(cudaMemcpyAsync(host, c->logits + (size_t)row0 * V, (size_t)nrows * V * 4, cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    return DFB_OK;
}

// ───────────────────────── allocation-free linear ─────────────────────────
// Some callers must not allocate device memory while they run: serving stacks that
// hand every byte of the GPU to their own caching allocator up front, and callers that
// cannot afford the device-wide synchronization cudaMalloc / cudaFree may imply in the
// middle of their work.  dfb_linear_noalloc serves them: the only scratch the dequant
// GEMM needs (split-tile partial sums and arrival counters) lives in the fixed arrays
// below, compiled into this library.  Every GPU that loads the library holds them
// (8 MiB + 8 KiB) until the process exits.
namespace {
constexpr int kNoallocGrid = 32;                      // CTAs per launch (bounds the scratch)
constexpr int kNoallocMaxTokens = 256;                // one token group
constexpr int kNoallocMaxGroups = (kNoallocMaxTokens + kMaxTok - 1) / kMaxTok;
constexpr int kNoallocMaxTiles = 2040;                // 128-row output tiles (lm_head of 261k vocab)
constexpr int kCntM = kNoallocMaxGroups * kNoallocMaxTiles;  // [groups x tiles] counters, then M, then the error flag
constexpr int kNoallocCnt = kCntM + 8;
static __device__ __align__(256) float g_noalloc_ws[(size_t)kNoallocGrid * 2 * kWsTile];
static __device__ __align__(256) int g_noalloc_cnt[kNoallocCnt];

struct NoallocDev {
    float *ws = nullptr;
    int *cnt = nullptr;
};
NoallocDev g_noalloc_dev[64];
std::mutex g_noalloc_mu;

// Zeroes the counters the launch will use and the error flag, stores M.
__global__ void noalloc_prep_kernel(int *cnt, int n_tiles, int M) {
    for (int i = threadIdx.x; i < kNoallocMaxGroups * n_tiles; i += blockDim.x) cnt[i] = 0;
    if (threadIdx.x == 0) {
        cnt[kCntM] = M;
        cnt[kCntM + 1] = 0;
    }
}

template <int WT>
int noalloc_launch(const WMat &w, const XMaps &xm, const EpiArgs &e, const NoallocDev &nd, int device, cudaStream_t st) {
    // the caller's x is a plain f16 matrix: one activation part (W_hi.x + W_lo.x)
    auto kern = dq_gemm_kernel<WT, EPI_F32, 1>;
    constexpr int smem = gemm_smem_bytes(WT, 1);
    static bool attr_set[64] = {false};  // once per device (the caller holds the device lock)
    if (!attr_set[device & 63]) {
        CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr_set[device & 63] = true;
    }
    const GemmParams p = gemm_params(w, nd.cnt + kCntM, nd.ws, nd.cnt, nd.cnt + kCntM + 1, e);
    const int n_pairs = std::min(kNoallocGrid / 2, (kMaxContrib - 2) * (w.n_tiles / 2));
    CK(launch_k(kern, dim3(2 * n_pairs), dim3(kThreads), smem, st, false, w.tm, xm, p));
    return DFB_OK;
}
}  // namespace

extern "C" int dfb_linear_noalloc(const dfb_model *m, int role, int layer, const void *x_f16_dev, int M,
                                  float *y_dev, void *stream) {
    if (!m || !x_f16_dev || !y_dev) return set_err(DFB_ERR_ARG, "null pointer");
    if (!m->finalized) return set_err(DFB_ERR_STATE, "model not finalized");
    if (reinterpret_cast<uintptr_t>(x_f16_dev) % 16)  // rows are read as 16-byte copies
        return set_err(DFB_ERR_ARG, "dfb_linear_noalloc: x must be 16-byte aligned");
    if (M <= 0 || M > kNoallocMaxTokens)
        return set_err(DFB_ERR_ARG, "dfb_linear_noalloc: M = %d outside [1, %d] (fixed scratch size)", M,
                       kNoallocMaxTokens);
    const WMat *w = nullptr;
    int K = 0;
    if (role == DFB_OUTPUT) { w = &m->lm_head; K = m->hp.n_embd; }
    else if (role == DFB_WO || role == DFB_DOWN) {
        if (layer < 0 || layer >= m->hp.n_layer) return set_err(DFB_ERR_ARG, "bad layer %d", layer);
        w = role == DFB_WO ? &m->layers[layer].o : &m->layers[layer].down;
        K = role == DFB_WO ? m->n_q : m->hp.n_ff;
    } else {
        return set_err(DFB_ERR_UNSUPPORTED, "dfb_linear_noalloc serves the unfused weights (attn_output, ffn_down, output)");
    }
    if (w->n_tiles > kNoallocMaxTiles)
        return set_err(DFB_ERR_ARG, "weight has %d output tiles, the fixed scratch holds %d", w->n_tiles, kNoallocMaxTiles);
    XMaps xm;  // host-side descriptors of the caller's matrix (no device memory)
    RET(make_xmaps(&xm, x_f16_dev, K, M, 1));
    std::lock_guard<std::mutex> lk(device_lock(m->device));
    CK(cudaSetDevice(m->device));
    NoallocDev nd;
    {
        // first call on this device: resolve the device addresses of the static arrays
        // (the host-side names are only stand-ins)
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        NoallocDev &d = g_noalloc_dev[m->device];
        if (!d.ws) {
            void *a = nullptr, *b = nullptr;
            CK(cudaGetSymbolAddress(&a, g_noalloc_ws));
            CK(cudaGetSymbolAddress(&b, g_noalloc_cnt));
            d.ws = static_cast<float *>(a);
            d.cnt = static_cast<int *>(b);
        }
        nd = d;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    noalloc_prep_kernel<<<1, 256, 0, st>>>(nd.cnt, w->n_tiles, M);
    CK(cudaGetLastError());
    EpiArgs e;
    e.out = y_dev;
    e.ld = w->n_true;
    e.n_valid = w->n_true;
    switch (w->wt) {
        case W_Q4K: RET(noalloc_launch<W_Q4K>(*w, xm, e, nd, m->device, st)); break;
        case W_Q6K: RET(noalloc_launch<W_Q6K>(*w, xm, e, nd, m->device, st)); break;
        case W_Q80: RET(noalloc_launch<W_Q80>(*w, xm, e, nd, m->device, st)); break;
        case W_F16: RET(noalloc_launch<W_F16>(*w, xm, e, nd, m->device, st)); break;
        case W_F32: RET(noalloc_launch<W_F32>(*w, xm, e, nd, m->device, st)); break;
        default: return set_err(DFB_ERR_STATE, "weight not uploaded");
    }
    CK(cudaStreamSynchronize(st));
    int err = 0;
    CK(cudaMemcpy(&err, nd.cnt + kCntM + 1, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) return set_err(DFB_ERR_TIMEOUT, "a GEMM stopped (code 0x%x: %s)", err, gemm_err_str(err));
    return DFB_OK;
}
