// Dequant-fused tcgen05 GEMM:  Y[tok][n] = sum_k X[tok][k] * W[n][k]
//
// Replaces every ggml_mul_mat(W, x) of the reference forward (src/diffuse-graph.cpp
// :61-63, 122, 136-140, 154 and the cached variants :451-453, 556, 570-574, 587).
//
// Operands.  W is the GGUF weight (Q4_K / Q6_K / Q8_0 raw blocks re-tiled at load,
// or F16), dequantized to f16 in registers; X is the f16 activation matrix [tokens][K].
// The MMA is "swap-AB": the 128-row A operand is a tile of 128 output features
// (dequantized into shared memory in the UMMA 128-byte-swizzled K-major layout) and
// the B operand is up to 256 tokens of X (TMA tensor loads, same swizzle).  The f32
// accumulator lives in TMEM: lane = output feature, column = token.
//
// Work split.  Units are (output tile, k-block of 256); a persistent grid of one CTA
// per SM takes an equal contiguous range of units ("stream-K").  A tile split across
// CTAs is finished by whichever contributor arrives last on the tile's counter: it
// sums every contributor's f32 partial in contributor order (so the result does not
// depend on timing) and applies the epilogue.  The token count M is read on the
// device, so one launch configuration serves every denoising step.
//
// Warp roles (480 threads): w0 activation TMA producer, w1 MMA issuer + TMEM owner,
// w2-w5 dequantizers (thread = weight row), w6-w9 and w11-w14 epilogue (thread = TMEM
// lane; the two warps of a lane quarter take alternate 16-column chunks), w10
// weight-chunk producer (bulk copies into shared memory, L2 prefetch ahead).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx.cuh"

namespace dfb {

// Per-CTA phase timestamps for pipeline analysis (compiled in only with -DDFB_GEMM_TRACE).
#ifdef DFB_GEMM_TRACE
#define GEMM_STAMP(p, slot)                                                                      \
    do {                                                                                         \
        if ((p).trace) (p).trace[(size_t)blockIdx.x * 16 + (slot)] = globaltimer();              \
    } while (0)
// Event streams of CTAs 0..3: stream s, event i -> trace[256*16 + (cta*8 + s)*64 + i].
#define GEMM_EVENT(p, stream, idx)                                                               \
    do {                                                                                         \
        if ((p).trace && blockIdx.x < 4 && (idx) < 64)                                           \
            (p).trace[256 * 16 + ((size_t)blockIdx.x * 8 + (stream)) * 64 + (idx)] = globaltimer(); \
    } while (0)
#else
#define GEMM_STAMP(p, slot) do {} while (0)
#define GEMM_EVENT(p, stream, idx) do {} while (0)
#endif

enum WType : int { W_Q4K = 0, W_Q6K = 1, W_Q80 = 2, W_F16 = 3 };
enum EpiKind : int { EPI_F32 = 0, EPI_F16 = 1, EPI_RESID = 2, EPI_QKV = 3, EPI_SWIGLU = 4, EPI_LOGITS = 5 };

// Bytes of one re-tiled chunk (128 rows x one k-block of 256 elements).
__host__ __device__ constexpr int raw_chunk_bytes(int wt) {
    return wt == W_Q4K ? 128 * 144 : wt == W_Q6K ? 128 * 210 : wt == W_Q80 ? 128 * 272 : 0;
}

struct EpiArgs {
    void *out = nullptr;   // F32/F16/RESID/SWIGLU/LOGITS destination
    int ld = 0;            // its row stride (elements)
    int n_valid = 0;       // valid output features (rows of W before padding)
    // QKV
    __half *q_out = nullptr;
    int ld_q = 0;
    __half *k_cache = nullptr, *v_cache = nullptr;  // [position][n_kv] of this layer
    int ld_kv = 0;
    int n_q_tiles = 0, n_k_tiles = 0;  // tiles in the (padded) Q and K sections
    int n_q = 0, n_kv = 0, head_dim = 0;
    const float *bias = nullptr;       // [(n_q_tiles + 2 n_k_tiles) * 128], section-padded, original order
    const float2 *rope = nullptr;      // [position][head_dim/2] (cos, sin)
    const int *pos = nullptr;          // [tokens] position of each row (QKV, LOGITS)
};

struct GemmParams {
    const uint8_t *w = nullptr;  // re-tiled weight chunks (quantized types)
    int n_tiles = 0;             // 128-row output tiles
    int kb = 0;                  // k-blocks of 256
    const int *m_dev = nullptr;  // token count (device)
    float *ws = nullptr;         // split-tile partials [grid][2][256 * 128]
    int *tile_cnt = nullptr;     // [n_tiles * 2] arrival counters, left at 0
    int *err = nullptr;          // first error code of any CTA
    unsigned long long *trace = nullptr;  // DFB_GEMM_TRACE builds only: [grid][16] globaltimer stamps
    EpiArgs epi;
};

constexpr int kThreads = 480;
constexpr int kEpiThreads = 256;  // two epilogue warps per TMEM lane quarter
constexpr int kPrefetchChunks = 6;  // weight chunks warmed in L2 ahead of the smem copy
constexpr int kStages = 3;
constexpr int kRawStages = 2;
constexpr int kABytes = 128 * 128;       // 128 rows x 64 f16
constexpr int kBBytes = 256 * 128;       // 256 tokens x 64 f16
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kMaxTok = 256;             // tokens per MMA (N)
constexpr int kWsTile = kMaxTok * 128;   // floats per partial tile
constexpr int kErrTimeout = 0x100;

constexpr int kMaxContrib = 64;  // split contributors of one tile tracked in shared memory
constexpr int kFixupPeers = (kStages * kStageBytes) / 32768;  // partial chunks the stage buffers hold
__host__ __device__ constexpr int gemm_smem_bytes(int wt) {
    return 1024 /*align slack*/ + kStages * kStageBytes + kRawStages * raw_chunk_bytes(wt) + 256 /*barriers*/ +
           4 * kMaxTok /*token positions*/ + 8 * kMaxContrib /*contributor partial offsets*/;
}

// Static stream-K schedule, recomputed identically by every role of every CTA.
struct Sched {
    int M, n_mg, gsz, kb, n_ot, U, G, u0, u1;
    __device__ __forceinline__ void init(int M_, int n_tiles, int kb_, int grid, int cta) {
        M = M_;
        kb = kb_;
        n_mg = (M + kMaxTok - 1) / kMaxTok;
        gsz = (((M + n_mg - 1) / n_mg) + 15) & ~15;
        n_ot = n_tiles * n_mg;
        U = n_ot * kb;
        G = grid < U ? grid : U;
        u0 = (int)((long long)cta * U / G);
        u1 = (int)((long long)(cta + 1) * U / G);
    }
    __device__ __forceinline__ int owner(int u) const { return (int)(((long long)(u + 1) * G - 1) / U); }
    __device__ __forceinline__ int begin_of(int c) const { return (int)((long long)c * U / G); }
};

struct Seg {
    int ot, tile, m0, ntok, nmma, nbox, k0, k1;
};
__device__ __forceinline__ Seg make_seg(const Sched &s, int u, int u1) {
    Seg g;
    g.ot = u / s.kb;
    g.k0 = u % s.kb;
    g.k1 = min(s.kb, g.k0 + (u1 - u));
    g.tile = g.ot / s.n_mg;
    const int mg = g.ot % s.n_mg;
    g.m0 = mg * s.gsz;
    g.ntok = min(s.gsz, s.M - g.m0);
    g.nmma = (g.ntok + 15) & ~15;
    g.nbox = (g.ntok + 63) / 64;
    return g;
}

// ───────────── dequantization of one 64-wide k-slice of one weight row ─────────────
// A stage: row r at r*128 B; logical 16-byte chunk c (k = 8c..8c+7) stored at c ^ (r & 7).
__device__ __forceinline__ void st_a(uint8_t *A, int r, int c, uint4 v) {
    *reinterpret_cast<uint4 *>(A + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Q4_K chunk layout (per 128 rows): [d,dmin f16 x2: 4 B/row][scales: 12 B/row at 512]
// [qs: 128 B/row at 2048, 16-byte chunk c stored at c ^ (row & 7)].
struct Q4KRow {
    __half2 d2;
    __half2 sc[8], nsc[8], nmo[8];  // sc, -1024*sc, -(dmin*m) per sub-block, as f16 pairs
};
__device__ __forceinline__ void q4k_load_meta(const uint8_t *R, int r, Q4KRow &m) {
    const uint32_t dm = *reinterpret_cast<const uint32_t *>(R + 4 * r);
    const __half d = __ushort_as_half((unsigned short)(dm & 0xFFFF));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
    m.d2 = __halves2half2(d, d);
    const uint32_t *sp = reinterpret_cast<const uint32_t *>(R + 512 + 12 * r);
    uint8_t q[12];
    const uint32_t s0 = sp[0], s1 = sp[1], s2 = sp[2];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        q[i] = (s0 >> (8 * i)) & 0xFF;
        q[4 + i] = (s1 >> (8 * i)) & 0xFF;
        q[8 + i] = (s2 >> (8 * i)) & 0xFF;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        if (j < 4) {
            sc = q[j] & 63;
            mn = q[j + 4] & 63;
        } else {
            sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
            mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
        }
        const __half hs = __int2half_rn(sc);
        m.sc[j] = __halves2half2(hs, hs);
        const __half hn = __int2half_rn(-1024 * sc);
        m.nsc[j] = __halves2half2(hn, hn);
        const __half ho = __float2half_rn(-(dmin * (float)mn));
        m.nmo[j] = __halves2half2(ho, ho);
    }
}
// 4 nibbles (one byte lane each, values 0..15) -> two f16 pairs of q*sc*d - dmin*m.
__device__ __forceinline__ void q4k_pair(uint32_t nib, const __half2 &sc, const __half2 &nsc, const __half2 &d2,
                                         const __half2 &nmo, uint32_t &o01, uint32_t &o23) {
    const uint32_t p01 = __byte_perm(nib, 0x64646464u, 0x4140);  // (1024 + q0, 1024 + q1)
    const uint32_t p23 = __byte_perm(nib, 0x64646464u, 0x4342);
    const __half2 t01 = __hfma2(u2h(p01), sc, nsc);  // q*sc, exact
    const __half2 t23 = __hfma2(u2h(p23), sc, nsc);
    o01 = h2u(__hfma2(t01, d2, nmo));
    o23 = h2u(__hfma2(t23, d2, nmo));
}
__device__ __forceinline__ void q4k_slice(const uint8_t *R, int r, int s, const Q4KRow &m, uint8_t *A) {
    const uint8_t *qrow = R + 2048 + 128 * r;
    const uint4 qa = *reinterpret_cast<const uint4 *>(qrow + (((2 * s) ^ (r & 7)) << 4));
    const uint4 qb = *reinterpret_cast<const uint4 *>(qrow + (((2 * s + 1) ^ (r & 7)) << 4));
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int jl = 2 * s, jh = 2 * s + 1;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint4 lo, hi;
        const uint32_t w0 = w[2 * c], w1 = w[2 * c + 1];
        q4k_pair(w0 & 0x0F0F0F0Fu, m.sc[jl], m.nsc[jl], m.d2, m.nmo[jl], lo.x, lo.y);
        q4k_pair(w1 & 0x0F0F0F0Fu, m.sc[jl], m.nsc[jl], m.d2, m.nmo[jl], lo.z, lo.w);
        q4k_pair((w0 >> 4) & 0x0F0F0F0Fu, m.sc[jh], m.nsc[jh], m.d2, m.nmo[jh], hi.x, hi.y);
        q4k_pair((w1 >> 4) & 0x0F0F0F0Fu, m.sc[jh], m.nsc[jh], m.d2, m.nmo[jh], hi.z, hi.w);
        st_a(A, r, c, lo);
        st_a(A, r, 4 + c, hi);
    }
}

// Q6_K chunk layout: [ql: 128 B/row, chunk c at c ^ (row & 7)]
// [qh: 64 B/row at 16384, chunk c at c ^ ((row >> 1) & 3)][scales i8: 16 B/row at 24576]
// [d f16: 2 B/row at 26624].
struct Q6KRow {
    __half2 ds[16];  // f16(d * scale) per 16-element group
};
__device__ __forceinline__ void q6k_load_meta(const uint8_t *R, int r, Q6KRow &m) {
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(R + 26624 + 2 * r)));
    const uint4 sv = *reinterpret_cast<const uint4 *>(R + 24576 + 16 * r);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int g = 0; g < 16; g++) {
        const int sc = (int)(int8_t)((sw[g >> 2] >> (8 * (g & 3))) & 0xFF);
        const __half h = __float2half_rn(d * (float)sc);
        m.ds[g] = __halves2half2(h, h);
    }
}
struct Q6KHalf {
    uint32_t ql[16];
    uint32_t qh[8];
};
__device__ __forceinline__ void q6k_load_half(const uint8_t *R, int r, int h, Q6KHalf &q) {
    const uint8_t *qlrow = R + 128 * r;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 v = *reinterpret_cast<const uint4 *>(qlrow + (((4 * h + c) ^ (r & 7)) << 4));
        q.ql[4 * c] = v.x; q.ql[4 * c + 1] = v.y; q.ql[4 * c + 2] = v.z; q.ql[4 * c + 3] = v.w;
    }
    const uint8_t *qhrow = R + 16384 + 64 * r;
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const uint4 v = *reinterpret_cast<const uint4 *>(qhrow + (((2 * h + c) ^ ((r >> 1) & 3)) << 4));
        q.qh[4 * c] = v.x; q.qh[4 * c + 1] = v.y; q.qh[4 * c + 2] = v.z; q.qh[4 * c + 3] = v.w;
    }
}
// 4 six-bit values (byte lanes) -> two f16 pairs of d*sc*(q-32).
__device__ __forceinline__ void q6k_pair(uint32_t q6, const __half2 &ds, uint32_t &o01, uint32_t &o23) {
    const __half2 k1056 = __halves2half2(__int2half_rn(1056), __int2half_rn(1056));
    const uint32_t p01 = __byte_perm(q6, 0x64646464u, 0x4140);
    const uint32_t p23 = __byte_perm(q6, 0x64646464u, 0x4342);
    o01 = h2u(__hmul2(__hsub2(u2h(p01), k1056), ds));
    o23 = h2u(__hmul2(__hsub2(u2h(p23), k1056), ds));
}
__device__ __forceinline__ void q6k_slice(const Q6KHalf &q, int r, int s, const Q6KRow &m, uint8_t *A) {
    const int s2 = s & 1;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int hiq = c >= 4 ? 1 : 0;
        const int shift = 4 * s2 + 2 * hiq;
        uint4 o;
#pragma unroll
        for (int hw = 0; hw < 2; hw++) {
            const uint32_t lw = q.ql[8 * hiq + 2 * (c & 3) + hw];
            const uint32_t hwd = q.qh[2 * (c & 3) + hw];
            const uint32_t nib = s2 ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
            const uint32_t q6 = nib | (((hwd >> shift) & 0x03030303u) << 4);
            uint32_t a, b;
            q6k_pair(q6, m.ds[4 * s + (c >> 1)], a, b);
            if (hw == 0) { o.x = a; o.y = b; } else { o.z = a; o.w = b; }
        }
        st_a(A, r, c, o);
    }
}

// Q8_0 chunk layout: [d f16 x 8: 16 B/row][qs: 256 B/row at 2048, chunk c at (c & 8) | ((c & 7) ^ (row & 7))].
__device__ __forceinline__ void q80_slice(const uint8_t *R, int r, int s, uint8_t *A) {
    const uint4 dv = *reinterpret_cast<const uint4 *>(R + 16 * r);
    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
    const uint8_t *qrow = R + 2048 + 256 * r;
    const __half2 k1152 = __halves2half2(__int2half_rn(1152), __int2half_rn(1152));
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        const int c = 4 * s + cc;
        const uint4 v = *reinterpret_cast<const uint4 *>(qrow + (((c & 8) | ((c & 7) ^ (r & 7))) << 4));
        const int blk = 2 * s + (cc >> 1);
        const unsigned short dbits = (unsigned short)((dw[blk >> 1] >> (16 * (blk & 1))) & 0xFFFF);
        const __half dh = __ushort_as_half(dbits);
        const __half2 d2 = __halves2half2(dh, dh);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int half_ = 0; half_ < 2; half_++) {
            uint4 o;
            uint32_t *op = &o.x;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const uint32_t x = w[2 * half_ + i] ^ 0x80808080u;
                const uint32_t p01 = __byte_perm(x, 0x64646464u, 0x4140);
                const uint32_t p23 = __byte_perm(x, 0x64646464u, 0x4342);
                op[2 * i] = h2u(__hmul2(__hsub2(u2h(p01), k1152), d2));
                op[2 * i + 1] = h2u(__hmul2(__hsub2(u2h(p23), k1152), d2));
            }
            st_a(A, r, 2 * cc + half_, o);
        }
    }
}

// ───────────── epilogues ─────────────

// Per-thread constants of one output tile (thread = TMEM lane = one output row).
struct EpiRow {
    int f;          // output feature written by this lane (after un-fusing)
    bool fvalid;    // f is a real feature (not tile padding)
    bool writer;    // this lane stores (SwiGLU: the gate lane of each pair)
    int sec;        // QKV: 0 Q, 1 K, 2 V
    int ipair;      // QKV: NEOX pair index i (angle index)
    int bpair;      // QKV: 0 for element i, 1 for element i + head_dim/2
    float bias;     // QKV bias of this row (0 without bias)
};

template <int EPI>
__device__ __forceinline__ EpiRow epi_row(const EpiArgs &e, int tile, int row) {
    EpiRow r{};
    if constexpr (EPI == EPI_SWIGLU) {
        // rows interleaved: 2i = gate_i, 2i+1 = up_i
        r.f = tile * 64 + (row >> 1);
        r.fvalid = 2 * r.f < e.n_valid;
        r.writer = (row & 1) == 0;
    } else if constexpr (EPI == EPI_QKV) {
        const int hd = e.head_dim;
        int lt;
        if (tile < e.n_q_tiles) { r.sec = 0; lt = tile; }
        else if (tile < e.n_q_tiles + e.n_k_tiles) { r.sec = 1; lt = tile - e.n_q_tiles; }
        else { r.sec = 2; lt = tile - e.n_q_tiles - e.n_k_tiles; }
        const int fl = lt * 128 + row;
        const int sec_off = r.sec == 0 ? 0 : r.sec == 1 ? e.n_q_tiles * 128 : (e.n_q_tiles + e.n_k_tiles) * 128;
        if (r.sec < 2) {
            // rows permuted within each head: local 2i+b <-> feature i + b*hd/2 (NEOX pairs)
            const int head = fl / hd, rr = fl % hd;
            r.ipair = rr >> 1;
            r.bpair = rr & 1;
            r.f = head * hd + r.ipair + r.bpair * (hd >> 1);
        } else {
            r.f = fl;
        }
        r.fvalid = r.f < (r.sec == 0 ? e.n_q : e.n_kv);
        r.bias = e.bias ? __ldg(e.bias + sec_off + r.f) : 0.f;
        r.writer = true;
    } else {
        r.f = tile * 128 + row;
        r.fvalid = r.f < e.n_valid;
        r.writer = true;
    }
    return r;
}

// Epilogue of 16 consecutive tokens (tl0 .. tl0+15 of the segment) for this lane's row.
// All global loads of a chunk are issued before any store, so they overlap.  Called
// by all 32 lanes of a warp together (paired epilogues exchange values with the
// neighbouring lane).  s_pos: positions of the segment's tokens (shared memory).
template <int EPI>
__device__ __forceinline__ void epi_chunk(const EpiArgs &e, const EpiRow &r, const int *s_pos, int m0, int tl0,
                                          int ntok, float (&v)[16]) {
    const int nvalid = r.fvalid ? min(16, ntok - tl0) : 0;  // tokens of this chunk that are stored
    if constexpr (EPI == EPI_F32 || EPI == EPI_F16) {
        const size_t base = (size_t)(m0 + tl0) * e.ld + r.f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (i < nvalid) {
                if constexpr (EPI == EPI_F32) reinterpret_cast<float *>(e.out)[base + (size_t)i * e.ld] = v[i];
                else reinterpret_cast<__half *>(e.out)[base + (size_t)i * e.ld] = __float2half_rn(v[i]);
            }
        }
    } else if constexpr (EPI == EPI_RESID) {
        float *x = reinterpret_cast<float *>(e.out) + (size_t)(m0 + tl0) * e.ld + r.f;
        float old[16];
#pragma unroll
        for (int i = 0; i < 16; i++) old[i] = i < nvalid ? x[(size_t)i * e.ld] : 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < nvalid) x[(size_t)i * e.ld] = v[i] + old[i];
    } else if constexpr (EPI == EPI_LOGITS) {
        float *out = reinterpret_cast<float *>(e.out) + r.f;
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < nvalid) out[(size_t)s_pos[tl0 + i] * e.ld] = v[i];
    } else if constexpr (EPI == EPI_SWIGLU) {
        __half *out = reinterpret_cast<__half *>(e.out) + (size_t)(m0 + tl0) * e.ld + r.f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const float up = __shfl_xor_sync(0xffffffffu, v[i], 1);
            const float g = v[i];
            const float h = g * up * (1.0f / (1.0f + __expf(-g)));
            if (r.writer && i < nvalid) out[(size_t)i * e.ld] = __float2half_rn(h);
        }
    } else if constexpr (EPI == EPI_QKV) {
        const int hh = e.head_dim >> 1;
        if (r.sec < 2) {
            float2 cs[16];
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int pp = tl0 + i < ntok ? s_pos[tl0 + i] : 0;
                cs[i] = __ldg(e.rope + (size_t)pp * hh + r.ipair);
            }
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const float x = v[i] + r.bias;
                const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
                const float o = r.bpair == 0 ? (x * cs[i].x - partner * cs[i].y) : (partner * cs[i].y + x * cs[i].x);
                if (i < nvalid) {
                    if (r.sec == 0) e.q_out[(size_t)(m0 + tl0 + i) * e.ld_q + r.f] = __float2half_rn(o);
                    else e.k_cache[(size_t)s_pos[tl0 + i] * e.ld_kv + r.f] = __float2half_rn(o);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (i < nvalid) e.v_cache[(size_t)s_pos[tl0 + i] * e.ld_kv + r.f] = __float2half_rn(v[i] + r.bias);
        }
    }
}

// ───────────── the kernel ─────────────
template <int WT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, GemmParams p) {
    constexpr int RAWB = raw_chunk_bytes(WT);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stages = smem;
    uint8_t *raw = smem + kStages * kStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(raw + kRawStages * RAWB);
    uint64_t *full_b = bars, *full_a = bars + 3, *empty = bars + 6, *raw_full = bars + 9, *raw_empty = bars + 11,
             *acc_full = bars + 13, *acc_empty = bars + 15, *drain = bars + 17;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 18);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 19);
    int *bcast = reinterpret_cast<int *>(bars + 20);
    volatile int *okflag = reinterpret_cast<volatile int *>(bars + 21);
    uint64_t *fix_bar = bars + 22;  // bulk loads of split-tile partials into the drained stage buffers
    int *s_pos = reinterpret_cast<int *>(bars + 32);                              // [kMaxTok]
    long long *s_contrib = reinterpret_cast<long long *>(s_pos + kMaxTok);        // [kMaxContrib]

    const int M = *p.m_dev;
    if (M <= 0) return;
    if (threadIdx.x == 0) GEMM_STAMP(p, 0);
    Sched S;
    S.init(M, p.n_tiles, p.kb, gridDim.x, blockIdx.x);
    if ((int)blockIdx.x >= S.G) return;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 3; i++) {
            mbar_init(&full_b[i], 1);
            mbar_init(&full_a[i], 4);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 4);
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiThreads / 32);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        mbar_init(fix_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_x);
        if (WT == W_F16) prefetch_tmap(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    if (threadIdx.x == 0) GEMM_STAMP(p, 1);

    if (warp == 0) {
        // ── activation TMA producer ──
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                    for (int s = 0; s < 4; s++) {
                        const int st = it % kStages;
                        if (!(ok = mbar_wait(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 2))) break;
                        uint8_t *A = stages + st * kStageBytes;
                        uint8_t *B = A + kABytes;
                        const uint32_t bytes = g.nbox * 8192 + (WT == W_F16 ? kABytes : 0);
                        mbar_arrive_expect_tx(&full_b[st], bytes);
                        for (int b = 0; b < g.nbox; b++)
                            tma_load_2d(B + b * 8192, &tm_x, kbi * 256 + s * 64, g.m0 + b * 64, &full_b[st]);
                        GEMM_EVENT(p, 0, it);
                        if constexpr (WT == W_F16) tma_load_2d(A, &tm_w, kbi * 256 + s * 64, g.tile * 128, &full_b[st]);
                        it++;
                    }
                }
                u += g.k1 - g.k0;
            }
            GEMM_STAMP(p, 2);
            if (!ok) {
                // let every copy this thread started land before the CTA exits
                for (int i = (it > kStages ? it - kStages : 0); i < it; i++)
                    spin_bounded(&full_b[i % kStages], (i / kStages) & 1);
            }
        }
        __syncwarp();
    } else if (warp == 10) {
        // ── weight-chunk producer: one re-tiled chunk (128 rows x 256 k) per k-block ──
        if constexpr (WT != W_F16) {
            if (lane == 0) {
                auto chunk = [&](int u) {
                    const int ot = u / S.kb, kbi = u % S.kb;
                    return p.w + ((size_t)(ot / S.n_mg) * p.kb + kbi) * RAWB;
                };
                for (int u = S.u0; u < S.u1 && u < S.u0 + kPrefetchChunks; u++) bulk_prefetch_l2(chunk(u), RAWB);
                int rit = 0;
                bool ok = true;
                for (int u = S.u0; u < S.u1 && ok; u++) {
                    const int r = rit % kRawStages;
                    if (!(ok = mbar_wait(&raw_empty[r], ((rit / kRawStages) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 1))) break;
                    if (u + kPrefetchChunks < S.u1) bulk_prefetch_l2(chunk(u + kPrefetchChunks), RAWB);
                    mbar_arrive_expect_tx(&raw_full[r], RAWB);
                    bulk_g2s(raw + r * RAWB, chunk(u), RAWB, &raw_full[r]);
                    GEMM_EVENT(p, 1, rit);
                    rit++;
                }
                if (!ok)
                    for (int i = (rit > kRawStages ? rit - kRawStages : 0); i < rit; i++)
                        spin_bounded(&raw_full[i % kRawStages], (i / kRawStages) & 1);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            int it = 0, si = 0;
            bool ok = true, issued = false;
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                const int acc = si & 1;
                if (!(ok = mbar_wait(&acc_empty[acc], ((si >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 3))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * 256;
                const uint32_t idesc = idesc_f16_m128((uint32_t)g.nmma);
                uint32_t accum = 0;
                for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                    for (int s = 0; s < 4; s++) {
                        const int st = it % kStages;
                        const uint32_t ph = (it / kStages) & 1;
                        if (!(ok = mbar_wait(&full_b[st], ph, abort_flag, p.err, kErrTimeout + 4))) break;
                        if constexpr (WT != W_F16)
                            if (!(ok = mbar_wait(&full_a[st], ph, abort_flag, p.err, kErrTimeout + 5))) break;
                        GEMM_EVENT(p, 4, it);
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(stages + st * kStageBytes);
                        const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                        for (int kk = 0; kk < 4; kk++) {
                            mma_f16_ss(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc, accum);
                            accum = 1;
                        }
                        issued = true;
                        mma_commit(&empty[st]);
                        GEMM_EVENT(p, 5, it);
                        it++;
                    }
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
                si++;
                u += g.k1 - g.k0;
            }
            GEMM_STAMP(p, 3);
            if (issued) {
                // every MMA must have retired before TMEM is released
                mma_commit(drain);
                spin_bounded(drain, 0);
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ── dequantizers: thread = weight row of the tile ──
        if constexpr (WT != W_F16) {
            const int r = threadIdx.x - 64;
            int it = 0, rit = 0;
            bool ok = true;
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                    const int rs = rit % kRawStages;
                    ok = __all_sync(0xffffffffu, mbar_wait(&raw_full[rs], (rit / kRawStages) & 1, abort_flag, p.err, kErrTimeout + 6));
                    if (!ok) break;
                    if (r == 0) GEMM_EVENT(p, 2, rit);
                    const uint8_t *R = raw + rs * RAWB;
                    if constexpr (WT == W_Q4K) {
                        Q4KRow meta;
                        q4k_load_meta(R, r, meta);
                        #pragma unroll
                        for (int s = 0; s < 4; s++) {
                            const int st = it % kStages;
                            ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 7));
                            if (!ok) break;
                            q4k_slice(R, r, s, meta, stages + st * kStageBytes);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&full_a[st]);
                            if (r == 0) GEMM_EVENT(p, 3, it);
                            it++;
                        }
                    } else if constexpr (WT == W_Q6K) {
                        Q6KRow meta;
                        q6k_load_meta(R, r, meta);
                        Q6KHalf qv;
                        #pragma unroll
                        for (int s = 0; s < 4; s++) {
                            if ((s & 1) == 0) q6k_load_half(R, r, s >> 1, qv);
                            const int st = it % kStages;
                            ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 7));
                            if (!ok) break;
                            q6k_slice(qv, r, s, meta, stages + st * kStageBytes);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&full_a[st]);
                            it++;
                        }
                    } else {
                        #pragma unroll
                        for (int s = 0; s < 4; s++) {
                            const int st = it % kStages;
                            ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((it / kStages) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 7));
                            if (!ok) break;
                            q80_slice(R, r, s, stages + st * kStageBytes);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&full_a[st]);
                            it++;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                    rit++;
                }
                u += g.k1 - g.k0;
            }
        }
    } else {
        // ── epilogue: thread = TMEM lane = output feature ──
        const int q = warp & 3;
        const int row = 32 * q + lane;
        const int half = warp >= 11 ? 1 : 0;
        const int et = half ? 128 + (int)threadIdx.x - 352 : (int)threadIdx.x - 192;  // 0..255
        uint32_t fix_phase = 0;
        int si = 0;
        bool ok = true;
        const int first_ot = S.begin_of(blockIdx.x) / S.kb;
        for (int u = S.u0; u < S.u1 && ok;) {
            const Seg g = make_seg(S, u, S.u1);
            const int acc = si & 1;
            // one thread waits, the barrier hands the outcome to the whole group
            if (et == 0) *okflag = mbar_wait(&acc_full[acc], (si >> 1) & 1, abort_flag, p.err, kErrTimeout + 8) ? 1 : 0;
            named_bar_sync(1, kEpiThreads);
            ok = *okflag != 0;
            if (!ok) break;
            if (et == 0 && si < 4) GEMM_STAMP(p, 4 + 2 * si);
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + acc * 256;
            const bool whole = g.k0 == 0 && g.k1 == S.kb;
            const EpiRow er = epi_row<EPI>(p.epi, g.tile, row);
            if constexpr (EPI == EPI_QKV || EPI == EPI_LOGITS) {
                for (int t = et; t < g.ntok; t += kEpiThreads) s_pos[t] = p.epi.pos[g.m0 + t];
                named_bar_sync(1, kEpiThreads);
            }
            // mode 0: whole tile straight from TMEM; 1: finisher with the other partials
            // bulk-staged in the drained stage buffers; 2: finisher reading partials from L2;
            // 3: not the finisher (nothing to emit)
            int mode = 0, nc = 1, me = 0;
            const bool last_seg = u + (g.k1 - g.k0) == S.u1;  // stage buffers drained after this one
            if (!whole) {
                // Split tile.  Partials are stored [64-column chunk][column][row] (32 KB per
                // chunk, coalesced for the writers, bank-conflict-free in shared memory).
                const int slot = g.ot == first_ot ? 0 : 1;
                float *wsl = p.ws + ((size_t)blockIdx.x * 2 + slot) * kWsTile;
                if (et == 0) GEMM_EVENT(p, 6, 5 * si + 0);
                for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                    uint32_t u16[16];
                    tmem_ld16(taddr + c0, u16);
                    tmem_ld_wait();
                    float *dst = wsl + (size_t)(c0 >> 6) * 8192 + (size_t)(c0 & 63) * 128 + row;
#pragma unroll
                    for (int i = 0; i < 16; i++) dst[i * 128] = __uint_as_float(u16[i]);
                }
                __threadfence();
                named_bar_sync(1, kEpiThreads);
                const int c_first = S.owner(g.ot * S.kb), c_last = S.owner((g.ot + 1) * S.kb - 1);
                nc = c_last - c_first + 1;
                me = blockIdx.x - c_first;
                if (et == 0) {
                    const int old = atomicAdd(&p.tile_cnt[g.ot], 1);
                    *bcast = (old == nc - 1) ? 1 : 0;
                    if (nc > kMaxContrib) atomicCAS(p.err, 0, kErrTimeout + 9);  // launcher keeps nc <= kMaxContrib
                }
                if (et < nc && et < kMaxContrib) {  // (et < kEpiThreads covers kMaxContrib)
                    const int c = c_first + et;
                    const int sl = (S.begin_of(c) / S.kb == g.ot) ? 0 : 1;
                    s_contrib[et] = ((long long)c * 2 + sl) * kWsTile;
                }
                named_bar_sync(1, kEpiThreads);
                if (et == 0) GEMM_EVENT(p, 6, 5 * si + 3);
                if (!*bcast || nc > kMaxContrib) mode = 3;
                else {
                    __threadfence();
                    mode = (last_seg && nc - 1 <= kFixupPeers) ? 1 : 2;
                }
            }
            if (mode >= 2) {
                // the accumulator is in the workspace: let the MMA warp reuse the TMEM buffer
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            if (mode != 3) {
                const float *sbuf = reinterpret_cast<const float *>(stages);
                bool staged_ok = true;
                for (int cb = 0; cb < g.nmma && staged_ok; cb += 64) {
                    if (mode == 1) {
                        // stage this 64-column chunk of every other contributor
                        const int cols = min(64, g.nmma - cb);
                        named_bar_sync(1, kEpiThreads);  // the previous chunk's buffers are consumed
                        if (et == 0) {
                            fence_proxy_async_smem();
                            mbar_arrive_expect_tx(fix_bar, (uint32_t)(nc - 1) * cols * 512);
                            for (int c = 0, k = 0; c < nc; c++) {
                                if (c == me) continue;
                                bulk_g2s(stages + (size_t)k * 32768, p.ws + s_contrib[c] + (size_t)(cb >> 6) * 8192,
                                         (uint32_t)cols * 512, fix_bar);
                                k++;
                            }
                            *okflag = mbar_wait(fix_bar, fix_phase, abort_flag, p.err, kErrTimeout + 10) ? 1 : 0;
                        }
                        fix_phase ^= 1;
                        named_bar_sync(1, kEpiThreads);
                        if (!*okflag) { staged_ok = false; break; }
                    }
                  for (int c0 = cb + 16 * half; c0 < min(cb + 64, g.nmma); c0 += 32) {
                    float v[16];
                    if (mode <= 1) {
                        uint32_t u16[16];
                        tmem_ld16(taddr + c0, u16);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; i++) v[i] = __uint_as_float(u16[i]);
                    }
                    if (mode >= 1) {
                        // ordered sum over contributors: the result does not depend on timing
                        float own[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) { own[i] = v[i]; v[i] = 0.f; }
                        for (int c = 0, k = 0; c < nc; c++) {
                            float t[16];
                            if (mode == 1 && c == me) {
#pragma unroll
                                for (int i = 0; i < 16; i++) t[i] = own[i];
                            } else if (mode == 1) {
                                const float *src = sbuf + (size_t)k * 8192 + (size_t)(c0 & 63) * 128 + row;
#pragma unroll
                                for (int i = 0; i < 16; i++) t[i] = src[i * 128];
                                k++;
                            } else {
                                const float *src = p.ws + s_contrib[c] + (size_t)(c0 >> 6) * 8192 + (size_t)(c0 & 63) * 128 + row;
#pragma unroll
                                for (int i = 0; i < 16; i++) t[i] = __ldcg(src + i * 128);
                            }
#pragma unroll
                            for (int i = 0; i < 16; i++) v[i] += t[i];
                        }
                    }
                    epi_chunk<EPI>(p.epi, er, s_pos, g.m0, c0, g.ntok, v);
                  }
                }
                if (mode >= 1 && et == 0) {
                    p.tile_cnt[g.ot] = 0;
                    GEMM_EVENT(p, 6, 5 * si + 4);
                }
            }
            if (mode <= 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            named_bar_sync(1, kEpiThreads);  // okflag / bcast are reused by the next segment
            if (et == 0 && si < 4) GEMM_STAMP(p, 5 + 2 * si);
            si++;
            u += g.k1 - g.k0;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) GEMM_STAMP(p, 12);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

}  // namespace dfb
