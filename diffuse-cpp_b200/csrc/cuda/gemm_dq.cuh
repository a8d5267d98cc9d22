// Dequant-fused tcgen05 GEMM:  Y[tok][n] = sum_k X[tok][k] * W[n][k]
//
// Replaces every ggml_mul_mat(W, x) of the reference forward (src/diffuse-graph.cpp
// :61-63, 122, 136-140, 154 and the cached variants :451-453, 556, 570-574, 587).
//
// Operands.  W is the GGUF weight (Q4_K / Q6_K / Q8_0 raw blocks re-tiled at load,
// or F16), dequantized to f16 in registers; X is the f16 activation matrix [tokens][K].
// The MMA is "swap-AB" and paired (tcgen05 cta_group::2, M = 256): the A operand is a
// tile of 256 output features, 128 dequantized into the TMEM of each CTA of a pair (F16
// weights: TMA-loaded into shared memory, 128-byte-swizzled K-major); the B operand is a
// group of up to 256 tokens of X, each CTA holding half of them (TMA tensor loads into
// shared memory, same swizzle).  The f32 accumulator lives in TMEM: lane = output
// feature, column = token.
//
// Work split.  Units are (pair tile of 256 output rows, token group, k-block of 256); a
// persistent grid of CTA pairs (one CTA per SM) takes equal contiguous unit ranges
// ("stream-K").  A tile split across pairs is finished by all of its contributors
// together once each has written its f32 partial: every contributor takes an equal
// share of the tile's token columns and sums all partials for them in contributor
// order (so the result does not depend on timing), then applies the epilogue.  The
// token count M is read on the device, so one launch configuration serves every
// denoising step.
//
// Warp roles (640 threads per CTA): see the kernel.
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
// Event streams of CTAs 0..3 (also -DDFB_GEMM_EVENTS, which perturbs the timing it records):
// stream s, event i -> trace[256*16 + (cta*8 + s)*64 + i].
#ifdef DFB_GEMM_EVENTS
#define GEMM_EVENT(p, stream, idx)                                                               \
    do {                                                                                         \
        if ((p).trace && blockIdx.x < 4 && (idx) < 64)                                           \
            (p).trace[256 * 16 + ((size_t)blockIdx.x * 8 + (stream)) * 64 + (idx)] = globaltimer(); \
    } while (0)
#else
#define GEMM_EVENT(p, stream, idx) do {} while (0)
#endif
#else
#define GEMM_STAMP(p, slot) do {} while (0)
#define GEMM_EVENT(p, stream, idx) do {} while (0)
#endif

enum WType : int { W_Q4K = 0, W_Q6K = 1, W_Q80 = 2, W_F16 = 3 };
enum EpiKind : int { EPI_F32 = 0, EPI_F16 = 1, EPI_QKV = 3, EPI_SWIGLU = 4, EPI_LOGITS = 5 };

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

// Activation tensor maps, one per token half-group size h = 16 (i + 1), i = 0..7: a 3-D
// view {64 k, rows, K / 64 k-blocks} of the row-major [rows][K] f16 matrix (strides: row,
// then 128 B), box {64, h, x_slices(h)}, 128-byte swizzle.  One load brings x_slices
// consecutive 64-wide k-slices of h rows, each in the canonical K-major SW128 layout.
constexpr int kXMaps = 8;
__host__ __device__ constexpr int x_slices(int h) { return h <= 32 ? 4 : h <= 64 ? 2 : 1; }
struct XMaps {
    CUtensorMap m[kXMaps];
};

struct GemmParams {
    const uint8_t *w = nullptr;  // re-tiled weight chunks (quantized types)
    int K = 0;                   // valid columns of the activations
    int n_tiles = 0;             // 128-row output tiles
    int kb = 0;                  // k-blocks of 256
    const int *m_dev = nullptr;  // token count (device)
    float *ws = nullptr;         // split-tile partials [grid][2][256 * 128]
    int *tile_cnt = nullptr;     // [n_tiles x token groups] arrival + departure counters, left at 0
    int *err = nullptr;          // first error code of any CTA
    unsigned long long *trace = nullptr;  // DFB_GEMM_TRACE builds only: [grid][16] globaltimer stamps
    EpiArgs epi;
};

constexpr int kThreads = 640;            // 20 warps, roles below
constexpr int kEpiThreads = 256;         // two epilogue warps per TMEM lane quarter
constexpr int kDeqWarps = 8;             // two sets of four: even / odd k-slices
constexpr int kSliceBytes = 128 * 128;   // one 64-wide k-slice of this CTA's 128 weight rows (f16)
constexpr int kABytes = kSliceBytes;      // one A stage: one k-slice
constexpr int kMaxTok = 256;             // tokens per MMA group (N) of the pair
constexpr int kDblTok = 192;             // groups up to this size double-buffer the accumulator
constexpr int kWsTile = kMaxTok * 128;   // floats per partial tile (one CTA's 128 rows)
constexpr int kErrTimeout = 0x100;
constexpr int kMaxAStages = 6, kMaxBSlots = 24, kMaxRawStages = 4;
// TMEM (512 columns per CTA): accumulators [0, 192) and [192, 384) for token groups of up
// to 192, one accumulator [0, 256) for larger groups (the MMA of the next segment then
// waits for the epilogue to drain it, which costs less than dequantizing the weights once
// per group of 128); dequantized A stages (quantized weights) at [384 + 32 st, +32):
// lane = weight row, one k-slice each.
constexpr int kTmemA = 2 * kDblTok;
constexpr int kTmemAStage = 32;

// Rings per weight type, sized so that shared memory (227 KB) holds them:
//  A        one k-slice per stage, four stages (one k-block): dequantized weights go to
//           TMEM (written by tcgen05.st, read by the MMA from TMEM: no shared-memory round
//           trip and no proxy fence, which cost ~1.2k cycles per warp and stage); F16
//           weights are TMA-loaded into a shared-memory ring instead;
//  B ring   this CTA's activation rows of 1-4 k-slices per slot (2-12 KB), so small
//           token counts keep many slices in flight and hide the L2 latency;
//  raw ring re-tiled weight chunks (one k-block of 256 for 128 rows), grouped.
__host__ __device__ constexpr int a_stages(int wt) { return 4; }
__host__ __device__ constexpr int a_ring_bytes(int wt) { return wt == W_F16 ? 4 * kABytes : 0; }
__host__ __device__ constexpr int b_ring_bytes(int wt) { return 96 * 1024; }
// A raw stage holds raw_cpr consecutive chunks of the CTA's unit range: the weight
// stream reached ~3.8 TB/s with 18 KB stages and ~6-7 TB/s with 36-72 KB stages
// (same bytes in flight), so small chunks are grouped.
__host__ __device__ constexpr int raw_stages(int wt) { return wt == W_Q4K ? 3 : wt == W_Q6K ? 4 : wt == W_Q80 ? 3 : 0; }
__host__ __device__ constexpr int raw_cpr(int wt) { return wt == W_Q4K ? 2 : 1; }

// Warp roles.  A warp runs on scheduler warp % 4 and may only access TMEM lanes
// 32*(warp % 4)..+31, so the dequantizers (they write A into TMEM) and the epilogue cover
// every lane quarter: w4-w7 dequantizer set 0, w8-w11 set 1, w12-w19 epilogue (each
// quarter twice); w0 activation producer, w1 MMA issuer, w2 weight-chunk producer, w3
// relay.
enum WarpRole : int { R_DEQ = 0, R_MMA = 1, R_BPROD = 2, R_WPROD = 3, R_EPI = 4, R_RELAY = 5 };
__host__ __device__ constexpr int warp_role(int w) {
    return w == 0 ? R_BPROD : w == 1 ? R_MMA : w == 2 ? R_WPROD : w == 3 ? R_RELAY : w < 12 ? R_DEQ : R_EPI;
}
// dequantizer index 0..7: set = index / 4 takes k-slices set and set + 2 of each k-block;
// its weight rows are the warp's TMEM lane quarter
__host__ __device__ constexpr int deq_index(int w) { return w - 4; }
// epilogue thread group: warps 12-15 and 16-19 each cover the four lane quarters
__host__ __device__ constexpr int epi_half(int w) { return w >= 16 ? 1 : 0; }

constexpr int kEpiStageBytes = 16 * 128 * 4;  // epilogue output staging per half: 16 tokens x 128 f32
constexpr int kMaxContrib = 64;     // split contributors (CTA pairs) of one tile tracked in shared memory
constexpr int kBarBytes = 80 * 8;   // mbarriers and flags, see the kernel's shared-memory map
__host__ __device__ constexpr int gemm_smem_bytes(int wt) {
    return 1024 /*align slack*/ + a_ring_bytes(wt) + b_ring_bytes(wt) + raw_stages(wt) * raw_cpr(wt) * raw_chunk_bytes(wt) +
           2 * kEpiStageBytes /*epilogue output staging*/ + kBarBytes /*barriers, flags*/ + 4 * kMaxTok /*token positions*/ + 8 * kMaxContrib /*contributor partial offsets*/;
}

// Static stream-K schedule over CTA pairs, recomputed identically by every role of
// both CTAs of a pair.  Units are (pair tile of 256 weight rows, token group, k-block).
struct Sched {
    int M, n_mg, gsz, kb, n_ot, U, G, u0, u1;
    bool dbl;                 // double-buffered accumulator (gsz <= kDblTok)
    int bh, spb, bslot, nbs;  // B ring: rows per CTA (widest group), slices per load, slot bytes, slots
    __device__ __forceinline__ void init(int M_, int n_ptiles, int kb_, int n_pairs, int pair, int ring_bytes) {
        M = M_;
        kb = kb_;
        n_mg = (M + kMaxTok - 1) / kMaxTok;
        gsz = (((M + n_mg - 1) / n_mg) + 15) & ~15;
        dbl = gsz <= kDblTok;
        n_ot = n_ptiles * n_mg;
        U = n_ot * kb;
        G = n_pairs < U ? n_pairs : U;
        if (M <= 0 || pair >= G) {
            u0 = u1 = 0;
        } else {
            u0 = (int)((long long)pair * U / G);
            u1 = (int)((long long)(pair + 1) * U / G);
        }
        bh = ((gsz + 31) & ~31) >> 1;  // 16..128
        if (bh < 16) bh = 16;
        spb = x_slices(bh);
        bslot = bh * 128 * spb;
        nbs = ring_bytes / bslot;
        if (nbs > kMaxBSlots) nbs = kMaxBSlots;
    }
    // accumulator buffer of segment si and how many segments used it before
    __device__ __forceinline__ int acc_of(int si) const { return dbl ? (si & 1) : 0; }
    __device__ __forceinline__ int acc_uses(int si) const { return dbl ? (si >> 1) : si; }
    __device__ __forceinline__ int owner(int u) const { return (int)(((long long)(u + 1) * G - 1) / U); }
    __device__ __forceinline__ int begin_of(int c) const { return (int)((long long)c * U / G); }
};

struct Seg {
    int ot, pt, m0, ntok, nmma, half, k0, k1;
};
__device__ __forceinline__ Seg make_seg(const Sched &s, int u, int u1) {
    Seg g;
    g.ot = u / s.kb;
    g.k0 = u % s.kb;
    g.k1 = min(s.kb, g.k0 + (u1 - u));
    g.pt = g.ot / s.n_mg;
    const int mg = g.ot % s.n_mg;
    g.m0 = mg * s.gsz;
    g.ntok = min(s.gsz, s.M - g.m0);
    g.nmma = (g.ntok + 31) & ~31;  // MMA N: split evenly over the pair, 16-row multiples each
    g.half = g.nmma >> 1;          // tokens [m0 + rank*half, +half) are this CTA's B rows
    return g;
}

// ───────────── dequantization of one 64-wide k-slice of one weight row ─────────────
// The slice is produced in 32 registers of f16 pairs in k order (register j holds k = 2j
// in its low half and 2j + 1 in its high half), the layout of one TMEM lane of a 32-column
// A operand; put() fills the 8 k-values of 16-byte chunk c.
__device__ __forceinline__ void put(uint32_t (&o)[32], int c, uint4 v) {
    o[4 * c] = v.x; o[4 * c + 1] = v.y; o[4 * c + 2] = v.z; o[4 * c + 3] = v.w;
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Q4_K chunk layout (per 128 rows): [d,dmin f16 x2: 4 B/row][scales: 12 B/row at 512]
// [qs: 128 B/row at 2048, 16-byte chunk c stored at c ^ (row & 7)].
// Scales of the four sub-blocks one dequant set uses: set p dequantizes k-slices p and
// p + 2, i.e. sub-blocks 2p, 2p + 1 (local 0, 1) and 2p + 4, 2p + 5 (local 2, 3).
struct Q4KMeta {
    __half2 d2;
    __half2 sc[4], nsc[4], nmo[4];  // sc, -1024*sc, -(dmin*m) per sub-block, as f16 pairs
};
__device__ __forceinline__ void q4k_load_meta(const uint8_t *R, int r, int set, Q4KMeta &m) {
    const uint32_t dm = *reinterpret_cast<const uint32_t *>(R + 4 * r);
    const __half d = __ushort_as_half((unsigned short)(dm & 0xFFFF));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
    m.d2 = __halves2half2(d, d);
    const uint32_t *sp = reinterpret_cast<const uint32_t *>(R + 512 + 12 * r);
    const uint32_t s0 = sp[0], s1 = sp[1], s2 = sp[2];
    // byte i of the 12 packed scale bytes (i may be a runtime value: no local array)
    auto qb = [&](int i) -> int { return (int)(((i < 4 ? s0 : i < 8 ? s1 : s2) >> (8 * (i & 3))) & 0xFF); };
#pragma unroll
    for (int l = 0; l < 4; l++) {
        // 6-bit scale / min of sub-block j (get_scale_min_k4 packing)
        const int j = 2 * set + (l & 1) + 4 * (l >> 1);
        int sc, mn;
        if (l < 2) {  // j < 4
            sc = qb(j) & 63;
            mn = qb(j + 4) & 63;
        } else {
            sc = (qb(j + 4) & 0xF) | ((qb(j - 4) >> 6) << 4);
            mn = (qb(j + 4) >> 4) | ((qb(j) >> 6) << 4);
        }
        const __half hs = __int2half_rn(sc);
        m.sc[l] = __halves2half2(hs, hs);
        const __half hn = __int2half_rn(-1024 * sc);
        m.nsc[l] = __halves2half2(hn, hn);
        const __half ho = __float2half_rn(-(dmin * (float)mn));
        m.nmo[l] = __halves2half2(ho, ho);
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
// Slice s (k = 64s .. 64s+63) of row r: low nibbles of qs bytes 32s.. are sub-block 2s,
// high nibbles sub-block 2s+1; lo = local meta index of sub-block 2s.
__device__ __forceinline__ void q4k_slice(const uint8_t *R, int r, int s, int lo, const Q4KMeta &m, uint32_t (&o)[32]) {
    const uint8_t *qrow = R + 2048 + 128 * r;
    const uint4 qa = *reinterpret_cast<const uint4 *>(qrow + (((2 * s) ^ (r & 7)) << 4));
    const uint4 qb = *reinterpret_cast<const uint4 *>(qrow + (((2 * s + 1) ^ (r & 7)) << 4));
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int jl = lo, jh = lo + 1;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint4 lo4, hi4;
        const uint32_t w0 = w[2 * c], w1 = w[2 * c + 1];
        q4k_pair(w0 & 0x0F0F0F0Fu, m.sc[jl], m.nsc[jl], m.d2, m.nmo[jl], lo4.x, lo4.y);
        q4k_pair(w1 & 0x0F0F0F0Fu, m.sc[jl], m.nsc[jl], m.d2, m.nmo[jl], lo4.z, lo4.w);
        q4k_pair((w0 >> 4) & 0x0F0F0F0Fu, m.sc[jh], m.nsc[jh], m.d2, m.nmo[jh], hi4.x, hi4.y);
        q4k_pair((w1 >> 4) & 0x0F0F0F0Fu, m.sc[jh], m.nsc[jh], m.d2, m.nmo[jh], hi4.z, hi4.w);
        put(o, c, lo4);
        put(o, 4 + c, hi4);
    }
}

// Q6_K chunk layout: [ql: 128 B/row, chunk c at c ^ (row & 7)]
// [qh: 64 B/row at 16384, chunk c at c ^ ((row >> 1) & 3)][scales i8: 16 B/row at 24576]
// [d f16: 2 B/row at 26624].
// d * scale of the eight 16-element groups one dequant set uses: set p takes slices p
// and p + 2, i.e. groups 4p .. 4p + 3 and 4p + 8 .. 4p + 11 (scale words p and p + 2).
struct Q6KMeta {
    __half2 ds[8];
};
__device__ __forceinline__ void q6k_load_meta(const uint8_t *R, int r, int set, Q6KMeta &m) {
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(R + 26624 + 2 * r)));
    const uint4 sv = *reinterpret_cast<const uint4 *>(R + 24576 + 16 * r);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int wi = set + 2 * h;  // scale word holding groups 4*wi .. 4*wi+3
        const uint32_t w = wi == 0 ? sv.x : wi == 1 ? sv.y : wi == 2 ? sv.z : sv.w;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int sc = (int)(int8_t)((w >> (8 * i)) & 0xFF);
            const __half hh = __float2half_rn(d * (float)sc);
            m.ds[4 * h + i] = __halves2half2(hh, hh);
        }
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
__device__ __forceinline__ void q6k_slice(const Q6KHalf &q, int s, int lo, const Q6KMeta &m, uint32_t (&out)[32]) {
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
            q6k_pair(q6, m.ds[lo + (c >> 1)], a, b);
            if (hw == 0) { o.x = a; o.y = b; } else { o.z = a; o.w = b; }
        }
        put(out, c, o);
    }
}

// Q8_0 chunk layout: [d f16 x 8: 16 B/row][qs: 256 B/row at 2048, chunk c at (c & 8) | ((c & 7) ^ (row & 7))].
__device__ __forceinline__ void q80_slice(const uint8_t *R, int r, int s, uint32_t (&out)[32]) {
    const uint4 dv = *reinterpret_cast<const uint4 *>(R + 16 * r);
    const uint8_t *qrow = R + 2048 + 256 * r;
    const __half2 k1152 = __halves2half2(__int2half_rn(1152), __int2half_rn(1152));
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        const int c = 4 * s + cc;
        const uint4 v = *reinterpret_cast<const uint4 *>(qrow + (((c & 8) | ((c & 7) ^ (r & 7))) << 4));
        const int blk = 2 * s + (cc >> 1);
        const int wi = blk >> 1;  // may be a runtime value: select, no local array
        const uint32_t dwd = wi == 0 ? dv.x : wi == 1 ? dv.y : wi == 2 ? dv.z : dv.w;
        const unsigned short dbits = (unsigned short)((dwd >> (16 * (blk & 1))) & 0xFFFF);
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
            put(out, 2 * cc + half_, o);
        }
    }
}

// ───────────── epilogues ─────────────

// Per-thread constants of one output tile (thread = TMEM lane = one output row).
struct EpiRow {
    int f;          // output feature written by this lane (after un-fusing)
    int col;        // its column in the tile's staging rows
    bool fvalid;    // f is a real feature (not tile padding)
    bool writer;    // this lane stores (SwiGLU: the gate lane of each pair)
    int sec;        // QKV: 0 Q, 1 K, 2 V
    int ipair;      // QKV: NEOX pair index i (angle index)
    int bpair;      // QKV: 0 for element i, 1 for element i + head_dim/2
    float bias;     // QKV bias of this row (0 without bias)
};

// QKV tile -> section (0 Q, 1 K, 2 V) and tile index within it.
__device__ __forceinline__ int qkv_section(const EpiArgs &e, int tile, int &lt) {
    if (tile < e.n_q_tiles) { lt = tile; return 0; }
    if (tile < e.n_q_tiles + e.n_k_tiles) { lt = tile - e.n_q_tiles; return 1; }
    lt = tile - e.n_q_tiles - e.n_k_tiles;
    return 2;
}

template <int EPI>
__device__ __forceinline__ EpiRow epi_row(const EpiArgs &e, int tile, int row) {
    EpiRow r{};
    if constexpr (EPI == EPI_SWIGLU) {
        // rows interleaved: 2i = gate_i, 2i+1 = up_i
        r.f = tile * 64 + (row >> 1);
        r.col = row >> 1;
        r.fvalid = 2 * r.f < e.n_valid;
        r.writer = (row & 1) == 0;
    } else if constexpr (EPI == EPI_QKV) {
        const int hd = e.head_dim;
        int lt;
        r.sec = qkv_section(e, tile, lt);
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
        r.col = r.f - lt * 128;  // heads divide the 128-row tile, so the tile's features stay in it
        r.fvalid = r.f < (r.sec == 0 ? e.n_q : e.n_kv);
        r.bias = (e.bias && r.fvalid) ? __ldg(e.bias + sec_off + r.f) : 0.f;
        r.writer = true;
    } else {
        r.f = tile * 128 + row;
        r.col = row;
        r.fvalid = r.f < e.n_valid;
        r.writer = true;
    }
    return r;
}

// Output staging: a chunk of 16 tokens x the tile's output features, one per epilogue
// half, written by the row threads and stored to global memory as whole token rows.
template <int EPI> struct EpiFmt {
    static constexpr int esize = (EPI == EPI_F32 || EPI == EPI_LOGITS) ? 4 : 2;
    static constexpr int width = EPI == EPI_SWIGLU ? 64 : 128;  // output features per tile
    static constexpr int row_bytes = esize * width;            // staging row pitch
};

// Where one tile's token rows go.
struct EpiDst {
    char *base;      // the tile's first output feature in row 0
    long long ld;    // bytes between rows
    int nbytes;      // valid bytes per row (0: the tile is padding)
    bool by_pos;     // row index = the token's position (else m0 + token)
    bool vec;        // 16-byte vector stores are aligned
};
template <int EPI>
__device__ __forceinline__ EpiDst epi_dst(const EpiArgs &e, int tile) {
    constexpr int es = EpiFmt<EPI>::esize, W = EpiFmt<EPI>::width;
    EpiDst d{};
    long long ld_el;
    int n_feat, f0;
    if constexpr (EPI == EPI_QKV) {
        int lt;
        const int sec = qkv_section(e, tile, lt);
        f0 = lt * 128;
        char *b = reinterpret_cast<char *>(sec == 0 ? e.q_out : sec == 1 ? e.k_cache : e.v_cache);
        d.base = b + (size_t)f0 * es;
        ld_el = sec == 0 ? e.ld_q : e.ld_kv;
        n_feat = (sec == 0 ? e.n_q : e.n_kv) - f0;
        d.by_pos = sec != 0;
    } else {
        f0 = tile * W;
        d.base = reinterpret_cast<char *>(e.out) + (size_t)f0 * es;
        ld_el = e.ld;
        n_feat = (EPI == EPI_SWIGLU ? e.n_valid / 2 : e.n_valid) - f0;
        d.by_pos = EPI == EPI_LOGITS;
    }
    d.ld = ld_el * es;
    d.nbytes = max(0, min(W, n_feat)) * es;
    d.vec = (reinterpret_cast<uintptr_t>(d.base) % 16 == 0) && (d.ld % 16 == 0);
    return d;
}

// Epilogue math of 16 consecutive tokens (tl0 .. tl0+15 of the segment) for this lane's
// row, into the staging rows.  Called by all 32 lanes of a warp together (paired
// epilogues exchange values with the neighbouring lane).  s_pos: positions of the
// segment's tokens (shared memory).
template <int EPI>
__device__ __forceinline__ void epi_values(const EpiArgs &e, const EpiRow &r, const int *s_pos, int tl0, int ntok,
                                           float (&v)[16], uint8_t *stage) {
    constexpr int RB = EpiFmt<EPI>::row_bytes;
    if constexpr (EPI == EPI_F32 || EPI == EPI_LOGITS) {
#pragma unroll
        for (int i = 0; i < 16; i++) reinterpret_cast<float *>(stage + i * RB)[r.col] = v[i];
    } else if constexpr (EPI == EPI_F16) {
#pragma unroll
        for (int i = 0; i < 16; i++) reinterpret_cast<__half *>(stage + i * RB)[r.col] = __float2half_rn(v[i]);
    } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const float up = __shfl_xor_sync(0xffffffffu, v[i], 1);
            const float g = v[i];
            const float h = __fdividef(g * up, 1.0f + __expf(-g));  // silu(g) * up
            if (r.writer) reinterpret_cast<__half *>(stage + i * RB)[r.col] = __float2half_rn(h);
        }
    } else if constexpr (EPI == EPI_QKV) {
        if (r.sec < 2) {
            const int hh = e.head_dim >> 1;
            float2 csv[16];
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int pp = tl0 + i < ntok ? s_pos[tl0 + i] : 0;
                csv[i] = __ldg(e.rope + (size_t)pp * hh + r.ipair);
            }
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const float2 cs = csv[i];
                const float x = v[i] + r.bias;
                const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
                const float o = r.bpair == 0 ? (x * cs.x - partner * cs.y) : (partner * cs.y + x * cs.x);
                if (r.col < 128) reinterpret_cast<__half *>(stage + i * RB)[r.col] = __float2half_rn(o);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (r.col < 128) reinterpret_cast<__half *>(stage + i * RB)[r.col] = __float2half_rn(v[i] + r.bias);
        }
    }
}

// Stores the staged chunk as token rows: lanes of a warp cover a row in 16-byte pieces.
// tid: 0..127 within the epilogue half.
template <int EPI>
__device__ __forceinline__ void epi_copyout(const EpiDst &d, const int *s_pos, int m0, int tl0, int ntok,
                                            const uint8_t *stage, int tid) {
    constexpr int es = EpiFmt<EPI>::esize, RB = EpiFmt<EPI>::row_bytes;
    constexpr int LPR = RB / 16, RPW = 32 / LPR;  // lanes per row, rows per warp pass
    const int w = tid >> 5, lane = tid & 31;
    const int off = (lane % LPR) * 16;
    if (off >= d.nbytes) return;
    for (int i = w * RPW + lane / LPR; i < 16; i += 4 * RPW) {
        const int t = tl0 + i;
        if (t >= ntok) break;
        const long long rowi = d.by_pos ? (long long)s_pos[t] : (long long)(m0 + t);
        char *dst = d.base + rowi * d.ld + off;
        const uint8_t *src = stage + i * RB + off;
        if (d.vec && off + 16 <= d.nbytes) {
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
        } else {
            const int nb = min(16, d.nbytes - off);
            for (int b = 0; b < nb; b += es) {
                if constexpr (es == 4) *reinterpret_cast<float *>(dst + b) = *reinterpret_cast<const float *>(src + b);
                else *reinterpret_cast<__half *>(dst + b) = *reinterpret_cast<const __half *>(src + b);
            }
        }
    }
}

// ───────────── the kernel ─────────────
// Launched as clusters of two CTAs (a pair on one TPC).  Pair p owns the stream-K unit
// range of pair tile pt = 256 weight rows: the even CTA (rank 0) dequantizes rows
// [256 pt, +128), the odd one rows [256 pt + 128, +128); each CTA loads its half of the
// token group's activation rows.  The even CTA issues the paired MMA (M = 256) and its
// commits arrive on the barriers of both CTAs; each CTA's epilogue drains its own TMEM.
// Barriers the MMA waits on (full_a, full_b, acc_empty) live in the even CTA; the odd
// CTA's loads and arrivals reach them through cluster addresses.
//
// Shared memory (per CTA): [A ring (F16 weights only): a_stages x 16 KB][B ring][raw ring]
// [barriers][token positions][contributor offsets].  Slice i (64 k) of the CTA's unit
// range uses A stage i % a_stages (TMEM columns kTmemA + 32 stage for quantized weights)
// and part i % spb of B slot (i / spb) % nbs.
//
// Warps (warp_role): w0 activation producer, w1 MMA issuer (even CTA) + TMEM owner, w2
// weight-chunk producer (F16 weights: A-tile TMA producer), w3 relay, w4-w11 dequantizers
// (two sets of four; thread = weight row = TMEM lane), w12-w19 epilogue (thread = TMEM
// lane; w12-15 and w16-19 take alternate 16-column chunks).
template <int WT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ XMaps xm, GemmParams p) {
    constexpr int RAWB = raw_chunk_bytes(WT);
    constexpr int NA = a_stages(WT), NRAW = raw_stages(WT), BRING = b_ring_bytes(WT), AR = a_ring_bytes(WT);
    constexpr int CPR = raw_cpr(WT), RSB = CPR * RAWB;  // chunks and bytes per raw stage
    // The relay frees the B slot of slice j - NA while it handles slice j, after waiting
    // for the B loads up to slice j - 1: with one slice per load (the widest group, 12 KB
    // loads) the producer needs 2 + (NA - 1) slots not to wait on itself.
    static_assert(BRING / (kMaxTok / 2 * 128) >= 2 + (NA - 1), "B ring too shallow for the A ring");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *aring = smem;  // F16 weights only
    uint8_t *bring = smem + AR;
    uint8_t *raw = bring + BRING;
    uint8_t *epi_stage = raw + NRAW * RSB;  // [2 halves][kEpiStageBytes]
    uint64_t *bars = reinterpret_cast<uint64_t *>(epi_stage + 2 * kEpiStageBytes);
    uint64_t *full_a = bars, *empty_a = bars + 6, *full_b = bars + 12, *empty_b = bars + 36, *raw_full = bars + 60,
             *raw_empty = bars + 64, *acc_full = bars + 68, *acc_empty = bars + 70, *drain = bars + 72,
             *fix_bar = bars + 73;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 74);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 75);
    volatile int *okflag = reinterpret_cast<volatile int *>(bars + 77);
    int *s_pos = reinterpret_cast<int *>(bars + kBarBytes / 8);                   // [kMaxTok]
    long long *s_contrib = reinterpret_cast<long long *>(s_pos + kMaxTok);        // [kMaxContrib]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    // the next kernel of the stream may be scheduled now; it waits for this grid itself
    griddep_launch_dependents();
    if (threadIdx.x == 0) {
        GEMM_STAMP(p, 0);
        for (int i = 0; i < NA; i++) {
            // both CTAs' relays + F16: the expect_tx / else four dequant warps per CTA
            mbar_init(&full_a[i], WT == W_F16 ? 3 : 10);
            mbar_init(&empty_a[i], 1);                   // the paired MMA's commit
        }
        for (int i = 0; i < kMaxBSlots; i++) {
            mbar_init(&full_b[i], 1);   // the producer's expect_tx
            mbar_init(&empty_b[i], 1);  // the relay, once the MMA that read the slot completed
        }
        for (int i = 0; i < NRAW; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kDeqWarps);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 2 * kEpiThreads / 32);  // every epilogue warp of both CTAs
        }
        mbar_init(drain, 1);
        mbar_init(fix_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    const int role = warp_role(warp);
    if (WT == W_F16 && role == R_WPROD && lane == 0) prefetch_tmap(&tm_w);
    if (role == R_MMA) {
        tmem_alloc2(tmem_holder, 512);
        tmem_relinquish2();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // barriers of both CTAs initialised, TMEM of both allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    // The schedule needs only the token count, which is final before any GEMM of a
    // forward starts (the step-preparation kernel or the host writes it ahead of the
    // forward's first launch), and the weights do not depend on the previous kernel.  So
    // the weight producer and the dequantizers start now and fill the pipeline while the
    // previous kernel finishes; the activation producer and the epilogue wait for it
    // (griddepcontrol.wait) before they read or write anything it touches, and the MMAs
    // wait for the activations.
    const int M = *reinterpret_cast<volatile const int *>(p.m_dev);
    Sched S;
    S.init(M, p.n_tiles >> 1, p.kb, n_pairs, pair, BRING);
    const int NBS = S.nbs;
    // barriers of the even CTA as cluster addresses
    const uint32_t full_a0 = mapa_shared(full_a, 0), acc_empty0 = mapa_shared(acc_empty, 0);

    if (role == R_BPROD) {
        // ── activation producer (both CTAs, local barriers): this CTA's half of the
        //    token group, spb k-slices per tensor load.  Few large loads: the TMA unit
        //    also streams the weights and handles only a few operations per microsecond. ──
        griddep_wait();  // the activations are the previous kernel's output
        if (lane == 0) {
            GEMM_STAMP(p, 1);
            if (*reinterpret_cast<volatile const int *>(p.m_dev) != M) atomicCAS(p.err, 0, kErrTimeout + 14);
            const CUtensorMap *xmap = &xm.m[S.bh / 16 - 1];
            int ob = 0, sl = 0;  // B loads issued, slot of the next one
            uint32_t ph = 0;     // ring pass parity of the next load
            bool ok = true;
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                const int row0 = g.m0 + (int)rank * g.half;
                for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                    for (int s = 0; s < 4; s += S.spb) {
                        if (!(ok = mbar_wait(&empty_b[sl], ph ^ 1, abort_flag, p.err, kErrTimeout + 2))) break;
                        mbar_arrive_expect_tx(&full_b[sl], S.bslot);
                        tma_load_3d(bring + sl * S.bslot, xmap, 0, row0, kbi * 4 + s, &full_b[sl]);
                        GEMM_EVENT(p, 0, ob);
                        ob++;
                        if (++sl == NBS) { sl = 0; ph ^= 1; }
                    }
                }
                u += g.k1 - g.k0;
            }
            GEMM_STAMP(p, 2);
            if (!ok) {
                // let the copies in flight land before the CTA can exit
                for (int i = (ob > NBS ? ob - NBS : 0); i < ob; i++) spin_bounded(&full_b[i % NBS], (i / NBS) & 1);
            }
        }
        __syncwarp();
    } else if (role == R_WPROD) {
        if constexpr (WT != W_F16) {
            // ── weight-chunk producer: this CTA's re-tiled chunk (128 rows x 256 k) per k-block ──
            if (lane == 0) {
                auto chunk = [&](int u) {
                    const int ot = u / S.kb, kbi = u % S.kb;
                    return p.w + ((size_t)(2 * (ot / S.n_mg) + rank) * p.kb + kbi) * RAWB;
                };
                int rit = 0;
                bool ok = true;
                for (int u = S.u0; u < S.u1 && ok; u += CPR) {
                    const int r = rit % NRAW;
                    if (!(ok = mbar_wait(&raw_empty[r], ((rit / NRAW) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 1))) break;
                    const int nch = min(CPR, S.u1 - u);
                    mbar_arrive_expect_tx(&raw_full[r], nch * RAWB);
                    for (int c = 0; c < nch; c++) bulk_g2s(raw + r * RSB + c * RAWB, chunk(u + c), RAWB, &raw_full[r]);
                    GEMM_EVENT(p, 1, rit);
                    rit++;
                }
                if (!ok)
                    for (int i = (rit > NRAW ? rit - NRAW : 0); i < rit; i++)
                        spin_bounded(&raw_full[i % NRAW], (i / NRAW) & 1);
            }
        } else {
            // ── F16 weights: A-tile TMA producer (completions counted on the even CTA) ──
            if (lane == 0) {
                int it = 0;
                bool ok = true;
                for (int u = S.u0; u < S.u1 && ok;) {
                    const Seg g = make_seg(S, u, S.u1);
                    for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                        for (int s = 0; s < 4; s++) {  // one stage = one k-slice
                            const int st = it % NA;
                            if (!(ok = mbar_wait(&empty_a[st], ((it / NA) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 11))) break;
                            if (rank == 0) mbar_arrive_expect_tx(&full_a[st], 2 * kABytes);
                            tma_load_2d_pair(aring + st * kABytes, &tm_w, kbi * 256 + s * 64, (2 * g.pt + (int)rank) * 128,
                                             full_a0 + 8 * st);
                            it++;
                        }
                    }
                    u += g.k1 - g.k0;
                }
                if (!ok) {
                    if (rank == 0)
                        for (int i = (it > NA ? it - NA : 0); i < it; i++) spin_bounded(&full_a[i % NA], (i / NA) & 1);
                    const uint64_t t0 = globaltimer();
                    while (globaltimer() - t0 < 50000) {}
                }
            }
        }
        __syncwarp();
    } else if (role == R_MMA) {
        // ── MMA issuer (even CTA) ──
        // Every instruction on this thread's path between two slices leaves the tensor
        // pipe idle (the queue holds about one MMA), so the per-slice work is only: wait
        // for the stage, fence, four MMAs, commit.  Each unit is one k-block = four
        // slices, so the A stage of slice s2 is s2 (a_stages == 4) and its barrier parity
        // flips per k-block; the four B descriptors are computed once per k-block.
        static_assert(NA == 4, "one A stage per k-slice of a k-block");
        if (lane == 0 && rank == 0) {
            int si = 0, ka = 0;  // accumulator segments, k-blocks consumed
            bool ok = true, issued = false;
#ifdef DFB_GEMM_TRACE
            long long tr_nwait = 0, tr_wcyc = 0, tr_t0 = clock64();
#endif
            const uint64_t bdesc0 = sw128_desc(smem_u32(bring)), adesc0 = sw128_desc(smem_u32(aring));
            const int lg_spb = S.spb == 1 ? 0 : S.spb == 2 ? 1 : 2;  // B slices per ring slot: 1, 2 or 4
            const uint32_t bpart_bytes = S.bh * 128;
            int bslot = 0;  // ring slot of the first slice of the next k-block
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                const int acc = S.acc_of(si);
                if (!(ok = mbar_wait(&acc_empty[acc], (S.acc_uses(si) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 3))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kDblTok;
                const uint32_t idesc = idesc_f16(256, (uint32_t)g.nmma);
                uint32_t accum = 0;
                for (int kbi = g.k0; kbi < g.k1; kbi++, ka++) {
                    uint64_t bd[4];
#pragma unroll
                    for (int s2 = 0; s2 < 4; s2++) {
                        int sl = bslot + (s2 >> lg_spb);
                        if (sl >= NBS) sl -= NBS;
                        bd[s2] = bdesc0 + (uint64_t)((sl * S.bslot + (s2 & (S.spb - 1)) * bpart_bytes) >> 4);
                    }
                    bslot += 4 >> lg_spb;
                    if (bslot >= NBS) bslot -= NBS;
                    const uint32_t par = ka & 1;
#pragma unroll
                    for (int s2 = 0; s2 < 4; s2++) {
                        // full_a also carries the relays' arrivals: this stage's B rows have landed
#ifdef DFB_GEMM_TRACE
                        if (!mbar_try_wait(&full_a[s2], par)) {
                            const long long w0 = clock64();
                            ok = mbar_wait(&full_a[s2], par, abort_flag, p.err, kErrTimeout + 5);
                            tr_nwait++;
                            tr_wcyc += clock64() - w0;
                        }
                        if (!ok) break;
#else
                        if (!(ok = mbar_wait(&full_a[s2], par, abort_flag, p.err, kErrTimeout + 5))) break;
#endif
                        tc_fence_after();
                        if constexpr (WT == W_F16)
                            mma2_f16_ss_k64(d_tmem, adesc0 + (uint64_t)((s2 * kABytes) >> 4), bd[s2], idesc, accum);
                        else
                            mma2_f16_ts_k64(d_tmem, tmem_base + kTmemA + s2 * kTmemAStage, bd[s2], idesc, accum);
                        accum = 1;
                        mma2_commit_mc(&empty_a[s2], 0x3);
                        GEMM_EVENT(p, 4, 4 * ka + s2);
                    }
                    issued = true;
                    if (!ok) break;
                }
                if (!ok) break;
                mma2_commit_mc(&acc_full[acc], 0x3);
                si++;
                u += g.k1 - g.k0;
            }
            GEMM_STAMP(p, 3);
#ifdef DFB_GEMM_TRACE
            if (p.trace && blockIdx.x < 4) {  // full_a waits that had to block: count, cycles; loop cycles; slices
                unsigned long long *tp = p.trace + 256 * 16 + ((size_t)blockIdx.x * 8 + 5) * 64 + 56;
                tp[0] = tr_nwait; tp[1] = tr_wcyc; tp[2] = clock64() - tr_t0; tp[3] = 4 * ka;
            }
#endif
            if (issued) {
                // every MMA must have retired before TMEM is released
                mma2_commit(drain);
                spin_bounded(drain, 0);
            }
        }
        __syncwarp();
    } else if (role == R_RELAY) {
        // ── relay (one thread per CTA), slice by slice: once the MMA of slice j - NA has
        //    completed (empty_a, the same wait the A writers do), its B slot is free again
        //    (after the last slice of the slot's load); once this CTA's B rows of slice j
        //    have landed (full_b), arrive on full_a of slice j in the even CTA.  The MMA issuer so waits on one barrier per stage, and no relay
        //    can fall a full phase behind the barriers it polls. ──
        if (lane == 0) {
            int n_it = 0;
            for (int u = S.u0; u < S.u1;) {
                const Seg g = make_seg(S, u, S.u1);
                n_it += 4 * (g.k1 - g.k0);
                u += g.k1 - g.k0;
            }
            bool ok = true;
            const int spb = S.spb;
            // running ring positions (no divisions): B load of slice j and of slice j - NA
            int fo_sl = 0, fo_part = 0, eo_sl = 0, eo_part = 0;
            uint32_t fo_ph = 0;
            for (int j = 0; j < n_it + NA && ok; j++) {  // A stage = slice j
                if (j >= NA) {
                    // MMA of slice j - NA done (phase (j - NA) / NA of empty_a[j % NA]); its B
                    // slot is free once the last slice of the slot's load is done
                    if (!(ok = mbar_wait(&empty_a[j % NA], ((j / NA) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 12))) break;
                    if (++eo_part == spb) {
                        eo_part = 0;
                        mbar_arrive(&empty_b[eo_sl]);
                        if (++eo_sl == NBS) eo_sl = 0;
                    }
                }
                if (j < n_it) {
                    if (fo_part == 0)
                        if (!(ok = mbar_wait(&full_b[fo_sl], fo_ph, abort_flag, p.err, kErrTimeout + 4))) break;
                    mbar_arrive_cluster(full_a0 + 8 * (j % NA));
                    if (++fo_part == spb) {
                        fo_part = 0;
                        if (++fo_sl == NBS) { fo_sl = 0; fo_ph ^= 1; }
                    }
                }
            }
        }
        __syncwarp();
    } else if (role == R_DEQ) {
        // ── dequantizers: thread = weight row of this CTA's tile; set p takes slices
        //    p and p + 2 of every k-block ──
        if constexpr (WT != W_F16) {
            const int di = deq_index(warp);
            const int set = di >> 2;
            const int r = (di & 3) * 32 + lane;
            int rit = 0;
            bool ok = true;
            // This warp's TMEM lane quarter holds its 32 weight rows of every A stage.
            const uint32_t a_lane = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + kTmemA;
            // The stage's tcgen05.st have completed; order them before the arrival the MMA
            // issuer waits on (no shared memory, so no proxy fence).
            auto publish = [&](int st) {
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(full_a0 + 8 * st);
            };
            // Lane 0 waits and the warp takes its verdict; then every
            // lane observes the completed phase itself (one try_wait, which succeeds: the
            // phase cannot advance further without this warp), for acquire ordering.
            auto wait_warp = [&](uint64_t *bar, uint32_t parity, int code) {
                int okw = 1;
                if (lane == 0) okw = mbar_wait(bar, parity, abort_flag, p.err, code);
                const bool okb = __shfl_sync(0xffffffffu, okw, 0) != 0;
                if (okb) (void)mbar_try_wait(bar, parity);
                return okb;
            };
            auto wait_a = [&](int ia) {
                return wait_warp(&empty_a[ia % NA], ((ia / NA) & 1) ^ 1, kErrTimeout + 7);
            };
            const int n_units = S.u1 - S.u0;
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                    // unit rit of the range: raw stage rit / CPR, chunk rit % CPR in it
                    const int rst = rit / CPR, rs = rst % NRAW;
                    if (rit % CPR == 0) {
                        ok = wait_warp(&raw_full[rs], (rst / NRAW) & 1, kErrTimeout + 6);
                        if (!ok) break;
                        if (r == 0 && set == 0) GEMM_EVENT(p, 2, rst);
                    }
                    const uint8_t *R = raw + rs * RSB + (rit % CPR) * RAWB;
                    // this set's k-slices of the k-block: set and set + 2, one A stage each
                    uint32_t o[32];
                    if constexpr (WT == W_Q4K) {
                        Q4KMeta meta;
                        q4k_load_meta(R, r, set, meta);
                        #pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int sl = set + 2 * h, ia = 4 * rit + sl;
                            q4k_slice(R, r, sl, 2 * h, meta, o);
                            if (!(ok = wait_a(ia))) break;
                            tc_fence_after();  // after the MMA that read this stage
                            if (r == 0 && ia < 32) GEMM_EVENT(p, 7, ia);
                            tmem_st32(a_lane + (ia % NA) * kTmemAStage, o);
                            publish(ia % NA);
                            if (r == 0) GEMM_EVENT(p, 3, ia);
                        }
                    } else if constexpr (WT == W_Q6K) {
                        Q6KMeta meta;
                        q6k_load_meta(R, r, set, meta);
                        #pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int sl = set + 2 * h, ia = 4 * rit + sl;
                            Q6KHalf qv;
                            q6k_load_half(R, r, h, qv);  // slice sl uses half sl / 2 = h of ql / qh
                            q6k_slice(qv, sl, 4 * h, meta, o);
                            if (!(ok = wait_a(ia))) break;
                            tc_fence_after();
                            tmem_st32(a_lane + (ia % NA) * kTmemAStage, o);
                            publish(ia % NA);
                        }
                    } else {
                        #pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int sl = set + 2 * h, ia = 4 * rit + sl;
                            q80_slice(R, r, sl, o);
                            if (!(ok = wait_a(ia))) break;
                            tc_fence_after();
                            tmem_st32(a_lane + (ia % NA) * kTmemAStage, o);
                            publish(ia % NA);
                        }
                    }
                    __syncwarp();
                    if (lane == 0 && (rit % CPR == CPR - 1 || rit == n_units - 1)) mbar_arrive(&raw_empty[rs]);
                    rit++;
                }
                u += g.k1 - g.k0;
            }
        }
    } else {
        // ── epilogue: thread = TMEM lane = output feature of this CTA's tile ──
        griddep_wait();  // outputs, workspace and counters are the previous kernel's until it completes
        // A whole tile is finished straight from TMEM.  A split tile's partial goes to
        // the workspace (f32 [column / 4][row][column % 4], slot 0 for the pair's first
        // tile, 1 for its last) and its arrival is counted; once every MMA of this CTA is done, each
        // contributor of a split tile finishes its share of the tile's 16-column chunks,
        // summing all contributors' partials in contributor order (so the result does
        // not depend on timing), staged into the drained rings by bulk copies.
        const int q = warp & 3;
        const int row = 32 * q + lane;
        const int half = epi_half(warp);
        const int et = half * 128 + q * 32 + lane;  // 0..255
        const int tid_h = q * 32 + lane;            // 0..127 within the half
        uint8_t *my_stage = epi_stage + half * kEpiStageBytes;
        int si = 0;
        bool ok = true;
        const int first_ot = S.begin_of(pair) / S.kb;
        int split_u0 = -1, split_u1 = -1;  // first units of this CTA's split segments (first, last)
        auto release_acc = [&](int acc) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * acc);
        };
        for (int u = S.u0; u < S.u1 && ok;) {
            const Seg g = make_seg(S, u, S.u1);
            const int tile = 2 * g.pt + (int)rank;
            const int acc = S.acc_of(si);
            // one thread waits, the barrier hands the outcome to the whole group
            if (et == 0) *okflag = mbar_wait(&acc_full[acc], S.acc_uses(si) & 1, abort_flag, p.err, kErrTimeout + 8) ? 1 : 0;
            named_bar_sync(1, kEpiThreads);
            ok = *okflag != 0;
            if (!ok) break;
            if (et == 0 && si < 4) GEMM_STAMP(p, 4 + 2 * si);
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + acc * kDblTok;
            const bool whole = g.k0 == 0 && g.k1 == S.kb;
            if (whole) {
                const EpiRow er = epi_row<EPI>(p.epi, tile, row);
                const EpiDst dd = epi_dst<EPI>(p.epi, tile);
                if constexpr (EPI == EPI_QKV || EPI == EPI_LOGITS) {
                    for (int t = et; t < g.ntok; t += kEpiThreads) s_pos[t] = p.epi.pos[g.m0 + t];
                    named_bar_sync(1, kEpiThreads);
                }
                for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                    uint32_t u16[16];
                    tmem_ld16(taddr + c0, u16);
                    tmem_ld_wait();
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(u16[i]);
                    epi_values<EPI>(p.epi, er, s_pos, c0, g.ntok, v, my_stage);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                    epi_copyout<EPI>(dd, s_pos, g.m0, c0, g.ntok, my_stage, tid_h);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                }
                release_acc(acc);
            } else {
                const int slot = g.ot == first_ot ? 0 : 1;
                float *wsl = p.ws + ((size_t)blockIdx.x * 2 + slot) * kWsTile;
                if (et == 0) GEMM_EVENT(p, 6, 5 * si + 0);
                for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                    uint32_t u16[16];
                    tmem_ld16(taddr + c0, u16);
                    tmem_ld_wait();
                    float *dst = wsl + (size_t)c0 * 128 + row * 4;  // column group c0/4, this row
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        *reinterpret_cast<uint4 *>(dst + j * 512) =
                            make_uint4(u16[4 * j], u16[4 * j + 1], u16[4 * j + 2], u16[4 * j + 3]);
                }
                // the accumulator is in registers / on its way to the workspace
                release_acc(acc);
                __threadfence();
                named_bar_sync(1, kEpiThreads);
                if (et == 0) atomicAdd(&p.tile_cnt[2 * g.ot + rank], 1);
                if (slot == 0) split_u0 = u;
                else split_u1 = u;
                if (et == 0) GEMM_EVENT(p, 6, 5 * si + 3);
            }
            named_bar_sync(1, kEpiThreads);  // okflag / s_pos are reused by the next segment
            if (et == 0 && si < 4) GEMM_STAMP(p, 5 + 2 * si);
            si++;
            u += g.k1 - g.k0;
        }

        // ── deferred split-tile fixups: every MMA of this CTA has completed, so the rings
        //    (everything below the barriers) are free for staging ──
        constexpr int kStageBytes = AR + BRING + NRAW * RSB;
        constexpr int kChunkBytes = 16 * 128 * 4;  // one 16-column chunk of one partial
        const float *sbuf = reinterpret_cast<const float *>(smem);
        uint32_t fix_phase = 0;
        for (int i = 0; i < 2 && ok; i++) {
            const int su = i == 0 ? split_u0 : split_u1;
            if (su < 0) continue;
            const Seg g = make_seg(S, su, S.u1);
            const int tile = 2 * g.pt + (int)rank;
            const int c_first = S.owner(g.ot * S.kb), c_last = S.owner((g.ot + 1) * S.kb - 1);
            const int nc = c_last - c_first + 1, me = pair - c_first;
            const int nch = g.nmma >> 4;
            const int ch0 = me * nch / nc, ch1 = (me + 1) * nch / nc;
            int *cntp = p.tile_cnt + 2 * g.ot + rank;
            if (et < nc && et < kMaxContrib) {
                const int c = c_first + et;
                const int sl = (S.begin_of(c) / S.kb == g.ot) ? 0 : 1;
                s_contrib[et] = ((long long)(2 * c + (int)rank) * 2 + sl) * kWsTile;
            }
            if constexpr (EPI == EPI_QKV || EPI == EPI_LOGITS) {
                for (int t = et; t < g.ntok; t += kEpiThreads) s_pos[t] = p.epi.pos[g.m0 + t];
            }
            if (et == 0) {
                int okw = nc <= kMaxContrib;  // the launcher keeps nc <= kMaxContrib
                if (!okw) atomicCAS(p.err, 0, kErrTimeout + 9);
                else okw = wait_count(cntp, nc, abort_flag, p.err, kErrTimeout + 13);
                *okflag = okw;
                if (okw) fence_proxy_async_all();  // the partials, seen here, before the bulk reads
            }
            named_bar_sync(1, kEpiThreads);
            ok = *okflag != 0;
            if (!ok) break;
            if (et == 0) GEMM_EVENT(p, 6, 5 * si + 0);
            const EpiRow er = epi_row<EPI>(p.epi, tile, row);
            const EpiDst dd = epi_dst<EPI>(p.epi, tile);
            const bool staged = nc * kChunkBytes <= kStageBytes;
            const int per_round = staged ? kStageBytes / (nc * kChunkBytes) : 1;
            for (int r0 = ch0; r0 < ch1; r0 += per_round) {
                const int nr = min(ch1, r0 + per_round) - r0;
                if (staged) {
                    if (et == 0) {
                        mbar_arrive_expect_tx(fix_bar, (uint32_t)(nc * nr * kChunkBytes));
                        for (int c = 0; c < nc; c++)
                            bulk_g2s(smem + (size_t)c * nr * kChunkBytes, p.ws + s_contrib[c] + (size_t)r0 * 2048,
                                     (uint32_t)(nr * kChunkBytes), fix_bar);
                        *okflag = mbar_wait(fix_bar, fix_phase, abort_flag, p.err, kErrTimeout + 10) ? 1 : 0;
                    }
                    fix_phase ^= 1;
                    named_bar_sync(1, kEpiThreads);
                    if (!*okflag) { ok = false; break; }
                    if (et == 0 && r0 == ch0) GEMM_EVENT(p, 6, 5 * si + 1);
                }
                for (int ch = r0 + half; ch < r0 + nr; ch += 2) {
                    float v[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) v[k] = 0.f;
                    for (int c = 0; c < nc; c++) {
                        float4 t[4];
                        if (staged) {
                            const float4 *src =
                                reinterpret_cast<const float4 *>(sbuf + ((size_t)c * nr + (ch - r0)) * 2048 + row * 4);
#pragma unroll
                            for (int j = 0; j < 4; j++) t[j] = src[j * 128];
                        } else {
                            const float4 *src = reinterpret_cast<const float4 *>(p.ws + s_contrib[c] + (size_t)ch * 2048 + row * 4);
#pragma unroll
                            for (int j = 0; j < 4; j++) t[j] = __ldcg(src + j * 128);
                        }
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            v[4 * j] += t[j].x;
                            v[4 * j + 1] += t[j].y;
                            v[4 * j + 2] += t[j].z;
                            v[4 * j + 3] += t[j].w;
                        }
                    }
                    epi_values<EPI>(p.epi, er, s_pos, ch * 16, g.ntok, v, my_stage);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                    epi_copyout<EPI>(dd, s_pos, g.m0, ch * 16, g.ntok, my_stage, tid_h);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                }
                // staged chunks consumed before the next round's copies; generic reads of the
                // staging area before the async-proxy writes
                named_bar_sync(1, kEpiThreads);
                if (et == 0) fence_proxy_async_smem();
                if (et == 0 && r0 == ch0) GEMM_EVENT(p, 6, 5 * si + 2);
            }
            if (!ok) break;
            // departure: the last of the nc contributors resets the counter for the next launch
            if (et == 0) {
                const int old = atomicAdd(cntp, 1);
                if (old == 2 * nc - 1) *cntp = 0;
                GEMM_EVENT(p, 6, 5 * si + 4);
            }
            named_bar_sync(1, kEpiThreads);  // s_contrib / s_pos / okflag reused
            si++;
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no remote arrival or copy of either CTA is still in flight
    if (threadIdx.x == 0) GEMM_STAMP(p, 12);
    if (role == R_MMA) {
        tc_fence_after();
        tmem_dealloc2(tmem_base, 512);
    }
}

}  // namespace dfb
