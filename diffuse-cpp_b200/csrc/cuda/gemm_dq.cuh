// Dequant-fused tcgen05 GEMM:  Y[tok][n] = sum_k X[tok][k] * W[n][k]
//
// Replaces every ggml_mul_mat(W, x) of the reference forward (src/diffuse-graph.cpp
// :61-63, 122, 136-140, 154 and the cached variants :451-453, 556, 570-574, 587).
//
// Precision.  Each operand is split, v = hi + lo with hi = f16(v), and the product is
// W_hi.X_hi + W_hi.X_lo + W_lo.X_hi in one f32 accumulator (the dropped W_lo.X_lo term is
// ~2^-22 of it): the main term as an f16 MMA, the two corrections (~2^-11 of it, needed
// to ~5 bits) as one E4M3 MMA (kind::f8f6f4, twice the f16 rate) over the operand pairs
// [W_hi 2^-10 | W_lo] x [X_lo 2^10 | X_hi], whose products land at their true scale.
// Per element that is ~2^-17 of the product, below the f32 accumulation error over K.
// Quantized weights are dequantized in f32 (exact: Q4_K d*sc*q - dmin*m is one f32
// rounding, Q6_K / Q8_0 products are exact) after a power-of-two pre-scale that puts the
// largest near 2^14; the epilogue undoes the scale.  F16 / F32 / BF16 weights come as
// precomputed f16 hi and E4M3 correction matrices.  For plain f16 activations (XS = 1, the
// allocation-free entry point) the weights are split into f16 hi and lo instead (two f16
// MMAs, exact products).
//
// Operands.  W is the GGUF weight (Q4_K / Q6_K / Q8_0 raw blocks re-tiled at load, or
// f16 matrices); X is the activation matrix [tokens][K] in "pair" layout: per 64-wide
// k-slice, 64 hi f16 then 64 E4M3 X_lo 2^10 and 64 E4M3 X_hi (256 bytes, dequant.cuh).
// The MMA is "swap-AB" and
// paired (tcgen05 cta_group::2, M = 256): the A operand is a tile of 256 output
// features, 128 dequantized into the TMEM of each CTA of a pair (f16 weights: TMA-loaded
// into shared memory, 128-byte-swizzled K-major); the B operand is a group of up to 256
// tokens of X, each CTA holding half of them (TMA tensor loads into shared memory, same
// swizzle).  The f32 accumulator lives in TMEM: lane = output feature, column = token.
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
#include <type_traits>
#include "dequant.cuh"
#include "ptx.cuh"

namespace dfb {

// W_F16: one f16 matrix (exact); W_F32: hi and lo f16 matrices of F32 / BF16 weights.
enum WType : int { W_Q4K = 0, W_Q6K = 1, W_Q80 = 2, W_F16 = 3, W_F32 = 4 };
__host__ __device__ constexpr bool w_smem(int wt) { return wt == W_F16 || wt == W_F32; }  // A by TMA into shared memory
__host__ __device__ constexpr bool w_split(int wt) { return wt != W_F16; }               // A has a lo part
// EPI_F32: f32 rows; EPI_QKV: Q rows and K/V cache rows (f32) with bias and RoPE;
// EPI_SWIGLU: silu(gate) * up as pair-layout rows (the down projection's X);
// EPI_LOGITS: f32 rows at the tokens' positions.
enum EpiKind : int { EPI_F32 = 0, EPI_QKV = 3, EPI_SWIGLU = 4, EPI_LOGITS = 5 };

// Bytes of one re-tiled chunk (128 rows x one k-block of 256 elements).
__host__ __device__ constexpr int raw_chunk_bytes(int wt) {
    return wt == W_Q4K ? 128 * 144 : wt == W_Q6K ? 128 * 210 : wt == W_Q80 ? 128 * 272 : 0;
}

struct EpiArgs {
    void *out = nullptr;   // F32 / SWIGLU / LOGITS destination
    int ld = 0;            // its row stride (elements; SWIGLU: f16 elements of the pair rows)
    int n_valid = 0;       // valid output features (rows of W before padding)
    float out_scale = 1.f; // undoes the weights' power-of-two pre-scale (exact)
    // QKV (f32 outputs)
    float *q_out = nullptr;
    int ld_q = 0;
    float *k_cache = nullptr, *v_cache = nullptr;  // [position][n_kv] of this layer
    int ld_kv = 0;
    int n_q_tiles = 0, n_k_tiles = 0;  // tiles in the (padded) Q and K sections
    int n_q = 0, n_kv = 0, head_dim = 0;
    const float *bias = nullptr;       // [(n_q_tiles + 2 n_k_tiles) * 128], section-padded, original order
    const float2 *rope = nullptr;      // [position][head_dim/2] (cos, sin)
    const int *pos = nullptr;          // [tokens] position of each row (QKV cache rows, LOGITS rows)
    const int *rope_pos = nullptr;     // [tokens] position within its sequence (QKV RoPE angles)
};

// Activation tensor maps, one per token half-group size h = 16 (i + 1), i = 0..7: a 3-D
// view {64 k, rows, XS * K / 64 slices} of the row-major activation matrix (XS = 2: pair
// layout, a hi slice then a lo slice per 64-wide k-slice; XS = 1: plain f16), strides
// row, then 128 B; box {64, h, XS * x_slices(h)}, 128-byte swizzle.  One load brings
// x_slices consecutive k-slices (both parts) of h rows, each part in the canonical
// K-major SW128 layout.
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
    float wscale = 1.f;          // power-of-two pre-scale of the dequantized weights
    int lo_row = 0;              // f16 tile weights: row of the lo matrix (W_F32) in the tensor map
    int corr_row = 0;            // f16 tile weights: row of the correction matrix in the tensor map
    const int *m_dev = nullptr;  // token count (device)
    float *ws = nullptr;         // split-tile partials [grid][2][256 * 128]
    int *tile_cnt = nullptr;     // [n_tiles x token groups] arrival + departure counters, left at 0
    int *err = nullptr;          // first error code of any CTA
    unsigned long long timeout_ns = 4000000000ull;  // limit of every wait (4 s; tests shorten it)
    EpiArgs epi;
};

constexpr int kThreads = 640;            // 20 warps, roles below
constexpr int kEpiThreads = 256;         // two epilogue warps per TMEM lane quarter
constexpr int kDeqWarps = 8;             // two sets of four: even / odd k-slices
constexpr int kSliceBytes = 128 * 128;   // one 64-wide k-slice of this CTA's 128 weight rows (f16)
constexpr int kMaxTok = 256;             // tokens per MMA group (N) of the pair
constexpr int kDblTok = 192;             // groups up to this size double-buffer the accumulator
// (an MMA's N is the group rounded up to 32: the limits are multiples of 32 so a
// double-buffered accumulator never reaches the next one or the A stages)
static_assert(kDblTok % 32 == 0, "double-buffered accumulator width");
constexpr int kDbl4Tok = 128;            // ... and groups up to this size also get four A stages
constexpr int kWsTile = kMaxTok * 128;   // floats per partial tile (one CTA's 128 rows)
constexpr int kErrTimeout = 0x100;
constexpr int kMaxAStages = 6, kMaxBSlots = 24, kMaxRawStages = 4;
// TMEM (512 columns per CTA), by token-group size (Sched::init):
//   <= 128: accumulators [0, 128), [128, 256), four A stages at [256, 512);
//   <= 192: accumulators [0, 192), [192, 384), two A stages at [384, 512);
//   larger: one accumulator [0, 256) (the MMA of the next segment waits for the epilogue to
//           drain it, which costs less than dequantizing the weights once per group of
//           128), four A stages at [256, 512).
// An A stage (quantized weights) holds one k-slice, lane = weight row: f16 hi in the first
// 32 columns, then the E4M3 correction pair (16 columns W_hi 2^-10, 16 columns W_lo), or
// f16 lo for XS = 1.  Dequantizer set p fills the stages of its slices (p, or p and p + 2
// alternately with four stages), so with four stages a set runs a whole slice ahead of the
// MMA that frees its previous stage.  f16 / f32 weight tiles come through shared memory
// (two stages) instead; their accumulators are always double-buffered ([0, 256), [256, 512)).
constexpr int kTmemAStage = 64;
constexpr int kTmemALo = 32;
constexpr int kNA = 2;                   // shared-memory A stages (f16 / f32 weight tiles)
constexpr int kMaxNA = 4;                // TMEM A stages
static_assert(2 * kDblTok + 2 * kTmemAStage <= 512 && 2 * kDbl4Tok + 4 * kTmemAStage <= 512 &&
              kMaxTok + 4 * kTmemAStage <= 512, "TMEM columns");
// The relay returns the activation slot of slice j - kRelayLag while it handles slice j.
constexpr int kRelayLag = 2;

// Rings per weight type, sized so that shared memory (227 KB) holds them:
//  A        one k-slice per stage: dequantized weights go to TMEM (two or four stages, see
//           above; written by tcgen05.st, read by the MMA from TMEM: no shared-memory round
//           trip and no proxy fence, which cost ~1.2k cycles per warp and stage); f16
//           weight tiles are TMA-loaded into a two-stage shared-memory ring instead (hi and
//           lo tiles for W_F32);
//  B ring   this CTA's activation rows of 1-4 k-slices per slot, so small token counts
//           keep many slices in flight and hide the L2 latency;
//  raw ring re-tiled weight chunks (one k-block of 256 for 128 rows), grouped.
__host__ __device__ constexpr int a_stages(int wt) { return kNA; }
// f16 tile weights: XS = 2 stages hold the hi and correction tiles, XS = 1 the hi tile
// (and the lo tile of W_F32)
__host__ __device__ constexpr int a_stage_bytes(int wt, int xs) {
    return (xs == 2 || wt == W_F32) ? 2 * kSliceBytes : kSliceBytes;
}
__host__ __device__ constexpr int a_ring_bytes(int wt, int xs) { return w_smem(wt) ? kNA * a_stage_bytes(wt, xs) : 0; }
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
__host__ __device__ constexpr int gemm_smem_bytes(int wt, int xs) {
    return 1024 /*align slack*/ + a_ring_bytes(wt, xs) + b_ring_bytes(wt) + raw_stages(wt) * raw_cpr(wt) * raw_chunk_bytes(wt) +
           2 * kEpiStageBytes /*epilogue output staging*/ + kBarBytes /*barriers, flags*/ + 8 * kMaxTok /*token positions*/ + 2 * 8 * kMaxContrib /*contributor partial offsets*/;
}

// Static stream-K schedule over CTA pairs, recomputed identically by every role of
// both CTAs of a pair.  Units are (pair tile of 256 weight rows, token group, k-block).
struct Sched {
    int M, n_mg, gsz, kb, n_ot, U, G, u0, u1;
    bool dbl;                 // double-buffered accumulator
    int na;                   // A stages (TMEM: 2 or 4; shared-memory tiles: 2)
    int acc_stride;           // TMEM columns between the two accumulators
    int tmem_a;               // TMEM column of A stage 0
    int bh, spb, bpart, bslot, nbs;  // B ring: rows per CTA (widest group), k-slices per load, bytes per
                                     // k-slice (all parts), slot bytes, slots
    __device__ __forceinline__ void init(int M_, int n_ptiles, int kb_, int n_pairs, int pair, int ring_bytes, int xs,
                                         bool a_in_tmem) {
        M = M_;
        kb = kb_;
        n_mg = (M + kMaxTok - 1) / kMaxTok;
        gsz = (((M + n_mg - 1) / n_mg) + 15) & ~15;
        if (!a_in_tmem) {
            dbl = true; na = kNA; acc_stride = kMaxTok; tmem_a = 0;
        } else if (gsz <= kDbl4Tok) {
            dbl = true; na = 4; acc_stride = kDbl4Tok; tmem_a = 2 * kDbl4Tok;
        } else if (gsz <= kDblTok) {
            dbl = true; na = 2; acc_stride = kDblTok; tmem_a = 2 * kDblTok;
        } else {
            dbl = false; na = 4; acc_stride = 0; tmem_a = kMaxTok;
        }
        n_ot = n_ptiles * n_mg;
        U = n_ot * kb;
        G = n_pairs < U ? n_pairs : U;
        // (unsigned 32-bit products: the launcher keeps (U + 1) * G below 2^32)
        if (M <= 0 || pair >= G) {
            u0 = u1 = 0;
        } else {
            u0 = (int)((unsigned)pair * (unsigned)U / (unsigned)G);
            u1 = (int)((unsigned)(pair + 1) * (unsigned)U / (unsigned)G);
        }
        bh = ((gsz + 31) & ~31) >> 1;  // 16..128
        if (bh < 16) bh = 16;
        spb = x_slices(bh);
        bpart = bh * 128 * xs;
        bslot = bpart * spb;
        nbs = ring_bytes / bslot;
        if (nbs > kMaxBSlots) nbs = kMaxBSlots;
    }
    // accumulator buffer of segment si and how many segments used it before
    __device__ __forceinline__ int acc_of(int si) const { return dbl ? (si & 1) : 0; }
    __device__ __forceinline__ int acc_uses(int si) const { return dbl ? (si >> 1) : si; }
    __device__ __forceinline__ int owner(int u) const { return (int)(((unsigned)(u + 1) * (unsigned)G - 1u) / (unsigned)U); }
    __device__ __forceinline__ int begin_of(int c) const { return (int)((unsigned)c * (unsigned)U / (unsigned)G); }
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

// ───────────── epilogues ─────────────

// Per-thread constants of one output tile (thread = TMEM lane = one output row).
struct EpiRow {
    int f;          // output feature written by this lane (after un-fusing)
    int col;        // its column in the tile's staging rows
    bool fvalid;    // f is a real feature (not tile padding)
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
    } else {
        r.f = tile * 128 + row;
        r.col = row;
        r.fvalid = r.f < e.n_valid;
    }
    return r;
}

// Output staging: a chunk of 16 tokens x the tile's output features, one per epilogue
// half, written by the row threads and stored to global memory as whole token rows.
// SwiGLU rows hold the tile's 64 features as one pair-layout slice (256 bytes).
template <int EPI> struct EpiFmt {
    static constexpr int esize = EPI == EPI_SWIGLU ? 2 : 4;
    static constexpr int width = 128;                  // staged elements per token row
    static constexpr int row_bytes = esize * width;    // staging row pitch
};

// Where one tile's token rows go.
struct EpiDst {
    char *base;      // the tile's first output element in row 0
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
    int n_el, e0;
    if constexpr (EPI == EPI_QKV) {
        int lt;
        const int sec = qkv_section(e, tile, lt);
        e0 = lt * 128;
        char *b = reinterpret_cast<char *>(sec == 0 ? e.q_out : sec == 1 ? e.k_cache : e.v_cache);
        d.base = b + (size_t)e0 * es;
        ld_el = sec == 0 ? e.ld_q : e.ld_kv;
        n_el = (sec == 0 ? e.n_q : e.n_kv) - e0;
        d.by_pos = sec != 0;
    } else if constexpr (EPI == EPI_SWIGLU) {
        // tile t holds features [64 t, +64): pair slice t of the output rows
        e0 = tile * 128;
        d.base = reinterpret_cast<char *>(e.out) + (size_t)e0 * es;
        ld_el = e.ld;
        n_el = (e.n_valid / 2 - tile * 64) > 0 ? 128 : 0;  // feature counts are multiples of 64
        d.by_pos = false;
    } else {
        e0 = tile * W;
        d.base = reinterpret_cast<char *>(e.out) + (size_t)e0 * es;
        ld_el = e.ld;
        n_el = e.n_valid - e0;
        d.by_pos = EPI == EPI_LOGITS;
    }
    d.ld = ld_el * es;
    d.nbytes = max(0, min(W, n_el)) * es;
    d.vec = (reinterpret_cast<uintptr_t>(d.base) % 16 == 0) && (d.ld % 16 == 0);
    return d;
}

// Epilogue math of 16 consecutive tokens (tl0 .. tl0+15 of the segment) for this lane's
// row, into the staging rows.  v holds the raw accumulator (pre-scaled weights): the
// first step multiplies by out_scale.  Called by all 32 lanes of a warp together (paired
// epilogues exchange values with the neighbouring lane).  s_rpos: the segment's token
// positions within their sequences (RoPE angles, shared memory).
template <int EPI>
__device__ __forceinline__ void epi_values(const EpiArgs &e, const EpiRow &r, const int *s_rpos, int tl0, int ntok,
                                           float (&v)[16], uint8_t *stage) {
    constexpr int RB = EpiFmt<EPI>::row_bytes;
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] *= e.out_scale;
    if constexpr (EPI == EPI_F32 || EPI == EPI_LOGITS) {
#pragma unroll
        for (int i = 0; i < 16; i++) reinterpret_cast<float *>(stage + i * RB)[r.col] = v[i];
    } else if constexpr (EPI == EPI_SWIGLU) {
        // lanes 2i (gate) and 2i + 1 (up) of feature i split the chunk's tokens: the even
        // lane takes tokens 0-7, the odd lane 8-15, each after receiving its partner's values
        // for them
        const bool odd = (threadIdx.x & 1) != 0;
        float g[8], up[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[8 + j], 1);
            g[j] = odd ? recv : v[j];
            up[j] = odd ? v[8 + j] : recv;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float hv = (g[j] / (1.0f + expf(-g[j]))) * up[j];  // silu(g) * up (ggml_silu, ggml_mul)
            // pair-layout slice: hi f16, then E4M3 lo 2^10, E4M3 hi
            const __half hh = __float2half_rn(hv);
            const float hf = __half2float(hh);
            uint8_t *row = stage + (j + (odd ? 8 : 0)) * RB;
            reinterpret_cast<__half *>(row)[r.col] = hh;
            const uint32_t c2 = e4m3x2((hv - hf) * 1024.0f, hf);
            row[128 + r.col] = (uint8_t)(c2 & 0xFF);
            row[192 + r.col] = (uint8_t)(c2 >> 8);
        }
    } else if constexpr (EPI == EPI_QKV) {
        if (r.sec < 2) {
            // (cos, sin) of this lane's angle, eight tokens at a time (the loads in flight
            // together, few registers)
            const int hh = e.head_dim >> 1;
#pragma unroll
            for (int i8 = 0; i8 < 16; i8 += 8) {
                float2 csv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int pp = tl0 + i8 + i < ntok ? s_rpos[tl0 + i8 + i] : 0;
                    csv[i] = __ldg(e.rope + (size_t)pp * hh + r.ipair);
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float2 cs = csv[i];
                    const float x = v[i8 + i] + r.bias;
                    const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
                    // ggml_rope_ext NEOX: (x0 cos - x1 sin, x0 sin + x1 cos)
                    const float o = r.bpair == 0 ? (x * cs.x - partner * cs.y) : (partner * cs.y + x * cs.x);
                    if (r.col < 128) reinterpret_cast<float *>(stage + (i8 + i) * RB)[r.col] = o;
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (r.col < 128) reinterpret_cast<float *>(stage + i * RB)[r.col] = v[i] + r.bias;
        }
    }
}

// Stores the staged chunk as token rows: lanes of a warp cover a row in 16-byte pieces.
// tid: 0..127 within the epilogue half.
template <int EPI>
__device__ __forceinline__ void epi_copyout(const EpiDst &d, const int *s_pos, int m0, int tl0, int ntok,
                                            const uint8_t *stage, int tid) {
    constexpr int es = EpiFmt<EPI>::esize, RB = EpiFmt<EPI>::row_bytes;
    constexpr int LPR = RB / 16, RPW = LPR >= 32 ? 1 : 32 / LPR;  // lanes per row, rows per warp pass
    const int w = tid >> 5, lane = tid & 31;
    for (int off = (lane % LPR) * 16; off < RB; off += 32 * 16) {
        if (off >= d.nbytes) return;
        for (int i = w * RPW + (LPR >= 32 ? 0 : lane / LPR); i < 16; i += 4 * RPW) {
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
// Shared memory (per CTA): [A ring (f16 weight tiles only): a_stages x a_stage_bytes]
// [B ring][raw ring][barriers][token positions][contributor offsets].  Slice i (64 k) of
// the CTA's unit range uses A stage i % na (TMEM columns tmem_a + 64 stage for quantized
// weights, Sched::init) and part i % spb of B slot (i / spb) % nbs; a part holds the
// slice's XS sub-slices (hi, then lo).
//
// MMAs per slice: W_hi.X_hi, W_hi.X_lo (XS = 2), W_lo.X_hi (weights with a lo part).
//
// Warps (warp_role): w0 activation producer, w1 MMA issuer (even CTA) + TMEM owner, w2
// weight-chunk producer (f16 weights: A-tile TMA producer), w3 relay, w4-w11 dequantizers
// (two sets of four; thread = weight row = TMEM lane), w12-w19 epilogue (thread = TMEM
// lane; w12-15 and w16-19 take alternate 16-column chunks).
template <int WT, int EPI, int XS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ XMaps xm, GemmParams p) {
    constexpr int RAWB = raw_chunk_bytes(WT);
    constexpr int NA = a_stages(WT), NRAW = raw_stages(WT), BRING = b_ring_bytes(WT), AR = a_ring_bytes(WT, XS);
    constexpr int ASB = a_stage_bytes(WT, XS);
    constexpr int CPR = raw_cpr(WT), RSB = CPR * RAWB;  // chunks and bytes per raw stage
    static_assert(gemm_smem_bytes(WT, XS) <= 227 * 1024, "shared memory per CTA");
    static_assert(XS == 1 || XS == 2, "activation parts");
    static_assert(NA == 2, "shared-memory A tiles: two stages");
    // The relay frees the B slot of slice j - kRelayLag while it handles slice j, after waiting
    // for the B loads up to slice j - 1: with one slice per load (the widest group, 16 or
    // 32 KB loads) the producer needs 2 + (kRelayLag - 1) slots not to wait on itself.
    static_assert(BRING / (kMaxTok / 2 * 128 * XS) >= 2 + (kRelayLag - 1), "B ring too shallow for the relay");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *aring = smem;  // f16 weight tiles only
    uint8_t *bring = smem + AR;
    uint8_t *raw = bring + BRING;
    uint8_t *epi_stage = raw + NRAW * RSB;  // [2 halves][kEpiStageBytes]
    uint64_t *bars = reinterpret_cast<uint64_t *>(epi_stage + 2 * kEpiStageBytes);
    uint64_t *full_a = bars, *empty_a = bars + 6, *full_b = bars + 12, *empty_b = bars + 36, *raw_full = bars + 60,
             *raw_empty = bars + 64, *acc_full = bars + 68, *acc_empty = bars + 70, *drain = bars + 72;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 74);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 75);
    volatile int *okflag = reinterpret_cast<volatile int *>(bars + 77);
    int *s_pos = reinterpret_cast<int *>(bars + kBarBytes / 8);                   // [kMaxTok]
    int *s_rpos = s_pos + kMaxTok;                                                // [kMaxTok]
    long long *s_contrib = reinterpret_cast<long long *>(s_rpos + kMaxTok);       // [2][kMaxContrib]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    // the next kernel of the stream may be scheduled now; it waits for this grid itself
    griddep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxNA; i++) {
            // both CTAs' relays + f16 tiles: the expect_tx / else four dequant warps per CTA
            mbar_init(&full_a[i], w_smem(WT) ? 3 : 10);
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
        *abort_flag = 0;
        fence_barrier_init();
    }
    const int role = warp_role(warp);
    if (w_smem(WT) && role == R_WPROD && lane == 0) prefetch_tmap(&tm_w);
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
    S.init(M, p.n_tiles >> 1, p.kb, n_pairs, pair, BRING, XS, !w_smem(WT));
    const int lg_na = S.na == 4 ? 2 : 1;
    const int NBS = S.nbs;
    // barriers of the even CTA as cluster addresses
    const uint32_t full_a0 = mapa_shared(full_a, 0), acc_empty0 = mapa_shared(acc_empty, 0);

    if (role == R_BPROD) {
        // ── activation producer (both CTAs, local barriers): this CTA's half of the
        //    token group, spb k-slices per tensor load.  Few large loads: the TMA unit
        //    also streams the weights and handles only a few operations per microsecond. ──
        griddep_wait();  // the activations are the previous kernel's output
        if (lane == 0) {
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
                        if (!(ok = mbar_wait(&empty_b[sl], ph ^ 1, abort_flag, p.err, kErrTimeout + 2, p.timeout_ns))) break;
                        mbar_arrive_expect_tx(&full_b[sl], S.bslot);
                        tma_load_3d(bring + sl * S.bslot, xmap, 0, row0, XS * (kbi * 4 + s), &full_b[sl]);
                        ob++;
                        if (++sl == NBS) { sl = 0; ph ^= 1; }
                    }
                }
                u += g.k1 - g.k0;
            }
            if (!ok) {
                // let the copies in flight land before the CTA can exit
                for (int i = (ob > NBS ? ob - NBS : 0); i < ob; i++) spin_bounded(&full_b[i % NBS], (i / NBS) & 1);
            }
        }
        __syncwarp();
    } else if (role == R_WPROD) {
        if constexpr (!w_smem(WT)) {
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
                    if (!(ok = mbar_wait(&raw_empty[r], ((rit / NRAW) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 1, p.timeout_ns))) break;
                    const int nch = min(CPR, S.u1 - u);
                    mbar_arrive_expect_tx(&raw_full[r], nch * RAWB);
                    for (int c = 0; c < nch; c++) bulk_g2s(raw + r * RSB + c * RAWB, chunk(u + c), RAWB, &raw_full[r]);
                    rit++;
                }
                if (!ok)
                    for (int i = (rit > NRAW ? rit - NRAW : 0); i < rit; i++)
                        spin_bounded(&raw_full[i % NRAW], (i / NRAW) & 1);
            }
        } else {
            // ── f16 weight tiles: A-tile TMA producer (completions counted on the even CTA);
            //    W_F32 stages hold the hi tile, then the lo tile (rows lo_row + ...) ──
            if (lane == 0) {
                int it = 0;
                bool ok = true;
                for (int u = S.u0; u < S.u1 && ok;) {
                    const Seg g = make_seg(S, u, S.u1);
                    for (int kbi = g.k0; kbi < g.k1 && ok; kbi++) {
                        for (int s = 0; s < 4; s++) {  // one stage = one k-slice
                            const int st = it % NA;
                            if (!(ok = mbar_wait(&empty_a[st], ((it / NA) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 11, p.timeout_ns))) break;
                            if (rank == 0) mbar_arrive_expect_tx(&full_a[st], 2 * ASB);
                            const int row = (2 * g.pt + (int)rank) * 128;
                            tma_load_2d_pair(aring + st * ASB, &tm_w, kbi * 256 + s * 64, row, full_a0 + 8 * st);
                            if constexpr (ASB == 2 * kSliceBytes)
                                tma_load_2d_pair(aring + st * ASB + kSliceBytes, &tm_w, kbi * 256 + s * 64,
                                                 (XS == 2 ? p.corr_row : p.lo_row) + row, full_a0 + 8 * st);
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
        // for the stage, fence, the slice's MMAs, commit.  Each unit is one k-block = four
        // slices; slice j of the range uses A stage j % na, whose barrier completes once per
        // use, so its parity is (j / na) & 1; the B descriptors are computed once per k-block.
        if (lane == 0 && rank == 0) {
            int si = 0;   // accumulator segments
            int kbc = 0;  // k-blocks issued
            bool ok = true, issued = false;
            const uint64_t bdesc0 = sw128_desc(smem_u32(bring)), adesc0 = sw128_desc(smem_u32(aring));
            const int lg_spb = S.spb == 1 ? 0 : S.spb == 2 ? 1 : 2;  // k-slices per ring slot: 1, 2 or 4
            const uint32_t bsub = S.bh * 128;  // bytes of one part (hi or lo) of a k-slice
            int bslot = 0;  // ring slot of the first slice of the next k-block
            for (int u = S.u0; u < S.u1 && ok;) {
                const Seg g = make_seg(S, u, S.u1);
                const int acc = S.acc_of(si);
                if (!(ok = mbar_wait(&acc_empty[acc], (S.acc_uses(si) & 1) ^ 1, abort_flag, p.err, kErrTimeout + 3, p.timeout_ns))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * S.acc_stride;
                const uint32_t idesc = idesc_f16(256, (uint32_t)g.nmma);
                uint32_t accum = 0;
                for (int kbi = g.k0; kbi < g.k1; kbi++) {
                    // (the ring may hold fewer slots than a k-block's four loads: wrap by modulo)
                    uint64_t bd[4];
#pragma unroll
                    for (int s2 = 0; s2 < 4; s2++) {
                        const int sl = (bslot + (s2 >> lg_spb)) % NBS;
                        bd[s2] = bdesc0 + (uint64_t)((sl * S.bslot + (s2 & (S.spb - 1)) * S.bpart) >> 4);
                    }
                    bslot = (bslot + (4 >> lg_spb)) % NBS;
#pragma unroll
                    for (int s2 = 0; s2 < 4; s2++) {
                        // slice j = 4 kbc + s2 of the range: stage j % na, use j / na of it
                        const int j = 4 * kbc + s2;
                        const int st = j & (S.na - 1);
                        // full_a also carries the relays' arrivals: this stage's B rows have landed
                        if (!(ok = mbar_wait(&full_a[st], (uint32_t)((j >> lg_na) & 1), abort_flag, p.err, kErrTimeout + 5, p.timeout_ns))) break;
                        tc_fence_after();
                        // main term (f16), then the corrections: XS = 2 one E4M3 MMA over the
                        // correction pairs, XS = 1 W_lo.X (f16) for weights with a lo part
                        const uint64_t bhi = bd[s2], bcor = bd[s2] + (uint64_t)(bsub >> 4);
                        if constexpr (w_smem(WT)) {
                            const uint64_t ahi = adesc0 + (uint64_t)((st * ASB) >> 4);
                            const uint64_t a2 = ahi + (uint64_t)(kSliceBytes >> 4);
                            mma2_f16_ss_k64(d_tmem, ahi, bhi, idesc, accum);
                            if constexpr (XS == 2) mma2_f8_ss_k128(d_tmem, a2, bcor, idesc);
                            else if constexpr (w_split(WT)) mma2_f16_ss_k64(d_tmem, a2, bhi, idesc, 1);
                        } else {
                            const uint32_t ahi = tmem_base + (uint32_t)S.tmem_a + st * kTmemAStage;
                            mma2_f16_ts_k64(d_tmem, ahi, bhi, idesc, accum);
                            if constexpr (XS == 2) mma2_f8_ts_k128(d_tmem, ahi + kTmemALo, bcor, idesc);
                            else mma2_f16_ts_k64(d_tmem, ahi + kTmemALo, bhi, idesc, 1);
                        }
                        accum = 1;
                        mma2_commit_mc(&empty_a[st], 0x3);
                    }
                    issued = true;
                    kbc++;
                    if (!ok) break;
                }
                if (!ok) break;
                mma2_commit_mc(&acc_full[acc], 0x3);
                si++;
                u += g.k1 - g.k0;
            }
            if (issued) {
                // every MMA must have retired before TMEM is released
                mma2_commit(drain);
                spin_bounded(drain, 0);
            }
        }
        __syncwarp();
    } else if (role == R_RELAY) {
        // ── relay (one thread per CTA), slice by slice: once the MMA of slice j - kRelayLag
        //    has completed (empty_a of its stage), its B slot is free again
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
            // running ring positions (no divisions): B load of slice j and of slice j - kRelayLag
            int fo_sl = 0, fo_part = 0, eo_sl = 0, eo_part = 0;
            uint32_t fo_ph = 0;
            for (int j = 0; j < n_it + kRelayLag && ok; j++) {  // A stage = slice j % na
                if (j >= kRelayLag) {
                    // MMA of slice jd = j - kRelayLag done (use jd / na of its stage; the stage's
                    // next use needs this relay's arrival for slice jd + na > j first, so the
                    // barrier cannot be a phase ahead); its B slot is free once the last slice
                    // of the slot's load is done
                    const int jd = j - kRelayLag;
                    if (!(ok = mbar_wait(&empty_a[jd & (S.na - 1)], (uint32_t)((jd >> lg_na) & 1), abort_flag, p.err,
                                         kErrTimeout + 12, p.timeout_ns))) break;
                    if (++eo_part == spb) {
                        eo_part = 0;
                        mbar_arrive(&empty_b[eo_sl]);
                        if (++eo_sl == NBS) eo_sl = 0;
                    }
                }
                if (j < n_it) {
                    if (fo_part == 0)
                        if (!(ok = mbar_wait(&full_b[fo_sl], fo_ph, abort_flag, p.err, kErrTimeout + 4, p.timeout_ns))) break;
                    mbar_arrive_cluster(full_a0 + 8 * (j & (S.na - 1)));
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
        if constexpr (!w_smem(WT)) {
            const int di = deq_index(warp);
            const int set = di >> 2;
            const int r = (di & 3) * 32 + lane;
            int rit = 0;
            bool ok = true;
            // This warp's TMEM lane quarter holds its 32 weight rows of every A stage.
            const uint32_t a_lane = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)S.tmem_a;
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
                if (lane == 0) okw = mbar_wait(bar, parity, abort_flag, p.err, code, p.timeout_ns);
                const bool okb = __shfl_sync(0xffffffffu, okw, 0) != 0;
                if (okb) (void)mbar_try_wait(bar, parity);
                return okb;
            };
            auto wait_a = [&](int ia) {
                return wait_warp(&empty_a[ia & (S.na - 1)], ((ia >> lg_na) & 1) ^ 1, kErrTimeout + 7);
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
                    }
                    const uint8_t *R = raw + rs * RSB + (rit % CPR) * RAWB;
                    // this set's k-slices of the k-block: set and set + 2 (A stage set, or set and
                    // set + 2 with four stages); each slice in two halves of 32 k.  XS = 2: f16 hi (16 columns per
                    // half), E4M3 hi 2^-10 and E4M3 lo (8 columns per half each, at 32 and 48);
                    // XS = 1: f16 hi and f16 lo (16 columns per half each, at 0 and 32).
                    using Half = typename std::conditional<XS == 2, HalfCorr, HalfSplit>::type;
                    [[maybe_unused]] Q4KMeta m4;
                    [[maybe_unused]] Q6KMeta m6;
                    [[maybe_unused]] Q6XMeta m6x;
                    if constexpr (WT == W_Q4K) q4k_load_meta(R, r, set, p.wscale, m4);
                    if constexpr (WT == W_Q6K && XS == 2) q6x_load_meta(R, r, set, p.wscale, m6x);
                    else if constexpr (WT == W_Q6K) q6k_load_meta(R, r, set, p.wscale, m6);
                    // Q6_K / Q8_0 with pair-row activations: f16 arithmetic (one conversion per
                    // weight fewer than the f32 route, dequant.cuh); otherwise f32
                    auto deq = [&](int hs, int hh, Half &o) {
                        const int sl = set + 2 * hs;
                        const int gi = 4 * hs + 2 * hh;  // Q6_K group of the half's first 16 values
                        if constexpr (WT == W_Q4K) q4k_half(R, r, sl, hh, m4.dsc[2 * hs + hh], m4.nm[2 * hs + hh], o);
                        else if constexpr (WT == W_Q6K && XS == 2)
                            q6x_half(R, r, sl, hh, m6x.dsh[gi], m6x.dsl[gi], m6x.dsh[gi + 1], m6x.dsl[gi + 1], o);
                        else if constexpr (WT == W_Q6K) q6k_half(R, r, sl, hh, m6.ds[gi], m6.ds[gi + 1], o);
                        else if constexpr (XS == 2) q8x_half(R, r, sl, hh, p.wscale, o);
                        else q80_half(R, r, sl, hh, p.wscale, o);
                    };
                    auto store = [&](uint32_t at, int hh, const Half &o) {
                        tmem_st16(at + 16 * hh, o.hi);
                        if constexpr (XS == 2) {
                            tmem_st8(at + kTmemALo + 8 * hh, o.ch);
                            tmem_st8(at + kTmemALo + 16 + 8 * hh, o.cl);
                        } else {
                            tmem_st16(at + kTmemALo + 16 * hh, o.lo);
                        }
                    };
#pragma unroll
                    for (int hs = 0; hs < 2; hs++) {
                        const int ia = 4 * rit + set + 2 * hs;  // slice of the range
                        const int st = ia & (S.na - 1);          // its stage: set, or set + 2 hs
                        const uint32_t at = a_lane + (uint32_t)(st * kTmemAStage);
                        Half o;
                        deq(hs, 0, o);
                        if (!(ok = wait_a(ia))) break;
                        tc_fence_after();  // after the MMA that read this stage
                        store(at, 0, o);
                        deq(hs, 1, o);
                        store(at, 1, o);
                        publish(st);
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
        // A whole tile is finished straight from TMEM.  A split tile's partial goes to the
        // workspace (f32 [column / 4][row][column % 4], slot 0 for the pair's first tile, 1
        // for its last) and its arrival is counted; once every MMA of this CTA is done, each
        // contributor of a split tile finishes its share of the tile's 16-column chunks,
        // summing all contributors' partials in contributor order (so the result does not
        // depend on timing).  A split segment whose accumulator no later segment reuses stays
        // in TMEM: only the other contributors' shares go to the workspace, and its own share
        // is read back from TMEM.
        const int q = warp & 3;
        const int row = 32 * q + lane;
        const int half = epi_half(warp);
        const int et = half * 128 + q * 32 + lane;  // 0..255
        const int tid_h = q * 32 + lane;            // 0..127 within the half
        uint8_t *my_stage = epi_stage + half * kEpiStageBytes;
        bool ok = true;
        const int first_ot = S.begin_of(pair) / S.kb;
        int nseg = 0;  // segments of this pair's range
        for (int u = S.u0; u < S.u1; nseg++) {
            const Seg g = make_seg(S, u, S.u1);
            u += g.k1 - g.k0;
        }
        // split tiles of this CTA: the pair's first and last tile (when split), with this
        // contributor's share of their chunks
        struct Fix {
            Seg g;
            int nc, me, ch0, ch1;
            int tm;  // TMEM column of the resident accumulator, or -1
        };
        Fix fx[2];
        int nfx = 0;
        auto release_acc = [&](int acc) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * acc);
        };
        // token positions of the token group starting at m0 (QKV cache rows and RoPE angles,
        // logits rows), loaded once per group: the first group's while the MMAs run
        int pos_m0 = -1;
        auto load_pos = [&](int m0, int ntok) {
            if constexpr (EPI == EPI_QKV || EPI == EPI_LOGITS) {
                if (m0 == pos_m0) return;
                named_bar_sync(1, kEpiThreads);  // earlier readers are done
                for (int t = et; t < ntok; t += kEpiThreads) {
                    s_pos[t] = p.epi.pos[m0 + t];
                    if constexpr (EPI == EPI_QKV) s_rpos[t] = p.epi.rope_pos[m0 + t];
                }
                named_bar_sync(1, kEpiThreads);
                pos_m0 = m0;
            }
        };
        if (S.u0 < S.u1) {
            const Seg g0 = make_seg(S, S.u0, S.u1);
            load_pos(g0.m0, g0.ntok);
        }
        int si = 0;
        for (int u = S.u0; u < S.u1 && ok;) {
            const Seg g = make_seg(S, u, S.u1);
            const int tile = 2 * g.pt + (int)rank;
            const int acc = S.acc_of(si);
            const bool whole = g.k0 == 0 && g.k1 == S.kb;
            if (whole) load_pos(g.m0, g.ntok);
            // one thread waits, the barrier hands the outcome to the whole group
            if (et == 0) *okflag = mbar_wait(&acc_full[acc], S.acc_uses(si) & 1, abort_flag, p.err, kErrTimeout + 8, p.timeout_ns) ? 1 : 0;
            named_bar_sync(1, kEpiThreads);
            ok = *okflag != 0;
            if (!ok) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + acc * S.acc_stride;
            if (whole) {
                const EpiRow er = epi_row<EPI>(p.epi, tile, row);
                const EpiDst dd = epi_dst<EPI>(p.epi, tile);
                // the next chunk's TMEM load is in flight while this chunk is handled (QKV,
                // whose RoPE loads take registers, loads each chunk when it needs it)
                constexpr bool kAhead = EPI != EPI_QKV;
                uint32_t u16[16];
                if (kAhead && 16 * half < g.nmma) tmem_ld16(taddr + 16 * half, u16);
                for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                    if (!kAhead) tmem_ld16(taddr + c0, u16);
                    tmem_ld_wait(u16);
                    float v[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(u16[i]);
                    if (kAhead && c0 + 32 < g.nmma) tmem_ld16(taddr + c0 + 32, u16);
                    epi_values<EPI>(p.epi, er, s_rpos, c0, g.ntok, v, my_stage);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                    epi_copyout<EPI>(dd, s_pos, g.m0, c0, g.ntok, my_stage, tid_h);
                    named_bar_sync(2 + half, kEpiThreads / 2);
                }
                release_acc(acc);
            } else {
                const int slot = g.ot == first_ot ? 0 : 1;
                Fix &f = fx[nfx++];
                f.g = g;
                const int c_first = S.owner(g.ot * S.kb), c_last = S.owner((g.ot + 1) * S.kb - 1);
                f.nc = c_last - c_first + 1;
                f.me = pair - c_first;
                const int nch = g.nmma >> 4;
                f.ch0 = f.me * nch / f.nc;
                f.ch1 = (f.me + 1) * nch / f.nc;
                // resident: no later segment of this pair reuses the accumulator
                const bool resident = si + (S.dbl ? 2 : 1) >= nseg;
                f.tm = resident ? acc * S.acc_stride : -1;
                if (et < f.nc && et < kMaxContrib) {
                    const int c = c_first + et;
                    const int sl = (S.begin_of(c) / S.kb == g.ot) ? 0 : 1;
                    s_contrib[(nfx - 1) * kMaxContrib + et] = ((long long)(2 * c + (int)rank) * 2 + sl) * kWsTile;
                }
                float *wsl = p.ws + ((size_t)blockIdx.x * 2 + slot) * kWsTile;
                if (resident) {
                    // the other contributors' shares only
                    for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                        if ((c0 >> 4) >= f.ch0 && (c0 >> 4) < f.ch1) continue;
                        uint32_t u16[16];
                        tmem_ld16(taddr + c0, u16);
                        tmem_ld_wait(u16);
                        float *dst = wsl + (size_t)c0 * 128 + row * 4;  // column group c0/4, this row
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            *reinterpret_cast<uint4 *>(dst + j * 512) =
                                make_uint4(u16[4 * j], u16[4 * j + 1], u16[4 * j + 2], u16[4 * j + 3]);
                    }
                } else {
                    uint32_t u16[16];
                    if (16 * half < g.nmma) tmem_ld16(taddr + 16 * half, u16);
                    for (int c0 = 16 * half; c0 < g.nmma; c0 += 32) {
                        tmem_ld_wait(u16);
                        uint4 qv[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) qv[j] = make_uint4(u16[4 * j], u16[4 * j + 1], u16[4 * j + 2], u16[4 * j + 3]);
                        if (c0 + 32 < g.nmma) tmem_ld16(taddr + c0 + 32, u16);
                        float *dst = wsl + (size_t)c0 * 128 + row * 4;
#pragma unroll
                        for (int j = 0; j < 4; j++) *reinterpret_cast<uint4 *>(dst + j * 512) = qv[j];
                    }
                    // the accumulator is in registers / on its way to the workspace
                    release_acc(acc);
                }
                __threadfence();
                named_bar_sync(1, kEpiThreads);
                if (et == 0) atomicAdd(&p.tile_cnt[2 * g.ot + rank], 1);
            }
            named_bar_sync(1, kEpiThreads);  // okflag is reused by the next segment
            si++;
            u += g.k1 - g.k0;
        }

        // ── deferred split-tile fixups, once every MMA of this CTA has completed (the rings
        //    are drained): both split tiles are waited for together, then each chunk of this
        //    contributor's shares is summed from the workspace (own share of a resident
        //    accumulator from TMEM) ──
        if (nfx > 0 && ok) {
            if (et == 0) {
                int okw = 1;
                for (int i = 0; i < nfx && okw; i++) {
                    if (fx[i].nc > kMaxContrib) {  // the launcher keeps nc <= kMaxContrib
                        atomicCAS(p.err, 0, kErrTimeout + 9);
                        okw = 0;
                    } else {
                        okw = wait_count(p.tile_cnt + 2 * fx[i].g.ot + rank, fx[i].nc, abort_flag, p.err, kErrTimeout + 13,
                                         p.timeout_ns);
                    }
                }
                *okflag = okw;
            }
            named_bar_sync(1, kEpiThreads);
            ok = *okflag != 0;
        }
        // Each thread prefetches, per chunk of its half, the other contributors' partials of
        // its row into its own slots of the drained rings by cp.async, one chunk ahead, so the
        // L2 latency of chunk n + 1 overlaps chunk n.  Slots per buffer: [remote contributor]
        // [4 float4][256 threads] (consecutive threads hold consecutive 16 bytes).  The layout
        // depends on the tile, so both halves finish a tile before either starts the next.
        constexpr int kStageBytes = AR + BRING + NRAW * RSB;
        for (int i = 0; i < nfx && ok; i++) {
            const Fix &f = fx[i];
            if (i > 0) named_bar_sync(1, kEpiThreads);
            load_pos(f.g.m0, f.g.ntok);
            const int tile = 2 * f.g.pt + (int)rank;
            const EpiRow er = epi_row<EPI>(p.epi, tile, row);
            const EpiDst dd = epi_dst<EPI>(p.epi, tile);
            const long long *contrib = s_contrib + i * kMaxContrib;
            const bool own_tm = f.tm >= 0;
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(own_tm ? f.tm : 0);
            const int part_bytes = (f.nc - (own_tm ? 1 : 0)) * 4 * 16 * kEpiThreads;
            const int buf_bytes = part_bytes;
            const int nbuf = 2 * buf_bytes <= kStageBytes ? 2 : buf_bytes <= kStageBytes ? 1 : 0;
            auto issue = [&](int ch, int b) {
                uint8_t *base = smem + (size_t)b * buf_bytes;
                int slot = 0;
                for (int c = 0; c < f.nc; c++) {
                    if (c == f.me && own_tm) continue;
                    const float *src = p.ws + contrib[c] + (size_t)ch * 2048 + row * 4;
#pragma unroll
                    for (int j = 0; j < 4; j++) cp_async16(base + ((size_t)(slot * 4 + j) * kEpiThreads + et) * 16, src + j * 512);
                    slot++;
                }
                cp_async_commit();
            };
            if (nbuf == 2 && f.ch0 + half < f.ch1) issue(f.ch0 + half, 0);
            int k = 0;
            for (int ch = f.ch0 + half; ch < f.ch1; ch += 2, k++) {
                const int b = nbuf == 2 ? (k & 1) : 0;
                if (nbuf == 2) {
                    if (ch + 2 < f.ch1) {
                        issue(ch + 2, b ^ 1);
                        cp_async_wait<1>();
                    } else {
                        cp_async_wait<0>();
                    }
                } else if (nbuf == 1) {
                    issue(ch, 0);
                    cp_async_wait<0>();
                }
                const uint8_t *base = smem + (size_t)b * buf_bytes;
                // contributors in order
                float v[16];
#pragma unroll
                for (int kk = 0; kk < 16; kk++) v[kk] = 0.f;
                int slot = 0;
                for (int c = 0; c < f.nc; c++) {
                    float4 t[4];
                    if (c == f.me && own_tm) {
                        uint32_t u16[16];
                        tmem_ld16(taddr + 16 * ch, u16);
                        tmem_ld_wait(u16);
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            t[j] = make_float4(__uint_as_float(u16[4 * j]), __uint_as_float(u16[4 * j + 1]),
                                               __uint_as_float(u16[4 * j + 2]), __uint_as_float(u16[4 * j + 3]));
                    } else if (nbuf) {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            t[j] = *reinterpret_cast<const float4 *>(base + ((size_t)(slot * 4 + j) * kEpiThreads + et) * 16);
                        slot++;
                    } else {
                        const float4 *src = reinterpret_cast<const float4 *>(p.ws + contrib[c] + (size_t)ch * 2048 + row * 4);
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
                epi_values<EPI>(p.epi, er, s_rpos, ch * 16, f.g.ntok, v, my_stage);
                named_bar_sync(2 + half, kEpiThreads / 2);
                epi_copyout<EPI>(dd, s_pos, f.g.m0, ch * 16, f.g.ntok, my_stage, tid_h);
                named_bar_sync(2 + half, kEpiThreads / 2);
            }
        }
        if (ok && et == 0) {
            // departure: the last of the nc contributors resets the counter for the next launch
            for (int i = 0; i < nfx; i++) {
                int *cntp = p.tile_cnt + 2 * fx[i].g.ot + rank;
                const int old = atomicAdd(cntp, 1);
                if (old == 2 * fx[i].nc - 1) *cntp = 0;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no remote arrival or copy of either CTA is still in flight
    if (role == R_MMA) {
        tc_fence_after();
        tmem_dealloc2(tmem_base, 512);
    }
}

}  // namespace dfb
