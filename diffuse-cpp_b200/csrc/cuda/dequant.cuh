// Dequantization of re-tiled GGUF weight chunks into hi / lo f16 pairs for the GEMM's
// A operand (one TMEM lane = one weight row).
//
// Each weight is computed in f32 (Q4_K d*sc*q - dmin*m with one rounding; Q6_K
// d*sc*(q-32) and Q8_0 d*q exactly) after multiplying the block scales by the GEMM's
// power-of-two pre-scale `ws`, then split: hi = f16(w), lo = f16(w - hi).  hi + lo
// carries ~22 significant bits.  The block formats are GGML's (Q4_K / Q6_K / Q8_0, the
// weight-format contract of the reference's GGUF files); the decode rules match
// gguf-py's dequantizers, which the host codec tests pin.
//
// The output of one call is one half of a 64-wide k-slice (32 k-values) in 16 registers
// of f16 pairs per part, in k order (register j holds k = 2j in its low half and 2j + 1
// in its high half): the layout of one TMEM lane of 16 columns of an f16 A operand.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace dfb {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Two f32 values -> f16 pairs of their hi and lo parts (a in the low halves).  a - hi is
// exact in f32 (hi holds a's leading 11 bits).
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    hi = h2u(h);
    lo = h2u(__floats2half2_rn(a - hf.x, b - hf.y));
}

// Byte k (0..3) of x as the float 2^23 + byte (exact for bytes 0..255).
template <int K>
__device__ __forceinline__ float byte_magic(uint32_t x) {
    return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u | K));
}
constexpr float kMagic = 8388608.0f;  // 2^23

// Four elements (bytes of x) through f(value) -> two hi pairs and two lo pairs.
template <typename F>
__device__ __forceinline__ void quad(uint32_t x, F f, uint32_t &h01, uint32_t &h23, uint32_t &l01, uint32_t &l23) {
    const float w0 = f(byte_magic<0>(x)), w1 = f(byte_magic<1>(x));
    const float w2 = f(byte_magic<2>(x)), w3 = f(byte_magic<3>(x));
    split2(w0, w1, h01, l01);
    split2(w2, w3, h23, l23);
}

// ── Q4_K ── chunk layout (per 128 rows): [d,dmin f16 x2: 4 B/row][scales: 12 B/row at 512]
// [qs: 128 B/row at 2048, 16-byte chunk c stored at c ^ (row & 7)].
// Set p dequantizes k-slices p and p + 2, i.e. sub-blocks 2p, 2p + 1 (local 0, 1) and
// 2p + 4, 2p + 5 (local 2, 3); one half-slice is one sub-block of 32.
struct Q4KMeta {
    float dsc[4], nm[4];  // ws*d*sc and -(ws*dmin*m) per local sub-block
};
__device__ __forceinline__ void q4k_load_meta(const uint8_t *R, int r, int set, float ws, Q4KMeta &m) {
    const uint32_t dm = *reinterpret_cast<const uint32_t *>(R + 4 * r);
    const float d = __half2float(__ushort_as_half((unsigned short)(dm & 0xFFFF))) * ws;
    const float dmin = __half2float(__ushort_as_half((unsigned short)(dm >> 16))) * ws;
    const uint32_t *sp = reinterpret_cast<const uint32_t *>(R + 512 + 12 * r);
    const uint32_t s0 = sp[0], s1 = sp[1], s2 = sp[2];
    // byte i of the 12 packed scale bytes (i may be a runtime value: no local array)
    auto qb = [&](int i) -> int { return (int)(((i < 4 ? s0 : i < 8 ? s1 : s2) >> (8 * (i & 3))) & 0xFF); };
#pragma unroll
    for (int l = 0; l < 4; l++) {
        // 6-bit scale / min of sub-block j (GGML's get_scale_min_k4 packing)
        const int j = 2 * set + (l & 1) + 4 * (l >> 1);
        int sc, mn;
        if (l < 2) {  // j < 4
            sc = qb(j) & 63;
            mn = qb(j + 4) & 63;
        } else {
            sc = (qb(j + 4) & 0xF) | ((qb(j - 4) >> 6) << 4);
            mn = (qb(j + 4) >> 4) | ((qb(j) >> 6) << 4);
        }
        m.dsc[l] = d * (float)sc;     // exact: 11 + 6 significant bits
        m.nm[l] = -(dmin * (float)mn);
    }
}
// Half h of slice s of row r: the low nibbles of qs bytes 32s .. 32s+31 are sub-block 2s
// (h = 0), the high nibbles sub-block 2s + 1 (h = 1); l = local meta index.
__device__ __forceinline__ void q4k_half(const uint8_t *R, int r, int s, int h, float dsc, float nm,
                                         uint32_t (&hi)[16], uint32_t (&lo)[16]) {
    const uint8_t *qrow = R + 2048 + 128 * r;
    const uint4 qa = *reinterpret_cast<const uint4 *>(qrow + (((2 * s) ^ (r & 7)) << 4));
    const uint4 qc = *reinterpret_cast<const uint4 *>(qrow + (((2 * s + 1) ^ (r & 7)) << 4));
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qc.x, qc.y, qc.z, qc.w};
    auto f = [&](float mg) { return fmaf(mg - kMagic, dsc, nm); };  // q exact, one rounding
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t nib = h ? ((w[i] >> 4) & 0x0F0F0F0Fu) : (w[i] & 0x0F0F0F0Fu);
        quad(nib, f, hi[2 * i], hi[2 * i + 1], lo[2 * i], lo[2 * i + 1]);
    }
}

// ── Q6_K ── chunk layout: [ql: 128 B/row, chunk c at c ^ (row & 7)]
// [qh: 64 B/row at 16384, chunk c at c ^ ((row >> 1) & 3)][scales i8: 16 B/row at 24576]
// [d f16: 2 B/row at 26624].
// ws*d*scale of the eight 16-element groups one dequant set uses: set p takes slices p
// and p + 2, i.e. groups 4p .. 4p + 3 and 4p + 8 .. 4p + 11 (scale words p and p + 2).
struct Q6KMeta {
    float ds[8];
};
__device__ __forceinline__ void q6k_load_meta(const uint8_t *R, int r, int set, float ws, Q6KMeta &m) {
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(R + 26624 + 2 * r))) * ws;
    const uint4 sv = *reinterpret_cast<const uint4 *>(R + 24576 + 16 * r);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int wi = set + 2 * h;  // scale word holding groups 4*wi .. 4*wi+3
        const uint32_t w = wi == 0 ? sv.x : wi == 1 ? sv.y : wi == 2 ? sv.z : sv.w;
#pragma unroll
        for (int i = 0; i < 4; i++) m.ds[4 * h + i] = d * (float)(int)(int8_t)((w >> (8 * i)) & 0xFF);  // exact
    }
}
// Half hh of slice s of row r (k = 64 s + 32 hh ..): 32 six-bit values, groups of 16 with
// scales ds0 (first 16) and ds1.  Slice s reads half s / 2 of ql / qh: ql bytes
// 64 (s/2) .. +63 (low nibbles for even s, high nibbles for odd s), qh bits 2 * (2 (s&1)
// + (byte >= 32)) of qh bytes 32 (s/2) + (l % 32).
__device__ __forceinline__ void q6k_half(const uint8_t *R, int r, int s, int hh, float ds0, float ds1,
                                         uint32_t (&hi)[16], uint32_t (&lo)[16]) {
    const int h = s >> 1, s2 = s & 1;
    const uint8_t *qlrow = R + 128 * r, *qhrow = R + 16384 + 64 * r;
    // ql bytes 64h + 32hh .. +31 and qh bytes 32h .. +31 (all of them: bit pair by hh)
    const uint4 l0 = *reinterpret_cast<const uint4 *>(qlrow + (((4 * h + 2 * hh) ^ (r & 7)) << 4));
    const uint4 l1 = *reinterpret_cast<const uint4 *>(qlrow + (((4 * h + 2 * hh + 1) ^ (r & 7)) << 4));
    const uint4 g0 = *reinterpret_cast<const uint4 *>(qhrow + (((2 * h) ^ ((r >> 1) & 3)) << 4));
    const uint4 g1 = *reinterpret_cast<const uint4 *>(qhrow + (((2 * h + 1) ^ ((r >> 1) & 3)) << 4));
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t qw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const int shift = 4 * s2 + 2 * hh;
    const float bias = kMagic + 32.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t nib = s2 ? ((lw[i] >> 4) & 0x0F0F0F0Fu) : (lw[i] & 0x0F0F0F0Fu);
        const uint32_t q6 = nib | (((qw[i] >> shift) & 0x03030303u) << 4);
        const float ds = i < 4 ? ds0 : ds1;
        auto f = [&](float mg) { return (mg - bias) * ds; };
        quad(q6, f, hi[2 * i], hi[2 * i + 1], lo[2 * i], lo[2 * i + 1]);
    }
}

// ── Q8_0 ── chunk layout: [d f16 x 8: 16 B/row][qs: 256 B/row at 2048, chunk c at
// (c & 8) | ((c & 7) ^ (row & 7))].  Half h of slice s is block 2s + h.
__device__ __forceinline__ void q80_half(const uint8_t *R, int r, int s, int h, float ws, uint32_t (&hi)[16],
                                         uint32_t (&lo)[16]) {
    const int blk = 2 * s + h;
    const uint4 dv = *reinterpret_cast<const uint4 *>(R + 16 * r);
    const int wi = blk >> 1;  // may be a runtime value: select, no local array
    const uint32_t dwd = wi == 0 ? dv.x : wi == 1 ? dv.y : wi == 2 ? dv.z : dv.w;
    const float d = __half2float(__ushort_as_half((unsigned short)((dwd >> (16 * (blk & 1))) & 0xFFFF))) * ws;
    const uint8_t *qrow = R + 2048 + 256 * r;
    const float bias = kMagic + 128.f;
    auto f = [&](float mg) { return (mg - bias) * d; };  // exact: 11 + 8 significant bits
#pragma unroll
    for (int cc = 0; cc < 2; cc++) {
        const int c = 2 * blk + cc;
        const uint4 v = *reinterpret_cast<const uint4 *>(qrow + (((c & 8) | ((c & 7) ^ (r & 7))) << 4));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int j = 4 * cc + i;
            quad(w[i] ^ 0x80808080u, f, hi[2 * j], hi[2 * j + 1], lo[2 * j], lo[2 * j + 1]);
        }
    }
}

}  // namespace dfb
