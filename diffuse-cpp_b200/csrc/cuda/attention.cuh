// Bidirectional (non-causal) attention over the inter-step K/V cache, in f32.
//
// Replaces the reference's per-head attention block: K^T Q (ggml_mul_mat of two f32
// tensors, an f32 dot product), scale 1/sqrt(head_dim), soft_max with no mask, V * P
// (src/diffuse-graph.cpp:97-119; cached variant :528-553 with keys [cached ‖ active]).
// Here the keys are every position of the sequence read straight from the cache (the
// QKV epilogue has already written the fresh rows of the active positions), so the full
// and the cached forward are the same kernel.  GQA: query head h reads kv head
// h / n_rep, as ggml_repeat's grouped layout does (graph.cpp:84-95).  RoPE was applied
// when K and Q were produced.
//
// Arithmetic: f32 FMAs on the CUDA cores, like the reference's f32 mul_mat; the softmax
// is the online (flash) form, exp2 of log2(e)-scaled scores, which equals the
// reference's expf(x - max) / sum up to f32 rounding.  16-bit tensor-core operands would
// round Q, K, P and V to 11 bits, which over 32 layers moves the logits by ~4e-3 of
// their magnitude; f32 keeps the forward within ~1e-5 of the model's exact mathematics.
//
// Work list: tiles {first active row, rows (<= 32), first key position, keys} of one
// sequence each (several sequences step together, their rows and cache positions
// concatenated); a CTA takes tile blockIdx.x of one head.
//
// One CTA = 32 query rows of one head, 128 threads; key tiles of 64 (cp.async, K of tile
// t + 1 loading during the P.V of tile t, V of tile t + 1 during the scores of t + 1).
// Thread (ty, tx) = (tid / 16, tid % 16) owns rows 4 ty .. 4 ty + 3: scores of keys
// tx + 16 j, and output dims of float4 chunks tx + 16 i.  The output rows are written in
// the GEMM's pair layout (hi f16, lo f16 per 64-wide slice) for the O projection.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "dequant.cuh"
#include "ptx.cuh"

namespace dfb {

constexpr int kAttnRows = 32, kAttnKeys = 64, kAttnThreads = 128;

template <int HD>
struct AttnSmem {
    static constexpr int QP = HD + 4;   // Q / K row pitch (floats): conflict-free float4 reads
    static constexpr int PP = 36;       // P^T row pitch
    static constexpr int q_off = 0;
    static constexpr int k_off = q_off + kAttnRows * QP;
    static constexpr int v_off = k_off + kAttnKeys * QP;
    static constexpr int p_off = v_off + kAttnKeys * HD;
    static constexpr int floats = p_off + kAttnKeys * PP;
    static constexpr int bytes = floats * 4;
};
template <int HD>
constexpr int attn_smem_bytes() { return AttnSmem<HD>::bytes; }

// q: [rows][ld_q] f32 (head h at h*HD), kc/vc: [positions][ld_kv] f32 (kv head at
// kvh*HD), o: pair rows of ld_o bytes (4 * n_q, dequant.cuh); tiles / n_tiles: the work list.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const float *__restrict__ q, int ld_q,
                                                           const float *__restrict__ kc, const float *__restrict__ vc,
                                                           int ld_kv, uint8_t *__restrict__ o, int ld_o,
                                                           const int4 *__restrict__ tiles, const int *__restrict__ n_tiles_dev,
                                                           int n_rep, float scale_log2) {
    using L = AttnSmem<HD>;
    constexpr int NC = HD / 4;                   // float4 chunks per row
    constexpr int CPT = (NC + 15) / 16;          // output chunks per thread
    extern __shared__ __align__(16) float att_smem[];
    float *Qs = att_smem + L::q_off, *Ks = att_smem + L::k_off, *Vs = att_smem + L::v_off, *Ps = att_smem + L::p_off;

    griddep_launch_dependents();
    griddep_wait();  // q, the K/V cache and the work list come from the previous kernels
    if ((int)blockIdx.x >= *n_tiles_dev) return;
    const int4 tile = tiles[blockIdx.x];
    const int q0 = tile.x, M = tile.x + tile.y, n_keys = tile.w;
    kc += (size_t)tile.z * ld_kv;  // the sequence's first cache position
    vc += (size_t)tile.z * ld_kv;
    const int h = blockIdx.y, kvh = h / n_rep;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

    auto load_rows = [&](float *dst, int pitch, const float *src, int k0) {
        for (int idx = tid; idx < kAttnKeys * NC; idx += kAttnThreads) {
            const int row = idx / NC, ch = idx % NC;
            const int key = k0 + row;
            const bool valid = key < n_keys;
            cp_async16(dst + row * pitch + 4 * ch, src + (size_t)(valid ? key : 0) * ld_kv + kvh * HD + 4 * ch, valid);
        }
        cp_async_commit();
    };
    const int n_tiles = (n_keys + kAttnKeys - 1) / kAttnKeys;
    load_rows(Ks, L::QP, kc, 0);
    load_rows(Vs, HD, vc, 0);
    // Q rows, pre-scaled by log2(e) / sqrt(HD); rows beyond M are zero
    for (int idx = tid; idx < kAttnRows * NC; idx += kAttnThreads) {
        const int row = idx / NC, ch = idx % NC;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + row < M) v = *reinterpret_cast<const float4 *>(q + (size_t)(q0 + row) * ld_q + h * HD + 4 * ch);
        v.x *= scale_log2; v.y *= scale_log2; v.z *= scale_log2; v.w *= scale_log2;
        *reinterpret_cast<float4 *>(Qs + row * L::QP + 4 * ch) = v;
    }

    float acc[4][CPT][4];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
        for (int i = 0; i < CPT; i++) acc[r][i][0] = acc[r][i][1] = acc[r][i][2] = acc[r][i][3] = 0.f;
    float m[4], l[4];
#pragma unroll
    for (int r = 0; r < 4; r++) { m[r] = -INFINITY; l[r] = 0.f; }

    for (int t = 0; t < n_tiles; t++) {
        cp_async_wait<1>();  // K of tile t (V of tile t may still be in flight)
        __syncthreads();
        // scores of rows 4ty + r, keys tx + 16 j
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; r++) s[r][0] = s[r][1] = s[r][2] = s[r][3] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int r = 0; r < 4; r++) qv[r] = *reinterpret_cast<const float4 *>(Qs + (4 * ty + r) * L::QP + d);
#pragma unroll
            for (int j = 0; j < 4; j++) kv[j] = *reinterpret_cast<const float4 *>(Ks + (tx + 16 * j) * L::QP + d);
#pragma unroll
            for (int r = 0; r < 4; r++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    s[r][j] = fmaf(qv[r].x, kv[j].x, s[r][j]);
                    s[r][j] = fmaf(qv[r].y, kv[j].y, s[r][j]);
                    s[r][j] = fmaf(qv[r].z, kv[j].z, s[r][j]);
                    s[r][j] = fmaf(qv[r].w, kv[j].w, s[r][j]);
                }
        }
        // online softmax: row max over the 16 threads of the row group, rescale
        const int kbase = t * kAttnKeys;
        float alpha[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (kbase + tx + 16 * j >= n_keys) s[r][j] = -INFINITY;
                mx = fmaxf(mx, s[r][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[r], mx);  // finite: every tile has a valid key
            alpha[r] = exp2f(m[r] - mn);       // 0 on the first tile
            m[r] = mn;
            float ls = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                s[r][j] = exp2f(s[r][j] - mn);
                ls += s[r][j];
            }
            l[r] = l[r] * alpha[r] + ls;
        }
        // P^T into shared memory: Ps[key][row]
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4 *>(Ps + (tx + 16 * j) * L::PP + 4 * ty) = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();  // P visible; K of tile t consumed
        if (t + 1 < n_tiles) {
            load_rows(Ks, L::QP, kc, (t + 1) * kAttnKeys);
            cp_async_wait<1>();  // V of tile t
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int i = 0; i < CPT; i++) {
                acc[r][i][0] *= alpha[r]; acc[r][i][1] *= alpha[r]; acc[r][i][2] *= alpha[r]; acc[r][i][3] *= alpha[r];
            }
#pragma unroll 4
        for (int k = 0; k < kAttnKeys; k++) {
            const float4 p4 = *reinterpret_cast<const float4 *>(Ps + k * L::PP + 4 * ty);
            const float pr[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int i = 0; i < CPT; i++) {
                const int c = tx + 16 * i;
                if (c < NC) {
                    const float4 v = *reinterpret_cast<const float4 *>(Vs + k * HD + 4 * c);
#pragma unroll
                    for (int r = 0; r < 4; r++) {
                        acc[r][i][0] = fmaf(pr[r], v.x, acc[r][i][0]);
                        acc[r][i][1] = fmaf(pr[r], v.y, acc[r][i][1]);
                        acc[r][i][2] = fmaf(pr[r], v.z, acc[r][i][2]);
                        acc[r][i][3] = fmaf(pr[r], v.w, acc[r][i][3]);
                    }
                }
            }
        }
        __syncthreads();  // V and P of tile t consumed
        if (t + 1 < n_tiles) load_rows(Vs, HD, vc, (t + 1) * kAttnKeys);
    }
    // row sums over the 16 threads of each row group, normalize, write pair rows
#pragma unroll
    for (int r = 0; r < 4; r++) {
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
        const int row = q0 + 4 * ty + r;
        if (row >= M) continue;
        const float inv = 1.f / l[r];
#pragma unroll
        for (int i = 0; i < CPT; i++) {
            const int c = tx + 16 * i;
            if (c >= NC) continue;
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) v[e] = acc[r][i][e] * inv;
            store_pair4(o + (size_t)row * ld_o, h * HD + 4 * c, v);  // features h*HD + 4c .. +3
        }
    }
}

}  // namespace dfb
