// Bidirectional (non-causal) flash attention over the inter-step K/V cache.
//
// Replaces the reference's per-head attention block: K^T Q (ggml_mul_mat), scale
// 1/sqrt(head_dim), soft_max with no mask, V * P (src/diffuse-graph.cpp:97-119; cached
// variant :528-553 with keys [cached ‖ active]).  Here the keys are every position of
// the sequence read straight from the cache (the QKV epilogue has already written the
// fresh rows of the active positions), so the full and the cached forward are the same
// kernel.  GQA: query head h reads kv head h / n_rep, as ggml_repeat's grouped layout
// does (graph.cpp:84-95).  RoPE was applied when K and Q were produced.
//
// One CTA = 64 query rows of one head, two groups of 4 warps: group g takes the key tiles
// t = g (mod 2) of 64 keys (its own cp.async double buffer) with an online softmax in f32
// registers; at the end group 1 hands its running max, sum and output rows to group 0
// through shared memory, which merges them (the log-sum-exp combination of two softmax
// partials) and writes the rows.  Two groups double the warps per SM at the same grid.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx.cuh"

namespace dfb {

constexpr int kAttnRows = 64, kAttnKeys = 64;

template <int HD>
__device__ __forceinline__ int attn_swz(int row, int chunk) {
    constexpr int nch = HD / 8;
    constexpr int msk = (nch < 8 ? nch : 8) - 1;
    return row * HD * 2 + ((chunk ^ (row & msk)) << 4);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    const int sz = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// Four 8x8 b16 matrices, not transposed: lane l addresses row l % 8 of matrix l / 8 and
// receives, of each matrix, row l / 4, elements 2 (l % 4) and 2 (l % 4) + 1.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// q: [M][ld_q] (head h at h*HD), kc/vc: [n_keys][ld_kv] (kv head at kvh*HD), o: [M][ld_o].
constexpr int kAttnThreads = 256;

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const __half *__restrict__ q, int ld_q,
                                                   const __half *__restrict__ kc, const __half *__restrict__ vc,
                                                   int ld_kv, __half *__restrict__ o, int ld_o,
                                                   const int *__restrict__ m_dev, int n_keys, int n_rep,
                                                   float scale_log2) {
    constexpr int NCH = HD / 8;           // 16-byte chunks per row
    constexpr int KT = HD / 16;           // k-steps for Q K^T
    constexpr int DT = HD / 8;            // n-tiles of the output
    extern __shared__ __align__(128) uint8_t att_smem[];
    const int grp = threadIdx.x >> 7, gtid = threadIdx.x & 127;
    uint8_t *Ks = att_smem + grp * 4 * kAttnKeys * HD * 2;  // this group's [2][64][HD]
    uint8_t *Vs = Ks + 2 * kAttnKeys * HD * 2;              // [2][64][HD]

    griddep_launch_dependents();
    griddep_wait();  // q and the K/V cache come from the previous kernels
    const int M = *m_dev;
    const int q0 = blockIdx.x * kAttnRows;
    if (q0 >= M) return;
    const int h = blockIdx.y, kvh = h / n_rep;
    const int warp = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;

    // Q fragments (rows beyond M read as zero)
    uint32_t qa[KT][4];
    {
        const __half *q_r0 = q + (size_t)min(r0, M - 1) * ld_q + h * HD;
        const __half *q_r1 = q + (size_t)min(r1, M - 1) * ld_q + h * HD;
        const bool v0 = r0 < M, v1 = r1 < M;
#pragma unroll
        for (int kk = 0; kk < KT; kk++) {
            const int c = 16 * kk + 2 * t;
            qa[kk][0] = v0 ? *reinterpret_cast<const uint32_t *>(q_r0 + c) : 0u;
            qa[kk][1] = v1 ? *reinterpret_cast<const uint32_t *>(q_r1 + c) : 0u;
            qa[kk][2] = v0 ? *reinterpret_cast<const uint32_t *>(q_r0 + c + 8) : 0u;
            qa[kk][3] = v1 ? *reinterpret_cast<const uint32_t *>(q_r1 + c + 8) : 0u;
        }
    }

    auto load_tile = [&](int tile, int buf) {
        const int k0 = tile * kAttnKeys;
        uint8_t *kd = Ks + buf * kAttnKeys * HD * 2, *vd = Vs + buf * kAttnKeys * HD * 2;
        for (int idx = gtid; idx < kAttnKeys * NCH; idx += 128) {
            const int row = idx / NCH, ch = idx % NCH;
            const int key = k0 + row;
            const bool valid = key < n_keys;
            const size_t off = (size_t)(valid ? key : 0) * ld_kv + kvh * HD + ch * 8;
            cp_async16(kd + attn_swz<HD>(row, ch), kc + off, valid);
            cp_async16(vd + attn_swz<HD>(row, ch), vc + off, valid);
        }
        cp_async_commit();
    };

    float acc[DT][4];
#pragma unroll
    for (int i = 0; i < DT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m_0 = -INFINITY, m_1 = -INFINITY, l_0 = 0.f, l_1 = 0.f;

    const int n_tiles = (n_keys + kAttnKeys - 1) / kAttnKeys;
    if (grp < n_tiles) load_tile(grp, 0);
    for (int tile = grp, it = 0; tile < n_tiles; tile += 2, it++) {
        const int buf = it & 1;
        if (tile + 2 < n_tiles) {
            load_tile(tile + 2, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        named_bar_sync(1 + grp, 128);
        const uint8_t *kb = Ks + buf * kAttnKeys * HD * 2;
        const uint8_t *vb = Vs + buf * kAttnKeys * HD * 2;

        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
            if constexpr (KT % 2 == 0) {
                // B fragments of two k-steps per ldmatrix: matrices = (keys nt*8..+7) x
                // (16-byte chunks 2kk, 2kk+1, 2kk+2, 2kk+3) of the K rows
                const uint32_t kaddr = static_cast<uint32_t>(__cvta_generic_to_shared(kb));
#pragma unroll
                for (int kk = 0; kk < KT; kk += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kaddr + attn_swz<HD>(nt * 8 + (lane & 7), 2 * kk + (lane >> 3)), b0, b1, b2, b3);
                    mma16816(s[nt], qa[kk], b0, b1);
                    mma16816(s[nt], qa[kk + 1], b2, b3);
                }
            } else {
                const int krow = nt * 8 + g;
#pragma unroll
                for (int kk = 0; kk < KT; kk++) {
                    const int col = 16 * kk + 2 * t;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kb + attn_swz<HD>(krow, col >> 3) + (col & 7) * 2);
                    const uint32_t b1 =
                        *reinterpret_cast<const uint32_t *>(kb + attn_swz<HD>(krow, (col + 8) >> 3) + (col & 7) * 2);
                    mma16816(s[nt], qa[kk], b0, b1);
                }
            }
        }
        // mask keys past the end, row max
        const int kbase = tile * kAttnKeys;
        float mx0 = m_0, mx1 = m_1;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int key = kbase + nt * 8 + 2 * t + (e & 1);
                float v = s[nt][e] * scale_log2;
                if (key >= n_keys) v = -INFINITY;
                s[nt][e] = v;
            }
            mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
            mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float c0 = exp2f(m_0 - mx0), c1 = exp2f(m_1 - mx1);
        m_0 = mx0;
        m_1 = mx1;
        float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            s[nt][0] = exp2f(s[nt][0] - mx0);
            s[nt][1] = exp2f(s[nt][1] - mx0);
            s[nt][2] = exp2f(s[nt][2] - mx1);
            s[nt][3] = exp2f(s[nt][3] - mx1);
            ls0 += s[nt][0] + s[nt][1];
            ls1 += s[nt][2] + s[nt][3];
        }
        l_0 = l_0 * c0 + ls0;
        l_1 = l_1 * c1 + ls1;
#pragma unroll
        for (int i = 0; i < DT; i++) {
            acc[i][0] *= c0; acc[i][1] *= c0;
            acc[i][2] *= c1; acc[i][3] *= c1;
        }
        // O += P V: 4 k-steps of 16 keys
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t pa[4];
            pa[0] = pack_h2(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack_h2(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int dt = 0; dt < DT; dt += 2) {
                const int mat = lane >> 3, rr = lane & 7;
                const int key = 16 * kk + (mat & 1) * 8 + rr;
                const int ch = dt + (mat >> 1);
                const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(vb + attn_swz<HD>(key, ch)));
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(addr, b0, b1, b2, b3);
                mma16816(acc[dt], pa, b0, b1);
                mma16816(acc[dt + 1], pa, b2, b3);
            }
        }
        named_bar_sync(1 + grp, 128);
    }
    // merge group 1 into group 0: per thread, the same rows and columns in both groups
    __syncthreads();  // both groups are done with their tiles; reuse the tile buffers
    float *xch = reinterpret_cast<float *>(att_smem);  // [DT*4 + 4][128]
    if (grp == 1) {
#pragma unroll
        for (int i = 0; i < DT; i++)
#pragma unroll
            for (int e = 0; e < 4; e++) xch[(i * 4 + e) * 128 + gtid] = acc[i][e];
        xch[(DT * 4 + 0) * 128 + gtid] = m_0;
        xch[(DT * 4 + 1) * 128 + gtid] = m_1;
        xch[(DT * 4 + 2) * 128 + gtid] = l_0;
        xch[(DT * 4 + 3) * 128 + gtid] = l_1;
    }
    __syncthreads();
    if (grp == 1) return;
    {
        const float bm0 = xch[(DT * 4 + 0) * 128 + gtid], bm1 = xch[(DT * 4 + 1) * 128 + gtid];
        const float nm0 = fmaxf(m_0, bm0), nm1 = fmaxf(m_1, bm1);
        // a group without tiles has max -inf and contributes nothing
        const float ca0 = m_0 == -INFINITY ? 0.f : exp2f(m_0 - nm0), cb0 = bm0 == -INFINITY ? 0.f : exp2f(bm0 - nm0);
        const float ca1 = m_1 == -INFINITY ? 0.f : exp2f(m_1 - nm1), cb1 = bm1 == -INFINITY ? 0.f : exp2f(bm1 - nm1);
        l_0 = l_0 * ca0 + xch[(DT * 4 + 2) * 128 + gtid] * cb0;
        l_1 = l_1 * ca1 + xch[(DT * 4 + 3) * 128 + gtid] * cb1;
#pragma unroll
        for (int i = 0; i < DT; i++) {
            acc[i][0] = acc[i][0] * ca0 + xch[(i * 4 + 0) * 128 + gtid] * cb0;
            acc[i][1] = acc[i][1] * ca0 + xch[(i * 4 + 1) * 128 + gtid] * cb0;
            acc[i][2] = acc[i][2] * ca1 + xch[(i * 4 + 2) * 128 + gtid] * cb1;
            acc[i][3] = acc[i][3] * ca1 + xch[(i * 4 + 3) * 128 + gtid] * cb1;
        }
    }
    l_0 += __shfl_xor_sync(0xffffffffu, l_0, 1);
    l_0 += __shfl_xor_sync(0xffffffffu, l_0, 2);
    l_1 += __shfl_xor_sync(0xffffffffu, l_1, 1);
    l_1 += __shfl_xor_sync(0xffffffffu, l_1, 2);
    const float i0 = 1.f / l_0, i1 = 1.f / l_1;
#pragma unroll
    for (int dt = 0; dt < DT; dt++) {
        const int col = h * HD + dt * 8 + 2 * t;
        if (r0 < M) *reinterpret_cast<uint32_t *>(o + (size_t)r0 * ld_o + col) = pack_h2(acc[dt][0] * i0, acc[dt][1] * i0);
        if (r1 < M) *reinterpret_cast<uint32_t *>(o + (size_t)r1 * ld_o + col) = pack_h2(acc[dt][2] * i1, acc[dt][3] * i1);
    }
}

template <int HD>
constexpr int attn_smem_bytes() {
    // two groups x double-buffered K and V tiles (the merge reuses the first group's)
    return 2 * 4 * kAttnKeys * HD * 2;
}
static_assert(attn_smem_bytes<16>() >= (16 / 8 * 4 + 4) * 128 * 4, "merge buffer fits in the tile buffers");

}  // namespace dfb
