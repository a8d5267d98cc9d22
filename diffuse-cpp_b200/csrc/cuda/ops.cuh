// Memory-bound kernels of one denoising step: active-set build, embedding gather,
// RMSNorm, and the remasking sampler (row statistics + ordering/commit).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "dequant.cuh"
#include "ptx.cuh"

namespace dfb {

// Device counters of a context: totals over its sequences (segments) ...
enum { CNT_M = 0, CNT_NMASKED = 1, CNT_NTILES = 2, CNT_ERR = 4, CNT_N = 8 };
// ... and per segment: active rows, masked positions, commits of the last step, whether the
// cached forward ran, offsets of the segment's rows in the active / masked lists.
enum { SEG_NACT = 0, SEG_NMASK = 1, SEG_COMMITTED = 2, SEG_USED_CACHE = 3, SEG_AOFF = 4, SEG_MOFF = 5, SEG_ERR = 6,
       SEG_N = 8 };
constexpr int kMaxSeg = 256;  // sequences one context steps together

// Block-wide exclusive scan of 0/1 flags for a 1024-thread block.  Returns this
// thread's offset; *total receives the block count.
__device__ __forceinline__ int block_scan_flag(bool flag, int *warp_tot, int *total) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned b = __ballot_sync(0xffffffffu, flag);
    const int in_warp = __popc(b & ((1u << lane) - 1));
    if (lane == 0) warp_tot[warp] = __popc(b);
    __syncthreads();
    if (warp == 0) {
        const int v = warp_tot[lane];
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        warp_tot[lane] = x - v;
        if (lane == 31) *total = x;
    }
    __syncthreads();
    const int off = warp_tot[warp] + in_warp;
    __syncthreads();
    return off;
}

// Active set of one step for segment blockIdx.x, positions [seg_off[s], seg_off[s+1])
// (diffuse-cache.h:78-115 and diffuse-sampler.cpp:143-182, per sequence).  full != 0:
// every position is active (step 0, cache off, refresh), last_changed is not touched
// (the reference does not call compute_active_set there).  Otherwise active = changed
// since the last forward ∪ masked ∪ changed within keep_active steps; an empty or
// complete active set falls back to the full forward like diffuse-sampler.cpp:165-173.
// A finished segment (done[s], no position left masked: the reference's loop has ended
// for it) contributes nothing.  Lists go to tmp_* at the segment's own offset; records
// prev_seq = seq (update_seq, cache.h:142-145).  One block of 1024 threads per segment.
__global__ void __launch_bounds__(1024) seg_prepare_kernel(int full, int step, int keep_active, const int *seg_off,
                                                           const uint8_t *done, int32_t *seq, int32_t *prev_seq,
                                                           int32_t *last_changed, const uint8_t *masked,
                                                           int *tmp_active, int *tmp_masked, int *seg_cnt) {
    __shared__ int warp_tot[32];
    __shared__ int tot;
    const int sg = blockIdx.x, p0 = seg_off[sg], n = seg_off[sg + 1] - p0;
    int *sc = seg_cnt + sg * SEG_N;
    if (done[sg]) {
        if (threadIdx.x == 0) { sc[SEG_NACT] = 0; sc[SEG_NMASK] = 0; sc[SEG_USED_CACHE] = 0; }
        return;
    }
    int base_a = 0, base_m = 0;
    for (int c0 = 0; c0 < n; c0 += 1024) {
        const int i = p0 + c0 + threadIdx.x;
        bool act = false, msk = false;
        if (c0 + (int)threadIdx.x < n) {
            msk = masked[i] != 0;
            if (full) act = true;
            else {
                const bool changed = seq[i] != prev_seq[i];
                if (changed) last_changed[i] = step;
                const int lc = last_changed[i];
                const bool recent = keep_active > 0 && lc >= 0 && (step - lc) <= keep_active;
                act = changed || msk || recent;
            }
        }
        const int oa = block_scan_flag(act, warp_tot, &tot);
        if (act) tmp_active[p0 + base_a + oa] = i;
        base_a += tot;
        __syncthreads();
        const int om = block_scan_flag(msk, warp_tot, &tot);
        if (msk) tmp_masked[p0 + base_m + om] = i;
        base_m += tot;
        __syncthreads();
    }
    const bool all = full || base_a == 0 || base_a >= n;
    for (int j = threadIdx.x; j < n; j += 1024) {
        if (all) tmp_active[p0 + j] = p0 + j;
        prev_seq[p0 + j] = seq[p0 + j];
    }
    if (threadIdx.x == 0) {
        sc[SEG_NACT] = all ? n : base_a;
        sc[SEG_NMASK] = base_m;
        sc[SEG_USED_CACHE] = all ? 0 : 1;
    }
}

// Dense lists over all segments: active rows (global positions, and positions within their
// sequence for RoPE), masked positions and the logits row each reads (Dream: max(i-1, 0)
// within its sequence, diffuse-sampler.cpp:74,235), attention tiles of <= 32 active rows
// of one segment {first row, rows, first key position, keys}, totals.  One block.
__global__ void __launch_bounds__(1024) seg_compact_kernel(int n_seg, const int *seg_off, const int *tmp_active,
                                                           const int *tmp_masked, int *seg_cnt, int shift,
                                                           int *active_pos, int *rope_pos, int *masked_pos,
                                                           int *masked_row, int4 *tiles, int *cnt) {
    __shared__ int aoff[kMaxSeg + 1], moff[kMaxSeg + 1];
    griddep_wait();
    if (threadIdx.x == 0) {
        int a = 0, m = 0, k = 0;
        for (int sg = 0; sg < n_seg; sg++) {
            int *sc = seg_cnt + sg * SEG_N;
            aoff[sg] = a;
            moff[sg] = m;
            sc[SEG_AOFF] = a;
            sc[SEG_MOFF] = m;
            const int na = sc[SEG_NACT], len = seg_off[sg + 1] - seg_off[sg];
            for (int r = 0; r < na; r += 32) tiles[k++] = make_int4(a + r, min(32, na - r), seg_off[sg], len);
            a += na;
            m += sc[SEG_NMASK];
        }
        aoff[n_seg] = a;
        moff[n_seg] = m;
        cnt[CNT_M] = a;
        cnt[CNT_NMASKED] = m;
        cnt[CNT_NTILES] = k;
    }
    __syncthreads();
    for (int sg = 0; sg < n_seg; sg++) {
        const int p0 = seg_off[sg], na = aoff[sg + 1] - aoff[sg], nm = moff[sg + 1] - moff[sg];
        for (int i = threadIdx.x; i < na; i += 1024) {
            const int pos = tmp_active[p0 + i];
            active_pos[aoff[sg] + i] = pos;
            rope_pos[aoff[sg] + i] = pos - p0;
        }
        for (int i = threadIdx.x; i < nm; i += 1024) {
            const int pos = tmp_masked[p0 + i];
            masked_pos[moff[sg] + i] = pos;
            masked_row[moff[sg] + i] = (shift && pos > p0) ? pos - 1 : pos;
        }
    }
}

// x[a] = token_embd[seq[active_pos[a]]] as f32 (ggml_get_rows, graph.cpp:43/433).
template <typename T>
__global__ void embed_kernel(const T *__restrict__ emb, int d, int n_vocab, const int32_t *__restrict__ seq,
                             const int *__restrict__ active_pos, int *__restrict__ cnt, float *__restrict__ x) {
    const int a = blockIdx.x;
    if (a >= cnt[CNT_M]) return;
    int tok = seq[active_pos[a]];
    if (tok < 0 || tok >= n_vocab) {  // a token id outside the vocabulary: report it, read row 0
        if (threadIdx.x == 0) atomicCAS(&cnt[CNT_ERR], 0, 1);
        tok = 0;
    }
    const T *src = emb + (size_t)tok * d;
    float *dst = x + (size_t)a * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        if constexpr (sizeof(T) == 2) dst[i] = __half2float(src[i]);
        else dst[i] = src[i];
    }
}

__device__ __forceinline__ uint32_t h2u_(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

__device__ __forceinline__ float block_sum(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float w = lane < nw ? red[lane] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const float r = red[32];
    __syncthreads();
    return r;
}

// h[a] = x[a] * (1 / sqrt(mean(x[a]^2) + eps)) * w  (ggml_rms_norm + ggml_mul,
// graph.cpp:51-58) as pair rows (4 bytes per value, dequant.cuh), with the residual add of the projection
// before it folded in when y is given: x[a] += y[a] first (ggml_add, graph.cpp:123 /
// :142), written back as the new residual stream.  One block per row; 8 elements per
// thread step (float4 loads); d is a multiple of 64.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float *__restrict__ x, const float *__restrict__ y,
                                                      const float *__restrict__ w, int d, float eps,
                                                      const int *__restrict__ cnt, uint8_t *__restrict__ h) {
    __shared__ float red[33];
    griddep_launch_dependents();
    griddep_wait();  // x, y and the row count come from the previous kernels
    const int a = blockIdx.x;
    if (a >= cnt[CNT_M]) return;
    float *xr = x + (size_t)a * d;
    const float *yr = y ? y + (size_t)a * d : nullptr;
    uint8_t *hr = h + (size_t)a * 4 * d;
    float ss = 0.f;
    for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
        float4 v0 = *reinterpret_cast<const float4 *>(xr + i);
        float4 v1 = *reinterpret_cast<const float4 *>(xr + i + 4);
        if (yr) {
            const float4 y0 = *reinterpret_cast<const float4 *>(yr + i);
            const float4 y1 = *reinterpret_cast<const float4 *>(yr + i + 4);
            v0.x += y0.x; v0.y += y0.y; v0.z += y0.z; v0.w += y0.w;
            v1.x += y1.x; v1.y += y1.y; v1.z += y1.z; v1.w += y1.w;
            *reinterpret_cast<float4 *>(xr + i) = v0;
            *reinterpret_cast<float4 *>(xr + i + 4) = v1;
        }
        ss += v0.x * v0.x + v0.y * v0.y + v0.z * v0.z + v0.w * v0.w;
        ss += v1.x * v1.x + v1.y * v1.y + v1.z * v1.z + v1.w * v1.w;
    }
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)d + eps);
    for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
        const float4 v0 = *reinterpret_cast<const float4 *>(xr + i);
        const float4 v1 = *reinterpret_cast<const float4 *>(xr + i + 4);
        const float4 w0 = __ldg(reinterpret_cast<const float4 *>(w + i));
        const float4 w1 = __ldg(reinterpret_cast<const float4 *>(w + i + 4));
        const float v[8] = {(v0.x * scale) * w0.x, (v0.y * scale) * w0.y, (v0.z * scale) * w0.z, (v0.w * scale) * w0.w,
                            (v1.x * scale) * w1.x, (v1.y * scale) * w1.y, (v1.z * scale) * w1.z, (v1.w * scale) * w1.w};
        store_pair8(hr, i, v);
    }
}

// Per-candidate statistics of one logits row (diffuse-sampler.cpp:34-57 and :239-255):
// top-1 value and first index (strict '>' keeps the lowest index), top-2 value (the
// largest value at any other index), entropy with the p > 1e-10 rule.  One block per
// masked position; masked_row gives the logits row it reads (Dream's shift applied).
struct Top2 {
    float best;
    int idx;
    float second;
};
__device__ __forceinline__ Top2 top2_merge(Top2 a, Top2 b) {
    Top2 r;
    const bool a_first = a.best > b.best || (a.best == b.best && a.idx < b.idx);
    if (a_first) { r.best = a.best; r.idx = a.idx; r.second = fmaxf(a.second, b.best); }
    else { r.best = b.best; r.idx = b.idx; r.second = fmaxf(b.second, a.best); }
    return r;
}

__global__ void __launch_bounds__(512) row_stats_kernel(const float *__restrict__ logits, int n_vocab,
                                                         const int *__restrict__ masked_row, int *__restrict__ cnt,
                                                         int margin, int32_t *__restrict__ cand_tok,
                                                         float *__restrict__ cand_conf, float *__restrict__ cand_ent) {
    __shared__ float red[33];
    __shared__ Top2 tred[16];
    const int b = blockIdx.x;
    if (b >= cnt[CNT_NMASKED]) return;
    const int row = masked_row[b];
    const float *z = logits + (size_t)row * n_vocab;
    // Each pass reads the row as float4 (n_vocab % 4 == 0) with four loads in flight per
    // thread; a thread visits its elements in increasing index order, so the strict '>'
    // still keeps the lowest index of equal maxima.
    const bool vec = (n_vocab & 3) == 0;
    const int n4 = n_vocab >> 2;
    const float4 *z4 = reinterpret_cast<const float4 *>(z);
    Top2 t{-INFINITY, 0x7fffffff, -1e30f};
    auto see = [&](float x, int v) {
        if (x > t.best) { t.second = fmaxf(t.second, t.best); t.best = x; t.idx = v; }
        else t.second = fmaxf(t.second, x);
    };
    if (vec) {
        int q = threadIdx.x;
        for (; q + 3 * (int)blockDim.x < n4; q += 4 * blockDim.x) {
            float4 f[4];
#pragma unroll
            for (int u = 0; u < 4; u++) f[u] = z4[q + u * blockDim.x];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int v = 4 * (q + u * blockDim.x);
                see(f[u].x, v); see(f[u].y, v + 1); see(f[u].z, v + 2); see(f[u].w, v + 3);
            }
        }
        for (; q < n4; q += blockDim.x) {
            const float4 f = z4[q];
            see(f.x, 4 * q); see(f.y, 4 * q + 1); see(f.z, 4 * q + 2); see(f.w, 4 * q + 3);
        }
    } else {
        for (int v = threadIdx.x; v < n_vocab; v += blockDim.x) see(z[v], v);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.best = __shfl_xor_sync(0xffffffffu, t.best, o);
        u.idx = __shfl_xor_sync(0xffffffffu, t.idx, o);
        u.second = __shfl_xor_sync(0xffffffffu, t.second, o);
        t = top2_merge(t, u);
    }
    if (lane == 0) tred[warp] = t;
    __syncthreads();
    if (warp == 0) {
        t = lane < (int)(blockDim.x >> 5) ? tred[lane] : Top2{-INFINITY, 0x7fffffff, -1e30f};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            Top2 u;
            u.best = __shfl_xor_sync(0xffffffffu, t.best, o);
            u.idx = __shfl_xor_sync(0xffffffffu, t.idx, o);
            u.second = __shfl_xor_sync(0xffffffffu, t.second, o);
            t = top2_merge(t, u);
        }
        if (lane == 0) tred[0] = t;
    }
    __syncthreads();
    t = tred[0];
    const float mx = t.best;
    float se = 0.f;
    if (vec) {
        int q = threadIdx.x;
        for (; q + 3 * (int)blockDim.x < n4; q += 4 * blockDim.x) {
            float4 f[4];
#pragma unroll
            for (int u = 0; u < 4; u++) f[u] = z4[q + u * blockDim.x];
#pragma unroll
            for (int u = 0; u < 4; u++) se += expf(f[u].x - mx) + expf(f[u].y - mx) + expf(f[u].z - mx) + expf(f[u].w - mx);
        }
        for (; q < n4; q += blockDim.x) {
            const float4 f = z4[q];
            se += expf(f.x - mx) + expf(f.y - mx) + expf(f.z - mx) + expf(f.w - mx);
        }
    } else {
        for (int v = threadIdx.x; v < n_vocab; v += blockDim.x) se += expf(z[v] - mx);
    }
    se = block_sum(se, red);
    const float log_sum = logf(se);
    float ent = 0.f;
    auto term = [&](float x) {
        const float lp = (x - mx) - log_sum;
        const float p = expf(lp);
        if (p > 1e-10f) ent -= p * lp;
    };
    if (vec) {
        int q = threadIdx.x;
        for (; q + 3 * (int)blockDim.x < n4; q += 4 * blockDim.x) {
            float4 f[4];
#pragma unroll
            for (int u = 0; u < 4; u++) f[u] = z4[q + u * blockDim.x];
#pragma unroll
            for (int u = 0; u < 4; u++) { term(f[u].x); term(f[u].y); term(f[u].z); term(f[u].w); }
        }
        for (; q < n4; q += blockDim.x) {
            const float4 f = z4[q];
            term(f.x); term(f.y); term(f.z); term(f.w);
        }
    } else {
        for (int v = threadIdx.x; v < n_vocab; v += blockDim.x) term(z[v]);
    }
    ent = block_sum(ent, red);
    if (threadIdx.x == 0) {
        if (t.idx < 0 || t.idx >= n_vocab) {  // no value compared greater than -inf (NaN logits): report it
            atomicCAS(&cnt[CNT_ERR], 0, 2);
            t.idx = 0;
        }
        cand_tok[b] = t.idx;
        cand_conf[b] = margin ? (t.best - t.second) : t.best;
        cand_ent[b] = ent;
    }
}

__device__ __forceinline__ uint32_t ordered_u32(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Ordering + commit (diffuse-sampler.cpp:277-323) of segment blockIdx.x: its candidates
// are [moff, moff + n) of the masked list, in ascending position order; keys: confidence
// descending (LOW_CONFIDENCE / MASKGIT_PLUS / TOPK_MARGIN) or entropy ascending
// (ENTROPY_EXIT), ties by ascending position; RANDOM uses the host's shuffle of the
// segment's candidate indices (order[moff ..]).  sched[s] is tokens_to_unmask of the
// segment's own loop; a negative value marks a finished segment.  One block of 1024
// threads per segment; dynamic shared memory holds the padded key array (8 bytes per
// candidate, power of two).
__global__ void __launch_bounds__(1024) select_commit_kernel(int remasking, const int *__restrict__ sched, float tau,
                                                             int key_cap, const int32_t *__restrict__ order,
                                                             const int *__restrict__ masked_pos,
                                                             const int32_t *__restrict__ cand_tok,
                                                             const float *__restrict__ cand_conf,
                                                             const float *__restrict__ cand_ent, int32_t *seq,
                                                             uint8_t *masked, int32_t *commit_pos,
                                                             int32_t *commit_tok, int *seg_cnt) {
    extern __shared__ unsigned long long keys[];
    __shared__ int n_easy_s;
    int *sc = seg_cnt + blockIdx.x * SEG_N;
    const int n = sc[SEG_NMASK], moff = sc[SEG_MOFF], n_unmask_sched = sched[blockIdx.x];
    if (n_unmask_sched < 0) {  // finished segment
        if (threadIdx.x == 0) sc[SEG_COMMITTED] = 0;
        return;
    }
    int np = 1;
    while (np < n) np <<= 1;
    if (np > key_cap) {  // host and device disagree on the candidate count: commit nothing
        if (threadIdx.x == 0) { sc[SEG_ERR] = 1; sc[SEG_COMMITTED] = 0; }
        return;
    }
    if (threadIdx.x == 0) n_easy_s = 0;
    __syncthreads();
    int easy = 0;
    for (int b = threadIdx.x; b < np; b += blockDim.x) {
        unsigned long long k = ~0ull;
        if (b < n) {
            uint32_t k32;
            if (remasking == 2) {
                k32 = ordered_u32(cand_ent[moff + b]);
                easy += cand_ent[moff + b] < tau ? 1 : 0;
            } else {
                k32 = ~ordered_u32(cand_conf[moff + b]);
            }
            k = ((unsigned long long)k32 << 32) | (uint32_t)b;
        }
        keys[b] = k;
    }
    if (remasking == 2 && easy) atomicAdd(&n_easy_s, easy);
    __syncthreads();
    if (remasking != 1) {
        for (int size = 2; size <= np; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = threadIdx.x; i < np; i += blockDim.x) {
                    const int j = i ^ stride;
                    if (j > i) {
                        const bool up = (i & size) == 0;
                        const unsigned long long a = keys[i], c = keys[j];
                        if ((a > c) == up) { keys[i] = c; keys[j] = a; }
                    }
                }
                __syncthreads();
            }
    }
    int n_unmask = n_unmask_sched;
    if (remasking == 2) n_unmask = max(n_unmask, n_easy_s);
    n_unmask = min(n_unmask, n);
    for (int j = threadIdx.x; j < n_unmask; j += blockDim.x) {
        const int b = remasking == 1 ? order[moff + j] : (int)(keys[j] & 0xffffffffu);
        const int pos = masked_pos[moff + b];
        const int tok = cand_tok[moff + b];
        seq[pos] = tok;
        masked[pos] = 0;
        commit_pos[moff + j] = pos;
        commit_tok[moff + j] = tok;
    }
    if (threadIdx.x == 0) {
        sc[SEG_COMMITTED] = n_unmask;
        sc[SEG_NMASK] = n - n_unmask;
    }
}

// X (f32 [rows][K], host-provided for dfb_linear) -> pair rows (4 K bytes each); K multiple of 64.
// ── tensor parallelism: the sampler statistics of vocabulary-parallel logits rows ──
// Each rank holds the logits of its vocabulary rows [v0, v0 + n).  Per candidate, rank r
// computes over its columns the maximum m_r, its first index, the second value s_r and
// se_r = sum exp(x - m_r) (tp_stats_kernel); after an all-gather every rank combines them
// (tp_combine_kernel): the maximum over ranks (ties to the lower vocabulary index, i.e. the
// lower rank), the second value (the largest at any other index), and
// Z = sum_r se_r exp(m_r - M); the entropy terms with the global max and log Z are then summed
// over each rank's columns (tp_entropy_kernel) and all-reduced.  The decisions are those of
// row_stats_kernel over the whole row up to the order of the f32 sums.
__global__ void __launch_bounds__(512) tp_stats_kernel(const float *__restrict__ logits, int n, int v0,
                                                        const int *__restrict__ masked_row, const int *__restrict__ cnt,
                                                        float4 *__restrict__ stats) {
    __shared__ float red[33];
    __shared__ Top2 tred[16];
    const int b = blockIdx.x;
    if (b >= cnt[CNT_NMASKED]) return;
    const float *z = logits + (size_t)masked_row[b] * n;
    Top2 t{-INFINITY, 0x7fffffff, -1e30f};
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
        const float x = z[v];
        if (x > t.best) { t.second = fmaxf(t.second, t.best); t.best = x; t.idx = v; }
        else t.second = fmaxf(t.second, x);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.best = __shfl_xor_sync(0xffffffffu, t.best, o);
        u.idx = __shfl_xor_sync(0xffffffffu, t.idx, o);
        u.second = __shfl_xor_sync(0xffffffffu, t.second, o);
        t = top2_merge(t, u);
    }
    if (lane == 0) tred[warp] = t;
    __syncthreads();
    if (warp == 0) {
        t = lane < (int)(blockDim.x >> 5) ? tred[lane] : Top2{-INFINITY, 0x7fffffff, -1e30f};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            Top2 u;
            u.best = __shfl_xor_sync(0xffffffffu, t.best, o);
            u.idx = __shfl_xor_sync(0xffffffffu, t.idx, o);
            u.second = __shfl_xor_sync(0xffffffffu, t.second, o);
            t = top2_merge(t, u);
        }
        if (lane == 0) tred[0] = t;
    }
    __syncthreads();
    t = tred[0];
    float se = 0.f;
    for (int v = threadIdx.x; v < n; v += blockDim.x) se += expf(z[v] - t.best);
    se = block_sum(se, red);
    if (threadIdx.x == 0) stats[b] = make_float4(t.best, t.second, se, __int_as_float(v0 + t.idx));
}
// gath: [ranks][candidates] of tp_stats_kernel's values; gstat[b] = (global max, log Z).
__global__ void tp_combine_kernel(const float4 *__restrict__ gath, int ranks, int stride, const int *__restrict__ cnt,
                                  int margin, int32_t *__restrict__ cand_tok, float *__restrict__ cand_conf,
                                  float2 *__restrict__ gstat) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= cnt[CNT_NMASKED]) return;
    float best = -INFINITY, second = -1e30f;
    int idx = 0x7fffffff, br = 0;
    for (int r = 0; r < ranks; r++) {  // ranks in vocabulary order: a tie keeps the lower index
        const float4 s = gath[(size_t)r * stride + b];
        if (s.x > best) { second = fmaxf(second, best); best = s.x; idx = __float_as_int(s.w); br = r; }
        else second = fmaxf(second, s.x);
        second = fmaxf(second, s.y);
    }
    (void)br;
    float Z = 0.f;
    for (int r = 0; r < ranks; r++) {
        const float4 s = gath[(size_t)r * stride + b];
        Z += s.z * expf(s.x - best);
    }
    cand_tok[b] = idx;
    cand_conf[b] = margin ? (best - second) : best;
    gstat[b] = make_float2(best, logf(Z));
}
__global__ void __launch_bounds__(512) tp_entropy_kernel(const float *__restrict__ logits, int n,
                                                          const int *__restrict__ masked_row, const int *__restrict__ cnt,
                                                          const float2 *__restrict__ gstat, float *__restrict__ ent_part) {
    __shared__ float red[33];
    const int b = blockIdx.x;
    if (b >= cnt[CNT_NMASKED]) return;
    const float *z = logits + (size_t)masked_row[b] * n;
    const float mx = gstat[b].x, log_sum = gstat[b].y;
    float ent = 0.f;
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
        const float lp = (z[v] - mx) - log_sum;
        const float p = expf(lp);
        if (p > 1e-10f) ent -= p * lp;
    }
    ent = block_sum(ent, red);
    if (threadIdx.x == 0) ent_part[b] = ent;
}

// Sampling at temperature > 0 (diffuse-sampler.cpp:256-269): probabilities
// p_v = expf((l_v - max) / T) / sum_v expf(...) in f32, then the draw of
// std::discrete_distribution<int>(p) with the uniform u the host took from the loop's
// mt19937 (std::generate_canonical<double, 53>, one per candidate in position order): the
// weights as doubles divided by their double sum, cumulative sums, the first index whose
// cumulative sum reaches u (the last index if rounding leaves every sum below u, as the
// distribution sets its last cumulative sum to 1).  The confidence is p of the drawn
// token.  The sums are block reductions here, serial in the reference, and the device
// expf is not the host libm's: p agrees to a few f32 ulp, so a draw can differ only when u
// falls within that distance of a cumulative sum.  One block per masked candidate.
__device__ __forceinline__ double block_sum_d(double v, double *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double w = lane < nw ? red[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const double r = red[32];
    __syncthreads();
    return r;
}
constexpr int kSampleThreads = 512;
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const float *__restrict__ logits, int n_vocab,
                                                                 const int *__restrict__ masked_row, const int *__restrict__ cnt,
                                                                 float temperature, const double *__restrict__ unif,
                                                                 int32_t *__restrict__ cand_tok, float *__restrict__ cand_conf) {
    __shared__ float red[33];
    __shared__ double redd[33];
    __shared__ double scan[kSampleThreads];
    const int b = blockIdx.x;
    if (b >= cnt[CNT_NMASKED]) return;
    const float *z = logits + (size_t)masked_row[b] * n_vocab;
    const int tid = threadIdx.x;
    // max
    float mx = -INFINITY;
    for (int v = tid; v < n_vocab; v += blockDim.x) mx = fmaxf(mx, z[v]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    if (tid < 32) {
        float w = tid < (int)(blockDim.x >> 5) ? red[tid] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (tid == 0) red[32] = w;
    }
    __syncthreads();
    mx = red[32];
    __syncthreads();
    auto prob = [&](int v) { return expf((z[v] - mx) / temperature); };
    float se = 0.f;
    for (int v = tid; v < n_vocab; v += blockDim.x) se += prob(v);
    const float S = block_sum(se, red);
    // the distribution's weights: p_v = f32(prob / S) as doubles, normalised by their sum
    double sd = 0.0;
    for (int v = tid; v < n_vocab; v += blockDim.x) sd += (double)(prob(v) / S);
    const double D = block_sum_d(sd, redd);
    // cumulative sums over contiguous chunks: thread t covers [t C, t C + C)
    const int C = (n_vocab + blockDim.x - 1) / blockDim.x;
    const int v0 = min(n_vocab, tid * C), v1 = min(n_vocab, v0 + C);
    double cs = 0.0;
    for (int v = v0; v < v1; v++) cs += (double)(prob(v) / S) / D;
    scan[tid] = cs;
    __syncthreads();
    for (int off = 1; off < (int)blockDim.x; off <<= 1) {  // inclusive scan (Hillis-Steele)
        const double add = tid >= off ? scan[tid - off] : 0.0;
        __syncthreads();
        scan[tid] += add;
        __syncthreads();
    }
    const double u = unif[b];
    const double before = tid ? scan[tid - 1] : 0.0;
    int pick = -1;
    if (u <= 0.0) {
        if (tid == 0) pick = 0;  // the first cumulative sum is >= 0
    } else if (before < u && scan[tid] >= u) {  // the crossing lies in this thread's chunk
        double c = before;
        for (int v = v0; v < v1; v++) {
            c += (double)(prob(v) / S) / D;
            if (c >= u) { pick = v; break; }
        }
        if (pick < 0) pick = v1 - 1;
    } else if (tid == (int)blockDim.x - 1 && scan[tid] < u) {
        pick = n_vocab - 1;
    }
    if (pick >= 0) {
        cand_tok[b] = pick;
        cand_conf[b] = prob(pick) / S;
    }
}

__global__ void f32_to_pair_kernel(const float *__restrict__ x, uint8_t *__restrict__ y, int rows, int K) {
    const size_t groups = (size_t)rows * (K / 8);
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < groups; g += (size_t)gridDim.x * blockDim.x) {
        const size_t r = g / (K / 8);
        const int i = (int)(g % (K / 8)) * 8;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = x[r * K + i + e];
        store_pair8(y + r * 4 * K, i, v);
    }
}

}  // namespace dfb
