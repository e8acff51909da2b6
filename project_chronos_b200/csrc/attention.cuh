// attention.cuh — one-token decode of the hybrid attention
// (chronos/model/hybrid_attention.py) and the residual add + RMSNorm of a block.
//
// Both decode kernels run one thread-block cluster per (kv head g, batch row
// b), `splits` CTAs of 256 threads that share the cached positions, and do, in
// one launch: the per-head RMSNorms of the new token's projections, RoPE at its
// position, the cache append, the scores of the group's n_rep query heads
// against every cached token, the softmax and the weighted sum.
// Arithmetic is fp32; values are rounded to the layer type where the
// reference's torch code holds a tensor in that type (norm and RoPE outputs,
// the new cache entries, the softmax probabilities, the output), so a bf16
// layer rounds where the reference's bf16 run rounds.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace chronos {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxRep = 8;

struct AttnParams {
    int heads, kv_heads, rep, head_dim, rope_dim, nope, latent, window, max_len, table_len;
    int stage_w;   // MLA: 1 = the group's weight slices are staged in shared memory
    int splits;    // CTAs per (kv head, batch row): the cluster size
    int cap;       // score slots per head and CTA: ceil(cached positions / splits)
    float eps, scale;
    const int32_t* pos;
    const void* proj;
    const void* norm_q;
    const void* norm_q2;
    const void* norm_kv;
    const void* w_krope;
    const void* w_knope;
    const void* w_v;
    const void* cos;
    const void* sin;
    void* cache_a;
    void* cache_b;
    void* out;
};

struct NormParams {
    int64_t rows;
    int width;
    float eps;
    int x_fp32;  // 1: x is fp32, rounded to T as read
    const void* x;
    const void* residual;
    void* sum_out;
    const void* weight;
    void* out;
};

template <typename T>
__device__ __forceinline__ float round_to(float v) {
    return to_f32<T>(from_f32<T>(v));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// In place: v = round(w * (v * rsqrt(mean(v^2) + eps))) over `len` values, by one warp.
template <typename T>
__device__ __forceinline__ void warp_rmsnorm(float* v, int len, const T* w, float eps, int lane) {
    float ss = 0.0f;
    for (int i = lane; i < len; i += 32) ss = fmaf(v[i], v[i], ss);
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(len) + eps);
    __syncwarp();
    for (int i = lane; i < len; i += 32) v[i] = round_to<T>(to_f32<T>(w[i]) * (v[i] * inv));
    __syncwarp();
}

// warp_rmsnorm with the norm weight already in shared memory (fp32).
template <typename T>
__device__ __forceinline__ void warp_rmsnorm_s(float* v, int len, const float* w, float eps, int lane) {
    float ss = 0.0f;
    for (int i = lane; i < len; i += 32) ss = fmaf(v[i], v[i], ss);
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(len) + eps);
    __syncwarp();
    for (int i = lane; i < len; i += 32) v[i] = round_to<T>(w[i] * (v[i] * inv));
    __syncwarp();
}

// RoPE as the reference writes it (minimind apply_rotary_pos_emb):
// x*cos + rotate_half(x)*sin over `len` values, with cos/sin the first `len`
// columns of the table row; each product and the sum rounded to T.  `tmp`
// holds the rotated values until every thread has read the inputs.
template <typename T>
__device__ __forceinline__ float rope_value(const float* x, int i, int len, const T* crow, const T* srow) {
    const int half = len >> 1;
    const float rot = i < half ? -x[i + half] : x[i - half];
    return round_to<T>(round_to<T>(x[i] * to_f32<T>(crow[i])) + round_to<T>(rot * to_f32<T>(srow[i])));
}

// rope_value with the cos/sin row already in shared memory (fp32).
template <typename T>
__device__ __forceinline__ float rope_value_s(const float* x, int i, int len, const float* c, const float* sn) {
    const int half = len >> 1;
    const float rot = i < half ? -x[i + half] : x[i - half];
    return round_to<T>(round_to<T>(x[i] * c[i]) + round_to<T>(rot * sn[i]));
}

// ---------------------------------------------------------------------------
// residual add + RMSNorm: out = RMSNorm(x + residual) * weight, one block per row
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) add_rmsnorm_kernel(NormParams p) {
    extern __shared__ float nsm[];
    float* xs = nsm;                     // [width]
    float* red = nsm + p.width;          // [kAttnWarps]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* x = static_cast<const T*>(p.x);
    const T* res = static_cast<const T*>(p.residual);
    const T* w = static_cast<const T*>(p.weight);
    T* sum_out = static_cast<T*>(p.sum_out);
    T* out = static_cast<T*>(p.out);
    pdl_wait();   // launched early behind the kernel that writes x (programmatic launch)
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const int64_t base = r * p.width;
        float ss = 0.0f;
        for (int c = threadIdx.x; c < p.width; c += kAttnThreads) {
            float v = p.x_fp32 ? round_to<T>(static_cast<const float*>(p.x)[base + c]) : to_f32<T>(x[base + c]);
            if (res != nullptr) v = round_to<T>(v + to_f32<T>(res[base + c]));
            if (sum_out != nullptr) sum_out[base + c] = from_f32<T>(v);
            xs[c] = v;
            ss = fmaf(v, v, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < kAttnWarps; ++i) tot += red[i];
        const float inv = rsqrtf(tot / static_cast<float>(p.width) + p.eps);
        for (int c = threadIdx.x; c < p.width; c += kAttnThreads)
            out[base + c] = from_f32<T>(to_f32<T>(w[c]) * (xs[c] * inv));
        __syncthreads();
    }
}

// The same with one warp per row (rows of width <= 256 * VPL, width % 8 == 0,
// 16-byte aligned): each lane keeps its VPL 8-column groups in registers, one
// warp sum, no block barrier.  8 rows per block.
template <typename T, int VPL>
__global__ void __launch_bounds__(kAttnThreads) add_rmsnorm_warp_kernel(NormParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kAttnWarps + warp;
    pdl_wait();   // launched early behind the kernel that writes x (programmatic launch)
    if (r >= p.rows) return;
    const int nv = p.width / 8;
    const int64_t base = r * p.width;
    const T* x = static_cast<const T*>(p.x) + base;
    const T* res = p.residual != nullptr ? static_cast<const T*>(p.residual) + base : nullptr;
    const T* w = static_cast<const T*>(p.weight);
    float v[VPL][8], wv[VPL][8];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c8 = lane + 32 * i;
        if (c8 < nv) {
            load8<T>(w + c8 * 8, wv[i]);   // issued with the row's loads, used after the sum
            if (p.x_fp32) {
                load8<float>(static_cast<const float*>(p.x) + base + c8 * 8, v[i]);
#pragma unroll
                for (int u = 0; u < 8; ++u) v[i][u] = round_to<T>(v[i][u]);
            } else {
                load8<T>(x + c8 * 8, v[i]);
            }
            if (res != nullptr) {
                float rr[8];
                load8<T>(res + c8 * 8, rr);
#pragma unroll
                for (int u = 0; u < 8; ++u) v[i][u] = round_to<T>(v[i][u] + rr[u]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) ss = fmaf(v[i][u], v[i][u], ss);
        }
    }
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(p.width) + p.eps);
    T* sum_out = p.sum_out != nullptr ? static_cast<T*>(p.sum_out) + base : nullptr;
    T* out = static_cast<T*>(p.out) + base;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c8 = lane + 32 * i;
        if (c8 < nv) {
            if (sum_out != nullptr) store8<T>(sum_out + c8 * 8, v[i]);
            float o[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) o[u] = wv[i][u] * (v[i][u] * inv);
            store8<T>(out + c8 * 8, o);
        }
    }
}

// ---------------------------------------------------------------------------
// arg-max of every row (the greedy pick of a decode step): the index of the
// first maximal value, NaN counting as the maximum (as torch.argmax does).
// One block per row, threads over columns, then a warp and a block reduction.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
    const bool vn = v != v, bn = bv != bv;
    if (vn || bn) return vn && (!bn || i < bi);
    return v > bv || (v == bv && i < bi);
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads) argmax_rows_kernel(const T* x, int64_t rows, int cols,
                                                                   int64_t* out) {
    __shared__ float s_v[kAttnWarps];
    __shared__ int s_i[kAttnWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();   // launched early behind the kernel that writes x (programmatic launch)
    // rows of 8-element groups on 16-byte boundaries: each thread loads up to 4
    // groups at once (one memory round trip for rows of up to 8192 elements)
    const bool vec = cols % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* row = x + r * cols;
        float bv = -INFINITY;
        int bi = cols;
        if (vec) {
            const int G = cols / 8;
            for (int g0 = threadIdx.x; g0 < G; g0 += 4 * kAttnThreads) {
                float v[4][8];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (g0 + j * kAttnThreads < G) load8<T>(row + (g0 + j * kAttnThreads) * 8, v[j]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int g = g0 + j * kAttnThreads;
                    if (g < G)
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            if (argmax_better(v[j][u], g * 8 + u, bv, bi)) { bv = v[j][u]; bi = g * 8 + u; }
                }
            }
        } else {
            for (int c = threadIdx.x; c < cols; c += kAttnThreads) {
                const float v = to_f32<T>(row[c]);
                if (argmax_better(v, c, bv, bi)) { bv = v; bi = c; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { s_v[warp] = bv; s_i[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kAttnWarps; ++w)
                if (argmax_better(s_v[w], s_i[w], bv, bi)) { bv = s_v[w]; bi = s_i[w]; }
            out[r] = bi < cols ? bi : 0;
        }
        __syncthreads();
    }
}

// Start copying `count` elements (a multiple of 16 bytes) into shared memory
// with 16-byte asynchronous copies (every copy of the block in flight at once);
// stage_rows_wait() then __syncthreads() make them visible.
template <typename T>
__device__ __forceinline__ void stage_rows(T* dst, const T* src, int count) {
    constexpr int EPV = 16 / static_cast<int>(sizeof(T));
    for (int i = threadIdx.x; i < count / EPV; i += kAttnThreads) {
        const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(reinterpret_cast<uint4*>(dst) + i));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d),
                     "l"(reinterpret_cast<const uint4*>(src) + i)
                     : "memory");
    }
}
__device__ __forceinline__ void stage_rows_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Lanes per cached row in the weighted sums: one lane per 8-column group,
// rounded up to a power of two (at least 4), so 32 / LPP rows per warp step.
__host__ __device__ constexpr int attn_lpp(int groups) {
    return groups <= 4 ? 4 : groups <= 8 ? 8 : groups <= 16 ? 16 : 32;
}

// Weighted sum of `n` cached rows for every head of the group:
// out[h][c] = sum_t p[h][t] * row_t[c] for the `width` (<= 256) columns of a
// row, rows `stride` elements apart; the row at `fresh_t` comes from shared
// memory (`fresh`, fp32) instead.  Lanes take 8-column groups (16-byte loads,
// a row read by consecutive lanes), the 32 / LPP row slots of a warp and the 8
// warps take every (8 * 32 / LPP)-th row; the slots are summed by shuffles,
// the warps through `red` [8][REP][width] in shared memory, in warp order.
// `emit(h, c, value)` receives each result.  Every thread of the block calls it.
template <typename T, int REP, typename Emit>
__device__ __forceinline__ void weighted_rows(const T* rows, int64_t stride, int n, int width, const float* p,
                                              int p_stride, int fresh_t, const float* fresh, float* red,
                                              int warp, int lane, Emit&& emit) {
    const int G = width / 8;
    const int lpp = attn_lpp(G), pp = 32 / lpp;
    const int gl = lane % lpp, ps = lane / lpp;
    float acc[REP][8];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[h][u] = 0.0f;
    if (gl < G) {
#pragma unroll 2
        for (int t = warp * pp + ps; t < n; t += kAttnWarps * pp) {
            float v[8];
            if (t == fresh_t) {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = fresh[gl * 8 + u];
            } else {
                load8<T>(rows + static_cast<int64_t>(t) * stride + gl * 8, v);
            }
#pragma unroll
            for (int h = 0; h < REP; ++h) {
                const float ph = p[h * p_stride + t];
#pragma unroll
                for (int u = 0; u < 8; ++u) acc[h][u] = fmaf(ph, v[u], acc[h][u]);
            }
        }
    }
    for (int o = lpp; o < 32; o <<= 1)
#pragma unroll
        for (int h = 0; h < REP; ++h)
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[h][u] += __shfl_xor_sync(0xffffffffu, acc[h][u], o);
    if (ps == 0 && gl < G)
#pragma unroll
        for (int h = 0; h < REP; ++h) {
            float4* dst = reinterpret_cast<float4*>(red + (warp * REP + h) * width + gl * 8);
            dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
            dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
        }
    __syncthreads();
    for (int i = threadIdx.x; i < REP * width; i += kAttnThreads) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) v += red[w * REP * width + i];
        emit(i / width, i % width, v);
    }
}

// ---------------------------------------------------------------------------
// Split decode.  The cached positions of one (kv head g, batch row b) are
// divided over a thread-block cluster of `splits` CTAs.  Every CTA computes the
// token's query (norms, RoPE) itself; CTA s scores positions
// [s*chunk, (s+1)*chunk).  The cluster agrees on each head's maximum and
// exponential sum through distributed shared memory before any probability is
// rounded, so every probability is the one a single block would round; each
// CTA then forms the weighted sum of its positions, and the partial sums are
// added in CTA order.  Four cluster barriers, reached by every thread of every
// CTA; the last keeps each CTA's shared memory alive until its peers have read
// it.  The kernels are instantiated per REP (query heads per kv head).
// ---------------------------------------------------------------------------

// Scores of positions [t_lo, t_hi) for every head of the group into
// sc[h * cap + t - t_lo].  Four lanes per position (lane sub takes the 8-column
// groups sub, sub + 4, ...), summed by two butterfly steps.  Column group
// q < w1/8 comes from `rows1` (row stride st1, query q1 [REP][w1]), the others
// from `rows2` (st2, q2 [REP][w2]); the row at `fresh_t` comes from shared
// memory (f1, f2) instead.  Queries are 16-byte aligned in shared memory.
template <typename T, int REP>
__device__ __forceinline__ void split_scores(const T* rows1, int64_t st1, const float* q1, int w1, const float* f1,
                                             const T* rows2, int64_t st2, const float* q2, int w2,
                                             const float* f2, int t_lo, int t_hi, int fresh_t, float scale,
                                             float* sc, int cap, int warp, int lane) {
    const int g1 = w1 / 8, gall = g1 + w2 / 8, sub = lane & 3;
    for (int base = t_lo + warp * 8; base < t_hi; base += kAttnWarps * 8) {   // uniform per warp
        const int t = base + (lane >> 2);
        const bool ok = t < t_hi;
        float acc[REP];
#pragma unroll
        for (int h = 0; h < REP; ++h) acc[h] = 0.0f;
        if (ok) {
            const bool fresh = t == fresh_t;
#pragma unroll 4
            for (int q = sub; q < gall; q += 4) {
                const bool first = q < g1;
                const int c = first ? q * 8 : (q - g1) * 8;
                float v[8];
                if (fresh) {
                    const float* f = first ? f1 : f2;
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = f[c + u];
                } else {
                    load8<T>(first ? rows1 + static_cast<int64_t>(t) * st1 + c
                                   : rows2 + static_cast<int64_t>(t) * st2 + c, v);
                }
                const float* qq = first ? q1 + c : q2 + c;
                const int qs = first ? w1 : w2;
#pragma unroll
                for (int h = 0; h < REP; ++h) {
                    const float4 a = reinterpret_cast<const float4*>(qq + h * qs)[0];
                    const float4 b = reinterpret_cast<const float4*>(qq + h * qs)[1];
                    acc[h] = fmaf(a.x, v[0], acc[h]);
                    acc[h] = fmaf(a.y, v[1], acc[h]);
                    acc[h] = fmaf(a.z, v[2], acc[h]);
                    acc[h] = fmaf(a.w, v[3], acc[h]);
                    acc[h] = fmaf(b.x, v[4], acc[h]);
                    acc[h] = fmaf(b.y, v[5], acc[h]);
                    acc[h] = fmaf(b.z, v[6], acc[h]);
                    acc[h] = fmaf(b.w, v[7], acc[h]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < REP; ++h) {
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
        }
        if (ok && sub == 0)
#pragma unroll
            for (int h = 0; h < REP; ++h) sc[h * cap + (t - t_lo)] = acc[h] * scale;
    }
}

// The cluster-wide softmax of the scores sc[h * cap + i], i < cnt, rounded to T
// in place.  Each CTA publishes its maximum m_r and sum l_r = sum exp(s - m_r)
// per head (red[0..REP) and red[kAttnMaxRep..+REP)); after one cluster barrier
// every CTA forms M = max m_r and L = sum_r l_r exp(m_r - M) in CTA order and
// rounds p = exp(s - M) / L.
template <typename T, int REP>
__device__ __forceinline__ void split_softmax(cooperative_groups::cluster_group& cluster, float* sc, int cap,
                                              int cnt, float* red, int warp, int lane) {
    const int splits = static_cast<int>(cluster.num_blocks());
    for (int h = warp; h < REP; h += kAttnWarps) {
        float m = -INFINITY;
        for (int i = lane; i < cnt; i += 32) m = fmaxf(m, sc[h * cap + i]);
        m = warp_max(m);
        float sum = 0.0f;
        for (int i = lane; i < cnt; i += 32) sum += __expf(sc[h * cap + i] - m);
        sum = warp_sum(sum);
        if (lane == 0) {
            red[h] = m;
            red[kAttnMaxRep + h] = sum;
        }
    }
    cluster.sync();
    for (int h = warp; h < REP; h += kAttnWarps) {
        float mr = lane < splits ? cluster.map_shared_rank(red, lane)[h] : -INFINITY;
        const float lr = lane < splits ? cluster.map_shared_rank(red, lane)[kAttnMaxRep + h] : 0.0f;
        const float M = warp_max(mr);
        // l_r exp(m_r - M), summed by lane 0 in CTA order (an empty CTA adds 0)
        const float term = lr > 0.0f ? lr * __expf(mr - M) : 0.0f;
        float tot = 0.0f;
        for (int r = 0; r < splits; ++r) tot += __shfl_sync(0xffffffffu, term, r);
        const float inv = 1.0f / tot;
        for (int i = lane; i < cnt; i += 32) sc[h * cap + i] = round_to<T>(__expf(sc[h * cap + i] - M) * inv);
    }
}

// Start moving rows [t_lo, t_hi) of a cache (`bytes` per row, rows `stride`
// elements apart) towards L2 while the CTA computes its query.
template <typename T>
__device__ __forceinline__ void prefetch_rows(const T* rows, int64_t stride, int t_lo, int t_hi, int bytes) {
    const int lines = (bytes + 127) / 128;
    for (int i = threadIdx.x; i < (t_hi - t_lo) * lines; i += kAttnThreads) {
        const int t = t_lo + i / lines, l = i % lines;
        prefetch_l2(reinterpret_cast<const uint8_t*>(rows + static_cast<int64_t>(t) * stride) + l * 128);
    }
}

// Floats of the weighted-sum reduction buffer of a CTA.
__host__ __device__ constexpr int attn_red_floats(int rep, int width) { return kAttnWarps * rep * width; }

// ---------------------------------------------------------------------------
// MLA decode (hybrid_attention.py:116-179 with a cache, S = 1)
// ---------------------------------------------------------------------------
template <typename T, int REP>
__global__ void __launch_bounds__(kAttnThreads, REP <= 4 ? 3 : 2) mla_decode_kernel(AttnParams p) {
    namespace cg = cooperative_groups;
    constexpr int rep = REP;
    extern __shared__ __align__(16) float msm[];
    cg::cluster_group cluster = cg::this_cluster();
    pdl_wait();   // launched early behind the projection that writes proj (programmatic launch)
    const int pos = *p.pos;   // first: the rotary rows and the CTA's positions depend on it
    const int splits = p.splits;
    const int sidx = blockIdx.x % splits, g = blockIdx.x / splits, b = blockIdx.y;
    const int nope = p.nope, R = p.rope_dim, L = p.latent, D = p.head_dim, cap = p.cap;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this CTA's output rows d0 .. d1 - 1 of the value up-projection
    const int dper = (D + splits - 1) / splits;
    const int d0 = min(D, sidx * dper), d1 = min(D, d0 + dper);
    // the group's k_nope_proj [nope, L] and k_rope_proj [R, L] slices and this
    // CTA's v_proj rows: staged in shared memory when they fit, else read in L2
    const T* wkn_g = static_cast<const T*>(p.w_knope) + static_cast<int64_t>(g) * nope * L;
    const T* wkr_g = static_cast<const T*>(p.w_krope) + static_cast<int64_t>(g) * R * L;
    const T* wv_g = static_cast<const T*>(p.w_v) + (static_cast<int64_t>(g) * D + d0) * L;
    T* wstage = reinterpret_cast<T*>(msm);
    const int wcount = p.stage_w ? L * (nope + R + dper) : 0;
    const T* wkn = p.stage_w ? wstage : wkn_g;
    const T* wkr = p.stage_w ? wstage + nope * L : wkr_g;
    const T* wv = p.stage_w ? wstage + (nope + R) * L : wv_g;   // rows d0 ..
    float* qn = reinterpret_cast<float*>(wstage + wcount);   // [rep][nope]
    float* qr = qn + rep * nope;           // [rep][R]
    float* qabs = qr + rep * R;            // [rep][L]
    float* ctx = qabs + rep * L;           // [rep][L] combined weighted latent
    float* part = ctx + rep * L;           // [rep][L] this CTA's weighted latent
    float* cnew = part + rep * L;          // [L]
    float* krn = cnew + L;                 // [R]
    float* tmp = krn + R;                  // [(rep+1)*R] rotated q_rope heads and k_rope
    float* wqn = tmp + (rep + 1) * R;      // [nope] q_nope norm weight
    float* wqr = wqn + nope;               // [R] q_rope norm weight
    float* wkv = wqr + R;                  // [L] latent norm weight
    float* cs = wkv + L;                   // [R] cos row
    float* sn = cs + R;                    // [R] sin row
    float* red = sn + R;                   // [2 * kAttnMaxRep]
    float* wred = red + 2 * kAttnMaxRep;   // [kAttnWarps][rep][L] weighted-sum reduction
    float* sc = wred + attn_red_floats(rep, L);   // [rep][cap]
    // what does not depend on the position first: the weight slices, this token's
    // projections, the norm weights
    const int width = p.heads * (nope + R) + L;
    const T* row = static_cast<const T*>(p.proj) + static_cast<int64_t>(b) * width;
    if (p.stage_w) {
        stage_rows<T>(wstage, wkn_g, nope * L);
        stage_rows<T>(wstage + nope * L, wkr_g, R * L);
        stage_rows<T>(wstage + (nope + R) * L, wv_g, (d1 - d0) * L);
    }
    for (int i = threadIdx.x; i < rep * nope; i += kAttnThreads)
        qn[i] = to_f32<T>(row[(g * rep) * nope + i]);
    for (int i = threadIdx.x; i < rep * R; i += kAttnThreads)
        qr[i] = to_f32<T>(row[p.heads * nope + (g * rep) * R + i]);
    for (int i = threadIdx.x; i < L; i += kAttnThreads) {
        cnew[i] = to_f32<T>(row[p.heads * (nope + R) + i]);
        wkv[i] = to_f32<T>(static_cast<const T*>(p.norm_kv)[i]);
    }
    for (int i = threadIdx.x; i < nope; i += kAttnThreads) wqn[i] = to_f32<T>(static_cast<const T*>(p.norm_q)[i]);
    for (int i = threadIdx.x; i < R; i += kAttnThreads) wqr[i] = to_f32<T>(static_cast<const T*>(p.norm_q2)[i]);
    T* out = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.heads + g * rep) * D;
    if (pos < 0 || pos >= p.max_len || pos >= p.table_len) {   // outside the cache: no access
        for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) out[i] = from_f32<T>(0.0f);
        return;   // every CTA of the cluster returns here (same pos)
    }
    const int n = pos + 1;
    T* cache_c = static_cast<T*>(p.cache_a) + static_cast<int64_t>(b) * p.max_len * L;
    T* cache_k = static_cast<T*>(p.cache_b) + static_cast<int64_t>(b) * p.max_len * p.kv_heads * R;
    // the rotary row (its first R columns), and this CTA's cache rows on their way
    for (int i = threadIdx.x; i < R; i += kAttnThreads) {
        cs[i] = to_f32<T>(static_cast<const T*>(p.cos)[static_cast<int64_t>(pos) * D + i]);
        sn[i] = to_f32<T>(static_cast<const T*>(p.sin)[static_cast<int64_t>(pos) * D + i]);
    }
    const int chunk = (n + splits - 1) / splits;
    const int t_lo = min(n, sidx * chunk), t_hi = min(n, t_lo + chunk), cnt = t_hi - t_lo;
    prefetch_rows<T>(cache_c, L, t_lo, t_hi, L * static_cast<int>(sizeof(T)));
    prefetch_rows<T>(cache_k + g * R, static_cast<int64_t>(p.kv_heads) * R, t_lo, t_hi,
                     R * static_cast<int>(sizeof(T)));
    if (p.stage_w) stage_rows_wait();
    __syncthreads();
    // per-head RMSNorms of q_nope and q_rope (each q_rope head then rotated by its
    // warp into tmp [rep][R]), RMSNorm of the latent
    for (int v = warp; v < 2 * rep + 1; v += kAttnWarps) {
        if (v < rep) {
            warp_rmsnorm_s<T>(qn + v * nope, nope, wqn, p.eps, lane);
        } else if (v < 2 * rep) {
            float* vec = qr + (v - rep) * R;
            warp_rmsnorm_s<T>(vec, R, wqr, p.eps, lane);
            for (int e = lane; e < R; e += 32) tmp[(v - rep) * R + e] = rope_value_s<T>(vec, e, R, cs, sn);
        } else {
            warp_rmsnorm_s<T>(cnew, L, wkv, p.eps, lane);
        }
    }
    __syncthreads();
    // k_rope of the new token: k_rope_proj(c) (rounded as the bf16 linear rounds); a
    // warp takes 4 output rows at once so their loads and warp sums interleave
    for (int r0 = warp * 4; r0 < R; r0 += kAttnWarps * 4) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int j = lane; j < L; j += 32) {
            const float c = cnew[j];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (r0 + q < R) acc[q] = fmaf(to_f32<T>(wkr[(r0 + q) * L + j]), c, acc[q]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = warp_sum(acc[q]);
        if (lane < 4 && r0 + lane < R) {
            float v = acc[0];
#pragma unroll
            for (int q = 1; q < 4; ++q) v = lane == q ? acc[q] : v;
            krn[r0 + lane] = round_to<T>(v);
        }
    }
    // q_abs = W_kn^T q_nope: the key up-projection folded into the query (an fp32
    // intermediate); eight terms loaded at a time into two interleaved sums
    for (int i = threadIdx.x; i < rep * L; i += kAttnThreads) {
        const int h = i / L, j = i % L;
        const float* q = qn + h * nope;
        float a0 = 0.0f, a1 = 0.0f;
        int d = 0;
        for (; d + 8 <= nope; d += 8) {
            float w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = to_f32<T>(wkn[(d + u) * L + j]);
#pragma unroll
            for (int u = 0; u < 8; u += 2) {
                a0 = fmaf(w[u], q[d + u], a0);
                a1 = fmaf(w[u + 1], q[d + u + 1], a1);
            }
        }
        for (; d < nope; ++d) a0 = fmaf(to_f32<T>(wkn[d * L + j]), q[d], a0);
        qabs[i] = a0 + a1;
    }
    __syncthreads();
    // RoPE at `pos` on the new k_rope: tmp + rep*R [R]
    for (int e = threadIdx.x; e < R; e += kAttnThreads) tmp[rep * R + e] = rope_value_s<T>(krn, e, R, cs, sn);
    __syncthreads();
    const float* qrot = tmp;
    const float* krot = tmp + rep * R;
    // append the new token to the cache (by CTA 0 of the cluster; the latent once, by group 0)
    if (sidx == 0) {
        if (g == 0)
            for (int j = threadIdx.x; j < L; j += kAttnThreads)
                cache_c[static_cast<int64_t>(pos) * L + j] = from_f32<T>(cnew[j]);
        for (int r = threadIdx.x; r < R; r += kAttnThreads)
            cache_k[(static_cast<int64_t>(pos) * p.kv_heads + g) * R + r] = from_f32<T>(krot[r]);
    }
    // this CTA's positions: latent against q_abs, rope key against q_rope
    split_scores<T, REP>(cache_c, L, qabs, L, cnew, cache_k + g * R, static_cast<int64_t>(p.kv_heads) * R, qrot, R,
                         krot, t_lo, t_hi, pos, p.scale, sc, cap, warp, lane);
    __syncthreads();
    split_softmax<T, REP>(cluster, sc, cap, cnt, red, warp, lane);
    __syncthreads();
    // this CTA's weighted latent sum_t p_t c_t per head
    weighted_rows<T, REP>(cache_c + static_cast<int64_t>(t_lo) * L, L, cnt, L, sc, cap, pos - t_lo, cnew, wred,
                          warp, lane, [&](int h, int c, float v) { part[h * L + c] = v; });
    cluster.sync();
    for (int i = threadIdx.x; i < rep * L; i += kAttnThreads) {
        float v = 0.0f;
        for (int r = 0; r < splits; ++r) v += cluster.map_shared_rank(part, r)[i];
        ctx[i] = v;
    }
    __syncthreads();
    // out = W_v ctx for this CTA's rows: the value up-projection applied once to the
    // weighted latent; a warp takes two rows at once so their sums interleave
    for (int d = d0 + 2 * warp; d < d1; d += 2 * kAttnWarps) {
        const bool two = d + 1 < d1;
        const T* wrow = wv + static_cast<int64_t>(d - d0) * L;
        float acc[2][REP];
#pragma unroll
        for (int h = 0; h < REP; ++h) acc[0][h] = acc[1][h] = 0.0f;
        for (int j = lane; j < L; j += 32) {
            const float w0 = to_f32<T>(wrow[j]);
            const float w1 = two ? to_f32<T>(wrow[L + j]) : 0.0f;
#pragma unroll
            for (int h = 0; h < REP; ++h) {
                const float c = ctx[h * L + j];
                acc[0][h] = fmaf(w0, c, acc[0][h]);
                acc[1][h] = fmaf(w1, c, acc[1][h]);
            }
        }
#pragma unroll
        for (int h = 0; h < REP; ++h) {
            acc[0][h] = warp_sum(acc[0][h]);
            acc[1][h] = warp_sum(acc[1][h]);
        }
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < REP; ++h) {
                out[h * D + d] = from_f32<T>(acc[0][h]);
                if (two) out[h * D + d + 1] = from_f32<T>(acc[1][h]);
            }
    }
    cluster.sync();   // no CTA leaves while a peer may still read its partial sums
}

// ---------------------------------------------------------------------------
// sliding-window decode (hybrid_attention.py:213-258 with a cache, S = 1)
// ---------------------------------------------------------------------------
template <typename T, int REP>
__global__ void __launch_bounds__(kAttnThreads, REP <= 4 ? 3 : 2) sw_decode_kernel(AttnParams p) {
    namespace cg = cooperative_groups;
    constexpr int rep = REP;
    extern __shared__ __align__(16) float ssm[];
    cg::cluster_group cluster = cg::this_cluster();
    pdl_wait();   // launched early behind the projection that writes proj (programmatic launch)
    const int pos = *p.pos;   // first: the rotary rows and the CTA's positions depend on it
    const int splits = p.splits;
    const int sidx = blockIdx.x % splits, g = blockIdx.x / splits, b = blockIdx.y;
    const int D = p.head_dim, W = p.window, cap = p.cap;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* q = ssm;                        // [rep][D]
    float* kn = q + rep * D;               // [D]
    float* vn = kn + D;                    // [D]
    float* tmp = vn + D;                   // [(rep+1)*D]
    float* wq = tmp + (rep + 1) * D;       // [D] q norm weight
    float* wk = wq + D;                    // [D] k norm weight
    float* cs = wk + D;                    // [D] cos row
    float* sn = cs + D;                    // [D] sin row
    float* part = sn + D;                  // [rep][D] this CTA's weighted values
    float* red = part + rep * D;           // [2 * kAttnMaxRep]
    float* wred = red + 2 * kAttnMaxRep;   // [kAttnWarps][rep][D] weighted-sum reduction
    float* sc = wred + attn_red_floats(rep, D);   // [rep][cap]
    // what does not depend on the position first: this token's projections, the norm weights
    const int width = (p.heads + 2 * p.kv_heads) * D;
    const T* row = static_cast<const T*>(p.proj) + static_cast<int64_t>(b) * width;
    for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) q[i] = to_f32<T>(row[(g * rep) * D + i]);
    for (int i = threadIdx.x; i < D; i += kAttnThreads) {
        kn[i] = to_f32<T>(row[(p.heads + g) * D + i]);
        vn[i] = to_f32<T>(row[(p.heads + p.kv_heads + g) * D + i]);
        wq[i] = to_f32<T>(static_cast<const T*>(p.norm_q)[i]);
        wk[i] = to_f32<T>(static_cast<const T*>(p.norm_q2)[i]);
    }
    T* out = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.heads + g * rep) * D;
    const int rpos = pos < W ? pos : W;    // the cache length before this token
    if (pos < 0 || rpos >= p.table_len) {
        for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) out[i] = from_f32<T>(0.0f);
        return;   // every CTA of the cluster returns here (same pos)
    }
    const int slot = pos % W;
    const int n = pos + 1 < W ? pos + 1 : W;
    T* kc = static_cast<T*>(p.cache_a) + static_cast<int64_t>(b) * W * p.kv_heads * D;
    T* vc = static_cast<T*>(p.cache_b) + static_cast<int64_t>(b) * W * p.kv_heads * D;
    const int64_t rs = static_cast<int64_t>(p.kv_heads) * D;
    // the rotary row, and this CTA's ring slots on their way while the query is formed
    for (int i = threadIdx.x; i < D; i += kAttnThreads) {
        cs[i] = to_f32<T>(static_cast<const T*>(p.cos)[static_cast<int64_t>(rpos) * D + i]);
        sn[i] = to_f32<T>(static_cast<const T*>(p.sin)[static_cast<int64_t>(rpos) * D + i]);
    }
    const int chunk = (n + splits - 1) / splits;
    const int t_lo = min(n, sidx * chunk), t_hi = min(n, t_lo + chunk), cnt = t_hi - t_lo;
    prefetch_rows<T>(kc + g * D, rs, t_lo, t_hi, D * static_cast<int>(sizeof(T)));
    prefetch_rows<T>(vc + g * D, rs, t_lo, t_hi, D * static_cast<int>(sizeof(T)));
    __syncthreads();
    // per warp: a head's RMSNorm, then its rotation into tmp [rep][D] (queries) and
    // tmp + rep*D [D] (the new key), with no block barrier between the two
    for (int v = warp; v < rep + 1; v += kAttnWarps) {
        float* vec = v < rep ? q + v * D : kn;
        warp_rmsnorm_s<T>(vec, D, v < rep ? wq : wk, p.eps, lane);
        for (int e = lane; e < D; e += 32) tmp[v * D + e] = rope_value_s<T>(vec, e, D, cs, sn);
    }
    __syncthreads();
    const float* qrot = tmp;
    const float* krot = tmp + rep * D;
    if (sidx == 0)
        for (int i = threadIdx.x; i < D; i += kAttnThreads) {
            kc[(static_cast<int64_t>(slot) * p.kv_heads + g) * D + i] = from_f32<T>(krot[i]);
            vc[(static_cast<int64_t>(slot) * p.kv_heads + g) * D + i] = from_f32<T>(vn[i]);
        }
    // scores of this CTA's ring slots; the new token's slot comes from shared memory
    split_scores<T, REP>(kc + g * D, rs, qrot, D, krot, kc, rs, qrot, 0, krot, t_lo, t_hi, slot, p.scale, sc,
                         cap, warp, lane);
    __syncthreads();
    split_softmax<T, REP>(cluster, sc, cap, cnt, red, warp, lane);
    __syncthreads();
    weighted_rows<T, REP>(vc + static_cast<int64_t>(t_lo) * rs + g * D, rs, cnt, D, sc, cap, slot - t_lo, vn,
                          wred, warp, lane, [&](int h, int c, float v) { part[h * D + c] = v; });
    cluster.sync();
    // this CTA's share of the outputs: the partial sums added in CTA order
    const int per = (rep * D + splits - 1) / splits;
    const int i1 = min(rep * D, (sidx + 1) * per);
    for (int i = sidx * per + threadIdx.x; i < i1; i += kAttnThreads) {
        float v = 0.0f;
        for (int r = 0; r < splits; ++r) v += cluster.map_shared_rank(part, r)[i];
        out[i] = from_f32<T>(v);
    }
    cluster.sync();   // no CTA leaves while a peer may still read its partial sums
}

}  // namespace chronos
