// attention.cuh — one-token decode of the hybrid attention
// (chronos/model/hybrid_attention.py) and the residual add + RMSNorm of a block.
//
// Both decode kernels run one block per (kv head g, batch row b), 256 threads,
// and do, in one launch: the per-head RMSNorms of the new token's projections,
// RoPE at its position, the cache append, the scores of the group's n_rep
// query heads against every cached token, the softmax and the weighted sum.
// Arithmetic is fp32; values are rounded to the layer type where the
// reference's torch code holds a tensor in that type (norm and RoPE outputs,
// the new cache entries, the softmax probabilities, the output), so a bf16
// layer rounds where the reference's bf16 run rounds.
#pragma once

#include "common.cuh"

namespace chronos {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxRep = 8;

struct AttnParams {
    int heads, kv_heads, rep, head_dim, rope_dim, nope, latent, window, max_len, table_len;
    int stage_w;   // MLA: 1 = the group's weight slices are staged in shared memory
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
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

// Softmax over each head's scores (one warp per head), probabilities rounded to T.
template <typename T>
__device__ __forceinline__ void heads_softmax(float* sc, int rep, int stride, int n, int warp, int lane) {
    for (int h = warp; h < rep; h += kAttnWarps) {
        float* s = sc + h * stride;
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, s[t]);
        m = warp_max(m);
        float sum = 0.0f;
        for (int t = lane; t < n; t += 32) {
            const float e = __expf(s[t] - m);
            s[t] = e;
            sum += e;
        }
        const float inv = 1.0f / warp_sum(sum);
        __syncwarp();
        for (int t = lane; t < n; t += 32) s[t] = round_to<T>(s[t] * inv);
    }
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
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const int64_t base = r * p.width;
        float ss = 0.0f;
        for (int c = threadIdx.x; c < p.width; c += kAttnThreads) {
            float v = to_f32<T>(x[base + c]);
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

// 8 consecutive values as fp32: one 16-byte load for 2-byte types, two for fp32
// (the caller guarantees 16-byte alignment).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

// Copy `count` elements (a multiple of 8) into shared memory with 16-byte vectors.
template <typename T>
__device__ __forceinline__ void stage_rows(T* dst, const T* src, int count) {
    constexpr int EPV = 16 / static_cast<int>(sizeof(T));
    for (int i = threadIdx.x; i < count / EPV; i += kAttnThreads)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

// Weighted sum of `n` cached rows for every head of the group:
// out[h][c] = sum_t p[h][t] * row_t[c] for the `width` columns of a row, rows
// `stride` elements apart; the row at `fresh_t` comes from shared memory
// (`fresh`, fp32) instead.  Warps take 8-column groups, lanes take every 32nd
// row (many independent 16-byte loads in flight), and a warp reduction
// gathers the lanes; `emit(h, c, value)` receives each result.
template <typename T, typename Emit>
__device__ __forceinline__ void weighted_rows(const T* rows, int64_t stride, int n, int width, const float* p,
                                              int p_stride, int rep, int fresh_t, const float* fresh, int warp,
                                              int lane, Emit&& emit) {
    for (int cg = warp; cg < width / 8; cg += kAttnWarps) {
        float acc[kAttnMaxRep][8];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[h][u] = 0.0f;
#pragma unroll 4
        for (int t = lane; t < n; t += 32) {
            float v[8];
            if (t == fresh_t) {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = fresh[cg * 8 + u];
            } else {
                load8<T>(rows + static_cast<int64_t>(t) * stride + cg * 8, v);
            }
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h) {
                if (h < rep) {
                    const float ph = p[h * p_stride + t];
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[h][u] = fmaf(ph, v[u], acc[h][u]);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) {
            if (h < rep) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float r = warp_sum(acc[h][u]);
                    if (lane == 0) emit(h, cg * 8 + u, r);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// MLA decode (hybrid_attention.py:116-179 with a cache, S = 1)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) mla_decode_kernel(AttnParams p) {
    extern __shared__ __align__(16) float msm[];
    const int g = blockIdx.x, b = blockIdx.y;
    const int rep = p.rep, nope = p.nope, R = p.rope_dim, L = p.latent, D = p.head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the group's slices of k_nope_proj [nope, L], k_rope_proj [R, L], v_proj [D, L]:
    // staged in shared memory when they fit, else read where they are (L2)
    const T* wkn_g = static_cast<const T*>(p.w_knope) + static_cast<int64_t>(g) * nope * L;
    const T* wkr_g = static_cast<const T*>(p.w_krope) + static_cast<int64_t>(g) * R * L;
    const T* wv_g = static_cast<const T*>(p.w_v) + static_cast<int64_t>(g) * D * L;
    T* wstage = reinterpret_cast<T*>(msm);
    const int wcount = p.stage_w ? L * (nope + R + D) : 0;
    const T* wkn = p.stage_w ? wstage : wkn_g;
    const T* wkr = p.stage_w ? wstage + nope * L : wkr_g;
    const T* wv = p.stage_w ? wstage + (nope + R) * L : wv_g;
    float* qn = reinterpret_cast<float*>(wstage + wcount);   // [rep][nope]
    float* qr = qn + rep * nope;           // [rep][R]
    float* qabs = qr + rep * R;            // [rep][L]
    float* ctx = qabs + rep * L;           // [rep][L]
    float* cnew = ctx + rep * L;           // [L]
    float* krn = cnew + L;                 // [R]
    float* tmp = krn + R;                  // [(rep+1)*R] rotated q_rope heads and k_rope
    float* sc = tmp + (rep + 1) * R;       // [rep][max_len]
    const int pos = *p.pos;
    T* out = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.heads + g * rep) * D;
    if (pos < 0 || pos >= p.max_len || pos >= p.table_len) {   // outside the cache: no access
        for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) out[i] = from_f32<T>(0.0f);
        return;
    }
    const int n = pos + 1;
    const int width = p.heads * (nope + R) + L;
    const T* row = static_cast<const T*>(p.proj) + static_cast<int64_t>(b) * width;
    if (p.stage_w) {
        stage_rows<T>(wstage, wkn_g, nope * L);
        stage_rows<T>(wstage + nope * L, wkr_g, R * L);
        stage_rows<T>(wstage + (nope + R) * L, wv_g, D * L);
    }
    for (int i = threadIdx.x; i < rep * nope; i += kAttnThreads)
        qn[i] = to_f32<T>(row[(g * rep) * nope + i]);
    for (int i = threadIdx.x; i < rep * R; i += kAttnThreads)
        qr[i] = to_f32<T>(row[p.heads * nope + (g * rep) * R + i]);
    for (int i = threadIdx.x; i < L; i += kAttnThreads) cnew[i] = to_f32<T>(row[p.heads * (nope + R) + i]);
    __syncthreads();
    // per-head RMSNorms of q_nope and q_rope, RMSNorm of the latent
    for (int v = warp; v < 2 * rep + 1; v += kAttnWarps) {
        if (v < rep) warp_rmsnorm<T>(qn + v * nope, nope, static_cast<const T*>(p.norm_q), p.eps, lane);
        else if (v < 2 * rep) warp_rmsnorm<T>(qr + (v - rep) * R, R, static_cast<const T*>(p.norm_q2), p.eps, lane);
        else warp_rmsnorm<T>(cnew, L, static_cast<const T*>(p.norm_kv), p.eps, lane);
    }
    __syncthreads();
    // k_rope of the new token: k_rope_proj(c) (rounded as the bf16 linear rounds)
    for (int r = threadIdx.x; r < R; r += kAttnThreads) {
        float acc = 0.0f;
        for (int j = 0; j < L; ++j) acc = fmaf(to_f32<T>(wkr[r * L + j]), cnew[j], acc);
        krn[r] = round_to<T>(acc);
    }
    // q_abs = W_kn^T q_nope: the key up-projection folded into the query
    for (int i = threadIdx.x; i < rep * L; i += kAttnThreads) {
        const int h = i / L, j = i % L;
        const float* q = qn + h * nope;
        float acc = 0.0f;
        for (int d = 0; d < nope; ++d) acc = fmaf(to_f32<T>(wkn[d * L + j]), q[d], acc);
        qabs[i] = acc;
    }
    __syncthreads();
    // RoPE at `pos` on q_rope (every head) and on the new k_rope
    const T* crow = static_cast<const T*>(p.cos) + static_cast<int64_t>(pos) * D;
    const T* srow = static_cast<const T*>(p.sin) + static_cast<int64_t>(pos) * D;
    for (int i = threadIdx.x; i < (rep + 1) * R; i += kAttnThreads) {
        const int h = i / R, e = i % R;
        tmp[i] = rope_value<T>(h < rep ? qr + h * R : krn, e, R, crow, srow);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < (rep + 1) * R; i += kAttnThreads) {
        const int h = i / R, e = i % R;
        (h < rep ? qr + h * R : krn)[e] = tmp[i];
    }
    __syncthreads();
    // append the new token to the cache (the latent once, by the group-0 block)
    T* cache_c = static_cast<T*>(p.cache_a) + static_cast<int64_t>(b) * p.max_len * L;
    T* cache_k = static_cast<T*>(p.cache_b) + static_cast<int64_t>(b) * p.max_len * p.kv_heads * R;
    if (g == 0)
        for (int j = threadIdx.x; j < L; j += kAttnThreads)
            cache_c[static_cast<int64_t>(pos) * L + j] = from_f32<T>(cnew[j]);
    for (int r = threadIdx.x; r < R; r += kAttnThreads)
        cache_k[(static_cast<int64_t>(pos) * p.kv_heads + g) * R + r] = from_f32<T>(krn[r]);
    // scores: one cached token per thread (its latent and rope key as 16-byte loads),
    // every head of the group
    for (int t = threadIdx.x; t < n; t += kAttnThreads) {
        float acc[kAttnMaxRep];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) acc[h] = 0.0f;
        const T* ct = cache_c + static_cast<int64_t>(t) * L;
#pragma unroll 4
        for (int j8 = 0; j8 < L; j8 += 8) {
            float c[8];
            if (t == pos) {
#pragma unroll
                for (int u = 0; u < 8; ++u) c[u] = cnew[j8 + u];
            } else {
                load8<T>(ct + j8, c);
            }
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep)
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[h] = fmaf(qabs[h * L + j8 + u], c[u], acc[h]);
        }
        const T* kt = cache_k + (static_cast<int64_t>(t) * p.kv_heads + g) * R;
#pragma unroll 4
        for (int r8 = 0; r8 < R; r8 += 8) {
            float k[8];
            if (t == pos) {
#pragma unroll
                for (int u = 0; u < 8; ++u) k[u] = krn[r8 + u];
            } else {
                load8<T>(kt + r8, k);
            }
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep)
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[h] = fmaf(qr[h * R + r8 + u], k[u], acc[h]);
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
            if (h < rep) sc[h * p.max_len + t] = acc[h] * p.scale;
    }
    __syncthreads();
    heads_softmax<T>(sc, rep, p.max_len, n, warp, lane);
    __syncthreads();
    // ctx = sum_t p_t c_t per head
    weighted_rows<T>(cache_c, L, n, L, sc, p.max_len, rep, pos, cnew, warp, lane,
                     [&](int h, int c, float v) { ctx[h * L + c] = v; });
    __syncthreads();
    // out = W_v ctx: the value up-projection applied once to the weighted latent
    for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) {
        const int h = i / D, d = i % D;
        const float* c = ctx + h * L;
        float acc = 0.0f;
        for (int j = 0; j < L; ++j) acc = fmaf(to_f32<T>(wv[d * L + j]), c[j], acc);
        out[i] = from_f32<T>(acc);
    }
}

// ---------------------------------------------------------------------------
// sliding-window decode (hybrid_attention.py:213-258 with a cache, S = 1)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) sw_decode_kernel(AttnParams p) {
    extern __shared__ __align__(16) float ssm[];
    const int g = blockIdx.x, b = blockIdx.y;
    const int rep = p.rep, D = p.head_dim, W = p.window;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* q = ssm;                        // [rep][D]
    float* kn = q + rep * D;               // [D]
    float* vn = kn + D;                    // [D]
    float* tmp = vn + D;                   // [(rep+1)*D]
    float* sc = tmp + (rep + 1) * D;       // [rep][W]
    const int pos = *p.pos;
    T* out = static_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.heads + g * rep) * D;
    const int rpos = pos < W ? pos : W;    // the cache length before this token
    if (pos < 0 || rpos >= p.table_len) {
        for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) out[i] = from_f32<T>(0.0f);
        return;
    }
    const int slot = pos % W;
    const int n = pos + 1 < W ? pos + 1 : W;
    const int width = (p.heads + 2 * p.kv_heads) * D;
    const T* row = static_cast<const T*>(p.proj) + static_cast<int64_t>(b) * width;
    for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) q[i] = to_f32<T>(row[(g * rep) * D + i]);
    for (int i = threadIdx.x; i < D; i += kAttnThreads) {
        kn[i] = to_f32<T>(row[(p.heads + g) * D + i]);
        vn[i] = to_f32<T>(row[(p.heads + p.kv_heads + g) * D + i]);
    }
    __syncthreads();
    for (int v = warp; v < rep + 1; v += kAttnWarps) {
        if (v < rep) warp_rmsnorm<T>(q + v * D, D, static_cast<const T*>(p.norm_q), p.eps, lane);
        else warp_rmsnorm<T>(kn, D, static_cast<const T*>(p.norm_q2), p.eps, lane);
    }
    __syncthreads();
    const T* crow = static_cast<const T*>(p.cos) + static_cast<int64_t>(rpos) * D;
    const T* srow = static_cast<const T*>(p.sin) + static_cast<int64_t>(rpos) * D;
    for (int i = threadIdx.x; i < (rep + 1) * D; i += kAttnThreads) {
        const int h = i / D, e = i % D;
        tmp[i] = rope_value<T>(h < rep ? q + h * D : kn, e, D, crow, srow);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < (rep + 1) * D; i += kAttnThreads) {
        const int h = i / D, e = i % D;
        (h < rep ? q + h * D : kn)[e] = tmp[i];
    }
    __syncthreads();
    T* kc = static_cast<T*>(p.cache_a) + static_cast<int64_t>(b) * W * p.kv_heads * D;
    T* vc = static_cast<T*>(p.cache_b) + static_cast<int64_t>(b) * W * p.kv_heads * D;
    for (int i = threadIdx.x; i < D; i += kAttnThreads) {
        kc[(static_cast<int64_t>(slot) * p.kv_heads + g) * D + i] = from_f32<T>(kn[i]);
        vc[(static_cast<int64_t>(slot) * p.kv_heads + g) * D + i] = from_f32<T>(vn[i]);
    }
    // scores: one ring slot per thread, its key as 16-byte loads
    for (int t = threadIdx.x; t < n; t += kAttnThreads) {
        float acc[kAttnMaxRep];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) acc[h] = 0.0f;
        const T* kt = kc + (static_cast<int64_t>(t) * p.kv_heads + g) * D;
#pragma unroll 4
        for (int d8 = 0; d8 < D; d8 += 8) {
            float k[8];
            if (t == slot) {
#pragma unroll
                for (int u = 0; u < 8; ++u) k[u] = kn[d8 + u];
            } else {
                load8<T>(kt + d8, k);
            }
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep)
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[h] = fmaf(q[h * D + d8 + u], k[u], acc[h]);
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
            if (h < rep) sc[h * W + t] = acc[h] * p.scale;
    }
    __syncthreads();
    heads_softmax<T>(sc, rep, W, n, warp, lane);
    __syncthreads();
    weighted_rows<T>(vc + static_cast<int64_t>(g) * D, static_cast<int64_t>(p.kv_heads) * D, n, D, sc, W, rep,
                     slot, vn, warp, lane, [&](int h, int c, float v) { out[h * D + c] = from_f32<T>(v); });
}

}  // namespace chronos
