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

// ---------------------------------------------------------------------------
// MLA decode (hybrid_attention.py:116-179 with a cache, S = 1)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kAttnThreads) mla_decode_kernel(AttnParams p) {
    extern __shared__ float msm[];
    const int g = blockIdx.x, b = blockIdx.y;
    const int rep = p.rep, nope = p.nope, R = p.rope_dim, L = p.latent, D = p.head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* qn = msm;                       // [rep][nope]
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
    const T* wkr = static_cast<const T*>(p.w_krope) + static_cast<int64_t>(g) * R * L;
    for (int r = threadIdx.x; r < R; r += kAttnThreads) {
        float acc = 0.0f;
        for (int j = 0; j < L; ++j) acc = fmaf(to_f32<T>(wkr[r * L + j]), cnew[j], acc);
        krn[r] = round_to<T>(acc);
    }
    // q_abs = W_kn^T q_nope: the key up-projection folded into the query
    const T* wkn = static_cast<const T*>(p.w_knope) + static_cast<int64_t>(g) * nope * L;
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
    // scores: one token per thread, every head of the group
    for (int t = threadIdx.x; t < n; t += kAttnThreads) {
        float acc[kAttnMaxRep];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) acc[h] = 0.0f;
        const T* ct = cache_c + static_cast<int64_t>(t) * L;
        for (int j = 0; j < L; ++j) {
            const float c = t == pos ? cnew[j] : to_f32<T>(ct[j]);
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep) acc[h] = fmaf(qabs[h * L + j], c, acc[h]);
        }
        const T* kt = cache_k + (static_cast<int64_t>(t) * p.kv_heads + g) * R;
        for (int r = 0; r < R; ++r) {
            const float k = t == pos ? krn[r] : to_f32<T>(kt[r]);
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep) acc[h] = fmaf(qr[h * R + r], k, acc[h]);
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
            if (h < rep) sc[h * p.max_len + t] = acc[h] * p.scale;
    }
    __syncthreads();
    heads_softmax<T>(sc, rep, p.max_len, n, warp, lane);
    __syncthreads();
    // ctx = sum_t p_t c_t per head
    for (int i = threadIdx.x; i < rep * L; i += kAttnThreads) {
        const int h = i / L, j = i % L;
        const float* ph = sc + h * p.max_len;
        float acc = 0.0f;
        for (int t = 0; t < pos; ++t) acc = fmaf(ph[t], to_f32<T>(cache_c[static_cast<int64_t>(t) * L + j]), acc);
        ctx[i] = fmaf(ph[pos], cnew[j], acc);
    }
    __syncthreads();
    // out = W_v ctx: the value up-projection applied once to the weighted latent
    const T* wv = static_cast<const T*>(p.w_v) + static_cast<int64_t>(g) * D * L;
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
    extern __shared__ float ssm[];
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
    for (int t = threadIdx.x; t < n; t += kAttnThreads) {
        float acc[kAttnMaxRep];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) acc[h] = 0.0f;
        const T* kt = kc + (static_cast<int64_t>(t) * p.kv_heads + g) * D;
        for (int d = 0; d < D; ++d) {
            const float k = t == slot ? kn[d] : to_f32<T>(kt[d]);
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h)
                if (h < rep) acc[h] = fmaf(q[h * D + d], k, acc[h]);
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
            if (h < rep) sc[h * W + t] = acc[h] * p.scale;
    }
    __syncthreads();
    heads_softmax<T>(sc, rep, W, n, warp, lane);
    __syncthreads();
    for (int i = threadIdx.x; i < rep * D; i += kAttnThreads) {
        const int h = i / D, d = i % D;
        const float* ph = sc + h * W;
        float acc = 0.0f;
        for (int t = 0; t < n; ++t) {
            const float v = t == slot ? vn[d] : to_f32<T>(vc[(static_cast<int64_t>(t) * p.kv_heads + g) * D + d]);
            acc = fmaf(ph[t], v, acc);
        }
        out[i] = from_f32<T>(acc);
    }
}

}  // namespace chronos
