// router.cuh — router GEMM + softmax + top-k + blend coefficients.
//
// Restates chronos/model/moe_chronos.py:112-128 (gate Linear, softmax, topk,
// norm_topk_prob renormalisation) under the bit-exact routing contract of
// include/chronos_moe.h: a logit is the in-order fp32 sum of 128-element chunk
// partials, each partial one thread's fmaf chain over its chunk in increasing
// h, so the ranking is identical on every run and equal to the CPU oracle's.
//
// Two logit kernels produce the same bits, both writing the chunk partials
// chunk-major, partials[c][t][e] ([C, N, E], coalesced along experts):
//   route_partials_kernel  small batches: one thread per (expert, chunk, group
//                          of 8 tokens) (parallel over chunks, so a decode
//                          token's 64 logits are not 2048-long serial chains);
//   route_tiled_kernel     large batches: 128-token x 64-expert register-tiled
//                          SIMT GEMM, each block over 4 chunks (512 h) of K
//                          (the K split gives the grid enough blocks to fill
//                          every SM; the in-order fold stays in the select).
// route_select_kernel (one warp per token) then sums the partials in chunk
// order, applies the bias, softmax and top-k, and writes the per-token blend
// coefficient of the shared experts (1 + sum_k w*(1-a)) / S_h
// (moe_chronos.py:255-268), the within-expert position of every available
// selection (for the permutation) and zeroes the token's fp32 accumulator row.
#pragma once

#include "common.cuh"

namespace chronos {

constexpr int kRouteChunk = 128;       // h per partial (the contract's chunk)
constexpr int kRouteGroup = 8;         // tokens per thread in the partials kernel
constexpr int kRouteSmallMax = 256;    // largest batch routed by the partials kernel
constexpr int kRouteTile = 64;         // experts per tiled block
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 256;

struct RouteParams {
    const void* x;
    const void* w;
    const float* bias;
    const float* avail;
    int avail_mask;  // 1: a_e = (avail[e] > 0)
    const int32_t* slot_of_expert;
    int64_t n;
    int h, e, k, num_shared, norm_topk, prerouted;
    int nchunks;          // chunk partials per logit
    float* partials;      // [nchunks, N, E]
    void* probs;          // [N, E] T or null
    int32_t* topk_idx;    // [N, k]
    float* topk_w;        // [N, k]
    int32_t* counts_all;  // [E] or null
    float* mass_all;      // [E] or null
    int32_t* grp_count;   // [E + 1] routed-group sizes (selections with a > 0), then a ticket counter
    int32_t* pos;         // [N, k] position within the expert group, -1 when a == 0
    float* sel_coef;      // [N, k] w * a
    float* shared_coef;   // [N] (1 + sum w (1 - a)) / S_h
    float* y_acc;         // [N, H] fp32, zeroed here (or null)
    void* y_direct;       // k = 1, no shared experts: the output [N, H]; rows of tokens
                          // whose one selection is unavailable are zeroed here (or null)
};

// The logit kernels run first in a call: their first block zeroes the
// per-call counters (group sizes and the optional per-expert statistics) that
// the select kernel, launched after them, accumulates into.
__device__ __forceinline__ void zero_route_counters(const RouteParams& p) {
    if (threadIdx.x == 0) p.grp_count[p.e] = 0;  // ticket of the decode select + plan kernel
    for (int i = threadIdx.x; i < p.e; i += blockDim.x) {
        p.grp_count[i] = 0;
        if (p.counts_all) p.counts_all[i] = 0;
        if (p.mass_all) p.mass_all[i] = 0.0f;
    }
}

inline int route_chunks(int h) { return (h + kRouteChunk - 1) / kRouteChunk; }

// 4 consecutive elements as fp32 (8-byte loads for 16-bit types, 16 bytes for fp32).
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}

// ---------------------------------------------------------------------------
// small batches: chunk partials
// ---------------------------------------------------------------------------
constexpr int kPartialThreads = 64;  // experts per block (one thread each)

// Block (token group g, chunk c, expert block eb): the group's x chunk
// [8 tokens x 128 h] is staged in shared memory as fp32, and the block's
// weight chunk [64 experts x 128 h] is copied in with coalesced 16-byte loads
// (rows padded by 16 bytes so each thread's row reads are conflict-free).
// Then every thread runs its expert's 8 chunk chains.
template <typename T>
__global__ void __launch_bounds__(kPartialThreads) route_partials_kernel(RouteParams p) {
    constexpr int ROW = kRouteChunk * static_cast<int>(sizeof(T)) + 16;  // padded row bytes
    constexpr int V16 = kRouteChunk * static_cast<int>(sizeof(T)) / 16;  // 16-byte vectors per row
    constexpr int EPV = 16 / static_cast<int>(sizeof(T));                // elements per vector
    __shared__ __align__(16) float xs[kRouteGroup][kRouteChunk];
    __shared__ __align__(16) uint8_t ws[kPartialThreads * ROW];
    pdl_trigger();
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) zero_route_counters(p);
    const int E = p.e, H = p.h;
    const int c = blockIdx.y;
    const int e0 = blockIdx.z * kPartialThreads;
    const int e = e0 + threadIdx.x;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRouteGroup;
    const int64_t left = p.n - t0;
    const int nt = left < kRouteGroup ? static_cast<int>(left) : kRouteGroup;
    const int h0 = c * kRouteChunk;
    const int len = min(kRouteChunk, H - h0);  // multiple of 4
    const T* x = static_cast<const T*>(p.x);
    const T* w = static_cast<const T*>(p.w);
    // weights: row r = expert e0 + r, vector v = elements [v*EPV, v*EPV + EPV) of the
    // chunk; every thread issues all of its V16 loads before any store (one latency)
    const bool vec_ok = (H % EPV) == 0;  // 16-byte aligned rows
    {
        uint4 val[V16];
#pragma unroll
        for (int it = 0; it < V16; ++it) {
            const int i = it * kPartialThreads + threadIdx.x;
            const int r = i / V16, v = i % V16;
            const int er = e0 + r;
            val[it] = make_uint4(0u, 0u, 0u, 0u);
            if (er < E) {
                const T* src = w + static_cast<int64_t>(er) * H + h0 + v * EPV;
                if (vec_ok && v * EPV + EPV <= len) {
                    val[it] = *reinterpret_cast<const uint4*>(src);
                } else {
                    T tmp[EPV];
#pragma unroll
                    for (int u = 0; u < EPV; ++u) tmp[u] = (v * EPV + u < len) ? src[u] : from_f32<T>(0.0f);
                    val[it] = *reinterpret_cast<const uint4*>(tmp);
                }
            }
        }
#pragma unroll
        for (int it = 0; it < V16; ++it) {
            const int i = it * kPartialThreads + threadIdx.x;
            *reinterpret_cast<uint4*>(ws + (i / V16) * ROW + (i % V16) * 16) = val[it];
        }
    }
    // x chunk of the token group, as fp32 (loads first, then stores)
    {
        constexpr int XV = kRouteGroup * (kRouteChunk / 4) / kPartialThreads;
        float4 xv[XV];
#pragma unroll
        for (int it = 0; it < XV; ++it) {
            const int i = it * kPartialThreads + threadIdx.x;
            const int r = i / (kRouteChunk / 4), q4 = (i % (kRouteChunk / 4)) * 4;
            xv[it] = (r < nt && q4 < len) ? load4<T>(x + (t0 + r) * H + h0 + q4)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int it = 0; it < XV; ++it) {
            const int i = it * kPartialThreads + threadIdx.x;
            *reinterpret_cast<float4*>(&xs[i / (kRouteChunk / 4)][(i % (kRouteChunk / 4)) * 4]) = xv[it];
        }
    }
    __syncthreads();
    if (e >= E) return;
    float acc[kRouteGroup];
#pragma unroll
    for (int i = 0; i < kRouteGroup; ++i) acc[i] = 0.0f;
    // chains over h in increasing order; elements past `len` are zero pairs and
    // leave the sums unchanged
    const uint8_t* wrow = ws + threadIdx.x * ROW;
#pragma unroll 4
    for (int q = 0; q < kRouteChunk; q += 4) {
        const float4 b = load4<T>(reinterpret_cast<const T*>(wrow) + q);
#pragma unroll
        for (int i = 0; i < kRouteGroup; ++i) {
            const float4 a = *reinterpret_cast<const float4*>(&xs[i][q]);
            acc[i] = fmaf(a.x, b.x, acc[i]);
            acc[i] = fmaf(a.y, b.y, acc[i]);
            acc[i] = fmaf(a.z, b.z, acc[i]);
            acc[i] = fmaf(a.w, b.w, acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < kRouteGroup; ++i)
        if (i < nt) p.partials[(static_cast<int64_t>(c) * p.n + t0 + i) * E + e] = acc[i];
}

// ---------------------------------------------------------------------------
// large batches: register-tiled SIMT GEMM, chunk partials folded in order
// ---------------------------------------------------------------------------
constexpr int kTiledThreads = 256;
constexpr int kTiledTokens = 128;  // tokens per block (8 per thread)
constexpr int kTiledChunks = 4;    // chunks of K per block (blockIdx.z)
// h per shared-memory stage: 32 for 2-byte inputs (a stage computes for about
// as long as a DRAM round trip takes, so the one-stage-ahead register prefetch
// is hidden), 16 for fp32 inputs (their prefetch registers are twice as many)
template <typename T>
__host__ __device__ constexpr int tiled_k() { return sizeof(T) == 2 ? 32 : 16; }
template <typename T>
__host__ __device__ constexpr int tiled_smem_bytes() {
    return 2 * (kTiledTokens + kRouteTile) * (tiled_k<T>() + 4) * 4;  // double-buffered fp32 stages
}

// 4 consecutive inputs as loaded from global memory (converted when staged)
template <typename T>
struct Raw4 {
    uint2 v;
};
template <>
struct Raw4<float> {
    float4 v;
};
template <typename T>
__device__ __forceinline__ Raw4<T> load_raw4(const T* p) {
    Raw4<T> r;
    r.v = *reinterpret_cast<const decltype(r.v)*>(p);
    return r;
}
template <typename T>
__device__ __forceinline__ float4 raw4_to_f32(const Raw4<T>& r) {
    return load4<T>(reinterpret_cast<const T*>(&r.v));
}

// Block = 128 tokens x 64 experts x 4 chunks of K; thread = 8 tokens x 4
// experts (tokens tg + 16 i, experts eg + 16 j), one fmaf chain per (token, expert, chunk) in
// increasing h; at each chunk end the partial is written and the chain restarts.
// Stages of K_T h are double-buffered in shared memory (fp32); the next stage's
// inputs are held in registers as loaded while the current one is computed.
template <typename T>
__global__ void __launch_bounds__(kTiledThreads, 2) route_tiled_kernel(RouteParams p) {
    constexpr int KT_H = tiled_k<T>();
    constexpr int PAD = KT_H + 4;
    constexpr int EX = KT_H / 2;  // x elements per thread per stage (2 threads per row)
    constexpr int EW = KT_H / 4;  // w elements per thread per stage (4 threads per row)
    extern __shared__ __align__(16) float route_smem[];
    float* xs = route_smem;                        // [2][kTiledTokens][PAD]
    float* ws = route_smem + 2 * kTiledTokens * PAD;  // [2][kRouteTile][PAD]
    pdl_trigger();
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) zero_route_counters(p);
    const int tid = threadIdx.x;
    // tokens tg + 16 i: a warp's two token groups read adjacent shared-memory rows
    // (different banks), not rows 8 apart (the same banks at this row pitch)
    const int tg = tid >> 4;
    const int eg = tid & 15;  // experts eg + 16 j
    const int H = p.h, E = p.e;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTiledTokens;
    const int e0 = blockIdx.y * kRouteTile;
    const T* x = static_cast<const T*>(p.x);
    const T* w = static_cast<const T*>(p.w);
    // loaders: x row xr, EX consecutive h at xk; w row wr, EW consecutive h at wk
    const int xr = tid >> 1, xk = (tid & 1) * EX;
    const int wr = tid >> 2, wk = (tid & 3) * EW;
    const bool xrow_ok = t0 + xr < p.n;
    const bool wrow_ok = e0 + wr < E;
    const T* xrow = x + (t0 + xr) * H;
    const T* wrow = w + static_cast<int64_t>(e0 + wr) * H;
    Raw4<T> xraw[EX / 4], wraw[EW / 4];
    auto gload = [&](int kt) {
        const int h = kt * KT_H;
        Raw4<T> z;
        z.v = {};
#pragma unroll
        for (int q = 0; q < EX / 4; ++q)  // H % 4 == 0: each group of 4 is in or out as a whole
            xraw[q] = (xrow_ok && h + xk + 4 * q < H) ? load_raw4<T>(xrow + h + xk + 4 * q) : z;
#pragma unroll
        for (int q = 0; q < EW / 4; ++q)
            wraw[q] = (wrow_ok && h + wk + 4 * q < H) ? load_raw4<T>(wrow + h + wk + 4 * q) : z;
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int q = 0; q < EX / 4; ++q)
            *reinterpret_cast<float4*>(&xs[(buf * kTiledTokens + xr) * PAD + xk + 4 * q]) = raw4_to_f32<T>(xraw[q]);
#pragma unroll
        for (int q = 0; q < EW / 4; ++q)
            *reinterpret_cast<float4*>(&ws[(buf * kRouteTile + wr) * PAD + wk + 4 * q]) = raw4_to_f32<T>(wraw[q]);
    };
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    const int KT = (H + KT_H - 1) / KT_H;
    constexpr int kTilesPerChunk = kRouteChunk / KT_H;
    const int kt_begin = blockIdx.z * kTiledChunks * kTilesPerChunk;
    const int kt_end = min(KT, kt_begin + kTiledChunks * kTilesPerChunk);
    gload(kt_begin);
    sstore(0);
    __syncthreads();
    for (int kt = kt_begin; kt < kt_end; ++kt) {
        const int buf = (kt - kt_begin) & 1;
        if (kt + 1 < kt_end) gload(kt + 1);
        const float* xb = xs + (buf * kTiledTokens + tg) * PAD;
        const float* wb = ws + (buf * kRouteTile + eg) * PAD;
#pragma unroll
        for (int kk = 0; kk < KT_H; kk += 4) {
            float4 a[8], b[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = *reinterpret_cast<const float4*>(xb + 16 * i * PAD + kk);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(wb + 16 * j * PAD + kk);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
                    acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
                    acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
                    acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
                }
        }
        if ((kt + 1) % kTilesPerChunk == 0 || kt + 1 == KT) {
            // chunk finished: its partials, experts contiguous across the threads
            float* out = p.partials + static_cast<int64_t>(kt / kTilesPerChunk) * p.n * E;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t t = t0 + tg + 16 * i;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int e = e0 + eg + 16 * j;
                    if (t < p.n && e < E) out[t * E + e] = acc[i][j];
                    acc[i][j] = 0.0f;
                }
            }
        }
        if (kt + 1 < kt_end) sstore(buf ^ 1);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// per token: finish logits, softmax, top-k, blend coefficients
// ---------------------------------------------------------------------------
constexpr int kSelectThreads = 512;

__device__ __forceinline__ float expert_avail(const RouteParams& p, int e) {
    if (e < 0 || e >= p.e) return 0.0f;  // a padding selection of a pre-routed row
    float a = p.avail ? p.avail[e] : 1.0f;
    if (p.avail_mask) a = a > 0.0f ? 1.0f : 0.0f;
    if (p.slot_of_expert && p.slot_of_expert[e] < 0) a = 0.0f;
    return a;
}

// Finish one token's routing (one warp): logits from the chunk partials in
// chunk order (+ bias), softmax, top-k by (logit desc, index asc), optional
// renormalisation; or, with pre-routed inputs, read the given top-k.  Lane
// j < k returns choice j (expert, weight, availability) and has written its
// top-k outputs; every lane returns the token's shared-expert extra weight
// sum_k w (1 - a).  EPL = experts per lane (E <= 32 * EPL).  The per-expert
// statistics go to s_counts / s_mass (shared memory, the caller adds them to
// the global ones once per block) when given, else straight to global memory.
template <typename T, int EPL, typename Logits>
__device__ __forceinline__ void select_from_logits(const RouteParams& p, int64_t t, int lane, Logits&& logits,
                                                   int& mine_e, float& mine_w, float& mine_a,
                                                   float& shared_extra, int* s_counts, float* s_mass);

template <typename T, int EPL>
__device__ __forceinline__ void select_token(const RouteParams& p, int64_t t, int lane, int& mine_e,
                                             float& mine_w, float& mine_a, float& shared_extra,
                                             int* s_counts = nullptr, float* s_mass = nullptr) {
    mine_e = 0;
    mine_w = 0.0f;
    mine_a = 0.0f;
    shared_extra = 0.0f;
    if (p.prerouted) {
        for (int j = 0; j < p.k; ++j) {
            const int e = p.topk_idx[t * p.k + j];
            const float wt = p.topk_w[t * p.k + j];
            const float a = expert_avail(p, e);
            shared_extra += wt * (1.0f - a);
            if (lane == j) {
                mine_e = e;
                mine_w = wt;
                mine_a = a;
            }
        }
        if (lane < p.k) p.sel_coef[t * p.k + lane] = mine_w * mine_a;
        return;
    }
    const int C = p.nchunks;
    const int E = p.e;
    // partials[c][t][e] in global memory: the warp's lanes read consecutive experts,
    // loads in groups of 16 ahead of the in-order adds
    select_from_logits<T, EPL>(p, t, lane, [&](int e) {
        const float* pp = p.partials + t * E + e;
        const int64_t cs = p.n * E;
        float s = 0.0f;
        int c = 0;
        for (; c + 16 <= C; c += 16) {
            float r[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) r[u] = pp[(c + u) * cs];
#pragma unroll
            for (int u = 0; u < 16; ++u) s = s + r[u];
        }
        for (; c < C; ++c) s = s + pp[c * cs];
        if (p.bias) s = s + p.bias[e];
        return s;
    }, mine_e, mine_w, mine_a, shared_extra, s_counts, s_mass);
}

// The rest of a token's routing given its logits (`logits(e)`: the in-order
// chunk sum plus bias of expert e): softmax, top-k by (logit desc, index asc),
// optional renormalisation, availability, the top-k outputs and statistics.
template <typename T, int EPL, typename Logits>
__device__ __forceinline__ void select_from_logits(const RouteParams& p, int64_t t, int lane, Logits&& logits,
                                                   int& mine_e, float& mine_w, float& mine_a,
                                                   float& shared_extra, int* s_counts, float* s_mass) {
    const int E = p.e;
    mine_e = 0;
    mine_w = 0.0f;
    mine_a = 0.0f;
    shared_extra = 0.0f;
    float v[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < EPL; ++q) {
        const int e = lane + 32 * q;
        const float lg = e < E ? logits(e) : -INFINITY;
        v[q] = lg;
        m = fmaxf(m, lg);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
    float ex[EPL];
#pragma unroll
    for (int q = 0; q < EPL; ++q) {
        ex[q] = (lane + 32 * q < E) ? __expf(v[q] - m) : 0.0f;
        s += ex[q];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
    if (p.probs) {
        T* pr = static_cast<T*>(p.probs);
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
            const int e = lane + 32 * q;
            if (e < E) pr[t * E + e] = from_f32<T>(ex[q] * inv);
        }
    }
    // top-k by (logit desc, index asc); lane j keeps choice j
    unsigned taken = 0u;  // bit q: v[q] already chosen
    float wsum = 0.0f;
    for (int j = 0; j < p.k; ++j) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
            const int e = lane + 32 * q;
            if (e < E && !((taken >> q) & 1u)) {
                if (v[q] > bv || (v[q] == bv && e < bi)) {
                    bv = v[q];
                    bi = e;
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi >= E) {
            // no finite candidate (NaN logits): take the lowest unchosen index so
            // every access stays in bounds; routing of NaN rows is unspecified
            int lo = 0x7fffffff;
#pragma unroll
            for (int q = 0; q < EPL; ++q) {
                const int e = lane + 32 * q;
                if (e < E && !((taken >> q) & 1u)) lo = min(lo, e);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            bi = lo;
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        // probability of the chosen expert, broadcast from its owner lane
        float pe = 0.0f;
#pragma unroll
        for (int q = 0; q < EPL; ++q)
            if ((bi >> 5) == q) pe = ex[q] * inv;
        pe = __shfl_sync(0xffffffffu, pe, bi & 31);
        if (lane == j) {
            mine_e = bi;
            mine_w = pe;
        }
        wsum += pe;
    }
    if (p.norm_topk) mine_w = mine_w / (wsum + 1e-20f);
    if (lane < p.k) mine_a = expert_avail(p, mine_e);
    float extra = lane < p.k ? mine_w * (1.0f - mine_a) : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) extra += __shfl_xor_sync(0xffffffffu, extra, o);
    shared_extra = extra;
    if (lane < p.k) {
        const int64_t o = t * p.k + lane;
        p.topk_idx[o] = mine_e;
        p.topk_w[o] = mine_w;
        p.sel_coef[o] = mine_w * mine_a;
        if (p.counts_all) atomicAdd(s_counts ? &s_counts[mine_e] : &p.counts_all[mine_e], 1);
        if (p.mass_all) atomicAdd(s_mass ? &s_mass[mine_e] : &p.mass_all[mine_e], mine_w);
    }
}

// Direct-output calls (k = 1, no shared experts): a token whose selection is
// unavailable gets no contribution, so its output row is zeroed here.
template <typename T>
__device__ __forceinline__ void zero_direct_row(const RouteParams& p, int64_t t, int lane, float mine_a) {
    if (p.y_direct == nullptr) return;
    const float a0 = __shfl_sync(0xffffffffu, mine_a, 0);
    if (a0 > 0.0f) return;
    uint4* yv = reinterpret_cast<uint4*>(static_cast<T*>(p.y_direct) + t * p.h);
    const int n16 = p.h * static_cast<int>(sizeof(T)) / 16;
    for (int i = lane; i < n16; i += 32) yv[i] = make_uint4(0u, 0u, 0u, 0u);
}

// One warp per token: select; each available selection gets its position in
// its expert group.  The block's selections are counted per expert in shared
// memory first and one global atomic per (block, expert) reserves the block's
// positions, so a popular expert's counter sees one atomic per block instead
// of one per selection (the same for the routing statistics).
template <typename T, int EPL>
__global__ void __launch_bounds__(kSelectThreads) route_select_kernel(RouteParams p) {
    __shared__ int s_cnt[kMaxExperts];    // available selections per expert
    __shared__ int s_base[kMaxExperts];   // first group position of this block's selections
    __shared__ int s_hits[kMaxExperts];   // all selections per expert (statistics)
    __shared__ float s_mass[kMaxExperts];
    const int tid = threadIdx.x;
    for (int e = tid; e < p.e; e += kSelectThreads) {
        s_cnt[e] = 0;
        s_hits[e] = 0;
        s_mass[e] = 0.0f;
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();  // partials and zeroed counters from the logit kernel
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (kSelectThreads / 32) + warp;
    const bool valid = t < p.n;
    int mine_e = 0, rank = -1;
    float mine_w = 0.0f, mine_a = 0.0f, shared_extra = 0.0f;
    if (valid) {
        if (p.y_acc != nullptr) {
            float4* yv = reinterpret_cast<float4*>(p.y_acc + t * p.h);
            for (int i = lane; i < p.h / 4; i += 32) yv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        select_token<T, EPL>(p, t, lane, mine_e, mine_w, mine_a, shared_extra, s_hits, s_mass);
        if (lane < p.k && mine_a > 0.0f) rank = atomicAdd(&s_cnt[mine_e], 1);
        if (lane == 0 && p.num_shared > 0)
            p.shared_coef[t] = (1.0f + shared_extra) / static_cast<float>(p.num_shared);
        zero_direct_row<T>(p, t, lane, mine_a);
    }
    __syncthreads();
    for (int e = tid; e < p.e; e += kSelectThreads) {
        const int c = s_cnt[e];
        if (c > 0) s_base[e] = atomicAdd(&p.grp_count[e], c);
        if (p.counts_all && s_hits[e] > 0) atomicAdd(&p.counts_all[e], s_hits[e]);
        if (p.mass_all && s_hits[e] > 0) atomicAdd(&p.mass_all[e], s_mass[e]);
    }
    __syncthreads();
    if (valid && lane < p.k) p.pos[t * p.k + lane] = rank >= 0 ? s_base[mine_e] + rank : -1;
}

}  // namespace chronos
