// router.cuh — fused router GEMM + softmax + top-k + blend coefficients.
//
// Restates chronos/model/moe_chronos.py:112-128 (gate Linear, softmax, topk,
// norm_topk_prob renormalisation) under the bit-exact routing contract of
// include/chronos_moe.h: every logit is one thread's fmaf chain over
// h = 0..H-1 in increasing order, so the ranking is identical on every run and
// equal to the CPU oracle's.  Also produces, per token, the coefficient of the
// shared-expert term (1 + sum_k w*(1-a)) / S_h (moe_chronos.py:255-268) and,
// per selection with a > 0, the within-expert position used by the
// permutation; zeroes the fp32 output accumulator rows of its tokens.
#pragma once

#include "common.cuh"

namespace chronos {

constexpr int kRouteTokens = 32;   // tokens per block
constexpr int kRouteExperts = 64;  // experts per smem chunk
constexpr int kRouteK = 64;        // h per smem chunk
constexpr int kRouteThreads = 256;
constexpr int kRoutePad = kRouteK + 4;  // row pitch (floats) of the smem tiles
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 256;

struct RouteParams {
    const void* x;
    const void* w;
    const float* bias;
    const float* avail;
    const int32_t* slot_of_expert;
    int64_t n;
    int h, e, k, num_shared, norm_topk, prerouted;
    void* probs;          // [N, E] T or null
    int32_t* topk_idx;    // [N, k]
    float* topk_w;        // [N, k]
    int32_t* counts_all;  // [E] or null
    float* mass_all;      // [E] or null
    int32_t* grp_count;   // [E] routed-group sizes (selections with a > 0); zeroed by the caller
    int32_t* pos;         // [N, k] position within the expert group, -1 when a == 0
    float* sel_coef;      // [N, k] w * a
    float* shared_coef;   // [N] (1 + sum w (1 - a)) / S_h
    float* y_acc;         // [N, H] fp32, zeroed here
};

template <typename T>
__device__ __forceinline__ float expert_avail(const RouteParams& p, int e) {
    float a = p.avail ? p.avail[e] : 1.0f;
    if (p.slot_of_expert && p.slot_of_expert[e] < 0) a = 0.0f;
    return a;
}

template <typename T>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteParams p) {
    extern __shared__ float4 route_smem_f4[];
    float* smem = reinterpret_cast<float*>(route_smem_f4);
    float* xs = smem;                                  // [32][kRoutePad]
    float* ws = xs + kRouteTokens * kRoutePad;         // [64][kRoutePad]
    float* lg = ws + kRouteExperts * kRoutePad;        // [32][E]
    const int tid = threadIdx.x;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kRouteTokens;
    const int64_t left = p.n - t0;
    const int nt = left < kRouteTokens ? static_cast<int>(left) : kRouteTokens;
    const T* x = static_cast<const T*>(p.x);
    const T* w = static_cast<const T*>(p.w);
    const int H = p.h, E = p.e;

    // zero this block's rows of the fp32 accumulator
    if (p.y_acc != nullptr) {
        float4* yv = reinterpret_cast<float4*>(p.y_acc + t0 * H);
        const int nv = nt * H / 4;
        for (int i = tid; i < nv; i += kRouteThreads) yv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    if (!p.prerouted) {
        // ---- logits: thread (tg, eg) owns tokens {2tg, 2tg+1} x experts {eg + 16j} ----
        const int eg = tid & 15;
        const int tg = tid >> 4;
        for (int ec = 0; ec < E; ec += kRouteExperts) {
            float acc[2][4];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
            for (int kc = 0; kc < H; kc += kRouteK) {
                const int kw = min(kRouteK, H - kc);
                __syncthreads();
                for (int i = tid; i < kRouteTokens * kRouteK; i += kRouteThreads) {
                    const int r = i / kRouteK, c = i % kRouteK;
                    float v = 0.0f;
                    if (r < nt && c < kw) v = to_f32<T>(x[(t0 + r) * H + kc + c]);
                    xs[r * kRoutePad + c] = v;
                }
                for (int i = tid; i < kRouteExperts * kRouteK; i += kRouteThreads) {
                    const int r = i / kRouteK, c = i % kRouteK;
                    float v = 0.0f;
                    if (ec + r < E && c < kw) v = to_f32<T>(w[static_cast<int64_t>(ec + r) * H + kc + c]);
                    ws[r * kRoutePad + c] = v;
                }
                __syncthreads();
                const float* x0 = xs + (2 * tg) * kRoutePad;
                const float* x1 = x0 + kRoutePad;
                for (int c = 0; c < kw; c += 4) {
                    const float4 a0 = *reinterpret_cast<const float4*>(x0 + c);
                    const float4 a1 = *reinterpret_cast<const float4*>(x1 + c);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 b = *reinterpret_cast<const float4*>(ws + (eg + 16 * j) * kRoutePad + c);
                        // sequential in h: c, c+1, c+2, c+3 (zero padding past kw adds exact zeros)
                        acc[0][j] = fmaf(a0.x, b.x, acc[0][j]);
                        acc[0][j] = fmaf(a0.y, b.y, acc[0][j]);
                        acc[0][j] = fmaf(a0.z, b.z, acc[0][j]);
                        acc[0][j] = fmaf(a0.w, b.w, acc[0][j]);
                        acc[1][j] = fmaf(a1.x, b.x, acc[1][j]);
                        acc[1][j] = fmaf(a1.y, b.y, acc[1][j]);
                        acc[1][j] = fmaf(a1.z, b.z, acc[1][j]);
                        acc[1][j] = fmaf(a1.w, b.w, acc[1][j]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int e = ec + eg + 16 * j;
                    if (e < E) {
                        float v = acc[i][j];
                        if (p.bias) v = v + p.bias[e];
                        lg[(2 * tg + i) * E + e] = v;
                    }
                }
        }
    }
    __syncthreads();

    // ---- per token: softmax, top-k, blend coefficients (one warp per token) ----
    const int warp = tid >> 5, lane = tid & 31;
    const int per_lane = (E + 31) / 32;
    for (int r = warp; r < nt; r += kRouteThreads / 32) {
        const int64_t t = t0 + r;
        if (p.prerouted) {
            // weights and indices come from an earlier routing call
            float shared_extra = 0.0f;
            for (int j = 0; j < p.k; ++j) {
                const int e = p.topk_idx[t * p.k + j];
                const float wt = p.topk_w[t * p.k + j];
                const float a = expert_avail<T>(p, e);
                shared_extra += wt * (1.0f - a);
                if (lane == 0) {
                    p.sel_coef[t * p.k + j] = wt * a;
                    p.pos[t * p.k + j] = a > 0.0f ? atomicAdd(&p.grp_count[e], 1) : -1;
                }
            }
            if (lane == 0 && p.num_shared > 0)
                p.shared_coef[t] = (1.0f + shared_extra) / static_cast<float>(p.num_shared);
            continue;
        }
        float v[kMaxExperts / 32];
        float m = -INFINITY;
#pragma unroll
        for (int q = 0; q < kMaxExperts / 32; ++q) {
            const int e = lane + 32 * q;
            v[q] = (q < per_lane && e < E) ? lg[r * E + e] : -INFINITY;
            m = fmaxf(m, v[q]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float s = 0.0f;
        float ex[kMaxExperts / 32];
#pragma unroll
        for (int q = 0; q < kMaxExperts / 32; ++q) {
            const int e = lane + 32 * q;
            ex[q] = (q < per_lane && e < E) ? __expf(v[q] - m) : 0.0f;
            s += ex[q];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float inv = 1.0f / s;
        if (p.probs) {
            T* pr = static_cast<T*>(p.probs);
#pragma unroll
            for (int q = 0; q < kMaxExperts / 32; ++q) {
                const int e = lane + 32 * q;
                if (q < per_lane && e < E) pr[t * E + e] = from_f32<T>(ex[q] * inv);
            }
        }
        // top-k by (logit desc, index asc)
        unsigned taken = 0u;  // bit q: v[q] already chosen
        float wsel[kMaxTopK];
        int isel[kMaxTopK];
        float wsum = 0.0f;
        for (int j = 0; j < p.k; ++j) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int q = 0; q < kMaxExperts / 32; ++q) {
                const int e = lane + 32 * q;
                if (q < per_lane && e < E && !((taken >> q) & 1u)) {
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
                for (int q = 0; q < kMaxExperts / 32; ++q) {
                    const int e = lane + 32 * q;
                    if (q < per_lane && e < E && !((taken >> q) & 1u)) lo = min(lo, e);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                bi = lo;
            }
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            // probability of the chosen expert, broadcast from its owner lane
            float pe = 0.0f;
#pragma unroll
            for (int q = 0; q < kMaxExperts / 32; ++q)
                if ((bi >> 5) == q) pe = ex[q] * inv;
            pe = __shfl_sync(0xffffffffu, pe, bi & 31);
            wsel[j] = pe;
            isel[j] = bi;
            wsum += pe;
        }
        if (p.norm_topk) {
            const float d = wsum + 1e-20f;
            for (int j = 0; j < p.k; ++j) wsel[j] = wsel[j] / d;
        }
        float shared_extra = 0.0f;
        for (int j = 0; j < p.k; ++j) {
            const int e = isel[j];
            const float a = expert_avail<T>(p, e);
            shared_extra += wsel[j] * (1.0f - a);
            if (lane == j % 32) {
                p.topk_idx[t * p.k + j] = e;
                p.topk_w[t * p.k + j] = wsel[j];
                p.sel_coef[t * p.k + j] = wsel[j] * a;
                p.pos[t * p.k + j] = a > 0.0f ? atomicAdd(&p.grp_count[e], 1) : -1;
                if (p.counts_all) atomicAdd(&p.counts_all[e], 1);
                if (p.mass_all) atomicAdd(&p.mass_all[e], wsel[j]);
            }
        }
        if (lane == 0 && p.num_shared > 0)
            p.shared_coef[t] = (1.0f + shared_extra) / static_cast<float>(p.num_shared);
    }
}

inline size_t route_smem_bytes(int num_experts) {
    return sizeof(float) * (static_cast<size_t>(kRouteTokens) * kRoutePad +
                            static_cast<size_t>(kRouteExperts) * kRoutePad +
                            static_cast<size_t>(kRouteTokens) * num_experts);
}

}  // namespace chronos
