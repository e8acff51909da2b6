// lookahead.cuh — the lookahead router's two projections, SiLU and softmaxes
// in one kernel (chronos/model/lookahead_router.py:36-55).
//
// Block = a group of TB tokens (TB * H fp32 staged in shared memory), 256
// threads.  Phase 1: one warp per inner unit j (strided), lanes stride over H,
// every W1 row read once for the TB tokens; warp sums, SiLU -> h1 [TB][inner]
// in shared memory.  Phase 2: one warp per output o = s*E + e, same pattern
// over W2 -> logits [TB][E*K].  Phase 3: one warp per (token, step): max, exp,
// sum, normalise, write probs in the output type.
#pragma once

#include "common.cuh"

namespace chronos {

constexpr int kLookaheadThreads = 256;
constexpr int kLookaheadWarps = kLookaheadThreads / 32;
constexpr int kLookaheadMaxTB = 8;

struct LookaheadParams {
    const void* x;
    const void* w1;
    const void* w2;
    void* probs;
    int64_t n;
    int h, inner, e, k, tb;
};

template <typename T>
__global__ void __launch_bounds__(kLookaheadThreads) lookahead_kernel(LookaheadParams p) {
    extern __shared__ float la_smem[];
    const int tb = p.tb;
    float* xs = la_smem;                     // [tb][h]
    float* h1 = xs + tb * p.h;               // [tb][inner]
    float* lg = h1 + tb * p.inner;           // [tb][e*k]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tb;
    const int nt = static_cast<int>(p.n - t0 < tb ? p.n - t0 : tb);
    const T* x = static_cast<const T*>(p.x);
    for (int i = threadIdx.x; i < tb * p.h; i += kLookaheadThreads) {
        const int r = i / p.h, c = i % p.h;
        xs[i] = r < nt ? to_f32<T>(x[(t0 + r) * p.h + c]) : 0.0f;
    }
    __syncthreads();
    // phase 1: h1 = silu(W1 . x)
    const T* w1 = static_cast<const T*>(p.w1);
    for (int j = warp; j < p.inner; j += kLookaheadWarps) {
        float acc[kLookaheadMaxTB];
#pragma unroll
        for (int r = 0; r < kLookaheadMaxTB; ++r) acc[r] = 0.0f;
        const T* row = w1 + static_cast<int64_t>(j) * p.h;
        for (int c = lane; c < p.h; c += 32) {
            const float wv = to_f32<T>(row[c]);
#pragma unroll
            for (int r = 0; r < kLookaheadMaxTB; ++r)
                if (r < tb) acc[r] = fmaf(wv, xs[r * p.h + c], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < kLookaheadMaxTB; ++r) {
            float v = acc[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && r < tb) h1[r * p.inner + j] = silu_f32(v);
        }
    }
    __syncthreads();
    // phase 2: logits = W2 . h1
    const T* w2 = static_cast<const T*>(p.w2);
    const int ek = p.e * p.k;
    for (int o = warp; o < ek; o += kLookaheadWarps) {
        float acc[kLookaheadMaxTB];
#pragma unroll
        for (int r = 0; r < kLookaheadMaxTB; ++r) acc[r] = 0.0f;
        const T* row = w2 + static_cast<int64_t>(o) * p.inner;
        for (int c = lane; c < p.inner; c += 32) {
            const float wv = to_f32<T>(row[c]);
#pragma unroll
            for (int r = 0; r < kLookaheadMaxTB; ++r)
                if (r < tb) acc[r] = fmaf(wv, h1[r * p.inner + c], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < kLookaheadMaxTB; ++r) {
            float v = acc[r];
#pragma unroll
            for (int q = 16; q > 0; q >>= 1) v += __shfl_xor_sync(0xffffffffu, v, q);
            if (lane == 0 && r < tb) lg[r * ek + o] = v;
        }
    }
    __syncthreads();
    // phase 3: a softmax over the E experts of every (token, step)
    T* probs = static_cast<T*>(p.probs);
    for (int g = warp; g < nt * p.k; g += kLookaheadWarps) {
        const int r = g / p.k, s = g % p.k;
        const float* l = lg + r * ek + s * p.e;
        float m = -INFINITY;
        for (int e = lane; e < p.e; e += 32) m = fmaxf(m, l[e]);
#pragma unroll
        for (int q = 16; q > 0; q >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, q));
        float sum = 0.0f;
        for (int e = lane; e < p.e; e += 32) sum += __expf(l[e] - m);
#pragma unroll
        for (int q = 16; q > 0; q >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, q);
        const float inv = 1.0f / sum;
        T* out = probs + ((t0 + r) * p.k + s) * p.e;
        for (int e = lane; e < p.e; e += 32) out[e] = from_f32<T>(__expf(l[e] - m) * inv);
    }
}

}  // namespace chronos
