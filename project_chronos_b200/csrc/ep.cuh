// ep.cuh — expert-parallel dispatch (send-buffer packing) and combine.
//
// Rank g owns the routed experts [g*epr, (g+1)*epr).  Dispatch turns this
// rank's routing (topk_idx / topk_weight from the router kernels) into the
// all-to-all send buffers:
//   ep_count_kernel  one thread per (token, choice): a = avail[e], the shared
//                    experts' share w*(1-a), and for a > 0 the selection's
//                    position among those bound for (expert chunk, rank e/epr)
//                    (global atomics on C*G counters, zeroed by the caller);
//   ep_pack_kernel   one warp per (token, choice): send row = prefix of the
//                    counts + position (or, with fixed segments, rank * seg_rows
//                    + position); metadata (local expert, w*a) and the x
//                    row copied with 16-byte vectors, every load of a lane
//                    issued before its stores.
// With `pairs` > 1 (one expert chunk) the rows are deduplicated: one send row
// per (token, destination rank), opened by the token's first available
// selection on that rank, its metadata [pairs][2] listing every available
// selection of the token on that rank in choice order (padding: expert -1);
// the other selections' pair_slot is -1, their contribution comes back in the
// opening selection's row.
// ep_combine_kernel folds the returned rows back: one block per token,
// y_t = y_shared_t + sum_j recv[pair_slot(t, j)] in fp32, j ascending, so the
// result does not depend on the (atomic) order of rows inside a rank.
#pragma once

#include "common.cuh"

namespace chronos {

constexpr int kEpMaxRanks = 32;
constexpr int kMaxTopKEp = 16;
constexpr int kEpPackThreads = 256;
constexpr int kEpCombineThreads = 128;

struct EpParams {
    const void* x;
    int64_t n;
    int h, e, k, g, epr;
    int chunks;             // expert chunks per rank (1: unchunked)
    int chunk_experts;      // local experts per chunk (epr / chunks)
    int pairs;              // > 1: one send row per (token, destination rank) carrying up to
                            // `pairs` selections (deduplicated); 1: one row per selection
    int64_t seg_rows;       // > 0 (one chunk): rank g's rows start at row g * seg_rows (fixed
                            // all-to-all splits); the unused rows of each segment get padding
                            // metadata.  0: rows packed by the prefix sums of the counts
    const int32_t* topk_idx;
    const float* topk_w;
    const float* avail;
    int32_t* counts;      // [G]
    int32_t* pos;         // [N*k]
    void* send_x;         // [N*k, H]
    int32_t* send_meta;   // [N*k, 2] (local expert, fp32 bits of w*a)
    int32_t* pair_slot;   // [N*k]
    float* shared_w;      // [N, k]
};

__device__ __forceinline__ float ep_avail(const EpParams& p, int e) {
    if (e < 0 || e >= p.e) return 0.0f;
    if (p.avail == nullptr) return 1.0f;
    const float a = p.avail[e];
    return a > 1.0f ? 1.0f : (a > 0.0f ? a : 0.0f);
}

// Deduplicated dispatch: selection j of token t opens the send row of its
// destination rank when it is the token's first available selection bound
// for that rank (the rank's other selections of the token ride in that row's
// metadata).
__device__ __forceinline__ bool ep_first_for_rank(const EpParams& p, int64_t t, int j, int dest) {
    for (int q = 0; q < j; ++q) {
        const int eq = p.topk_idx[t * p.k + q];
        if (ep_avail(p, eq) > 0.0f && eq / p.epr == dest) return false;
    }
    return true;
}

__global__ void __launch_bounds__(kEpPackThreads) ep_count_kernel(EpParams p) {
    pdl_trigger();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * kEpPackThreads + threadIdx.x;
    if (i >= p.n * p.k) return;
    const int e = p.topk_idx[i];
    const float w = p.topk_w[i];
    const float a = ep_avail(p, e);
    p.shared_w[i] = w * (1.0f - a);
    bool opens = a > 0.0f;
    if (opens && p.pairs > 1) opens = ep_first_for_rank(p, i / p.k, static_cast<int>(i % p.k), e / p.epr);
    const int key = opens ? ((e % p.epr) / p.chunk_experts) * p.g + e / p.epr : 0;
    p.pos[i] = opens ? atomicAdd(&p.counts[key], 1) : -1;
}

template <typename T>
__global__ void __launch_bounds__(kEpPackThreads) ep_pack_kernel(EpParams p) {
    __shared__ int s_off[kEpMaxRanks];
    pdl_trigger();
    pdl_wait();  // counts and positions
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < 32) {
        const int c = lane < p.chunks * p.g ? p.counts[lane] : 0;
        int v = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += u;
        }
        s_off[lane] = v - c;
    }
    if (p.seg_rows > 0 && tid < 32) s_off[lane] = lane < p.g ? static_cast<int>(lane * p.seg_rows) : 0;
    __syncthreads();
    if (p.seg_rows > 0) {
        // padding metadata (expert -1, weight 0) for the rows of each segment past its count
        const int64_t total = p.g * p.seg_rows;
        const int64_t stride = static_cast<int64_t>(gridDim.x) * kEpPackThreads;
        for (int64_t r = static_cast<int64_t>(blockIdx.x) * kEpPackThreads + tid; r < total; r += stride) {
            const int g = static_cast<int>(r / p.seg_rows);
            if (r - g * p.seg_rows < p.counts[g]) continue;
            int32_t* m = p.send_meta + 2 * r * p.pairs;
            for (int q = 0; q < p.pairs; ++q) {
                m[2 * q] = -1;
                m[2 * q + 1] = __float_as_int(0.0f);
            }
        }
    }
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * (kEpPackThreads / 32) + (tid >> 5);
    if (gw >= p.n * p.k) return;
    const int ps = p.pos[gw];
    if (ps < 0) {
        if (lane == 0) p.pair_slot[gw] = -1;
        return;
    }
    const int e = p.topk_idx[gw];
    const int dest = e / p.epr;
    const int key = ((e % p.epr) / p.chunk_experts) * p.g + dest;
    const int64_t slot = static_cast<int64_t>(s_off[key]) + ps;
    const int64_t t = gw / p.k;
    if (lane == 0) {
        p.pair_slot[gw] = static_cast<int32_t>(slot);
        if (p.pairs > 1) {
            // the token's available selections on this rank, in choice order, padded
            int32_t* m = p.send_meta + 2 * slot * p.pairs;
            int q = 0;
            for (int j = static_cast<int>(gw % p.k); j < p.k && q < p.pairs; ++j) {
                const int ej = p.topk_idx[t * p.k + j];
                const float aj = ep_avail(p, ej);
                if (aj > 0.0f && ej / p.epr == dest) {
                    m[2 * q] = ej - dest * p.epr;
                    m[2 * q + 1] = __float_as_int(p.topk_w[t * p.k + j] * aj);
                    ++q;
                }
            }
            for (; q < p.pairs; ++q) {
                m[2 * q] = -1;
                m[2 * q + 1] = __float_as_int(0.0f);
            }
        } else {
            p.send_meta[2 * slot] = e - dest * p.epr;
            p.send_meta[2 * slot + 1] = __float_as_int(p.topk_w[gw] * ep_avail(p, e));
        }
    }
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + t * p.h);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(p.send_x) + slot * p.h);
    const int n16 = p.h * static_cast<int>(sizeof(T)) / 16;
    int i = lane;
    for (; i + 32 * 7 < n16; i += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = src[i + 32 * u];
#pragma unroll
        for (int u = 0; u < 8; ++u) dst[i + 32 * u] = v[u];
    }
    for (; i < n16; i += 32) dst[i] = src[i];
}

struct EpCombineParams {
    const void* y_shared;   // [N, H] or null
    const void* recv_y;     // [rows, H]
    const int32_t* pair_slot;
    void* y;                // [N, H]
    int64_t n;
    int h, k;
};

// 8 elements of T in one 16-byte vector (bf16/fp16), or 4 (fp32).
template <typename T>
struct Vec16 {
    static constexpr int kElems = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void vec_add_f32(float* acc, const uint4& v) {
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < Vec16<T>::kElems; ++i) acc[i] += to_f32<T>(e[i]);
}

template <typename T>
__global__ void __launch_bounds__(kEpCombineThreads) ep_combine_kernel(EpCombineParams p) {
    constexpr int EL = Vec16<T>::kElems;
    __shared__ int s_slot[kMaxTopKEp];
    pdl_trigger();
    pdl_wait();
    const int64_t t = blockIdx.x;
    if (threadIdx.x < p.k) s_slot[threadIdx.x] = p.pair_slot[t * p.k + threadIdx.x];
    __syncthreads();
    const int n16 = p.h / EL;
    const uint4* ysh = p.y_shared ? reinterpret_cast<const uint4*>(static_cast<const T*>(p.y_shared) + t * p.h)
                                  : nullptr;
    const T* recv = static_cast<const T*>(p.recv_y);
    uint4* out = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + t * p.h);
    for (int v = threadIdx.x; v < n16; v += kEpCombineThreads) {
        uint4 in[kMaxTopKEp + 1];
        const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
        in[0] = ysh ? ysh[v] : zero;
#pragma unroll
        for (int j = 0; j < kMaxTopKEp; ++j) {
            if (j < p.k) {
                const int s = s_slot[j];
                in[j + 1] = s >= 0 ? reinterpret_cast<const uint4*>(recv + static_cast<int64_t>(s) * p.h)[v]
                                   : zero;
            }
        }
        float acc[EL];
#pragma unroll
        for (int i = 0; i < EL; ++i) acc[i] = 0.0f;
        vec_add_f32<T>(acc, in[0]);
#pragma unroll
        for (int j = 0; j < kMaxTopKEp; ++j)
            if (j < p.k) vec_add_f32<T>(acc, in[j + 1]);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < EL; ++i) oe[i] = from_f32<T>(acc[i]);
        out[v] = o;
    }
}

}  // namespace chronos
