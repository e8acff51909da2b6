// lookahead.cuh — the lookahead router's two projections, SiLU and softmaxes
// in one kernel (chronos/model/lookahead_router.py:36-55).
//
// One thread-block cluster per group of TB tokens (TB <= 8), CS CTAs (<= 8),
// 256 threads each.  W1's rows are split over the cluster's CTAs (RPC rows
// each), so a decode batch of 32 tokens runs on 32 SMs and every W1 row is read
// by one CTA per token group.
//   Phase 1: the group's x rows are staged in shared memory as fp32; each warp
//   takes 4 W1 rows at a time (16-byte loads, lanes over 8-column groups) and
//   accumulates 4 rows x TB tokens in registers, so one shared-memory read of x
//   feeds 4 FMAs; warp sums, SiLU -> h1 slice [TB][RPC] in shared memory.
//   Cluster barrier.
//   Phase 2: CTA r handles tokens r, r + CS, ...: it gathers the token's h1 row
//   from every CTA's slice (distributed shared memory), computes the E*K logits
//   (a warp per output, W2 rows with 16-byte loads) and the K softmaxes.
//   Cluster barrier (no CTA leaves while a peer may read its slice).
// Summation order of a dot product: lane partials in increasing column, then
// the warp's butterfly sum — the same for any cluster size.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace chronos {

constexpr int kLookaheadThreads = 256;
constexpr int kLookaheadWarps = kLookaheadThreads / 32;
constexpr int kLookaheadMaxTB = 8;
constexpr int kLookaheadRowsPerWarp = 4;
constexpr int kLookaheadMaxCluster = 8;
constexpr int kLookaheadXBytes = 128 << 10;   // the staged x rows of a group

struct LookaheadParams {
    const void* x;
    const void* w1;
    const void* w2;
    void* probs;
    int64_t n;
    int h, inner, e, k;
    int tb;     // tokens per cluster
    int rpc;    // W1 rows per CTA
    int vec1;   // 1: x and W1 rows read as 8-element vectors (H % 8 == 0, 16-byte aligned)
    int vec2;   // 1: W2 rows read as 8-element vectors (inner % 8 == 0, aligned)
};

// Shared memory of one CTA, in floats: x [tb][h], h1 slice [tb][rpc], the
// gathered h1 row [inner], logits [e*k].
inline size_t lookahead_smem(int tb, int h, int rpc, int inner, int ek) {
    return (static_cast<size_t>(tb) * h + static_cast<size_t>(tb) * rpc + inner + ek) * sizeof(float);
}

template <typename T>
__global__ void __launch_bounds__(kLookaheadThreads) lookahead_kernel(LookaheadParams p) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) float la_smem[];
    cg::cluster_group cluster = cg::this_cluster();
    pdl_wait();   // launched early behind the kernel that writes x (programmatic launch)
    const int rank = static_cast<int>(cluster.block_rank());
    const int cs = static_cast<int>(cluster.num_blocks());
    const int tb = p.tb, H = p.h, rpc = p.rpc, inner = p.inner, ek = p.e * p.k;
    float* xs = la_smem;                                       // [tb][h]
    float* h1s = xs + static_cast<size_t>(tb) * H;             // [tb][rpc]
    float* hrow = h1s + static_cast<size_t>(tb) * rpc;         // [inner]
    float* lg = hrow + inner;                                  // [ek]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x / cs) * tb;
    const int nt = static_cast<int>(p.n - t0 < tb ? p.n - t0 : tb);
    const T* x = static_cast<const T*>(p.x);

    // x rows of the group.  Vector layout: the 8 columns of group q of row r
    // split in two float4 halves, lo at [r][0][q] and hi at [r][1][q], so that
    // lanes reading consecutive groups touch consecutive 16-byte words.
    const int q8 = H / 8;
    if (p.vec1) {
        float4* xs4 = reinterpret_cast<float4*>(xs);
        for (int i = tid; i < tb * q8; i += kLookaheadThreads) {
            const int r = i / q8, q = i % q8;
            float v[8];
            if (r < nt) {
                load8<T>(x + (t0 + r) * H + q * 8, v);
            } else {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = 0.0f;
            }
            xs4[(r * 2) * q8 + q] = make_float4(v[0], v[1], v[2], v[3]);
            xs4[(r * 2 + 1) * q8 + q] = make_float4(v[4], v[5], v[6], v[7]);
        }
    } else {
        for (int i = tid; i < tb * H; i += kLookaheadThreads) {
            const int r = i / H, c = i % H;
            xs[i] = r < nt ? to_f32<T>(x[(t0 + r) * H + c]) : 0.0f;
        }
    }
    __syncthreads();

    // phase 1: this CTA's W1 rows j0 .. j0 + rpc - 1, 4 rows per warp at a time
    const T* w1 = static_cast<const T*>(p.w1);
    const int j0 = rank * rpc;
    constexpr int R = kLookaheadRowsPerWarp;
    for (int jb = warp * R; jb < rpc; jb += kLookaheadWarps * R) {
        float acc[R][kLookaheadMaxTB];
#pragma unroll
        for (int q = 0; q < R; ++q)
#pragma unroll
            for (int r = 0; r < kLookaheadMaxTB; ++r) acc[q][r] = 0.0f;
        bool live[R];
        const T* rows[R];
#pragma unroll
        for (int q = 0; q < R; ++q) {
            live[q] = jb + q < rpc && j0 + jb + q < inner;
            rows[q] = w1 + static_cast<int64_t>(live[q] ? j0 + jb + q : 0) * H;
        }
        if (p.vec1) {
            const float4* xs4 = reinterpret_cast<const float4*>(xs);
            for (int q = lane; q < q8; q += 32) {
                float w[R][8];
#pragma unroll
                for (int rr = 0; rr < R; ++rr) {
                    if (live[rr]) {
                        load8<T>(rows[rr] + q * 8, w[rr]);
                    } else {
#pragma unroll
                        for (int u = 0; u < 8; ++u) w[rr][u] = 0.0f;
                    }
                }
#pragma unroll
                for (int r = 0; r < kLookaheadMaxTB; ++r) {
                    if (r >= tb) break;
                    const float4 lo = xs4[(r * 2) * q8 + q], hi = xs4[(r * 2 + 1) * q8 + q];
                    const float xv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                    for (int rr = 0; rr < R; ++rr)
#pragma unroll
                        for (int u = 0; u < 8; ++u) acc[rr][r] = fmaf(w[rr][u], xv[u], acc[rr][r]);
                }
            }
        } else {
            for (int c = lane; c < H; c += 32) {
                float w[R];
#pragma unroll
                for (int rr = 0; rr < R; ++rr) w[rr] = live[rr] ? to_f32<T>(rows[rr][c]) : 0.0f;
#pragma unroll
                for (int r = 0; r < kLookaheadMaxTB; ++r) {
                    if (r >= tb) break;
                    const float xv = xs[r * H + c];
#pragma unroll
                    for (int rr = 0; rr < R; ++rr) acc[rr][r] = fmaf(w[rr], xv, acc[rr][r]);
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr)
#pragma unroll
            for (int r = 0; r < kLookaheadMaxTB; ++r) {
                const float v = warp_sum(acc[rr][r]);
                if (lane == 0 && live[rr] && r < tb) h1s[r * rpc + jb + rr] = silu_f32(v);
            }
    }
    cluster.sync();   // every CTA's h1 slice is complete and visible to the cluster

    // phase 2: logits and softmaxes of tokens rank, rank + cs, ...
    const T* w2 = static_cast<const T*>(p.w2);
    T* probs = static_cast<T*>(p.probs);
    for (int r = rank; r < nt; r += cs) {
        for (int j = tid; j < inner; j += kLookaheadThreads) {
            const int owner = j / rpc;
            hrow[j] = cluster.map_shared_rank(h1s, owner)[r * rpc + (j - owner * rpc)];
        }
        __syncthreads();
        for (int o = warp; o < ek; o += kLookaheadWarps) {
            const T* row = w2 + static_cast<int64_t>(o) * inner;
            float acc = 0.0f;
            if (p.vec2) {
                for (int c8 = lane * 8; c8 < inner; c8 += 256) {
                    float w[8];
                    load8<T>(row + c8, w);
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc = fmaf(w[u], hrow[c8 + u], acc);
                }
            } else {
                for (int c = lane; c < inner; c += 32) acc = fmaf(to_f32<T>(row[c]), hrow[c], acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) lg[o] = acc;
        }
        __syncthreads();
        for (int s = warp; s < p.k; s += kLookaheadWarps) {
            const float* l = lg + s * p.e;
            float m = -INFINITY;
            for (int e = lane; e < p.e; e += 32) m = fmaxf(m, l[e]);
#pragma unroll
            for (int q = 16; q > 0; q >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, q));
            float sum = 0.0f;
            for (int e = lane; e < p.e; e += 32) sum += __expf(l[e] - m);
            sum = warp_sum(sum);
            const float inv = 1.0f / sum;
            T* out = probs + ((t0 + r) * p.k + s) * p.e;
            for (int e = lane; e < p.e; e += 32) out[e] = from_f32<T>(__expf(l[e] - m) * inv);
        }
        __syncthreads();   // hrow and lg are rewritten by the next token
    }
    cluster.sync();   // the slices stay alive until every peer has gathered its rows
}

}  // namespace chronos
