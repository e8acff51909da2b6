// route_fused.cuh — decode routing in ONE launch: chunk partial logits,
// selection, plan and slot tables, as one thread-block cluster.
//
// Decode batches (N <= 64 tokens) spend more time in launch and dependency
// latency than in routing arithmetic.  This kernel replaces the two launches
// of the decode path (route_partials_kernel, route_select_plan_kernel) by one
// cluster of up to 8 CTAs, 256 threads each:
//
//   1. CTA r computes the chunk partials of chunks r, r + ncta, ... (one fmaf
//      chain per 128-element chunk, the routing contract of router.cuh) for
//      every (token, expert) into its own shared memory;
//   2. cluster barrier; one warp per token then sums its 16-or-fewer chunk
//      partials IN CHUNK ORDER, reading the other CTAs' shared memory
//      (distributed shared memory), and selects (select_from_logits, the same
//      code as the select kernels); group positions and the per-expert
//      statistics are counted with atomics on CTA 0's shared memory;
//   3. cluster barrier; CTA 0 scans the group sizes and writes the plan and
//      slot tables (plan_tables, as the select + plan kernel does).
//
// Nothing is counted in global memory, so nothing has to be zeroed before the
// launch; the barriers are the hardware's cluster barriers, reached by every
// thread of every CTA (no CTA returns before the second one, so shared memory
// another CTA reads is never released early).  The logits are bit-identical
// to the two-kernel path (same chains, same order of the chunk sums).
#pragma once

#include <cooperative_groups.h>

#include "plan.cuh"
#include "router.cuh"

namespace chronos {

constexpr int kFusedRouteThreads = 256;
constexpr int kFusedRouteWarps = kFusedRouteThreads / 32;
constexpr int kFusedRouteMaxCtas = 8;   // the portable cluster size
constexpr int kFusedRouteMaxTokens = 64;
constexpr int kFusedRouteMaxChunks = 32;  // H <= 4096: at most 4 chunks per CTA

// Dynamic shared memory of one CTA: x chunk rows (fp32, token count padded to
// a group of 8), the chunk's weight rows (16-byte padded, as the partials
// kernel stages them), the CTA's partials [cpc][N][E].
template <typename T>
__host__ __device__ constexpr int fused_route_row_bytes() {
    return kRouteChunk * static_cast<int>(sizeof(T)) + 16;
}
template <typename T>
inline size_t fused_route_smem(int64_t n, int e, int cpc) {
    const int64_t npad = (n + kRouteGroup - 1) / kRouteGroup * kRouteGroup;
    return static_cast<size_t>(npad) * kRouteChunk * 4 + static_cast<size_t>(e) * fused_route_row_bytes<T>() +
           static_cast<size_t>(cpc) * n * e * 4;
}

template <typename T, int EPL>
__global__ void __launch_bounds__(kFusedRouteThreads)
    route_decode_fused_kernel(RouteParams rp, PlanParams pp, ScatterParams sp, int cpc) {
    namespace cg = cooperative_groups;
    constexpr int ROW = fused_route_row_bytes<T>();
    constexpr int V16 = kRouteChunk * static_cast<int>(sizeof(T)) / 16;
    constexpr int EPV = 16 / static_cast<int>(sizeof(T));
    extern __shared__ __align__(16) uint8_t frs[];
    __shared__ int s_cnt[kMaxExperts];      // CTA 0: available selections per expert
    __shared__ int s_hits[kMaxExperts];     // CTA 0: all selections per expert (statistics)
    __shared__ float s_mass[kMaxExperts];   // CTA 0: selected weight per expert (statistics)
    __shared__ int s_off[kMaxExperts];
    __shared__ int s_scratch[kFusedRouteWarps];
    __shared__ int s_tot[4];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int ncta = static_cast<int>(cluster.num_blocks());
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = static_cast<int>(rp.n), E = rp.e, H = rp.h, C = rp.nchunks, k = rp.k;
    const int npad = (N + kRouteGroup - 1) / kRouteGroup * kRouteGroup;
    float* xs = reinterpret_cast<float*>(frs);                              // [npad][128]
    uint8_t* ws = frs + static_cast<size_t>(npad) * kRouteChunk * 4;        // [E][ROW]
    float* part = reinterpret_cast<float*>(ws + static_cast<size_t>(E) * ROW);  // [cpc][N][E]
    pdl_trigger();

    if (rank == 0)
        for (int i = tid; i < kMaxExperts; i += kFusedRouteThreads) {
            s_cnt[i] = 0;
            s_hits[i] = 0;
            s_mass[i] = 0.0f;
        }
    if (sp.slot_map != nullptr)
        for (int i = rank * kFusedRouteThreads + tid; i < E * N; i += ncta * kFusedRouteThreads)
            sp.slot_map[i] = -1;

    // 1) this CTA's chunk partials, in shared memory
    const T* x = static_cast<const T*>(rp.x);
    const T* w = static_cast<const T*>(rp.w);
    const bool vec_ok = (H % EPV) == 0;
    const int groups = npad / kRouteGroup;
    for (int j = 0; j < cpc; ++j) {
        const int c = rank + j * ncta;   // the same for every thread of the CTA
        if (c >= C) break;
        const int h0 = c * kRouteChunk;
        const int len = min(kRouteChunk, H - h0);  // multiple of 4
        for (int i = tid; i < E * V16; i += kFusedRouteThreads) {
            const int r = i / V16, v = i % V16;
            const T* src = w + static_cast<int64_t>(r) * H + h0 + v * EPV;
            uint4 val;
            if (vec_ok && v * EPV + EPV <= len) {
                val = *reinterpret_cast<const uint4*>(src);
            } else {
                T tmp[EPV];
#pragma unroll
                for (int u = 0; u < EPV; ++u) tmp[u] = (v * EPV + u < len) ? src[u] : from_f32<T>(0.0f);
                val = *reinterpret_cast<const uint4*>(tmp);
            }
            *reinterpret_cast<uint4*>(ws + r * ROW + v * 16) = val;
        }
        for (int i = tid; i < npad * (kRouteChunk / 4); i += kFusedRouteThreads) {
            const int r = i / (kRouteChunk / 4), q4 = (i % (kRouteChunk / 4)) * 4;
            const float4 xv = (r < N && q4 < len) ? load4<T>(x + static_cast<int64_t>(r) * H + h0 + q4)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(xs + r * kRouteChunk + q4) = xv;
        }
        __syncthreads();
        // item = (expert, group of 8 tokens): 8 chains over h in increasing order
        for (int item = tid; item < E * groups; item += kFusedRouteThreads) {
            const int e = item % E, g = item / E;
            float acc[kRouteGroup];
#pragma unroll
            for (int i = 0; i < kRouteGroup; ++i) acc[i] = 0.0f;
            const uint8_t* wrow = ws + e * ROW;
            const float* xg = xs + g * kRouteGroup * kRouteChunk;
#pragma unroll 4
            for (int q = 0; q < kRouteChunk; q += 4) {
                const float4 b = load4<T>(reinterpret_cast<const T*>(wrow) + q);
#pragma unroll
                for (int i = 0; i < kRouteGroup; ++i) {
                    const float4 a = *reinterpret_cast<const float4*>(xg + i * kRouteChunk + q);
                    acc[i] = fmaf(a.x, b.x, acc[i]);
                    acc[i] = fmaf(a.y, b.y, acc[i]);
                    acc[i] = fmaf(a.z, b.z, acc[i]);
                    acc[i] = fmaf(a.w, b.w, acc[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < kRouteGroup; ++i) {
                const int t = g * kRouteGroup + i;
                if (t < N) part[(static_cast<size_t>(j) * N + t) * E + e] = acc[i];
            }
        }
        __syncthreads();
    }
    cluster.sync();  // every chunk's partials and CTA 0's zeroed counters are visible

    // 2) one warp per token: token t on CTA t % ncta, warp t / ncta
    int* cnt0 = cluster.map_shared_rank(s_cnt, 0);
    int* hits0 = cluster.map_shared_rank(s_hits, 0);
    float* mass0 = cluster.map_shared_rank(s_mass, 0);
    for (int t = rank + ncta * warp; t < N; t += ncta * kFusedRouteWarps) {
        if (rp.y_acc != nullptr) {
            float4* yv = reinterpret_cast<float4*>(rp.y_acc + static_cast<int64_t>(t) * H);
            for (int i = lane; i < H / 4; i += 32) yv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        int mine_e;
        float mine_w, mine_a, shared_extra;
        select_from_logits<T, EPL>(rp, t, lane, [&](int e) {
            // every remote load issued before the in-order adds (C <= 32 chunks)
            float r[kFusedRouteMaxChunks];
#pragma unroll
            for (int c = 0; c < kFusedRouteMaxChunks; ++c)
                r[c] = c < C ? cluster.map_shared_rank(part, c % ncta)[(static_cast<size_t>(c / ncta) * N + t) * E + e]
                             : 0.0f;
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < kFusedRouteMaxChunks; ++c)
                if (c < C) s = s + r[c];
            if (rp.bias) s = s + rp.bias[e];
            return s;
        }, mine_e, mine_w, mine_a, shared_extra, rp.counts_all ? hits0 : nullptr,
            rp.mass_all ? mass0 : nullptr);
        if (lane < k) rp.pos[static_cast<int64_t>(t) * k + lane] = mine_a > 0.0f ? atomicAdd(&cnt0[mine_e], 1) : -1;
        if (lane == 0 && rp.num_shared > 0)
            rp.shared_coef[t] = (1.0f + shared_extra) / static_cast<float>(rp.num_shared);
        zero_direct_row<T>(rp, t, lane, mine_a);
    }
    __threadfence();
    cluster.sync();  // every selection, position and count is in place
    if (rank != 0) return;

    // 3) CTA 0: statistics, plan, slot tables
    for (int e = tid; e < E; e += kFusedRouteThreads) {
        if (rp.counts_all) rp.counts_all[e] = s_hits[e];
        if (rp.mass_all) rp.mass_all[e] = s_mass[e];
    }
    const int cnt = tid < pp.e ? s_cnt[tid] : 0;
    const int inc = block_inclusive_scan<kFusedRouteThreads>(cnt, s_scratch);
    if (tid < pp.e) s_off[tid] = inc - cnt;
    plan_tables<kFusedRouteThreads>(pp, cnt, inc, s_scratch, s_tot);
    __syncthreads();
    const int64_t total = static_cast<int64_t>(N) * k;
    for (int64_t i = tid; i < total; i += kFusedRouteThreads) {
        const int64_t tt = i / k;
        const int j = static_cast<int>(i % k);
        const int ps = __ldcg(rp.pos + i);
        const int e = __ldcg(rp.topk_idx + i);
        const float c = __ldcg(rp.sel_coef + i);
        if (j == 0 && sp.num_shared > 0) {
            const float sc = __ldcg(rp.shared_coef + tt);
            for (int q = 0; q < sp.num_shared; ++q) {
                const int64_t slot = sp.n * k + q * sp.n + tt;
                sp.slot_tok[slot] = static_cast<int32_t>(tt);
                sp.slot_coef[slot] = sc;
            }
        }
        if (ps < 0) continue;
        const int64_t slot = static_cast<int64_t>(s_off[e]) + ps;
        sp.slot_tok[slot] = static_cast<int32_t>(tt);
        sp.slot_coef[slot] = c;
        if (sp.slot_map != nullptr) sp.slot_map[static_cast<int64_t>(e) * sp.n + tt] = static_cast<int32_t>(slot);
    }
}

}  // namespace chronos
