// plan.cuh — token-to-expert permutation and the small elementwise kernels.
//
// Replaces the reference's per-expert host loop (moe_chronos.py:149-154 and
// :207-262: `(topk_idx == i)`, `.nonzero()`, `x_flat[token_idx]`, with one or
// two host syncs per expert) by three device steps:
//   plan    one block: exclusive scan of the expert-group sizes into slot
//           offsets, the list of active groups (routed experts with at least
//           one available selection, then the shared experts) and the
//           per-group tile counts the persistent GEMMs walk;
//   scatter one warp per (token, choice): slot = offset[e] + position,
//           slot -> (token, w*a), and the x row copied into the expert-sorted
//           buffer with 16-byte loads/stores;
//   finalize fp32 accumulator -> output dtype.
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace chronos {

// Written by plan_kernel, read by every later kernel of the call.
struct PlanHeader {
    int32_t num_active;      // active groups
    int32_t routed_rows;     // routed slots in use (<= N*k)
    int32_t units_gu;        // work units of the gate/up GEMM
    int32_t units_dn;        // work units of the down GEMM
    int32_t max_rows;        // largest group
    int32_t dn_done;         // down GEMM CTAs whose routed units are complete (shared-last mode)
    int32_t pad[2];
};

struct PlanParams {
    int64_t n;
    int e, k, num_shared;
    int tok_tile;                 // token rows per gate/up GEMM tile
    int tok_tile_dn;              // token rows per down GEMM tile
    int mt_gu, mt_dn;             // weight-row tiles per group (gate/up, down)
    int splits_dn;                // K splits per down tile
    int shared_fin;               // shared experts run last in the down GEMM, merged (no down units here)
    const int32_t* grp_count;     // [E]
    const int32_t* slot_of_expert;  // [E] or null
    PlanHeader* hdr;
    int32_t* grp_off;             // [E] first slot of routed group e
    // active groups, [E + S_h] each (+1 for the unit prefix arrays)
    int32_t* act_rows;
    int32_t* act_xrow;   // first row of the group's token rows in its B source
    int32_t* act_hrow;   // first row of the group in the hidden buffer
    int32_t* act_wslot;  // weight slot (routed pool slot, or shared index)
    int32_t* act_eid;    // routed expert id, or -1 for a shared group
    int32_t* ustart_gu;  // [A + 1]
    int32_t* ustart_dn;  // [A + 1]
    int32_t* tile_cnt;   // [n_tile_cnt] down output-tile counters (folded finalize), zeroed here; or null
    int n_tile_cnt;
    int splits_gu;       // K splits of a routed gate/up tile (decode, dense mode); shared tiles whole
    int32_t* gu_cnt;     // [n_gu_cnt] routed gate/up tile arrival counters, zeroed here; or null
    int n_gu_cnt;
};

constexpr int kPlanThreads = 256;  // >= the 256 experts the ABI accepts: one expert per thread

// Inclusive scan over the block (NT values, NT = blockDim.x), warp shuffles +
// one pass over the warp totals.  `scratch` holds NT / 32 ints.
template <int NT = kPlanThreads>
__device__ __forceinline__ int block_inclusive_scan(int v, int* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int s = lane < NT / 32 ? scratch[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += n;
        }
        if (lane < NT / 32) scratch[lane] = s;
    }
    __syncthreads();
    if (warp > 0) v += scratch[warp - 1];
    __syncthreads();
    return v;
}

// The plan tables (active groups, unit prefixes, header); called by one block
// of NT threads.  `cnt` / `inc_cnt`: this thread's expert group size and its
// inclusive scan.
template <int NT = kPlanThreads>
__device__ __forceinline__ void plan_tables(const PlanParams& p, int cnt, int inc_cnt, int* s_scratch,
                                            int* s_tot) {
    const int tid = threadIdx.x;
    const int E = p.e;
    const int S = p.num_shared;
    const int N = static_cast<int>(p.n);
    const int is_act = (tid < E && cnt > 0) ? 1 : 0;
    const int tt = (cnt + p.tok_tile - 1) / p.tok_tile;
    const int tt_dn = (cnt + p.tok_tile_dn - 1) / p.tok_tile_dn;
    const int ugu = is_act ? tt * p.mt_gu * (p.splits_gu > 1 ? p.splits_gu : 1) : 0;
    const int udn = is_act ? tt_dn * p.mt_dn * p.splits_dn : 0;
    const int inc_act = block_inclusive_scan<NT>(is_act, s_scratch);
    const int inc_gu = block_inclusive_scan<NT>(ugu, s_scratch);
    const int inc_dn = block_inclusive_scan<NT>(udn, s_scratch);
    if (tid == NT - 1) {
        s_tot[0] = inc_cnt;
        s_tot[1] = inc_act;
        s_tot[2] = inc_gu;
        s_tot[3] = inc_dn;
    }
    __syncthreads();
    // shared groups first (the largest: N rows each), then routed groups in expert order
    const int tt_sh = (N + p.tok_tile - 1) / p.tok_tile;
    const int tt_sh_dn = (N + p.tok_tile_dn - 1) / p.tok_tile_dn;
    const int sh_gu = tt_sh * p.mt_gu;
    const int sh_dn = p.shared_fin ? 0 : tt_sh_dn * p.mt_dn * p.splits_dn;
    if (tid < E) {
        const int off = inc_cnt - cnt;
        p.grp_off[tid] = off;
        if (is_act) {
            const int a = S + inc_act - 1;
            p.act_rows[a] = cnt;
            p.act_xrow[a] = off;
            p.act_hrow[a] = off;
            p.act_wslot[a] = p.slot_of_expert ? p.slot_of_expert[tid] : tid;
            p.act_eid[a] = tid;
            p.ustart_gu[a] = S * sh_gu + inc_gu - ugu;
            p.ustart_dn[a] = S * sh_dn + inc_dn - udn;
        }
    }
    for (int i = tid; i < p.n_tile_cnt; i += NT) p.tile_cnt[i] = 0;
    for (int i = tid; i < p.n_gu_cnt; i += NT) p.gu_cnt[i] = 0;
    if (tid < S) {
        p.act_rows[tid] = N;
        p.act_xrow[tid] = 0;
        p.act_hrow[tid] = N * p.k + tid * N;
        p.act_wslot[tid] = tid;
        p.act_eid[tid] = -1;
        p.ustart_gu[tid] = tid * sh_gu;
        p.ustart_dn[tid] = tid * sh_dn;
    }
    if (tid == 0) {
        const int A = S + s_tot[1];
        const int tot_gu = S * sh_gu + s_tot[2];
        const int tot_dn = S * sh_dn + s_tot[3];
        p.ustart_gu[A] = tot_gu;
        p.ustart_dn[A] = tot_dn;
        p.hdr->num_active = A;
        p.hdr->routed_rows = s_tot[0];
        p.hdr->units_gu = tot_gu;
        p.hdr->units_dn = tot_dn;
        p.hdr->max_rows = S > 0 ? N : 0;
        p.hdr->dn_done = 0;
    }
}

struct ScatterParams {
    const void* x;
    int64_t n;
    int h, k, num_shared;
    const int32_t* topk_idx;
    const int32_t* pos;
    const float* sel_coef;
    const float* shared_coef;
    const int32_t* grp_off;
    void* xp;             // [N*k, H] expert-sorted copies of x rows
    int32_t* slot_tok;    // [N*k + S*N]
    float* slot_coef;     // [N*k + S*N]
    int copy_rows;        // 0: only the slot tables (B operand read from x by row index)
    int32_t* slot_map;    // decode batches: [E, N] slot of (expert, token) or -1
    int e;                // experts (rows of slot_map)
    int32_t* pair_slot;   // [N, k] slot of (token, choice), -1 if unavailable; or null
};

constexpr int kScatterThreads = kPlanThreads;
constexpr int kScatterWarps = kScatterThreads / 32;

// Plan + permutation in one launch.  Every block scans the E group sizes
// itself (E <= 256 values) to get the group offsets; block 0 also writes the
// plan tables the GEMMs walk.  Then one warp per (token, choice) writes the
// slot tables and copies the x row into expert order (all of a lane's 16-byte
// loads issued before its stores).  Warps with choice index 0 also fill the
// shared experts' slot tables.
template <typename T>
__global__ void __launch_bounds__(kScatterThreads) plan_scatter_kernel(PlanParams pp, ScatterParams p) {
    __shared__ int s_scratch[kPlanThreads / 32];
    __shared__ int s_tot[4];
    __shared__ int s_off[kPlanThreads];
    const int tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();  // routing results
    const int cnt = tid < pp.e ? pp.grp_count[tid] : 0;
    const int inc_cnt = block_inclusive_scan(cnt, s_scratch);
    s_off[tid] = inc_cnt - cnt;
    if (blockIdx.x == 0) plan_tables(pp, cnt, inc_cnt, s_scratch, s_tot);
    __syncthreads();

    const int64_t gw = static_cast<int64_t>(blockIdx.x) * kScatterWarps + (tid >> 5);
    const int lane = tid & 31;
    const int64_t total = p.n * p.k;
    if (gw >= total) return;
    const int64_t t = gw / p.k;
    const int j = static_cast<int>(gw % p.k);
    if (j == 0 && lane < p.num_shared) {
        const int64_t s = p.n * p.k + lane * p.n + t;
        p.slot_tok[s] = static_cast<int32_t>(t);
        p.slot_coef[s] = p.shared_coef[t];
    }
    const int ps = p.pos[gw];
    if (ps < 0) {
        if (lane == 0 && p.pair_slot != nullptr) p.pair_slot[gw] = -1;
        return;
    }
    const int e = p.topk_idx[gw];
    const int64_t slot = static_cast<int64_t>(s_off[e]) + ps;
    if (lane == 0) {
        p.slot_tok[slot] = static_cast<int32_t>(t);
        p.slot_coef[slot] = p.sel_coef[gw];
        if (p.pair_slot != nullptr) p.pair_slot[gw] = static_cast<int32_t>(slot);
    }
    if (!p.copy_rows) return;
    const T* src = static_cast<const T*>(p.x) + t * p.h;
    T* dst = static_cast<T*>(p.xp) + slot * p.h;
    const int bytes = p.h * static_cast<int>(sizeof(T));
    if ((bytes & 15) == 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        const int n16 = bytes / 16;
        int i = lane;
        for (; i + 32 * 7 < n16; i += 32 * 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = s4[i + 32 * u];
#pragma unroll
            for (int u = 0; u < 8; ++u) d4[i + 32 * u] = v[u];
        }
        for (; i < n16; i += 32) d4[i] = s4[i];
    } else {
        for (int i = lane; i < p.h; i += 32) dst[i] = src[i];
    }
}

// Decode batches (<= kSelectPlanMaxTokens tokens): routing selection, plan and
// slot tables in ONE launch.  One warp per token selects (blocks of 8 tokens,
// so a 64-token batch selects on 8 SMs), a global atomic gives each available
// selection its position in its expert group, and the last block to finish
// (a ticket counter, zeroed with the group counters) scans the group sizes and
// writes the plan and slot tables plus the (expert, token) -> slot map.
// Nothing is copied: the gate/up GEMM reads the token rows of x itself.
// Replaces the select + plan/scatter launches of larger batches.
constexpr int kSelectPlanThreads = kPlanThreads;
constexpr int kSelectPlanWarps = kSelectPlanThreads / 32;
constexpr int kSelectPlanMaxTokens = 64;
constexpr int kSelectPlanWideThreads = 1024;   // one block, one warp per token, up to 32 tokens

template <typename T, int EPL, int NT = kSelectPlanThreads>
__global__ void __launch_bounds__(NT)
    route_select_plan_kernel(RouteParams rp, PlanParams pp, ScatterParams sp, int32_t* ticket) {
    __shared__ int s_off[kMaxExperts];
    __shared__ int s_scratch[(NT / 32)];
    __shared__ int s_tot[4];
    __shared__ int s_last;
    // one block (<= NT / 32 tokens): group counts by shared-memory atomics and the
    // per-(token, choice) results kept in shared memory, no ticket or re-reads
    constexpr int kPairs = (NT / 32) * kMaxTopK;
    __shared__ int s_cnt[kMaxExperts];
    __shared__ int s_pe[kPairs];
    __shared__ int s_pp[kPairs];
    __shared__ float s_pc[kPairs];
    __shared__ float s_sc[(NT / 32)];
    const bool single = gridDim.x == 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t gtid = static_cast<int64_t>(blockIdx.x) * NT + tid;
    const int64_t gthreads = static_cast<int64_t>(gridDim.x) * NT;
    pdl_trigger();
    if (sp.slot_map != nullptr)
        for (int64_t i = gtid; i < static_cast<int64_t>(sp.e) * sp.n; i += gthreads) sp.slot_map[i] = -1;
    if (single) {
        for (int i = tid; i < kMaxExperts; i += NT) s_cnt[i] = 0;
        __syncthreads();
    }
    pdl_wait();  // chunk partials and zeroed counters from the logit kernel

    // 1) one warp per token: select, position within the expert group
    const int k = rp.k;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * (NT / 32) + warp;
    if (t < rp.n) {
        if (rp.y_acc != nullptr) {
            float4* yv = reinterpret_cast<float4*>(rp.y_acc + t * rp.h);
            for (int i = lane; i < rp.h / 4; i += 32) yv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        int mine_e;
        float mine_w, mine_a, shared_extra;
        select_token<T, EPL>(rp, t, lane, mine_e, mine_w, mine_a, shared_extra);
        if (lane < k) {
            const int ps = mine_a > 0.0f ? atomicAdd(single ? &s_cnt[mine_e] : &rp.grp_count[mine_e], 1) : -1;
            rp.pos[t * k + lane] = ps;
            if (single) {
                s_pe[warp * k + lane] = mine_e;
                s_pp[warp * k + lane] = ps;
                s_pc[warp * k + lane] = mine_w * mine_a;
            }
        }
        const float sc = (1.0f + shared_extra) / static_cast<float>(rp.num_shared > 0 ? rp.num_shared : 1);
        if (lane == 0 && rp.num_shared > 0) {
            rp.shared_coef[t] = sc;
            if (single) s_sc[warp] = sc;
        }
        zero_direct_row<T>(rp, t, lane, mine_a);
    }

    // 2) several blocks: the last to arrive sees every block's counts and tables
    if (single) {
        __syncthreads();
    } else {
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
    }

    // 3) plan: group offsets and the GEMM work tables
    const int cnt = tid < pp.e ? (single ? s_cnt[tid] : __ldcg(rp.grp_count + tid)) : 0;
    const int inc = block_inclusive_scan<NT>(cnt, s_scratch);
    if (tid < pp.e) s_off[tid] = inc - cnt;
    plan_tables<NT>(pp, cnt, inc, s_scratch, s_tot);
    __syncthreads();

    // 4) slot tables, one thread per (token, choice)
    const int64_t total = rp.n * k;
    for (int64_t i = tid; i < total; i += NT) {
        const int64_t tt = i / k;
        const int j = static_cast<int>(i % k);
        const int ps = single ? s_pp[i] : __ldcg(rp.pos + i);
        const int e = single ? s_pe[i] : __ldcg(rp.topk_idx + i);
        const float c = single ? s_pc[i] : __ldcg(rp.sel_coef + i);
        if (j == 0 && sp.num_shared > 0) {
            const float sc = single ? s_sc[tt] : __ldcg(rp.shared_coef + tt);
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

template <typename T>
__global__ void finalize_kernel(const float* __restrict__ y_acc, T* __restrict__ y, int64_t count4) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(y_acc)[i];
        T* d = y + 4 * i;
        d[0] = from_f32<T>(v.x);
        d[1] = from_f32<T>(v.y);
        d[2] = from_f32<T>(v.z);
        d[3] = from_f32<T>(v.w);
    }
}

}  // namespace chronos
