// gemm_tc.cuh — persistent grouped expert GEMMs on tcgen05 / TMEM, fed by TMA.
//
// One kernel template serves both halves of the expert SwiGLU
// (minimind FeedForward, restated at chronos/mlx/moe.py:13-23):
//
//   GATEUP: for every active group (routed expert or shared expert) and every
//           tile of 128 rows of its gate/up weights x BN token rows,
//             G = W_gate[rows] . X^T,  U = W_up[rows] . X^T   (two MMAs, one
//           shared B tile), epilogue h[token][f] = silu(G) * U in the input
//           dtype;
//   DOWN:   D = W_down[rows] . h^T, epilogue y_acc[token][n] += coef * D with
//           coef = w * a for routed slots and (1 + sum w (1-a)) / S_h for
//           shared slots — the availability blend and the weighted combine of
//           moe_chronos.py:255-268 fused into the GEMM.
//
// Orientation: weights are the M = 128 operand (A), tokens the N = BN operand
// (B), so decode batches of 1..64 tokens use narrow N tiles instead of padding
// M.  Both operands are K-major bf16/fp16 tiles of 64 elements (128 B, one
// 128-byte swizzle atom) staged by TMA into an STAGES-deep shared-memory ring.
//
// Warp roles (192 threads, one CTA per SM, persistent over the work units):
//   warp 0      TMA producer (one thread)
//   warp 1      TMEM allocator + MMA issuer (one thread)
//   warps 2..5  epilogue: tcgen05.ld of the accumulator rows, math, stores
// The accumulator is double-buffered in TMEM so the epilogue of one unit
// overlaps the MMAs of the next.  Every wait is bounded (globaltimer) and
// reports CHRONOS_ERR_PIPELINE_TIMEOUT instead of hanging.
#pragma once

#include "common.cuh"
#include "plan.cuh"

namespace chronos {

constexpr int kTcThreads = 192;
constexpr int kTcBM = 128;  // weight rows per tile (MMA M)
constexpr int kTcBK = 64;   // K per pipeline stage (one 128-byte swizzle atom)
constexpr uint64_t kPipelineLimitNs = 4000000000ull;

struct TcGemmParams {
    const PlanHeader* hdr;
    const int32_t* act_rows;
    const int32_t* act_xrow;
    const int32_t* act_hrow;
    const int32_t* act_wslot;
    const int32_t* act_eid;
    const int32_t* ustart;
    int k_tiles;       // K / 64
    int kt_per_split;  // k tiles per split
    int m_tiles;       // weight-row tiles per group
    int w_rows;        // weight rows per slot (F for gate/up, H for down)
    int out_cols;      // F (gate/up) or H (down)
    int f, h;
    void* hid;               // GATEUP: [slots, F]
    float* y_acc;            // DOWN: [N, H]
    const int32_t* slot_tok;
    const float* slot_coef;
    const int32_t* ready_flags;
    int32_t ready_epoch;
    uint64_t ready_limit_ns;
    int32_t* status;
    // DENSE gate/up (decode batches, N <= BN): slot of (expert, token), -1 if
    // the token did not choose the expert (or it is unavailable); [E, n_tokens]
    const int32_t* slot_map;
    int64_t n_tokens;
    // DOWN, one contribution per token (k = 1, no shared experts): rows of
    // coef * D stored straight into the output [N, H] (x dtype) instead of
    // reduce-added into y_acc; null otherwise
    void* y_direct;
    // DOWN, shared experts last (sf_shared = S_h > 0): after the routed units
    // (units_dn of them) come the shared units, one per (128 output columns,
    // BN tokens), each a K = S_h * F product over the S_h shared experts'
    // hidden rows (sh_hrow + s * n_tokens + token).  Their epilogue waits until
    // every CTA with routed units has counted itself in *dn_done, then writes
    // y_out = y_acc + shared_coef * D in the output dtype: the finalize pass
    // and the shared experts' reduce-adds are folded in.
    int sf_shared;
    int64_t sh_hrow;
    int32_t* dn_done;
    void* y_out;
    // DENSE gate/up (decode): the first pre_units units are the shared experts'
    // (S_h x m_tiles, one token tile each), run before this call's plan exists;
    // their hidden rows start at sh_hrow + s * n_tokens
    int pre_units;
    // Token-major down, two-phase combine (shared-last mode, large batches):
    // routed units STORE coef * D rounded to the layer dtype into ys[slot]
    // ([slots, H], no fp32 reduce-adds, no accumulator); the shared units then
    // write y = sum_j ys[pair_slot[t, j]] (j ascending, fp32) + shared_coef * D.
    // Null: routed units reduce-add into y_acc.
    void* ys;
    const int32_t* pair_slot;  // [n_tokens, k_pairs], -1 = no contribution
    int k_pairs;
    // Weight-major down (decode), finalize folded in: when a unit's reduce-adds
    // into output-column tile m are complete, its CTA counts them in
    // tile_cnt[m]; the CTA whose count completes the tile (units_dn / m_tiles
    // units) writes that tile of y_fold = y_acc in the output dtype.  Null: a
    // finalize kernel follows.
    int32_t* tile_cnt;
    void* y_fold;
    // Dense gate/up, routed units split along K (gu_splits > 1): each split
    // writes its fp32 G and U columns of the call's tokens to
    // gu_part[tile][split][G, U][token][128], counts itself in gu_cnt[tile]
    // (tile = (group - num_shared) * m_tiles + weight-row tile, zeroed by the
    // plan), and the split completing the tile sums the partials in split
    // order and writes silu(G) * U.
    int gu_splits;
    int num_shared;
    int32_t* gu_cnt;
    float* gu_part;
    // Dense gate/up, batches that select nearly every expert: before waiting for
    // the plan, a CTA past the shared units prefetches into L2 the first spec_kt
    // k tiles of the routed unit it would run first if all spec_experts experts
    // (weight slot = expert id) were active.  A hint: a wrong guess only moves
    // bytes while the HBM is otherwise idle.  0: no prefetch.
    // spec_avail (null: every expert available): the call's availability input;
    // experts with spec_avail[e] <= 0 form no group, so the guess skips them.
    int spec_kt;
    int spec_experts;
    const float* spec_avail;
};

__host__ __device__ constexpr int tc_stage_bytes(int bn, bool gateup) {
    return kTcBM * kTcBK * 2 * (gateup ? 2 : 1) + bn * kTcBK * 2;
}
// Epilogue staging: one output row per token of the tile, written to global
// memory by per-token bulk copies (h rows: 128 bf16; down: 128 fp32 to reduce
// into the accumulator, or 128 output elements stored directly).
__host__ __device__ constexpr int tc_stage_row_bytes(bool gateup) {
    return gateup ? kTcBM * 2 : kTcBM * 4;
}
// Dynamic shared memory of one CTA: the per-CTA limit (227 KB) minus the
// 1024-byte alignment slack, the barriers (256 B) and the per-unit slot tables.
__host__ __device__ constexpr int tc_ring_budget(int bn) { return 232448 - 1024 - 256 - 4 * bn * 4; }
// At most kTcMaxStages stages: the barrier block (256 B) holds 2 * stages + 5
// mbarriers and the CTA's flag words.
constexpr int kTcMaxStages = 8;
__host__ __device__ constexpr int tc_stages_with(int bn, bool gateup, int sub) {
    return (tc_ring_budget(bn) - sub * tc_stage_row_bytes(gateup)) / tc_stage_bytes(bn, gateup) > kTcMaxStages
               ? kTcMaxStages
               : (tc_ring_budget(bn) - sub * tc_stage_row_bytes(gateup)) / tc_stage_bytes(bn, gateup);
}
// Rows staged at a time.  Gate/up: the most (128, 64, 32 or 16, at most BN)
// that still leaves the TMA ring as many stages as the smallest staging would
// (a 128-token tile stages 64 rows: 4 stages instead of 3).  Down: up to 128
// rows; its fp32 rows are drained by reductions, and draining a 256-token tile
// in smaller pieces measured slower than the extra stage gains.
__host__ __device__ constexpr int tc_staging_rows(int bn, bool gateup) {
    return !gateup ? (bn < 128 ? bn : 128)
           : (bn >= 128 && tc_stages_with(bn, gateup, 128) >= tc_stages_with(bn, gateup, 16)) ? 128
           : (bn >= 64 && tc_stages_with(bn, gateup, 64) >= tc_stages_with(bn, gateup, 16))   ? 64
           : (bn >= 32 && tc_stages_with(bn, gateup, 32) >= tc_stages_with(bn, gateup, 16))   ? 32
                                                                                                 : 16;
}
__host__ __device__ constexpr int tc_staging_bytes(int bn, bool gateup) {
    return tc_staging_rows(bn, gateup) * tc_stage_row_bytes(gateup);
}
__host__ __device__ constexpr int tc_stages(int bn, bool gateup) {
    return tc_stages_with(bn, gateup, tc_staging_rows(bn, gateup));
}
__host__ __device__ constexpr int tc_tmem_cols(int bn, bool gateup) {
    // two accumulator buffers of (gateup ? 2 : 1) * bn fp32 columns, power of two >= 32
    return (2 * bn * (gateup ? 2 : 1)) <= 32    ? 32
           : (2 * bn * (gateup ? 2 : 1)) <= 64  ? 64
           : (2 * bn * (gateup ? 2 : 1)) <= 128 ? 128
           : (2 * bn * (gateup ? 2 : 1)) <= 256 ? 256
                                                 : 512;
}
__host__ __device__ constexpr int tc_smem_bytes(int bn, bool gateup) {
    return 1024 /* alignment slack */ + tc_stages(bn, gateup) * tc_stage_bytes(bn, gateup) +
           tc_staging_bytes(bn, gateup) + 4 * bn * 4 /* per-unit slot tables x2 */ + 256;
}

struct TcUnit {
    int a, tok_tile, mtile, split;
};

__device__ __forceinline__ TcUnit tc_decode(const TcGemmParams& p, int num_active, int u, int bn,
                                           int splits) {
    int lo = 0, hi = num_active - 1;
    while (lo < hi) {  // largest a with ustart[a] <= u
        const int mid = (lo + hi + 1) >> 1;
        if (p.ustart[mid] <= u) lo = mid; else hi = mid - 1;
    }
    TcUnit r;
    r.a = lo;
    int rem = u - p.ustart[lo];
    const int tt = (p.act_rows[lo] + bn - 1) / bn;
    r.tok_tile = rem % tt;
    rem /= tt;
    r.mtile = rem % p.m_tiles;
    r.split = rem / p.m_tiles;
    (void)splits;
    return r;
}

// Group of unit u for a warp whose previous unit was in group `a`: a CTA visits
// its units in increasing order, so the 32 lanes test the next 32 group starts
// at once (one memory round trip for most units instead of a binary search's
// chain).  Every lane of the warp must call it; all get the same result.
__device__ __forceinline__ int tc_group_warp(const TcGemmParams& p, int num_active, int a, int u, int lane) {
    while (true) {
        const int cand = a + 1 + lane;
        const bool ok = cand < num_active && p.ustart[cand] <= u;
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        if (m == 0u) return a;
        a += 32 - __clz(m);  // highest passing lane (group starts are increasing)
        if (m != 0xffffffffu) return a;
    }
}

// Unit u of group a: token tile, weight-row tile and K split.
__device__ __forceinline__ TcUnit tc_unit_at(const TcGemmParams& p, int a, int u, int bn) {
    TcUnit r;
    r.a = a;
    int rem = u - p.ustart[a];
    const int tt = (p.act_rows[a] + bn - 1) / bn;
    r.tok_tile = rem % tt;
    rem /= tt;
    r.mtile = rem % p.m_tiles;
    r.split = rem / p.m_tiles;
    return r;
}

// Shared-last down GEMM: an epilogue's routed reduce-adds are complete; count
// its CTA in (all 128 epilogue threads call this together).
__device__ __forceinline__ void tc_count_routed_done(int32_t* counter, int et) {
    bulk_wait_all();
    fence_proxy_async_global();
    epilogue_bar_sync(128);
    if (et == 0) {
        __threadfence();
        red_release_add_s32(counter, 1);
    }
}

template <typename T, int BN, bool GATEUP, bool DENSE = false>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_grouped_gemm(const __grid_constant__ CUtensorMap tm_a0r,  // routed gate (or down)
                    const __grid_constant__ CUtensorMap tm_a1r,  // routed up
                    const __grid_constant__ CUtensorMap tm_a0s,  // shared gate (or down)
                    const __grid_constant__ CUtensorMap tm_a1s,  // shared up
                    const __grid_constant__ CUtensorMap tm_br,   // routed token rows (Xp or h)
                    const __grid_constant__ CUtensorMap tm_bs,   // shared token rows (x or h)
                    TcGemmParams p) {
    constexpr int A_BYTES = kTcBM * kTcBK * 2;
    constexpr int B_BYTES = BN * kTcBK * 2;
    constexpr int STAGE_BYTES = tc_stage_bytes(BN, GATEUP);
    constexpr int STAGES = tc_stages(BN, GATEUP);
    constexpr int ROW_BYTES = tc_stage_row_bytes(GATEUP);
    constexpr int ACC_COLS = GATEUP ? 2 * BN : BN;
    constexpr int TMEM_COLS = tc_tmem_cols(BN, GATEUP);
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N must be a multiple of 16");
    static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0,
                  "operand tiles must keep the 1024-byte alignment of the 128-B swizzle atoms");
    static_assert(2 * ACC_COLS <= 512, "two accumulator buffers must fit in TMEM");
    static_assert(STAGES >= 2, "shared memory holds fewer than two pipeline stages");
    static_assert(tc_smem_bytes(BN, GATEUP) <= 232448, "shared memory over the per-CTA limit");
    static_assert((2 * STAGES + 5) * 8 + 20 <= 256, "barriers and flag words over their 256 bytes");

    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* staging = smem + STAGES * STAGE_BYTES;  // [tc_staging_rows(BN, GATEUP)][ROW_BYTES]
    // per-unit slot tables of the tile (coefficient, token), double-buffered by accumulator
    float* s_coef = reinterpret_cast<float*>(staging + tc_staging_rows(BN, GATEUP) * ROW_BYTES);  // [2][BN]
    int32_t* s_tok = reinterpret_cast<int32_t*>(s_coef + 2 * BN);                          // [2][BN]
    uint64_t* full = reinterpret_cast<uint64_t*>(s_tok + 2 * BN);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* ybar = tempty + 2;  // shared-last units: accumulator rows landed in staging
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ybar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        mbar_init(ybar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_a0r);
        prefetch_tmap(&tm_br);
        prefetch_tmap(&tm_a0s);
        prefetch_tmap(&tm_bs);
        if (GATEUP) {
            prefetch_tmap(&tm_a1r);
            prefetch_tmap(&tm_a1s);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    // Decode gate/up: the shared experts' units come first in the unit order and
    // their tables follow from the shape, so they run before this call's plan
    // exists (while the routing kernels are still running).  Everything else
    // waits for the earlier kernels of the call before reading the plan.
    const int pre_units = (GATEUP && DENSE) ? p.pre_units : 0;
    int num_active = 0, total_main = 0, sf_tt = 0, total = 0;
    bool planned = false;
    auto load_plan = [&]() {
        pdl_wait();
        num_active = p.hdr->num_active;
        total_main = GATEUP ? p.hdr->units_gu : p.hdr->units_dn;
        // shared-last units of the down GEMM: (output column tile, token tile) pairs after the routed ones
        sf_tt = (!GATEUP && p.sf_shared > 0) ? static_cast<int>((p.n_tokens + BN - 1) / BN) : 0;
        total = total_main + sf_tt * p.m_tiles;
        planned = true;
    };
    if (pre_units == 0) load_plan();
    const int splits_unused = 0;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        // the warp decodes the units, lane 0 issues the waits and the copies
        int stage = 0;
        uint32_t phase = 0;
        int polled_eid = -1;
        int ga = 0;
        // decode tiles (one token tile per group): weights streamed once, evict first
        constexpr bool kStreamA = BN <= 64;
        const uint64_t pol_a = kStreamA ? l2_evict_first_policy() : 0ull;
        if constexpr (GATEUP && DENSE) {
            if (p.spec_kt > 0 && static_cast<int>(blockIdx.x) >= pre_units) {
                // routed unit r = blockIdx.x - pre_units is weight-row tile r % m_tiles of
                // the (r / m_tiles)-th available expert when every available expert is
                // selected (groups in expert order)
                const int r = static_cast<int>(blockIdx.x) - pre_units;
                const int q = r / p.m_tiles;
                int e = q;
                if (p.spec_avail != nullptr) {
                    // the q-th expert with availability > 0: a warp scan over the input
                    e = -1;
                    int seen = 0;
                    for (int base = 0; base < p.spec_experts && e < 0; base += 32) {
                        const int ee = base + lane;
                        const uint32_t m =
                            __ballot_sync(0xffffffffu, ee < p.spec_experts && p.spec_avail[ee] > 0.0f);
                        const int c = __popc(m);
                        if (q < seen + c) {
                            uint32_t mm = m;
                            for (int i = 0; i < q - seen; ++i) mm &= mm - 1u;
                            e = base + __ffs(static_cast<int>(mm)) - 1;
                        }
                        seen += c;
                    }
                }
                if (lane == 0 && e >= 0 && e < p.spec_experts) {
                    const int a_row = e * p.w_rows + (r - q * p.m_tiles) * kTcBM;
                    for (int kt = 0; kt < p.spec_kt && kt < p.k_tiles; ++kt) {
                        tma_prefetch_2d(&tm_a0r, kt * kTcBK, a_row);
                        tma_prefetch_2d(&tm_a1r, kt * kTcBK, a_row);
                    }
                }
            }
        }
        for (int u = blockIdx.x;; u += gridDim.x) {
            if (u >= pre_units) {
                if (!planned) load_plan();
                if (u >= total) break;
            }
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            if constexpr (GATEUP && DENSE) {
                if (u < pre_units) {
                    // shared expert u / m_tiles, weight-row tile u % m_tiles; B = x rows [0, BN)
                    if (lane == 0) {
                        const int sx = u / p.m_tiles;
                        const int a_row = sx * p.w_rows + (u - sx * p.m_tiles) * kTcBM;
                        for (int kt = 0; kt < p.k_tiles; ++kt) {
                            if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                                *abort_flag = 1;
                                report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                                break;
                            }
                            uint8_t* sb = smem + stage * STAGE_BYTES;
                            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                            tma_load_2d_hint(sb, &tm_a0s, &full[stage], kt * kTcBK, a_row, pol_a);
                            tma_load_2d_hint(sb + A_BYTES, &tm_a1s, &full[stage], kt * kTcBK, a_row, pol_a);
                            tma_load_2d(sb + 2 * A_BYTES, &tm_bs, &full[stage], kt * kTcBK, 0);
                            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                        }
                    }
                    __syncwarp();
                    continue;
                }
            }
            if constexpr (!GATEUP) {
                if (u >= total_main) {
                    // shared-last unit: K runs over the S_h shared experts back to back
                    if (lane == 0) {
                        const int rem = u - total_main;
                        const int tok0 = (rem % sf_tt) * BN;
                        const int m0 = (rem / sf_tt) * kTcBM;
                        const int ktot = p.sf_shared * p.k_tiles;
                        for (int kt = 0; kt < ktot; ++kt) {
                            const int sx = kt / p.k_tiles;
                            const int kk = kt - sx * p.k_tiles;
                            if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                                *abort_flag = 1;
                                report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                                break;
                            }
                            uint8_t* sb = smem + stage * STAGE_BYTES;
                            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                            const int a_row = sx * p.w_rows + m0;
                            const int b_row = static_cast<int>(p.sh_hrow + sx * p.n_tokens) + tok0;
                            if constexpr (kStreamA)
                                tma_load_2d_hint(sb, &tm_a0s, &full[stage], kk * kTcBK, a_row, pol_a);
                            else
                                tma_load_2d(sb, &tm_a0s, &full[stage], kk * kTcBK, a_row);
                            tma_load_2d(sb + A_BYTES, &tm_br, &full[stage], kk * kTcBK, b_row);
                            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                        }
                    }
                    __syncwarp();
                    continue;
                }
            }
            ga = tc_group_warp(p, num_active, ga, u, lane);
            if (lane == 0) {
                const TcUnit w = tc_unit_at(p, ga, u, BN);
                const int eid = p.act_eid[w.a];
                const bool shared = eid < 0;
                if (!shared && p.ready_flags != nullptr && eid != polled_eid) {
                    // wait (bounded) for this selected expert's weights to be resident
                    const uint64_t t0 = globaltimer_ns();
                    bool ok = true;
                    while (ld_acquire_gpu(p.ready_flags + eid) < p.ready_epoch) {
                        if (globaltimer_ns() - t0 > p.ready_limit_ns) { ok = false; break; }
                        __nanosleep(256);
                    }
                    if (!ok) report_status(p.status, CHRONOS_ERR_EXPERT_NOT_READY);
                    fence_proxy_async_global();
                    polled_eid = eid;
                }
                const int a_row = p.act_wslot[w.a] * p.w_rows + w.mtile * kTcBM;
                const int b_row = (GATEUP ? p.act_xrow[w.a] : p.act_hrow[w.a]) + w.tok_tile * BN;
                const int kt0 = w.split * p.kt_per_split;
                const int kt1 = min(p.k_tiles, kt0 + p.kt_per_split);
                const CUtensorMap* ma0 = shared ? &tm_a0s : &tm_a0r;
                const CUtensorMap* ma1 = shared ? &tm_a1s : &tm_a1r;
                // DENSE: every group's B tile is x rows [0, BN) (all N <= BN tokens);
                // the epilogue keeps the columns of the tokens routed to the group
                const CUtensorMap* mb = ((GATEUP && shared) || DENSE) ? &tm_bs : &tm_br;
                const int b_row_eff = DENSE ? 0 : b_row;
                for (int kt = kt0; kt < kt1; ++kt) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        break;
                    }
                    uint8_t* sb = smem + stage * STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    if constexpr (kStreamA) {
                        // decode tiles: every weight tile is read once per call
                        tma_load_2d_hint(sb, ma0, &full[stage], kt * kTcBK, a_row, pol_a);
                        if (GATEUP) tma_load_2d_hint(sb + A_BYTES, ma1, &full[stage], kt * kTcBK, a_row, pol_a);
                    } else {
                        tma_load_2d(sb, ma0, &full[stage], kt * kTcBK, a_row);
                        if (GATEUP) tma_load_2d(sb + A_BYTES, ma1, &full[stage], kt * kTcBK, a_row);
                    }
                    tma_load_2d(sb + (GATEUP ? 2 : 1) * A_BYTES, mb, &full[stage], kt * kTcBK, b_row_eff);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------ MMA issuer ------------------------------
            constexpr uint32_t IDESC = idesc_f16(kTcBM, BN, AbFormat<T>::value);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            const bool unsplit = p.kt_per_split >= p.k_tiles;
            for (int u = blockIdx.x; !*abort_flag; u += gridDim.x) {
                if (u >= pre_units) {
                    if (!planned) load_plan();
                    if (u >= total) break;
                }
                // without K splits every unit spans the whole K: no unit decode on this path;
                // the dense gate/up's pre-plan (shared) units are never split
                const bool sfu = !GATEUP && u >= total_main;
                const bool pre = GATEUP && DENSE && u < pre_units;
                const int split =
                    (unsplit || sfu || pre) ? 0 : tc_decode(p, num_active, u, BN, splits_unused).split;
                const int kt0 = split * p.kt_per_split;
                const int kt1 = sfu   ? p.sf_shared * p.k_tiles
                                : pre ? p.k_tiles
                                      : min(p.k_tiles, kt0 + p.kt_per_split);
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
                const uint32_t d1 = d0 + BN;
                bool failed = false;
                for (int kt = kt0; kt < kt1; ++kt) {
                    if (!mbar_wait_bounded(&full[stage], phase, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa0 = smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t sa1 = sa0 + A_BYTES;
                    const uint32_t sbb = sa0 + (GATEUP ? 2 : 1) * A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 16; ++kk) {
                        const uint32_t accum = (kt > kt0 || kk > 0) ? 1u : 0u;
                        const uint64_t db = sdesc_k_sw128(sbb + kk * 32);
                        umma_f16(d0, sdesc_k_sw128(sa0 + kk * 32), db, IDESC, accum);
                        if (GATEUP) umma_f16(d1, sdesc_k_sw128(sa1 + kk * 32), db, IDESC, accum);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (failed) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        // Each unit: TMEM -> registers -> staging rows in shared memory (one row
        // per token, 128 output columns), then one bulk copy per valid token
        // row: a TMA reduce-add into the fp32 accumulator (down) or a plain
        // bulk store (gate/up hidden rows; down rows in direct-output mode).
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row_in_tile = q * 32 + lane;
        const int et = threadIdx.x - 64;  // 0..127 among the epilogue threads
        volatile int* ep_ok = abort_flag + 1;  // outcome of the accumulator wait, shared
        int acc = 0;
        uint32_t acc_phase = 0;
        int ga = 0;
        // shared-last mode: a CTA with routed units counts itself in once their
        // reduce-adds are complete; shared-last units wait until all such CTAs have
        const bool sf_count = !GATEUP && p.sf_shared > 0 && static_cast<int>(blockIdx.x) < total_main;
        const int sf_target = min(static_cast<int>(gridDim.x), total_main);
        bool sf_counted = false, sf_ready = false;
        uint32_t yphase = 0;
        // folded finalize: the output-column tile of the previous unit, counted in
        // once its reduce-adds are complete (one unit later: no wait on the newest)
        int fold_pending = -1;
        volatile int* fold_last = abort_flag + 2;
        volatile int* gu_last = abort_flag + 3;  // split gate/up: this CTA completed the tile
        auto fold_retire = [&](int tile) {
            fence_proxy_async_global();
            epilogue_bar_sync(128);
            if (et == 0) {
                __threadfence();
                const int done = atomicAdd(p.tile_cnt + tile, 1) + 1;
                const bool last = done == p.hdr->units_dn / p.m_tiles;
                if (last) __threadfence();
                *fold_last = last ? 1 : 0;
            }
            epilogue_bar_sync(128);
            if (*fold_last) {
                const int m0f = tile * kTcBM;
                const int ncf = min(kTcBM, p.out_cols - m0f);
                const int64_t cnt = p.n_tokens * ncf;
                for (int64_t i = et; i < cnt; i += 128) {
                    const int64_t t = i / ncf;
                    const int c = static_cast<int>(i - t * ncf);
                    static_cast<T*>(p.y_fold)[t * p.h + m0f + c] =
                        from_f32<T>(__ldcg(p.y_acc + t * p.h + m0f + c));
                }
            }
        };
        for (int u = blockIdx.x;; u += gridDim.x) {
            if (u >= pre_units) {
                if (!planned) load_plan();
                if (u >= total) break;
            }
            if constexpr (!GATEUP) {
                if (u >= total_main) {
                    // ---- shared-last unit: y_out = y_acc + shared_coef * D ----
                    if (sf_count && !sf_counted) {
                        tc_count_routed_done(p.dn_done, et);
                        sf_counted = true;
                    }
                    const int rem = u - total_main;
                    const int tok0 = (rem % sf_tt) * BN;
                    const int m0 = (rem / sf_tt) * kTcBM;
                    const int ncols = min(kTcBM, p.out_cols - m0);
                    float* cf = s_coef + acc * BN;
                    for (int r = et; r < BN; r += 128) {
                        const int64_t tok = tok0 + r;
                        cf[r] = tok < p.n_tokens ? p.slot_coef[p.sh_hrow + tok] : 0.0f;
                    }
                    if (et == 0) {
                        bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, kPipelineLimitNs, abort_flag);
                        if (ok && !sf_ready) {
                            // every routed contribution must be in the accumulator
                            const uint64_t t0 = globaltimer_ns();
                            while (ld_acquire_gpu(p.dn_done) < sf_target) {
                                if (*abort_flag || globaltimer_ns() - t0 > kPipelineLimitNs) {
                                    ok = false;
                                    break;
                                }
                                __nanosleep(64);
                            }
                        }
                        if (!ok) {
                            *abort_flag = 1;
                            report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        }
                        *ep_ok = ok ? 1 : 0;
                    }
                    sf_ready = true;
                    bulk_wait_read();
                    epilogue_bar_sync(128);
                    if (!*ep_ok) break;
                    tc_fence_after();
                    fence_proxy_async_global();  // accumulator rows are read by bulk copies below
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                           static_cast<uint32_t>(acc * ACC_COLS);
                    constexpr int SUB = tc_staging_rows(BN, GATEUP);
                    constexpr int ROW_F = ROW_BYTES / 4;
                    const float* ys = reinterpret_cast<const float*>(staging);
    #pragma unroll 1
                    for (int c0 = 0; c0 < BN; c0 += SUB) {
                        const int64_t left = p.n_tokens - (tok0 + c0);
                        const int nrows = left < SUB ? static_cast<int>(left) : SUB;
                        if (nrows <= 0) break;
                        const bool last = c0 + SUB >= BN || tok0 + c0 + SUB >= p.n_tokens;
                        if (c0 > 0) bulk_wait_read();
                        if (et == 0) mbar_arrive_expect_tx(ybar, static_cast<uint32_t>(nrows * ncols * 4));
                        epilogue_bar_sync(128);
                        // the SUB accumulator rows of these tokens -> staging (fp32)
                        if (et < nrows)
                            bulk_load(staging + et * ROW_BYTES, p.y_acc + (tok0 + c0 + et) * p.h + m0,
                                      static_cast<uint32_t>(ncols * 4), ybar);
                        if (!mbar_wait_bounded(ybar, yphase, kPipelineLimitNs, abort_flag)) {
                            *abort_flag = 1;
                            report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        }
                        yphase ^= 1u;
    #pragma unroll 1
                        for (int c = c0; c < c0 + SUB; c += 16) {
                            float g[16];
                            tmem_ld16(taddr + c, g);
                            tmem_wait_ld();
                            float yv[16];
    #pragma unroll
                            for (int j = 0; j < 16; ++j) yv[j] = ys[(c - c0 + j) * ROW_F + row_in_tile];
                            // all 128 columns of these 16 rows read before they are overwritten
                            epilogue_bar_sync(128);
    #pragma unroll
                            for (int j = 0; j < 16; ++j)
                                reinterpret_cast<T*>(staging + (c - c0 + j) * ROW_BYTES)[row_in_tile] =
                                    from_f32<T>(fmaf(cf[c + j], g[j], yv[j]));
                        }
                        if (last) {
                            tc_fence_before();
                            mbar_arrive(&tempty[acc]);
                        }
                        fence_proxy_async_smem();
                        epilogue_bar_sync(128);
                        if (et < nrows)
                            bulk_store(static_cast<T*>(p.y_out) + (tok0 + c0 + et) * p.h + m0,
                                       staging + et * ROW_BYTES, static_cast<uint32_t>(ncols * sizeof(T)));
                        bulk_commit();
                    }
                    if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
                    continue;
                }
            }
            TcUnit w;
            int rows, eid;
            int64_t hrow0;
            if (GATEUP && DENSE && u < pre_units) {
                // shared expert before the plan: all tokens, hidden rows after the routed slots
                const int sx = u / p.m_tiles;
                w.a = sx;
                w.tok_tile = 0;
                w.mtile = u - sx * p.m_tiles;
                w.split = 0;
                rows = static_cast<int>(p.n_tokens);
                eid = -1;
                hrow0 = p.sh_hrow + sx * p.n_tokens;
            } else {
                ga = tc_group_warp(p, num_active, ga, u, lane);
                w = tc_unit_at(p, ga, u, BN);
                rows = p.act_rows[w.a];
                eid = p.act_eid[w.a];
                hrow0 = p.act_hrow[w.a];
            }
            const int tok0 = w.tok_tile * BN;
            float* cf = s_coef + acc * BN;
            int32_t* tk = s_tok + acc * BN;
            if constexpr (!GATEUP) {
                // this tile's slot coefficients and tokens, read once (the other
                // buffer may still be read by threads finishing the previous unit)
                for (int r = et; r < BN; r += 128) {
                    const int tok = tok0 + r;
                    const bool ok = tok < rows;
                    cf[r] = ok ? p.slot_coef[hrow0 + tok] : 0.0f;
                    tk[r] = ok ? p.slot_tok[hrow0 + tok] : 0;
                }
            }
            // one thread waits (bounded) for the accumulator; the barrier hands its
            // outcome to the other 127, so they all leave together on a timeout
            if (et == 0) {
                const bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, kPipelineLimitNs, abort_flag);
                if (!ok) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                }
                *ep_ok = ok ? 1 : 0;
            }
            // the previous unit's bulk copies must also be done reading the staging rows
            bulk_wait_read();
            epilogue_bar_sync(128);
            if (!*ep_ok) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * ACC_COLS);
            const int m0 = w.mtile * kTcBM;
            const int ncols = min(kTcBM, p.out_cols - m0);
            constexpr int SUB = tc_staging_rows(BN, GATEUP);
            if constexpr (GATEUP && DENSE) {
                if (p.gu_splits > 1 && u >= pre_units) {
                    // ---- routed unit of a K-split tile ----
                    const int nt = static_cast<int>(p.n_tokens);  // <= BN
                    const int tile = (w.a - p.num_shared) * p.m_tiles + w.mtile;
                    const int64_t tstride = static_cast<int64_t>(nt) * kTcBM;  // one of G / U of one split
                    float* part = p.gu_part + (static_cast<int64_t>(tile) * p.gu_splits + w.split) * 2 * tstride;
#pragma unroll 1
                    for (int c = 0; c < nt; c += 16) {  // uniform: the TMEM loads are warp-wide
                        float g[16], uu[16];
                        tmem_ld16(taddr + c, g);
                        tmem_ld16(taddr + BN + c, uu);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (c + j < nt) {
                                part[(c + j) * kTcBM + row_in_tile] = g[j];
                                part[tstride + (c + j) * kTcBM + row_in_tile] = uu[j];
                            }
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);  // accumulator copied out: back to the MMA warp
                    __threadfence();
                    epilogue_bar_sync(128);
                    if (et == 0) {
                        const int done = atomicAdd(p.gu_cnt + tile, 1) + 1;
                        const bool last = done == p.gu_splits;
                        if (last) __threadfence();
                        *gu_last = last ? 1 : 0;
                    }
                    epilogue_bar_sync(128);
                    if (*gu_last) {
                        // every split's partial is in: sum in split order, SiLU-mul
                        __threadfence();
                        const float* tb = p.gu_part + static_cast<int64_t>(tile) * p.gu_splits * 2 * tstride;
#pragma unroll 1
                        for (int c0 = 0; c0 < BN; c0 += SUB) {
                            if (c0 >= nt) break;
                            if (c0 > 0) {
                                bulk_wait_read();
                                epilogue_bar_sync(128);
                            }
#pragma unroll 1
                            for (int c = c0; c < c0 + SUB; ++c) {
                                float gs = 0.0f, us = 0.0f;
                                if (c < nt) {
                                    for (int sp = 0; sp < p.gu_splits; ++sp) {
                                        gs += __ldcg(tb + sp * 2 * tstride + c * kTcBM + row_in_tile);
                                        us += __ldcg(tb + (sp * 2 + 1) * tstride + c * kTcBM + row_in_tile);
                                    }
                                }
                                reinterpret_cast<T*>(staging + (c - c0) * ROW_BYTES)[row_in_tile] =
                                    from_f32<T>(silu_f32(gs) * us);
                            }
                            fence_proxy_async_smem();
                            epilogue_bar_sync(128);
                            for (int r = et; r < SUB; r += 128) {
                                const int tok = c0 + r;
                                if (tok >= nt) continue;
                                const int64_t slot =
                                    eid < 0 ? hrow0 + tok : p.slot_map[static_cast<int64_t>(eid) * p.n_tokens + tok];
                                if (slot < 0) continue;
                                bulk_store(static_cast<T*>(p.hid) + slot * p.f + m0, staging + r * ROW_BYTES,
                                           static_cast<uint32_t>(ncols * sizeof(T)));
                            }
                            bulk_commit();
                        }
                    }
                    if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
                    continue;
                }
            }
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += SUB) {
                if (c0 > 0) {
                    // the staging rows are reused for the next SUB tokens of the tile
                    bulk_wait_read();
                    epilogue_bar_sync(128);
                }
#pragma unroll 1
                for (int c = c0; c < c0 + SUB; c += 16) {
                    float g[16];
                    tmem_ld16(taddr + c, g);
                    if constexpr (GATEUP) {
                        float uu[16];
                        tmem_ld16(taddr + BN + c, uu);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            uint8_t* row = staging + (c - c0 + j) * ROW_BYTES;
                            reinterpret_cast<T*>(row)[row_in_tile] = from_f32<T>(silu_f32(g[j]) * uu[j]);
                        }
                    } else {
                        tmem_wait_ld();
                        if (p.y_direct != nullptr) {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                reinterpret_cast<T*>(staging + (c - c0 + j) * ROW_BYTES)[row_in_tile] =
                                    from_f32<T>(cf[c + j] * g[j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                reinterpret_cast<float*>(staging + (c - c0 + j) * ROW_BYTES)[row_in_tile] =
                                    cf[c + j] * g[j];
                        }
                    }
                }
                if (c0 + SUB >= BN) {
                    // accumulator drained: hand the TMEM buffer back to the MMA warp
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                // staging rows complete -> per-token bulk copies
                fence_proxy_async_smem();
                epilogue_bar_sync(128);
                for (int r = et; r < SUB; r += 128) {
                    const int tok = tok0 + c0 + r;
                    int64_t slot;
                    if constexpr (DENSE) {
                        // column = token id; keep it only if the token chose this group
                        if (tok >= p.n_tokens) continue;
                        slot = eid < 0 ? hrow0 + tok : p.slot_map[static_cast<int64_t>(eid) * p.n_tokens + tok];
                        if (slot < 0) continue;
                    } else {
                        if (tok >= rows) continue;
                        slot = hrow0 + tok;
                    }
                    const uint8_t* row = staging + r * ROW_BYTES;
                    if constexpr (GATEUP) {
                        bulk_store(static_cast<T*>(p.hid) + slot * p.f + m0, row,
                                   static_cast<uint32_t>(ncols * sizeof(T)));
                    } else {
                        const int64_t t = tk[c0 + r];
                        if (p.y_direct != nullptr)
                            bulk_store(static_cast<T*>(p.y_direct) + t * p.h + m0, row,
                                       static_cast<uint32_t>(ncols * sizeof(T)));
                        else
                            bulk_reduce_add_f32(p.y_acc + t * p.h + m0, row,
                                                static_cast<uint32_t>(ncols * 4));
                    }
                }
                bulk_commit();
            }
            if constexpr (!GATEUP) {
                if (p.y_fold != nullptr) {
                    // one bulk group per unit (BN <= 128 staging rows): waiting for all
                    // but the newest leaves the previous unit's reduce-adds complete
                    static_assert(GATEUP || BN <= 128, "one bulk group per down unit");
                    if (fold_pending >= 0) {
                        bulk_wait_group_1();
                        fold_retire(fold_pending);
                    }
                    fold_pending = w.mtile;
                }
            }
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        // a CTA without shared-last units (or that stopped early) still counts itself in
        if (sf_count && !sf_counted) tc_count_routed_done(p.dn_done, et);
        bulk_wait_all();
        if constexpr (!GATEUP) {
            if (p.y_fold != nullptr && fold_pending >= 0 && *ep_ok) fold_retire(fold_pending);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}


// ---------------------------------------------------------------------------
// Token-major gate/up for large batches.  A = 128 token rows of the group
// (M = 128), B = the group's 128 gate rows followed by its 128 up rows (one
// 256-row K-major operand), one MMA of M = 128, N = 256 per 16 k: the token
// tile is read from shared memory once per k-step for both projections (the
// weight-major form reads it twice), 3/4 of the operand bytes per FLOP.  The
// accumulator row is a token: columns [0, 128) gate, [128, 256) up; the
// epilogue writes each token's h = silu(g) * u segment with one bulk store.
// ---------------------------------------------------------------------------
constexpr int kTmTokens = 128;
constexpr int kTmABytes = kTmTokens * kTcBK * 2;                  // 16 KB
constexpr int kTmStageBytes = kTmABytes + 2 * kTcBM * kTcBK * 2;  // + 32 KB
constexpr int kTmHalf = 64;                                       // f columns per epilogue pass
constexpr int kTmRowBytes = kTmHalf * 2 + 16;                     // padded: conflict-free rows
constexpr int kTmStagingBytes = kTmTokens * kTmRowBytes;
constexpr int kTmStages = (232448 - 1024 - 256 - kTmStagingBytes) / kTmStageBytes > 8
                              ? 8
                              : (232448 - 1024 - 256 - kTmStagingBytes) / kTmStageBytes;
constexpr int kTmSmemBytes = 1024 + kTmStages * kTmStageBytes + kTmStagingBytes + 256;

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gateup_tm(const __grid_constant__ CUtensorMap tm_gr,   // routed gate [P*F, H]
                 const __grid_constant__ CUtensorMap tm_ur,   // routed up
                 const __grid_constant__ CUtensorMap tm_gs,   // shared gate [S*F, H]
                 const __grid_constant__ CUtensorMap tm_us,   // shared up
                 const __grid_constant__ CUtensorMap tm_xr,   // expert-ordered token rows (Xp)
                 const __grid_constant__ CUtensorMap tm_xs,   // token rows of x (shared groups)
                 TcGemmParams p) {
    constexpr int STAGES = kTmStages;
    constexpr int ACC_COLS = 2 * kTcBM;  // gate | up
    constexpr int TMEM_COLS = 512;
    static_assert(STAGES >= 2, "shared memory holds fewer than two pipeline stages");
    static_assert(kTmSmemBytes <= 232448, "shared memory over the per-CTA limit");

    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* staging = smem + STAGES * kTmStageBytes;  // [128 tokens][kTmRowBytes]
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + kTmStagingBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_gr);
        prefetch_tmap(&tm_xr);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    pdl_wait();
    const int num_active = p.hdr->num_active;
    const int total = p.hdr->units_gu;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        int stage = 0;
        uint32_t phase = 0;
        int polled_eid = -1;
        int ga = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            ga = tc_group_warp(p, num_active, ga, u, lane);
            if (lane == 0) {
                const TcUnit w = tc_unit_at(p, ga, u, kTmTokens);
                const int eid = p.act_eid[w.a];
                const bool shared = eid < 0;
                if (!shared && p.ready_flags != nullptr && eid != polled_eid) {
                    const uint64_t t0 = globaltimer_ns();
                    bool ok = true;
                    while (ld_acquire_gpu(p.ready_flags + eid) < p.ready_epoch) {
                        if (globaltimer_ns() - t0 > p.ready_limit_ns) { ok = false; break; }
                        __nanosleep(256);
                    }
                    if (!ok) report_status(p.status, CHRONOS_ERR_EXPERT_NOT_READY);
                    fence_proxy_async_global();
                    polled_eid = eid;
                }
                const int w_row = p.act_wslot[w.a] * p.w_rows + w.mtile * kTcBM;
                const int x_row = p.act_xrow[w.a] + w.tok_tile * kTmTokens;
                const CUtensorMap* mg = shared ? &tm_gs : &tm_gr;
                const CUtensorMap* mu = shared ? &tm_us : &tm_ur;
                const CUtensorMap* mx = shared ? &tm_xs : &tm_xr;
                for (int kt = 0; kt < p.k_tiles; ++kt) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        break;
                    }
                    uint8_t* sb = smem + stage * kTmStageBytes;
                    mbar_arrive_expect_tx(&full[stage], kTmStageBytes);
                    tma_load_2d(sb, mx, &full[stage], kt * kTcBK, x_row);
                    tma_load_2d(sb + kTmABytes, mg, &full[stage], kt * kTcBK, w_row);
                    tma_load_2d(sb + kTmABytes + kTcBM * kTcBK * 2, mu, &full[stage], kt * kTcBK, w_row);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------ MMA issuer ------------------------------
            constexpr uint32_t IDESC = idesc_f16(kTmTokens, ACC_COLS, AbFormat<T>::value);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
                bool failed = false;
                for (int kt = 0; kt < p.k_tiles; ++kt) {
                    if (!mbar_wait_bounded(&full[stage], phase, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sx = smem_u32(smem + stage * kTmStageBytes);
                    const uint32_t sw = sx + kTmABytes;
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 16; ++kk) {
                        const uint32_t accum = (kt > 0 || kk > 0) ? 1u : 0u;
                        umma_f16(d, sdesc_k_sw128(sx + kk * 32), sdesc_k_sw128(sw + kk * 32), IDESC, accum);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (failed) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        // thread = one token row of the tile (TMEM lane), two passes of 64 f each
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        const int et = threadIdx.x - 64;
        volatile int* ep_ok = abort_flag + 1;
        uint8_t* my_row = staging + row_in_tile * kTmRowBytes;
        int acc = 0;
        uint32_t acc_phase = 0;
        int ga = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            ga = tc_group_warp(p, num_active, ga, u, lane);
            const TcUnit w = tc_unit_at(p, ga, u, kTmTokens);
            const int rows = p.act_rows[w.a];
            const int64_t hrow0 = p.act_hrow[w.a];
            const int tok = w.tok_tile * kTmTokens + row_in_tile;
            const int m0 = w.mtile * kTcBM;
            const int ncols = min(kTcBM, p.out_cols - m0);
            if (et == 0) {
                const bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, kPipelineLimitNs, abort_flag);
                if (!ok) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                }
                *ep_ok = ok ? 1 : 0;
            }
            bulk_wait_read();  // the previous unit's stores are done reading the staging rows
            epilogue_bar_sync(128);
            if (!*ep_ok) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * ACC_COLS);
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                if (half == 1) bulk_wait_read();  // this thread's first-half store has read its row
#pragma unroll 1
                for (int c = half * kTmHalf; c < half * kTmHalf + kTmHalf; c += 16) {
                    float g[16], uu[16];
                    tmem_ld16(taddr + c, g);
                    tmem_ld16(taddr + kTcBM + c, uu);
                    tmem_wait_ld();
                    T h[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) h[j] = from_f32<T>(silu_f32(g[j]) * uu[j]);
                    uint4* dst = reinterpret_cast<uint4*>(my_row + (c - half * kTmHalf) * 2);
                    dst[0] = reinterpret_cast<const uint4*>(h)[0];
                    dst[1] = reinterpret_cast<const uint4*>(h)[1];
                }
                if (half == 1) {
                    // accumulator drained: hand the TMEM buffer back to the MMA warp
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                fence_proxy_async_smem();
                if (tok < rows && half * kTmHalf < ncols)
                    bulk_store(static_cast<T*>(p.hid) + (hrow0 + tok) * p.f + m0 + half * kTmHalf, my_row,
                               static_cast<uint32_t>(kTmHalf * sizeof(T)));
                bulk_commit();
            }
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}


// ---------------------------------------------------------------------------
// Token-major down GEMM for large batches.  A = 128 hidden rows of the group
// (its tokens, M = 128), B = 256 rows of the group's down weights (two
// 128-row boxes, N = 256), K = F.  Token tiles of 128 rows leave less padding
// in small expert groups than 256-token tiles, at the same operand bytes per
// FLOP.  The accumulator row is a token: the epilogue thread owning it scales
// the row by the slot coefficient and reduce-adds it into the token's y_acc
// row, PASS columns at a time, through its own padded staging row (no
// transposition, no barriers between the epilogue threads).  Direct output
// (k = 1, no shared experts) and shared-last units (sf_shared > 0) behave as
// in tc_grouped_gemm: shared-last units follow the routed ones, run K over
// the S_h shared experts back to back and write y_out = y_acc + coef * D.
// ---------------------------------------------------------------------------
constexpr int kDmCols = 256;                                    // output columns per tile (MMA N)
constexpr int kDmStageBytes = kTmABytes + kDmCols * kTcBK * 2;  // 16 KB tokens + 32 KB weights
__host__ __device__ constexpr int tc_dm_row_bytes(int pass) { return pass * 4 + 16; }
// No alignment slack: the dynamic shared memory of a CTA that has no static
// shared memory starts 1024-byte aligned (the kernel checks it and reports
// CHRONOS_ERR_CUDA otherwise), which buys the ring its fourth stage.
__host__ __device__ constexpr int tc_dm_stages(int pass) {
    return (232448 - 256 - kTmTokens * tc_dm_row_bytes(pass)) / kDmStageBytes > 8
               ? 8
               : (232448 - 256 - kTmTokens * tc_dm_row_bytes(pass)) / kDmStageBytes;
}
__host__ __device__ constexpr int tc_dm_smem_bytes(int pass) {
    return tc_dm_stages(pass) * kDmStageBytes + kTmTokens * tc_dm_row_bytes(pass) + 256;
}

template <typename T, int PASS>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_down_tm(const __grid_constant__ CUtensorMap tm_dr,  // routed down [P*H, F], 128-row boxes
               const __grid_constant__ CUtensorMap tm_ds,  // shared down [S*H, F]
               const __grid_constant__ CUtensorMap tm_h,   // hidden rows [slots, F], 128-row boxes
               TcGemmParams p) {
    constexpr int STAGES = tc_dm_stages(PASS);
    constexpr int ROW_BYTES = tc_dm_row_bytes(PASS);
    constexpr int ACC_COLS = kDmCols;
    constexpr int TMEM_COLS = 512;
    static_assert(kDmCols % PASS == 0 && PASS % 16 == 0, "passes must tile the 256 columns");
    static_assert(STAGES >= 2, "shared memory holds fewer than two pipeline stages");
    static_assert(tc_dm_smem_bytes(PASS) <= 232448, "shared memory over the per-CTA limit");

    extern __shared__ __align__(1024) uint8_t tc_dm_smem[];
    if ((smem_u32(tc_dm_smem) & 1023u) != 0u) {
        // operand tiles need 1024-byte alignment (128-byte swizzle atoms)
        if (threadIdx.x == 0) report_status(p.status, CHRONOS_ERR_CUDA);
        return;
    }
    uint8_t* smem = tc_dm_smem;
    uint8_t* staging = smem + STAGES * kDmStageBytes;  // [128 tokens][ROW_BYTES]
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + kTmTokens * ROW_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* ybar = tempty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ybar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        mbar_init(ybar, 1);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tm_dr);
        prefetch_tmap(&tm_h);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    pdl_wait();
    const int num_active = p.hdr->num_active;
    const int total_main = p.hdr->units_dn;
    const int sf_tt = p.sf_shared > 0 ? static_cast<int>((p.n_tokens + kTmTokens - 1) / kTmTokens) : 0;
    const int total = total_main + sf_tt * p.m_tiles;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        int stage = 0;
        uint32_t phase = 0;
        int polled_eid = -1;
        int ga = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            const bool sfu = u >= total_main;
            if (!sfu) ga = tc_group_warp(p, num_active, ga, u, lane);
            if (lane == 0) {
                int h_row, w_row, ktot;
                const CUtensorMap* mw;
                if (sfu) {
                    const int rem = u - total_main;
                    h_row = static_cast<int>(p.sh_hrow) + (rem % sf_tt) * kTmTokens;
                    w_row = (rem / sf_tt) * kDmCols;
                    ktot = p.sf_shared * p.k_tiles;
                    mw = &tm_ds;
                } else {
                    const TcUnit w = tc_unit_at(p, ga, u, kTmTokens);
                    const int eid = p.act_eid[w.a];
                    const bool shared = eid < 0;
                    if (!shared && p.ready_flags != nullptr && eid != polled_eid) {
                        const uint64_t t0 = globaltimer_ns();
                        bool ok = true;
                        while (ld_acquire_gpu(p.ready_flags + eid) < p.ready_epoch) {
                            if (globaltimer_ns() - t0 > p.ready_limit_ns) { ok = false; break; }
                            __nanosleep(256);
                        }
                        if (!ok) report_status(p.status, CHRONOS_ERR_EXPERT_NOT_READY);
                        fence_proxy_async_global();
                        polled_eid = eid;
                    }
                    h_row = p.act_hrow[w.a] + w.tok_tile * kTmTokens;
                    w_row = p.act_wslot[w.a] * p.w_rows + w.mtile * kDmCols;
                    ktot = p.k_tiles;
                    mw = shared ? &tm_ds : &tm_dr;
                }
                for (int kt = 0; kt < ktot; ++kt) {
                    // shared-last units: k tiles of shared expert sx, whose hidden rows
                    // follow the previous expert's N rows
                    const int sx = sfu ? kt / p.k_tiles : 0;
                    const int kk = kt - sx * p.k_tiles;
                    const int hr = h_row + static_cast<int>(sx * p.n_tokens);
                    const int wr = w_row + sx * p.w_rows;
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        break;
                    }
                    uint8_t* sb = smem + stage * kDmStageBytes;
                    mbar_arrive_expect_tx(&full[stage], kDmStageBytes);
                    tma_load_2d(sb, &tm_h, &full[stage], kk * kTcBK, hr);
                    tma_load_2d(sb + kTmABytes, mw, &full[stage], kk * kTcBK, wr);
                    tma_load_2d(sb + kTmABytes + kTcBM * kTcBK * 2, mw, &full[stage], kk * kTcBK, wr + kTcBM);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------ MMA issuer ------------------------------
            constexpr uint32_t IDESC = idesc_f16(kTmTokens, kDmCols, AbFormat<T>::value);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
                const int ktot = u >= total_main ? p.sf_shared * p.k_tiles : p.k_tiles;
                if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, kPipelineLimitNs, abort_flag)) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
                bool failed = false;
                for (int kt = 0; kt < ktot; ++kt) {
                    if (!mbar_wait_bounded(&full[stage], phase, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sh = smem_u32(smem + stage * kDmStageBytes);
                    const uint32_t sw = sh + kTmABytes;
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 16; ++kk) {
                        const uint32_t accum = (kt > 0 || kk > 0) ? 1u : 0u;
                        umma_f16(d, sdesc_k_sw128(sh + kk * 32), sdesc_k_sw128(sw + kk * 32), IDESC, accum);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (failed) break;
                umma_commit(&tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        // thread = one token row of the tile (TMEM lane)
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        const int et = threadIdx.x - 64;
        volatile int* ep_ok = abort_flag + 1;
        uint8_t* my_row = staging + row_in_tile * ROW_BYTES;
        int acc = 0;
        uint32_t acc_phase = 0;
        int ga = 0;
        const bool sf_count = p.sf_shared > 0 && static_cast<int>(blockIdx.x) < total_main;
        const int sf_target = min(static_cast<int>(gridDim.x), total_main);
        bool sf_counted = false, sf_ready = false;
        uint32_t yphase = 0;
        const bool two_phase = p.ys != nullptr;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            const bool sfu = u >= total_main;
            int64_t out_row = -1;  // y row of this thread's token, -1: padding row
            int64_t out_slot = -1; // two-phase routed units: the row's slot in ys
            float coef = 0.0f;
            int n0;
            if (sfu) {
                if (sf_count && !sf_counted) {
                    tc_count_routed_done(p.dn_done, et);
                    sf_counted = true;
                }
                const int rem = u - total_main;
                const int64_t tok = static_cast<int64_t>(rem % sf_tt) * kTmTokens + row_in_tile;
                n0 = (rem / sf_tt) * kDmCols;
                if (tok < p.n_tokens) {
                    out_row = tok;
                    coef = p.slot_coef[p.sh_hrow + tok];
                }
            } else {
                ga = tc_group_warp(p, num_active, ga, u, lane);
                const TcUnit w = tc_unit_at(p, ga, u, kTmTokens);
                const int tok = w.tok_tile * kTmTokens + row_in_tile;
                n0 = w.mtile * kDmCols;
                if (tok < p.act_rows[w.a]) {
                    const int64_t slot = p.act_hrow[w.a] + tok;
                    out_row = p.slot_tok[slot];
                    out_slot = slot;
                    coef = p.slot_coef[slot];
                }
            }
            const int ncols = min(kDmCols, p.out_cols - n0);
            if (et == 0) {
                bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, kPipelineLimitNs, abort_flag);
                if (ok && sfu && !sf_ready) {
                    // every routed contribution must be in the accumulator
                    const uint64_t t0 = globaltimer_ns();
                    while (ld_acquire_gpu(p.dn_done) < sf_target) {
                        if (*abort_flag || globaltimer_ns() - t0 > kPipelineLimitNs) {
                            ok = false;
                            break;
                        }
                        __nanosleep(64);
                    }
                }
                if (!ok) {
                    *abort_flag = 1;
                    report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                }
                *ep_ok = ok ? 1 : 0;
            }
            if (sfu) sf_ready = true;
            // two-phase shared units: this token's slot rows, read once per unit
            // (all k loads in flight together)
            constexpr int kPairBatch = 8;
            constexpr int kPairMax = 2 * kPairBatch;  // >= kMaxTopK
            int sls[kPairMax];
#pragma unroll
            for (int q2 = 0; q2 < kPairMax; ++q2)
                sls[q2] = (sfu && two_phase && out_row >= 0 && q2 < p.k_pairs)
                              ? __ldcg(p.pair_slot + out_row * p.k_pairs + q2)
                              : -1;
            bulk_wait_read();  // this thread's previous copies are done reading its row
            epilogue_bar_sync(128);
            if (!*ep_ok) break;
            tc_fence_after();
            if (sfu) fence_proxy_async_global();  // accumulator rows are read by bulk copies below
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * ACC_COLS);
#pragma unroll 1
            for (int c0 = 0; c0 < kDmCols; c0 += PASS) {
                const int nc = min(PASS, ncols - c0);  // uniform over the tile
                if (nc <= 0) break;
                const bool last = c0 + PASS >= ncols;
                // this pass's accumulator columns -> registers first: the TMEM reads
                // overlap the wait for the staging row, and the last pass hands the
                // accumulator back before the row is written
                float g[PASS];
#pragma unroll
                for (int j = 0; j < PASS; j += 16) tmem_ld16(taddr + c0 + j, *reinterpret_cast<float(*)[16]>(g + j));
                tmem_wait_ld();
                if (last) {
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                if (c0 > 0) bulk_wait_read();  // this thread's previous copy has read its row
                float4* row4 = reinterpret_cast<float4*>(my_row);
                if (sfu && !two_phase) {
                    // the pass's accumulator segment of every valid token row -> its
                    // staging row (the barrier orders the expected bytes before the copies)
                    const int64_t tile_tok0 = static_cast<int64_t>((u - total_main) % sf_tt) * kTmTokens;
                    const int64_t left = p.n_tokens - tile_tok0;
                    const int nrows = left < kTmTokens ? static_cast<int>(left) : kTmTokens;
                    if (et == 0) mbar_arrive_expect_tx(ybar, static_cast<uint32_t>(nrows * nc * 4));
                    epilogue_bar_sync(128);
                    if (out_row >= 0)
                        bulk_load(my_row, p.y_acc + out_row * p.h + n0 + c0, static_cast<uint32_t>(nc * 4), ybar);
                    if (!mbar_wait_bounded(ybar, yphase, kPipelineLimitNs, abort_flag)) {
                        *abort_flag = 1;
                        report_status(p.status, CHRONOS_ERR_PIPELINE_TIMEOUT);
                    }
                    yphase ^= 1u;
                }
                if (sfu || p.y_direct != nullptr || two_phase) {
                    // output dtype, written over the front of the row (2 bytes per
                    // column behind the 4-byte columns already read)
#pragma unroll
                    for (int c = 0; c < PASS; c += 16) {
                        float yv[16];
                        if (sfu && two_phase) {
                            // the token's routed contributions, in choice order; the
                            // loads of up to 8 slot rows are issued before any is used
#pragma unroll
                            for (int j = 0; j < 16; ++j) yv[j] = 0.0f;
#pragma unroll
                            for (int qb = 0; qb < kPairMax; qb += kPairBatch) {
                                if (qb >= p.k_pairs) break;
                                uint4 v[kPairBatch][2];
#pragma unroll
                                for (int j = 0; j < kPairBatch; ++j) {
                                    if (sls[qb + j] >= 0) {
                                        const uint4* src = reinterpret_cast<const uint4*>(
                                            static_cast<const T*>(p.ys) + static_cast<int64_t>(sls[qb + j]) * p.h +
                                            n0 + c0 + c);
                                        v[j][0] = __ldcg(src);
                                        v[j][1] = __ldcg(src + 1);
                                    }
                                }
#pragma unroll
                                for (int j = 0; j < kPairBatch; ++j) {
                                    if (sls[qb + j] < 0) continue;
                                    const T* e0 = reinterpret_cast<const T*>(&v[j][0]);
                                    const T* e1 = reinterpret_cast<const T*>(&v[j][1]);
#pragma unroll
                                    for (int u = 0; u < 8; ++u) {
                                        yv[u] += to_f32<T>(e0[u]);
                                        yv[8 + u] += to_f32<T>(e1[u]);
                                    }
                                }
                            }
                        } else if (sfu) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float4 v = row4[c / 4 + j];
                                yv[4 * j] = v.x;
                                yv[4 * j + 1] = v.y;
                                yv[4 * j + 2] = v.z;
                                yv[4 * j + 3] = v.w;
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j) yv[j] = 0.0f;
                        }
                        T o[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) o[j] = from_f32<T>(fmaf(coef, g[c + j], yv[j]));
                        uint4* dst = reinterpret_cast<uint4*>(my_row + c * 2);
                        dst[0] = reinterpret_cast<const uint4*>(o)[0];
                        dst[1] = reinterpret_cast<const uint4*>(o)[1];
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < PASS; c += 4)
                        row4[c / 4] = make_float4(coef * g[c], coef * g[c + 1], coef * g[c + 2], coef * g[c + 3]);
                }
                fence_proxy_async_smem();
                if (out_row >= 0) {
                    if (sfu)
                        bulk_store(static_cast<T*>(p.y_out) + out_row * p.h + n0 + c0, my_row,
                                   static_cast<uint32_t>(nc * sizeof(T)));
                    else if (two_phase)
                        bulk_store(static_cast<T*>(p.ys) + out_slot * p.h + n0 + c0, my_row,
                                   static_cast<uint32_t>(nc * sizeof(T)));
                    else if (p.y_direct != nullptr)
                        bulk_store(static_cast<T*>(p.y_direct) + out_row * p.h + n0 + c0, my_row,
                                   static_cast<uint32_t>(nc * sizeof(T)));
                    else
                        bulk_reduce_add_f32(p.y_acc + out_row * p.h + n0 + c0, my_row,
                                            static_cast<uint32_t>(nc * 4));
                }
                bulk_commit();
            }
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
        if (sf_count && !sf_counted) tc_count_routed_done(p.dn_done, et);
        bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace chronos
