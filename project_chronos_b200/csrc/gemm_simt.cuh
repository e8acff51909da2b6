// gemm_simt.cuh — grouped expert GEMMs on the CUDA cores with fp32 FMA.
//
// Used for fp32 layers (tcgen05 has no fp32 kind; rel-L2 1e-5 parity needs
// true fp32 arithmetic) and for bf16/fp16 layers whose H or F is not a
// multiple of 64 (the TMA/128-byte-swizzle tiling of gemm_tc.cuh).  Same
// work decomposition and epilogues as the tensor-core kernels: tiles of 64
// token rows x 64 weight rows per active group, token rows read by slot ->
// token index (no permuted copy of x needed).
#pragma once

#include "common.cuh"
#include "plan.cuh"

namespace chronos {

constexpr int kSimtTile = 64;
constexpr int kSimtBK = 16;
constexpr int kSimtThreads = 256;

struct SimtGemmParams {
    const PlanHeader* hdr;
    const int32_t* act_rows;
    const int32_t* act_hrow;
    const int32_t* act_wslot;
    const int32_t* act_eid;
    const int32_t* ustart;
    int m_tiles;
    int kdim;        // H (gate/up) or F (down)
    int out_cols;    // F (gate/up) or H (down)
    int f, h;
    const void* x;          // GATEUP: token rows of x, by slot_tok
    const void* hid_in;     // DOWN: [slots, F]
    const void* w0r;        // routed gate (or down) pool
    const void* w1r;        // routed up pool
    const void* w0s;        // shared gate (or down)
    const void* w1s;        // shared up
    void* hid_out;          // GATEUP: [slots, F]
    float* y_acc;           // DOWN
    const int32_t* slot_tok;
    const float* slot_coef;
    // expert readiness: wait (bounded) until ready_flags[e] >= ready_epoch
    const int32_t* ready_flags;
    int32_t ready_epoch;
    uint64_t ready_limit_ns;
    int32_t* status;
};

template <typename T, bool GATEUP>
__global__ void __launch_bounds__(kSimtThreads) simt_grouped_gemm(SimtGemmParams p) {
    __shared__ float as[kSimtBK][kSimtTile + 4];
    __shared__ float bs0[kSimtBK][kSimtTile + 4];
    __shared__ float bs1[GATEUP ? kSimtBK : 1][kSimtTile + 4];
    __shared__ int64_t s_arow[kSimtTile];
    int polled_eid = -1;  // meaningful in thread 0 only

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    pdl_trigger();
    pdl_wait();
    const int num_active = p.hdr->num_active;
    const int total = GATEUP ? p.hdr->units_gu : p.hdr->units_dn;
    const int K = p.kdim;

    for (int u = blockIdx.x; u < total; u += gridDim.x) {
        int lo = 0, hi = num_active - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.ustart[mid] <= u) lo = mid; else hi = mid - 1;
        }
        const int a = lo;
        const int rows = p.act_rows[a];
        const int tt = (rows + kSimtTile - 1) / kSimtTile;
        int rem = u - p.ustart[a];
        const int tok_tile = rem % tt;
        const int mtile = rem / tt;
        const bool shared = p.act_eid[a] < 0;
        const int64_t hrow0 = p.act_hrow[a];
        const int64_t wslot = p.act_wslot[a];
        const T* w0 = static_cast<const T*>(shared ? p.w0s : p.w0r) + wslot * p.out_cols * K;
        const T* w1 = GATEUP ? static_cast<const T*>(shared ? p.w1s : p.w1r) + wslot * p.out_cols * K
                             : nullptr;
        if (tid == 0 && !shared && p.ready_flags != nullptr && p.act_eid[a] != polled_eid) {
            // wait (bounded) for this selected expert's weights to be resident
            const int eid = p.act_eid[a];
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_gpu(p.ready_flags + eid) < p.ready_epoch) {
                if (globaltimer_ns() - t0 > p.ready_limit_ns) {
                    report_status(p.status, CHRONOS_ERR_EXPERT_NOT_READY);
                    break;
                }
                __nanosleep(256);
            }
            polled_eid = eid;
        }
        __syncthreads();
        if (tid < kSimtTile) {
            const int tok = tok_tile * kSimtTile + tid;
            int64_t r = -1;
            if (tok < rows) r = GATEUP ? static_cast<int64_t>(p.slot_tok[hrow0 + tok]) : hrow0 + tok;
            s_arow[tid] = r;
        }
        float acc0[4][4], acc1[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) { acc0[i][j] = 0.f; acc1[i][j] = 0.f; }
        const T* asrc = static_cast<const T*>(GATEUP ? p.x : p.hid_in);
        for (int kc = 0; kc < K; kc += kSimtBK) {
            __syncthreads();
            for (int i = tid; i < kSimtBK * kSimtTile; i += kSimtThreads) {
                const int r = i / kSimtBK, c = i % kSimtBK;
                const int64_t ar = s_arow[r];
                const int kk = kc + c;
                as[c][r] = (ar >= 0 && kk < K) ? to_f32<T>(asrc[ar * K + kk]) : 0.f;
                const int wr = mtile * kSimtTile + r;
                const bool wok = wr < p.out_cols && kk < K;
                bs0[c][r] = wok ? to_f32<T>(w0[static_cast<int64_t>(wr) * K + kk]) : 0.f;
                if (GATEUP) bs1[c][r] = wok ? to_f32<T>(w1[static_cast<int64_t>(wr) * K + kk]) : 0.f;
            }
            __syncthreads();
#pragma unroll
            for (int c = 0; c < kSimtBK; ++c) {
                float av[4], bv0[4], bv1[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = as[c][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    bv0[j] = bs0[c][tx * 4 + j];
                    bv1[j] = GATEUP ? bs1[c][tx * 4 + j] : 0.f;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc0[i][j] = fmaf(av[i], bv0[j], acc0[i][j]);
                        if (GATEUP) acc1[i][j] = fmaf(av[i], bv1[j], acc1[i][j]);
                    }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = tok_tile * kSimtTile + ty * 4 + i;
            if (tok >= rows) continue;
            const int64_t slot = hrow0 + tok;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = mtile * kSimtTile + tx * 4 + j;
                if (col >= p.out_cols) continue;
                if constexpr (GATEUP) {
                    static_cast<T*>(p.hid_out)[slot * p.f + col] =
                        from_f32<T>(silu_f32(acc0[i][j]) * acc1[i][j]);
                } else {
                    const int64_t t = p.slot_tok[slot];
                    atomicAdd(p.y_acc + t * p.h + col, p.slot_coef[slot] * acc0[i][j]);
                }
            }
        }
    }
}

}  // namespace chronos
