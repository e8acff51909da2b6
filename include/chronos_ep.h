/*
 * chronos_ep.h — C ABI of the expert-parallel dispatch / combine kernels.
 *
 * No counterpart in the reference: FonaTech/Project_Chronos runs every expert
 * of a layer on one device (chronos/model/moe_chronos.py:146-173, 190-268;
 * no torch.distributed anywhere).  These entry points split that same
 * arithmetic across G ranks, rank g owning the contiguous routed experts
 * [g*E/G, (g+1)*E/G) while the router and the shared experts are replicated:
 *
 *   y_t = shared_t * (1 + sum_j w_tj (1 - a_e))          (on the token's rank)
 *         + sum_j w_tj a_e SwiGLU_e(x_t)                  (on expert e's rank)
 *
 * the blend of chronos/mlx/moe.py:160-166 with the selections of one token
 * sent to the ranks that own their experts.  The exchange itself (counts,
 * rows, returned rows) is the caller's all-to-all (NCCL over NVLink); these
 * kernels build its send buffers and fold the returned rows back.
 *
 * Conventions as in chronos_moe.h: device pointers, row-major contiguous
 * tensors, caller-allocated buffers, stream-ordered, nothing aborts.
 */
#ifndef CHRONOS_EP_H_
#define CHRONOS_EP_H_

#include <stddef.h>
#include <stdint.h>

#include "chronos_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

#define CHRONOS_EP_MAX_RANKS 32

typedef struct ChronosEpDispatchArgs {
    int64_t num_tokens;        /* N tokens on this rank */
    int32_t hidden;            /* H; H * element size must be a multiple of 16 bytes */
    int32_t num_experts;       /* E routed experts in total (a multiple of world_size) */
    int32_t top_k;             /* k */
    int32_t world_size;        /* G, 1..CHRONOS_EP_MAX_RANKS */
    int32_t dtype;             /* CHRONOS_DTYPE_* of x and send_x */
    int32_t num_chunks;        /* C >= 1 dividing E/G: each rank's local experts split into C
                                  chunks of E/(G*C); send rows ordered by (expert chunk,
                                  destination rank); C * G <= CHRONOS_EP_MAX_RANKS */
    int32_t meta_pairs;        /* 0 or 1: one send row per available selection, send_meta
                                  [rows, 2]; P >= min(k, E/G) (C = 1): deduplicated, one
                                  send row per (token, destination rank), send_meta
                                  [rows, P, 2] = that rank's available selections of the
                                  token in choice order, padded with (-1, 0.0f) */
    const void* x;             /* [N, H] */
    const int32_t* topk_idx;   /* [N, k] global expert ids (chronos_moe_route) */
    const float* topk_weight;  /* [N, k] */
    const float* avail;        /* [E] availability a_e in [0, 1], or NULL for all 1 */
    int32_t* send_counts;      /* [C, G] out: selections of each expert chunk sent to each rank */
    void* send_x;              /* [N*k, H] out: x rows grouped by destination rank */
    int32_t* send_meta;        /* [N*k, P or 1, 2] out: (expert id local to the destination
                                  rank, fp32 bits of w * a) per send row and selection */
    int32_t* pair_slot;        /* [N*k] out: send row of selection (t, j), -1 when a = 0 (and,
                                  deduplicated, for all but the token's first selection on
                                  each rank) */
    float* shared_weight;      /* [N, k] out: w * (1 - a), the shared experts' share */
    int32_t* scratch;          /* [N*k] int32 scratch */
    int64_t seg_rows;          /* 0: rows packed (rank g's rows follow rank g-1's).  > 0 (one
                                  chunk): fixed all-to-all segments, rank g's rows at
                                  [g * seg_rows, g * seg_rows + send_counts[g]); the rest of
                                  each segment gets padding metadata (expert -1, weight 0) and
                                  unspecified x rows.  seg_rows >= N (deduplicated) or
                                  N * min(k, E/G); send_x and send_meta then hold G * seg_rows
                                  rows.  With equal splits no host needs the counts before the
                                  exchange. */
} ChronosEpDispatchArgs;

/* Builds the send buffers of one rank: rows are grouped by (expert chunk,
 * destination rank), chunk-major (first send_counts[0][0] rows: chunk 0 to
 * rank 0, ...), so each chunk's rows form one contiguous all-to-all send
 * buffer and a receiver can run each chunk's experts as soon as it lands
 * (reading each expert's weights once); within a group the row order is
 * unspecified.  Selections with a_e = 0 are not sent.  Deduplicated
 * (meta_pairs > 1), a token's selections on one rank share one row, so the
 * exchange carries each x row at most once per destination and the
 * receiver runs its experts on the row with top_k = P (pre-routed, padding
 * selections skipped). */
CHRONOS_API int chronos_ep_dispatch(const ChronosEpDispatchArgs* args, void* cuda_stream);

typedef struct ChronosEpCombineArgs {
    int64_t num_tokens;        /* N */
    int32_t hidden;            /* H (as for dispatch) */
    int32_t top_k;             /* k */
    int32_t dtype;             /* CHRONOS_DTYPE_* of every row buffer */
    const void* y_shared;      /* [N, H] shared term (1 + sum_j shared_weight) * shared_t, or NULL */
    const void* recv_y;        /* [sum(send_counts), H] returned rows (w*a*SwiGLU_e), send order */
    const int32_t* pair_slot;  /* [N*k] from chronos_ep_dispatch */
    void* y;                   /* [N, H] out */
} ChronosEpCombineArgs;

/* y_t = y_shared_t + sum over j = 0..k-1 (ascending) of recv_y[pair_slot[t*k + j]],
 * accumulated in fp32, rounded once to the output type. */
CHRONOS_API int chronos_ep_combine(const ChronosEpCombineArgs* args, void* cuda_stream);

/* sizeof of the two structs as compiled into the library (FFI mirror checks). */
CHRONOS_API size_t chronos_ep_dispatch_args_size(void);
CHRONOS_API size_t chronos_ep_combine_args_size(void);

#ifdef __cplusplus
}
#endif

#endif /* CHRONOS_EP_H_ */
