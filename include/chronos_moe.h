/*
 * chronos_moe.h — C ABI of the sm_100a MoE feed-forward extension.
 *
 * One call computes the Chronos MoE feed-forward layer
 * (chronos/model/moe_chronos.py:95-281, ChronosMOEFeedForward.forward):
 *
 *   scores   = softmax(x @ router_w^T [+ router_bias])            (:112)
 *   topk     = top_k(scores), optional renormalisation            (:124-128)
 *   shared   = mean_j SwiGLU_j(x)                                 (:90-93)
 *   y_t      = sum_k w_tk * (a_e * SwiGLU_e(x_t) + (1 - a_e) * shared_t)
 *              + shared_t                                          (:190-268,
 *                                                                   chronos/mlx/moe.py:160-166)
 *
 * where SwiGLU(x) = down(silu(gate(x)) * up(x)) is the bias-free expert of
 * the minimind FeedForward (restated at chronos/mlx/moe.py:13-23) and a_e is
 * the effective availability of routed expert e (1 = resident, 0 = cache
 * miss served by the shared experts).
 *
 * Routing contract (bit-exact, identical on every run): a logit is the
 * in-order fp32 sum of chunk partials, partial c being one chain of fused
 * multiply-adds over h in [128c, min(128c + 128, H)) starting from 0
 * (operands widened to fp32), plus router_bias[e] when given.  Experts are
 * ranked by (logit descending, expert index ascending); the top-k weights
 * are the fp32 softmax probabilities of the chosen experts, renormalised by
 * (sum + 1e-20) when norm_topk is set.
 *
 * Conventions: every pointer in ChronosMoeArgs is a DEVICE pointer unless
 * stated otherwise; all matrices are row-major and contiguous with the
 * nn.Linear [out, in] layout.  The caller allocates every buffer, including
 * the workspace (size from chronos_moe_workspace_size).  Calls are ordered
 * on the given stream; nothing here synchronises the host unless the
 * function's comment says so.  No function aborts, traps or exits.
 */
#ifndef CHRONOS_MOE_H_
#define CHRONOS_MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CHRONOS_API __attribute__((visibility("default")))
#else
#define CHRONOS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CHRONOS_MOE_ABI_VERSION 2

/* Return codes. */
#define CHRONOS_OK 0
#define CHRONOS_ERR_INVALID_ARG 1
#define CHRONOS_ERR_WORKSPACE_TOO_SMALL 2
#define CHRONOS_ERR_CUDA 3
#define CHRONOS_ERR_EXPERT_NOT_READY 4 /* a device-side ready-flag wait ran out */
#define CHRONOS_ERR_NCCL 5
#define CHRONOS_ERR_PIPELINE_TIMEOUT 6 /* an internal pipeline wait ran out */

/* Element types of x, router_w, the expert weights, y and router_probs. */
#define CHRONOS_DTYPE_BF16 0
#define CHRONOS_DTYPE_FP16 1
#define CHRONOS_DTYPE_FP32 2

/* Flags (ChronosMoeArgs.flags). */
/* topk_idx / topk_weight are INPUTS produced by an earlier
 * chronos_moe_route call (the host-hook slow path); routing is skipped. */
#define CHRONOS_FLAG_PREROUTED 0x1
/* avail is a residency mask: a_e = 1 where avail[e] > 0, else 0 (the caller's
 * mask passed as it is, no thresholding pass before the call). */
#define CHRONOS_FLAG_AVAIL_MASK 0x2
/* y is an fp32 [N, H] buffer (16-byte aligned) that receives the layer's fp32
 * accumulator itself: no rounding to the layer dtype, no finalize pass.  For a
 * caller whose next kernel reads the output anyway (a residual add + RMSNorm
 * that rounds it to the layer dtype first, chronos_add_rmsnorm's x_fp32). */
#define CHRONOS_FLAG_ACC_OUT 0x4

typedef struct ChronosMoeShape {
    int64_t num_tokens;  /* N = B*S (x.view(-1, H), moe_chronos.py:110-111); 0 is allowed */
    int32_t hidden;      /* H = hidden_size */
    int32_t num_experts; /* E = num_experts (routed) */
    int32_t top_k;       /* k = num_experts_per_tok, 1 <= k <= min(E, 16) */
    int32_t ffn;         /* F = moe_intermediate_size */
    int32_t num_shared;  /* S_h = num_shared_experts, 0..8 */
    int32_t dtype;       /* CHRONOS_DTYPE_* */
} ChronosMoeShape;

typedef struct ChronosMoeArgs {
    ChronosMoeShape shape;
    int32_t norm_topk; /* config.norm_topk_prob (moe_chronos.py:127-128) */
    int32_t flags;     /* CHRONOS_FLAG_* */

    const void* x;            /* [N, H] */
    const void* router_w;     /* [E, H]  gate.weight (moe_chronos.py:54) */
    const float* router_bias; /* [E] fp32 added to the logits, or NULL */

    /* Routed expert weights, stacked: slot p holds one expert.
     * w_gate/w_up: [P, F, H] (experts[e].gate_proj / up_proj .weight),
     * w_down: [P, H, F] (experts[e].down_proj.weight). */
    const void* w_gate;
    const void* w_up;
    const void* w_down;
    int32_t pool_slots;             /* P */
    const int32_t* slot_of_expert;  /* [E] slot of expert e, or NULL for slot == e.
                                       A negative slot means "not resident": the
                                       expert is treated as a = 0 (shared fallback). */
    /* Shared experts (moe_chronos.py:59-62): [S_h, F, H], [S_h, F, H], [S_h, H, F]. */
    const void* w_shared_gate;
    const void* w_shared_up;
    const void* w_shared_down;

    const float* avail; /* [E] effective availability a_e in [0, 1], or NULL for all 1 */

    /* Expert readiness (chronos/io/expert_store.py:480-543): when ready_flags is
     * non-NULL the grouped GEMMs wait, per SELECTED expert only, until
     * ready_flags[e] >= ready_epoch before reading its weights.  A wait longer
     * than spin_limit_ns records CHRONOS_ERR_EXPERT_NOT_READY in *status and
     * the kernel goes on with whatever the slot holds, so that expert's
     * contribution to this call is undefined (the status says so). */
    const int32_t* ready_flags;
    int32_t ready_epoch;
    int64_t spin_limit_ns; /* <= 0 selects the default (2 s) */

    /* Outputs. */
    void* y;              /* [N, H], required */
    void* router_probs;   /* [N, E] softmax probabilities in x dtype, or NULL */
    int32_t* topk_idx;    /* [N, k], or NULL (an input with CHRONOS_FLAG_PREROUTED) */
    float* topk_weight;   /* [N, k], or NULL (an input with CHRONOS_FLAG_PREROUTED) */
    int32_t* expert_counts; /* [E] tokens routed to each expert (all selections), or NULL */
    float* expert_mass;     /* [E] sum of top-k weights routed to each expert, or NULL */

    void* workspace;       /* >= chronos_moe_workspace_size(&shape) bytes, 256-byte aligned */
    size_t workspace_bytes;
    int32_t* status;       /* [1] device word; kernels write a CHRONOS_ERR_* code on a
                              device-side failure.  The caller zeroes it.  May be NULL. */
    int32_t max_ctas;      /* > 0: the persistent expert GEMMs use at most this many CTAs
                              (one per SM), leaving SMs free for concurrent work such as an
                              all-to-all on another stream; 0 = every SM */
} ChronosMoeArgs;

/* Bytes of workspace one chronos_moe_forward / chronos_moe_route call with
 * this shape needs (a function of the shape only, never of the routing).
 * Returns 0 for an invalid shape; chronos_moe_last_error() says why. */
CHRONOS_API size_t chronos_moe_workspace_size(const ChronosMoeShape* shape);

/* The whole layer (replaces ChronosMOEFeedForward.forward's arithmetic,
 * moe_chronos.py:110-268, both the standard and the masked branch). */
CHRONOS_API int chronos_moe_forward(const ChronosMoeArgs* args, void* cuda_stream);

/* Routing only (moe_chronos.py:112-128): writes topk_idx, topk_weight and,
 * when given, router_probs, expert_counts and expert_mass.  Used by hosts
 * that must see the selected experts before the expert GEMMs run (runtime
 * hooks `runtime_touch_expert` / `runtime_on_demand_loader`,
 * moe_chronos.py:228-248).  topk_idx and topk_weight are required. */
CHRONOS_API int chronos_moe_route(const ChronosMoeArgs* args, void* cuda_stream);

/* Largest workspace chronos_moe_forward_noalloc can serve: 16 MiB, enough
 * for decode batches (e.g. up to 64 tokens of a d_model 2048, 64-expert top-6
 * layer with d_ff 1408 and 2 shared experts). */
#define CHRONOS_NOALLOC_SCRATCH_BYTES (16u << 20)

/* chronos_moe_forward for callers that cannot allocate device memory.
 *
 * No counterpart in the reference (its layer allocates through PyTorch).
 * Some hosts cannot hand this library a workspace: an engine embedding the
 * layer through FFI with no handle on the GPU allocator, a runtime whose
 * device memory pool is sized once at start-up and handed out to its own
 * tensors only, or a real-time server that forbids cudaMalloc after start-up
 * because it synchronises the device and can fail under fragmentation.  This entry point
 * computes exactly what chronos_moe_forward computes, but ignores
 * args->workspace / args->workspace_bytes and uses one scratch array built
 * into the library (CHRONOS_NOALLOC_SCRATCH_BYTES of device memory, reserved
 * on every GPU that loads the library and held until the process exits).  It
 * calls no cudaMalloc, cudaFree or other allocating routine; the caller
 * still passes x, the weights and every output buffer.
 *
 * - Shapes whose chronos_moe_workspace_size exceeds the limit are rejected
 *   with CHRONOS_ERR_INVALID_ARG before anything is launched.
 * - The first call on a device looks up the scratch array's device address
 *   (with that device current); make that first call before any stream
 *   capture on the device.
 * - Every call shares the one array: calls that can overlap on the GPU (on
 *   different streams, or from different host threads without ordering)
 *   race on it and give undefined results.  Calls ordered on one stream are
 *   safe; each call re-initialises the scratch state it relies on. */
CHRONOS_API int chronos_moe_forward_noalloc(const ChronosMoeArgs* args, void* cuda_stream);

/* Message of the last failing call on this host thread ("" if none). */
CHRONOS_API const char* chronos_moe_last_error(void);

/* CHRONOS_MOE_ABI_VERSION of the loaded library. */
CHRONOS_API int chronos_moe_abi_version(void);

/* sizeof(ChronosMoeArgs) as compiled into the library, so an FFI binding can
 * check its mirror of the struct. */
CHRONOS_API size_t chronos_moe_args_size(void);

/* ---- measurement aids (no counterpart in the reference, which has no
 * profiling of this path) ---- */

/* Stages of one chronos_moe_forward call, in launch order. */
#define CHRONOS_STAGE_ROUTE 0
#define CHRONOS_STAGE_PLAN 1
#define CHRONOS_STAGE_SCATTER 2
#define CHRONOS_STAGE_GATEUP 3
#define CHRONOS_STAGE_ACT 4 /* no kernel: SiLU-mul runs in the gate/up epilogue */
#define CHRONOS_STAGE_DOWN 5
#define CHRONOS_STAGE_FINALIZE 6 /* empty when the down GEMM writes the output itself (direct
                                  output; shared experts last at large batches) */
#define CHRONOS_NUM_STAGES 7

/* After chronos_moe_profile_begin(max_calls), the next max_calls forward
 * calls made on this host thread record CUDA events on their stream around
 * each stage's kernel.  chronos_moe_profile_end synchronises on those events
 * and writes, per stage, the summed device milliseconds and the number of
 * kernel launches; it returns the number of calls recorded (or a negative
 * CHRONOS_ERR_* code) and ends profiling. */
CHRONOS_API int chronos_moe_profile_begin(int max_calls);
CHRONOS_API int chronos_moe_profile_end(float* stage_ms, int32_t* stage_launches, int max_stages);

/* Kernels launched by this library since it was loaded (all threads). */
CHRONOS_API uint64_t chronos_moe_kernel_launches(void);

/* Process-wide switches of the launch sequence (no counterpart in the
 * reference; the routing is bit-identical either way, the outputs agree to the
 * layer dtype's rounding):
 *   "fused_route"  1: a decode call (N <= 64 tokens, d_model <= 4096) routes in
 *                  ONE launch, a thread-block cluster that computes the chunk
 *                  partials, the selection and the plan; 0 (default): the logit
 *                  kernel and the select + plan kernel.
 *   "two_phase_combine"  1: a large call whose shared experts run last in the
 *                  token-major down GEMM combines in two phases: routed units
 *                  store coef * expert(x) rounded to the layer dtype per slot,
 *                  the shared units sum each token's slots in choice order
 *                  (deterministic; no fp32 accumulator); 0 (default, measured
 *                  faster): fp32 reduce-adds into an accumulator.
 *   "fold_finalize"  1: a call below 1024 tokens with shared experts writes
 *                  its output from the down GEMM, each 128-column tile
 *                  converted by the CTA whose contribution completes it; 0
 *                  (default, measured faster): a separate finalize kernel.
 *   "down_split_target"  -1 (default): the weight-major down GEMM of a decode
 *                  call halves K once its unsplit work units fill at least two
 *                  rounds of the SMs; n in 0..64: split until it has about n
 *                  units per SM (0: no split).
 *   "gateup_split"  1: a decode call (N <= 64) whose gate/up units would not
 *                  cover the SMs splits the routed units along K (2 or 4 ways);
 *                  the split completing a tile sums the fp32 partials in split
 *                  order and applies SiLU-mul; 0 (default, measured faster): never.
 *                  Set it before sizing a workspace (it reserves the partials).
 *   "select_plan_one_block"  1: decode calls of 9..32 tokens select and plan
 *                  in one block of a warp per token; 0 (default, measured
 *                  faster): blocks of 8 tokens and a last-block plan.
 *   "gateup_prefetch_mb"  0..1024, default 128: in a decode call that leaves
 *                  an expert unselected with probability (1 - k/E)^N <= 10 %
 *                  and has no slot_of_expert map, each gate/up CTA past the
 *                  shared experts' units prefetches into L2, while the routing
 *                  kernels run, the first k tiles of the routed unit it would
 *                  run first if every available expert were selected (at most
 *                  this many MB over all CTAs); 0: off.  A hint only.
 *   "model_pdl"  1: chronos_add_rmsnorm, the attention decode kernels,
 *                  chronos_lookahead_forward and chronos_argmax_rows launch as
 *                  programmatic dependents of the previous kernel on the stream
 *                  (their blocks start early and wait for it before touching
 *                  memory); 0 (default, measured faster): ordinary stream order.
 * Returns CHRONOS_OK, or CHRONOS_ERR_INVALID_ARG for an unknown name or a value
 * out of range. */
CHRONOS_API int chronos_moe_set_option(const char* name, int64_t value);

#ifdef __cplusplus
}
#endif

#endif /* CHRONOS_MOE_H_ */
