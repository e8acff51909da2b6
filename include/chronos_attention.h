/*
 * chronos_attention.h — C ABI of the hybrid-attention decode kernels.
 *
 * Replaces the one-token (S = 1, cached) step of the two attention modules of
 * FonaTech/Project_Chronos's hybrid attention, and the residual add + RMSNorm
 * around them:
 *
 *   chronos_mla_decode  MLAAttention.forward with a cache
 *                       (chronos/model/hybrid_attention.py:116-179), even layers;
 *   chronos_sw_decode   SlidingWindowAttention.forward with a cache
 *                       (chronos/model/hybrid_attention.py:213-258), odd layers;
 *   chronos_add_rmsnorm ChronosBlock's `hidden + residual` followed by
 *                       RMSNorm (chronos/model/model_chronos.py:47-56; minimind
 *                       RMSNorm: x * rsqrt(mean(x^2) + eps) * weight in fp32,
 *                       rounded to the input type).
 *
 * The caller runs the input projections (one GEMM with the concatenated
 * projection weights) and o_proj; each decode kernel takes the projection
 * output of its B tokens and does everything between: the per-head RMSNorms,
 * RoPE, the cache append and the attention, in one launch.
 *
 * MLA (one block per (kv head, row)).  proj = [q_nope (nH*nope) | q_rope
 * (nH*R) | kv_down (L)] per row.  The cache holds the normalised latent
 * c_t [B, max_len, L] and the rotated rope keys krope_t [B, max_len, nKV, R]
 * (k_rope_proj(c_t) rotated at position t), so a step never recomputes keys
 * or values of past tokens: with W_kn the k_nope_proj rows and W_v the v_proj
 * rows of the head's kv group,
 *     score_t = ((W_kn^T q_nope) . c_t + q_rope . krope_t) / sqrt(head_dim)
 *     out     = W_v (sum_t softmax(score)_t c_t)
 * which is q.k_t and sum_t p_t v_t of the reference with k and v expanded
 * from the latent.  RoPE uses the first R columns of the model's cos/sin
 * tables at the token's position, as the reference slices them.
 *
 * Sliding window (one block per (kv head, row)).  proj = [q (nH*D) | k
 * (nKV*D) | v (nKV*D)] per row.  The cache is a ring of `window` slots per
 * row: the token at position p goes to slot p % window; a step attends to
 * min(p + 1, window) slots.  As in the reference, the rotary position of a
 * new token is the cache length before it, min(p, window)
 * (hybrid_attention.py:217-234: the cached keys are cut to the window, and
 * past_len is read from the cut cache).
 *
 * `pos` is a DEVICE int32: the position of the new token (= tokens already
 * cached), the same for every row, read by the kernels so that a captured
 * CUDA graph replays correctly as it advances.  Conventions as in
 * chronos_moe.h (return codes, stream-ordered, nothing allocated).
 */
#ifndef CHRONOS_ATTENTION_H_
#define CHRONOS_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#include "chronos_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ChronosAttnArgs {
    int32_t batch;        /* B rows, one new token each */
    int32_t heads;        /* nH */
    int32_t kv_heads;     /* nKV, divides nH; nH/nKV <= 8 */
    int32_t head_dim;     /* D, even, <= 256 */
    int32_t rope_dim;     /* MLA: R (even, < D, nope = D - R); sliding window: D */
    int32_t latent;       /* MLA: L <= 256; sliding window: 0 */
    int32_t window;       /* sliding window: ring slots per row (>= 1); MLA: 0 */
    int32_t max_len;      /* MLA: cache positions per row (<= 8192); SW: = window */
    int32_t table_len;    /* rows of the cos/sin tables */
    int32_t dtype;        /* CHRONOS_DTYPE_* of proj, weights, tables, caches and out */
    float eps;            /* rms_norm_eps */
    const int32_t* pos;   /* device: position of the new token */
    const void* proj;     /* [B, proj_width] input-projection output */
    const void* norm_q;   /* MLA: q_nope_norm.weight [nope]; SW: q_norm.weight [D] */
    const void* norm_q2;  /* MLA: q_rope_norm.weight [R];    SW: k_norm.weight [D] */
    const void* norm_kv;  /* MLA: kv_down_norm.weight [L];   SW: NULL */
    const void* w_krope;  /* MLA: k_rope_proj.weight [nKV*R, L]; SW: NULL */
    const void* w_knope;  /* MLA: k_nope_proj.weight [nKV*nope, L]; SW: NULL */
    const void* w_v;      /* MLA: v_proj.weight [nKV*D, L]; SW: NULL */
    const void* cos;      /* [table_len, D] */
    const void* sin;      /* [table_len, D] */
    void* cache_a;        /* MLA: latent [B, max_len, L];     SW: keys [B, window, nKV, D] */
    void* cache_b;        /* MLA: krope [B, max_len, nKV, R]; SW: values [B, window, nKV, D] */
    void* out;            /* [B, nH*D] attention output (o_proj input) */
} ChronosAttnArgs;

CHRONOS_API int chronos_mla_decode(const ChronosAttnArgs* args, void* cuda_stream);
CHRONOS_API int chronos_sw_decode(const ChronosAttnArgs* args, void* cuda_stream);

typedef struct ChronosNormArgs {
    int64_t rows;
    int32_t width;        /* <= 16384 */
    int32_t dtype;
    float eps;
    int32_t x_fp32;       /* 1: x is fp32 (e.g. a layer's fp32 accumulator, CHRONOS_FLAG_ACC_OUT),
                             rounded to dtype as it is read; 0: x is dtype */
    const void* x;        /* [rows, width] */
    const void* residual; /* [rows, width] added to x first, or NULL */
    void* sum_out;        /* x + residual (rounded), or NULL; may alias x or residual */
    const void* weight;   /* [width] */
    void* out;            /* RMSNorm(x + residual) * weight */
} ChronosNormArgs;

CHRONOS_API int chronos_add_rmsnorm(const ChronosNormArgs* args, void* cuda_stream);

/* The index of the first maximal value of every row of x [rows, cols] (NaN
 * counts as the maximum), into out [rows] (int64): the greedy pick of a decode
 * step, torch.argmax(logits, dim=-1).  One block per row. */
CHRONOS_API int chronos_argmax_rows(const void* x, int64_t rows, int32_t cols, int32_t dtype, int64_t* out,
                                    void* cuda_stream);

CHRONOS_API size_t chronos_attn_args_size(void);
CHRONOS_API size_t chronos_norm_args_size(void);

#ifdef __cplusplus
}
#endif

#endif /* CHRONOS_ATTENTION_H_ */
