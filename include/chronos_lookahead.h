/*
 * chronos_lookahead.h — C ABI of the fused lookahead-router kernel.
 *
 * Replaces LookaheadRouter.forward (chronos/model/lookahead_router.py:36-55):
 *
 *   logits = W2 . silu(W1 . x)        W1 [H/4, H], W2 [E*K, H/4], bias-free
 *   probs[t, s, :] = softmax(logits[t, s*E : (s+1)*E])    s = 0..K-1
 *
 * with K = lookahead_steps + 1 (s = 0 the current step, s >= 1 the predicted
 * future steps).  One launch per call: both projections, the SiLU and the K
 * softmaxes of a group of up to 8 tokens run in one thread-block cluster (W1's
 * rows split over its CTAs), accumulating in fp32 and rounding once to the
 * output type.  Conventions as in chronos_moe.h.
 */
#ifndef CHRONOS_LOOKAHEAD_H_
#define CHRONOS_LOOKAHEAD_H_

#include <stddef.h>
#include <stdint.h>

#include "chronos_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ChronosLookaheadArgs {
    int64_t num_tokens;   /* N = B*S */
    int32_t hidden;       /* H, 1..8192 */
    int32_t inner;        /* H/4 (proj[0] out_features), 1..2048 */
    int32_t num_experts;  /* E */
    int32_t steps;        /* K = lookahead_steps + 1, E*K <= 4096 */
    int32_t dtype;        /* CHRONOS_DTYPE_* of x, the weights and probs */
    const void* x;        /* [N, H] */
    const void* w1;       /* [inner, H]   proj[0].weight */
    const void* w2;       /* [E*K, inner] proj[2].weight */
    void* probs;          /* [N, K, E] out */
} ChronosLookaheadArgs;

CHRONOS_API int chronos_lookahead_forward(const ChronosLookaheadArgs* args, void* cuda_stream);

/* sizeof(ChronosLookaheadArgs) as compiled into the library. */
CHRONOS_API size_t chronos_lookahead_args_size(void);

#ifdef __cplusplus
}
#endif

#endif /* CHRONOS_LOOKAHEAD_H_ */
