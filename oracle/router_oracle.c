/*
 * router_oracle.c — CPU restatement of the Chronos MoE router, TEST
 * INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU legs may load this file's library; it is the checker, never the
 * product.
 *
 * Restates chronos/model/moe_chronos.py:112 (gate GEMM + softmax) and
 * :124-128 (top-k + optional renormalisation) under the bit-exact routing
 * contract of include/chronos_moe.h:
 *   partial[c] = fmaf chain over h in [128c, min(128c + 128, H)), from 0.0f
 *   logit      = ((0.0f + partial[0]) + partial[1]) + ... (+ bias[e])
 *   rank experts by (logit desc, index asc), keep k
 *   prob = softmax(logit) in fp32; weight = prob of the chosen experts,
 *   divided by (sum + 1e-20) when norm_topk (moe_chronos.py:127-128).
 * The chunk chains and their in-order sum are exactly the operations the CUDA
 * router performs, so top-k indices match bit for bit.  Softmax uses libm
 * expf, so probabilities/weights match the device within a few ulp (compared
 * with a tolerance, never bitwise).
 *
 * Inputs are fp32 arrays holding the operand values (bf16/fp16 inputs are
 * widened exactly before the call).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ROUTER_CHUNK 128

static float logit_of(const float* xr, const float* wr, int h) {
    float total = 0.0f;
    for (int c0 = 0; c0 < h; c0 += ROUTER_CHUNK) {
        const int c1 = c0 + ROUTER_CHUNK < h ? c0 + ROUTER_CHUNK : h;
        float acc = 0.0f;
        for (int i = c0; i < c1; ++i) acc = fmaf(xr[i], wr[i], acc);
        total = total + acc;
    }
    return total;
}

/* logits [N, E] only: the bit-exact part of the contract. */
void oracle_router_logits(const float* x, const float* w, const float* bias,
                          int64_t n, int h, int e, float* logits) {
    for (int64_t t = 0; t < n; ++t) {
        const float* xr = x + t * (int64_t)h;
        for (int j = 0; j < e; ++j) {
            float acc = logit_of(xr, w + (int64_t)j * h, h);
            if (bias) acc = acc + bias[j];
            logits[t * e + j] = acc;
        }
    }
}

/* Full routing.  idx [N, k] int32 in rank order, weight [N, k] fp32,
 * probs [N, E] fp32 (may be NULL), logits [N, E] fp32 (may be NULL). */
void oracle_route(const float* x, const float* w, const float* bias, int64_t n,
                  int h, int e, int k, int norm_topk, int32_t* idx,
                  float* weight, float* probs, float* logits_out) {
    float* lg = (float*)malloc(sizeof(float) * (size_t)e);
    float* pr = (float*)malloc(sizeof(float) * (size_t)e);
    unsigned char* taken = (unsigned char*)malloc((size_t)e);
    for (int64_t t = 0; t < n; ++t) {
        oracle_router_logits(x + t * (int64_t)h, w, bias, 1, h, e, lg);
        float m = lg[0];
        for (int j = 1; j < e; ++j) m = lg[j] > m ? lg[j] : m;
        float s = 0.0f;
        for (int j = 0; j < e; ++j) {
            pr[j] = expf(lg[j] - m);
            s += pr[j];
        }
        for (int j = 0; j < e; ++j) pr[j] = pr[j] / s;
        memset(taken, 0, (size_t)e);
        float wsum = 0.0f;
        for (int r = 0; r < k; ++r) {
            int best = -1;
            for (int j = 0; j < e; ++j) {
                if (taken[j]) continue;
                if (best < 0 || lg[j] > lg[best]) best = j; /* strict >: ties keep the lower index */
            }
            taken[best] = 1;
            idx[t * k + r] = best;
            weight[t * k + r] = pr[best];
            wsum += pr[best];
        }
        if (norm_topk) {
            for (int r = 0; r < k; ++r) weight[t * k + r] = weight[t * k + r] / (wsum + 1e-20f);
        }
        if (probs) memcpy(probs + t * e, pr, sizeof(float) * (size_t)e);
        if (logits_out) memcpy(logits_out + t * e, lg, sizeof(float) * (size_t)e);
    }
    free(lg);
    free(pr);
    free(taken);
}
