/* Model-harness entry points of libce_b200.so (batch-1 mixture-of-experts
 * GEMVs for the gpt-oss-20b-shaped decoder of benchmark config 2).  They are
 * not part of the eviction overlay: the reference runs that model inside
 * SGLang, whose MoE layers have no counterpart here.  Conventions as in
 * ce_api.h (device pointers, a cudaStream_t as void*, int status). */
#ifndef CE_MODEL_H
#define CE_MODEL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* g[k, i] = silu(W1[ids[k], i] . x) * (W1[ids[k], inter + i] . x) for
 * k < num_experts_chosen, i < inter.  x [dim] bf16 (dim a multiple of 8,
 * <= 8192), W1 [num_experts, 2 * inter, dim] bf16 row-major, g [k, inter]
 * bf16.  An id outside [0, num_experts) flags CE_EW_INDEX and leaves its row
 * of g unwritten. */
int ce_moe_gate_up(const void* x, const void* w1, const int32_t* ids, int32_t num_experts_chosen,
                   int32_t num_experts, int32_t inter, int32_t dim, void* g, int32_t* err, void* stream);

/* x[d] += sum_k weights[k] * (W2[ids[k], d] . g[k]) for d < dim: the experts'
 * down projections, weighted by the router and added to the residual x (bf16,
 * in place).  W2 [num_experts, dim, inter] bf16 row-major (inter a multiple
 * of 8), weights [k] fp32. */
int ce_moe_down(const void* g, const void* w2, const int32_t* ids, const float* weights,
                int32_t num_experts_chosen, int32_t num_experts, int32_t inter, int32_t dim, void* x,
                int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CE_MODEL_H */
