/*
 * MoE top-k routing on the GPU: the reference's aether_route_top_k
 * (Sain-Kai/noel include/sparsity.h:33, src/sparsity.c:46-79) for a batch of
 * tokens whose gate logits are in device memory.
 */
#ifndef NOEL_ROUTER_H
#define NOEL_ROUTER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as the reference's moe_routing_t (sparsity.h:12-15). */
typedef struct {
    int32_t expert_id;
    float weight;
} noel_moe_routing_t;

/*
 * d_routing[t * top_k + k] = aether_route_top_k(d_gate_logits + t * ld,
 * n_experts, top_k)[k] for t in [0, n_tokens): the top_k experts by (logit
 * desc, id asc) among logits strictly above -1e9 (then (-1, weight of a -1e9
 * slot) slots), with softmax weights over the selected logits.  Expert ids
 * are exact; weights are within 1e-5 relative of the reference's (CUDA's
 * single-precision expf, within 2 units in the last place of the C
 * library's).  1 <= n_experts <= 256, 1 <= top_k <= 64,
 * ld >= n_experts.  Returns NOEL_OK or a negative status
 * (noel_sampler_cuda_last_error_message() says why).  Asynchronous on stream.
 */
int noel_moe_route_top_k(const float *d_gate_logits, int n_tokens, int n_experts, size_t ld, int top_k,
                         noel_moe_routing_t *d_routing, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NOEL_ROUTER_H */
