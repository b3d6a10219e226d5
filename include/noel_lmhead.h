/*
 * The LM head feeding the sampler on the GPU: the reference's final
 * projection and sampling call (Sain-Kai/noel src/engine.c:377-387:
 * noel_gemv_quantized, src/dequant.c:412-470, then noel_sampler_sample) for a
 * batch of tokens whose hidden states and output weights are on the device.
 */
#ifndef NOEL_LMHEAD_H
#define NOEL_LMHEAD_H

#include <stddef.h>
#include <stdint.h>

#include "sampler.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Row formats of the output weight, with the reference's GGML type ids
 * (include/gguf_loader.h:20-48). */
enum { NOEL_HEAD_F32 = 0, NOEL_HEAD_F16 = 1, NOEL_HEAD_BF16 = 30 };

/*
 * d_logits[b][v] = d_weight[v] . d_hidden[b] for v < vocab, b < batch, in
 * noel_gemv_quantized's summation order (the logits equal the reference's bit
 * for bit), then noel_sampler_sample_batch on those logits in the same stream
 * (histories, RNG states, ids and probabilities as there).  d_weight rows are
 * ldw elements apart and 16-byte aligned; hidden_dim must be a multiple of 8;
 * d_hidden rows are ldh floats apart (16-byte aligned).  d_logits [batch][vocab]
 * receives the logits (they stay in L2 for the sampler when batch x vocab x 4
 * bytes fits).  The weights are read once per eight tokens.  Returns NOEL_OK or
 * a negative status (noel_sampler_cuda_last_error_message() says why).
 */
int noel_lmhead_sample(const noel_sampler_config_t *cfg, const void *d_weight, int weight_type, size_t ldw,
                       const float *d_hidden, size_t ldh, int batch, int hidden_dim, int vocab,
                       const int32_t *d_history, int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                       float *d_probs, float *d_logits, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NOEL_LMHEAD_H */
