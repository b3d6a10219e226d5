/*
 * The pipeline's sibling sampler on the GPU: the reference's
 * aether_postreq_apply_penalties, aether_postreq_grammar_mask and
 * aether_postreq_sample (Sain-Kai/noel include/pipeline_stages.h:58-67,
 * src/pipeline_stages.c:64-189).  Its semantics differ from
 * noel_sampler_sample: a softmax over the whole vocabulary, top-k capped at
 * 256 and taken by probability, an absolute top-p over the normalised
 * probabilities, and a uniform from the C library's rand().
 */
#ifndef NOEL_POSTREQ_H
#define NOEL_POSTREQ_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same layout as the reference's aether_sampling_params_t
 * (pipeline_stages.h:13-20). */
typedef struct {
    float temperature;
    float top_p;
    int top_k;
    float repetition_penalty;
    int repetition_window;
    bool grammar_enforce_json;
} noel_postreq_params_t;

/*
 * aether_postreq_sample (pipeline_stages.c:103-189) on B rows of fp32 logits
 * in device memory (row b at d_logits + b * ld), each row modified in place
 * as the reference modifies its buffer (non-greedy rows end up holding the
 * softmax probabilities).  d_uniform[b] is the row's uniform, the
 * reference's (float)rand() / (float)RAND_MAX; d_ids[b] receives the token
 * (-1 when no probability of the row is a number, as in the reference).
 * Token ids equal the reference's except where the uniform lies within
 * rounding of a cumulative-probability boundary; probabilities are within
 * 1e-5 relative (CUDA's single-precision expf, within 2 units in the last
 * place of the C library's).  Asynchronous on stream.
 */
int noel_postreq_sample_batch(const noel_postreq_params_t *params, float *d_logits, int batch, int vocab,
                              size_t ld, const float *d_uniform, int32_t *d_ids, void *stream);

/* aether_postreq_apply_penalties (pipeline_stages.c:64-79) on B rows:
 * history row b at d_history + b * hld, history_len ids. */
int noel_postreq_apply_penalties_batch(float *d_logits, int batch, int vocab, size_t ld, const int32_t *d_history,
                                       int history_len, size_t hld, float penalty, int window, void *stream);

/* aether_postreq_grammar_mask (pipeline_stages.c:81-94) on B rows: the
 * state of row b is d_fsm_state[b], or fsm_state for every row when
 * d_fsm_state is NULL. */
int noel_postreq_grammar_mask_batch(float *d_logits, int batch, int vocab, size_t ld, const int32_t *d_fsm_state,
                                    int fsm_state, void *stream);

/*
 * Drop-in for aether_postreq_sample on one row, host or device logits:
 * draws its uniform from rand() on the calling thread exactly where the
 * reference does (non-greedy calls only), samples on the GPU and leaves the
 * row as the reference would.  Returns the token; on a device failure 0,
 * with noel_sampler_cuda_last_error() saying why.
 */
int32_t noel_postreq_sample(float *logits, int vocab_size, const noel_postreq_params_t *params);

#ifdef __cplusplus
}
#endif

#endif /* NOEL_POSTREQ_H */
