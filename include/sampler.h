/*
 * Token sampler C ABI, unchanged from the reference so existing callers link
 * against libnoel_sampler_cuda.so without edits.
 *
 * Every declaration below keeps the reference's name, argument meaning, struct
 * layout and error behaviour (Sain-Kai/noel include/sampler.h:12-61); the
 * bodies are new and run the sampling on a B200 (noel_b200/csrc/).
 */
#ifndef NOEL_SAMPLER_H
#define NOEL_SAMPLER_H

#include <stdint.h>
#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces noel_sampler_config_t, include/sampler.h:12-19 (32 bytes). */
typedef struct {
    float temperature;         /* <= 1e-4: greedy argmax; else stochastic */
    float top_p;               /* nucleus threshold; applied when 0 < top_p < 1 */
    int top_k;                 /* candidate limit; <= 0 disables */
    float repetition_penalty;  /* > 1.0 penalises tokens of the history */
    int repetition_window;     /* most recent tokens to scan (0 = whole history) */
    uint64_t seed;             /* PRNG seed (0 = seed from the clock) */
} noel_sampler_config_t;

/* Replaces noel_token_prob_t, include/sampler.h:21-24. */
typedef struct {
    int32_t id;
    float val;
} noel_token_prob_t;

/* Replaces noel_sampler_t, include/sampler.h:26-31.  Callers embed it by
 * value and write config fields directly; device state is kept outside it. */
typedef struct {
    noel_sampler_config_t config;
    uint64_t rng_state[2];
    noel_token_prob_t *candidates;
    int candidate_capacity;
} noel_sampler_t;

/* Replaces include/sampler.h:36 (src/sampler.c:23-52).  NULL cfg gives
 * temperature 0.7, top-p 0.9, top-k 40, penalty 1.1, window 64, clock seed. */
void noel_sampler_init(noel_sampler_t *sampler, const noel_sampler_config_t *cfg, int max_vocab);

/* Replaces include/sampler.h:41 (src/sampler.c:54-61). */
void noel_sampler_free(noel_sampler_t *sampler);

/* Replaces include/sampler.h:46 (src/sampler.c:63-70): reseeds if seed != 0. */
void noel_sampler_set_config(noel_sampler_t *sampler, const noel_sampler_config_t *cfg);

/*
 * Replaces include/sampler.h:52-56 (src/sampler.c:80-192).  logits may be a
 * host or a device pointer; penalised entries are written back in place.
 * Returns 0 on invalid arguments, like the reference; a device failure also
 * returns 0 and is reported by noel_sampler_cuda_last_error().
 * After the call, candidates[0..n) holds the list the token was drawn from
 * (id, unnormalised weight), sorted, with n = min(n_final, capacity).
 */
int32_t noel_sampler_sample(noel_sampler_t *sampler,
                            float *logits,
                            int vocab_size,
                            const int32_t *history,
                            int history_len);

/* Replaces include/sampler.h:61 (src/sampler.c:17-21): one xorshift128+ step
 * of the sampler's state, as a 24-bit uniform in [0, 1). */
float noel_sampler_random_f32(noel_sampler_t *sampler);

#ifdef __cplusplus
}
#endif

#endif /* NOEL_SAMPLER_H */
