/*
 * Batch driver around the reference sampler itself (Sain-Kai/noel
 * src/sampler.c, compiled from the reference sources by oracle/Makefile into
 * oracle/_ref/libsampler_ref.so).  TEST INFRASTRUCTURE ONLY: it is used to
 * pin the oracle restatement, to make the golden fixtures and as the timed
 * CPU baseline; the shipped library never loads it.
 *
 * Each row gets its own noel_sampler_t whose rng_state is set from the
 * caller's per-row state (sampler.h:27-28), so every row draws from an
 * independent, reproducible stream.  After each call the reference leaves
 * its sorted candidate list in sampler->candidates (sampler.c:133-152);
 * the driver copies the first n_list entries out together with the
 * recomputed candidate count.
 */
#include "sampler.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int ref_sampler_sizeof(void) { return (int)sizeof(noel_sampler_t); }
int ref_config_sizeof(void) { return (int)sizeof(noel_sampler_config_t); }

int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/*
 * cfg: the reference config; logits row b at logits + b*ld (copied unless
 * in_place); history row b at hist + b*hld with H entries (hist may be NULL);
 * rng[2b..2b+1] in/out.  num_cands[b] (may be NULL) receives the count of
 * candidates the reference built; cand_ids/cand_vals[b*n_list + i] (may be
 * NULL) its sorted list, -1/0 padded.
 */
void ref_sample_batch(const noel_sampler_config_t *cfg, const float *logits, int B,
                      int V, size_t ld, const int32_t *hist, int H, size_t hld,
                      uint64_t *rng, int32_t *ids, int32_t *num_cands,
                      int32_t *cand_ids, float *cand_vals, int n_list, int in_place,
                      int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        noel_sampler_t s;
        noel_sampler_config_t c = *cfg;
        c.seed = 1; /* any non-zero seed: the state is overwritten per row */
        noel_sampler_init(&s, &c, V);
        float *row = in_place ? NULL : (float *)malloc((size_t)V * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int b = 0; b < B; ++b) {
            float *x = in_place ? (float *)logits + (size_t)b * ld : row;
            if (!in_place) memcpy(row, logits + (size_t)b * ld, (size_t)V * sizeof(float));
            s.config = *cfg;
            s.rng_state[0] = rng[2 * (size_t)b];
            s.rng_state[1] = rng[2 * (size_t)b + 1];
            const int32_t *h = hist ? hist + (size_t)b * hld : NULL;
            ids[b] = noel_sampler_sample(&s, x, V, h, hist ? H : 0);
            rng[2 * (size_t)b] = s.rng_state[0];
            rng[2 * (size_t)b + 1] = s.rng_state[1];
            if (num_cands || cand_ids) {
                int n = 0;
                if (cfg->temperature > 1e-4f) {
                    /* the reference's own predicate on the penalised row */
                    float mx = x[0];
                    for (int i = 1; i < V; ++i) if (x[i] > mx) mx = x[i];
                    float inv_t = 1.0f / cfg->temperature;
                    for (int i = 0; i < V; ++i)
                        if ((x[i] - mx) * inv_t > -15.0f) ++n;
                    if (n == 0) n = 1;
                }
                if (num_cands) num_cands[b] = n;
                if (cand_ids) {
                    for (int i = 0; i < n_list; ++i) {
                        int ok = i < n;
                        cand_ids[(size_t)b * n_list + i] = ok ? s.candidates[i].id : -1;
                        if (cand_vals)
                            cand_vals[(size_t)b * n_list + i] = ok ? s.candidates[i].val : 0.0f;
                    }
                }
            }
        }
        free(row);
        noel_sampler_free(&s);
    }
}

/* Reference init/set_config/random_f32 round trip for the ABI tests. */
void ref_init_state(const noel_sampler_config_t *cfg, int use_null_cfg, uint64_t out_state[2],
                    noel_sampler_config_t *out_cfg) {
    noel_sampler_t s;
    noel_sampler_init(&s, use_null_cfg ? NULL : cfg, 16);
    out_state[0] = s.rng_state[0];
    out_state[1] = s.rng_state[1];
    if (out_cfg) *out_cfg = s.config;
    noel_sampler_free(&s);
}
