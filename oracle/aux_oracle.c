/*
 * Oracle for the paths next to the sampler: a CPU restatement of the
 * reference's MoE router (Sain-Kai/noel src/sparsity.c:46-79), used ONLY as
 * the checker by tests/ and bench.py's CPU leg.  Nothing in the shipped
 * library links, loads or calls this code.
 *
 * Parity pinning: checked against the reference's known-answer test
 * (tests/test_engine.c:128-142) and against the reference's own sparsity.c,
 * compiled from its sources into oracle/_ref/libaux_ref.so by
 * oracle/Makefile, on seeded inputs (tests/test_router.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

/* sparsity.c:46-79 for tokens t in [0, T): logits row t at logits + t * ld;
 * ids / weights [T][top_k]. */
void orc_route_top_k(const float *logits, int T, int E, size_t ld, int top_k, int32_t *ids, float *weights) {
    for (int t = 0; t < T; ++t) {
        const float *x = logits + (size_t)t * ld;
        int32_t *id = ids + (size_t)t * top_k;
        float *w = weights + (size_t)t * top_k;
        for (int k = 0; k < top_k; ++k) { /* sparsity.c:48-51 */
            id[k] = -1;
            w[k] = -1e9f;
        }
        for (int e = 0; e < E; ++e) { /* sparsity.c:53-65: first slot it strictly beats */
            const float v = x[e];
            for (int k = 0; k < top_k; ++k) {
                if (v > w[k]) {
                    for (int m = top_k - 1; m > k; --m) {
                        id[m] = id[m - 1];
                        w[m] = w[m - 1];
                    }
                    id[k] = e;
                    w[k] = v;
                    break;
                }
            }
        }
        const float mx = w[0]; /* sparsity.c:67-78 */
        float sum = 0.0f;
        for (int k = 0; k < top_k; ++k) {
            w[k] = expf(w[k] - mx);
            sum += w[k];
        }
        const float inv = sum > 0.0f ? (1.0f / sum) : 0.0f;
        for (int k = 0; k < top_k; ++k) w[k] *= inv;
    }
}
