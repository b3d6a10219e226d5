/*
 * CPU restatement of the reference token sampler (Sain-Kai/noel
 * src/sampler.c).  TEST INFRASTRUCTURE ONLY: this is the oracle the CUDA
 * path is checked against; the shipped library never links or calls it.
 *
 * Every stage cites the reference lines it restates.  The arithmetic is the
 * reference's, operation for operation, in fp32 with glibc's expf, so the
 * results are bit-identical to the reference built with gcc on the same
 * machine (checked by tests/test_oracle.py against oracle/_ref/).
 */
#include "sampler_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* sampler.c:8-15: xorshift128+ with shifts 23, 18, 5; returns s[1] + s0. */
uint64_t orc_xorshift128plus(uint64_t s[2]) {
    uint64_t a = s[0];
    const uint64_t b = s[1];
    s[0] = b;
    a ^= a << 23;
    s[1] = a ^ b ^ (a >> 18) ^ (b >> 5);
    return s[1] + b;
}

/* sampler.c:17-21: top 24 bits of the step, scaled by 2^-24. */
float orc_random_f32(uint64_t s[2]) {
    uint64_t v = orc_xorshift128plus(s);
    return (float)(v >> 40) * (1.0f / 16777216.0f);
}

/* sampler.c:42-47 (init with a non-zero seed) and :66-69 (set_config). */
void orc_seed_state(uint64_t seed, uint64_t s[2]) {
    s[0] = seed;
    s[1] = seed ^ 0x9E3779B97F4A7C15ULL;
    if (s[0] == 0 && s[1] == 0) {
        s[0] = 123456789ULL;
        s[1] = 987654321ULL;
    }
}

/* sampler.c:87-103: penalty per occurrence, in place, inside the window. */
static void orc_penalize(const orc_config_t *cfg, float *logits, int vocab,
                         const int32_t *history, int history_len) {
    if (!(cfg->repetition_penalty > 1.0f) || !history || history_len <= 0) return;
    int w = cfg->repetition_window;
    int first = (w > 0 && w < history_len) ? history_len - w : 0;
    const float rep = cfg->repetition_penalty;
    for (int i = first; i < history_len; ++i) {
        int32_t t = history[i];
        if (t < 0 || t >= vocab) continue;
        float x = logits[t];
        logits[t] = (x > 0.0f) ? x / rep : x * rep;
    }
}

/* sampler.c:106-115: first index holding the strict running maximum. */
static int32_t orc_argmax(const float *logits, int vocab) {
    int32_t best = 0;
    float bv = logits[0];
    for (int i = 1; i < vocab; ++i)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    return best;
}

/*
 * Stable ordering of candidates by value, largest first (sampler.c:72-78 and
 * :152).  glibc's qsort sorts this array with a stable merge, so among equal
 * values the candidate built first -- the lower id -- stays first; this
 * bottom-up merge gives the same order.
 */
static void orc_sort_desc(int32_t *ids, float *vals, int n, int32_t *tid, float *tval) {
    for (int width = 1; width < n; width *= 2) {
        for (int lo = 0; lo < n; lo += 2 * width) {
            int mid = lo + width < n ? lo + width : n;
            int hi = lo + 2 * width < n ? lo + 2 * width : n;
            int a = lo, b = mid, o = lo;
            while (a < mid && b < hi) {
                /* take from the right run only if strictly larger */
                if (vals[b] > vals[a]) { tid[o] = ids[b]; tval[o++] = vals[b++]; }
                else { tid[o] = ids[a]; tval[o++] = vals[a++]; }
            }
            while (a < mid) { tid[o] = ids[a]; tval[o++] = vals[a++]; }
            while (b < hi) { tid[o] = ids[b]; tval[o++] = vals[b++]; }
        }
        memcpy(ids, tid, (size_t)n * sizeof(int32_t));
        memcpy(vals, tval, (size_t)n * sizeof(float));
    }
}

int32_t orc_sample_row(const orc_config_t *cfg, float *logits, int vocab,
                       const int32_t *history, int history_len, uint64_t rng[2],
                       int32_t *cand_ids, float *cand_vals, orc_row_diag_t *diag) {
    orc_row_diag_t d;
    memset(&d, 0, sizeof(d));
    if (!cfg || !logits || vocab <= 0) {           /* sampler.c:85 */
        if (diag) *diag = d;
        return 0;
    }
    orc_penalize(cfg, logits, vocab, history, history_len);

    if (cfg->temperature <= 1e-4f) {                /* sampler.c:106 */
        d.greedy = 1;
        d.id = orc_argmax(logits, vocab);
        d.max_val = logits[d.id];
        if (diag) *diag = d;
        return d.id;
    }

    /* sampler.c:119-124: max over the penalised row (strict >, from [0]). */
    float mx = logits[0];
    for (int i = 1; i < vocab; ++i)
        if (logits[i] > mx) mx = logits[i];
    d.max_val = mx;

    int32_t *ids = cand_ids ? cand_ids : (int32_t *)malloc((size_t)vocab * sizeof(int32_t));
    float *vals = cand_vals ? cand_vals : (float *)malloc((size_t)vocab * sizeof(float));

    /* sampler.c:132-143: scaled difference, the -15 cut, unnormalised expf. */
    const float inv_t = 1.0f / cfg->temperature;
    int n = 0;
    for (int i = 0; i < vocab; ++i) {
        float diff = (logits[i] - mx) * inv_t;
        if (diff > -15.0f) { ids[n] = i; vals[n] = expf(diff); ++n; }
    }
    if (n == 0) { ids[0] = 0; vals[0] = 1.0f; n = 1; }   /* sampler.c:145-149 */
    d.num_cands = n;

    {
        int32_t *tid = (int32_t *)malloc((size_t)n * sizeof(int32_t));
        float *tval = (float *)malloc((size_t)n * sizeof(float));
        orc_sort_desc(ids, vals, n, tid, tval);
        free(tid);
        free(tval);
    }

    if (cfg->top_k > 0 && cfg->top_k < n) n = cfg->top_k;   /* sampler.c:155-157 */
    d.n_topk = n;

    /* sampler.c:160-179: sequential mass, inclusive nucleus cut. */
    float mass = 0.0f;
    for (int i = 0; i < n; ++i) mass += vals[i];
    const float p = cfg->top_p;
    if (p > 0.0f && p < 1.0f) {
        const float cutoff = p * mass;
        float cum = 0.0f;
        int keep = 0;
        for (int i = 0; i < n; ++i) {
            cum += vals[i];
            ++keep;
            if (cum >= cutoff) break;
        }
        n = keep;
        mass = cum;
    }
    d.n_final = n;
    d.total_mass = mass;

    /* sampler.c:182-191: one RNG step, first prefix sum reaching r. */
    d.u = orc_random_f32(rng);
    const float r = d.u * mass;
    d.r = r;
    float acc = 0.0f;
    d.pos = 0;
    d.id = ids[0];
    for (int i = 0; i < n; ++i) {
        acc += vals[i];
        if (r <= acc || i == n - 1) { d.pos = i; d.id = ids[i]; break; }
    }
    if (!cand_ids) free(ids);
    if (!cand_vals) free(vals);
    if (diag) *diag = d;
    return d.id;
}

static void orc_batch_common(const orc_config_t *cfg, const float *logits_f32,
                             const uint16_t *logits_bf16, int B, int V, size_t ld,
                             const int32_t *hist, int H, size_t hld, uint64_t *rng,
                             int32_t *out_ids, float *probs, orc_row_diag_t *diag,
                             int32_t *topn_ids, float *topn_probs, int n_list,
                             int in_place, int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float *row = (float *)malloc((size_t)V * sizeof(float));
        int32_t *ids = (int32_t *)malloc((size_t)V * sizeof(int32_t));
        float *vals = (float *)malloc((size_t)V * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int b = 0; b < B; ++b) {
            float *x;
            if (logits_bf16) {
                const uint16_t *src = logits_bf16 + (size_t)b * ld;
                for (int i = 0; i < V; ++i) {
                    uint32_t u = (uint32_t)src[i] << 16;
                    memcpy(&row[i], &u, 4);
                }
                x = row;
            } else if (in_place) {
                x = (float *)logits_f32 + (size_t)b * ld;
            } else {
                memcpy(row, logits_f32 + (size_t)b * ld, (size_t)V * sizeof(float));
                x = row;
            }
            orc_row_diag_t d;
            const int32_t *h = hist ? hist + (size_t)b * hld : NULL;
            int32_t id = orc_sample_row(cfg, x, V, h, hist ? H : 0, rng + 2 * (size_t)b,
                                        ids, vals, &d);
            out_ids[b] = id;
            if (probs) probs[b] = d.greedy ? 1.0f : vals[d.pos] / d.total_mass;
            if (diag) diag[b] = d;
            if (topn_ids) {
                int n = d.greedy ? 1 : d.n_final;
                for (int i = 0; i < n_list; ++i) {
                    if (i < n) {
                        topn_ids[(size_t)b * n_list + i] = d.greedy ? id : ids[i];
                        if (topn_probs)
                            topn_probs[(size_t)b * n_list + i] =
                                d.greedy ? 1.0f : vals[i] / d.total_mass;
                    } else {
                        topn_ids[(size_t)b * n_list + i] = -1;
                        if (topn_probs) topn_probs[(size_t)b * n_list + i] = 0.0f;
                    }
                }
            }
        }
        free(row);
        free(ids);
        free(vals);
    }
}

void orc_sample_batch(const orc_config_t *cfg, const float *logits, int B, int V,
                      size_t ld, const int32_t *hist, int H, size_t hld,
                      uint64_t *rng, int32_t *ids, float *probs,
                      orc_row_diag_t *diag, int32_t *topn_ids, float *topn_probs,
                      int n_list, int in_place, int nthreads) {
    orc_batch_common(cfg, logits, NULL, B, V, ld, hist, H, hld, rng, ids, probs, diag,
                     topn_ids, topn_probs, n_list, in_place, nthreads);
}

void orc_sample_batch_bf16(const orc_config_t *cfg, const uint16_t *logits, int B,
                           int V, size_t ld, const int32_t *hist, int H, size_t hld,
                           uint64_t *rng, int32_t *ids, float *probs,
                           orc_row_diag_t *diag, int32_t *topn_ids,
                           float *topn_probs, int n_list, int nthreads) {
    orc_batch_common(cfg, NULL, logits, B, V, ld, hist, H, hld, rng, ids, probs, diag,
                     topn_ids, topn_probs, n_list, 0, nthreads);
}

void orc_expf_range(uint32_t lo_bits, uint32_t n, float *out) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint32_t u = lo_bits + (uint32_t)i;
        float x;
        memcpy(&x, &u, 4);
        out[i] = expf(x);
    }
}

/* splitmix64 finaliser: a commutative per-element hash summed over a chunk,
 * so a parallel GPU reduction can reproduce the same checksum. */
static inline uint64_t orc_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void orc_expf_domain_checksums(int chunk_log2, uint64_t *out, int n_chunks, int nthreads) {
    const uint32_t first = 0x80000000u, last = 0xC1700000u; /* -0.0 .. -15.0 (excl.) */
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (int c = 0; c < n_chunks; ++c) {
        uint64_t h = 0;
        uint64_t lo = (uint64_t)first + ((uint64_t)c << chunk_log2);
        uint64_t hi = lo + (1ULL << chunk_log2);
        if (hi > last) hi = last;
        for (uint64_t u = lo; u < hi; ++u) {
            uint32_t ub = (uint32_t)u;
            float x, y;
            memcpy(&x, &ub, 4);
            y = expf(x);
            uint32_t yb;
            memcpy(&yb, &y, 4);
            h += orc_mix64(((uint64_t)ub << 32) | yb);
        }
        out[c] = h;
    }
}
