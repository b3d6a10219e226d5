/*
 * Oracle for the paths next to the sampler: CPU restatements of the
 * reference's MoE router (Sain-Kai/noel src/sparsity.c:46-79), of the
 * pipeline's sibling sampler (src/pipeline_stages.c:64-189) and of its
 * LM-head GEMV for unquantised rows (src/dequant.c:412-470), used ONLY as
 * checkers by tests/ and bench.py's CPU leg.  Nothing in the shipped library
 * links, loads or calls this code.
 *
 * Parity pinning: checked against the reference's known-answer test of the
 * router (tests/test_engine.c:128-142) and against the reference's own
 * sparsity.c and pipeline_stages.c, compiled from their sources into
 * oracle/_ref/libaux_ref.so by oracle/Makefile, on seeded inputs
 * (tests/test_router.py, tests/test_postreq.py, tests/test_lmhead.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

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

/* ------------------------------------------------------------------------ */
/* the pipeline's sibling sampler (src/pipeline_stages.c:64-189)            */

/* pipeline_stages.c:64-79: per occurrence, in place, ids outside [0, V) skipped */
void orc_postreq_apply_penalties(float *logits, int V, const int32_t *hist, int H, float pen, int window) {
    if (pen <= 1.0f || H <= 0) return;
    const int first = (window > 0 && H > window) ? H - window : 0;
    for (int i = first; i < H; ++i) {
        const int32_t t = hist[i];
        if (t < 0 || t >= V) continue;
        logits[t] = logits[t] > 0.0f ? logits[t] / pen : logits[t] * pen;
    }
}

/* pipeline_stages.c:81-94: state 0 keeps only '{' */
void orc_postreq_grammar_mask(float *logits, int V, int state) {
    if (state != 0) return;
    for (int v = 0; v < V; ++v)
        if (v != '{') logits[v] = -1e9f;
}

/* pipeline_stages.c:103-189 with the uniform r given (the reference draws it
 * from rand() at :180); the row is modified in place as the reference does */
int32_t orc_postreq_sample(float *logits, int V, float T, float top_p, int top_k, float r) {
    if (T <= 1e-4f) { /* :105-115 first strict maximum */
        int32_t best = 0;
        float bv = logits[0];
        for (int v = 1; v < V; ++v)
            if (logits[v] > bv) {
                bv = logits[v];
                best = v;
            }
        return best;
    }
    const float inv_t = 1.0f / T; /* :118-121 */
    for (int v = 0; v < V; ++v) logits[v] *= inv_t;
    float m = logits[0]; /* :124-127 */
    for (int v = 1; v < V; ++v)
        if (logits[v] > m) m = logits[v];
    float sum = 0.0f; /* :128-136 */
    for (int v = 0; v < V; ++v) {
        logits[v] = expf(logits[v] - m);
        sum += logits[v];
    }
    const float inv_sum = sum > 0.0f ? 1.0f / sum : 0.0f;
    for (int v = 0; v < V; ++v) logits[v] *= inv_sum;
    int K = top_k; /* :138-158: the K best by (p desc, id asc), slots of (-1, -1) */
    if (K <= 0 || K > V) K = V;
    if (K > 256) K = 256;
    int32_t cid[256];
    float cp[256];
    for (int i = 0; i < K; ++i) {
        cid[i] = -1;
        cp[i] = -1.0f;
    }
    for (int v = 0; v < V; ++v) {
        const float p = logits[v];
        if (!(p > cp[K - 1])) continue;
        int at = K - 1; /* below every slot it does not strictly beat */
        while (at > 0 && p > cp[at - 1]) {
            cp[at] = cp[at - 1];
            cid[at] = cid[at - 1];
            --at;
        }
        cp[at] = p;
        cid[at] = v;
    }
    float cum = 0.0f; /* :160-168 */
    int n = 0;
    for (int i = 0; i < K && cid[i] >= 0; ++i) {
        cum += cp[i];
        ++n;
        if (cum >= top_p) break;
    }
    const float inv_cum = 1.0f / cum; /* :170-174 */
    for (int i = 0; i < n; ++i) cp[i] *= inv_cum;
    float run = 0.0f; /* :180-188 */
    for (int i = 0; i < n; ++i) {
        run += cp[i];
        if (r <= run || i == n - 1) return cid[i];
    }
    return cid[0];
}

/* B rows (row b at logits + b * ld), uniforms r[b] */
void orc_postreq_sample_batch(float *logits, int B, int V, size_t ld, float T, float top_p, int top_k, const float *r,
                              int32_t *ids) {
    for (int b = 0; b < B; ++b) ids[b] = orc_postreq_sample(logits + (size_t)b * ld, V, T, top_p, top_k, r[b]);
}

/* ------------------------------------------------------------------------ */
/* LM-head GEMV (src/dequant.c:412-470) for F32 (type 0), F16 (1), BF16 (30) */

static float orc_half(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t f;
    if (e == 0u) {
        if (m == 0u) f = sign;
        else { /* subnormal half: normalise */
            int k = -1;
            uint32_t mm = m;
            do { mm <<= 1; ++k; } while (!(mm & 1024u));
            f = sign | ((uint32_t)(112 - k) << 23) | ((mm & 1023u) << 13);
        }
    } else if (e == 31u) {
        f = sign | 0x7F800000u | (m << 13);
    } else {
        f = sign | ((e + 112u) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &f, 4);
    return r;
}

static float orc_elem(int type, const void *row, int j) {
    if (type == 0) return ((const float *)row)[j];
    const uint16_t h = ((const uint16_t *)row)[j];
    if (type == 30) {
        const uint32_t f = (uint32_t)h << 16;
        float r;
        memcpy(&r, &f, 4);
        return r;
    }
    return orc_half(h);
}

/* y[b][r] for rows r < rows, tokens b < B, cols a multiple of 8: eight fused
 * multiply-add accumulators over blocks of eight columns, combined as
 * ((a0 + a4) + (a1 + a5)) + ((a2 + a6) + (a3 + a7)) (dequant.c:437-452).
 * The reference's scalar loop over a ragged tail (:454-456) is left to its
 * compiler's scheduling (it matches neither one fused multiply-add per
 * column nor a multiply and an add), so other widths are not restated. */
void orc_gemv(int type, const void *W, size_t ldw, const float *x, size_t ldx, int B, int rows, int cols, float *y,
              size_t ldy) {
    const size_t es = type == 0 ? 4 : 2;
    for (int b = 0; b < B; ++b) {
        const float *xb = x + (size_t)b * ldx;
        for (int r = 0; r < rows; ++r) {
            const void *row = (const char *)W + (size_t)r * ldw * es;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int j = 0;
            for (; j + 8 <= cols; j += 8)
                for (int k = 0; k < 8; ++k) a[k] = fmaf(orc_elem(type, row, j + k), xb[j + k], a[k]);
            float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
            const float dot = (s0 + s1) + (s2 + s3);
            y[(size_t)b * ldy + r] = dot;
        }
    }
}
