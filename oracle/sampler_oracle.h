/*
 * Oracle for the token-sampling path: a CPU restatement of the reference
 * sampler (Sain-Kai/noel src/sampler.c:8-192), used ONLY as the checker by
 * tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py.
 * Nothing in the shipped library links, loads or calls this code.
 *
 * Parity pinning: the restatement is checked against the reference's own
 * known-answer tests (tests/test_engine.c:700-748) and against the reference
 * sampler itself, compiled from its sources into oracle/_ref/ by
 * oracle/Makefile, on seeded inputs (tests/test_oracle.py) and on the
 * committed golden fixtures under tests/golden/.
 */
#ifndef NOEL_SAMPLER_ORACLE_H
#define NOEL_SAMPLER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order and types as noel_sampler_config_t (include/sampler.h). */
typedef struct {
    float temperature;
    float top_p;
    int top_k;
    float repetition_penalty;
    int repetition_window;
    uint64_t seed;
} orc_config_t;

/* Per-row diagnostics of one sampling call (what the reference keeps in
 * locals): counts after each stage, the masses and the scaled uniform. */
typedef struct {
    int32_t id;          /* returned token */
    int32_t greedy;      /* 1 if the argmax branch ran (no RNG step) */
    int32_t num_cands;   /* candidates passing diff > -15 (1 after fallback) */
    int32_t n_topk;      /* after top-k truncation */
    int32_t n_final;     /* after top-p truncation (the drawn-from list) */
    int32_t pos;         /* index of the returned id in the sorted list */
    float max_val;       /* row max after the penalty */
    float total_mass;    /* mass of the drawn-from list */
    float u;             /* the U[0,1) draw */
    float r;             /* u * total_mass */
} orc_row_diag_t;

/* xorshift128+ step (sampler.c:8-15). */
uint64_t orc_xorshift128plus(uint64_t s[2]);
/* 24-bit uniform in [0,1) (sampler.c:17-21). */
float orc_random_f32(uint64_t s[2]);
/* State for a non-zero seed (sampler.c:42-47 and :66-69). */
void orc_seed_state(uint64_t seed, uint64_t s[2]);

/*
 * Sample one row in place (logits are penalised in the caller's buffer,
 * like the reference).  rng is the row's 2-word state, advanced exactly as
 * the reference advances it.  cand_ids/cand_vals (capacity >= vocab, may be
 * NULL) receive the full sorted candidate list; diag (may be NULL) the
 * per-stage counts.  Returns the sampled id.
 */
int32_t orc_sample_row(const orc_config_t *cfg, float *logits, int vocab,
                       const int32_t *history, int history_len, uint64_t rng[2],
                       int32_t *cand_ids, float *cand_vals, orc_row_diag_t *diag);

/*
 * Batched driver: rows b in [0,B) are logits + b*ld (copied to private
 * scratch unless in_place), histories hist + b*hld (H entries, may be NULL),
 * RNG states rng[2b..2b+1] (in/out).  Outputs: ids[b]; probs[b] (may be
 * NULL) = val(chosen)/total_mass; diag[b] (may be NULL); top-n lists
 * (may be NULL): topn_ids/topn_probs[b*n_list + i] for i < min(n_final,
 * n_list), -1 / 0 padded.  nthreads <= 0 uses all OpenMP threads.
 */
void orc_sample_batch(const orc_config_t *cfg, const float *logits, int B, int V,
                      size_t ld, const int32_t *hist, int H, size_t hld,
                      uint64_t *rng, int32_t *ids, float *probs,
                      orc_row_diag_t *diag, int32_t *topn_ids, float *topn_probs,
                      int n_list, int in_place, int nthreads);

/* Same as orc_sample_batch for bf16 logits (upcast exactly to fp32). */
void orc_sample_batch_bf16(const orc_config_t *cfg, const uint16_t *logits, int B,
                           int V, size_t ld, const int32_t *hist, int H, size_t hld,
                           uint64_t *rng, int32_t *ids, float *probs,
                           orc_row_diag_t *diag, int32_t *topn_ids,
                           float *topn_probs, int n_list, int nthreads);

/* glibc expf over [lo, hi] float bit patterns, for the exp-parity checks. */
void orc_expf_range(uint32_t lo_bits, uint32_t n, float *out);
/* FNV-style checksum of expf(x) bits for every float x in (-15, 0], in
 * chunks of 2^chunk_log2 bit patterns starting at -0.0 (0x80000000). */
void orc_expf_domain_checksums(int chunk_log2, uint64_t *out, int n_chunks, int nthreads);

#ifdef __cplusplus
}
#endif

#endif
