/*
 * Batched B200 entry points of the token sampler (libnoel_sampler_cuda.so).
 *
 * The reference samples one host row per call (Sain-Kai/noel
 * src/sampler.c:80, called from src/engine.c:387).  These entry points run
 * the same computation for a batch of rows resident on the GPU: per row the
 * repetition penalty over its history, temperature, top-k, top-p and one
 * draw from the row's own xorshift128+ state, with results identical to the
 * reference's for the same row, history, config and state.  They have no
 * counterpart in the reference beyond that per-row function; each cites the
 * reference lines whose semantics it carries.
 *
 * Conventions: plain pointers and sizes; "d_" pointers are device memory of
 * the current device; stream is a cudaStream_t (NULL = default stream).
 * Every function returns NOEL_OK (0) or a negative status; the calling
 * thread's last status and message are kept for noel_sampler_cuda_last_error().
 */
#ifndef NOEL_SAMPLER_CUDA_H
#define NOEL_SAMPLER_CUDA_H

#include "sampler.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    NOEL_OK = 0,
    NOEL_ERR_INVALID_ARG = -1,   /* NULL pointer, bad size or misaligned row */
    NOEL_ERR_CUDA = -2,          /* a CUDA runtime call failed */
    NOEL_ERR_NO_DEVICE = -3,     /* no usable sm_100 device */
    NOEL_ERR_TOO_LARGE = -4,     /* size beyond what the entry point supports */
    NOEL_ERR_UNSUPPORTED = -5,   /* option combination not supported */
    NOEL_ERR_DEVICE_WAIT = -6,   /* a kernel's bounded wait ran out; results of that call are invalid */
};

enum { NOEL_DTYPE_F32 = 0, NOEL_DTYPE_BF16 = 1 };

/* Per-row statistics (out_stats, 4 x int32 per row). */
enum {
    NOEL_STAT_NUM_CANDS = 0,  /* candidates with diff > -15, or -1 if > the kept set */
    NOEL_STAT_N_TOPK = 1,     /* list length after top-k (sampler.c:155-157) */
    NOEL_STAT_N_FINAL = 2,    /* list length after top-p (sampler.c:165-179) */
    NOEL_STAT_FLAGS = 3,      /* NOEL_ROW_* bits */
};
enum {
    NOEL_ROW_GREEDY = 1,      /* argmax branch, no RNG step (sampler.c:106-116) */
    NOEL_ROW_EXACT_PASS = 2,  /* finished by the two-pass exact kernel */
    NOEL_ROW_FALLBACK = 4,    /* no candidate: {0, 1.0} (sampler.c:145-149) */
};

/* Optional outputs and options of one batched call. */
typedef struct {
    float *d_probs;           /* [B] val(chosen)/mass, or NULL (1.0 for greedy) */
    int32_t *d_list_ids;      /* [B][list_len] drawn-from list, sorted, -1 padded, or NULL */
    float *d_list_probs;      /* [B][list_len] their probabilities, or NULL */
    int list_len;
    int list_weights;         /* 1: d_list_probs gets the unnormalised weights (sampler.c:140) */
    int32_t *d_stats;         /* [B][4] NOEL_STAT_* per row, or NULL */
    int write_back;           /* 1: store penalised values into the fp32 logits (sampler.c:96-100) */
} noel_sample_extras_t;

/*
 * Sample B rows on the device.  Replaces B calls of noel_sampler_sample
 * (sampler.c:80-192) with one launch sequence.
 *   d_logits   [B][ld] fp32 or bf16 (dtype), row b at d_logits + b*ld elements;
 *              ld >= vocab; the base must be aligned to the element size.
 *   d_history  [B][hld] int32 token ids or NULL; the first history_len are used
 *              (window per cfg->repetition_window, sampler.c:89-90).
 *   d_rng      [B][2] xorshift128+ states, advanced once per non-greedy row.
 *   d_ids      [B] sampled ids.
 *   d_probs    [B] probability of the sampled id, or NULL.
 */
int noel_sampler_sample_batch(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                              int batch, int vocab, size_t ld, const int32_t *d_history,
                              int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                              float *d_probs, void *stream);

/* As noel_sampler_sample_batch, with the optional outputs of extras (may be NULL). */
int noel_sampler_sample_batch_ex(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                                 int batch, int vocab, size_t ld, const int32_t *d_history,
                                 int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                                 const noel_sample_extras_t *extras, void *stream);

/*
 * noel_sampler_sample_batch for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some callers can't call cudaMalloc: a
 * serving loop that fixed its device-memory budget at start-up and must not
 * grow it (or risk cudaMalloc synchronising the device mid-stream), or an
 * embedding application whose allocator owns all device memory and gives the
 * sampler none.  This entry point allocates nothing: the scratch of the
 * two-pass kernel lives in a static device array of the library image
 * (8,421,632 bytes, held by every GPU that loads the library until exit).
 * Limits: batch <= 8192 rows, vocab <= 262144; larger calls return
 * NOEL_ERR_TOO_LARGE.  The first call on each device does a one-time set-up
 * (looks up the array's device address and sets kernel attributes) and should
 * come before any stream capture.  All calls share the array and it keeps the
 * last call's contents (the call clears what must start empty), so calls that
 * overlap on one GPU (issued on different streams) race: issue them on one
 * stream per device.  Arguments as noel_sampler_sample_batch.
 */
int noel_sampler_sample_batch_noalloc(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                                      int batch, int vocab, size_t ld, const int32_t *d_history,
                                      int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                                      float *d_probs, void *stream);

/*
 * Vocab-sharded rows: the vocabulary split into column ranges, one per GPU
 * (rank r holds [v_begin_r, v_begin_r + shard_vocab_r), ranks in ascending
 * order covering the whole vocabulary).  No counterpart in the reference,
 * which samples whole rows on the host (sampler.c:80-192); the result equals
 * noel_sampler_sample on the full row.  Three steps:
 *
 *   1. noel_sampler_shard_select on every GPU: per row, a list of
 *      L = noel_sampler_shard_list_len(cfg) entries (global id, penalised
 *      logit bits) by (logit desc, id asc), id -1 past the listed ones, then a
 *      trailer (largest penalised logit bits, flags): d_lists [B][L + 1][2]
 *      u32.  Greedy lists the shard's best element; top-k (k <= 120) its best
 *      k + 8; top-k off or above 120 its elements within the -15 cut under
 *      its own maximum (at most 256).
 *   2. an exchange that gives the rank merging rows [r0, r1) every shard's
 *      lists of those rows, shard-major: [n_shards][r1 - r0][L + 1][2]
 *      (an all-to-all of contiguous row blocks, or an all-gather of
 *      everything).
 *   3. noel_sampler_shard_merge: the rows' samples from those lists, with
 *      their RNG states d_rng [rows][2] (in/out).  A row that cannot be
 *      decided from them (a weight tie at the top-k boundary reaching below
 *      the gathered entries, or a full-list shard that left out elements
 *      within the row's cut) gets status 1 and keeps its RNG state: sample it
 *      from its full row (gather the row's shards) with
 *      noel_sampler_sample_batch.
 *
 * The penalty applies to the history ids inside the shard; d_history holds
 * global ids.  d_logits points at the shard's first column; ld is its row
 * stride.  A full-list shard whose history table and list do not fit the
 * streaming kernel's shared memory returns NOEL_ERR_UNSUPPORTED.
 */
int noel_sampler_shard_list_len(const noel_sampler_config_t *cfg);
int noel_sampler_shard_select(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                              int batch, int shard_vocab, size_t ld, int v_begin,
                              const int32_t *d_history, int history_len, size_t hld,
                              uint32_t *d_lists, void *stream);
/* d_lists [n_shards][batch][L + 1][2]; d_rng [batch][2] in/out, d_ids [batch],
 * d_probs [batch] or NULL, d_status [batch]. */
int noel_sampler_shard_merge(const noel_sampler_config_t *cfg, int n_shards, int batch,
                             const uint32_t *d_lists, uint64_t *d_rng, int32_t *d_ids, float *d_probs,
                             int32_t *d_status, void *stream);

/*
 * Host-buffer form of noel_sampler_sample_batch for callers whose logits are
 * in host memory (the reference engine's layout, src/engine.c:59): copies the
 * rows, histories and states to the device, samples, and copies ids, states
 * and (if h_probs) probabilities back; synchronous.  Pinned host memory gives
 * the fastest copies.  logits rows are h_logits + b*ld fp32 or bf16 elements.
 */
int noel_sampler_sample_batch_host(const noel_sampler_config_t *cfg, const void *h_logits, int dtype,
                                   int batch, int vocab, size_t ld, const int32_t *h_history,
                                   int history_len, size_t hld, uint64_t *h_rng, int32_t *h_ids,
                                   float *h_probs);

/*
 * Wait for the work queued on stream and report device-side failures of the
 * batched calls made on it since the last check: NOEL_ERR_DEVICE_WAIT if a
 * wait of the streaming kernel (for a ring stage, a prepared row or the
 * consumers of a row) ran out of its limit; the kernel then returns instead
 * of hanging and the results of that call are invalid.  Clears the flag.
 */
int noel_sampler_cuda_sync_check(void *stream);

/*
 * Limit of every device-side wait of the batched calls this thread makes
 * next, in nanoseconds of the GPU's global timer (0 restores the default of
 * 2 s).  stall_next_call = 1 makes the next batched call's kernel issue no
 * row loads, so its waits run out and noel_sampler_cuda_sync_check reports
 * NOEL_ERR_DEVICE_WAIT: the failure-detection path, exercised without a GPU
 * fault.  No counterpart in the reference (its sampler never waits).
 */
int noel_sampler_cuda_set_wait_limit(long long wait_ns, int stall_next_call);

/* Calling thread's last status (NOEL_OK after a successful call). */
int noel_sampler_cuda_last_error(void);
/* Calling thread's last error message ("" if none). */
const char *noel_sampler_cuda_last_error_message(void);
/* Static name of a status code. */
const char *noel_sampler_cuda_status_string(int status);

/*
 * Profiling hook: record ev_before / ev_after (cudaEvent_t, or NULL to stop)
 * on the launching stream around the single-pass sampling kernel of every
 * later batched call made by this thread, so a caller can time that kernel
 * alone with CUDA events.
 */
int noel_sampler_cuda_profile_events(void *ev_before, void *ev_after);

/* Number of inputs x in (-15, 0] whose exp weight comes from the C-library
 * table rather than the correctly rounded exp (diagnostic). */
int noel_sampler_cuda_expf_table_size(void);

/*
 * Checksum of the device's exp weight bits over every float in (-15, 0]
 * (bit patterns 0x80000000 .. 0xC1700000), in chunks of 2^chunk_log2 inputs:
 * out[c] = sum over the chunk of mix64((x_bits << 32) | weight_bits).  The
 * same sums over the C library's expf pin the device weights to it.
 * d_out has room for ceil(0x41700000 / 2^chunk_log2) uint64 values.
 */
int noel_sampler_cuda_expf_checksums(int chunk_log2, uint64_t *d_out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NOEL_SAMPLER_CUDA_H */
