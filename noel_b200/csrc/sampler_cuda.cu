/*
 * Host side of libnoel_sampler_cuda.so: the reference's sampler ABI
 * (include/sampler.h) and the batched entry points (include/noel_sampler_cuda.h).
 *
 * Device state never lives in noel_sampler_t (callers embed it by value and
 * poke its fields, Sain-Kai/noel src/main.c:259-262): it is kept per device in
 * a process-global context, the way the reference keeps its CUDA context in
 * a global (src/cuda_backend.c:8), plus per-thread staging buffers and stream
 * for the single-row ABI.  There is no CPU fallback: a missing or
 * unsupported device is an error.
 */
#include <cuda_runtime.h>

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <map>
#include <mutex>
#include <vector>

#include "noel_lmhead.h"
#include "noel_postreq.h"
#include "noel_router.h"
#include "noel_sampler_cuda.h"
#include "lmhead.cuh"
#include "postreq.cuh"
#include "router.cuh"
#include "sampler_stream.cuh"

#define NOEL_EXPF_QUAL static __device__ const
#include "_gen/expf_table.inc"

using namespace noel;

namespace {

/* ------------------------------------------------------------------ errors */
thread_local int t_status = NOEL_OK;
thread_local char t_msg[512] = "";

int fail(int code, const char *fmt, ...) {
    t_status = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return code;
}
int ok() {
    t_status = NOEL_OK;
    t_msg[0] = '\0';
    return NOEL_OK;
}

#define CUDA_TRY(call)                                                                     \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess) return fail(NOEL_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

/* -------------------------------------------------------- device context */
struct Workspace {
    int32_t *counters = nullptr;  // 4 ints
    int32_t *rows = nullptr;      // row list of the exact kernel
    uint2 *slots = nullptr;       // nslots x 2 x vocab
    uint4 *gsplit = nullptr;      // per row: greedy rows split over CTAs (zeroed, re-armed by the kernel)
    int rows_cap = 0, vocab_cap = 0, nslots = 0;
};

struct DeviceCtx {
    bool ready = false;
    int sms = 0;
    size_t smem_optin = 0;
    ExpTable et{};
    std::map<cudaStream_t, Workspace> ws;
    std::map<const void *, size_t> smem_set;  // kernel -> dynamic smem attribute set
};

std::mutex g_mu;
std::vector<DeviceCtx> g_dev;

int device_ctx(DeviceCtx **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(NOEL_ERR_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
    DeviceCtx &c = g_dev[dev];
    if (!c.ready) {
        cudaDeviceProp p;
        CUDA_TRY(cudaGetDeviceProperties(&p, dev));
        if (p.major != 10)
            return fail(NOEL_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                        p.major, p.minor);
        c.sms = p.multiProcessorCount;
        c.smem_optin = p.sharedMemPerBlockOptin;
        void *k = nullptr, *v = nullptr, *o = nullptr;
        CUDA_TRY(cudaGetSymbolAddress(&k, kExpfExcKeys));
        CUDA_TRY(cudaGetSymbolAddress(&v, kExpfExcVals));
        CUDA_TRY(cudaGetSymbolAddress(&o, kExpfExcOffs));
        c.et.keys = static_cast<const uint32_t *>(k);
        c.et.vals = static_cast<const uint32_t *>(v);
        c.et.offs = static_cast<const uint32_t *>(o);
        c.et.near = NOEL_EXPF_NEAR;
        c.ready = true;
    }
    *out = &c;
    return NOEL_OK;
}

/* Per-(device, stream) scratch of the exact kernel.  Calls on one stream run
 * in order, so they can share it; calls on different streams get their own. */
int workspace(DeviceCtx *c, cudaStream_t s, int rows, int vocab, Workspace **out) {
    std::lock_guard<std::mutex> lk(g_mu);
    Workspace &w = c->ws[s];
    const int nslots = rows < 64 ? rows : 64;
    if (w.counters && rows <= w.rows_cap && vocab <= w.vocab_cap && nslots <= w.nslots) {
        *out = &w;
        return NOEL_OK;
    }
    /* growing synchronises the stream and frees the old buffers, which a
     * stream being captured into a CUDA graph cannot do: the first call of
     * each shape on a stream must come before capture */
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone)
        return fail(NOEL_ERR_UNSUPPORTED,
                    "the stream is being captured and its scratch must grow: make one call of this shape "
                    "(%d rows x %d tokens) on the stream before capturing", rows, vocab);
    /* grow to cover both the old and the new shape, so calls that alternate
     * between shapes settle at once */
    int rc = rows > 1 ? rows : 1, vc = vocab, ns = nslots > 1 ? nslots : 1;
    if (w.counters) {
        rc = rc > w.rows_cap ? rc : w.rows_cap;
        vc = vc > w.vocab_cap ? vc : w.vocab_cap;
        ns = ns > w.nslots ? ns : w.nslots;
        CUDA_TRY(cudaStreamSynchronize(s));
        cudaFree(w.counters);
        cudaFree(w.rows);
        cudaFree(w.slots);
        cudaFree(w.gsplit);
        w = Workspace{};
    }
    CUDA_TRY(cudaMalloc(&w.counters, 4 * sizeof(int32_t)));
    CUDA_TRY(cudaMemset(w.counters, 0, 4 * sizeof(int32_t)));
    CUDA_TRY(cudaMalloc(&w.rows, (size_t)rc * sizeof(int32_t)));
    CUDA_TRY(cudaMalloc(&w.slots, (size_t)ns * 2 * (size_t)vc * sizeof(uint2)));
    CUDA_TRY(cudaMalloc(&w.gsplit, (size_t)rc * sizeof(uint4)));
    CUDA_TRY(cudaMemset(w.gsplit, 0, (size_t)rc * sizeof(uint4)));
    w.rows_cap = rc;
    w.vocab_cap = vc;
    w.nslots = ns;
    *out = &w;
    return NOEL_OK;
}

/* events recorded around the next main-kernel launches of this thread (profiling hook) */
thread_local cudaEvent_t t_ev_before = nullptr, t_ev_after = nullptr;

/* limit of the streaming kernel's device-side waits, and the failure-
 * detection hook (the next call's kernel issues no row loads) */
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;
thread_local unsigned long long t_wait_ns = kDefaultWaitNs;
thread_local int t_stall_next = 0;

int set_smem(DeviceCtx *c, const void *kernel, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    size_t &cur = c->smem_set[kernel];
    if (bytes > cur) {
        CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
        cur = bytes;
    }
    return NOEL_OK;
}

int pow2_at_least(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

constexpr int kMaxKprime = 1024;     // top-k mode up to k = 1016
constexpr size_t kStreamStaticReserve = 10240;  // static shared memory of the streaming kernel, rounded up
static_assert(sizeof(StreamShared) <= kStreamStaticReserve, "streaming kernel's static shared memory");
/* modes the persistent streaming kernel serves; the others use the one-CTA-
 * per-row kernels, measured faster for them on B200 (1024 x 152,064 fp32:
 * top-k 40 with a penalty 166 vs 281 us, greedy 113 vs 174 us).  A build
 * with -DNOEL_STREAM_MODES=7 streams every mode (all parity tests pass). */
#ifndef NOEL_STREAM_MODES
#define NOEL_STREAM_MODES (1u << kFullList)
#endif
constexpr unsigned kStreamModes = NOEL_STREAM_MODES;
constexpr int kWarpKprimeMax = 128;  // warp-streaming kernel up to k = 120
constexpr int kCapMax = 4096;

template <typename T>
int launch_t(const SampleArgs &a0, int mode, bool block_kernel, bool wide, bool stream, bool exact_only,
             size_t smem_main, size_t smem_exact, DeviceCtx *c, cudaStream_t s) {
    const void *kmain = nullptr;
    if (stream) kmain = mode == kGreedy ? (const void *)stream_rows_kernel<T, kGreedy>
                        : mode == kTopK ? (const void *)stream_rows_kernel<T, kTopK>
                                        : (const void *)stream_rows_kernel<T, kFullList>;
    else if (block_kernel) kmain = (const void *)sample_rows_block_kernel<T, kTopK>;
    else if (mode == kGreedy) kmain = (const void *)sample_rows_kernel<T, kGreedy, 1>;
    else if (mode == kTopK) kmain = wide ? (const void *)sample_rows_kernel<T, kTopK, 4>
                                         : (const void *)sample_rows_kernel<T, kTopK, 1>;
    else kmain = wide ? (const void *)sample_rows_kernel<T, kFullList, 4>
                      : (const void *)sample_rows_kernel<T, kFullList, 1>;
    const void *kexact = (const void *)exact_rows_kernel<T>;
    int r = exact_only ? NOEL_OK : set_smem(c, kmain, smem_main);
    if (r) return r;
    r = set_smem(c, kexact, smem_exact);
    if (r) return r;
    if (t_ev_before) CUDA_TRY(cudaEventRecord(t_ev_before, s));
    /* one CTA per row, or per range of a split greedy row (the streaming
     * kernel: one per SM, rows in turn) */
    const int grid = a0.gsplit ? a0.batch * a0.split : a0.batch;
    const int sgrid = a0.batch < c->sms ? a0.batch : c->sms;
    if (exact_only) list_all_rows_kernel<<<(a0.batch + 255) / 256 < c->sms ? (a0.batch + 255) / 256 : c->sms, 256, 0,
                                            s>>>(a0);
    else if (stream && mode == kGreedy) stream_rows_kernel<T, kGreedy><<<sgrid, kSThreads, smem_main, s>>>(a0);
    else if (stream && mode == kTopK) stream_rows_kernel<T, kTopK><<<sgrid, kSThreads, smem_main, s>>>(a0);
    else if (stream) stream_rows_kernel<T, kFullList><<<sgrid, kSThreads, smem_main, s>>>(a0);
    else if (block_kernel) sample_rows_block_kernel<T, kTopK><<<grid, kMainThreads, smem_main, s>>>(a0);
    else if (mode == kGreedy) sample_rows_kernel<T, kGreedy, 1><<<grid, kRowThreads, smem_main, s>>>(a0);
    else if (mode == kTopK && wide) sample_rows_kernel<T, kTopK, 4><<<grid, kRowThreads, smem_main, s>>>(a0);
    else if (mode == kTopK) sample_rows_kernel<T, kTopK, 1><<<grid, kRowThreads, smem_main, s>>>(a0);
    else if (wide) sample_rows_kernel<T, kFullList, 4><<<grid, kRowThreads, smem_main, s>>>(a0);
    else sample_rows_kernel<T, kFullList, 1><<<grid, kRowThreads, smem_main, s>>>(a0);
    CUDA_TRY(cudaGetLastError());
    if (t_ev_after) CUDA_TRY(cudaEventRecord(t_ev_after, s));
    if (mode != kGreedy) {
        /* launched as a programmatic dependent of the main kernel, which
         * allows it at its start: its launch overlaps the main kernel's last
         * CTAs, and it waits for that grid (griddepcontrol.wait) before it
         * reads the row list */
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(a0.nslots);
        lc.blockDim = dim3(kExactThreads);
        lc.dynamicSmemBytes = smem_exact;
        lc.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        CUDA_TRY(cudaLaunchKernelEx(&lc, exact_rows_kernel<T>, a0));
        CUDA_TRY(cudaGetLastError());
    }
    return NOEL_OK;
}

/* vocab shard output of sample_batch (see SampleArgs) */
struct ShardOut {
    int id_off;
    uint2 *lists;
    int split = 0, split_vocab = 0;  // row splitting (see SampleArgs)
};

/* Entries a warp of the single-pass kernel keeps when its buffer fills.  A
 * row falls to the two-pass kernel when one warp holds more of the row's K'
 * best than it keeps; warps take batches dynamically and may stream well over
 * a quarter of the row, so they keep all K' for K' <= 32 and 3K'/4 for
 * K' = 64, which only a warp streaming most of the row could exceed.  At
 * K' = 128 (top-k 57..120) half is as safe: a warp's share of the 128 best
 * stays near 32.  Keeping all K' everywhere makes compactions frequent and
 * costs more than it saves. */
/* Rank r of the single-pass warm-up's starting filter, the r-th largest of
 * a uniform sample of s of a row's v elements: the smallest r for which the
 * row's K' largest put r or more elements in the sample with probability at
 * most 1e-9 (the Poisson tail of mean K' s / v, which bounds the sample's
 * hypergeometric count from above).  Fewer than r of them in the sample
 * leave K' row elements above the filter; otherwise the row end finds fewer
 * than K' passed and the row goes to the two-pass kernel.  K' when the
 * sample is the whole row (the filter is then proved). */
int warm_rank(int kprime, long long s, long long v) {
    if (s >= v) return kprime;
    const double x = (double)kprime * (double)s / (double)v;
    double p = exp(-x), cdf = 0.0;  // p = P(count = r - 1)
    for (int r = 1; r < kprime; ++r) {
        cdf += p;
        if (1.0 - cdf <= 1e-9) return r;
        p *= x / r;
    }
    return kprime;
}

int warp_keep(int kprime) { return kprime <= 32 ? kprime : (kprime <= 64 ? 3 * kprime / 4 : kprime / 2); }

/* Entries of a warp's candidate buffer: a compaction sorts the buffer and
 * keeps kw, so a small buffer compacts often (the filters rise sooner) and a
 * large one rarely; 128 entries measured best for K' = 16, 64 and 128. */
int warp_buffer(int kw) { return 2 * kw > 128 ? 2 * kw : 128; }

/* How a config is vocab-sharded: greedy lists each shard's best element
 * (selected among its 16 best); top-k with k <= 120 its best k + 8 (selected
 * among its K' = pow2(k + 8) best); top-k off or above 120 every element
 * within the -15 cut under its own maximum, up to kShardFullLen of them. */
struct ShardPlan {
    int mode, kprime, len;
};
ShardPlan shard_plan(const noel_sampler_config_t *cfg) {
    if (cfg->temperature <= 1e-4f) return {kTopK, 16, 1};  // sampler.c:106
    if (cfg->top_k > 0 && cfg->top_k <= kWarpKprimeMax - 8)
        return {kTopK, pow2_at_least(cfg->top_k + 8 > 16 ? cfg->top_k + 8 : 16), cfg->top_k + 8};
    return {kFullList, 0, kShardFullLen};
}

/* B rows of V columns, one CTA per row (or per range of a row, with a shard
 * output) */
int sample_batch(const noel_sampler_config_t *cfg, const void *logits, int dtype, int B, int V,
                 size_t ld, const int32_t *hist, int H, size_t hld, uint64_t *rng, int32_t *ids,
                 const noel_sample_extras_t *ex, cudaStream_t s, const Workspace *fixed_ws = nullptr,
                 const ShardOut *so = nullptr) {
    if (!cfg) return fail(NOEL_ERR_INVALID_ARG, "cfg is NULL");
    if (B < 0 || V <= 0) return fail(NOEL_ERR_INVALID_ARG, "batch %d / vocab %d", B, V);
    if (B == 0) return ok();
    if (!logits || (!so && (!rng || !ids))) return fail(NOEL_ERR_INVALID_ARG, "logits, rng and ids are required");
    if (so && (!so->lists || so->id_off < 0))
        return fail(NOEL_ERR_INVALID_ARG, "shard lists are required, v_begin >= 0");
    if (dtype != NOEL_DTYPE_F32 && dtype != NOEL_DTYPE_BF16) return fail(NOEL_ERR_INVALID_ARG, "dtype %d", dtype);
    if (ld < (size_t)V) return fail(NOEL_ERR_INVALID_ARG, "ld %zu < vocab %d", ld, V);
    const int es = dtype == NOEL_DTYPE_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(logits) % es) return fail(NOEL_ERR_INVALID_ARG, "logits not %d-byte aligned", es);
    if (H < 0) return fail(NOEL_ERR_INVALID_ARG, "history_len %d", H);
    if (hist && H > 0 && hld < (size_t)H) return fail(NOEL_ERR_INVALID_ARG, "hld %zu < history_len %d", hld, H);
    if (ex && ex->list_len < 0) return fail(NOEL_ERR_INVALID_ARG, "list_len %d", ex->list_len);
    if (ex && ex->write_back && dtype != NOEL_DTYPE_F32)
        return fail(NOEL_ERR_UNSUPPORTED, "write_back needs fp32 logits");
    if (ex && ex->d_stats && (reinterpret_cast<uintptr_t>(ex->d_stats) & 15))
        return fail(NOEL_ERR_INVALID_ARG, "d_stats must be 16-byte aligned");

    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;

    SampleArgs a{};
    a.logits = logits;
    a.ld = (int64_t)ld;
    a.vocab = V;
    a.batch = B;
    a.penalty = (cfg->repetition_penalty > 1.0f && hist && H > 0) ? 1 : 0;  // sampler.c:88
    if (a.penalty) {
        const int w = cfg->repetition_window;                                 // sampler.c:89-90
        a.hist = hist;
        a.hld = (int64_t)hld;
        a.hist_len = H;
        a.hist_start = (w > 0 && w < H) ? H - w : 0;
    }
    a.rep = cfg->repetition_penalty;
    const float T = cfg->temperature;
    a.inv_t = 1.0f / T;  // sampler.c:132
    a.top_p = cfg->top_p;
    a.top_k = cfg->top_k;
    a.rng = rng;
    a.ids = ids;
    if (ex) {
        a.probs = ex->d_probs;
        a.list_ids = ex->d_list_ids;
        a.list_probs = ex->d_list_probs;
        a.list_len = ex->d_list_ids ? ex->list_len : 0;
        a.list_weights = ex->list_weights;
        a.stats = ex->d_stats;
        if (ex->write_back && a.penalty) a.wb = const_cast<float *>(static_cast<const float *>(logits));
    }
    a.et = c->et;

    int mode;
    const ShardPlan sp = so ? shard_plan(cfg) : ShardPlan{0, 0, 0};
    if (so) mode = sp.mode;          // a vocab shard lists its best elements
    else if (T <= 1e-4f) mode = kGreedy;  // sampler.c:106
    else if (cfg->top_k > 0 && cfg->top_k <= kMaxKprime - 8) mode = kTopK;
    else mode = kFullList;
    bool block_kernel = false;
    if (so) {
        a.id_off = so->id_off;
        a.shard_lists = so->lists;
        a.shard_len = sp.len;
        a.split = so->split;
        a.split_vocab = so->split_vocab;
        if (mode == kTopK) {
            a.kprime = sp.kprime;
            a.kw = warp_keep(a.kprime);
            a.cap = warp_buffer(a.kw);
        } else {
            a.cap = 256;
        }
    } else if (mode == kTopK) {
        a.kprime = pow2_at_least(cfg->top_k + 8 > 16 ? cfg->top_k + 8 : 16);
        if (a.kprime <= kWarpKprimeMax) {
            a.kw = warp_keep(a.kprime);
            a.cap = warp_buffer(a.kw);
        } else {
            block_kernel = true;
            const int cap = pow2_at_least(4 * a.kprime);
            a.cap = cap < 512 ? 512 : (cap > kCapMax ? kCapMax : cap);
            a.warm_rank = warm_rank(a.kprime, (long long)kMainThreads * 2 * 16, V);  // 8192 sampled elements
        }
    } else if (mode == kFullList) {
        a.cap = 256;
    }

    size_t hist_bytes = 0;
    if (a.penalty) {
        const size_t W = ((size_t)V + 31) / 32, G = (W + 7) / 8;
        hist_bytes = W * 4 + (G + 1) * 4 + (size_t)(H - a.hist_start > 1 ? H - a.hist_start : 1) * 4;
        hist_bytes = (hist_bytes + 15) & ~size_t(15);
    }
    size_t smem_main = 0;
    bool wide = false;
    /* the persistent streaming kernel wherever its ring fits next to the
     * four row sets (greedy, top-k with K' <= 128, full lists) */
    bool stream = !block_kernel && ((kStreamModes >> mode) & 1u);
    if (stream) {
        if (a.penalty) {
            const int win = H - a.hist_start > 1 ? H - a.hist_start : 1;
            a.hcap = pow2_at_least(2 * win > 64 ? 2 * win : 64);
        }
        const StreamLayout l0 = stream_layout(mode, V, a.penalty, a.hcap, a.kprime, 0);
        const size_t avail = c->smem_optin - kStreamStaticReserve;
        const long long ns = l0.total < avail ? (long long)((avail - l0.total) / kStageBytes) : 0;
        /* at least the chunks a finisher reads for a row's starting filter
         * plus one chunk per consumer group */
        const long long nsc = ns < kMaxStages ? ns : kMaxStages;
        if (nsc >= kMinStages) {
            a.nstages = (int)nsc;
            a.wait_ns = t_wait_ns;
            a.test_stall = t_stall_next;
            t_stall_next = 0;
            smem_main = stream_layout(mode, V, a.penalty, a.hcap, a.kprime, a.nstages).total;
        } else {
            stream = false;
            a.hcap = 0;
        }
    }
    /* a full-list vocab shard whose history table and list do not fit the
     * streaming kernel: every row goes to the two-pass kernel */
    const bool exact_only = so && mode == kFullList && !stream;
    if (stream || exact_only) {
    } else if (block_kernel) {
        /* the block kernel's history also holds the id of each rank while
         * it computes the penalised values */
        const size_t idr = a.penalty ? (size_t)(H - a.hist_start > 1 ? H - a.hist_start : 1) * 4 : 0;
        smem_main = ((hist_bytes + idr + 15) & ~size_t(15)) + (size_t)a.cap * 8 + kWarmBins * 4;
    } else {
        /* single-pass kernel: bitmap of 8-id blocks + (id, count) table of the window,
         * per-warp buffers, and one area reused by the warm-up histogram and
         * the row-end gather (keys, ids, then the sort keys) */
        smem_main = 0;
        if (a.penalty) {
            const int win = H - a.hist_start > 1 ? H - a.hist_start : 1;
            a.hcap = pow2_at_least(2 * win > 64 ? 2 * win : 64);
            smem_main += (size_t)((hs_blk_words(V) + 3) & ~3) * 4 + (size_t)a.hcap * 8;
        }
        if (mode != kGreedy) {
            const int nw = kRowWarps;
            /* a batch too small to fill the GPU at 7 rows per SM streams each
             * row with batches four times as wide (2 rows per SM) */
            wide = B <= 2 * c->sms;
            const int u = (dtype == NOEL_DTYPE_F32 ? 2 : 1) * (wide ? 4 : 1);  // vectors per lane and batch
            a.qcap = 32 * u > kQueueCap ? 32 * u : kQueueCap;
            if (mode == kTopK) a.warm_rank = warm_rank(a.kprime, (long long)nw * 32 * 16 * (wide ? 4 : 1), V);
            /* the row-end union: every warp's whole buffer for K' > 32, each
             * warp's best kw below */
            a.ucap = mode == kTopK && a.kprime <= 32 ? nw * a.kw : nw * a.cap;
            const size_t gather = (size_t)a.ucap * 8 + (size_t)pow2_at_least(a.ucap) * 8;
            const size_t warm = mode == kTopK ? (size_t)2 * kWarpBins * 4 : 0;
            smem_main += (size_t)nw * a.qcap * (sizeof(V8) + 4) + (size_t)nw * a.cap * 8 +
                         (gather > warm ? gather : warm);
        }
    }
    const size_t smem_exact = a.penalty && !a.wb ? hist_bytes : 0;
    if (smem_main > c->smem_optin - 2048 || smem_exact > c->smem_optin - 16384)
        return fail(NOEL_ERR_TOO_LARGE, "vocab %d / history %d need %zu B of shared memory", V, H, smem_main);

    const Workspace *ws = fixed_ws;  // caller-provided scratch (the allocation-free entry point)
    if (!ws) {
        Workspace *w = nullptr;
        r = workspace(c, s, B, V, &w);
        if (r) return r;
        ws = w;
    }
    a.counters = ws->counters;
    a.exact_list = ws->rows;
    a.slots = ws->slots;
    a.nslots = ws->nslots;
    /* greedy rows too few to fill the GPU at 8 CTAs per SM: each row split
     * into ranges of at least 8192 tokens, one CTA per range, that fold
     * their best into the row's (the row's last CTA writes it) */
    if (mode == kGreedy && !so && !stream && ws->gsplit) {
        const int slots = 8 * c->sms;
        int sp = B < slots / 2 ? slots / B : 1;
        sp = sp < 16 ? sp : 16;
        const int maxsp = V / 8192;
        sp = sp < maxsp ? sp : maxsp;
        if (sp > 1) {
            const int width = (((V + sp - 1) / sp) + 63) & ~63;  // ranges start 256-byte apart from the row's start
            a.split = (V + width - 1) / width;
            a.split_vocab = V;
            a.vocab = width;
            a.gsplit = ws->gsplit;
        }
    }
    r = dtype == NOEL_DTYPE_F32
            ? launch_t<float>(a, mode, block_kernel, wide, stream, exact_only, smem_main, smem_exact, c, s)
            : launch_t<uint16_t>(a, mode, block_kernel, wide, stream, exact_only, smem_main, smem_exact, c, s);
    if (r) return r;
    return ok();
}

/* ------------------------------------------- per-thread single-row state */
struct Staging {
    int dev = -1;
    cudaStream_t stream = nullptr;
    float *d_logits = nullptr;
    size_t logits_cap = 0;
    int32_t *d_hist = nullptr;
    size_t hist_cap = 0;
    uint64_t *d_rng = nullptr;
    int32_t *d_out = nullptr;       // id, stats[4]
    int32_t *d_list = nullptr;
    float *d_listw = nullptr;
    int list_cap = 0;
    void *h_pin = nullptr;    // pinned: ids + stats, RNG state, list ids and weights
    size_t pin_cap = 0;
    ~Staging() {
        if (dev >= 0) {
            cudaFreeHost(h_pin);
            cudaFree(d_logits);
            cudaFree(d_hist);
            cudaFree(d_rng);
            cudaFree(d_out);
            cudaFree(d_list);
            cudaFree(d_listw);
            if (stream) cudaStreamDestroy(stream);
        }
    }
};
thread_local Staging t_stage;

int grow(void **p, size_t *cap, size_t need) {
    if (*cap >= need) return NOEL_OK;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    CUDA_TRY(cudaMalloc(p, need));
    *cap = need;
    return NOEL_OK;
}

/* sampler.c:87-103 on the caller's host row: the penalty written back in
 * place, one application per occurrence in the window, in history order */
void host_penalize(float *logits, int V, const int32_t *hist, int H, const noel_sampler_config_t *cfg) {
    const int w = cfg->repetition_window;
    const int start = (w > 0 && w < H) ? H - w : 0;
    const float rep = cfg->repetition_penalty;
    for (int i = start; i < H; ++i) {
        const int t = hist[i];
        if (t < 0 || t >= V) continue;
        logits[t] = logits[t] > 0.0f ? logits[t] / rep : logits[t] * rep;
    }
}

bool is_device_ptr(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace

/* ========================================================================= */
/* reference ABI (include/sampler.h)                                          */

extern "C" void noel_sampler_init(noel_sampler_t *sampler, const noel_sampler_config_t *cfg, int max_vocab) {
    if (!sampler) return;  // sampler.c:24
    memset(sampler, 0, sizeof(*sampler));
    if (cfg) {
        sampler->config = *cfg;
    } else {  // sampler.c:29-36
        sampler->config.temperature = 0.7f;
        sampler->config.top_p = 0.9f;
        sampler->config.top_k = 40;
        sampler->config.repetition_penalty = 1.1f;
        sampler->config.repetition_window = 64;
        sampler->config.seed = 0;
    }
    uint64_t seed = sampler->config.seed;  // sampler.c:38-47
    if (seed == 0) seed = (uint64_t)time(NULL) ^ ((uint64_t)(uintptr_t)sampler << 16);
    sampler->rng_state[0] = seed;
    sampler->rng_state[1] = seed ^ 0x9E3779B97F4A7C15ULL;
    if (sampler->rng_state[0] == 0 && sampler->rng_state[1] == 0) {
        sampler->rng_state[0] = 123456789ULL;
        sampler->rng_state[1] = 987654321ULL;
    }
    const int cap = max_vocab > 1024 ? max_vocab : 1024;  // sampler.c:49-51
    sampler->candidates = (noel_token_prob_t *)malloc((size_t)cap * sizeof(noel_token_prob_t));
    sampler->candidate_capacity = sampler->candidates ? cap : 0;
}

extern "C" void noel_sampler_free(noel_sampler_t *sampler) {
    if (!sampler) return;  // sampler.c:54-61
    free(sampler->candidates);
    sampler->candidates = NULL;
    sampler->candidate_capacity = 0;
}

extern "C" void noel_sampler_set_config(noel_sampler_t *sampler, const noel_sampler_config_t *cfg) {
    if (!sampler || !cfg) return;  // sampler.c:63-70
    sampler->config = *cfg;
    if (cfg->seed != 0) {
        sampler->rng_state[0] = cfg->seed;
        sampler->rng_state[1] = cfg->seed ^ 0x9E3779B97F4A7C15ULL;
    }
}

extern "C" float noel_sampler_random_f32(noel_sampler_t *sampler) {
    if (!sampler) return 0.0f;  // sampler.c:17-21
    uint64_t *s = sampler->rng_state;
    uint64_t a = s[0];
    const uint64_t b = s[1];
    s[0] = b;
    a ^= a << 23;
    s[1] = a ^ b ^ (a >> 18) ^ (b >> 5);
    return (float)((s[1] + b) >> 40) * (1.0f / 16777216.0f);
}

extern "C" int32_t noel_sampler_sample(noel_sampler_t *sampler, float *logits, int vocab_size,
                                       const int32_t *history, int history_len) {
    if (!sampler || !logits || vocab_size <= 0) {  // sampler.c:85
        fail(NOEL_ERR_INVALID_ARG, "sampler, logits and vocab_size > 0 are required");
        return 0;
    }
    Staging &st = t_stage;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        fail(NOEL_ERR_NO_DEVICE, "no CUDA device");
        return 0;
    }
    if (st.dev != dev) {
        st.~Staging();
        new (&st) Staging();
        st.dev = dev;
        if (cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaMalloc(&st.d_rng, 2 * sizeof(uint64_t)) != cudaSuccess ||
            cudaMalloc(&st.d_out, 8 * sizeof(int32_t)) != cudaSuccess) {
            fail(NOEL_ERR_CUDA, "staging allocation failed");
            st.dev = -1;
            return 0;
        }
    }
    cudaStream_t s = st.stream;
    const bool dev_logits = is_device_ptr(logits);
    const bool penalty = sampler->config.repetition_penalty > 1.0f && history && history_len > 0;
    const size_t row_bytes = (size_t)vocab_size * sizeof(float);
    float *d_row = logits;
    if (!dev_logits) {
        if (grow((void **)&st.d_logits, &st.logits_cap, row_bytes)) return 0;
        d_row = st.d_logits;
        if (cudaMemcpyAsync(d_row, logits, row_bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            fail(NOEL_ERR_CUDA, "row copy failed");
            return 0;
        }
    }
    const int32_t *d_hist = nullptr;
    if (penalty) {
        if (is_device_ptr(history)) {
            d_hist = history;
        } else {
            if (grow((void **)&st.d_hist, &st.hist_cap, (size_t)history_len * sizeof(int32_t))) return 0;
            if (cudaMemcpyAsync(st.d_hist, history, (size_t)history_len * sizeof(int32_t),
                                cudaMemcpyHostToDevice, s) != cudaSuccess) {
                fail(NOEL_ERR_CUDA, "history copy failed");
                return 0;
            }
            d_hist = st.d_hist;
        }
    }
    /* the drawn-from list: at most top_k entries when top-k applies */
    const noel_sampler_config_t &cf = sampler->config;
    int list = sampler->candidate_capacity < 4096 ? sampler->candidate_capacity : 4096;
    if (cf.temperature <= 1e-4f) list = list < 1 ? list : 1;
    else if (cf.top_k > 0 && cf.top_k < list) list = cf.top_k;
    if (list > st.list_cap) {
        cudaFree(st.d_list);
        cudaFree(st.d_listw);
        st.d_list = nullptr;
        st.d_listw = nullptr;
        st.list_cap = 0;
        if (cudaMalloc(&st.d_list, (size_t)list * 4) != cudaSuccess ||
            cudaMalloc(&st.d_listw, (size_t)list * 4) != cudaSuccess) {
            fail(NOEL_ERR_CUDA, "staging allocation failed");
            return 0;
        }
        st.list_cap = list;
    }
    if (cudaMemcpyAsync(st.d_rng, sampler->rng_state, 16, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fail(NOEL_ERR_CUDA, "state copy failed");
        return 0;
    }
    /* the penalised entries go back to a host row from the host (the same
     * fp32 operations, without copying the row back); a device row is
     * written on the device */
    const bool host_wb = penalty && !dev_logits && !is_device_ptr(history);
    noel_sample_extras_t ex{};
    ex.d_list_ids = list > 0 ? st.d_list : nullptr;
    ex.d_list_probs = list > 0 ? st.d_listw : nullptr;
    ex.list_len = list;
    ex.list_weights = 1;
    ex.d_stats = st.d_out + 4;
    ex.write_back = penalty && !host_wb ? 1 : 0;
    /* one row: the single-pass kernel's wide batches (a batch this small
     * runs at 2 CTAs per SM, each row with four times the loads in flight) */
    const int hl = penalty ? history_len : 0;
    if (sample_batch(&sampler->config, d_row, NOEL_DTYPE_F32, 1, vocab_size, (size_t)vocab_size, d_hist, hl,
                     (size_t)history_len, st.d_rng, st.d_out, &ex, s))
        return 0;
    /* results through one pinned block, one synchronisation */
    const size_t pin_need = 64 + (size_t)(list > 0 ? list : 0) * 8;
    if (st.pin_cap < pin_need) {
        cudaFreeHost(st.h_pin);
        st.h_pin = nullptr;
        st.pin_cap = 0;
        if (cudaHostAlloc(&st.h_pin, pin_need, cudaHostAllocDefault) != cudaSuccess) {
            fail(NOEL_ERR_CUDA, "pinned staging allocation failed");
            return 0;
        }
        st.pin_cap = pin_need;
    }
    int32_t *out = static_cast<int32_t *>(st.h_pin);                         // id, stats[4]
    uint64_t *rng_out = reinterpret_cast<uint64_t *>(static_cast<char *>(st.h_pin) + 32);
    int32_t *lid = reinterpret_cast<int32_t *>(static_cast<char *>(st.h_pin) + 64);
    float *lw = reinterpret_cast<float *>(lid + (list > 0 ? list : 0));
    cudaMemcpyAsync(out, st.d_out, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    cudaMemcpyAsync(rng_out, st.d_rng, 16, cudaMemcpyDeviceToHost, s);
    if (list > 0) {
        cudaMemcpyAsync(lid, st.d_list, (size_t)list * 4, cudaMemcpyDeviceToHost, s);
        cudaMemcpyAsync(lw, st.d_listw, (size_t)list * 4, cudaMemcpyDeviceToHost, s);
    }
    if (ex.write_back && !dev_logits) cudaMemcpyAsync(logits, d_row, row_bytes, cudaMemcpyDeviceToHost, s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        fail(NOEL_ERR_CUDA, "sampling failed: %s", cudaGetErrorString(e));
        return 0;
    }
    sampler->rng_state[0] = rng_out[0];
    sampler->rng_state[1] = rng_out[1];
    if (host_wb) host_penalize(logits, vocab_size, history, history_len, &sampler->config);
    const int nfinal = out[4 + NOEL_STAT_N_FINAL];
    for (int i = 0; i < list && i < nfinal; ++i) {
        sampler->candidates[i].id = lid[i];
        sampler->candidates[i].val = lw[i];
    }
    ok();
    return out[0];
}

/* ========================================================================= */
/* batched entry points (include/noel_sampler_cuda.h)                         */

extern "C" int noel_sampler_sample_batch(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                                         int batch, int vocab, size_t ld, const int32_t *d_history,
                                         int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                                         float *d_probs, void *stream) {
    noel_sample_extras_t ex{};
    ex.d_probs = d_probs;
    return sample_batch(cfg, d_logits, dtype, batch, vocab, ld, d_history, history_len, hld, d_rng, d_ids,
                        &ex, static_cast<cudaStream_t>(stream));
}

extern "C" int noel_sampler_sample_batch_ex(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                                            int batch, int vocab, size_t ld, const int32_t *d_history,
                                            int history_len, size_t hld, uint64_t *d_rng, int32_t *d_ids,
                                            const noel_sample_extras_t *extras, void *stream) {
    return sample_batch(cfg, d_logits, dtype, batch, vocab, ld, d_history, history_len, hld, d_rng, d_ids,
                        extras, static_cast<cudaStream_t>(stream));
}

namespace {
struct HostBatchStage {
    int dev = -1;
    cudaStream_t stream = nullptr;
    void *d_logits = nullptr;
    size_t logits_cap = 0;
    void *d_hist = nullptr;
    size_t hist_cap = 0;
    void *d_rng = nullptr;
    size_t rng_cap = 0;
    void *d_ids = nullptr;
    size_t ids_cap = 0;
    void *d_probs = nullptr;
    size_t probs_cap = 0;
    /* the buffers and stream of the device they were made on, freed with
     * that device current (a thread that moves to another device frees them
     * first) */
    void release() {
        if (dev < 0) return;
        int cur = -1;
        cudaGetDevice(&cur);
        cudaSetDevice(dev);
        if (stream) cudaStreamSynchronize(stream);
        cudaFree(d_logits);
        cudaFree(d_hist);
        cudaFree(d_rng);
        cudaFree(d_ids);
        cudaFree(d_probs);
        if (stream) cudaStreamDestroy(stream);
        if (cur >= 0) cudaSetDevice(cur);
        *this = HostBatchStage{};
    }
    ~HostBatchStage() { release(); }
};
thread_local HostBatchStage t_hb;
}  // namespace

/* ------------------------------------------------------ vocab-sharded rows */
/* ------------------------------------------------ the pipeline's sampler */
static_assert(sizeof(noel_postreq_params_t) == 24, "aether_sampling_params_t layout");

extern "C" int noel_postreq_sample_batch(const noel_postreq_params_t *params, float *d_logits, int batch, int vocab,
                                         size_t ld, const float *d_uniform, int32_t *d_ids, void *stream) {
    if (!params) return fail(NOEL_ERR_INVALID_ARG, "params is NULL");
    if (batch < 0 || vocab <= 0) return fail(NOEL_ERR_INVALID_ARG, "batch %d / vocab %d", batch, vocab);
    if (ld < (size_t)vocab) return fail(NOEL_ERR_INVALID_ARG, "ld %zu < vocab %d", ld, vocab);
    if (batch == 0) return ok();
    if (!d_logits || !d_ids || (!d_uniform && params->temperature > 1e-4f))
        return fail(NOEL_ERR_INVALID_ARG, "logits, ids and (non-greedy) uniforms are required");
    if (reinterpret_cast<uintptr_t>(d_logits) & 3) return fail(NOEL_ERR_INVALID_ARG, "logits not 4-byte aligned");
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    PostArgs pa{};
    pa.logits = d_logits;
    pa.ld = (int64_t)ld;
    pa.batch = batch;
    pa.vocab = vocab;
    pa.temperature = params->temperature;
    pa.top_p = params->top_p;
    pa.top_k = params->top_k;
    pa.uniform = d_uniform;
    pa.ids = d_ids;
    pa.et = c->et;
    postreq_sample_kernel<<<batch, kPostThreads, 0, static_cast<cudaStream_t>(stream)>>>(pa);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

extern "C" int noel_postreq_apply_penalties_batch(float *d_logits, int batch, int vocab, size_t ld,
                                                  const int32_t *d_history, int history_len, size_t hld,
                                                  float penalty, int window, void *stream) {
    if (batch < 0 || vocab <= 0) return fail(NOEL_ERR_INVALID_ARG, "batch %d / vocab %d", batch, vocab);
    if (penalty <= 1.0f || history_len <= 0 || batch == 0) return ok();  // pipeline_stages.c:67
    if (!d_logits || !d_history) return fail(NOEL_ERR_INVALID_ARG, "logits and history are required");
    if (ld < (size_t)vocab || hld < (size_t)history_len) return fail(NOEL_ERR_INVALID_ARG, "ld / hld too small");
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    const int start = (window > 0 && history_len > window) ? history_len - window : 0;  // pipeline_stages.c:69
    const int n = history_len - start;
    const int cap = pow2_at_least(2 * n > 64 ? 2 * n : 64);
    const size_t smem = (size_t)cap * 8;
    if (smem > c->smem_optin - 1024) return fail(NOEL_ERR_TOO_LARGE, "history window %d", n);
    r = set_smem(c, (const void *)postreq_penalty_kernel, smem);
    if (r) return r;
    postreq_penalty_kernel<<<batch, kPostThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        d_logits, (int64_t)ld, vocab, d_history, (int64_t)hld, history_len, start, penalty, cap);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

extern "C" int noel_postreq_grammar_mask_batch(float *d_logits, int batch, int vocab, size_t ld,
                                               const int32_t *d_fsm_state, int fsm_state, void *stream) {
    if (batch < 0 || vocab <= 0) return fail(NOEL_ERR_INVALID_ARG, "batch %d / vocab %d", batch, vocab);
    if (batch == 0) return ok();
    if (!d_logits || ld < (size_t)vocab) return fail(NOEL_ERR_INVALID_ARG, "logits / ld");
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    const size_t n = (size_t)batch * (size_t)vocab;
    const size_t want = (n + 255) / 256;
    const int grid = (int)(want < (size_t)(c->sms * 8) ? want : (size_t)(c->sms * 8));
    postreq_grammar_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_logits, (int64_t)ld, batch, vocab,
                                                                               d_fsm_state, fsm_state);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

namespace {
/* per-thread buffers of the single-row pipeline sampler */
struct PostStage {
    int dev = -1;
    float *d_row = nullptr, *h_row = nullptr, *d_u = nullptr;
    int32_t *d_id = nullptr, *h_id = nullptr;
    int cap = 0;
    cudaStream_t stream = nullptr;
    void release() {
        if (dev < 0) return;
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(dev);
        if (stream) cudaStreamSynchronize(stream);
        cudaFree(d_row);
        cudaFree(d_u);
        cudaFree(d_id);
        cudaFreeHost(h_row);
        cudaFreeHost(h_id);
        if (stream) cudaStreamDestroy(stream);
        cudaSetDevice(cur);
        *this = PostStage{};
    }
    ~PostStage() { release(); }
};
thread_local PostStage t_post;
}  // namespace

extern "C" int32_t noel_postreq_sample(float *logits, int vocab_size, const noel_postreq_params_t *params) {
    if (!logits || vocab_size <= 0 || !params) {
        fail(NOEL_ERR_INVALID_ARG, "logits, vocab_size and params are required");
        return 0;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        fail(NOEL_ERR_NO_DEVICE, "no CUDA device");
        return 0;
    }
    PostStage &st = t_post;
    if (st.dev != dev) st.release();
    const bool greedy = params->temperature <= 1e-4f;
    /* the reference draws once, after the softmax, on non-greedy calls
     * (pipeline_stages.c:180); drawing here keeps the caller's rand() stream
     * where the reference would leave it */
    const float u = greedy ? 0.0f : (float)rand() / (float)RAND_MAX;
    auto step = [&]() -> int {
        if (!st.stream) {
            st.dev = dev;
            CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
            CUDA_TRY(cudaMalloc(&st.d_u, sizeof(float)));
            CUDA_TRY(cudaMalloc(&st.d_id, sizeof(int32_t)));
            CUDA_TRY(cudaMallocHost(&st.h_id, sizeof(int32_t)));
        }
        const bool on_dev = is_device_ptr(logits);
        float *row = logits;
        if (!on_dev) {
            if (st.cap < vocab_size) {
                cudaFree(st.d_row);
                cudaFreeHost(st.h_row);
                st.d_row = nullptr;
                st.h_row = nullptr;
                st.cap = 0;
                CUDA_TRY(cudaMalloc(&st.d_row, (size_t)vocab_size * sizeof(float)));
                CUDA_TRY(cudaMallocHost(&st.h_row, (size_t)vocab_size * sizeof(float)));
                st.cap = vocab_size;
            }
            memcpy(st.h_row, logits, (size_t)vocab_size * sizeof(float));
            CUDA_TRY(cudaMemcpyAsync(st.d_row, st.h_row, (size_t)vocab_size * sizeof(float), cudaMemcpyHostToDevice,
                                     st.stream));
            row = st.d_row;
        }
        CUDA_TRY(cudaMemcpyAsync(st.d_u, &u, sizeof(float), cudaMemcpyHostToDevice, st.stream));
        int r2 = noel_postreq_sample_batch(params, row, 1, vocab_size, (size_t)vocab_size, st.d_u, st.d_id, st.stream);
        if (r2) return r2;
        CUDA_TRY(cudaMemcpyAsync(st.h_id, st.d_id, sizeof(int32_t), cudaMemcpyDeviceToHost, st.stream));
        if (!on_dev && !greedy)  // the row now holds the probabilities, as in the reference
            CUDA_TRY(cudaMemcpyAsync(st.h_row, st.d_row, (size_t)vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                                     st.stream));
        CUDA_TRY(cudaStreamSynchronize(st.stream));
        if (!on_dev && !greedy) memcpy(logits, st.h_row, (size_t)vocab_size * sizeof(float));
        return NOEL_OK;
    };
    if (step() != NOEL_OK) return 0;
    ok();
    return *st.h_id;
}

/* ------------------------------------------------ LM head -> sampler */
namespace {
template <int WT, int NB>
int head_launch_nb(DeviceCtx *c, const HeadArgs &h, cudaStream_t s) {
    const int grid = (h.rows + kHeadThreads - 1) / kHeadThreads;
    const int r = set_smem(c, (const void *)lmhead_gemv_kernel<WT, NB>, head_smem_bytes());
    if (r) return r;
    lmhead_gemv_kernel<WT, NB><<<grid, kHeadThreads, head_smem_bytes(), s>>>(h);
    CUDA_TRY(cudaGetLastError());
    return NOEL_OK;
}
template <int WT>
int head_launch(DeviceCtx *c, const HeadArgs &h, int nb, cudaStream_t s) {
    switch (nb) {
        case 8: return head_launch_nb<WT, 8>(c, h, s);
        case 4: return head_launch_nb<WT, 4>(c, h, s);
        case 2: return head_launch_nb<WT, 2>(c, h, s);
        default: return head_launch_nb<WT, 1>(c, h, s);
    }
}
}  // namespace

extern "C" int noel_lmhead_sample(const noel_sampler_config_t *cfg, const void *d_weight, int weight_type,
                                  size_t ldw, const float *d_hidden, size_t ldh, int batch, int hidden_dim, int vocab,
                                  const int32_t *d_history, int history_len, size_t hld, uint64_t *d_rng,
                                  int32_t *d_ids, float *d_probs, float *d_logits, void *stream) {
    if (!cfg || !d_weight || !d_hidden || !d_logits) return fail(NOEL_ERR_INVALID_ARG, "cfg, weight, hidden and logits are required");
    if (weight_type != NOEL_HEAD_F32 && weight_type != NOEL_HEAD_F16 && weight_type != NOEL_HEAD_BF16)
        return fail(NOEL_ERR_UNSUPPORTED, "weight type %d (F32 0, F16 1, BF16 30)", weight_type);
    if (batch < 0 || vocab <= 0 || hidden_dim <= 0) return fail(NOEL_ERR_INVALID_ARG, "batch / vocab / hidden_dim");
    if (hidden_dim % 8) return fail(NOEL_ERR_UNSUPPORTED, "hidden_dim %d is not a multiple of 8", hidden_dim);
    if (ldw < (size_t)hidden_dim || ldw % 8 || ldh < (size_t)hidden_dim || ldh % 4)
        return fail(NOEL_ERR_INVALID_ARG, "ldw %zu (multiple of 8) / ldh %zu (multiple of 4)", ldw, ldh);
    if ((reinterpret_cast<uintptr_t>(d_weight) & 15) || (reinterpret_cast<uintptr_t>(d_hidden) & 15) ||
        (reinterpret_cast<uintptr_t>(d_logits) & 3))
        return fail(NOEL_ERR_INVALID_ARG, "weight and hidden must be 16-byte aligned");
    if (batch == 0) return ok();
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int t0 = 0; t0 < batch;) {
        const int left = batch - t0;
        const int nb = left >= 8 ? 8 : (left >= 4 ? 4 : (left >= 2 ? 2 : 1));
        HeadArgs h{};
        h.w = d_weight;
        h.ldw = (int64_t)ldw;
        h.x = d_hidden + (size_t)t0 * ldh;
        h.ldx = (int64_t)ldh;
        h.rows = vocab;
        h.cols = hidden_dim;
        h.y = d_logits + (size_t)t0 * (size_t)vocab;
        h.ldy = vocab;
        r = weight_type == NOEL_HEAD_F32 ? head_launch<kHeadF32>(c, h, nb, s)
            : weight_type == NOEL_HEAD_F16 ? head_launch<kHeadF16>(c, h, nb, s)
                                           : head_launch<kHeadBF16>(c, h, nb, s);
        if (r) return r;
        t0 += nb;
    }
    noel_sample_extras_t ex{};
    ex.d_probs = d_probs;
    return sample_batch(cfg, d_logits, NOEL_DTYPE_F32, batch, vocab, (size_t)vocab, d_history, history_len, hld,
                        d_rng, d_ids, &ex, s);
}

extern "C" int noel_moe_route_top_k(const float *d_gate_logits, int n_tokens, int n_experts, size_t ld, int top_k,
                                    noel_moe_routing_t *d_routing, void *stream) {
    if (n_tokens < 0) return fail(NOEL_ERR_INVALID_ARG, "n_tokens %d", n_tokens);
    if (n_experts < 1 || n_experts > kRouterMaxExperts)
        return fail(NOEL_ERR_TOO_LARGE, "n_experts %d (1..%d)", n_experts, kRouterMaxExperts);
    if (top_k < 1 || top_k > kRouterMaxTopK) return fail(NOEL_ERR_TOO_LARGE, "top_k %d (1..%d)", top_k, kRouterMaxTopK);
    if (ld < (size_t)n_experts) return fail(NOEL_ERR_INVALID_ARG, "ld %zu < n_experts %d", ld, n_experts);
    if (n_tokens == 0) return ok();
    if (!d_gate_logits || !d_routing) return fail(NOEL_ERR_INVALID_ARG, "gate logits and routing are required");
    if ((reinterpret_cast<uintptr_t>(d_gate_logits) & 3) || (reinterpret_cast<uintptr_t>(d_routing) & 7))
        return fail(NOEL_ERR_INVALID_ARG, "gate logits must be 4-byte and routing 8-byte aligned");
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    RouterArgs ra{};
    ra.logits = d_gate_logits;
    ra.ld = (int64_t)ld;
    ra.tokens = n_tokens;
    ra.experts = n_experts;
    ra.top_k = top_k;
    ra.out = reinterpret_cast<uint2 *>(d_routing);
    ra.et = c->et;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int tgrid = (n_tokens + kRouterThreads - 1) / kRouterThreads;
    if (top_k <= 8) moe_route_thread_kernel<8><<<tgrid, kRouterThreads, 0, s>>>(ra);
    else if (top_k <= 16) moe_route_thread_kernel<16><<<tgrid, kRouterThreads, 0, s>>>(ra);
    else moe_route_kernel<<<(n_tokens + kRouterWarps - 1) / kRouterWarps, 32 * kRouterWarps, 0, s>>>(ra);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

extern "C" int noel_sampler_shard_list_len(const noel_sampler_config_t *cfg) {
    if (!cfg) return fail(NOEL_ERR_INVALID_ARG, "cfg is NULL");
    return shard_plan(cfg).len;
}

extern "C" int noel_sampler_shard_select(const noel_sampler_config_t *cfg, const void *d_logits, int dtype,
                                         int batch, int shard_vocab, size_t ld, int v_begin,
                                         const int32_t *d_history, int history_len, size_t hld,
                                         uint32_t *d_lists, void *stream) {
    ShardOut so{v_begin, reinterpret_cast<uint2 *>(d_lists)};
    if (reinterpret_cast<uintptr_t>(d_lists) & 7) return fail(NOEL_ERR_INVALID_ARG, "d_lists must be 8-byte aligned");
    return sample_batch(cfg, d_logits, dtype, batch, shard_vocab, ld, d_history, history_len, hld, nullptr, nullptr,
                        nullptr, static_cast<cudaStream_t>(stream), nullptr, &so);
}

extern "C" int noel_sampler_shard_merge(const noel_sampler_config_t *cfg, int n_shards, int batch,
                                        const uint32_t *d_lists, uint64_t *d_rng, int32_t *d_ids, float *d_probs,
                                        int32_t *d_status, void *stream) {
    if (!cfg) return fail(NOEL_ERR_INVALID_ARG, "cfg is NULL");
    if (n_shards <= 0 || batch < 0) return fail(NOEL_ERR_INVALID_ARG, "n_shards %d / batch %d", n_shards, batch);
    if (batch == 0) return ok();
    const ShardPlan sp = shard_plan(cfg);
    const int K = sp.len;
    if (!d_lists || !d_rng || !d_ids || !d_status)
        return fail(NOEL_ERR_INVALID_ARG, "lists, rng, ids and status are required");
    if (reinterpret_cast<uintptr_t>(d_lists) & 7) return fail(NOEL_ERR_INVALID_ARG, "d_lists must be 8-byte aligned");
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    const size_t smem = (size_t)kMergeWarps * merge_warp_bytes(n_shards, K);
    if (smem > c->smem_optin - 1024) return fail(NOEL_ERR_TOO_LARGE, "%d shards x %d entries need %zu B of shared memory",
                                                 n_shards, K, smem);
    r = set_smem(c, (const void *)shard_merge_kernel, smem);
    if (r) return r;
    MergeArgs m{};
    m.n_shards = n_shards;
    m.batch = batch;
    m.len = K;
    m.full = sp.mode == kFullList;
    m.lists = reinterpret_cast<const uint2 *>(d_lists);
    m.greedy = cfg->temperature <= 1e-4f;  // sampler.c:106
    m.inv_t = 1.0f / cfg->temperature;     // sampler.c:132
    m.top_p = cfg->top_p;
    m.top_k = cfg->top_k;
    m.rng = d_rng;
    m.ids = d_ids;
    m.probs = d_probs;
    m.status = d_status;
    m.et = c->et;
    const int grid = (batch + kMergeWarps - 1) / kMergeWarps;
    shard_merge_kernel<<<grid, 32 * kMergeWarps, smem, static_cast<cudaStream_t>(stream)>>>(m);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

extern "C" int noel_sampler_sample_batch_host(const noel_sampler_config_t *cfg, const void *h_logits, int dtype,
                                              int batch, int vocab, size_t ld, const int32_t *h_history,
                                              int history_len, size_t hld, uint64_t *h_rng, int32_t *h_ids,
                                              float *h_probs) {
    if (!cfg || !h_logits || !h_rng || !h_ids || batch < 0 || vocab <= 0 || ld < (size_t)vocab)
        return fail(NOEL_ERR_INVALID_ARG, "invalid arguments");
    if (dtype != NOEL_DTYPE_F32 && dtype != NOEL_DTYPE_BF16) return fail(NOEL_ERR_INVALID_ARG, "dtype %d", dtype);
    if (h_history && history_len > 0 && hld < (size_t)history_len)
        return fail(NOEL_ERR_INVALID_ARG, "hld %zu < history_len %d", hld, history_len);
    if (batch == 0) return ok();
    HostBatchStage &st = t_hb;
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (st.dev != dev) {
        st.release();
        st.dev = dev;
        CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
    }
    cudaStream_t s = st.stream;
    const size_t es = dtype == NOEL_DTYPE_F32 ? 4 : 2;
    const size_t row_bytes = (size_t)vocab * es;
    int r;
    if ((r = grow(&st.d_logits, &st.logits_cap, (size_t)batch * row_bytes))) return r;
    if ((r = grow(&st.d_rng, &st.rng_cap, (size_t)batch * 16))) return r;
    if ((r = grow(&st.d_ids, &st.ids_cap, (size_t)batch * 4))) return r;
    if (h_probs && (r = grow(&st.d_probs, &st.probs_cap, (size_t)batch * 4))) return r;
    if (ld == (size_t)vocab)
        CUDA_TRY(cudaMemcpyAsync(st.d_logits, h_logits, (size_t)batch * row_bytes, cudaMemcpyHostToDevice, s));
    else
        CUDA_TRY(cudaMemcpy2DAsync(st.d_logits, row_bytes, h_logits, ld * es, row_bytes, batch,
                                   cudaMemcpyHostToDevice, s));
    const bool use_hist = h_history && history_len > 0;
    if (use_hist) {
        if ((r = grow(&st.d_hist, &st.hist_cap, (size_t)batch * history_len * 4))) return r;
        CUDA_TRY(cudaMemcpy2DAsync(st.d_hist, (size_t)history_len * 4, h_history, hld * 4,
                                   (size_t)history_len * 4, batch, cudaMemcpyHostToDevice, s));
    }
    CUDA_TRY(cudaMemcpyAsync(st.d_rng, h_rng, (size_t)batch * 16, cudaMemcpyHostToDevice, s));
    noel_sample_extras_t ex{};
    ex.d_probs = h_probs ? static_cast<float *>(st.d_probs) : nullptr;
    r = sample_batch(cfg, st.d_logits, dtype, batch, vocab, (size_t)vocab,
                     use_hist ? static_cast<const int32_t *>(st.d_hist) : nullptr, use_hist ? history_len : 0,
                     (size_t)history_len, static_cast<uint64_t *>(st.d_rng), static_cast<int32_t *>(st.d_ids),
                     &ex, s);
    if (r) return r;
    CUDA_TRY(cudaMemcpyAsync(h_ids, st.d_ids, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaMemcpyAsync(h_rng, st.d_rng, (size_t)batch * 16, cudaMemcpyDeviceToHost, s));
    if (h_probs) CUDA_TRY(cudaMemcpyAsync(h_probs, st.d_probs, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    return ok();
}

extern "C" int noel_sampler_cuda_sync_check(void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CUDA_TRY(cudaStreamSynchronize(s));
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    int32_t *flag = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = c->ws.find(s);
        if (it != c->ws.end()) flag = it->second.counters + 3;
    }
    if (!flag) return ok();
    int32_t v = 0;
    CUDA_TRY(cudaMemcpy(&v, flag, sizeof(v), cudaMemcpyDeviceToHost));
    if (v) {
        CUDA_TRY(cudaMemset(flag, 0, sizeof(v)));
        return fail(NOEL_ERR_DEVICE_WAIT, "a device-side wait ran out of its limit");
    }
    return ok();
}

extern "C" int noel_sampler_cuda_set_wait_limit(long long wait_ns, int stall_next_call) {
    if (wait_ns < 0) return fail(NOEL_ERR_INVALID_ARG, "wait_ns %lld", wait_ns);
    t_wait_ns = wait_ns == 0 ? kDefaultWaitNs : (unsigned long long)wait_ns;
    t_stall_next = stall_next_call ? 1 : 0;
    return ok();
}

extern "C" int noel_sampler_cuda_last_error(void) { return t_status; }
extern "C" const char *noel_sampler_cuda_last_error_message(void) { return t_msg; }
extern "C" const char *noel_sampler_cuda_status_string(int status) {
    switch (status) {
        case NOEL_OK: return "ok";
        case NOEL_ERR_INVALID_ARG: return "invalid argument";
        case NOEL_ERR_CUDA: return "CUDA error";
        case NOEL_ERR_NO_DEVICE: return "no usable device";
        case NOEL_ERR_TOO_LARGE: return "size too large";
        case NOEL_ERR_UNSUPPORTED: return "unsupported option";
        case NOEL_ERR_DEVICE_WAIT: return "device-side wait ran out";
        default: return "unknown status";
    }
}

extern "C" int noel_sampler_cuda_expf_table_size(void) { return NOEL_EXPF_NEXC; }

extern "C" int noel_sampler_cuda_profile_events(void *ev_before, void *ev_after) {
    t_ev_before = static_cast<cudaEvent_t>(ev_before);
    t_ev_after = static_cast<cudaEvent_t>(ev_after);
    return ok();
}

extern "C" int noel_sampler_cuda_expf_checksums(int chunk_log2, uint64_t *d_out, void *stream) {
    if (!d_out || chunk_log2 < 10 || chunk_log2 > 30) return fail(NOEL_ERR_INVALID_ARG, "chunk_log2 %d", chunk_log2);
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    const uint64_t span = (uint64_t)(NOEL_EXPF_DOMAIN_END - NOEL_EXPF_DOMAIN_FIRST);
    const unsigned nch = (unsigned)((span + (1ull << chunk_log2) - 1) >> chunk_log2);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CUDA_TRY(cudaMemsetAsync(d_out, 0, (size_t)nch * 8, s));
    dim3 grid(nch, 64);
    expf_checksum_kernel<<<grid, 256, 0, s>>>(chunk_log2, d_out, c->et);
    CUDA_TRY(cudaGetLastError());
    return ok();
}

/* ========================================================================= */
/* allocation-free entry point                                                */

namespace {

/*
 * Scratch of noel_sampler_sample_batch_noalloc, held in the library's device
 * image: every GPU that loads the library keeps these kNoAllocBytes
 * (8,421,632 B) until the process exits.  Layout: 4 counters (padded to
 * 256 B), the row list of the two-pass kernel (kNoAllocMaxRows int32), and
 * kNoAllocSlots candidate slots of 2 x kNoAllocMaxVocab (x, id) pairs.
 */
constexpr int kNoAllocMaxRows = 8192;
constexpr int kNoAllocMaxVocab = 262144;
constexpr int kNoAllocSlots = 2;
constexpr size_t kNoAllocRowsOff = 256;
constexpr size_t kNoAllocSlotsOff = kNoAllocRowsOff + (size_t)kNoAllocMaxRows * sizeof(int32_t);
constexpr size_t kNoAllocBytes = kNoAllocSlotsOff + (size_t)kNoAllocSlots * 2 * kNoAllocMaxVocab * sizeof(uint2);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct NoAllocDev {
    bool ready = false;
    Workspace ws;
};
std::mutex g_noalloc_mu;
NoAllocDev g_noalloc_dev[64];  // per device ordinal; fixed storage, nothing allocated per call

template <typename T>
int preset_attrs(DeviceCtx *c) {
    const size_t mx = c->smem_optin;
    const void *ks[] = {(const void *)sample_rows_kernel<T, kGreedy, 1>, (const void *)sample_rows_kernel<T, kTopK, 1>,
                        (const void *)sample_rows_kernel<T, kTopK, 4>, (const void *)sample_rows_kernel<T, kFullList, 1>,
                        (const void *)sample_rows_kernel<T, kFullList, 4>, (const void *)sample_rows_block_kernel<T, kTopK>,
                        (const void *)exact_rows_kernel<T>, (const void *)stream_rows_kernel<T, kGreedy>,
                        (const void *)stream_rows_kernel<T, kTopK>, (const void *)stream_rows_kernel<T, kFullList>};
    for (const void *k : ks) {
        cudaFuncAttributes fa;
        CUDA_TRY(cudaFuncGetAttributes(&fa, k));
        int r = set_smem(c, k, mx - fa.sharedSizeBytes);  // dynamic limit: opt-in minus static
        if (r) return r;
    }
    return NOEL_OK;
}

/* once per device, with that device current: the scratch's device address */
int noalloc_setup(int dev, DeviceCtx *c, const Workspace **out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDev &d = g_noalloc_dev[dev];
    if (!d.ready) {
        void *base = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&base, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(NOEL_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        int r = preset_attrs<float>(c);
        if (!r) r = preset_attrs<uint16_t>(c);
        if (r) return r;
        unsigned char *b = static_cast<unsigned char *>(base);
        d.ws.counters = reinterpret_cast<int32_t *>(b);
        d.ws.rows = reinterpret_cast<int32_t *>(b + kNoAllocRowsOff);
        d.ws.slots = reinterpret_cast<uint2 *>(b + kNoAllocSlotsOff);
        d.ws.rows_cap = kNoAllocMaxRows;
        d.ws.vocab_cap = kNoAllocMaxVocab;
        d.ws.nslots = kNoAllocSlots;
        d.ready = true;
    }
    *out = &d.ws;
    return NOEL_OK;
}

}  // namespace

extern "C" int noel_sampler_sample_batch_noalloc(const noel_sampler_config_t *cfg, const void *d_logits,
                                                 int dtype, int batch, int vocab, size_t ld,
                                                 const int32_t *d_history, int history_len, size_t hld,
                                                 uint64_t *d_rng, int32_t *d_ids, float *d_probs, void *stream) {
    if (batch > kNoAllocMaxRows || vocab > kNoAllocMaxVocab)
        return fail(NOEL_ERR_TOO_LARGE,
                    "noalloc entry point handles at most %d rows of at most %d tokens (got %d x %d); "
                    "use noel_sampler_sample_batch",
                    kNoAllocMaxRows, kNoAllocMaxVocab, batch, vocab);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(NOEL_ERR_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(NOEL_ERR_NO_DEVICE, "device ordinal %d", dev);
    DeviceCtx *c = nullptr;
    int r = device_ctx(&c);
    if (r) return r;
    const Workspace *ws = nullptr;
    r = noalloc_setup(dev, c, &ws);
    if (r) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    /* the array keeps the last call's contents: the row list starts empty */
    CUDA_TRY(cudaMemsetAsync(ws->counters, 0, 4 * sizeof(int32_t), s));
    noel_sample_extras_t ex{};
    ex.d_probs = d_probs;
    return sample_batch(cfg, d_logits, dtype, batch, vocab, ld, d_history, history_len, hld, d_rng, d_ids, &ex,
                        s, ws);
}
