/*
 * The single-pass sampling kernel for greedy rows, top-k rows with k <= 120
 * and full-list rows (top-k off): one CTA of 4 warps per row, warps that
 * stream the row without block barriers, and a shared-memory footprint small
 * enough for 7-8 CTAs per SM, so 1024 rows run in one wave.
 *
 * Row start: the window of the row's history becomes a bitmap of 8-id blocks
 * and an open-addressing table of (id, occurrences) (sampler.c:87-93).
 * Streaming: 256-bit ld.global.nc.L1::no_allocate.L2::evict_first loads; each
 * lane takes the maximum of each vector and only looks at single elements when
 * that raw maximum can pass the current filter.  The repetition penalty only
 * lowers values (sampler.c:96-100), so it is applied exactly, but only to
 * vectors that can pass.
 *   greedy  - a quarter of the row per warp, one batch prefetched in
 *             registers; the running (value desc, id asc) maximum
 *             (sampler.c:106-116).
 *   top-k   - the K' = pow2(k+8) best (logit desc, id asc).  Warps take
 *             batches of the row as they free up and queue passing vectors
 *             in shared memory; a drain tests them element by element, keeps
 *             the warp's best kw in a shared-memory buffer (register bitonic
 *             sort when it fills) and publishes a ladder of kept keys; any
 *             combination with K' retained keys above it is a valid filter
 *             for every warp.  A block warm-up on the first batches starts
 *             the filter near the K'-th largest.
 *   full    - the -15 cut under the running maximum (sampler.c:137-138).
 * Row end: warp 0 gathers the kept keys, selects the K' best, checks that no
 * excluded element could belong to the top k (else the row goes to the
 * two-pass kernel), computes the weights and runs the sequential mass /
 * nucleus / draw loops of sampler.c:160-191; for a vocab shard it writes the
 * shard's K' best instead.
 */
#pragma once

#include "sampler_device.cuh"

namespace noel {

constexpr int kRowWarps = 4;  // warps streaming one row

constexpr int kRowThreads = 32 * kRowWarps;
constexpr int kWarpBins = 512;    // per level of the warm-up histogram (9 key bits)

/* ---------------------------------------------------------------------- */
/* the row's history: a bitmap of 8-id blocks + open addressing (id -> n)   */

struct HistSet {
    uint32_t *blk;    // bit b: some history id in [8b, 8b + 8); (V + 255) / 256 words
    uint32_t *key;    // cap: id + 1, 0 = empty
    uint32_t *val;    // cap: occurrences in the window while building, then the
                      // penalised logit (float bits)
    int cap;          // power of two >= 2 x window
};

__host__ __device__ inline int hs_blk_words(int V) { return (V + 255) / 256; }

__device__ __forceinline__ uint32_t hs_hash(uint32_t id) {
    return id * 0x9E3779B1u;  // Fibonacci hashing
}

/* The window's distinct ids with their occurrence counts, then each id's
 * penalised logit, computed once per row: the penalty applies per occurrence
 * (sampler.c:93-102), so an id seen c times takes c dependent roundings, and
 * the streaming code only substitutes the stored value. */
template <typename T, int NT>
__device__ void hs_build(const HistSet &h, const int32_t *hrow, int first, int H, int V, int id_off,
                         const void *rowp, float rep) {
    for (int i = threadIdx.x; i < hs_blk_words(V); i += NT) h.blk[i] = 0u;
    for (int i = threadIdx.x; i < h.cap; i += NT) {
        h.key[i] = 0u;
        h.val[i] = 0u;
    }
    __syncthreads();
    constexpr int R = kHistBatch;
    const int bits = __ffs(h.cap) - 1;
    for (int b0 = first; b0 < H; b0 += NT * R) {  // R rounds of whole warps, their loads issued together
        int gv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = b0 + r * NT + (int)threadIdx.x;
            gv[r] = i < H ? hrow[i] : -1;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = b0 + r * NT + (int)threadIdx.x;
            const int gt = gv[r];
            const bool in = i < H && gt >= id_off && gt - id_off < V;  // sampler.c:95 (ids of this shard)
            if (!in) continue;
            const uint32_t t = (uint32_t)(gt - id_off);
            atomicOr(&h.blk[t >> 8], 1u << ((t >> 3) & 31));
            uint32_t p = bits ? (hs_hash(t) >> (32 - bits)) : 0u;
            for (int probe = 0; probe < h.cap; ++probe) {
                const uint32_t prev = atomicCAS(&h.key[p], 0u, t + 1u);
                if (prev == 0u || prev == t + 1u) {  // claimed, or the id's slot already
                    atomicAdd(&h.val[p], 1u);
                    break;
                }
                p = (p + 1) & (uint32_t)(h.cap - 1);
            }
        }
    }
    __syncthreads();
    for (int s0 = threadIdx.x; s0 < h.cap; s0 += NT * R) {  // R logits loaded together
        float xs[R];
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const int s = s0 + k * NT;
            const uint32_t key = s < h.cap ? h.key[s] : 0u;
            xs[k] = key ? Fmt<T>::scalar(rowp, (int)(key - 1u)) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const int s = s0 + k * NT;
            if (s < h.cap && h.key[s]) h.val[s] = __float_as_uint(apply_penalty(xs[k], h.val[s], rep));
        }
    }
    __syncthreads();
}

/* the penalised logit of id if id is in the window */
__device__ __forceinline__ bool hs_find(const HistSet &h, uint32_t id, float &x) {
    if (!((h.blk[id >> 8] >> ((id >> 3) & 31)) & 1u)) return false;
    const int bits = __ffs(h.cap) - 1;
    uint32_t p = bits ? (hs_hash(id) >> (32 - bits)) : 0u;
    for (int probe = 0; probe < h.cap; ++probe) {
        const uint32_t k = h.key[p];
        if (k == id + 1u) {
            x = __uint_as_float(h.val[p]);
            return true;
        }
        if (k == 0u) return false;
        p = (p + 1) & (uint32_t)(h.cap - 1);
    }
    return false;
}

/* the penalty on N consecutive ids starting at id0 (sampler.c:93-102): one or
 * two bitmap words say whether any of them is in the window; an id in it
 * takes its penalised logit from the table */
template <int N>
__device__ __forceinline__ void hs_penalize(const HistSet &h, uint32_t id0, float *x) {
    const uint32_t b0 = id0 >> 3, b1 = (id0 + N - 1) >> 3;  // at most 3 blocks
    uint32_t any = 0u;
    for (uint32_t bb = b0; bb <= b1; ++bb) any |= (h.blk[bb >> 5] >> (bb & 31)) & 1u;
    if (!any) return;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        float v;
        if (hs_find(h, id0 + j, v)) x[j] = v;
    }
}

/* penalised values written back to the caller's fp32 row, once per distinct id */
template <int NT>
__device__ void hs_write_back(const SampleArgs &a, const HistSet &h, int row) {
    float *wrow = a.wb + (size_t)row_span(a, row).off;
    for (int s = threadIdx.x; s < h.cap; s += NT) {
        const uint32_t k = h.key[s];
        if (k) wrow[k - 1] = __uint_as_float(h.val[s]);
    }
}

/* Bin of the K-th largest count of a kWarpBins histogram (counted from the top
 * bin down), found by all NT threads; -1 if the total is below K.
 * *need_in_bin = how many of that bin's entries are needed. */
template <int NT>
__device__ int block_find_bin_desc(const uint32_t *h, int K, int *s_w, int *s_res, int *need_in_bin) {
    constexpr int PER = kWarpBins / NT;
    const int hi = kWarpBins - 1 - threadIdx.x * PER;
    int c[PER], sum = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        c[j] = (int)h[hi - j];
        sum += c[j];
    }
    int total;
    const int before = block_excl_scan<NT>(sum, s_w, total);
    if (threadIdx.x == 0) s_res[0] = -1;
    __syncthreads();
    if (before < K && K <= before + sum) {
        int cum = before;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            if (cum < K && K <= cum + c[j]) {
                s_res[0] = hi - j;
                s_res[1] = K - cum;
            }
            cum += c[j];
        }
    }
    __syncthreads();
    *need_in_bin = s_res[1];
    return s_res[0];
}


/* 16 elements per lane per batch: two 8-float vectors or one 16-bf16 vector */
template <typename T>
struct WarpFmt;
template <>
struct WarpFmt<float> {
    static constexpr int VEC = 8, U = 2;
};
template <>
struct WarpFmt<uint16_t> {
    static constexpr int VEC = 16, U = 1;
};
constexpr int kLaneElems = 16;
constexpr int kQueueCap = 64;  // queued vectors per warp at one-wave occupancy (>= the vectors of one batch)

/* one lane's batch, passed by value to the out-of-line paths */
struct LaneBatch {
    float v[kLaneElems];
};

/* a 32-byte vector to / from shared memory as two 16-byte accesses */
__device__ __forceinline__ void st_vec(V8 *dst, const V8 &v) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    d[0] = make_uint4(v.v[0], v.v[1], v.v[2], v.v[3]);
    d[1] = make_uint4(v.v[4], v.v[5], v.v[6], v.v[7]);
}
__device__ __forceinline__ V8 ld_vec(const V8 *src) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    const uint4 a = s[0], b = s[1];
    V8 v;
    v.v[0] = a.x, v.v[1] = a.y, v.v[2] = a.z, v.v[3] = a.w;
    v.v[4] = b.x, v.v[5] = b.y, v.v[6] = b.z, v.v[7] = b.w;
    return v;
}

/* ---------------------------------------------------------------------- */
/* the row's shared state                                                   */

struct RowShared {
    unsigned long long tsh;                 // best shared top-k filter
    unsigned long long taus[kRowWarps];     // each warp's own exclusion threshold
    unsigned long long lad[3][kRowWarps];   // each warp's (2kw/NW)-th, (kw/2)-th, kw-th kept key
    int res[2];
    uint32_t maxkey;                        // running maximum key (full list)
    int flags, l0nan, trunc;
    int wcnt[kRowWarps];
    int wfill[kRowWarps];
    int next;                               // next batch to stream (queued modes)
    int w[kRowWarps + 1];
    uint32_t wmax[kRowWarps];               // each warp's largest raw sample key (warm-up)
    float gx[kRowWarps];
    uint32_t gid[kRowWarps];
};
__shared__ RowShared rs;
extern __shared__ __align__(32) unsigned char row_smem[];

/* Dynamic shared memory of one row, recomputed from the arguments wherever it
 * is needed: vector queues, the history set, per-warp candidate buffers and
 * one area reused by the warm-up histogram and the row-end gather. */
struct RowLayout {
    V8 *q;              // this warp's queue
    uint32_t *qid;      // id of each queued vector's first element
    HistSet hs;
    uint32_t *wkey, *wid;  // this warp's candidate buffer
    uint32_t *area, *ukey, *uid;
    uint64_t *sk;
};

template <int MODE>
__device__ __forceinline__ RowLayout row_layout(const SampleArgs &a, int warp) {
    constexpr int NW = kRowWarps;
    unsigned char *sp = row_smem;
    RowLayout L;
    L.q = nullptr;
    L.qid = nullptr;
    if (MODE != kGreedy) {
        L.q = reinterpret_cast<V8 *>(sp) + warp * a.qcap;
        sp += NW * a.qcap * sizeof(V8);
        L.qid = reinterpret_cast<uint32_t *>(sp) + warp * a.qcap;
        sp += NW * a.qcap * 4;
    }
    L.hs = HistSet{nullptr, nullptr, nullptr, 0};
    if (a.penalty) {
        L.hs.blk = reinterpret_cast<uint32_t *>(sp);
        sp += ((hs_blk_words(a.vocab) + 3) & ~3) * 4;  // keeps 16-byte alignment
        L.hs.cap = a.hcap;
        L.hs.key = reinterpret_cast<uint32_t *>(sp);
        sp += a.hcap * 4;
        L.hs.val = reinterpret_cast<uint32_t *>(sp);
        sp += a.hcap * 4;
    }
    L.wkey = L.wid = L.area = L.ukey = L.uid = nullptr;
    L.sk = nullptr;
    if (MODE != kGreedy) {
        L.wkey = reinterpret_cast<uint32_t *>(sp) + warp * a.cap * 2;
        L.wid = L.wkey + a.cap;
        sp += NW * a.cap * 8;
        /* warm-up bins (2 x kWarpBins), later the gather (ucap keys and ids)
         * followed by the sort keys (pow2(ucap) x u64) */
        L.area = reinterpret_cast<uint32_t *>(sp);
        L.ukey = L.area;
        L.uid = L.area + a.ucap;
        L.sk = reinterpret_cast<uint64_t *>(L.area + 2 * a.ucap);
    }
    return L;
}

__device__ __forceinline__ int warp_kw(const SampleArgs &a) { return a.kw; }

/* ---------------------------------------------------------------------- */
/* out-of-line paths                                                        */

/* Insertion of every lane's pend elements of x (ids id0 + e) into the warp's
 * buffer (all lanes call it): positions from a warp prefix sum of the lanes'
 * counts, since the warp is its buffer's only writer.  Clears pend for the
 * elements that found a slot. */
template <int N>
__device__ __forceinline__ void buffer_insert(const RowLayout &L, int warp, int capw, const float (&x)[N],
                                              uint32_t id0, uint32_t &pend) {
    const int lane = threadIdx.x & 31;
    const int cnt = __popc(pend);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
    }
    const int total = __shfl_sync(kFull, incl, 31);
    const int wf = *(volatile int *)&rs.wfill[warp];
    int pos = wf + incl - cnt;
#pragma unroll
    for (int j = 0; j < N; ++j)
        if (((pend >> j) & 1u) && pos < capw) {
            L.wkey[pos] = ord_key(x[j]);
            L.wid[pos] = id0 + (uint32_t)j;
            pend &= ~(1u << j);
            ++pos;
        }
    __syncwarp();
    if (lane == 0) rs.wfill[warp] = min(wf + total, capw);
    __syncwarp();
}

/* Keep the warp's best kw entries, publish its threshold and ladder, and raise
 * the row's shared filter to the best combination the ladders prove. */
__device__ __forceinline__ unsigned long long warp_compact(const RowLayout &L, int warp, int capw, int kw,
                                                           int kprime) {
    const int lane = threadIdx.x & 31;
    __syncwarp();
    const int n = min(*(volatile int *)&rs.wfill[warp], capw);
    __syncwarp();
    uint64_t lad[3];
    /* kw <= 96 (K' <= 128), within a 4-register sort */
    const unsigned long long tau_w =
        warp_topk_sorted_r<4>(L.wkey, L.wid, n, kw, lad, max(1, kprime / kRowWarps));
    if (lane == 0) {
        rs.wfill[warp] = kw;
        rs.taus[warp] = tau_w;
        rs.lad[0][warp] = lad[0];
        rs.lad[1][warp] = lad[1];
        rs.lad[2][warp] = lad[2];
        __threadfence_block();
        /* K' retained elements beat each of: every warp's (K'/NW)-th, the 4th
         * largest (kw/2)-th, the 2nd largest kw-th, and (when kw >= K') the
         * largest kw-th */
        unsigned long long mn = ~0ull, q4[4] = {0ull, 0ull, 0ull, 0ull}, c1 = 0ull, c2 = 0ull;
        for (int w = 0; w < kRowWarps; ++w) {
            const unsigned long long l0 = *(volatile unsigned long long *)&rs.lad[0][w];
            const unsigned long long l1 = *(volatile unsigned long long *)&rs.lad[1][w];
            const unsigned long long l2 = *(volatile unsigned long long *)&rs.lad[2][w];
            mn = min(mn, l0);
            for (int q = 0; q < 4; ++q)
                if (l1 > q4[q]) {
                    for (int z = 3; z > q; --z) q4[z] = q4[z - 1];
                    q4[q] = l1;
                    break;
                }
            if (l2 > c1) {
                c2 = c1;
                c1 = l2;
            } else if (l2 > c2) {
                c2 = l2;
            }
        }
        if (kRowWarps < 4) q4[3] = 0ull;
        atomicMax(&rs.tsh, max(max(mn, q4[3]), max(c2, kw >= kprime ? c1 : 0ull)));
    }
    __syncwarp();
    return tau_w;
}

/* Top-k drain of the warp's n queued vectors, one per lane per round: the
 * penalty, the exact (logit desc, id asc) test against the current filter,
 * insertion, and compaction whenever the buffer fills.  Returns the warp's
 * own threshold. */
template <typename T>
__device__ __forceinline__ unsigned long long topk_drain(const SampleArgs &a, int n, unsigned long long tau_w) {
    constexpr int VEC = Fmt<T>::VEC;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const RowLayout L = row_layout<kTopK>(a, warp);
    const int capw = a.cap, kw = warp_kw(a);
    for (int r = 0; r < n; r += 32) {
        const int i = r + lane;
        float x[VEC];
        uint32_t id0 = 0u, pend = 0u;
        if (i < n) {
            Fmt<T>::unpack(ld_vec(L.q + i), x);
            id0 = L.qid[i];
            if (a.penalty) hs_penalize<VEC>(L.hs, id0, x);
            const unsigned long long te = max(tau_w, *(volatile unsigned long long *)&rs.tsh);
            const uint32_t tk = (uint32_t)(te >> 32);
            const float tau_f = tk == 0u ? -INFINITY : key_float(tk);
            const uint32_t tau_id = 0xFFFFFFFFu - (uint32_t)te;  // ties at tau_f pass below this id
#pragma unroll
            for (int j = 0; j < VEC; ++j)
                if (x[j] > tau_f || (x[j] == tau_f && id0 + j < tau_id)) pend |= 1u << j;
        }
        for (;;) {
            if (!__any_sync(kFull, pend != 0u)) break;
            buffer_insert<VEC>(L, warp, capw, x, id0, pend);
            if (!__any_sync(kFull, pend != 0u)) break;
            tau_w = warp_compact(L, warp, capw, kw, a.kprime);  // the buffer is full
            const unsigned long long te = max(tau_w, *(volatile unsigned long long *)&rs.tsh);
#pragma unroll
            for (int j = 0; j < VEC; ++j)
                if (((pend >> j) & 1u) && !(comp_key(ord_key(x[j]), id0 + j) > te)) pend &= ~(1u << j);
        }
    }
    return tau_w;
}

/* Full-list drain (top-k off): penalises the queued vectors, raises the
 * running maximum, inserts what passes the -15 cut under it and drops what
 * the new maximum cuts when the buffer fills.  Sets kOverflow when the kept
 * list outgrows the buffer. */
template <typename T>
__device__ __forceinline__ void full_drain(const SampleArgs &a, int n) {
    constexpr int VEC = Fmt<T>::VEC;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const RowLayout L = row_layout<kFullList>(a, warp);
    const int capw = a.cap;
    for (int r = 0; r < n; r += 32) {
        const int i = r + lane;
        float x[VEC];
        uint32_t id0 = 0u, pend = 0u;
        float lm = -INFINITY;
        if (i < n) {
            Fmt<T>::unpack(ld_vec(L.q + i), x);
            id0 = L.qid[i];
            if (a.penalty) hs_penalize<VEC>(L.hs, id0, x);
#pragma unroll
            for (int j = 0; j < VEC; ++j) lm = fmaxf(lm, x[j]);
        }
        lm = warp_max_f(lm);
        if (lane == 0 && lm > -INFINITY) atomicMax(&rs.maxkey, ord_key(lm));
        __syncwarp();
        float m = key_float(*(volatile uint32_t *)&rs.maxkey);
        if (i < n) {
#pragma unroll
            for (int j = 0; j < VEC; ++j)
                if (scaled_diff(x[j], m, a.inv_t) > -15.0f) pend |= 1u << j;
        }
        for (;;) {
            if (!__any_sync(kFull, pend != 0u)) break;
            buffer_insert<VEC>(L, warp, capw, x, id0, pend);
            if (!__any_sync(kFull, pend != 0u)) break;
            __syncwarp();
            int nb = min(*(volatile int *)&rs.wfill[warp], capw);
            __syncwarp();
            m = key_float(*(volatile uint32_t *)&rs.maxkey);
            nb = warp_filter_by_max(L.wkey, L.wid, nb, m, a.inv_t);
            if (lane == 0) rs.wfill[warp] = nb;
            __syncwarp();
            if (nb > capw / 2) {
                if (lane == 0) atomicOr(&rs.flags, kOverflow);
                return;
            }
#pragma unroll
            for (int j = 0; j < VEC; ++j)
                if (((pend >> j) & 1u) && !(scaled_diff(x[j], m, a.inv_t) > -15.0f)) pend &= ~(1u << j);
        }
    }
}

/* Greedy slow path for one lane (repetition penalty on): penalises the
 * candidate vectors and folds them into the lane's (value desc, id asc) best. */
template <int VEC, int U>
__device__ __noinline__ uint64_t greedy_take(const SampleArgs &a, uint32_t id0, uint32_t cand, float gx,
                                             uint32_t gid, LaneBatch b) {
    const RowLayout L = row_layout<kGreedy>(a, threadIdx.x >> 5);
#pragma unroll
    for (int u = 0; u < U; ++u) {
        if (!((cand >> u) & 1u)) continue;
        const uint32_t v0 = id0 + (uint32_t)(u * 32 * VEC);
        float x[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) x[j] = b.v[u * VEC + j];
        hs_penalize<VEC>(L.hs, v0, x);
#pragma unroll
        for (int j = 0; j < VEC; ++j)
            if (x[j] > gx || (x[j] == gx && v0 + j < gid)) {
                gx = x[j];
                gid = v0 + j;
            }
    }
    return ((uint64_t)__float_as_uint(gx) << 32) | gid;
}

/* Vector of the row's body that warm-up sample slot (warp, u, lane) reads:
 * the block's NW * 32 * U slots spread evenly over the body (a uniform
 * sample of the row whatever the order of its ids), or the whole body when
 * it is shorter; -1 for a slot past it. */
template <int U>
__device__ __forceinline__ int warm_vec(int nvec, int warp, int u, int lane) {
    constexpr int NS = kRowWarps * 32 * U;
    const int j = (warp * U + u) * 32 + lane;
    if (nvec >= NS) return (int)(((long long)j * nvec) / NS);
    return j < nvec ? j : -1;
}

/* Block warm-up on the row's sample (all threads of the block; slot (u,
 * lane) of each warp's queue holds the vector warm_vec names): the smallest
 * raw lane maximum of a warp has 32 raw elements above it and becomes the
 * warp's own threshold (an exclusion threshold checked at the row end, so it
 * needs no proof); the second largest of those, lo_key, bounds a histogram
 * of the larger sample elements, penalised, in 512 bins over [lo_key, the
 * sample's largest raw key], and the floor of the bin holding the r-th
 * largest (r = warm_rank) becomes the row's starting filter.  With r < K' the filter is a bet, not a
 * proof: it drops elements below it, and the row end sends the row to the
 * two-pass kernel when fewer than K' elements passed it.  The penalty only
 * lowers values, so only elements whose raw value reaches the histogram are
 * looked up.  Returns the warp's own threshold. */
template <typename T, int UX>
__device__ __forceinline__ unsigned long long row_warmup(const SampleArgs &a, int head, int nvec) {
    using F = Fmt<T>;
    constexpr int NT = kRowThreads, NW = kRowWarps;
    constexpr int VEC = WarpFmt<T>::VEC, U = WarpFmt<T>::U * UX, NE = U * VEC;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const RowLayout L = row_layout<kTopK>(a, warp);
    float xw[NE];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        if (warm_vec<U>(nvec, warp, u, lane) >= 0) {
            F::unpack(ld_vec(L.q + u * 32 + lane), xw + u * VEC);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) xw[u * VEC + j] = -INFINITY;
        }
    }
    unsigned long long tau_w = 0ull;
    float lmax = -INFINITY;
#pragma unroll
    for (int e = 0; e < NE; ++e) lmax = fmaxf(lmax, xw[e]);  // NaN-ignoring
    const float t0 = warp_min_f(lmax);
    if (t0 > -INFINITY) {
        tau_w = (unsigned long long)ord_key(t0) << 32;  // 32 of this warp's raw elements beat it
        if (lane == 0) rs.taus[warp] = tau_w;
    }
    {
        const float wm = warp_max_f(lmax);
        if (lane == 0) rs.wmax[warp] = wm > -INFINITY ? ord_key(wm) : 0u;
    }
    __syncthreads();
    unsigned long long t1 = 0ull, t2 = 0ull;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const unsigned long long tw = rs.taus[w];
        if (tw > t1) {
            t2 = t1;
            t1 = tw;
        } else if (tw > t2) {
            t2 = tw;
        }
    }
    const uint32_t lo_key = (uint32_t)(t2 >> 32);
    /* 512 bins over the sample's key range [lo_key, largest raw key] (the
     * penalty only lowers keys, so a penalised key above lo_key stays in it) */
    uint32_t hi_key = 0u;
#pragma unroll
    for (int w = 0; w < NW; ++w) hi_key = max(hi_key, rs.wmax[w]);
    const uint32_t span = hi_key > lo_key ? hi_key - lo_key : 0u;
    const int shift = span < (uint32_t)kWarpBins ? 0 : (32 - __clz((int)span)) - 9;
    auto bin1 = [&](uint32_t key) -> uint32_t { return min((uint32_t)(kWarpBins - 1), (key - lo_key) >> shift); };
    /* The elements whose raw value reaches a floor form a bitmask; one
     * compact loop takes each one's value back from this warp's queue (which
     * still holds the batch) and its penalised value from the table (the
     * penalty only lowers values, so the raw test loses nothing).  With wide
     * batches (64 elements per lane) this saves about 10 us per row over
     * lookups unrolled across all NE registers; with 16 per lane the unrolled
     * form is slightly faster and stays. */
    const V8 *const wq = L.q;
    auto value = [&](int e) -> float {
        const int u = e / VEC, j = e - (e / VEC) * VEC;
        float x = F::scalar(wq + u * 32 + lane, j);
        float pv;
        if (a.penalty && hs_find(L.hs, (uint32_t)(head + warm_vec<U>(nvec, warp, u, lane) * VEC + j), pv)) x = pv;
        return x;
    };
    auto reach = [&](uint32_t floor_key) -> uint64_t {
        uint64_t m = 0ull;
#pragma unroll
        for (int e = 0; e < NE; ++e) {
            const float xv = xw[e];
            if (xv == xv && xv > -INFINITY && ord_key(xv) >= floor_key) m |= 1ull << e;
        }
        return m;
    };
    if (UX > 1) {
        for (uint64_t m = reach(lo_key); m; m &= m - 1) {
            const float xv = value(__ffsll((long long)m) - 1);
            if (ord_key(xv) >= lo_key) atomicAdd(&L.area[bin1(ord_key(xv))], 1u);
        }
    } else {
        if (a.penalty) {  // only what reaches the histogram needs its penalised value
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint32_t id0 = (uint32_t)(head + warm_vec<U>(nvec, warp, u, lane) * VEC);
#pragma unroll
                for (int j = 0; j < VEC; ++j) {
                    float &xv = xw[u * VEC + j];
                    float pv;
                    if (xv == xv && xv > -INFINITY && ord_key(xv) >= lo_key && hs_find(L.hs, id0 + (uint32_t)j, pv)) xv = pv;
                }
            }
        }
#pragma unroll
        for (int e = 0; e < NE; ++e) {
            const float xv = xw[e];
            if (xv == xv && xv > -INFINITY && ord_key(xv) >= lo_key) atomicAdd(&L.area[bin1(ord_key(xv))], 1u);
        }
    }
    __syncthreads();
    int need;
    const int wb1 = block_find_bin_desc<NT>(L.area, a.warm_rank > 0 ? a.warm_rank : a.kprime, rs.w, rs.res, &need);
    if (tid == 0 && wb1 >= 0)  // the bin's floor: r sample elements reach it
        rs.tsh = (unsigned long long)(lo_key + ((uint32_t)wb1 << shift)) << 32;
    __syncthreads();
    return tau_w;
}

/* Row end (all threads of the block): gather, exactness check, weights and
 * the sequential tail of sampler.c:160-191. */
template <typename T, int MODE>
__device__ __forceinline__ void row_finish(const SampleArgs &a, unsigned long long tau_w, float gx, uint32_t gid) {
    constexpr int NT = kRowThreads, NW = kRowWarps;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x;
    const RowLayout L = row_layout<MODE>(a, warp);
    const int capw = a.cap, kw = warp_kw(a);
    bool wtrunc = tau_w != 0ull;
    int wcount = 0;
    if (MODE == kGreedy) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ox = __shfl_xor_sync(kFull, gx, o);
            const uint32_t oid = __shfl_xor_sync(kFull, gid, o);
            if (ox > gx || (ox == gx && oid < gid)) {
                gx = ox;
                gid = oid;
            }
        }
        if (lane == 0) {
            rs.gx[warp] = gx;
            rs.gid[warp] = gid;
        }
        __syncthreads();
        if (a.wb && a.penalty) hs_write_back<NT>(a, L.hs, row);
        if (tid == 0) {
            float bx = rs.gx[0];
            uint32_t bid = rs.gid[0];
            for (int w = 1; w < NW; ++w)
                if (rs.gx[w] > bx || (rs.gx[w] == bx && rs.gid[w] < bid)) {
                    bx = rs.gx[w];
                    bid = rs.gid[w];
                }
            int orow = row;
            bool nan0 = rs.l0nan;
            if (a.gsplit) {
                /* a range of a split row: fold this range's best into the
                 * row's; the row's last CTA writes the result and re-arms */
                const RowSpan sp = row_span(a, row);
                uint4 *gs = a.gsplit + sp.hrow;
                unsigned long long *best = reinterpret_cast<unsigned long long *>(gs);
                if (bid != 0xFFFFFFFFu) atomicMax(best, comp_key(ord_key(bx), bid + (uint32_t)sp.id_off));
                if (sp.id_off == 0 && rs.l0nan) atomicExch(&gs->w, 1u);
                __threadfence();
                if (atomicAdd(&gs->z, 1u) != (uint32_t)a.split - 1u) return;
                __threadfence();
                const unsigned long long b = atomicExch(best, 0ull);
                nan0 = atomicExch(&gs->w, 0u) != 0u;
                gs->z = 0u;
                bid = b ? 0xFFFFFFFFu - (uint32_t)b : 0xFFFFFFFFu;
                orow = sp.hrow;
            }
            const int row = orow;
            RowOut o;
            o.id = (nan0 || bid == 0xFFFFFFFFu) ? 0 : (int)bid;  // sampler.c:106-116
            o.prob = 1.0f;
            o.mass = 1.0f;
            o.n_topk = o.n_final = o.num_cands = 1;
            o.flags = NOEL_ROW_GREEDY;
            write_row_stats(a, row, o);
            if (a.list_ids)
                for (int i = 0; i < a.list_len; ++i) {
                    a.list_ids[(size_t)row * a.list_len + i] = i == 0 ? o.id : -1;
                    if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = i == 0 ? 1.0f : 0.0f;
                }
        }
        return;
    }

    wcount = min(*(volatile int *)&rs.wfill[warp], capw);
    __syncthreads();  // all warps done streaming: rs.maxkey, rs.flags final
    if (a.wb && a.penalty) hs_write_back<NT>(a, L.hs, row);
    if (MODE == kFullList && (rs.flags & kOverflow)) {
        if (tid == 0) list_exact_row(a, row);
        return;
    }
    const float Mfull = rs.l0nan ? __uint_as_float(0x7FC00000u) : key_float(rs.maxkey);
    /* K' > 32: the whole block sorts the union of the warps' buffers; small
     * K': each warp brings its best kw and warp 0 selects from their union
     * (a sort of up to NW buffers costs more than those small selections) */
    const bool bsort = MODE == kTopK && a.kprime > 32;
    if (MODE == kTopK) {
        /* entries below the shared filter are excluded like every element
         * the filter dropped while streaming */
        const unsigned long long t2 = rs.tsh;
        if (t2) {
            int wn = 0;
            for (int b0 = 0; b0 < wcount; b0 += 32) {
                const int i = b0 + lane;
                const bool ok = i < wcount;
                const uint32_t k = ok ? L.wkey[i] : 0u, v = ok ? L.wid[i] : 0u;
                const bool keep = ok && comp_key(k, v) >= t2;
                const uint32_t bal = __ballot_sync(kFull, keep);
                __syncwarp();
                if (keep) {
                    const int pos = wn + __popc(bal & lanemask_lt());
                    L.wkey[pos] = k;
                    L.wid[pos] = v;
                }
                wn += __popc(bal);
                __syncwarp();
            }
            wcount = wn;
        }
        if (!bsort && wcount > kw) {
            tau_w = warp_topk_sorted_r<4>(L.wkey, L.wid, wcount, kw, nullptr, 1);
            wcount = kw;
            wtrunc = true;
        }
    } else {
        wcount = warp_filter_by_max(L.wkey, L.wid, wcount, Mfull, a.inv_t);
    }
    if (lane == 0) {
        rs.wcnt[warp] = wcount;
        rs.taus[warp] = wtrunc ? tau_w : 0ull;  // final exclusion threshold of this warp
        if (wtrunc) rs.trunc = 1;
    }
    __syncthreads();
    int off = 0, nu = 0;
    for (int w = 0; w < NW; ++w) {
        if (w < warp) off += rs.wcnt[w];
        nu += rs.wcnt[w];
    }
    if (nu > a.ucap) {  // full list larger than the gather area: two-pass kernel
        if (tid == 0) list_exact_row(a, row);
        return;
    }
    if (bsort) {
        /* the union (at most NW buffers) as composite keys, sorted by the
         * whole block; its best min(nu, K') go to ukey / uid in order */
        int P = 2;
        while (P < nu) P <<= 1;
        for (int i = lane; i < wcount; i += 32) L.sk[off + i] = comp_key(L.wkey[i], L.wid[i]);
        for (int i = nu + tid; i < P; i += NT) L.sk[i] = 0ull;
        __syncthreads();
        block_bitonic_pairs_desc<NT>(L.sk, P);
        for (int i = tid; i < min(nu, a.kprime); i += NT) {
            const uint64_t k = L.sk[i];
            L.ukey[i] = (uint32_t)(k >> 32);
            L.uid[i] = 0xFFFFFFFFu - (uint32_t)k;
        }
    } else {
        for (int i = lane; i < wcount; i += 32) {
            L.ukey[off + i] = L.wkey[i];
            L.uid[off + i] = L.wid[i];
        }
    }
    __syncthreads();
    if (warp != 0) return;

    /* ---- warp 0: the row's finish ---- */
    int n = nu;
    bool trunc = rs.trunc != 0 || rs.tsh != 0ull;
    uint32_t t_last = 0u;
    if (MODE == kTopK && (n > a.kprime || trunc)) {
        /* Every excluded element must rank below the K'-th kept one: the
         * shared filter guarantees it once K' elements passed it (every kept
         * one did); a warp's own cut does when the K'-th kept key beats that
         * warp's final threshold. */
        unsigned long long worst = 0ull;
        for (int w = 0; w < NW; ++w) worst = max(worst, rs.taus[w]);
        const unsigned long long T = n < a.kprime ? 0ull
                                     : bsort ? (unsigned long long)L.sk[a.kprime - 1]
                                             : warp_topk_sorted_r<4>(L.ukey, L.uid, n, a.kprime, nullptr, 1);
        if (n < a.kprime || T < worst) {  // a warp's cut excludes only keys strictly below it
            if (lane == 0) list_exact_row(a, row);
            return;
        }
        t_last = (uint32_t)(T >> 32);
        n = a.kprime;
        trunc = true;
    }
    if (MODE == kTopK && a.shard_lists) {
        /* vocab shard: its best shard_len of its K' best by (logit desc, id
         * asc), its largest penalised logit, and whether it holds more
         * elements than listed */
        if (!trunc && !bsort) warp_topk_sorted_r<4>(L.ukey, L.uid, n, a.kprime, nullptr, 1);
        const int m = min(n, a.shard_len);
        const int id_off = row_span(a, row).id_off;
        shard_write(a, row, id_off, m, n > 0 ? key_float(L.ukey[0]) : -INFINITY,
                    (rs.l0nan && id_off == 0 ? kShardNaN0 : 0) | (trunc || n > m ? kShardMore : 0),
                    [&](int i) { return make_uint2(L.uid[i], L.ukey[i]); });
        return;
    }
    float M = Mfull;
    if (MODE == kTopK) {
        uint32_t mk = 0u;
        if (trunc) mk = L.ukey[0];  // the kept entries are sorted: [0] is the row max
        else
            for (int i = lane; i < n; i += 32) mk = max(mk, L.ukey[i]);
        mk = warp_max_u(mk);
        M = (rs.l0nan || n == 0) ? __uint_as_float(0x7FC00000u) : key_float(mk);
    }
    int P = 1;
    while (P < n) P <<= 1;
    int ncand = 0;
    for (int b0 = 0; b0 < P; b0 += 32) {
        const int i = b0 + lane;
        uint64_t kv = 0ull;
        bool cand = false;
        if (i < n) {
            const float d = scaled_diff(key_float(L.ukey[i]), M, a.inv_t);
            if (d > -15.0f) {
                kv = ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - L.uid[i]);
                cand = true;
            }
        }
        if (i < P) L.sk[i] = kv;
        ncand += __popc(__ballot_sync(kFull, cand));
    }
    __syncwarp();
    {
        /* Kept top-k entries arrive sorted by (logit desc, id asc); weights are
         * monotone in the logit, so that is the (weight desc, id asc) order
         * unless two adjacent candidates have equal weights. */
        bool sorted = MODE == kTopK && trunc;
        if (sorted) {
            bool bad = false;
            for (int b0 = 0; b0 + 1 < ncand; b0 += 32) {
                const int i = b0 + lane;
                bad |= (i + 1 < ncand) && ((uint32_t)(L.sk[i] >> 32) == (uint32_t)(L.sk[i + 1] >> 32));
            }
            sorted = !__any_sync(kFull, bad);
        }
        if (!sorted) warp_bitonic_desc(L.sk, P);
    }

    bool more = false, exact = true;
    if (MODE == kTopK && trunc && ncand == n) {
        more = true;  // every kept entry is a candidate: the row has more
        const float dl = scaled_diff(key_float(t_last), M, a.inv_t);
        const float v_last = dl > -15.0f ? ref_weight(dl, a.et) : 0.0f;
        const float v_k = __uint_as_float((uint32_t)(L.sk[a.top_k - 1] >> 32));
        exact = v_last < v_k;
    }
    if (!exact) {
        if (lane == 0) list_exact_row(a, row);
        return;
    }
    const bool fb = ncand == 0;
    int nfin = 0;
    float mass = 0.0f;
    uint64_t st[2] = {0ull, 0ull};
    if (lane == 0) {
        st[0] = a.rng[2 * (size_t)row];
        st[1] = a.rng[2 * (size_t)row + 1];
    }
    auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float((uint32_t)(L.sk[i] >> 32)); };
    /* the running sums go where the gathered keys were (no longer read) */
    const TailOut t = warp_tail(fb ? 1 : ncand, more, a.top_k, a.top_p, st, w, reinterpret_cast<float *>(L.ukey));
    if (lane == 0) {
        a.rng[2 * (size_t)row] = st[0];
        a.rng[2 * (size_t)row + 1] = st[1];
        RowOut o;
        o.id = fb ? 0 : (int)(0xFFFFFFFFu - (uint32_t)L.sk[t.pos]);
        o.prob = __fdiv_rn(w(t.pos), t.mass);
        o.mass = t.mass;
        o.n_topk = t.n_topk;
        o.n_final = t.n_final;
        o.num_cands = more ? -1 : (fb ? 1 : ncand);
        o.flags = fb ? NOEL_ROW_FALLBACK : 0;
        write_row_stats(a, row, o);
        nfin = t.n_final;
        mass = t.mass;
    }
    nfin = __shfl_sync(kFull, nfin, 0);
    mass = __shfl_sync(kFull, mass, 0);
    if (a.list_ids) {
        for (int i = lane; i < a.list_len; i += 32) {
            int id = -1;
            float p = 0.0f;
            if (i < nfin) {
                if (fb) {
                    id = 0;
                    p = 1.0f;
                } else {
                    id = (int)(0xFFFFFFFFu - (uint32_t)L.sk[i]);
                    p = __uint_as_float((uint32_t)(L.sk[i] >> 32));
                    if (!a.list_weights) p = __fdiv_rn(p, mass);
                }
            }
            a.list_ids[(size_t)row * a.list_len + i] = id;
            if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = p;
        }
    }
}

/* Greedy fits 8 CTAs per SM at 64 registers; the queued modes get 72 (7 per
 * SM, still one wave for 1024 rows), which removes most of their spills. */
template <int MODE, int UX>
struct RowOcc {
    static constexpr int kCtas = UX > 1 ? 2 : (MODE == kGreedy ? 8 : 7);
};

/* UX = 1: batches of 16 elements per lane, 7-8 CTAs per SM (a batch that
 * fills the GPU).  UX = 4: batches four times as wide at 2 CTAs per SM, for
 * batches too small to fill the GPU: one row's loads in flight grow fourfold,
 * and a row streams at about four times the rate. */
template <typename T, int MODE, int UX>
__global__ void __launch_bounds__(kRowThreads, (RowOcc<MODE, UX>::kCtas))
    sample_rows_kernel(const __grid_constant__ SampleArgs a) {
    allow_dependent_launch();
    using F = Fmt<T>;
    constexpr int NT = kRowThreads, NW = kRowWarps;
    constexpr int VEC = WarpFmt<T>::VEC, U = WarpFmt<T>::U * UX, NE = U * VEC;
    static_assert(MODE != kGreedy || NE == kLaneElems, "greedy: sixteen elements per lane and batch");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x;
    const RowSpan span = row_span(a, row);
    const int V = span.V;
    const void *rowp = static_cast<const char *>(a.logits) + (size_t)span.off * F::ES;
    const RowGeom g = row_geom<T>(rowp, V);
    const V8 *vbase = reinterpret_cast<const V8 *>(static_cast<const char *>(rowp) + (size_t)g.head * F::ES);

    /* top-k: the warm-up sample is copied into each warp's queue (still
     * empty) while the history table is built */
    const bool warm = MODE == kTopK && min(g.nvec, NW * 32 * U) * VEC >= 4 * a.kprime;
    if (warm) {
        V8 *const q = reinterpret_cast<V8 *>(row_smem) + warp * a.qcap;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int vi = warm_vec<U>(g.nvec, warp, u, lane);
            if (vi >= 0) {
                cp_async16(q + u * 32 + lane, vbase + vi);
                cp_async16(reinterpret_cast<char *>(q + u * 32 + lane) + 16,
                           reinterpret_cast<const char *>(vbase + vi) + 16);
            }
        }
        cp_async_commit();
    }

    {
        const RowLayout L = row_layout<MODE>(a, warp);
        if (tid < NW) {
            rs.wfill[tid] = 0;
            rs.taus[tid] = 0ull;
            rs.lad[0][tid] = rs.lad[1][tid] = rs.lad[2][tid] = 0ull;
        }
        if (MODE == kTopK)
            for (int i = tid; i < kWarpBins; i += NT) L.area[i] = 0u;
        if (tid == 0) {
            rs.tsh = 0ull;
            rs.maxkey = kKeyNegInf;
            rs.flags = 0;
            rs.trunc = 0;
            const float x0 = F::scalar(rowp, 0);
            rs.l0nan = x0 != x0;  // a NaN at id 0 (the penalty keeps it NaN)
            rs.next = NW;
        }
        if (a.penalty)
            hs_build<T, NT>(L.hs, a.hist + (size_t)span.hrow * a.hld, a.hist_start, a.hist_len, V, span.id_off, rowp,
                            a.rep);
        __syncthreads();
    }

    /* greedy: a quarter of the row per warp; queued modes: batches of 32U
     * vectors handed out by ticket, ticket w first for warp w, the rest taken
     * as warps free up.  Ticket t names batch (t mod 4) * bq + t / 4: the first
     * four tickets start at the quarters of the row and later ones walk the
     * quarters in turn, so the early thresholds see the whole row (tickets
     * past the row end name no batch). */
    const int nbat = (g.nvec + 32 * U - 1) / (32 * U), bq = (nbat + 3) / 4;
    auto ticket_batch = [&](int t) -> int {
        const int b = (t & 3) * bq + (t >> 2);
        return (t >> 2) < bq && b < nbat ? b : -1;
    };
    const int first_b = MODE == kGreedy ? warp : ticket_batch(warp);
    const int per = MODE == kGreedy ? (g.nvec + NW - 1) / NW : 32 * U;
    const int v0 = first_b < 0 ? g.nvec : min(g.nvec, first_b * per), v1 = min(g.nvec, v0 + per);

    float gx = -INFINITY;
    uint32_t gid = 0xFFFFFFFFu;

    /* ---- scalar head / tail (warp 0) ---- */
    if (warp == 0) {
        const RowLayout L = row_layout<MODE>(a, warp);
        const bool have = lane < g.nscalar;
        float xs = 0.0f;
        int ids = 0;
        if (have) {
            ids = scalar_id(g, lane);
            xs = F::scalar(rowp, ids);
            if (a.penalty) {
                float v;
                if (hs_find(L.hs, (uint32_t)ids, v)) xs = v;
            }
        }
        if (MODE == kGreedy) {
            if (have && (xs > gx || (xs == gx && (uint32_t)ids < gid))) {
                gx = xs;
                gid = (uint32_t)ids;
            }
        } else {
            const bool ins = have && xs == xs;
            const uint32_t b = __ballot_sync(kFull, ins);
            if (ins) {
                const int pos = __popc(b & lanemask_lt());
                L.wkey[pos] = ord_key(xs);
                L.wid[pos] = (uint32_t)ids;
            }
            if (lane == 0) rs.wfill[0] = __popc(b);
            if (MODE == kFullList) {
                const float m = warp_max_f(ins ? xs : -INFINITY);
                if (lane == 0 && m > -INFINITY) atomicMax(&rs.maxkey, ord_key(m));
            }
            __syncwarp();
        }
    }

    /* greedy: first batch of this warp's slice, prefetched */
    V8 nxt[U];
    if (MODE == kGreedy) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int vi = v0 + u * 32 + lane;
            if (vi < v1) nxt[u] = ld_stream(vbase + vi);
        }
    }

    unsigned long long tau_w = 0ull;
    if (warm) {
        cp_async_wait<0>();  // this lane's sample slots have landed
        __syncwarp();
        tau_w = row_warmup<T, UX>(a, g.head, g.nvec);
    }

    /* ---- the warp's slice of the vector body ---- */
    if (MODE == kGreedy) {
        /* load (one batch prefetched), vector maxima, one comparison */
        for (int base = v0; base < v1; base += 32 * U) {
            V8 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = nxt[u];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = base + 32 * U + u * 32 + lane;
                if (vi < v1) nxt[u] = ld_stream(vbase + vi);
            }
            const uint32_t id0 = (uint32_t)(g.head + (base + lane) * VEC);
            uint32_t cand = 0u;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float x[VEC];
                F::unpack(v[u], x);
                float m = x[0];
#pragma unroll
                for (int j = 1; j < VEC; ++j) m = fmaxf(m, x[j]);
                /* raw maximum: NaN only if the whole vector is NaN; the
                 * penalty only lowers values */
                if (base + u * 32 + lane < v1 && m >= gx) cand |= 1u << u;
            }
            if (cand) {
                LaneBatch bt;
#pragma unroll
                for (int u = 0; u < U; ++u) F::unpack(v[u], bt.v + u * VEC);
                if (a.penalty) {
                    const uint64_t r = greedy_take<VEC, U>(a, id0, cand, gx, gid, bt);
                    gx = __uint_as_float((uint32_t)(r >> 32));
                    gid = (uint32_t)r;
                } else {
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        if (!((cand >> u) & 1u)) continue;
#pragma unroll
                        for (int j = 0; j < VEC; ++j) {
                            const float xv = bt.v[u * VEC + j];
                            const uint32_t id = id0 + (uint32_t)(u * 32 * VEC + j);
                            if (xv > gx || (xv == gx && id < gid)) {
                                gx = xv;
                                gid = id;
                            }
                        }
                    }
                }
            }
        }
    } else {
        /* Top-k / full list: load, vector maxima, one comparison; vectors
         * that pass are queued.  When the queue would overflow, the inner
         * loop stops before that batch, the queue is drained (one queued
         * vector per lane) and streaming resumes at the same batch.  Warps
         * take batches as they free up, so a warp that drained more does
         * not hold up the row end.  28 warps per SM keep enough loads in
         * flight without a register prefetch. */
        V8 *const wq = reinterpret_cast<V8 *>(row_smem) + warp * a.qcap;
        uint32_t *const wqid = reinterpret_cast<uint32_t *>(row_smem + NW * a.qcap * sizeof(V8)) + warp * a.qcap;
        int qfill = 0;  // warp-uniform
        auto take = [&]() -> int {  // the next ticket's batch, nbat when none is left
            for (;;) {
                int t = 0;
                if (lane == 0) t = atomicAdd(&rs.next, 1);
                t = __shfl_sync(kFull, t, 0);
                if (t >= 4 * bq) return nbat;
                const int b = ticket_batch(t);
                if (b >= 0) return b;
            }
        };
        int cur = first_b >= 0 ? first_b : take();  // batch being streamed (warp-uniform)
        int nextb = -1;                             // the batch after it, once taken
        for (;;) {
            while (cur < nbat) {
                const int base = cur * 32 * U, end = min(g.nvec, base + 32 * U);
                V8 v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int vi = base + u * 32 + lane;
                    if (vi < end) v[u] = ld_stream(vbase + vi);
                }
                if (nextb < 0) nextb = take();  // the following batch, while the loads fly
                float bound;  // raw maxima below it cannot pass
                if (MODE == kTopK) {
                    const unsigned long long te = max(tau_w, *(volatile unsigned long long *)&rs.tsh);
                    const uint32_t tk = (uint32_t)(te >> 32);
                    bound = tk == 0u ? -INFINITY : key_float(tk);
                } else {
                    bound = key_float(*(volatile uint32_t *)&rs.maxkey);
                }
                bool c[U];
                uint32_t bal[U];
                int nq = 0;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    float x[VEC];
                    F::unpack(v[u], x);
                    float m = x[0];
#pragma unroll
                    for (int j = 1; j < VEC; ++j) m = fmaxf(m, x[j]);
                    /* raw maximum: NaN only if the whole vector is NaN; the
                     * penalty only lowers values */
                    const bool live = base + u * 32 + lane < end;
                    c[u] = live && (MODE == kTopK ? m >= bound : scaled_diff(m, bound, a.inv_t) > -15.0f);
                    bal[u] = __ballot_sync(kFull, c[u]);
                    nq += __popc(bal[u]);
                }
                if (nq) {
                    if (qfill + nq > a.qcap) break;  // drain, then redo this batch (qcap >= 32U)
                    const uint32_t id0 = (uint32_t)(g.head + (base + lane) * VEC);
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        if (c[u]) {
                            const int p = qfill + __popc(bal[u] & lanemask_lt());
                            st_vec(wq + p, v[u]);
                            wqid[p] = id0 + (uint32_t)(u * 32 * VEC);
                        }
                        qfill += __popc(bal[u]);
                    }
                }
                cur = nextb;
                nextb = -1;
            }
            if (qfill > 0) {
                __syncwarp();
                if (MODE == kTopK) tau_w = topk_drain<T>(a, qfill, tau_w);
                else full_drain<T>(a, qfill);
                qfill = 0;
                __syncwarp();
                if (MODE == kFullList && (__shfl_sync(kFull, *(volatile int *)&rs.flags, 0) & kOverflow)) break;
            }
            if (cur >= nbat) break;
        }
    }
    row_finish<T, MODE>(a, tau_w, gx, gid);
}

}  // namespace noel
