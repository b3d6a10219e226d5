/*
 * The persistent streaming kernel: one CTA per SM walks its rows one after
 * another (rows b, b + G, b + 2G, ... for CTA b of G), so that every phase of
 * a row other than reading it overlaps the reading of other rows.
 *
 * Warp roles (one CTA of 21 warps):
 *   producer   (warp 0)    one lane issues cp.async.bulk copies of the rows'
 *                          16-byte-aligned bodies, 16 KB at a time, into a
 *                          ring of shared-memory stages; each stage has a
 *                          "full" mbarrier (transaction bytes) and an "empty"
 *                          one (released by the consumers).  The stream never
 *                          stops at a row boundary.  A shared counter of the
 *                          copies issued so far tells a waiter which fill of a
 *                          stage its parity refers to.
 *   consumers  (warps 1-16) chunks of the stream go to four groups of four
 *                          consumer warps in turn (chunk q to group q mod 4,
 *                          one 4 KB quarter per warp), so four stages are read
 *                          at once; a lane reads eight 16-byte pieces of its
 *                          quarter (32 fp32 or 64 bf16 elements) and compares
 *                          their raw maxima with the row's current filter.
 *                          Only a piece that can pass is penalised (the
 *                          penalty only lowers values, sampler.c:96-100) and
 *                          tested element by element, by its own lane, one
 *                          such piece per lane per round:
 *                            greedy  per-lane (value desc, id asc) best
 *                                    (sampler.c:105-116);
 *                            top-k   elements above the row's shared filter
 *                                    are appended to the row's candidate
 *                                    buffer (one shared atomic each);
 *                            full    elements within the -15 cut under the
 *                                    running maximum (sampler.c:119-143) are
 *                                    appended.
 *                          Apart from its group's warm-up meeting, a consumer
 *                          warp never waits for the others: it goes from one
 *                          row to the next as soon as the next row's set is
 *                          ready.
 *   finishers  (warps 17-20) finisher f owns row set f (rows j = f, f + 4, ...
 *                          of the CTA): the row state, the history table and
 *                          the candidate buffer.  It prepares a row (history
 *                          bitmap and penalised values, the unaligned head and
 *                          tail elements, NaN at id 0) while the consumers
 *                          still read the rows before it.  While its row
 *                          streams it keeps the top-k filter tight: a two-pass
 *                          radix count over the keys appended so far gives a
 *                          16-bit key prefix with at least K' of them at or
 *                          above it.  When the row has streamed it runs the
 *                          row end: selection of the K' best, weights and the
 *                          sequential mass / nucleus / draw of
 *                          sampler.c:155-191, or the K' best of a vocab shard.
 *                          With four sets, a row end and the next preparation
 *                          of its set overlap the streaming of three rows.
 *
 * Starting filter: each consumer warp first takes its lanes' maxima over
 * pieces of its group's first chunk of the row that hold no history id (their
 * values are final).  Full list: the largest starts the running maximum.
 * Top-k: the group's four warps meet (one mbarrier per group, no wait for the
 * other groups), each raises the filter to the K'-th largest of their 128
 * lane maxima, and the group publishes a ladder of them to the row set; every
 * group then combines all ladders published so far (K' lane maxima across
 * groups above a value), so the last group to arrive sets a filter from all
 * four chunks.  Every lane maximum is an element that passes the filter when
 * its group reads the chunk.
 *
 * Exactness: every element that reaches the buffer stays there, and every
 * filter value f has at least K' elements with composite key >= f that reach
 * the buffer (or, for a raised filter, are in it), so an element left out
 * ranks below K' others.  A buffer that overflows, or a tie of weights at the
 * top-k boundary, sends the row to the two-pass kernel.
 *
 * Every wait is bounded (SampleArgs::wait_ns of %globaltimer): a wait that
 * runs out sets counters[3] and the CTA's error flag, every role leaves its
 * loop, and the producer first waits for its own copies in flight.
 */
#pragma once

#include "sampler_kernels.cuh"
#include "sampler_warp.cuh"

namespace noel {

constexpr int kSCons = 16;                       // consumer warps
constexpr int kSFin = 4;                         // finisher warps = row sets
constexpr int kSWarps = 1 + kSCons + kSFin;
constexpr int kSThreads = 32 * kSWarps;
constexpr int kStageBytes = 16384;               // one stage: one bulk copy
constexpr int kParts = 4;                        // consumer warps sharing a chunk
constexpr int kGroups = kSCons / kParts;         // chunks read at once
constexpr int kPartBytes = kStageBytes / kParts; // one consumer warp's part of a chunk
constexpr int kPieces = kPartBytes / (16 * 32);  // 16-byte pieces per lane and part
constexpr int kMaxStages = 16;
constexpr int kMinStages = 8;                    // two chunks per consumer group
constexpr int kRowBuf = 1024;                    // candidate entries per row set
constexpr int kFullSortMax = 512;                // full-list candidates a finisher sorts itself
static_assert(kPieces == 8, "eight 16-byte pieces per lane");

/* state of one row set, shared by the consumers and the set's finisher */
constexpr int kLadders = 4;                      // ladder slots a group publishes per row

struct StreamRow {
    unsigned long long tsh;             // top-k filter: an element passes iff comp_key > tsh
    unsigned long long lad[kGroups][kLadders];  // group g's ladder: slot i has ladder_count(i) lane maxima above it
    uint32_t pub;                       // groups whose ladder is published
    float gx[kSCons];                   // greedy: each warp's best
    uint32_t gid[kSCons];
    float sgx;                          // greedy: best head / tail element
    uint32_t sgid;
    uint32_t maxkey;                    // full list: running maximum key
    int cnt;                            // entries appended (more than kRowBuf: overflow)
    int l0nan;                          // NaN at the row's first element
};

struct StreamShared {
    unsigned long long full[kMaxStages], empty[kMaxStages];
    unsigned long long ready[kSFin];    // finisher -> consumers: set prepared for its next row
    unsigned long long done[kSFin];     // consumers -> finisher: row streamed
    unsigned long long gmeet[kGroups];  // a group's four warps meet once per row (top-k warm-up)
    unsigned long long glad[2][kGroups][kParts][32];  // their sorted lane maxima, by row parity
    StreamRow st[kSFin];
    uint32_t issued;                    // chunks the producer has issued (release / acquire)
    int err;
};

/* ---------------------------------------------------------------------- */
/* mbarrier, bulk copy and timer                                          */

__device__ __forceinline__ uint32_t sm_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(unsigned long long *b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sm_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mb_try(unsigned long long *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sm_addr(b)), "r"(parity)
        : "memory");
    return ok != 0u;
}
/* try_wait that may suspend the thread until the phase completes or about
 * hint_ns pass (no spinning while the phase is far off) */
__device__ __forceinline__ bool mb_try_sleep(unsigned long long *b, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sm_addr(b)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0u;
}
__device__ __forceinline__ void mb_arrive(unsigned long long *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm_addr(b)) : "memory");
}
__device__ __forceinline__ void mb_expect_tx(unsigned long long *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_addr(b)), "r"(bytes) : "memory");
}
/* global -> shared bulk copy (no multicast), completion counted on mbarrier b */
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, unsigned long long *b,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(sm_addr(dst)),
        "l"(src), "r"(bytes), "r"(sm_addr(b)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire_shared(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(sm_addr(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_shared(uint32_t *p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(sm_addr(p)), "r"(v) : "memory");
}

/* One thread's bounded wait for the phase of the given parity.  False when
 * the limit ran out (flags set) or another role gave up. */
__device__ __noinline__ bool mb_wait_thread(unsigned long long *b, uint32_t parity, const SampleArgs &a,
                                            StreamShared &sh) {
    if (mb_try(b, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        if (mb_try_sleep(b, parity, 100000u)) return true;  // sleeps until the phase completes, 0.1 ms at most
        if (*(volatile int *)&sh.err) return false;
        if (gtimer() - t0 > a.wait_ns) {
            sh.err = 1;
            atomicExch(&a.counters[3], 1);
            return false;
        }
    }
}

/* A warp's bounded wait: lane 0 waits, then every lane observes the phase
 * itself (the acquire that makes the stage's bytes visible to it). */
__device__ __forceinline__ bool mb_wait_warp(unsigned long long *b, uint32_t parity, const SampleArgs &a,
                                             StreamShared &sh) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0 && !mb_try(b, parity)) ok = mb_wait_thread(b, parity, a, sh) ? 1 : 0;
    ok = __shfl_sync(kFull, ok, 0);
    if (!ok) return false;
    /* the phase has completed and cannot advance again before this warp
     * arrives somewhere, so this ends at once; bounded all the same */
    for (int i = 0; i < (1 << 20) && !mb_try(b, parity); ++i) {
    }
    return true;
}

/* A warp's bounded wait for chunk q of the CTA's stream (stage q mod S, fill
 * q / S).  The producer issues chunk q only after the stage's previous fill
 * was released, so once the issue counter has passed q the stage's barrier
 * is in the phase of fill q / S or past it, and the parity names that fill. */
__device__ __forceinline__ bool chunk_wait(uint32_t q, int S, const SampleArgs &a, StreamShared &sh) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0 && ld_acquire_shared(&sh.issued) <= q) {
        const uint64_t t0 = gtimer();
        while (ld_acquire_shared(&sh.issued) <= q) {
            if (*(volatile int *)&sh.err) {
                ok = 0;
                break;
            }
            if (gtimer() - t0 > a.wait_ns) {
                sh.err = 1;
                atomicExch(&a.counters[3], 1);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!__shfl_sync(kFull, ok, 0)) return false;
    return mb_wait_warp(&sh.full[q % (uint32_t)S], (q / (uint32_t)S) & 1u, a, sh);
}

/* ---------------------------------------------------------------------- */
/* geometry and layout                                                    */

/* a row as an unaligned head, a 16-byte-aligned body copied in stages, and
 * an unaligned tail */
struct BulkGeom {
    int head, tail0, nscalar, nchunks;
    long long body;  // bytes
};
template <typename T>
__device__ __forceinline__ BulkGeom bulk_geom(const void *rowp, int V) {
    constexpr int ES = (int)sizeof(T);
    BulkGeom g;
    const uintptr_t p = reinterpret_cast<uintptr_t>(rowp);
    g.head = (int)(((16u - (unsigned)(p & 15u)) & 15u) / ES);
    if (g.head > V) g.head = V;
    g.body = ((long long)(V - g.head) * ES) & ~15ll;
    g.tail0 = g.head + (int)(g.body / ES);
    g.nscalar = g.head + (V - g.tail0);
    g.nchunks = (int)((g.body + kStageBytes - 1) / kStageBytes);
    return g;
}
__device__ __forceinline__ int bulk_scalar_id(const BulkGeom &g, int s) { return s < g.head ? s : g.tail0 + (s - g.head); }

/* Dynamic shared memory: the ring, then per set the history (8-id block
 * bitmap, table keys and values) and the candidate buffer (keys, ids), then
 * per finisher its sort keys, running sums and a radix histogram. */
struct StreamLayout {
    int blk_words, set_bytes, hs_key, hs_val, bkey, bid, fin_bytes, sk, ps, rh, skcap;
    size_t ring, total;
};
__host__ __device__ inline int stream_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}
__host__ __device__ inline StreamLayout stream_layout(int mode, int vocab, int penalty, int hcap, int kprime,
                                                      int nstages) {
    StreamLayout L{};
    L.ring = (size_t)nstages * kStageBytes;
    int off = 0;
    if (penalty) {
        L.blk_words = (((vocab + 255) / 256) + 3) & ~3;
        L.hs_key = L.blk_words * 4;
        L.hs_val = L.hs_key + hcap * 4;
        off = L.hs_val + hcap * 4;
    }
    L.bkey = off;
    L.bid = off + kRowBuf * 4;
    if (mode != kGreedy) off += kRowBuf * 8;
    L.set_bytes = (off + 127) & ~127;
    L.skcap = mode == kTopK ? stream_pow2(kprime) : (mode == kFullList ? kFullSortMax : 0);
    L.sk = 0;
    L.ps = L.skcap * 8;
    L.rh = L.ps + L.skcap * 4;
    L.fin_bytes = mode == kGreedy ? 0 : ((L.rh + 1024 + 127) & ~127);
    L.total = L.ring + (size_t)kSFin * (L.set_bytes + L.fin_bytes);
    return L;
}

/* warm-up ladder slot i counts (i + 1) K' / 4 lane maxima of a group (at
 * most its 128) */
__device__ __forceinline__ int ladder_count(int i, int kprime) { return max(1, kprime / kLadders) * (i + 1); }

/* The largest published ladder value f such that the published groups hold
 * at least K' lane maxima above it (summing, over groups, the largest count
 * among that group's slots whose value is >= f); 0 if none. */
__device__ __forceinline__ unsigned long long ladder_pool(const StreamRow &st, uint32_t pub, int kprime) {
    const int lane = threadIdx.x & 31;
    unsigned long long r = 0ull;
    if (lane < kGroups * kLadders && ((pub >> (lane / kLadders)) & 1u)) {
        const unsigned long long cand = *(volatile const unsigned long long *)&st.lad[lane / kLadders][lane % kLadders];
        int tot = 0;
#pragma unroll
        for (int g = 0; g < kGroups; ++g) {
            if (!((pub >> g) & 1u)) continue;
            int best = 0;
#pragma unroll
            for (int i = 0; i < kLadders; ++i) {
                const unsigned long long f = *(volatile const unsigned long long *)&st.lad[g][i];
                if (f && f >= cand) best = ladder_count(i, kprime);
            }
            tot += best;
        }
        if (cand && tot >= kprime) r = cand;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(kFull, r, o);
        r = t > r ? t : r;
    }
    return r;
}

/* views of a set */
struct SetView {
    HistSet hs;
    uint32_t *bkey, *bid;
};
__device__ __forceinline__ SetView set_view(unsigned char *smem, const StreamLayout &L, const SampleArgs &a, int f) {
    unsigned char *base = smem + L.ring + (size_t)f * L.set_bytes;
    SetView v;
    v.hs = HistSet{nullptr, nullptr, nullptr, 0};
    if (a.penalty) {
        v.hs.blk = reinterpret_cast<uint32_t *>(base);
        v.hs.key = reinterpret_cast<uint32_t *>(base + L.hs_key);
        v.hs.val = reinterpret_cast<uint32_t *>(base + L.hs_val);
        v.hs.cap = a.hcap;
    }
    v.bkey = reinterpret_cast<uint32_t *>(base + L.bkey);
    v.bid = reinterpret_cast<uint32_t *>(base + L.bid);
    return v;
}

/* one 16-byte piece as PE floats (fp32, or bf16 widened exactly) */
template <typename T>
__device__ __forceinline__ void piece_unpack(const uint4 &q, float *x) {
    if (sizeof(T) == 4) {
        x[0] = __uint_as_float(q.x), x[1] = __uint_as_float(q.y), x[2] = __uint_as_float(q.z), x[3] = __uint_as_float(q.w);
    } else {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            x[2 * e] = __uint_as_float(w[e] << 16);
            x[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
        }
    }
}

/* true if any of the N ids from id0 is in the row's window (bitmap only) */
template <int N>
__device__ __forceinline__ bool hs_touches(const HistSet &h, uint32_t id0) {
    const uint32_t b0 = id0 >> 3, b1 = (id0 + N - 1) >> 3;
    uint32_t any = 0u;
    for (uint32_t bb = b0; bb <= b1; ++bb) any |= (h.blk[bb >> 5] >> (bb & 31)) & 1u;
    return any != 0u;
}

/* one element into the row's buffer (dropped, with the count still raised,
 * once the buffer is full: the row then overflows) */
__device__ __forceinline__ void row_append(StreamRow &st, const SetView &v, float x, uint32_t id) {
    const int pos = atomicAdd(&st.cnt, 1);
    if (pos < kRowBuf) {
        v.bid[pos] = id;
        v.bkey[pos] = ord_key(x);
    }
}

/* ---------------------------------------------------------------------- */
/* finisher: preparing a row                                              */

/* the window's distinct ids, each with its penalised logit computed once
 * (sampler.c:87-102), by one warp */
template <typename T>
__device__ void hs_build_warp(const HistSet &h, const int32_t *hrow, int first, int H, int V, int id_off,
                              const void *rowp, float rep) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < hs_blk_words(V); i += 32) h.blk[i] = 0u;
    for (int i = lane; i < h.cap; i += 32) {
        h.key[i] = 0u;
        h.val[i] = 0u;
    }
    __syncwarp();
    const int bits = __ffs(h.cap) - 1;
    for (int b0 = first; b0 < H; b0 += 32 * 8) {  // eight ids per lane loaded at once
        int gts[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = b0 + u * 32 + lane;
            gts[u] = i < H ? hrow[i] : -1;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (b0 + u * 32 >= H) break;  // warp-uniform
            const int i = b0 + u * 32 + lane;
            const int gt = gts[u];
            const bool in = i < H && gt >= id_off && gt - id_off < V;  // sampler.c:95
            if (in) {  // lanes with the same id: one claims the slot, every lane counts
                const uint32_t t = (uint32_t)(gt - id_off);
                atomicOr(&h.blk[t >> 8], 1u << ((t >> 3) & 31));
                uint32_t p = bits ? (hs_hash(t) >> (32 - bits)) : 0u;
                for (int probe = 0; probe < h.cap; ++probe) {
                    const uint32_t prev = atomicCAS(&h.key[p], 0u, t + 1u);
                    if (prev == 0u || prev == t + 1u) {
                        atomicAdd(&h.val[p], 1u);
                        break;
                    }
                    p = (p + 1) & (uint32_t)(h.cap - 1);
                }
            }
            __syncwarp();
        }
    }
    __syncwarp();
    /* each distinct id's penalised logit; a lane's loads go out eight at a
     * time before their division chains */
    for (int s0 = 0; s0 < h.cap; s0 += 32 * 8) {
        float x[8];
        uint32_t kk[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int sl = s0 + u * 32 + lane;
            kk[u] = sl < h.cap ? h.key[sl] : 0u;
            x[u] = kk[u] ? Fmt<T>::scalar(rowp, (int)(kk[u] - 1u)) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int sl = s0 + u * 32 + lane;
            if (kk[u]) h.val[sl] = __float_as_uint(apply_penalty(x[u], h.val[sl], rep));
        }
    }
    __syncwarp();
}

/* the consumers' float bound of a top-k filter: a piece can pass only if its
 * raw maximum reaches it (a prefix at or below -inf's key bounds nothing) */
__device__ __forceinline__ float filter_bound(unsigned long long te) {
    const uint32_t hi = (uint32_t)(te >> 32);
    return hi <= kKeyNegInf ? -INFINITY : key_float(hi);
}

/* Prepare a row of the set: its state, the history table, the unaligned head
 * and tail elements and NaN at id 0. */
template <typename T, int MODE>
__device__ __noinline__ void stream_prepare(const SampleArgs &a, StreamRow &st, const SetView &v, int row) {
    using F = Fmt<T>;
    const int lane = threadIdx.x & 31;
    const RowSpan span = row_span(a, row);
    const void *rowp = static_cast<const char *>(a.logits) + (size_t)span.off * F::ES;
    if (lane < kSCons) {
        st.gx[lane] = -INFINITY;
        st.gid[lane] = 0xFFFFFFFFu;
    }
    /* the row's loads that do not depend on one another go out first: id
     * 0 (NaN test) and the unaligned head and tail (at most 14 elements) */
    const BulkGeom g = bulk_geom<T>(rowp, span.V);
    const bool have = lane < g.nscalar;
    uint32_t ids = have ? (uint32_t)bulk_scalar_id(g, lane) : 0u;
    float xs = have ? F::scalar(rowp, (int)ids) : 0.0f;
    const float x0 = lane == 0 ? F::scalar(rowp, 0) : 0.0f;
    if (lane < kGroups * kLadders) st.lad[lane / kLadders][lane % kLadders] = 0ull;
    if (lane == 0) {
        st.pub = 0u;
        st.tsh = 0ull;
        st.maxkey = kKeyNegInf;
        st.cnt = 0;
        st.l0nan = x0 != x0;  // the penalty keeps a NaN a NaN
    }
    if (a.penalty)
        hs_build_warp<T>(v.hs, a.hist + (size_t)span.hrow * a.hld, a.hist_start, a.hist_len, span.V, span.id_off, rowp,
                         a.rep);
    __syncwarp();
    if (have) {
        float pv;
        if (a.penalty && hs_find(v.hs, ids, pv)) xs = pv;
    }
    if (MODE == kGreedy) {
        float bx = have && xs == xs ? xs : -INFINITY;  // NaN never wins (sampler.c:108-115)
        uint32_t bid = have && xs == xs ? ids : 0xFFFFFFFFu;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ox = __shfl_xor_sync(kFull, bx, o);
            const uint32_t oid = __shfl_xor_sync(kFull, bid, o);
            if (ox > bx || (ox == bx && oid < bid)) {
                bx = ox;
                bid = oid;
            }
        }
        if (lane == 0) {
            st.sgx = bx;
            st.sgid = bid;
        }
        __syncwarp();
        return;
    }

    if (MODE == kTopK)  // unwritten entries read as key 0 while the filter is refreshed
        for (int i = lane; i < kRowBuf / 4; i += 32) reinterpret_cast<uint4 *>(v.bkey)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
    const bool ins = have && xs == xs;
    const uint32_t b = __ballot_sync(kFull, ins);
    if (ins) {
        const int pos = __popc(b & lanemask_lt());
        v.bkey[pos] = ord_key(xs);
        v.bid[pos] = ids;
    }
    if (lane == 0) st.cnt = __popc(b);
    if (MODE == kFullList) {
        const float m = warp_max_f(ins ? xs : -INFINITY);
        if (lane == 0 && m > -INFINITY) st.maxkey = max(st.maxkey, ord_key(m));
    }
    __syncwarp();
}

/* ---------------------------------------------------------------------- */
/* finisher: the filter while the row streams                             */

/* 256-bin histogram of (v >> shift) & 255 over entries v >= floor with
 * (v & mask) == prefix; returns how many entries were counted */
__device__ __noinline__ int warp_hist_floor(uint32_t *hist, const uint32_t *v, int n, uint32_t floor, uint32_t mask,
                                               uint32_t prefix, int shift) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 256; i += 32) hist[i] = 0u;
    __syncwarp();
    int total = 0;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const uint32_t x = i < n ? *(volatile const uint32_t *)&v[i] : 0u;
        const bool ok = i < n && x >= floor && (x & mask) == prefix;
        const uint32_t d = ok ? (x >> shift) & 255u : 256u + lane;  // unique tag when not counted
        const uint32_t peers = __match_any_sync(kFull, d);
        if (ok && (peers & lanemask_lt()) == 0u) hist[d] += (uint32_t)__popc(peers);
        total += __popc(__ballot_sync(kFull, ok));
        __syncwarp();
    }
    return total;
}

/* A filter from the keys appended so far: the largest 16-bit key prefix t
 * with at least K keys >= t << 16 among the first n entries (each is a real
 * element that stays in the buffer), as a composite filter (t << 16) << 32,
 * which every such key passes; 0 if fewer than K keys reach floor. */
__device__ __noinline__ unsigned long long refresh_filter(const uint32_t *bkey, int n, int K, uint32_t floor,
                                                             uint32_t *hist) {
    int d1, before, eq;
    if (warp_hist_floor(hist, bkey, n, max(floor, 1u), 0u, 0u, 24) < K) return 0ull;
    warp_find_digit(hist, K, true, d1, before, eq);
    const int need = K - before;
    __syncwarp();
    warp_hist_floor(hist, bkey, n, max(floor, 1u), 0xFF000000u, (uint32_t)d1 << 24, 16);
    int d2;
    warp_find_digit(hist, need, true, d2, before, eq);
    __syncwarp();
    const uint32_t t = ((uint32_t)d1 << 24) | ((uint32_t)d2 << 16);
    return (unsigned long long)t << 32;
}

/* The set's finisher while its row streams (top-k): a tighter filter from
 * all keys appended so far each time their number has grown by half (at
 * K', 1.5 K', 2.25 K', ...: the early refreshes, when the filter is weakest,
 * are the cheap ones); returns when the consumers are done with the row
 * (false if a wait ran out). */
__device__ __noinline__ bool stream_maintain(const SampleArgs &a, StreamShared &sh, StreamRow &st, const SetView &v,
                                uint32_t *hist, unsigned long long *done, uint32_t parity) {
    const int lane = threadIdx.x & 31;
    const uint64_t t0 = gtimer();
    int last = 0;
    for (uint32_t i = 0;; ++i) {
        int fin = 0;
        if (lane == 0) fin = mb_try(done, parity) ? 1 : 0;
        if (__shfl_sync(kFull, fin, 0)) break;
        const int n = min(__shfl_sync(kFull, *(volatile int *)&st.cnt, 0), kRowBuf);
        if (n >= a.kprime && n >= last + max(32, last / 2)) {
            const unsigned long long cur = *(volatile unsigned long long *)&st.tsh;
            const unsigned long long f = refresh_filter(v.bkey, n, a.kprime, (uint32_t)(cur >> 32), hist);
            if (lane == 0 && f > cur) atomicMax(&st.tsh, f);
            last = n;
        } else {
            __nanosleep(1000);
        }
        if ((i & 15u) == 15u) {
            int bad = 0;
            if (lane == 0) {
                if (*(volatile int *)&sh.err) bad = 1;
                else if (gtimer() - t0 > a.wait_ns) {
                    sh.err = 1;
                    atomicExch(&a.counters[3], 1);
                    bad = 1;
                }
            }
            if (__shfl_sync(kFull, bad, 0)) return false;
        }
    }
    /* every lane observes the phase itself (acquire of the consumers' writes) */
    for (int k = 0; k < (1 << 20) && !mb_try(done, parity); ++k) {
    }
    return true;
}

/* ---------------------------------------------------------------------- */
/* finisher: the row end                                                  */

__device__ __noinline__ void stream_list_out(const SampleArgs &a, int row, int nfin, bool fb, float mass,
                                                const uint64_t *sk) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < a.list_len; i += 32) {
        int id = -1;
        float p = 0.0f;
        if (i < nfin) {
            if (fb) {
                id = 0;
                p = 1.0f;
            } else {
                id = (int)(0xFFFFFFFFu - (uint32_t)sk[i]);
                p = __uint_as_float((uint32_t)(sk[i] >> 32));
                if (!a.list_weights) p = __fdiv_rn(p, mass);
            }
        }
        a.list_ids[(size_t)row * a.list_len + i] = id;
        if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = p;
    }
}

/* the tail over sk[0, ncand) sorted by (weight desc, id asc): sampler.c:
 * 155-191, the row's RNG step, outputs and lists */
__device__ __noinline__ void stream_tail(const SampleArgs &a, int row, const uint64_t *sk, int ncand, bool more,
                                            float *P) {
    const int lane = threadIdx.x & 31;
    const bool fb = ncand == 0;
    uint64_t rs_[2] = {0ull, 0ull};
    if (lane == 0) {
        rs_[0] = a.rng[2 * (size_t)row];
        rs_[1] = a.rng[2 * (size_t)row + 1];
    }
    auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float((uint32_t)(sk[i] >> 32)); };
    const TailOut t = warp_tail(fb ? 1 : ncand, more, a.top_k, a.top_p, rs_, w, P);
    int nfin = 0;
    float mass = 0.0f;
    if (lane == 0) {
        a.rng[2 * (size_t)row] = rs_[0];
        a.rng[2 * (size_t)row + 1] = rs_[1];
        RowOut o;
        o.id = fb ? 0 : (int)(0xFFFFFFFFu - (uint32_t)sk[t.pos]);
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
    if (a.list_ids) stream_list_out(a, row, nfin, fb, mass, sk);
}

/* stable in-place compaction of the buffer's entries that keep(k, id) */
template <typename Keep>
__device__ __forceinline__ int buf_compact(uint32_t *bk, uint32_t *bi, int n, Keep keep) {
    const int lane = threadIdx.x & 31;
    int w = 0;
    for (int b0 = 0; b0 < n; b0 += 32) {
        const int i = b0 + lane;
        const bool ok = i < n;
        const uint32_t k = ok ? bk[i] : 0u, id = ok ? bi[i] : 0u;
        const bool kp = ok && keep(k, id);
        const uint32_t bal = __ballot_sync(kFull, kp);
        __syncwarp();
        if (kp) {
            const int pos = w + __popc(bal & lanemask_lt());
            bk[pos] = k;
            bi[pos] = id;
        }
        w += __popc(bal);
        __syncwarp();
    }
    return w;
}

template <int R>
__device__ __noinline__ uint64_t stream_select(uint32_t *gk, uint32_t *gi, int n, int kprime) {
    return warp_topk_sorted_r<R>(gk, gi, n, kprime, nullptr, 1);
}

template <typename T, int MODE>
__device__ __noinline__ void stream_finish(const SampleArgs &a, const StreamRow &st, const SetView &v, unsigned char *fin,
                              const StreamLayout &L, int row) {
    const int lane = threadIdx.x & 31;
    const RowSpan span = row_span(a, row);
    if (a.wb && a.penalty) {  // penalised values into the caller's row (the row has been read)
        float *wrow = a.wb + (size_t)span.off;
        for (int s = lane; s < v.hs.cap; s += 32) {
            const uint32_t k = v.hs.key[s];
            if (k) wrow[k - 1] = __uint_as_float(v.hs.val[s]);
        }
    }
    if (MODE == kGreedy) {
        float bx = lane < kSCons ? st.gx[lane] : (lane == kSCons ? st.sgx : -INFINITY);
        uint32_t bid = lane < kSCons ? st.gid[lane] : (lane == kSCons ? st.sgid : 0xFFFFFFFFu);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ox = __shfl_xor_sync(kFull, bx, o);
            const uint32_t oid = __shfl_xor_sync(kFull, bid, o);
            if (ox > bx || (ox == bx && oid < bid)) {
                bx = ox;
                bid = oid;
            }
        }
        const int id = (st.l0nan || bid == 0xFFFFFFFFu) ? 0 : (int)bid;  // sampler.c:106-116
        if (lane == 0) {
            RowOut o;
            o.id = id;
            o.prob = 1.0f;
            o.mass = 1.0f;
            o.n_topk = o.n_final = o.num_cands = 1;
            o.flags = NOEL_ROW_GREEDY;
            write_row_stats(a, row, o);
        }
        if (a.list_ids)
            for (int i = lane; i < a.list_len; i += 32) {
                a.list_ids[(size_t)row * a.list_len + i] = i == 0 ? id : -1;
                if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = i == 0 ? 1.0f : 0.0f;
            }
        __syncwarp();
        return;
    }

    uint64_t *sk = reinterpret_cast<uint64_t *>(fin + L.sk);
    float *P = reinterpret_cast<float *>(fin + L.ps);
    uint32_t *gk = v.bkey, *gi = v.bid;
    const int cnt = st.cnt;
    if (cnt > kRowBuf) {  // the buffer overflowed
        if (lane == 0) list_exact_row(a, row);
        __syncwarp();
        return;
    }
    if (MODE == kFullList) {
        /* the candidates: entries within the -15 cut under the row maximum */
        /* NaN at the row's id 0 (for a vocab shard: at global id 0 only) */
        const bool nan0 = st.l0nan && span.id_off == 0;
        const float Mfull = nan0 ? __uint_as_float(0x7FC00000u) : key_float(st.maxkey);
        const int n = buf_compact(gk, gi, cnt, [&](uint32_t k, uint32_t) {
            return scaled_diff(key_float(k), Mfull, a.inv_t) > -15.0f;
        });
        if (n > kFullSortMax) {
            if (lane == 0) list_exact_row(a, row);
            __syncwarp();
            return;
        }
        const int Pn = stream_pow2(max(n, 1));
        if (a.shard_lists) {
            /* vocab shard: its candidates under its own maximum (a superset
             * of its elements within the cut under the row's maximum) by
             * (logit desc, id asc), at most shard_len of them */
            for (int i = lane; i < Pn; i += 32) sk[i] = i < n ? comp_key(gk[i], gi[i]) : 0ull;
            __syncwarp();
            if (n > 1) warp_bitonic_desc(sk, Pn);
            __syncwarp();
            const int m = min(n, a.shard_len);
            const uint32_t mk = *(volatile uint32_t *)&st.maxkey;
            shard_write(a, row, span.id_off, m, nan0 ? __uint_as_float(0x7FC00000u) : key_float(mk),
                        (nan0 ? kShardNaN0 : 0) | (n > m ? kShardMore : 0),
                        [&](int i) { return make_uint2(0xFFFFFFFFu - (uint32_t)sk[i], (uint32_t)(sk[i] >> 32)); });
            __syncwarp();
            return;
        }
        for (int i = lane; i < Pn; i += 32) {
            uint64_t kv = 0ull;
            if (i < n) {
                const float d = scaled_diff(key_float(gk[i]), Mfull, a.inv_t);
                kv = ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - gi[i]);
            }
            sk[i] = kv;
        }
        __syncwarp();
        if (n > 1) warp_bitonic_desc(sk, Pn);
        __syncwarp();
        stream_tail(a, row, sk, n, false, P);
        __syncwarp();
        return;
    }

    /* ---- top-k: the entries at or above the final filter ---- */
    const unsigned long long f = st.tsh;
    int n = f ? buf_compact(gk, gi, cnt, [&](uint32_t k, uint32_t id) { return comp_key(k, id) >= f; }) : cnt;
    bool trunc = f != 0ull;  // elements were left out
    uint64_t tk = 0ull;
    {
        const int R = a.kprime <= 64 ? 4 : 8;
        int m = n;
        if (n > 32 * R) {  // radix-select the K' best first (kept in id order), then sort them
            uint32_t ithr;
            warp_select_top(gk, gi, n, a.kprime, reinterpret_cast<uint32_t *>(fin + L.rh), &ithr);
            __syncwarp();
            m = a.kprime;
        }
        if (m > 0) tk = R == 4 ? stream_select<4>(gk, gi, m, a.kprime) : stream_select<8>(gk, gi, m, a.kprime);
    }
    uint32_t t_last = 0u;
    if (n > a.kprime || trunc) {
        if (n < a.kprime) {  // cannot happen with a valid filter; decided exactly all the same
            if (lane == 0) list_exact_row(a, row);
            __syncwarp();
            return;
        }
        t_last = (uint32_t)(tk >> 32);
        n = a.kprime;
        trunc = true;
    }
    if (a.shard_lists) {
        /* vocab shard: its best shard_len by (logit desc, id asc), its
         * largest penalised logit, and whether it holds more elements than
         * listed */
        const int m = min(n, a.shard_len);
        shard_write(a, row, span.id_off, m, n > 0 ? key_float(gk[0]) : -INFINITY,
                    (st.l0nan && span.id_off == 0 ? kShardNaN0 : 0) | (trunc || n > m ? kShardMore : 0),
                    [&](int i) { return make_uint2(gi[i], gk[i]); });
        __syncwarp();
        return;
    }
    const float M = (st.l0nan || n == 0) ? __uint_as_float(0x7FC00000u) : key_float(gk[0]);
    const int Pn = stream_pow2(max(n, 1));
    int ncand = 0;
    for (int b0 = 0; b0 < Pn; b0 += 32) {
        const int i = b0 + lane;
        uint64_t kv = 0ull;
        bool cand = false;
        if (i < n) {
            const float d = scaled_diff(key_float(gk[i]), M, a.inv_t);
            if (d > -15.0f) {
                kv = ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - gi[i]);
                cand = true;
            }
        }
        if (i < Pn) sk[i] = kv;
        ncand += __popc(__ballot_sync(kFull, cand));
    }
    __syncwarp();
    {
        /* sorted by (logit desc, id asc), which is (weight desc, id asc)
         * unless two adjacent candidates have equal weights */
        bool bad = false;
        for (int b0 = 0; b0 + 1 < ncand; b0 += 32) {
            const int i = b0 + lane;
            bad |= (i + 1 < ncand) && ((uint32_t)(sk[i] >> 32) == (uint32_t)(sk[i + 1] >> 32));
        }
        if (__any_sync(kFull, bad)) warp_bitonic_desc(sk, Pn);
        __syncwarp();
    }
    bool more = false, exact = true;
    if (trunc && ncand == n) {
        more = true;  // every kept entry is a candidate: the row has more
        const float dl = scaled_diff(key_float(t_last), M, a.inv_t);
        const float v_last = dl > -15.0f ? ref_weight(dl, a.et) : 0.0f;
        const float v_k = __uint_as_float((uint32_t)(sk[a.top_k - 1] >> 32));
        exact = v_last < v_k;
    }
    if (!exact) {
        if (lane == 0) list_exact_row(a, row);
        __syncwarp();
        return;
    }
    stream_tail(a, row, sk, ncand, more, P);
    __syncwarp();
}

/* ---------------------------------------------------------------------- */
/* consumers                                                              */

/* One consumer warp's part of a stage: piece p of a lane is the 16 bytes at
 * (p * 32 + lane) * 16 of the part.  Returns the pieces whose raw maximum
 * reaches bound (pass(m)) as a mask; with warm, also this lane's largest
 * element among pieces holding no history id (their values are final). */
template <typename T, bool WARM, typename Pass>
__device__ __forceinline__ uint32_t part_scan(const unsigned char *pbase, int nbw, uint32_t id_lane, const HistSet &hs,
                                              bool penalty, Pass pass, float &lm, uint32_t &lid) {
    constexpr int PE = 16 / (int)sizeof(T);
    const int lane = threadIdx.x & 31;
    uint32_t cm = 0u;
    const bool whole = nbw == kPartBytes;  // every piece inside: no per-piece bounds
#pragma unroll
    for (int p = 0; p < kPieces; ++p) {
        const int o = (p * 32 + lane) * 16;
        if (!whole && o >= nbw) continue;
        float x[PE];
        piece_unpack<T>(*reinterpret_cast<const uint4 *>(pbase + o), x);
        float m = x[0];
#pragma unroll
        for (int e = 1; e < PE; ++e) m = fmaxf(m, x[e]);  // NaN only if all NaN
        if (pass(m)) cm |= 1u << p;
        if (WARM && (m > lm || lid == 0xFFFFFFFFu) && !(penalty && hs_touches<PE>(hs, id_lane + (uint32_t)(p * 32 * PE)))) {
#pragma unroll
            for (int e = 0; e < PE; ++e)
                if (x[e] > lm || (x[e] == lm && lid == 0xFFFFFFFFu)) {  // NaN never taken
                    lm = x[e];
                    lid = id_lane + (uint32_t)(p * 32 * PE + e);
                }
        }
    }
    return cm;
}

template <typename T, int MODE>
__device__ void stream_consume(const SampleArgs &a, StreamShared &sh, unsigned char *smem, const StreamLayout &L,
                               int cw) {
    constexpr int ES = (int)sizeof(T);
    constexpr int PE = 16 / ES;        // elements per 16-byte piece
    using F = Fmt<T>;
    const int lane = threadIdx.x & 31;
    const int G = (int)gridDim.x;
    const int S = a.nstages;
    const int grp = cw / kParts, part = cw % kParts;
    unsigned char *ring = smem;
    uint32_t q = 0u;  // the next chunk of the CTA's stream
    int j = 0;
    for (int row = blockIdx.x; row < a.batch; row += G, ++j) {
        const int f = j % kSFin;
        const uint32_t use = (uint32_t)(j / kSFin) & 1u;
        StreamRow &st = sh.st[f];
        if (!mb_wait_warp(&sh.ready[f], use, a, sh)) return;
        const SetView v = set_view(smem, L, a, f);
        const RowSpan span = row_span(a, row);
        const void *rowp = static_cast<const char *>(a.logits) + (size_t)span.off * F::ES;
        const BulkGeom g = bulk_geom<T>(rowp, span.V);

        float gx = -INFINITY;
        uint32_t gid = 0xFFFFFFFFu;
        /* this group's chunks of the row: chunk c is stream chunk q + c */
        const int c0 = (int)(((uint32_t)grp + kGroups - q % kGroups) % kGroups);
        if (MODE != kGreedy) {
            /* warm-up on the group's first chunk of the row: lane maxima over
             * pieces holding no history id (final values).  Full list: their
             * maximum starts the running maximum.  Top-k: the group's four
             * warps meet and take the K'-th largest of their 128 lane maxima,
             * less one, as a filter; those K' elements pass it when the group
             * reads the chunk next. */
            float lm = -INFINITY;
            uint32_t lid = 0xFFFFFFFFu;
            if (c0 < g.nchunks) {
                const uint32_t qc = q + (uint32_t)c0;
                if (!chunk_wait(qc, S, a, sh)) return;
                const long long rem = g.body - (long long)c0 * kStageBytes - (long long)part * kPartBytes;
                const int nbw = rem <= 0 ? 0 : (int)min((long long)kPartBytes, rem);
                const uint32_t id_lane =
                    (uint32_t)(g.head + ((long long)c0 * kStageBytes + (long long)part * kPartBytes) / ES) +
                    (uint32_t)(lane * PE);
                part_scan<T, true>(ring + (size_t)(qc % (uint32_t)S) * kStageBytes + (size_t)part * kPartBytes, nbw,
                                   id_lane, v.hs, a.penalty != 0, [](float) { return false; }, lm, lid);
            }
            if (MODE == kTopK) {
                uint64_t k1[1] = {lid != 0xFFFFFFFFu ? comp_key(ord_key(lm), lid) : 0ull};
                warp_sort_desc<1>(k1);
                unsigned long long(*gl)[32] = sh.glad[j & 1][grp];
                gl[part][lane] = k1[0];
                __syncwarp();
                if (lane == 0) mb_arrive(&sh.gmeet[grp]);
                if (!mb_wait_warp(&sh.gmeet[grp], (uint32_t)j & 1u, a, sh)) return;
                uint64_t k4[kParts];
#pragma unroll
                for (int w = 0; w < kParts; ++w) k4[w] = gl[w][lane];
                warp_sort_desc<kParts>(k4);
                /* sorted position p sits in lane p / kParts, slot p % kParts;
                 * ladder slot i is the value at position ladder_count(i) - 1,
                 * less one (those lane maxima pass a filter below them) */
                {
                    /* every warp of the group: the group's own filter (K'-th
                     * of its 128 lane maxima) before it reads the chunk */
                    const int pk = min(a.kprime, kParts * 32) - 1;
                    uint64_t kk = 0ull;
#pragma unroll
                    for (int w = 0; w < kParts; ++w)
                        if (w == pk % kParts) kk = k4[w];
                    kk = __shfl_sync(kFull, kk, pk / kParts);
                    if (lane == 0 && kk && a.kprime <= kParts * 32) atomicMax(&st.tsh, kk - 1ull);
                }
                if (part == 0) {
#pragma unroll
                    for (int i = 0; i < kLadders; ++i) {
                        const int pk = min(ladder_count(i, a.kprime), kParts * 32) - 1;
                        uint64_t kk = 0ull;
#pragma unroll
                        for (int w = 0; w < kParts; ++w)
                            if (w == pk % kParts) kk = k4[w];
                        kk = __shfl_sync(kFull, kk, pk / kParts);
                        if (lane == 0)
                            st.lad[grp][i] = (kk && ladder_count(i, a.kprime) <= kParts * 32) ? kk - 1ull : 0ull;
                    }
                    __syncwarp();
                    __threadfence_block();
                    uint32_t pub = 0u;
                    if (lane == 0) pub = atomicOr(&st.pub, 1u << grp) | (1u << grp);
                    pub = __shfl_sync(kFull, pub, 0);
                    __threadfence_block();
                    const unsigned long long pf = ladder_pool(st, pub, a.kprime);
                    if (lane == 0 && pf) atomicMax(&st.tsh, pf);
                }
            } else {
                const float m = warp_max_f(lid != 0xFFFFFFFFu ? lm : -INFINITY);
                if (lane == 0 && m > -INFINITY) atomicMax(&st.maxkey, ord_key(m));
            }
        }
        int c = c0;
        for (; c < g.nchunks; c += kGroups) {
            const uint32_t qc = q + (uint32_t)c;
            if (!chunk_wait(qc, S, a, sh)) return;
            const int stg = (int)(qc % (uint32_t)S);
            const unsigned char *pb = ring + (size_t)stg * kStageBytes + (size_t)part * kPartBytes;
            const long long rem = g.body - (long long)c * kStageBytes - (long long)part * kPartBytes;
            const int nbw = rem <= 0 ? 0 : (int)min((long long)kPartBytes, rem);
            const uint32_t id_lane = (uint32_t)(g.head + ((long long)c * kStageBytes + (long long)part * kPartBytes) / ES) +
                                     (uint32_t)(lane * PE);
            float lm_unused = 0.0f;
            uint32_t lid_unused = 0u;
            uint32_t cm;
            if (MODE == kGreedy) {
                const float bnd = gx;  // the penalty only lowers values
                cm = part_scan<T, false>(pb, nbw, id_lane, v.hs, false, [&](float m) { return m >= bnd; }, lm_unused,
                                         lid_unused);
            } else if (MODE == kTopK) {
                const float bnd = filter_bound(*(volatile unsigned long long *)&st.tsh);
                cm = part_scan<T, false>(pb, nbw, id_lane, v.hs, false, [&](float m) { return m >= bnd; }, lm_unused,
                                         lid_unused);
            } else {
                const float M = key_float(*(volatile uint32_t *)&st.maxkey);
                const float it = a.inv_t;
                cm = part_scan<T, false>(pb, nbw, id_lane, v.hs, false,
                                         [&](float m) { return m == m && scaled_diff(m, M, it) > -15.0f; },
                                         lm_unused, lid_unused);
            }
            /* one candidate piece per lane per round, re-read from the
             * stage, penalised and tested by its lane */
            while (__any_sync(kFull, cm != 0u)) {
                if (cm) {
                    const int p = __ffs(cm) - 1;
                    cm &= cm - 1u;
                    const uint32_t id0 = id_lane + (uint32_t)(p * 32 * PE);
                    float x[PE];
                    piece_unpack<T>(*reinterpret_cast<const uint4 *>(pb + (p * 32 + lane) * 16), x);
                    if (a.penalty) hs_penalize<PE>(v.hs, id0, x);
                    if (MODE == kGreedy) {
#pragma unroll
                        for (int e = 0; e < PE; ++e)
                            if (x[e] > gx || (x[e] == gx && id0 + (uint32_t)e < gid)) {
                                gx = x[e];
                                gid = id0 + (uint32_t)e;
                            }
                    } else if (MODE == kTopK) {
                        const unsigned long long t2 = *(volatile unsigned long long *)&st.tsh;
#pragma unroll
                        for (int e = 0; e < PE; ++e)
                            if (x[e] == x[e] && comp_key(ord_key(x[e]), id0 + (uint32_t)e) > t2)
                                row_append(st, v, x[e], id0 + (uint32_t)e);
                    } else {
                        float m = -INFINITY;
#pragma unroll
                        for (int e = 0; e < PE; ++e) m = fmaxf(m, x[e]);
                        if (m > -INFINITY) atomicMax(&st.maxkey, ord_key(m));
                        const float M = key_float(*(volatile uint32_t *)&st.maxkey);
#pragma unroll
                        for (int e = 0; e < PE; ++e)
                            if (scaled_diff(x[e], M, a.inv_t) > -15.0f) row_append(st, v, x[e], id0 + (uint32_t)e);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mb_arrive(&sh.empty[stg]);
        }
        q += (uint32_t)g.nchunks;
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
                st.gx[cw] = gx;
                st.gid[cw] = gid;
            }
        }
        __syncwarp();
        if (lane == 0) mb_arrive(&sh.done[f]);
    }
}

/* ---------------------------------------------------------------------- */
/* the kernel                                                             */

template <typename T, int MODE>
__global__ void __launch_bounds__(kSThreads, 1) stream_rows_kernel(const __grid_constant__ SampleArgs a) {
    allow_dependent_launch();
    using F = Fmt<T>;
    extern __shared__ __align__(1024) unsigned char stream_smem[];
    __shared__ StreamShared sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = (int)gridDim.x;
    const int S = a.nstages;
    const StreamLayout L = stream_layout(MODE, a.vocab, a.penalty, a.hcap, a.kprime, S);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mb_init(&sh.full[s], 1);
            mb_init(&sh.empty[s], kParts);  // released by the chunk's group of consumer warps
        }
        for (int f = 0; f < kSFin; ++f) {
            mb_init(&sh.ready[f], 1);
            mb_init(&sh.done[f], kSCons);
        }
        for (int g = 0; g < kGroups; ++g) mb_init(&sh.gmeet[g], kParts);
        sh.issued = 0u;
        sh.err = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        /* ---- producer ---- */
        if (lane != 0 || a.test_stall) return;
        const uint64_t pol = l2_evict_first();
        uint32_t q = 0u;  // chunks issued
        bool alive = true;
        for (int row = blockIdx.x; row < a.batch && alive; row += G) {
            const RowSpan span = row_span(a, row);
            const char *rowp = static_cast<const char *>(a.logits) + (size_t)span.off * F::ES;
            const BulkGeom g = bulk_geom<T>(rowp, span.V);
            const char *src = rowp + (size_t)g.head * F::ES;
            long long left = g.body;
            for (int c = 0; c < g.nchunks; ++c, ++q) {
                const int s = (int)(q % (uint32_t)S);
                const uint32_t fill = q / (uint32_t)S;
                /* the consumers released the stage's previous fill (none on the first lap) */
                if (fill > 0u && !mb_try(&sh.empty[s], (fill - 1u) & 1u) &&
                    !mb_wait_thread(&sh.empty[s], (fill - 1u) & 1u, a, sh)) {
                    alive = false;
                    break;
                }
                const uint32_t nb = left < kStageBytes ? (uint32_t)left : (uint32_t)kStageBytes;
                mb_expect_tx(&sh.full[s], nb);
                bulk_load(stream_smem + (size_t)s * kStageBytes, src, nb, &sh.full[s], pol);
                st_release_shared(&sh.issued, q + 1u);
                src += nb;
                left -= nb;
            }
        }
        /* copies still in flight land before the CTA may leave: the last
         * fill of each stage */
        for (uint32_t i = 0; i < (uint32_t)S && i < q; ++i) {
            const uint32_t par = ((q - 1u - i) / (uint32_t)S) & 1u;
            if (!mb_try(&sh.full[i], par)) {
                const uint64_t t0 = gtimer();
                while (!mb_try(&sh.full[i], par))
                    if (gtimer() - t0 > a.wait_ns) {
                        atomicExch(&a.counters[3], 1);
                        break;
                    }
            }
        }
        return;
    }
    if (warp <= kSCons) {
        stream_consume<T, MODE>(a, sh, stream_smem, L, warp - 1);
        return;
    }

    /* ---- finisher f: rows j = f, f + kSFin, ... of this CTA ---- */
    const int f = warp - 1 - kSCons;
    const SetView v = set_view(stream_smem, L, a, f);
    unsigned char *fin = stream_smem + L.ring + (size_t)kSFin * L.set_bytes + (size_t)f * L.fin_bytes;
    uint32_t *hist = reinterpret_cast<uint32_t *>(fin + L.rh);
    StreamRow &st = sh.st[f];
    int j = f;
    int row = blockIdx.x + j * G;
    if (row < a.batch) {
        stream_prepare<T, MODE>(a, st, v, row);
        if (lane == 0) mb_arrive(&sh.ready[f]);
    }
    for (; row < a.batch; j += kSFin, row += kSFin * G) {
        const uint32_t par = (uint32_t)(j / kSFin) & 1u;
        if (MODE == kTopK) {
            if (!stream_maintain(a, sh, st, v, hist, &sh.done[f], par)) return;
        } else if (!mb_wait_warp(&sh.done[f], par, a, sh)) {
            return;
        }
        stream_finish<T, MODE>(a, st, v, fin, L, row);
        const int nrow = row + kSFin * G;
        if (nrow < a.batch) {
            stream_prepare<T, MODE>(a, st, v, nrow);
            if (lane == 0) mb_arrive(&sh.ready[f]);
        }
    }
}

}  // namespace noel
