/*
 * Device code of the B200 token sampler (sm_100a): the argument block, the
 * reference's scalar rules, and the warp / block primitives the kernels share.
 *
 * One pass of the reference sampler (Sain-Kai/noel src/sampler.c:80-192) per
 * logits row, restructured for a GPU that streams rows from HBM:
 *
 *   sample_rows_kernel        (sampler_warp.cuh) one CTA of 4 warps per row;
 *                             greedy, top-k with k <= 120, and full lists.
 *   sample_rows_block_kernel  (sampler_kernels.cuh) top-k with k > 120.
 *   exact_rows_kernel         (sampler_kernels.cuh) rows the others cannot
 *                             finish exactly (a candidate set larger than
 *                             shared memory, or a tie of weights at the top-k
 *                             boundary reaching below the kept set), redone in
 *                             two passes with the candidate list in global
 *                             scratch and a stable radix sort.
 *   shard_merge_kernel        (sampler_shard.cuh) rows split across GPUs.
 *
 * Why selecting by logit is exact: the weight w = expf((x - max) * (1/T)) is
 * non-decreasing in x (fp subtraction and multiplication by a positive are
 * monotone; glibc's expf is monotone on (-15, 0], checked exhaustively), so
 * the k-th largest weight is the weight of the k-th largest logit and every
 * element outside the kept set has a weight <= the weight of the smallest
 * kept logit.  When that weight is strictly below the k-th weight the kept
 * set holds the whole top-k; otherwise the row is sent to the exact kernel.
 */
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ref_expf.h"

namespace noel {

constexpr uint32_t kFull = 0xFFFFFFFFu;

enum Mode { kGreedy = 0, kTopK = 1, kFullList = 2 };

/* Flags kept per row in shared memory. */
enum { kTruncated = 1, kOverflow = 2, kNeedExact = 4, kWarmBet = 8 };

struct ExpTable {
    const uint32_t *keys, *vals, *offs;
    long long near;  // exceptions lie within this many double ulps of a midpoint
};

/* Kernel arguments (by value). */
struct SampleArgs {
    const void *logits;
    int64_t ld;
    int vocab, batch;
    const int32_t *hist;
    int64_t hld;
    int hist_len, hist_start;   // window [hist_start, hist_len)
    int penalty;                // repetition penalty active (sampler.c:88)
    float rep;
    float inv_t;                // 1.0f / temperature (sampler.c:132)
    float top_p;
    int top_k;
    int kprime;                 // kept-set size for top-k
    int warm_rank;              // rank of the single-pass warm-up's starting filter (0: K')
    int kw;                     // entries a warp keeps when it compacts (single-pass kernel)
    int cap;                    // candidate buffer entries
    int hcap;                   // history hash-table slots (single-pass kernel)
    int ucap;                   // gathered-candidate entries (single-pass kernel)
    uint64_t *rng;
    int32_t *ids;
    float *probs;
    int32_t *list_ids;
    float *list_probs;
    int list_len;
    int list_weights;           // list_probs receives unnormalised weights
    int32_t *stats;
    float *wb;                  // penalised values written here (fp32 rows) or NULL
    int32_t *exact_list;        // rows for exact_rows_kernel
    int32_t *counters;          // [0] rows listed, [1] next row, [2] CTAs done
    uint2 *slots;               // exact kernel scratch: nslots x 2 x vocab
    int nslots;
    ExpTable et;
    /* vocab shard (the row holds columns [id_off, id_off + vocab) of the full
     * vocabulary): history ids are global; instead of sampling, the kernels
     * write per row the shard's best shard_len (global id, penalised logit)
     * by (logit desc, id asc) -- for a full-list config only elements within
     * the -15 cut under the shard's maximum -- and then a trailer (largest
     * penalised logit, flags) */
    int id_off;
    uint2 *shard_lists;         // [B][shard_len + 1], id -1 past the listed ones; NULL: no shard output
    int shard_len;
    /* split rows (with shard output): kernel row r is columns
     * [s * vocab, s * vocab + vocab) of caller row r / split, s = r % split,
     * of a row of split_vocab columns; 0 or 1: rows are the caller's rows */
    int split, split_vocab;
    /* greedy rows split over `split` CTAs (no shard output): per caller row,
     * the best composite key (value desc, id asc) so far, the CTAs done and
     * NaN at id 0; zero between calls (the row's last CTA re-arms it) */
    uint4 *gsplit;
    int qcap;                   // queued vectors per warp (single-pass kernel, queued modes)
    /* persistent streaming kernel */
    int nstages;                // shared-memory ring stages of 16 KB
    int test_stall;             // 1: issue no row loads, so every wait runs out (failure-detection test)
    unsigned long long wait_ns; // limit of every device-side wait (%globaltimer ns)
};

/* where kernel row r lives: element offset, columns, global id of its first
 * column, history row */
struct RowSpan {
    int64_t off;
    int V, id_off, hrow;
};
__device__ __forceinline__ RowSpan row_span(const SampleArgs &a, int r) {
    RowSpan s;
    if (a.split > 1) {
        const int b = r / a.split, q = r - b * a.split;
        s.off = (int64_t)b * a.ld + (int64_t)q * a.vocab;
        s.V = min(a.vocab, a.split_vocab - q * a.vocab);
        s.id_off = a.id_off + q * a.vocab;
        s.hrow = b;
    } else {
        s.off = (int64_t)r * a.ld;
        s.V = a.vocab;
        s.id_off = a.id_off;
        s.hrow = r;
    }
    return s;
}

/* shard flags */
enum { kShardNaN0 = 1, kShardMore = 2 };


/* ---------------------------------------------------------------------- */
/* scalar helpers                                                          */

/* order-preserving key of a non-NaN float; -0 and +0 share a key */
__device__ __forceinline__ uint32_t ord_key(float x) {
    const uint32_t u = __float_as_uint(__fadd_rn(x, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
constexpr uint32_t kKeyNegInf = 0x007FFFFFu;   // ord_key(-inf)

/* One row's shard list: m listed entries from get(i) -> (local id, key),
 * padding, then the trailer.  By the calling warp. */
template <typename Get>
__device__ __forceinline__ void shard_write(const SampleArgs &a, int row, int id_off, int m, float mx, int flags,
                                            Get get) {
    const int lane = threadIdx.x & 31;
    uint2 *out = a.shard_lists + (size_t)row * (size_t)(a.shard_len + 1);
    for (int i = lane; i < a.shard_len; i += 32) {
        uint2 e = make_uint2(0xFFFFFFFFu, 0u);
        if (i < m) {
            const uint2 ik = get(i);
            e = make_uint2(ik.x + (uint32_t)id_off, __float_as_uint(key_float(ik.y)));
        }
        out[i] = e;
    }
    if (lane == 0) out[a.shard_len] = make_uint2(__float_as_uint(mx), (uint32_t)flags);
}

/* sampler.c:96-100 applied c times (one per occurrence in the window) */
__device__ __forceinline__ float apply_penalty(float x, uint32_t c, float rep) {
    /* the sign never changes (a positive value stays positive, zero stays
     * zero), so the branch of sampler.c:97-100 is taken once */
    if (x > 0.0f)
        for (uint32_t i = 0; i < c; ++i) x = __fdiv_rn(x, rep);
    else
        for (uint32_t i = 0; i < c; ++i) x = __fmul_rn(x, rep);
    return x;
}

/* sampler.c:8-21: xorshift128+ step, top 24 bits scaled by 2^-24 */
__device__ __forceinline__ float rng_uniform(uint64_t *s) {
    uint64_t a = s[0];
    const uint64_t b = s[1];
    s[0] = b;
    a ^= a << 23;
    s[1] = a ^ b ^ (a >> 18) ^ (b >> 5);
    const uint64_t v = s[1] + b;
    return __fmul_rn((float)(uint32_t)(v >> 40), 1.0f / 16777216.0f);
}

/* sampler.c:137: diff = (x - max) * inv_t, without contraction */
__device__ __forceinline__ float scaled_diff(float x, float m, float inv_t) {
    return __fmul_rn(__fsub_rn(x, m), inv_t);
}

__device__ __forceinline__ float ref_weight(float d, const ExpTable &et) {
    return noel_ref_expf(d, et.keys, et.vals, et.offs, et.near);
}

/* ---------------------------------------------------------------------- */
/* warp / block primitives                                                 */

__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

/* exclusive scan of one int per thread; s_w has NT/32+1 ints */
template <int NT>
__device__ __forceinline__ int block_excl_scan(int v, int *s_w, int &total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int inc = warp_incl_scan(v);
    if (lane == 31) s_w[w] = inc;
    __syncthreads();
    if (w == 0) {
        const int x = lane < NW ? s_w[lane] : 0;
        const int ix = warp_incl_scan(x);
        if (lane < NW) s_w[lane] = ix - x;
        if (lane == NW - 1) s_w[NW] = ix;
    }
    __syncthreads();
    total = s_w[NW];
    const int r = s_w[w] + inc - v;
    __syncthreads();
    return r;
}

template <int NT>
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t *s_w) {
    constexpr int NW = NT / 32;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
    if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = s_w[0];
    for (int i = 1; i < NW; ++i) r = max(r, s_w[i]);
    __syncthreads();
    return r;
}

template <int NT>
__device__ __forceinline__ int block_sum_int(int v, int *s_w) {
    int total;
    block_excl_scan<NT>(v, s_w, total);
    return total;
}

/* descending bitonic sort of P (power of two) 64-bit keys in shared memory */
template <int NT>
__device__ void bitonic_sort_desc(uint64_t *a, int P) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += NT) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t ai = a[i], aj = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (ai < aj) : (ai > aj)) {
                        a[i] = aj;
                        a[ixj] = ai;
                    }
                }
            }
            __syncthreads();
        }
    }
}

/* Descending bitonic sort of P (a power of two) keys in shared memory by a
 * whole block, each thread taking pairs (i, i + j) rather than indices, so no
 * thread idles in a step; ends with a barrier. */
template <int NT>
__device__ __forceinline__ void block_bitonic_pairs_desc(uint64_t *a, int P) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int p = threadIdx.x; p < (P >> 1); p += NT) {
                const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));  // lower index of pair p at distance j
                const uint64_t ai = a[i], aj = a[i + j];
                if ((i & k) == 0 ? (ai < aj) : (ai > aj)) {
                    a[i] = aj;
                    a[i + j] = ai;
                }
            }
            __syncthreads();
        }
    }
}

/* ---------------------------------------------------------------------- */
/* history: bitmap of ids in the window, rank -> occurrence count           */

struct HistView {
    uint32_t *bm;    // ceil(V/32) words
    uint32_t *gpre;  // set bits before each 8-word group; [G] = total
    uint32_t *cnt;   // per distinct id, indexed by rank: occurrences, or (with
                     // idr) the penalised logit as float bits once built
    int words;
    uint32_t *idr;   // optional scratch: id of each rank while building
};

__device__ __forceinline__ int hist_rank(const HistView &h, int t) {
    const int w = t >> 5, g = t >> 8;
    int r = (int)h.gpre[g];
    for (int ww = g << 3; ww < w; ++ww) r += __popc(h.bm[ww]);
    return r + __popc(h.bm[w] & ((1u << (t & 31)) - 1u));
}

/* sampler.c:88-93: the window of the row's history, ids in [0, V) only.
 * Lanes of a warp whose ids share a bitmap word set it with one atomic, and
 * lanes holding the same id count it once (a skewed window repeats a few low
 * ids in most lanes).  With h.idr, every distinct id's count then becomes its
 * penalised logit (sampler.c:96-100, once per occurrence), computed once per
 * row with the ranks spread over the threads. */
constexpr int kHistBatch = 8;  // history rounds (and penalised logits) whose loads are issued together

template <int NT, typename T = float>
__device__ void build_history(const HistView &h, const int32_t *hrow, int first, int H, int V,
                              int *s_w, int id_off = 0, const void *rowp = nullptr, float rep = 1.0f) {
    constexpr int R = kHistBatch;
    const int W = h.words, G = (W + 7) >> 3;
    for (int i = threadIdx.x; i < W; i += NT) h.bm[i] = 0u;
    __syncthreads();
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
            const int g = gv[r];
            const bool in = i < H && g >= id_off && g - id_off < V;  // sampler.c:95 (ids of this shard)
            const int t = g - id_off;
            if (in) atomicOr(&h.bm[t >> 5], 1u << (t & 31));
        }
    }
    __syncthreads();
    const int per = (G + NT - 1) / NT;
    const int g0 = threadIdx.x * per, g1 = min(G, g0 + per);
    int mine = 0;
    for (int g = g0; g < g1; ++g) {
        int s = 0;
        for (int w = g * 8; w < min(W, g * 8 + 8); ++w) s += __popc(h.bm[w]);
        h.gpre[g] = (uint32_t)s;
        mine += s;
    }
    int total;
    int base = block_excl_scan<NT>(mine, s_w, total);
    for (int g = g0; g < g1; ++g) {
        const int s = (int)h.gpre[g];
        h.gpre[g] = (uint32_t)base;
        base += s;
    }
    if (threadIdx.x == 0) h.gpre[G] = (uint32_t)total;
    for (int i = threadIdx.x; i < total; i += NT) h.cnt[i] = 0u;
    __syncthreads();
    for (int b0 = first; b0 < H; b0 += NT * R) {
        int gv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = b0 + r * NT + (int)threadIdx.x;
            gv[r] = i < H ? hrow[i] : -1;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = b0 + r * NT + (int)threadIdx.x;
            const int g = gv[r];
            const bool in = i < H && g >= id_off && g - id_off < V;
            if (in) {
                const int rk = hist_rank(h, g - id_off);
                const uint32_t before = atomicAdd(&h.cnt[rk], 1u);
                if (h.idr && before == 0u) h.idr[rk] = (uint32_t)(g - id_off);  // the first count names the rank
            }
        }
    }
    __syncthreads();
    if (h.idr) {
        const int total = (int)h.gpre[G];
        for (int r0 = threadIdx.x; r0 < total; r0 += NT * R) {  // R logits loaded together
            float xs[R];
#pragma unroll
            for (int k = 0; k < R; ++k) {
                const int r = r0 + k * NT;
                xs[k] = 0.0f;
                if (r < total) {
                    const int id = (int)h.idr[r];
                    xs[k] = sizeof(T) == 4 ? static_cast<const float *>(rowp)[id]  // fp32, or bf16 widened
                                           : __uint_as_float((uint32_t)static_cast<const uint16_t *>(rowp)[id] << 16);
                }
            }
#pragma unroll
            for (int k = 0; k < R; ++k) {
                const int r = r0 + k * NT;
                if (r < total) h.cnt[r] = __float_as_uint(apply_penalty(xs[k], h.cnt[r], rep));
            }
        }
        __syncthreads();
    }
}

/* penalty bits of ids [id0, id0+n) (n <= 16) */
__device__ __forceinline__ uint32_t hist_bits(const HistView &h, int id0, int n) {
    const int w = id0 >> 5, sh = id0 & 31;
    uint32_t b = h.bm[w] >> sh;
    if (sh + n > 32 && w + 1 < h.words) b |= h.bm[w + 1] << (32 - sh);
    return b & ((1u << n) - 1u);
}

/* the penalty for the group of N consecutive ids starting at id0 */
template <int N>
__device__ __forceinline__ void penalize_group(const HistView &hv, int id0, float *x, float rep) {
    uint32_t bits = hist_bits(hv, id0, N);
    while (bits) {
        const int j = __ffs(bits) - 1;
        bits &= bits - 1;
        const uint32_t c = hv.cnt[hist_rank(hv, id0 + j)];
#pragma unroll
        for (int jj = 0; jj < N; ++jj)
            if (jj == j) x[jj] = apply_penalty(x[jj], c, rep);
    }
}

/* ---------------------------------------------------------------------- */
/* element formats                                                          */

/* 32-byte vector: Blackwell loads 256 bits per thread in one instruction */
struct alignas(32) V8 {
    uint32_t v[8];
};

template <typename T>
struct Fmt;
template <>
struct Fmt<float> {
    static constexpr int VEC = 8, ES = 4, U = 4;
    __device__ static __forceinline__ void unpack(const V8 &v, float *x) {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __uint_as_float(v.v[i]);
    }
    __device__ static __forceinline__ float scalar(const void *row, int i) {
        return static_cast<const float *>(row)[i];
    }
};
template <>
struct Fmt<uint16_t> {  // bf16 bit patterns; upcast is exact
    static constexpr int VEC = 16, ES = 2, U = 2;
    __device__ static __forceinline__ void unpack(const V8 &v, float *x) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x[2 * i] = __uint_as_float(v.v[i] << 16);
            x[2 * i + 1] = __uint_as_float(v.v[i] & 0xFFFF0000u);
        }
    }
    __device__ static __forceinline__ float scalar(const void *row, int i) {
        return __uint_as_float((uint32_t)static_cast<const uint16_t *>(row)[i] << 16);
    }
};

/* streaming 256-bit load that keeps the row out of L1 and evicts it first from L2 */
__device__ __forceinline__ V8 ld_stream(const V8 *p) {
    V8 r;
    asm volatile(
        "ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
          "=r"(r.v[6]), "=r"(r.v[7])
        : "l"(p));
    return r;
}

/* Called at the start of every kernel the two-pass kernel follows (a
 * programmatic dependent launch): once every CTA of this grid has called it,
 * the dependent grid may be scheduled, and its launch overlaps this grid's
 * last CTAs.  The dependent still waits (griddepcontrol.wait) until this
 * grid has finished and its writes are visible. */
__device__ __forceinline__ void allow_dependent_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

/* Bulk prefetch of [p, p + bytes) into L2 by the copy engine (no registers,
 * nothing to wait for); p 16-byte aligned, bytes a multiple of 16. */
__device__ __forceinline__ void l2_prefetch(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

/* 16-byte global -> shared copies that bypass the registers (and L1) */
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

/* Row geometry: scalar head until 32-byte alignment, vector body, scalar tail. */
struct RowGeom {
    int head, nvec, tail0, nscalar;
};
template <typename T>
__device__ __forceinline__ RowGeom row_geom(const void *row, int V) {
    using F = Fmt<T>;
    RowGeom g;
    const uintptr_t a = reinterpret_cast<uintptr_t>(row);
    g.head = (int)(((32u - (a & 31u)) & 31u) / F::ES);
    if (g.head > V) g.head = V;
    g.nvec = (V - g.head) / F::VEC;
    g.tail0 = g.head + g.nvec * F::VEC;
    g.nscalar = g.head + (V - g.tail0);
    return g;
}
__device__ __forceinline__ int scalar_id(const RowGeom &g, int s) {
    return s < g.head ? s : g.tail0 + (s - g.head);
}

/* ---------------------------------------------------------------------- */
/* candidate buffer and its compaction                                      */

struct Buf {
    uint32_t *key;  // ord_key of the (penalised) logit
    uint32_t *id;
};

struct SelShared {
    uint32_t hist[256];
    int digit, above, eq;
};

/*
 * Keep the K largest entries by (key desc, id asc); entries land in [0, K).
 * Returns the K-th key; *id_thr is the largest kept id among entries with
 * that key when ties had to be cut, else 0xFFFFFFFF.
 */
template <int NT, int EPT>
__device__ uint32_t select_top(Buf b, int n, int K, SelShared &ss, int *s_w, uint32_t *id_thr) {
    uint32_t prefix = 0, mask = 0;
    int need = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) ss.hist[i] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += NT) {
            const uint32_t k = b.key[i];
            if ((k & mask) == prefix) atomicAdd(&ss.hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            int c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // lane covers digits 255-8*lane .. 248-8*lane
                c[j] = (int)ss.hist[255 - 8 * lane - j];
                s += c[j];
            }
            const int inc = warp_incl_scan(s);
            const int before = inc - s;
            if (before < need && need <= inc) {
                int cum = before;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (cum < need && need <= cum + c[j]) {
                        ss.digit = 255 - 8 * lane - j;
                        ss.above = cum;
                        ss.eq = c[j];
                    }
                    cum += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= (uint32_t)ss.digit << shift;
        mask |= 0xFFu << shift;
        need -= ss.above;
        __syncthreads();
    }
    const uint32_t t = prefix;
    const int eq = ss.eq;
    uint32_t ithr = 0xFFFFFFFFu;
    if (eq > need) {  // cut ties at t by ascending id
        uint32_t ip = 0, im = 0;
        int need2 = need;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += NT) ss.hist[i] = 0u;
            __syncthreads();
            for (int i = threadIdx.x; i < n; i += NT) {
                const uint32_t id = b.id[i];
                if (b.key[i] == t && (id & im) == ip) atomicAdd(&ss.hist[(id >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                int c[8], s = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    c[j] = (int)ss.hist[8 * lane + j];
                    s += c[j];
                }
                const int inc = warp_incl_scan(s);
                const int before = inc - s;
                if (before < need2 && need2 <= inc) {
                    int cum = before;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (cum < need2 && need2 <= cum + c[j]) {
                            ss.digit = 8 * lane + j;
                            ss.above = cum;
                        }
                        cum += c[j];
                    }
                }
            }
            __syncthreads();
            ip |= (uint32_t)ss.digit << shift;
            im |= 0xFFu << shift;
            need2 -= ss.above;
            __syncthreads();
        }
        ithr = ip;
    }
    /* stable in-place compaction of the kept entries */
    uint32_t kk[EPT], ki[EPT];
    const int per = (n + NT - 1) / NT;
    const int i0 = threadIdx.x * per;
    int mine = 0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
        const int i = i0 + e;
        kk[e] = 0u;
        ki[e] = 0u;
        if (e < per && i < n) {
            kk[e] = b.key[i];
            ki[e] = b.id[i];
            if (kk[e] > t || (kk[e] == t && ki[e] <= ithr)) ++mine;
        }
    }
    int total;
    int pos = block_excl_scan<NT>(mine, s_w, total);  // its barriers order reads before writes
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
        const int i = i0 + e;
        if (e < per && i < n && (kk[e] > t || (kk[e] == t && ki[e] <= ithr))) {
            b.key[pos] = kk[e];
            b.id[pos] = ki[e];
            ++pos;
        }
    }
    __syncthreads();
    *id_thr = ithr;
    return t;
}

/* Full-list mode: drop entries that fail the -15 cut under max m. */
template <int NT, int EPT>
__device__ int filter_by_max(Buf b, int n, float m, float inv_t, int *s_w) {
    uint32_t kk[EPT], ki[EPT];
    const int per = (n + NT - 1) / NT;
    const int i0 = threadIdx.x * per;
    int mine = 0;
    bool keep[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
        const int i = i0 + e;
        keep[e] = false;
        kk[e] = 0u;
        ki[e] = 0u;
        if (e < per && i < n) {
            kk[e] = b.key[i];
            ki[e] = b.id[i];
            keep[e] = scaled_diff(key_float(kk[e]), m, inv_t) > -15.0f;
            mine += keep[e];
        }
    }
    int total;
    int pos = block_excl_scan<NT>(mine, s_w, total);
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
        if (keep[e]) {
            b.key[pos] = kk[e];
            b.id[pos] = ki[e];
            ++pos;
        }
    }
    __syncthreads();
    return total;
}

/* ---------------------------------------------------------------------- */
/* the sequential tail of sampler.c:155-191 over a sorted weight list       */

struct TailOut {
    int n_topk, n_final, pos;
    float mass;
};

/* w(i) returns the i-th weight of the list sorted by (weight desc, id asc) */
template <typename WeightAt>
__device__ __forceinline__ TailOut run_tail(int num_cands, bool more_than_listed, int top_k,
                                            float top_p, uint64_t *rng, WeightAt w) {
    TailOut o;
    int n = num_cands;
    if (top_k > 0 && (more_than_listed || top_k < n)) n = top_k;  // sampler.c:155-157
    o.n_topk = n;
    float mass = 0.0f;                                             // sampler.c:160-163
    for (int i = 0; i < n; ++i) mass = __fadd_rn(mass, w(i));
    if (top_p > 0.0f && top_p < 1.0f) {                            // sampler.c:165-179
        const float cutoff = __fmul_rn(top_p, mass);
        float cum = 0.0f;
        int keep = 0;
        for (int i = 0; i < n; ++i) {
            cum = __fadd_rn(cum, w(i));
            ++keep;
            if (cum >= cutoff) break;
        }
        n = keep;
        mass = cum;
    }
    o.n_final = n;
    o.mass = mass;
    const float r = __fmul_rn(rng_uniform(rng), mass);            // sampler.c:182-191
    float acc = 0.0f;
    o.pos = n - 1;
    for (int i = 0; i < n; ++i) {
        acc = __fadd_rn(acc, w(i));
        if (r <= acc) {
            o.pos = i;
            break;
        }
    }
    return o;
}

/* First i < n with P[i] >= t (P non-decreasing), else n - 1; the whole warp. */
__device__ __forceinline__ int warp_first_at_least(const float *P, int n, float t) {
    const int lane = threadIdx.x & 31;
    for (int b = 0; b < n; b += 32) {
        const int i = b + lane;
        const unsigned hit = __ballot_sync(0xFFFFFFFFu, i < n && P[i] >= t);
        if (hit) return b + __ffs(hit) - 1;
    }
    return n - 1;
}

/* First i in [0, n) with P[i] >= t for a non-decreasing P in global memory
 * (whole warp): 32-way narrowing, then one ballot; n - 1 if there is none. */
__device__ __forceinline__ int warp_search_at_least(const float *P, int n, float t) {
    const int lane = threadIdx.x & 31;
    int lo = 0, hi = n;  // the answer, if any, is in [lo, hi)
    while (hi - lo > 32) {
        const int step = (hi - lo + 31) / 32;
        const int idx = lo + lane * step;
        const unsigned hit = __ballot_sync(0xFFFFFFFFu, idx < hi && P[idx] >= t);
        if (hit & 1u) return lo;  // P[lo] >= t
        if (hit) {
            const int L = __ffs(hit) - 1;  // P[lo + L step] >= t > P[lo + (L - 1) step]
            hi = lo + L * step + 1;
            lo = lo + (L - 1) * step + 1;
        } else {
            lo += ((hi - 1 - lo) / step) * step + 1;  // past the last sampled index
        }
    }
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, lo + lane < hi && P[lo + lane] >= t);
    return hit ? lo + __ffs(hit) - 1 : n - 1;
}

/* warp_tail for long lists held in global memory (the two-pass kernel):
 * the warp stages 256 weights at a time in shared memory (stage), lane 0
 * adds them in order, the running sums go to P (global, n floats), and the
 * cut and the draw are 32-way searches over P. */
template <typename WeightAt>
__device__ __forceinline__ TailOut warp_tail_global(int num_cands, bool more_than_listed, int top_k, float top_p,
                                                    uint64_t *rng, WeightAt w, float *P, float *stage) {
    const int lane = threadIdx.x & 31;
    TailOut o;
    int n = num_cands;
    if (top_k > 0 && (more_than_listed || top_k < n)) n = top_k;  // sampler.c:155-157
    o.n_topk = n;
    float m = 0.0f;  // sampler.c:160-163, keeping every partial sum (lane 0's)
    for (int b = 0; b < n; b += 256) {
        const int c = min(256, n - b);
        for (int j = lane; j < c; j += 32) stage[j] = w(b + j);
        __syncwarp();
        if (lane == 0) {
            int j = 0;
            for (; j + 8 <= c; j += 8) {
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = stage[j + q];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    m = __fadd_rn(m, v[q]);
                    stage[j + q] = m;
                }
            }
            for (; j < c; ++j) {
                m = __fadd_rn(m, stage[j]);
                stage[j] = m;
            }
        }
        __syncwarp();
        for (int j = lane; j < c; j += 32) P[b + j] = stage[j];
        __syncwarp();
    }
    __threadfence_block();
    __syncwarp();
    float mass = __shfl_sync(0xFFFFFFFFu, m, 0);
    if (top_p > 0.0f && top_p < 1.0f && n > 0) {  // sampler.c:165-179
        const int keep = warp_search_at_least(P, n, __fmul_rn(top_p, mass)) + 1;
        n = keep;
        mass = P[keep - 1];
    }
    o.n_final = n;
    o.mass = mass;
    float r = 0.0f;  // sampler.c:182-191
    if (lane == 0) r = __fmul_rn(rng_uniform(rng), mass);
    r = __shfl_sync(0xFFFFFFFFu, r, 0);
    o.pos = n > 0 ? warp_search_at_least(P, n, r) : -1;
    __syncwarp();
    return o;
}

/* run_tail for a whole warp.  The mass, nucleus and draw loops of
 * sampler.c:160-191 all walk the same running sum of the sorted weights, so
 * lane 0 computes that sum once, in order and with the same roundings, into
 * P[0, n) (shared memory), and the cut (first running sum >= top_p * mass)
 * and the draw (first running sum >= r) become warp searches: adding
 * non-negative weights never lowers a rounded sum, so P is non-decreasing.
 * rng is read and advanced by lane 0 only; every lane gets the result. */
template <typename WeightAt>
__device__ __forceinline__ TailOut warp_tail(int num_cands, bool more_than_listed, int top_k, float top_p,
                                             uint64_t *rng, WeightAt w, float *P) {
    const int lane = threadIdx.x & 31;
    TailOut o;
    int n = num_cands;
    if (top_k > 0 && (more_than_listed || top_k < n)) n = top_k;  // sampler.c:155-157
    o.n_topk = n;
    if (lane == 0) {  // sampler.c:160-163, keeping every partial sum
        float m = 0.0f;
        int i = 0;
        for (; i + 8 <= n; i += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = w(i + j);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                m = __fadd_rn(m, v[j]);
                P[i + j] = m;
            }
        }
        for (; i < n; ++i) {
            m = __fadd_rn(m, w(i));
            P[i] = m;
        }
    }
    __syncwarp();
    float mass = n > 0 ? P[n - 1] : 0.0f;
    if (top_p > 0.0f && top_p < 1.0f && n > 0) {  // sampler.c:165-179
        const int keep = warp_first_at_least(P, n, __fmul_rn(top_p, mass)) + 1;
        n = keep;
        mass = P[keep - 1];
    }
    o.n_final = n;
    o.mass = mass;
    float r = 0.0f;  // sampler.c:182-191
    if (lane == 0) r = __fmul_rn(rng_uniform(rng), mass);
    r = __shfl_sync(0xFFFFFFFFu, r, 0);
    o.pos = n > 0 ? warp_first_at_least(P, n, r) : -1;
    __syncwarp();
    return o;
}

}  // namespace noel

namespace noel {

/* ---------------------------------------------------------------------- */
/* warp-level candidate buffer primitives (no block barriers)              */

__device__ __forceinline__ uint32_t lanemask_lt() {
    return (1u << (threadIdx.x & 31)) - 1u;
}

/* digit d (searching from the top when desc) whose cumulative count crosses need */
__device__ __forceinline__ void warp_find_digit(const uint32_t *hist, int need, bool desc, int &digit,
                                                int &before_cnt, int &eq) {
    const int lane = threadIdx.x & 31;
    int c[8], s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        c[j] = (int)hist[desc ? 255 - 8 * lane - j : 8 * lane + j];
        s += c[j];
    }
    const int inc = warp_incl_scan(s);
    const int before = inc - s;
    const uint32_t sel = __ballot_sync(kFull, before < need && need <= inc);
    const int src = sel ? __ffs(sel) - 1 : 31;
    int d = 0, ab = 0, e = 0;
    if (lane == src) {
        int cum = before;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (cum < need && need <= cum + c[j] && e == 0) {
                d = desc ? 255 - 8 * lane - j : 8 * lane + j;
                ab = cum;
                e = c[j];
            }
            cum += c[j];
        }
    }
    digit = __shfl_sync(kFull, d, src);
    before_cnt = __shfl_sync(kFull, ab, src);
    eq = __shfl_sync(kFull, e, src);
}

/*
 * 256-bin histogram of digit (v >> shift) & 255 over the entries whose value
 * matches prefix under mask (and, if sel_key is given, whose sel_key equals
 * sel).  Equal digits within a warp-wide batch are counted once by their
 * leader (match_any), so heavily repeated digits do not serialise atomics.
 */
__device__ __forceinline__ void warp_digit_hist(uint32_t *hist, const uint32_t *v, const uint32_t *sel_key,
                                                uint32_t sel, int n, uint32_t mask, uint32_t prefix, int shift) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < 256; i += 32) hist[i] = 0u;
    __syncwarp();
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        bool ok = i < n;
        uint32_t x = 0u;
        if (ok) {
            x = v[i];
            ok = (x & mask) == prefix && (sel_key == nullptr || sel_key[i] == sel);
        }
        const uint32_t d = ok ? (x >> shift) & 255u : 256u + lane;  // unique tag when not counted
        const uint32_t peers = __match_any_sync(kFull, d);
        if (ok && (peers & lanemask_lt()) == 0u) hist[d] += (uint32_t)__popc(peers);
        __syncwarp();
    }
}

/*
 * Keep the K largest of n (K <= n) entries by (key desc, id asc), compacted
 * in place (stable) into [0, K).  Returns the K-th key; *ithr = largest kept id
 * among entries with that key when ties were cut, else 0xFFFFFFFF.
 * hist: 256 words of this warp's shared memory.
 */
__device__ uint32_t warp_select_top(uint32_t *key, uint32_t *id, int n, int K, uint32_t *hist, uint32_t *ithr) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, mask = 0;
    int need = K, eq = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        warp_digit_hist(hist, key, nullptr, 0u, n, mask, prefix, shift);
        int d, before;
        warp_find_digit(hist, need, true, d, before, eq);
        prefix |= (uint32_t)d << shift;
        mask |= 0xFFu << shift;
        need -= before;
        __syncwarp();
    }
    const uint32_t t = prefix;
    uint32_t it = 0xFFFFFFFFu;
    if (eq > need) {
        uint32_t ip = 0, im = 0;
        int need2 = need, eq2;
        for (int shift = 24; shift >= 0; shift -= 8) {
            warp_digit_hist(hist, id, key, t, n, im, ip, shift);
            int d, before;
            warp_find_digit(hist, need2, false, d, before, eq2);
            ip |= (uint32_t)d << shift;
            im |= 0xFFu << shift;
            need2 -= before;
            __syncwarp();
        }
        it = ip;
    }
    int w = 0;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const bool ok = i < n;
        const uint32_t k = ok ? key[i] : 0u, v = ok ? id[i] : 0u;
        const bool keep = ok && (k > t || (k == t && v <= it));
        const uint32_t b = __ballot_sync(kFull, keep);
        __syncwarp();
        if (keep) {
            const int pos = w + __popc(b & lanemask_lt());
            key[pos] = k;
            id[pos] = v;
        }
        w += __popc(b);
        __syncwarp();
    }
    *ithr = it;
    return t;
}

/* keep entries passing the -15 cut under max m (sampler.c:137-138); returns the count */
__device__ int warp_filter_by_max(uint32_t *key, uint32_t *id, int n, float m, float inv_t) {
    const int lane = threadIdx.x & 31;
    int w = 0;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const bool ok = i < n;
        const uint32_t k = ok ? key[i] : 0u, v = ok ? id[i] : 0u;
        const bool keep = ok && scaled_diff(key_float(k), m, inv_t) > -15.0f;
        const uint32_t b = __ballot_sync(kFull, keep);
        __syncwarp();
        if (keep) {
            const int pos = w + __popc(b & lanemask_lt());
            key[pos] = k;
            id[pos] = v;
        }
        w += __popc(b);
        __syncwarp();
    }
    return w;
}

/* descending bitonic sort of P (power of two) 64-bit keys by one warp */
__device__ void warp_bitonic_desc(uint64_t *a, int P) {
    const int lane = threadIdx.x & 31;
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < P; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t ai = a[i], aj = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (ai < aj) : (ai > aj)) {
                        a[i] = aj;
                        a[ixj] = ai;
                    }
                }
            }
            __syncwarp();
        }
    }
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ uint32_t warp_max_u(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
    return v;
}
__device__ __forceinline__ float warp_min_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

}  // namespace noel

namespace noel {

/* ---------------------------------------------------------------------- */
/* register-resident warp sort of 32*R 64-bit keys                         */

/* Descending bitonic sort; element i = lane*R + r is k[r] of lane i/R. */
template <int R>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&k)[R]) {
    const int lane = threadIdx.x & 31;
    constexpr int N = 32 * R;
#pragma unroll
    for (int kk = 2; kk <= N; kk <<= 1) {
#pragma unroll
        for (int j = kk >> 1; j > 0; j >>= 1) {
            if (j >= R) {
                const int lj = j / R;
                const bool lower = (lane & lj) == 0;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int i = lane * R + r;
                    const uint64_t o = __shfl_xor_sync(kFull, k[r], lj);
                    const bool desc = (i & kk) == 0;
                    k[r] = (desc == lower) ? (k[r] > o ? k[r] : o) : (k[r] < o ? k[r] : o);
                }
            } else {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int rp = r ^ j;
                    if (rp > r) {
                        const int i = lane * R + r;
                        const bool desc = (i & kk) == 0;
                        const uint64_t a = k[r], b = k[rp];
                        const bool sw = desc ? (a < b) : (a > b);
                        k[r] = sw ? b : a;
                        k[rp] = sw ? a : b;
                    }
                }
            }
        }
    }
}

/* (key desc, id asc) as one 64-bit key: larger is better */
__device__ __forceinline__ uint64_t comp_key(uint32_t key, uint32_t id) {
    return ((uint64_t)key << 32) | (uint64_t)(0xFFFFFFFFu - id);
}

/*
 * Top-K of n entries (key[], id[]) by (key desc, id asc) with a running
 * register sort of 32*R at a time (the best K so far plus the next 32*R-K
 * entries; K < 32*R).  Entries are read and written at r*32 + lane
 * (conflict-free); the sort runs on the lane-major order (input order is
 * irrelevant to a selection).  The kept entries are written back sorted to
 * [0, min(n, K)), and ladder[0..2] receive the composite keys
 * at sorted positions lad0-1, K/2-1 and K-1.  Returns the K-th composite
 * key (0 if n < K); the kept count is min(n, K).  Out of line: it runs
 * rarely and its unrolled network would otherwise crowd the streaming loop.
 */
template <int R>
__device__ __forceinline__ uint64_t warp_topk_sorted_r(uint32_t *key, uint32_t *id, int n, int K, uint64_t *ladder,
                                                   int lad0) {
    constexpr int N = 32 * R;
    const int lane = threadIdx.x & 31;
    uint64_t k[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        k[r] = i < n ? comp_key(key[i], id[i]) : 0ull;
    }
    warp_sort_desc<R>(k);
    /* each round replaces the N - K entries below the kept ones; callers pass
     * K <= N - 32 (the step never drops below 32, so a larger K ends the
     * loop too) */
    const int step = N - K > 32 ? N - K : 32;
    for (int next = N; next < n; next += step) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int p = lane * R + r;  // sorted position held here
            if (p >= K) {
                const int src = next + (p - K);
                k[r] = src < n ? comp_key(key[src], id[src]) : 0ull;
            }
        }
        warp_sort_desc<R>(k);
    }
    __syncwarp();
    uint64_t l0 = 0ull, l1 = 0ull, l2 = 0ull;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int p = lane * R + r;
        if (p < K && p < n) {  // kept entries, contiguous and sorted
            key[p] = (uint32_t)(k[r] >> 32);
            id[p] = 0xFFFFFFFFu - (uint32_t)k[r];
        }
        if (p == lad0 - 1) l0 = k[r];
        if (p == K / 2 - 1) l1 = k[r];
        if (p == K - 1) l2 = k[r];
    }
    l0 = __shfl_sync(kFull, l0, (lad0 - 1) / R);
    l1 = __shfl_sync(kFull, l1, (K / 2 - 1) / R);
    l2 = __shfl_sync(kFull, l2, (K - 1) / R);
    if (ladder) {
        ladder[0] = l0;
        ladder[1] = l1;
        ladder[2] = l2;
    }
    __syncwarp();
    return n >= K ? l2 : 0ull;
}


}  // namespace noel
