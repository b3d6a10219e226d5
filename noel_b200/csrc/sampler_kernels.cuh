/*
 * Kernels of the B200 token sampler.  See sampler_device.cuh for the design.
 */
#pragma once

#include "noel_sampler_cuda.h"
#include "sampler_device.cuh"

namespace noel {

constexpr int kMainThreads = 256;
constexpr int kEPT = 16;         // buffer entries per thread in compactions (cap <= 4096)
constexpr int kWarmBins = 2048;  // warm-up histogram on the top 11 key bits
constexpr int kExactThreads = 256;
#ifndef NOEL_BLOCK_PREFETCH
#define NOEL_BLOCK_PREFETCH 1
#endif
/* Chunks (NT * U vectors, 32 KB) of the block kernel's row kept prefetched
 * into L2 ahead of the one being read: each chunk ends in a block barrier,
 * so without them every chunk pays a full memory latency. */
constexpr int kBlockPrefetch = NOEL_BLOCK_PREFETCH;

struct RowOut {
    int id, n_topk, n_final, num_cands, flags;
    float prob, mass;
};

__device__ __forceinline__ void write_row_stats(const SampleArgs &a, int row, const RowOut &o) {
    a.ids[row] = o.id;
    if (a.probs) a.probs[row] = o.prob;
    if (a.stats) {
        int4 s = make_int4(o.num_cands, o.n_topk, o.n_final, o.flags);
        reinterpret_cast<int4 *>(a.stats)[row] = s;
    }
}

/* Penalised write-back of the row's history ids (sampler.c:96-100 mutates the
 * caller's logits).  Runs after the row has been read, from the original
 * values, once per distinct id. */
template <int NT>
__device__ void write_back_penalty(const SampleArgs &a, const HistView &hv, int row) {
    float *wrow = a.wb + (size_t)row * a.ld;
    for (int w = threadIdx.x; w < hv.words; w += NT) {
        uint32_t bits = hv.bm[w];
        while (bits) {
            const int j = __ffs(bits) - 1;
            bits &= bits - 1;
            const int id = w * 32 + j;
            wrow[id] = __uint_as_float(hv.cnt[hist_rank(hv, id)]);  // penalised value
        }
    }
}

__device__ __forceinline__ void list_exact_row(const SampleArgs &a, int row) {
    const int q = atomicAdd(&a.counters[0], 1);
    a.exact_list[q] = row;
}

/* Every row of the launch for exact_rows_kernel (the rows of a full-list
 * vocab shard whose history and list do not fit the streaming kernel). */
__global__ void list_all_rows_kernel(const SampleArgs a) {
    allow_dependent_launch();
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < a.batch; r += gridDim.x * blockDim.x) a.exact_list[r] = r;
    if (blockIdx.x == 0 && threadIdx.x == 0) a.counters[0] = a.batch;
}

/* ====================================================================== */
/* block-level kernel for large kept sets (k > 120): one CTA per row       */

/* Bin of an NB-bin histogram holding the K-th largest entry, counted from the
 * top bin down (warp 0, every lane): -1 if the total is below K; *need = how
 * many of that bin's entries are needed. */
template <int NB>
__device__ int warp_find_bin_desc(const uint32_t *h, int K, int *need) {
    const int lane = threadIdx.x & 31;
    constexpr int PER = NB / 32;
    int sum = 0;
    for (int j = 0; j < PER; ++j) sum += (int)h[NB - 1 - lane * PER - j];
    const int inc = warp_incl_scan(sum);
    int bin = -1, nd = 0;
    if (inc - sum < K && K <= inc) {
        int cum = inc - sum;
        for (int j = 0; j < PER; ++j) {
            const int b = NB - 1 - lane * PER - j;
            const int c = (int)h[b];
            if (cum + c >= K) {
                bin = b;
                nd = K - cum;
                break;
            }
            cum += c;
        }
    }
    const uint32_t m = __ballot_sync(kFull, bin >= 0);
    if (!m) return -1;
    const int src = __ffs(m) - 1;
    *need = __shfl_sync(kFull, nd, src);
    return __shfl_sync(kFull, bin, src);
}

/* Vector of the row's body read by sample slot j of the block kernel's
 * warm-up: NS slots spread evenly over the body, or the whole body when it is
 * shorter; -1 for a slot past it. */
template <int NS>
__device__ __forceinline__ int block_sample_vec(int j, int nvec) {
    if (nvec >= NS) return (int)(((long long)j * nvec) / NS);
    return j < nvec ? j : -1;
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kMainThreads, 2) sample_rows_block_kernel(const SampleArgs a) {
    allow_dependent_launch();
    using F = Fmt<T>;
    constexpr int NT = kMainThreads;
    constexpr int VEC = F::VEC, U = F::U, NE = U * VEC;
    static_assert(NE <= 32, "pending mask is 32 bits");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ SelShared ss;
    __shared__ int s_w[NT / 32 + 1];
    __shared__ uint32_t s_wu[NT / 32];
    __shared__ int s_n, s_flags, s_l0nan, s_fin_n;
    __shared__ uint32_t s_tau_key, s_tau_id, s_maxkey;
    __shared__ float s_fin_mass;
    __shared__ uint32_t s_gbest_key[NT / 32], s_gbest_id[NT / 32];
    __shared__ int s_wb1, s_wneed;

    const int tid = threadIdx.x, lane = tid & 31;
    const int row = blockIdx.x;
    const int V = a.vocab;
    const void *rowp = static_cast<const char *>(a.logits) + (size_t)row * (size_t)a.ld * F::ES;
    const RowGeom g = row_geom<T>(rowp, V);
    const V8 *vbase = reinterpret_cast<const V8 *>(static_cast<const char *>(rowp) + (size_t)g.head * F::ES);
    auto prefetch_chunk = [&](int it) {
        const int v0 = it * NT * U;
        if (v0 < g.nvec) l2_prefetch(vbase + v0, (uint32_t)(min(g.nvec - v0, NT * U) * (int)sizeof(V8)));
    };
    if (tid < kBlockPrefetch) prefetch_chunk(tid);  // land while the history is built

    /* shared-memory carve-up */
    unsigned char *sp = smem;
    HistView hv{nullptr, nullptr, nullptr, 0};
    if (a.penalty) {
        hv.words = (V + 31) >> 5;
        const int G = (hv.words + 7) >> 3;
        hv.bm = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)hv.words * 4;
        hv.gpre = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)(G + 1) * 4;
        hv.cnt = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)max(1, a.hist_len - a.hist_start) * 4;
        hv.idr = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)max(1, a.hist_len - a.hist_start) * 4;
        sp = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(sp) + 15) & ~uintptr_t(15));
    }
    Buf buf{nullptr, nullptr};
    uint32_t *whist = nullptr;
    if (MODE != kGreedy) {
        buf.key = reinterpret_cast<uint32_t *>(sp);
        buf.id = buf.key + a.cap;
        sp += (size_t)a.cap * 8;
    }
    if (MODE == kTopK) whist = reinterpret_cast<uint32_t *>(sp);

    if (tid == 0) {
        s_n = 0;
        s_flags = 0;
        s_l0nan = 0;
        s_tau_key = kKeyNegInf;
        s_tau_id = 0xFFFFFFFFu;
        s_maxkey = kKeyNegInf;
    }
    if (a.penalty)  // hv.cnt then holds penalised values
        build_history<NT, T>(hv, a.hist + (size_t)row * a.hld, a.hist_start, a.hist_len, V, s_w, a.id_off, rowp,
                             a.rep);
    __syncthreads();

    /* running state */
    float gx = -INFINITY;
    uint32_t gid = 0xFFFFFFFFu;
    float tmax = -INFINITY;

    /* ---- scalar head / tail elements ---- */
    if (tid < g.nscalar) {
        const int id = scalar_id(g, tid);
        float x = F::scalar(rowp, id);
        if (a.penalty && ((hv.bm[id >> 5] >> (id & 31)) & 1u))
            x = __uint_as_float(hv.cnt[hist_rank(hv, id)]);
        if (id == 0 && x != x) s_l0nan = 1;
        if (MODE == kGreedy) {
            if (x > gx || (x == gx && (uint32_t)id < gid)) {
                gx = x;
                gid = (uint32_t)id;
            }
        } else if (x == x) {
            tmax = fmaxf(tmax, x);
            const int slot = atomicAdd(&s_n, 1);
            buf.key[slot] = ord_key(x);
            buf.id[slot] = (uint32_t)id;
        }
    }
    if (MODE == kFullList && tmax > -INFINITY) atomicMax(&s_maxkey, ord_key(tmax));
    __syncthreads();

    /* ---- vector body ---- */
    const int per_iter = NT * U;
    const int iters = (g.nvec + per_iter - 1) / per_iter;
    const bool warm = (MODE == kTopK) && min(g.nvec, per_iter) * VEC >= 2 * a.kprime;

    /* Warm-up (top-k): a sample of NT * U vectors spread evenly over the row,
     * penalised; a two-level histogram (11 key bits, then the next 11 inside
     * the chosen bin) of it gives the floor of the bin holding its r-th
     * largest (r = warm_rank) as the starting filter.  With r < K' the filter
     * is a bet: the row end sends the row to the two-pass kernel when fewer
     * than K' elements passed it. */
    if (warm) {
        const int r = a.warm_rank > 0 ? a.warm_rank : a.kprime;
        float xs[NE];
        {
            V8 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = block_sample_vec<NT * U>(u * NT + tid, g.nvec);
                if (vi >= 0) v[u] = ld_stream(vbase + vi);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = block_sample_vec<NT * U>(u * NT + tid, g.nvec);
                if (vi >= 0) {
                    F::unpack(v[u], xs + u * VEC);
                    if (a.penalty) {
                        const int id0 = g.head + vi * VEC;
                        uint32_t bits = hist_bits(hv, id0, VEC);
                        while (bits) {
                            const int j = __ffs(bits) - 1;
                            bits &= bits - 1;
                            const float pv = __uint_as_float(hv.cnt[hist_rank(hv, id0 + j)]);
#pragma unroll
                            for (int jj = 0; jj < VEC; ++jj)
                                if (jj == j) xs[u * VEC + jj] = pv;
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < VEC; ++j) xs[u * VEC + j] = __uint_as_float(0x7FC00000u);  // not counted
                }
            }
        }
        for (int i = tid; i < kWarmBins; i += NT) whist[i] = 0u;
        __syncthreads();
#pragma unroll
        for (int e = 0; e < NE; ++e)
            if (xs[e] == xs[e]) atomicAdd(&whist[ord_key(xs[e]) >> 21], 1u);
        __syncthreads();
        if (tid < 32) {
            int need = 0;
            const int b1 = warp_find_bin_desc<kWarmBins>(whist, r, &need);
            if (lane == 0) {
                s_wb1 = b1;
                s_wneed = need;
            }
        }
        __syncthreads();
        const int b1 = s_wb1;
        if (b1 >= 0) {
            for (int i = tid; i < kWarmBins; i += NT) whist[i] = 0u;
            __syncthreads();
#pragma unroll
            for (int e = 0; e < NE; ++e)
                if (xs[e] == xs[e] && (int)(ord_key(xs[e]) >> 21) == b1)
                    atomicAdd(&whist[(ord_key(xs[e]) >> 10) & (kWarmBins - 1)], 1u);
            __syncthreads();
            if (tid < 32) {
                int need2 = 0;
                const int b2 = warp_find_bin_desc<kWarmBins>(whist, s_wneed, &need2);
                if (lane == 0 && b2 >= 0) {
                    s_tau_key = ((uint32_t)b1 << 21) | ((uint32_t)b2 << 10);  // r sample elements reach it
                    s_tau_id = 0xFFFFFFFFu;
                    s_flags |= kTruncated | (r < a.kprime ? kWarmBet : 0);
                }
            }
            __syncthreads();
        }
    }

    for (int it = 0; it < iters; ++it) {
        if (kBlockPrefetch > 0 && tid == 0) prefetch_chunk(it + kBlockPrefetch);
        float x[NE];
        uint32_t valid = 0u;
        {
            V8 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = it * per_iter + u * NT + tid;
                if (vi < g.nvec) v[u] = ld_stream(vbase + vi);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = it * per_iter + u * NT + tid;
                if (vi < g.nvec) {
                    F::unpack(v[u], x + u * VEC);
                    valid |= ((1u << VEC) - 1u) << (u * VEC);
                } else {
#pragma unroll
                    for (int j = 0; j < VEC; ++j) x[u * VEC + j] = 0.0f;
                }
            }
        }
        if (a.penalty) {
            /* Top-k after the warm-up: the penalty only lowers values, so an
             * element whose raw value is below the current threshold fails
             * the filter either way and needs no history lookup. */
            const float ptau = MODE == kTopK ? key_float(s_tau_key) : -INFINITY;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = it * per_iter + u * NT + tid;
                if (vi < g.nvec) {
                    const int id0 = g.head + vi * VEC;
                    uint32_t bits = hist_bits(hv, id0, VEC);
                    if (MODE == kTopK && bits) {
                        uint32_t need = 0u;
#pragma unroll
                        for (int j = 0; j < VEC; ++j)
                            if (x[u * VEC + j] >= ptau) need |= 1u << j;
                        bits &= need;
                    }
                    while (bits) {
                        const int j = __ffs(bits) - 1;
                        bits &= bits - 1;
                        const float pv = __uint_as_float(hv.cnt[hist_rank(hv, id0 + j)]);  // penalised value
#pragma unroll
                        for (int jj = 0; jj < VEC; ++jj)
                            if (jj == j) x[u * VEC + jj] = pv;
                    }
                }
            }
        }
        if (it == 0 && tid == 0 && g.head == 0 && g.nvec > 0 && x[0] != x[0]) s_l0nan = 1;

        if (MODE == kGreedy) {
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                if ((valid >> e) & 1u) {
                    const int u = e / VEC, j = e % VEC;
                    const uint32_t id = (uint32_t)(g.head + (it * per_iter + u * NT + tid) * VEC + j);
                    if (x[e] > gx || (x[e] == gx && id < gid)) {
                        gx = x[e];
                        gid = id;
                    }
                }
            }
            continue;
        }

        /* ---- candidate filter ---- */
        float m_cur = 0.0f;
        if (MODE == kFullList) {
            float lm = -INFINITY;
#pragma unroll
            for (int e = 0; e < NE; ++e)
                if ((valid >> e) & 1u) lm = fmaxf(lm, x[e]);
            tmax = fmaxf(tmax, lm);
            if (lm > -INFINITY) atomicMax(&s_maxkey, ord_key(lm));
            m_cur = key_float(*(volatile uint32_t *)&s_maxkey);
        }

        uint32_t pend = 0u;
        {
            const float tau_f = key_float(s_tau_key);
            const uint32_t tau_id = s_tau_id;
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                if ((valid >> e) & 1u) {
                    bool pass;
                    if (MODE == kTopK) {
                        const int u = e / VEC, j = e % VEC;
                        const uint32_t id = (uint32_t)(g.head + (it * per_iter + u * NT + tid) * VEC + j);
                        pass = x[e] >= tau_f && (x[e] > tau_f || id < tau_id);
                    } else {
                        pass = scaled_diff(x[e], m_cur, a.inv_t) > -15.0f;
                    }
                    if (pass) pend |= 1u << e;
                }
            }
        }

        bool stop = false;
        for (;;) {
            const int c = __popc(pend);
            if (__any_sync(kFull, c != 0)) {
                const int inc = warp_incl_scan(c);
                const int tot = __shfl_sync(kFull, inc, 31);
                int wbase = 0;
                if (lane == 31 && tot) wbase = atomicAdd(&s_n, tot);
                wbase = __shfl_sync(kFull, wbase, 31);
                int slot = wbase + inc - c;
                uint32_t pp = pend;
                while (pp) {
                    const int e = __ffs(pp) - 1;
                    pp &= pp - 1;
                    if (slot < a.cap) {
                        const int u = e / VEC, j = e % VEC;
                        float xv = 0.0f;
#pragma unroll
                        for (int ee = 0; ee < NE; ++ee)
                            if (ee == e) xv = x[ee];
                        buf.key[slot] = ord_key(xv);
                        buf.id[slot] = (uint32_t)(g.head + (it * per_iter + u * NT + tid) * VEC + j);
                        pend &= ~(1u << e);
                    }
                    ++slot;
                }
            }
            if (!__syncthreads_or(pend != 0u)) break;
            /* the buffer is full: compact it and raise the threshold */
            if (tid == 0) s_n = min(s_n, a.cap);
            __syncthreads();
            if (MODE == kTopK) {
                uint32_t ithr;
                const uint32_t t = select_top<NT, kEPT>(buf, s_n, a.kprime, ss, s_w, &ithr);
                if (tid == 0) {
                    s_n = a.kprime;
                    s_tau_key = t;
                    s_tau_id = ithr;
                    s_flags |= kTruncated;
                }
                __syncthreads();
                const float tau_f = key_float(t);
                uint32_t pp = pend;
                while (pp) {
                    const int e = __ffs(pp) - 1;
                    pp &= pp - 1;
                    const int u = e / VEC, j = e % VEC;
                    const uint32_t id = (uint32_t)(g.head + (it * per_iter + u * NT + tid) * VEC + j);
                    float xv = 0.0f;
#pragma unroll
                    for (int ee = 0; ee < NE; ++ee)
                        if (ee == e) xv = x[ee];
                    if (!(xv > tau_f || (xv == tau_f && id < ithr))) pend &= ~(1u << e);
                }
            } else {
                const float m = key_float(s_maxkey);
                const int nn = filter_by_max<NT, kEPT>(buf, s_n, m, a.inv_t, s_w);
                if (tid == 0) {
                    s_n = nn;
                    if (nn > a.cap / 2) s_flags |= kOverflow;
                }
                __syncthreads();
                if (s_flags & kOverflow) {
                    stop = true;
                    break;
                }
                uint32_t pp = pend;
                while (pp) {
                    const int e = __ffs(pp) - 1;
                    pp &= pp - 1;
                    float xv = 0.0f;
#pragma unroll
                    for (int ee = 0; ee < NE; ++ee)
                        if (ee == e) xv = x[ee];
                    if (!(scaled_diff(xv, m, a.inv_t) > -15.0f)) pend &= ~(1u << e);
                }
            }
        }
        if (stop) break;
    }

    /* ====================== finish the row ====================== */
    if (MODE == kGreedy) {
        /* block argmax by (value desc, id asc); NaN never wins (sampler.c:106-116) */
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
            s_gbest_key[tid >> 5] = __float_as_uint(gx);
            s_gbest_id[tid >> 5] = gid;
        }
        __syncthreads();
        if (a.wb && a.penalty) write_back_penalty<NT>(a, hv, row);
        if (tid == 0) {
            float bx = __uint_as_float(s_gbest_key[0]);
            uint32_t bid = s_gbest_id[0];
            for (int w = 1; w < NT / 32; ++w) {
                const float ox = __uint_as_float(s_gbest_key[w]);
                const uint32_t oid = s_gbest_id[w];
                if (ox > bx || (ox == bx && oid < bid)) {
                    bx = ox;
                    bid = oid;
                }
            }
            RowOut o;
            o.id = (s_l0nan || bid == 0xFFFFFFFFu) ? 0 : (int)bid;
            o.prob = 1.0f;
            o.mass = 1.0f;
            o.n_topk = o.n_final = o.num_cands = 1;
            o.flags = NOEL_ROW_GREEDY;
            write_row_stats(a, row, o);
            if (a.list_ids) {
                for (int i = 0; i < a.list_len; ++i) {
                    a.list_ids[(size_t)row * a.list_len + i] = i == 0 ? o.id : -1;
                    if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = i == 0 ? 1.0f : 0.0f;
                }
            }
        }
        return;
    }

    __syncthreads();
    if (a.wb && a.penalty) write_back_penalty<NT>(a, hv, row);
    if (MODE == kFullList) {
        if (tmax > -INFINITY) atomicMax(&s_maxkey, ord_key(tmax));
        __syncthreads();
        if (s_flags & kOverflow) {
            if (tid == 0) list_exact_row(a, row);
            return;
        }
    }

    int n = s_n;
    if (MODE == kTopK && (s_flags & kWarmBet) && n < a.kprime) {  // the warm-up's bet lost
        if (tid == 0) list_exact_row(a, row);
        return;
    }
    bool trunc = (s_flags & kTruncated) != 0;
    uint32_t t_last = 0u;
    if (MODE == kTopK && (n > a.kprime || trunc)) {
        uint32_t ithr;
        t_last = select_top<NT, kEPT>(buf, n, a.kprime, ss, s_w, &ithr);
        n = a.kprime;
        trunc = true;
    }
    float M;
    if (MODE == kTopK) {
        uint32_t mk = 0u;
        for (int i = tid; i < n; i += NT) mk = max(mk, buf.key[i]);
        mk = block_max_u32<NT>(mk, s_wu);
        M = (s_l0nan || n == 0) ? __uint_as_float(0x7FC00000u) : key_float(mk);
    } else {
        M = s_l0nan ? __uint_as_float(0x7FC00000u) : key_float(s_maxkey);
        n = filter_by_max<NT, kEPT>(buf, n, M, a.inv_t, s_w);
    }

    /* weights, then sort keys (weight desc, id asc) in place as u64 */
    int P = 1;
    while (P < n) P <<= 1;
    uint64_t *sk = reinterpret_cast<uint64_t *>(buf.key);
    int mine = 0;
    {
        uint64_t kv[kEPT];
        const int per = (n + NT - 1) / NT;
        const int i0 = tid * per;
#pragma unroll
        for (int e = 0; e < kEPT; ++e) {
            kv[e] = 0ull;
            const int i = i0 + e;
            if (e < per && i < n) {
                const float d = scaled_diff(key_float(buf.key[i]), M, a.inv_t);
                if (d > -15.0f) {
                    const float wgt = ref_weight(d, a.et);
                    kv[e] = ((uint64_t)__float_as_uint(wgt) << 32) | (uint64_t)(0xFFFFFFFFu - buf.id[i]);
                    ++mine;
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int e = 0; e < kEPT; ++e) {
            const int i = i0 + e;
            if (e < per && i < n) sk[i] = kv[e];
        }
        for (int i = n + tid; i < P; i += NT) sk[i] = 0ull;
    }
    const int ncand = block_sum_int<NT>(mine, s_w);  // its barriers publish sk
    block_bitonic_pairs_desc<NT>(sk, P);

    if (tid < 32) {  // warp 0
        bool more = false;
        bool exact = true;
        if (MODE == kTopK && trunc && ncand == n) {
            more = true;  // every kept entry is a candidate: the row has more
            const float dl = scaled_diff(key_float(t_last), M, a.inv_t);
            const float v_last = dl > -15.0f ? ref_weight(dl, a.et) : 0.0f;
            const float v_k = __uint_as_float((uint32_t)(sk[a.top_k - 1] >> 32));
            if (!(v_last < v_k)) exact = false;
        }
        if (!exact) {
            if (tid == 0) {
                list_exact_row(a, row);
                s_fin_n = -1;
            }
        } else {
            const bool fb = ncand == 0;
            uint64_t st[2] = {0ull, 0ull};
            if (tid == 0) {
                st[0] = a.rng[2 * (size_t)row];
                st[1] = a.rng[2 * (size_t)row + 1];
            }
            auto w = [&](int i) -> float {
                return fb ? 1.0f : __uint_as_float((uint32_t)(sk[i] >> 32));
            };
            /* the running sums go to the warm-up bins (2048 floats >= K') */
            const TailOut t = warp_tail(fb ? 1 : ncand, more, a.top_k, a.top_p, st, w, reinterpret_cast<float *>(whist));
            if (tid == 0) {
                a.rng[2 * (size_t)row] = st[0];
                a.rng[2 * (size_t)row + 1] = st[1];
                RowOut o;
                o.id = fb ? 0 : (int)(0xFFFFFFFFu - (uint32_t)sk[t.pos]);
                o.prob = __fdiv_rn(w(t.pos), t.mass);
                o.mass = t.mass;
                o.n_topk = t.n_topk;
                o.n_final = t.n_final;
                o.num_cands = more ? -1 : (fb ? 1 : ncand);
                o.flags = fb ? NOEL_ROW_FALLBACK : 0;
                write_row_stats(a, row, o);
                s_fin_n = fb ? -2 : t.n_final;
                s_fin_mass = t.mass;
            }
        }
    }
    __syncthreads();
    if (a.list_ids && s_fin_n != -1) {
        const int nf = s_fin_n == -2 ? 1 : s_fin_n;
        for (int i = tid; i < a.list_len; i += NT) {
            int id = -1;
            float p = 0.0f;
            if (i < nf) {
                if (s_fin_n == -2) {
                    id = 0;
                    p = 1.0f;
                } else {
                    id = (int)(0xFFFFFFFFu - (uint32_t)sk[i]);
                    p = __uint_as_float((uint32_t)(sk[i] >> 32));
                    if (!a.list_weights) p = __fdiv_rn(p, s_fin_mass);
                }
            }
            a.list_ids[(size_t)row * a.list_len + i] = id;
            if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = p;
        }
    }
}

}  // namespace noel

#include "sampler_warp.cuh"
#include "sampler_shard.cuh"

namespace noel {

/* ====================================================================== */
/* exact two-pass kernel for listed rows                                   */

/* stable LSD radix sort of n (x = key, y = payload) pairs by key ascending */
template <int NT>
__device__ uint2 *radix_sort_stable(uint2 *A, uint2 *B, int n, uint32_t *s_h, int *s_w, int *s_skip) {
    constexpr int NW = NT / 32;
    static_assert(NT == 256, "one digit per thread in the scan");
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int chunk = ((((n + NW - 1) / NW) + 31) / 32) * 32;
    const int c0 = min(n, w * chunk), c1 = min(n, c0 + chunk);
    const uint32_t lt = (1u << lane) - 1u;
    for (int shift = 0; shift < 32; shift += 8) {
        for (int i = threadIdx.x; i < NW * 256; i += NT) s_h[i] = 0u;
        if (threadIdx.x == 0) *s_skip = 0;
        __syncthreads();
        for (int base = c0; base < c1; base += 32) {
            const int i = base + lane;
            const bool ok = i < c1;
            const uint32_t mask = __ballot_sync(kFull, ok);
            if (ok) {
                const uint32_t d = (A[i].x >> shift) & 255u;
                const uint32_t peers = __match_any_sync(mask, d);
                if ((peers & lt) == 0u) s_h[w * 256 + d] += (uint32_t)__popc(peers);
            }
            __syncwarp();
        }
        __syncthreads();
        {
            const int d = threadIdx.x;
            int tot = 0;
            for (int ww = 0; ww < NW; ++ww) tot += (int)s_h[ww * 256 + d];
            if (tot == n) *s_skip = 1;
            int all;
            int base = block_excl_scan<NT>(tot, s_w, all);
            for (int ww = 0; ww < NW; ++ww) {
                const int c = (int)s_h[ww * 256 + d];
                s_h[ww * 256 + d] = (uint32_t)base;
                base += c;
            }
        }
        __syncthreads();
        if (*s_skip) continue;
        for (int base = c0; base < c1; base += 32) {
            const int i = base + lane;
            const bool ok = i < c1;
            const uint32_t mask = __ballot_sync(kFull, ok);
            uint32_t d = 0u, peers = 0u;
            if (ok) {
                const uint2 e = A[i];
                d = (e.x >> shift) & 255u;
                peers = __match_any_sync(mask, d);
                B[s_h[w * 256 + d] + __popc(peers & lt)] = e;
            }
            __syncwarp();
            if (ok && (peers & lt) == 0u) s_h[w * 256 + d] += (uint32_t)__popc(peers);
            __syncwarp();
        }
        __syncthreads();
        uint2 *t = A;
        A = B;
        B = t;
    }
    return A;
}

template <typename T>
__global__ void __launch_bounds__(kExactThreads) exact_rows_kernel(const SampleArgs a) {
    /* launched as a programmatic dependent of the main kernel: wait until
     * that grid has finished and its writes (the row list) are visible */
    asm volatile("griddepcontrol.wait;" ::: "memory");
    using F = Fmt<T>;
    constexpr int NT = kExactThreads, NW = NT / 32, IPT = 16;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t s_h[NW * 256];
    __shared__ int s_w[NT / 32 + 1];
    __shared__ uint32_t s_wu[NT / 32];
    __shared__ int s_row, s_skip, s_l0nan, s_fin_n;
    __shared__ float s_fin_mass;
    __shared__ uint2 *s_sorted;

    const int tid = threadIdx.x;
    const int V = a.vocab;
    const bool pen = a.penalty && !a.wb;  // with write-back the row is already penalised
    HistView hv{nullptr, nullptr, nullptr, 0};
    if (pen) {
        unsigned char *sp = smem;
        hv.words = (V + 31) >> 5;
        const int G = (hv.words + 7) >> 3;
        hv.bm = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)hv.words * 4;
        hv.gpre = reinterpret_cast<uint32_t *>(sp);
        sp += (size_t)(G + 1) * 4;
        hv.cnt = reinterpret_cast<uint32_t *>(sp);
    }
    uint2 *slotA = a.slots + (size_t)blockIdx.x * 2 * (size_t)V;
    uint2 *slotB = slotA + V;

    for (;;) {
        if (tid == 0) {
            const int q = atomicAdd(&a.counters[1], 1);
            s_row = q < *(volatile int *)&a.counters[0] ? a.exact_list[q] : -1;
            s_l0nan = 0;
        }
        __syncthreads();
        const int row = s_row;
        if (row < 0) break;
        const RowSpan span = row_span(a, row);
        const int Vr = span.V;
        const void *rowp = static_cast<const char *>(a.logits) + (size_t)span.off * F::ES;
        if (pen) build_history<NT>(hv, a.hist + (size_t)span.hrow * a.hld, a.hist_start, a.hist_len, Vr, s_w, span.id_off);

        auto load = [&](int i) -> float {
            float x = F::scalar(rowp, i);
            if (pen && ((hv.bm[i >> 5] >> (i & 31)) & 1u)) x = apply_penalty(x, hv.cnt[hist_rank(hv, i)], a.rep);
            return x;
        };
        /* pass 1: max of the penalised row (sampler.c:119-124) */
        float mx = -INFINITY;
        for (int i = tid; i < Vr; i += NT) {
            const float x = load(i);
            if (i == 0 && x != x && span.id_off == 0) s_l0nan = 1;
            mx = fmaxf(mx, x);
        }
        const uint32_t mk = block_max_u32<NT>(mx > -INFINITY ? ord_key(mx) : kKeyNegInf, s_wu);
        const float M = s_l0nan ? __uint_as_float(0x7FC00000u) : key_float(mk);

        /* pass 2: candidates in id order (sampler.c:136-143) as (~weight bits, id) */
        int n = 0;
        for (int t0 = 0; t0 < Vr; t0 += NT * IPT) {
            uint32_t wb[IPT];
            int c = 0;
#pragma unroll
            for (int e = 0; e < IPT; ++e) {
                const int i = t0 + tid * IPT + e;
                wb[e] = 0u;
                if (i < Vr) {
                    const float x = load(i);
                    if (a.shard_lists) {
                        /* a vocab shard lists every number by logit (greedy
                         * rows need them all; ord_key is never 0) */
                        if (x == x) {
                            wb[e] = ord_key(x);
                            ++c;
                        }
                    } else {
                        const float d = scaled_diff(x, M, a.inv_t);
                        if (d > -15.0f) {
                            wb[e] = __float_as_uint(ref_weight(d, a.et));
                            ++c;
                        }
                    }
                }
            }
            int tot;
            int pos = n + block_excl_scan<NT>(c, s_w, tot);
#pragma unroll
            for (int e = 0; e < IPT; ++e)
                if (wb[e]) slotA[pos++] = make_uint2(~wb[e], (uint32_t)(t0 + tid * IPT + e));
            n += tot;
        }
        __syncthreads();
        const bool fb = n == 0;
        uint2 *sorted = slotA;
        if (n > 1) sorted = radix_sort_stable<NT>(slotA, slotB, n, s_h, s_w, &s_skip);
        if (a.shard_lists) {
            /* vocab shard: its best shard_len by (logit desc, id asc) */
            if (tid < 32) {
                const int m = min(n, a.shard_len);
                shard_write(a, row, span.id_off, m, n > 0 ? key_float(mk) : -INFINITY,
                            (s_l0nan ? kShardNaN0 : 0) | (n > m ? kShardMore : 0),
                            [&](int i) { return make_uint2(sorted[i].y, ~sorted[i].x); });
            }
            __syncthreads();
            continue;
        }
        if (tid < 32) {  // warp 0: running sums into the other slot, staged through s_h
            uint64_t st[2] = {0ull, 0ull};
            if (tid == 0) {
                st[0] = a.rng[2 * (size_t)row];
                st[1] = a.rng[2 * (size_t)row + 1];
            }
            auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float(~sorted[i].x); };
            float *sums = reinterpret_cast<float *>(sorted == slotA ? slotB : slotA);
            const TailOut t = warp_tail_global(fb ? 1 : n, false, a.top_k, a.top_p, st, w, sums,
                                               reinterpret_cast<float *>(s_h));
            if (tid == 0) {
                a.rng[2 * (size_t)row] = st[0];
                a.rng[2 * (size_t)row + 1] = st[1];
                RowOut o;
                o.id = fb ? 0 : (int)sorted[t.pos].y;
                o.prob = __fdiv_rn(w(t.pos), t.mass);
                o.mass = t.mass;
                o.n_topk = t.n_topk;
                o.n_final = t.n_final;
                o.num_cands = fb ? 1 : n;
                o.flags = NOEL_ROW_EXACT_PASS | (fb ? NOEL_ROW_FALLBACK : 0);
                write_row_stats(a, row, o);
                s_fin_n = fb ? -2 : t.n_final;
                s_fin_mass = t.mass;
                s_sorted = sorted;
            }
        }
        __syncthreads();
        if (a.list_ids) {
            const int nf = s_fin_n == -2 ? 1 : s_fin_n;
            for (int i = tid; i < a.list_len; i += NT) {
                int id = -1;
                float p = 0.0f;
                if (i < nf) {
                    if (s_fin_n == -2) {
                        id = 0;
                        p = 1.0f;
                    } else {
                        id = (int)s_sorted[i].y;
                        p = __uint_as_float(~s_sorted[i].x);
                        if (!a.list_weights) p = __fdiv_rn(p, s_fin_mass);
                    }
                }
                a.list_ids[(size_t)row * a.list_len + i] = id;
                if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = p;
            }
        }
        __syncthreads();
    }
    /* the last CTA out re-arms the row list for the next call on this workspace */
    if (tid == 0) {
        __threadfence();
        const int d = atomicAdd(&a.counters[2], 1);
        if (d == (int)gridDim.x - 1) {
            a.counters[0] = 0;
            a.counters[1] = 0;
            a.counters[2] = 0;
            __threadfence();
        }
    }
}

/* ====================================================================== */
/* exp-parity checksums over every float in (-15, 0]                        */

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* grid (chunks, parts): block (c, s) sums part s of chunk c, one atomic per block */
__global__ void expf_checksum_kernel(int chunk_log2, uint64_t *out, ExpTable et) {
    __shared__ unsigned long long s_part[32];
    const uint64_t span = (uint64_t)(NOEL_EXPF_DOMAIN_END - NOEL_EXPF_DOMAIN_FIRST);
    const uint64_t csize = 1ull << chunk_log2;
    const uint64_t c0 = (uint64_t)blockIdx.x * csize;
    const uint64_t psize = (csize + gridDim.y - 1) / gridDim.y;
    const uint64_t lo = c0 + (uint64_t)blockIdx.y * psize;
    const uint64_t hi = min(min(lo + psize, c0 + csize), span);
    unsigned long long acc = 0ull;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const uint32_t ub = NOEL_EXPF_DOMAIN_FIRST + (uint32_t)i;
        const float y = ref_weight(__uint_as_float(ub), et);
        acc += mix64(((uint64_t)ub << 32) | __float_as_uint(y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0ull;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_part[w];
        if (lo < hi) atomicAdd(reinterpret_cast<unsigned long long *>(&out[blockIdx.x]), t);
    }
}

}  // namespace noel
