/*
 * The single-pass sampling kernel for greedy rows, top-k rows with k <= 120
 * and full-list rows (top-k off): one CTA per row, eight warps that stream
 * their own slices of the row without block barriers.
 *
 * Row start: the CTA builds the history bitmap and per-id counts in shared
 * memory (sampler.c:87-103).  Streaming: warp w reads its eighth of the row
 * with 256-bit loads (four in flight per lane), applies the penalty, takes
 * the maximum of each 8-element vector and only looks at single elements
 * when that maximum can pass the current threshold:
 *   top-k  - the best (logit desc, id asc) key that K' kept elements beat;
 *            every warp keeps its own buffer, compacts it by a warp radix
 *            select when it fills, and publishes its threshold to the other
 *            warps (a shared 64-bit atomicMax), which filter with it too;
 *   full   - the -15 cut under the row's running max, shared the same way;
 *   greedy - the running (value, lowest id) maximum.
 * Row end: the warps' candidates are gathered and warp 0 alone computes the
 * weights, sorts them and runs the sequential mass / nucleus / draw loops
 * (sampler.c:119-191) while the CTA's other warps retire, so other CTAs on
 * the SM keep the memory system busy.
 */
#pragma once

#include "sampler_device.cuh"

namespace noel {

constexpr int kUnionCap = 1024;  // row-end gather / sort area (entries)
constexpr int kRowWarps = 4;     // warps streaming one row
constexpr int kRowThreads = 32 * kRowWarps;

/* Bin of the K-th largest count in a 2048-bin histogram (counted from the top
 * bin down), found by all NT threads: each owns 2048/NT consecutive bins.
 * Returns the bin (or -1 if the total is below K); *need_in_bin = how many of
 * that bin's entries are needed. */
template <int NT>
__device__ int block_find_bin_desc(const uint32_t *h, int K, int *s_w, int *s_res, int *need_in_bin) {
    constexpr int PER = 2048 / NT;
    const int hi = 2047 - threadIdx.x * PER;  // this thread's bins: hi, hi-1, ..., hi-PER+1
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

template <typename T, int MODE>
__global__ void __launch_bounds__(kRowThreads, 16 / kRowWarps) sample_rows_kernel(const SampleArgs a) {
    using F = Fmt<T>;
    constexpr int NT = kRowThreads, NW = NT / 32;
    constexpr int VEC = F::VEC, U = F::U, NE = U * VEC;
    static_assert(NE <= 32, "pending mask is 32 bits");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ unsigned long long s_taus[NW];  // each warp's own exclusion threshold
    __shared__ unsigned long long s_btau;      // block warm-up threshold (top-k)
    __shared__ unsigned long long s_tsh;       // best shared filter (warm-up or ladders)
    __shared__ unsigned long long s_lad[3][NW];  // each warp's (2kw/NW)-th, (kw/2)-th, kw-th kept key
    __shared__ int s_res[2];
    __shared__ uint32_t s_maxkey;
    __shared__ int s_flags, s_l0nan, s_trunc;
    __shared__ int s_wcnt[NW];
    __shared__ int s_wfill[NW];  // entries each warp has claimed in its buffer
    __shared__ int s_w[NW + 1];
    __shared__ float s_gx[NW];
    __shared__ uint32_t s_gid[NW];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x;
    const int V = a.vocab;
    const void *rowp = static_cast<const char *>(a.logits) + (size_t)row * (size_t)a.ld * F::ES;

    /* ---- shared-memory carve-up ---- */
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
        sp = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(sp) + 15) & ~uintptr_t(15));
    }
    const int capw = a.cap;  // per-warp buffer entries
    uint32_t *wkey = nullptr, *wid = nullptr, *whist = nullptr;
    uint32_t *ukey = nullptr, *uid = nullptr;
    uint64_t *sk = nullptr;
    if (MODE != kGreedy) {
        uint32_t *wb = reinterpret_cast<uint32_t *>(sp);
        wkey = wb + (size_t)warp * capw * 2;
        wid = wkey + capw;
        sp += (size_t)NW * capw * 8;
        whist = reinterpret_cast<uint32_t *>(sp) + warp * 256;
        sp += (size_t)NW * 256 * 4;
        ukey = reinterpret_cast<uint32_t *>(sp);
        uid = ukey + kUnionCap;
        sp += (size_t)kUnionCap * 8;
        sk = reinterpret_cast<uint64_t *>(sp);
    }

    if (tid < NW) {
        s_wfill[tid] = 0;
        s_taus[tid] = 0ull;
        s_lad[0][tid] = s_lad[1][tid] = s_lad[2][tid] = 0ull;
    }
    if (MODE == kTopK)
        for (int i = tid; i < 2048; i += NT) ukey[i] = 0u;  // warm-up bins (the gather area)
    if (tid == 0) {
        s_btau = 0ull;
        s_tsh = 0ull;
        s_maxkey = kKeyNegInf;
        s_flags = 0;
        s_l0nan = 0;
        s_trunc = 0;
    }
    if (a.penalty) build_history<NT>(hv, a.hist + (size_t)row * a.hld, a.hist_start, a.hist_len, V, s_w);
    __syncthreads();

    const RowGeom g = row_geom<T>(rowp, V);
    const V8 *vbase = reinterpret_cast<const V8 *>(static_cast<const char *>(rowp) + (size_t)g.head * F::ES);
    const int per = (g.nvec + NW - 1) / NW;
    const int v0 = min(g.nvec, warp * per), v1 = min(g.nvec, v0 + per);

    const int kw = max(8, a.kprime / 2);  // entries a warp keeps (top-k mode)
    int wcount = 0;
    bool wtrunc = false;
    unsigned long long tau_w = 0ull;
    float gx = -INFINITY;
    uint32_t gid = 0xFFFFFFFFu;
    bool stop = false;

    /* ---- scalar head / tail (warp 0) ---- */
    if (warp == 0) {
        const bool have = lane < g.nscalar;
        float xs = 0.0f;
        int ids = 0;
        if (have) {
            ids = scalar_id(g, lane);
            xs = F::scalar(rowp, ids);
            if (a.penalty && ((hv.bm[ids >> 5] >> (ids & 31)) & 1u))
                xs = apply_penalty(xs, hv.cnt[hist_rank(hv, ids)], a.rep);
            if (ids == 0 && xs != xs) s_l0nan = 1;
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
                wkey[pos] = ord_key(xs);
                wid[pos] = (uint32_t)ids;
            }
            wcount = __popc(b);
            if (lane == 0) s_wfill[0] = wcount;
            if (MODE == kFullList) {
                const float m = warp_max_f(ins ? xs : -INFINITY);
                if (lane == 0 && m > -INFINITY) atomicMax(&s_maxkey, ord_key(m));
            }
            __syncwarp();
        }
    }

    /* ---- the warp's slice of the vector body, next batch prefetched ---- */
    V8 nxt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int vi = v0 + u * 32 + lane;
        if (vi < v1) nxt[u] = ld_stream(vbase + vi);
    }
    if (MODE == kTopK && min(g.nvec, NW * 32 * U) * VEC >= 4 * a.kprime) {
        /* Block warm-up on every warp's first batch: each warp's lane maxima
         * give it a threshold with 32 elements above; the second largest of
         * those bounds a histogram (2048 bins on the top 11 key bits) of the
         * batch's larger elements, whose bin holding the K'-th largest gives
         * the row's starting threshold. */
        float xw[NE];
        bool okw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int vi = v0 + u * 32 + lane;
            okw[u] = vi < v1;
            if (okw[u]) {
                F::unpack(nxt[u], xw + u * VEC);
                if (a.penalty) penalize_group<VEC>(hv, g.head + vi * VEC, xw + u * VEC, a.rep);
            } else {
#pragma unroll
                for (int j = 0; j < VEC; ++j) xw[u * VEC + j] = -INFINITY;
            }
        }
        float lmax = -INFINITY;
#pragma unroll
        for (int e = 0; e < NE; ++e) lmax = fmaxf(lmax, xw[e]);  // NaN-ignoring
        const float t0 = warp_min_f(lmax);
        if (t0 > -INFINITY) {
            tau_w = (unsigned long long)ord_key(t0) << 32;  // 32 elements of this warp beat it
            wtrunc = true;
            if (lane == 0) s_taus[warp] = tau_w;
        }
        __syncthreads();
        unsigned long long t1 = 0ull, t2 = 0ull;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const unsigned long long tw = s_taus[w];
            if (tw > t1) { t2 = t1; t1 = tw; } else if (tw > t2) { t2 = tw; }
        }
        const uint32_t lo_key = (uint32_t)(t2 >> 32);
#pragma unroll
        for (int e = 0; e < NE; ++e) {
            const float xv = xw[e];
            if (xv == xv && xv > -INFINITY && ord_key(xv) >= lo_key) atomicAdd(&ukey[ord_key(xv) >> 21], 1u);
        }
        __syncthreads();
        /* level 1: bin (top 11 key bits) of the K'-th largest; level 2: the next
         * 11 bits inside that bin */
        int need;
        const int wb = block_find_bin_desc<NT>(ukey, a.kprime, s_w, s_res, &need);
        if (wb >= 0) {
            uint32_t *h2 = ukey + 2048;  // second-level bins
            for (int i = tid; i < 2048; i += NT) h2[i] = 0u;
            __syncthreads();
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                const float xv = xw[e];
                if (xv == xv && xv > -INFINITY && (int)(ord_key(xv) >> 21) == wb)
                    atomicAdd(&h2[(ord_key(xv) >> 10) & 2047u], 1u);
            }
            __syncthreads();
            int need2;
            const int b2 = block_find_bin_desc<NT>(h2, need, s_w, s_res, &need2);
            if (tid == 0 && b2 >= 0) {
                const uint32_t key = ((uint32_t)wb << 21) | ((uint32_t)b2 << 10);
                s_btau = (unsigned long long)key << 32;
                s_tsh = s_btau;
            }
            __syncthreads();
        }
    }

    for (int base = v0; base < v1; base += 32 * U) {
        float x[NE];
        float vm[U];
        uint32_t valid = 0u;
        {
            V8 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = nxt[u];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = base + 32 * U + u * 32 + lane;
                if (vi < v1) nxt[u] = ld_stream(vbase + vi);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int vi = base + u * 32 + lane;
                if (vi < v1) {
                    F::unpack(v[u], x + u * VEC);
                    valid |= ((1u << VEC) - 1u) << (u * VEC);
                } else {
#pragma unroll
                    for (int j = 0; j < VEC; ++j) x[u * VEC + j] = -INFINITY;
                }
            }
        }
        if (base == 0 && lane == 0 && g.head == 0 && (valid & 1u) && x[0] != x[0]) s_l0nan = 1;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float m = x[u * VEC];
#pragma unroll
            for (int j = 1; j < VEC; ++j) m = fmaxf(m, x[u * VEC + j]);
            vm[u] = m;  // NaN-free unless the whole vector is NaN
        }

        /* The penalty only lowers values (sampler.c:96-100), so a vector whose
         * raw maximum cannot pass the filter needs no penalty lookup.  This
         * applies it to vector u and returns the penalised maximum. */
        uint32_t pdone = 0u;  // vectors already penalised in this batch
        auto penalize_vec = [&](int u) -> float {
            const int vi = base + u * 32 + lane;
            if (!a.penalty || vi >= v1 || ((pdone >> u) & 1u)) return vm[u];
            pdone |= 1u << u;
            const int id0 = g.head + vi * VEC;
            uint32_t bits = hist_bits(hv, id0, VEC);
            if (!bits) return vm[u];
            while (bits) {
                const int j = __ffs(bits) - 1;
                bits &= bits - 1;
                const uint32_t c = hv.cnt[hist_rank(hv, id0 + j)];
#pragma unroll
                for (int jj = 0; jj < VEC; ++jj)
                    if (jj == j) x[u * VEC + jj] = apply_penalty(x[u * VEC + jj], c, a.rep);
            }
            float m = x[u * VEC];
#pragma unroll
            for (int j = 1; j < VEC; ++j) m = fmaxf(m, x[u * VEC + j]);
            vm[u] = m;
            return m;
        };

        if (MODE == kGreedy) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (vm[u] >= gx && penalize_vec(u) >= gx) {
                    const uint32_t id0 = (uint32_t)(g.head + (base + u * 32 + lane) * VEC);
#pragma unroll
                    for (int j = 0; j < VEC; ++j) {
                        const float xv = x[u * VEC + j];
                        if (((valid >> (u * VEC + j)) & 1u) && (xv > gx || (xv == gx && id0 + j < gid))) {
                            gx = xv;
                            gid = id0 + j;
                        }
                    }
                }
            }
            continue;
        }

        uint32_t pend = 0u;
        float m_cur = 0.0f;
        unsigned long long tau_eff = 0ull;
        if (MODE == kTopK) {
            tau_eff = max(tau_w, *(volatile unsigned long long *)&s_tsh);
            const uint32_t tk = (uint32_t)(tau_eff >> 32);
            const float tau_f = tk == 0u ? -INFINITY : key_float(tk);
            const uint32_t tau_id = 0xFFFFFFFFu - (uint32_t)tau_eff;  // ties at tau_f pass below this id
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (vm[u] >= tau_f && penalize_vec(u) >= tau_f) {
                    const uint32_t id0 = (uint32_t)(g.head + (base + u * 32 + lane) * VEC);
#pragma unroll
                    for (int j = 0; j < VEC; ++j) {
                        const float xv = x[u * VEC + j];
                        const bool pass = xv > tau_f || (xv == tau_f && id0 + j < tau_id);
                        if (pass && ((valid >> (u * VEC + j)) & 1u)) pend |= 1u << (u * VEC + j);
                    }
                }
            }
        } else {
            if (__any_sync(kFull, (*(volatile int *)&s_flags & kOverflow) != 0)) break;
            /* the running max of penalised values: raw maxima are upper bounds,
             * so only vectors whose raw max exceeds it are penalised first */
            float lm = -INFINITY;
            {
                const float mk = key_float(*(volatile uint32_t *)&s_maxkey);
#pragma unroll
                for (int u = 0; u < U; ++u) lm = fmaxf(lm, vm[u] > mk ? penalize_vec(u) : vm[u]);
            }
            lm = warp_max_f(lm);
            if (lane == 0 && lm > -INFINITY) atomicMax(&s_maxkey, ord_key(lm));
            __syncwarp();
            m_cur = key_float(*(volatile uint32_t *)&s_maxkey);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (scaled_diff(vm[u], m_cur, a.inv_t) > -15.0f && scaled_diff(penalize_vec(u), m_cur, a.inv_t) > -15.0f) {
#pragma unroll
                    for (int j = 0; j < VEC; ++j)
                        if (((valid >> (u * VEC + j)) & 1u) && scaled_diff(x[u * VEC + j], m_cur, a.inv_t) > -15.0f)
                            pend |= 1u << (u * VEC + j);
                }
            }
        }

        /* ---- lane-local insert into the warp's buffer; compact when full ---- */
        for (;;) {
            if (!__any_sync(kFull, pend != 0u)) break;
            if (pend) {
                int slot = atomicAdd(&s_wfill[warp], __popc(pend));
                uint32_t pp = pend;
                while (pp) {  // compact loop: this path is rare
                    const int e = __ffs(pp) - 1;
                    pp &= pp - 1;
                    if (slot < capw) {
                        float xv = x[0];
#pragma unroll
                        for (int q = 1; q < NE; ++q) xv = (q == e) ? x[q] : xv;
                        wkey[slot] = ord_key(xv);
                        wid[slot] = (uint32_t)(g.head + (base + (e / VEC) * 32 + lane) * VEC + (e % VEC));
                        pend &= ~(1u << e);
                    }
                    ++slot;
                }
            }
            if (!__any_sync(kFull, pend != 0u)) break;
            __syncwarp();
            wcount = min(*(volatile int *)&s_wfill[warp], capw);
            __syncwarp();
            if (MODE == kTopK) {
                uint64_t lad[3];
                tau_w = warp_topk_sorted_r<4>(wkey, wid, wcount, kw, lad, max(1, 2 * kw / NW));
                wcount = kw;
                wtrunc = true;
                if (lane == 0) {
                    s_wfill[warp] = kw;
                    s_taus[warp] = tau_w;
                    s_lad[0][warp] = lad[0];
                    s_lad[1][warp] = lad[1];
                    s_lad[2][warp] = lad[2];
                    __threadfence_block();
                    /* K' retained elements beat each of: every warp's
                     * (2kw/NW)-th, the 4th largest (kw/2)-th (NW >= 4), the
                     * 2nd largest kw-th */
                    unsigned long long mn = ~0ull, b[4] = {0ull, 0ull, 0ull, 0ull}, c1 = 0ull, c2 = 0ull;
                    for (int w = 0; w < NW; ++w) {
                        const unsigned long long l0 = *(volatile unsigned long long *)&s_lad[0][w];
                        const unsigned long long l1 = *(volatile unsigned long long *)&s_lad[1][w];
                        const unsigned long long l2 = *(volatile unsigned long long *)&s_lad[2][w];
                        mn = min(mn, l0);
                        for (int q = 0; q < 4; ++q)
                            if (l1 > b[q]) {
                                for (int z = 3; z > q; --z) b[z] = b[z - 1];
                                b[q] = l1;
                                break;
                            }
                        if (l2 > c1) { c2 = c1; c1 = l2; } else if (l2 > c2) { c2 = l2; }
                    }
                    if (NW < 4) b[3] = 0ull;
                    atomicMax(&s_tsh, max(max(mn, b[3]), c2));
                }
                tau_eff = max(tau_w, *(volatile unsigned long long *)&s_tsh);
                __syncwarp();
#pragma unroll
                for (int e = 0; e < NE; ++e)
                    if ((pend >> e) & 1u) {
                        const uint32_t id = (uint32_t)(g.head + (base + (e / VEC) * 32 + lane) * VEC + (e % VEC));
                        if (!(comp_key(ord_key(x[e]), id) > tau_eff)) pend &= ~(1u << e);
                    }
            } else {
                const float m = key_float(*(volatile uint32_t *)&s_maxkey);
                wcount = warp_filter_by_max(wkey, wid, wcount, m, a.inv_t);
                if (lane == 0) s_wfill[warp] = wcount;
                __syncwarp();
                if (wcount > capw / 2) {
                    if (lane == 0) atomicOr(&s_flags, kOverflow);
                    stop = true;
                    break;
                }
#pragma unroll
                for (int e = 0; e < NE; ++e)
                    if (((pend >> e) & 1u) && !(scaled_diff(x[e], m, a.inv_t) > -15.0f)) pend &= ~(1u << e);
            }
        }
        if (stop) break;
    }

    /* ====================== finish the row ====================== */
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
            s_gx[warp] = gx;
            s_gid[warp] = gid;
        }
        __syncthreads();
        if (a.wb && a.penalty) write_back_penalty<NT>(a, hv, row);
        if (tid == 0) {
            float bx = s_gx[0];
            uint32_t bid = s_gid[0];
            for (int w = 1; w < NW; ++w)
                if (s_gx[w] > bx || (s_gx[w] == bx && s_gid[w] < bid)) {
                    bx = s_gx[w];
                    bid = s_gid[w];
                }
            RowOut o;
            o.id = (s_l0nan || bid == 0xFFFFFFFFu) ? 0 : (int)bid;  // sampler.c:106-116
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

    if (MODE != kGreedy) wcount = min(*(volatile int *)&s_wfill[warp], capw);
    __syncthreads();  // all warps done streaming: s_maxkey, s_flags final
    if (a.wb && a.penalty) write_back_penalty<NT>(a, hv, row);
    if (MODE == kFullList && (s_flags & kOverflow)) {
        if (tid == 0) list_exact_row(a, row);
        return;
    }
    const float Mfull = s_l0nan ? __uint_as_float(0x7FC00000u) : key_float(s_maxkey);
    if (MODE == kTopK) {
        /* entries below the second largest threshold cannot make the top K' */
        const unsigned long long t2 = s_tsh;
        if (t2) {
            int wn = 0;
            for (int b0 = 0; b0 < wcount; b0 += 32) {
                const int i = b0 + lane;
                const bool ok = i < wcount;
                const uint32_t k = ok ? wkey[i] : 0u, v = ok ? wid[i] : 0u;
                const bool keep = ok && comp_key(k, v) >= t2;
                const uint32_t bal = __ballot_sync(kFull, keep);
                __syncwarp();
                if (keep) {
                    const int pos = wn + __popc(bal & lanemask_lt());
                    wkey[pos] = k;
                    wid[pos] = v;
                }
                wn += __popc(bal);
                __syncwarp();
            }
            wcount = wn;
        }
        if (wcount > 2 * kw) {  // keeps the gather within its area
            tau_w = warp_topk_sorted_r<4>(wkey, wid, wcount, kw, nullptr, 1);
            wcount = kw;
            wtrunc = true;
        }
    } else {
        wcount = warp_filter_by_max(wkey, wid, wcount, Mfull, a.inv_t);
    }
    if (lane == 0) {
        s_wcnt[warp] = wcount;
        s_taus[warp] = wtrunc ? tau_w : 0ull;  // final exclusion threshold of this warp
        if (wtrunc) s_trunc = 1;
    }
    __syncthreads();
    int off = 0, nu = 0;
    for (int w = 0; w < NW; ++w) {
        if (w < warp) off += s_wcnt[w];
        nu += s_wcnt[w];
    }
    if (nu > kUnionCap) {  // full list larger than the gather area: two-pass kernel
        if (tid == 0) list_exact_row(a, row);
        return;
    }
    for (int i = lane; i < wcount; i += 32) {
        ukey[off + i] = wkey[i];
        uid[off + i] = wid[i];
    }
    __syncthreads();
    if (warp != 0) return;

    /* ---- warp 0: the row's finish ---- */
    int n = nu;
    bool trunc = s_trunc != 0 || s_tsh != 0ull;
    uint32_t t_last = 0u;
    if (MODE == kTopK && (n > a.kprime || trunc)) {
        /* Every excluded element must rank below the K'-th kept one: the
         * shared filter guarantees it; a warp's own cut does when the K'-th
         * kept key beats that warp's final threshold. */
        unsigned long long worst = 0ull;
        for (int w = 0; w < NW; ++w) worst = max(worst, s_taus[w]);
        const unsigned long long T =
            n < a.kprime ? 0ull
                         : (a.kprime < 128 ? warp_topk_sorted_r<4>(ukey, uid, n, a.kprime, nullptr, 1)
                                           : warp_topk_sorted_r<8>(ukey, uid, n, a.kprime, nullptr, 1));
        if (n < a.kprime || !(T > worst)) {
            if (lane == 0) list_exact_row(a, row);
            return;
        }
        t_last = (uint32_t)(T >> 32);
        n = a.kprime;
        trunc = true;
    }
    float M = Mfull;
    if (MODE == kTopK) {
        uint32_t mk = 0u;
        if (trunc) mk = ukey[0];  // the kept entries are sorted: [0] is the row max
        else
            for (int i = lane; i < n; i += 32) mk = max(mk, ukey[i]);
        mk = warp_max_u(mk);
        M = (s_l0nan || n == 0) ? __uint_as_float(0x7FC00000u) : key_float(mk);
    }
    int P = 1;
    while (P < n) P <<= 1;
    int ncand = 0;
    for (int b0 = 0; b0 < P; b0 += 32) {
        const int i = b0 + lane;
        uint64_t kv = 0ull;
        bool cand = false;
        if (i < n) {
            const int q = i;
            const float d = scaled_diff(key_float(ukey[q]), M, a.inv_t);
            if (d > -15.0f) {
                kv = ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - uid[q]);
                cand = true;
            }
        }
        if (i < P) sk[i] = kv;
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
                bad |= (i + 1 < ncand) && ((uint32_t)(sk[i] >> 32) == (uint32_t)(sk[i + 1] >> 32));
            }
            sorted = !__any_sync(kFull, bad);
        }
        if (!sorted) {
            warp_bitonic_desc(sk, P);
        }
    }

    bool more = false, exact = true;
    if (MODE == kTopK && trunc && ncand == n) {
        more = true;  // every kept entry is a candidate: the row has more
        const float dl = scaled_diff(key_float(t_last), M, a.inv_t);
        const float v_last = dl > -15.0f ? ref_weight(dl, a.et) : 0.0f;
        const float v_k = __uint_as_float((uint32_t)(sk[a.top_k - 1] >> 32));
        exact = v_last < v_k;
    }
    if (!exact) {
        if (lane == 0) list_exact_row(a, row);
        return;
    }
    const bool fb = ncand == 0;
    int nfin = 0;
    float mass = 0.0f;
    if (lane == 0) {
        uint64_t st[2] = {a.rng[2 * (size_t)row], a.rng[2 * (size_t)row + 1]};
        auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float((uint32_t)(sk[i] >> 32)); };
        const TailOut t = run_tail(fb ? 1 : ncand, more, a.top_k, a.top_p, st, w);
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
                    id = (int)(0xFFFFFFFFu - (uint32_t)sk[i]);
                    p = __uint_as_float((uint32_t)(sk[i] >> 32));
                    if (!a.list_weights) p = __fdiv_rn(p, mass);
                }
            }
            a.list_ids[(size_t)row * a.list_len + i] = id;
            if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = p;
        }
    }
}

}  // namespace noel
