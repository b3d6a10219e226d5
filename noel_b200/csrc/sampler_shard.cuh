/*
 * Merge of a vocab-sharded row (the full vocabulary split into column ranges
 * across GPUs, one range per rank in ascending order).
 *
 * Each shard contributes, per row, a list of L entries (global id, penalised
 * logit) by (logit desc, id asc), then a trailer (its largest penalised logit,
 * flags: NaN at global id 0; more elements than listed).
 *
 * Greedy and top-k (k + 8 = L): the union of the shards' best L holds the
 * row's best L (an element of the row's best is beaten only by elements of
 * the row's best, so at most L - 1 elements of its own shard beat it).  From
 * there the merge is the row end of the single-pass kernel: the row's maximum
 * (sampler.c:119-124; a NaN at id 0 makes it NaN), the weights of the -15 cut
 * (sampler.c:132-143), the (weight desc, id asc) order of the stable sort
 * (sampler.c:152), and the top-k / top-p / draw loops (sampler.c:155-191).  A
 * row whose top-k boundary ties with weights outside the gathered entries is
 * not decided here.
 *
 * Full list (top-k off, or above 120): each shard lists its elements within
 * the -15 cut under its own maximum, which holds all of its elements within
 * the cut under the row's maximum.  A shard that had more than L lists its
 * best L; the row is decided here when the smallest of them (and so every
 * element it left out) falls outside the row's cut, and then the merge sees
 * every candidate of the row.
 *
 * A row not decided here keeps its RNG state, its status is set, and the
 * caller samples it from the full row.
 */
#pragma once

#include "sampler_device.cuh"

namespace noel {

struct MergeArgs {
    int n_shards, batch, len;  // lists of len entries + 1 trailer, [n_shards][batch]
    int full;                  // full-list config: every candidate is gathered
    const uint2 *lists;
    int greedy;                // temperature <= 1e-4 (sampler.c:106)
    float inv_t, top_p;
    int top_k;
    uint64_t *rng;
    int32_t *ids;
    float *probs;          // optional
    int32_t *status;       // [batch] 0 decided here, 1 sample from the full row
    int32_t *list_ids;     // optional [batch][list_len]: the drawn-from list
    float *list_probs;
    int list_len, list_weights;
    int32_t *stats;        // optional [batch][4] (noel_sampler_cuda.h)
    ExpTable et;
};

constexpr int kMergeWarps = 4;
constexpr int kShardFullLen = 256;  // entries per row and shard of a full-list config

__host__ __device__ inline int merge_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}
/* shared memory of one warp: keys and ids of the union, then the sort keys
 * (the running sums reuse the union's keys) */
__host__ __device__ inline size_t merge_warp_bytes(int n_shards, int len) {
    return (size_t)n_shards * len * 8 + (size_t)merge_pow2(n_shards * len) * 8;
}

/* The tail of a merged row over sk[0, ncand) sorted by (weight desc, id
 * asc): sampler.c:145-191, the row's RNG step, outputs and lists. */
__device__ __noinline__ void merge_tail(const MergeArgs &a, int row, const uint64_t *sk, int ncand, bool more_c,
                                        float *sums) {
    const int lane = threadIdx.x & 31;
    const bool fb = ncand == 0;  // sampler.c:145-149
    int nfin = 0;
    float mass = 0.0f;
    uint64_t st[2] = {0ull, 0ull};
    if (lane == 0) {
        st[0] = a.rng[2 * (size_t)row];
        st[1] = a.rng[2 * (size_t)row + 1];
    }
    auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float((uint32_t)(sk[i] >> 32)); };
    const TailOut t = warp_tail(fb ? 1 : ncand, more_c, a.top_k, a.top_p, st, w, sums);
    if (lane == 0) {
        a.rng[2 * (size_t)row] = st[0];
        a.rng[2 * (size_t)row + 1] = st[1];
        a.ids[row] = fb ? 0 : (int)(0xFFFFFFFFu - (uint32_t)sk[t.pos]);
        if (a.probs) a.probs[row] = __fdiv_rn(w(t.pos), t.mass);
        a.status[row] = 0;
        if (a.stats)
            reinterpret_cast<int4 *>(a.stats)[row] =
                make_int4(more_c ? -1 : (fb ? 1 : ncand), t.n_topk, t.n_final, fb ? NOEL_ROW_FALLBACK : 0);
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

__global__ void __launch_bounds__(32 * kMergeWarps) shard_merge_kernel(const __grid_constant__ MergeArgs a) {
    extern __shared__ __align__(16) unsigned char msmem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * kMergeWarps + warp;
    if (row >= a.batch) return;  // whole warps; the kernel has no block barrier
    const int K = a.len, cap = a.n_shards * K;
    unsigned char *base = msmem + (size_t)warp * merge_warp_bytes(a.n_shards, K);
    uint32_t *ukey = reinterpret_cast<uint32_t *>(base);
    uint32_t *uid = ukey + cap;
    uint64_t *sk = reinterpret_cast<uint64_t *>(uid + cap);
    auto list = [&](int s) -> const uint2 * {
        return a.lists + ((size_t)s * a.batch + (size_t)row) * (size_t)(K + 1);
    };

    /* the shards' maxima and flags */
    bool more = false, nan0 = false;
    float mx = -INFINITY;
    for (int s = 0; s < a.n_shards; ++s) {
        const uint2 tr = list(s)[K];
        more |= (tr.y & kShardMore) != 0;
        if (s == 0) nan0 = (tr.y & kShardNaN0) != 0;
        mx = fmaxf(mx, __uint_as_float(tr.x));
    }
    const float M = nan0 ? __uint_as_float(0x7FC00000u) : mx;

    if (a.full && !a.greedy) {
        /* every candidate: decided when no shard left out an element within
         * the row's cut (its smallest listed one falls outside it) */
        bool undecided = false;
        for (int s = lane; s < a.n_shards; s += 32) {
            const uint2 tr = list(s)[K];
            if (tr.y & kShardMore) {
                const uint2 last = list(s)[K - 1];
                undecided |= scaled_diff(__uint_as_float(last.y), M, a.inv_t) > -15.0f;
            }
        }
        if (__any_sync(kFull, undecided)) {
            if (lane == 0) a.status[row] = 1;
            return;
        }
        int n = 0;
        for (int s = 0; s < a.n_shards; ++s) {
            const uint2 *e = list(s);
            for (int j0 = 0; j0 < K; j0 += 32) {
                const int j = j0 + lane;
                const uint2 v = j < K ? e[j] : make_uint2(0xFFFFFFFFu, 0u);
                float d = -INFINITY;
                if (v.x != 0xFFFFFFFFu) d = scaled_diff(__uint_as_float(v.y), M, a.inv_t);
                const bool ok = v.x != 0xFFFFFFFFu && d > -15.0f;
                const uint32_t bal = __ballot_sync(kFull, ok);
                if (ok) sk[n + __popc(bal & lanemask_lt())] =
                            ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - v.x);
                n += __popc(bal);
            }
        }
        const int P = merge_pow2(max(n, 1));
        for (int i = n + lane; i < P; i += 32) sk[i] = 0ull;
        __syncwarp();
        if (n > 1) warp_bitonic_desc(sk, P);
        __syncwarp();
        merge_tail(a, row, sk, n, false, reinterpret_cast<float *>(ukey));
        return;
    }

    /* A shard that listed K entries has K elements at or above its K-th, so
     * the row's K-th best is at least the largest such K-th entry: entries
     * below that floor cannot make the row's K best and are not gathered. */
    uint64_t floor_key = 0ull;
    for (int s = lane; s < a.n_shards; s += 32) {
        const uint2 v = list(s)[K - 1];
        if (v.x != 0xFFFFFFFFu) floor_key = max(floor_key, comp_key(ord_key(__uint_as_float(v.y)), v.x));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) floor_key = max(floor_key, __shfl_xor_sync(kFull, floor_key, o));

    /* gather the shards' lists */
    int n = 0;
    bool dropped = false;
    for (int s = 0; s < a.n_shards; ++s) {
        const uint2 *e = list(s);
        for (int j0 = 0; j0 < K; j0 += 32) {
            const int j = j0 + lane;
            const uint2 v = j < K ? e[j] : make_uint2(0xFFFFFFFFu, 0u);
            const bool listed = v.x != 0xFFFFFFFFu;
            const bool ok = listed && comp_key(ord_key(__uint_as_float(v.y)), v.x) >= floor_key;
            dropped |= listed && !ok;
            const uint32_t bal = __ballot_sync(kFull, ok);
            if (ok) {
                const int p = n + __popc(bal & lanemask_lt());
                ukey[p] = ord_key(__uint_as_float(v.y));
                uid[p] = v.x;
            }
            n += __popc(bal);
        }
    }
    __syncwarp();

    if (a.greedy) {
        /* sampler.c:106-116: the lowest id of the largest value; 0 when id 0
         * is NaN (nothing compares greater) or the row holds no number */
        uint64_t best = 0ull;
        for (int i = lane; i < n; i += 32) best = max(best, comp_key(ukey[i], uid[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(kFull, best, o));
        const int id = (nan0 || n == 0) ? 0 : (int)(0xFFFFFFFFu - (uint32_t)best);
        if (lane == 0) {
            a.ids[row] = id;
            if (a.probs) a.probs[row] = 1.0f;
            a.status[row] = 0;
            if (a.stats) reinterpret_cast<int4 *>(a.stats)[row] = make_int4(1, 1, 1, NOEL_ROW_GREEDY);
        }
        if (a.list_ids)
            for (int i = lane; i < a.list_len; i += 32) {
                a.list_ids[(size_t)row * a.list_len + i] = i == 0 ? id : -1;
                if (a.list_probs) a.list_probs[(size_t)row * a.list_len + i] = i == 0 ? 1.0f : 0.0f;
            }
        return;
    }

    /* the row's K best by (logit desc, id asc), sorted */
    const unsigned long long T = K <= 96 ? warp_topk_sorted_r<4>(ukey, uid, n, K, nullptr, 1)
                                         : warp_topk_sorted_r<8>(ukey, uid, n, K, nullptr, 1);
    const bool trunc = more || n > K || __any_sync(kFull, dropped);
    const int m = min(n, K);
    const int P = merge_pow2(max(m, 1));
    int ncand = 0;
    for (int b0 = 0; b0 < P; b0 += 32) {
        const int i = b0 + lane;
        uint64_t kv = 0ull;
        bool cand = false;
        if (i < m) {
            const float d = scaled_diff(key_float(ukey[i]), M, a.inv_t);
            if (d > -15.0f) {
                kv = ((uint64_t)__float_as_uint(ref_weight(d, a.et)) << 32) | (uint64_t)(0xFFFFFFFFu - uid[i]);
                cand = true;
            }
        }
        if (i < P) sk[i] = kv;
        ncand += __popc(__ballot_sync(kFull, cand));
    }
    __syncwarp();
    {
        /* logit order is weight order unless adjacent candidates tie on weight */
        bool bad = false;
        for (int b0 = 0; b0 + 1 < ncand; b0 += 32) {
            const int i = b0 + lane;
            bad |= (i + 1 < ncand) && ((uint32_t)(sk[i] >> 32) == (uint32_t)(sk[i + 1] >> 32));
        }
        if (__any_sync(kFull, bad)) warp_bitonic_desc(sk, P);
    }
    bool more_c = false, exact = true;
    if (trunc && m == K && ncand == K) {
        /* every kept entry is a candidate and the row has more: the k-th
         * weight must beat the weight of the smallest kept logit */
        more_c = true;
        const float dl = scaled_diff(key_float((uint32_t)(T >> 32)), M, a.inv_t);
        const float v_last = dl > -15.0f ? ref_weight(dl, a.et) : 0.0f;
        const float v_k = __uint_as_float((uint32_t)(sk[a.top_k - 1] >> 32));
        exact = v_last < v_k;
    }
    if (!exact) {
        if (lane == 0) a.status[row] = 1;
        return;
    }
    /* the running sums go where the gathered keys were (no longer read) */
    merge_tail(a, row, sk, ncand, more_c, reinterpret_cast<float *>(ukey));
}

}  // namespace noel
