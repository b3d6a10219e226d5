/*
 * Merge of a vocab-sharded row (the full vocabulary split into column ranges
 * across GPUs, one range per rank in ascending order).
 *
 * Each shard contributes, per row, its kprime best (global id, penalised
 * logit) by (logit desc, id asc), its largest penalised logit and two flags
 * (NaN at global id 0; more elements than listed).  The union of the shards'
 * kprime best holds the row's kprime best: an element of the row's best is
 * beaten only by elements of the row's best, so at most kprime - 1 elements of
 * its own shard beat it.  From there the merge is the row end of the
 * single-pass kernel: the row's maximum (sampler.c:119-124; a NaN at id 0
 * makes it NaN), the weights of the -15 cut (sampler.c:132-143), the
 * (weight desc, id asc) order of the stable sort (sampler.c:152), and the
 * top-k / top-p / draw loops (sampler.c:155-191).  A row whose top-k boundary
 * ties with weights outside the gathered entries is not decided here: its
 * status is set, its RNG state is left as it was, and the caller samples it
 * from the full row.
 */
#pragma once

#include "sampler_device.cuh"

namespace noel {

struct MergeArgs {
    int n_shards, batch, kprime;
    int es, eb;            // list (shard s, row b) is list s * es + b * eb
    const uint2 *entries;  // lists of kprime entries
    const float *maxes;    // one per list
    const int32_t *flags;  // one per list
    int greedy;            // temperature <= 1e-4 (sampler.c:106)
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

/* shared memory of one warp: keys and ids of the union, then the sort keys */
__host__ __device__ inline size_t merge_warp_bytes(int n_shards, int kprime) {
    int p = 1;
    while (p < kprime) p <<= 1;
    return (size_t)n_shards * kprime * 8 + (size_t)p * 8;
}

__global__ void __launch_bounds__(32 * kMergeWarps) shard_merge_kernel(const __grid_constant__ MergeArgs a) {
    extern __shared__ __align__(16) unsigned char msmem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * kMergeWarps + warp;
    if (row >= a.batch) return;  // whole warps; the kernel has no block barrier
    const int K = a.kprime, cap = a.n_shards * K;
    unsigned char *base = msmem + (size_t)warp * merge_warp_bytes(a.n_shards, K);
    uint32_t *ukey = reinterpret_cast<uint32_t *>(base);
    uint32_t *uid = ukey + cap;
    uint64_t *sk = reinterpret_cast<uint64_t *>(uid + cap);

    /* A shard that listed K entries has K elements at or above its K-th, so
     * the row's K-th best is at least the largest such K-th entry: entries
     * below that floor cannot make the row's K best and are not gathered. */
    uint64_t floor_key = 0ull;
    for (int s = lane; s < a.n_shards; s += 32) {
        const uint2 v = a.entries[((size_t)s * a.es + (size_t)row * a.eb) * K + (K - 1)];
        if (v.x != 0xFFFFFFFFu) floor_key = max(floor_key, comp_key(ord_key(__uint_as_float(v.y)), v.x));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) floor_key = max(floor_key, __shfl_xor_sync(kFull, floor_key, o));

    /* gather the shards' lists, maxima and flags */
    int n = 0;
    bool more = false, nan0 = false, dropped = false;
    float mx = -INFINITY;
    for (int s = 0; s < a.n_shards; ++s) {
        const size_t li = (size_t)s * a.es + (size_t)row * a.eb;
        const int fl = a.flags[li];
        more |= (fl & kShardMore) != 0;
        if (s == 0) nan0 = (fl & kShardNaN0) != 0;
        mx = fmaxf(mx, a.maxes[li]);
        const uint2 *e = a.entries + li * K;
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
    const unsigned long long T = K < 128 ? warp_topk_sorted_r<4>(ukey, uid, n, K, nullptr, 1)
                                         : warp_topk_sorted_r<8>(ukey, uid, n, K, nullptr, 1);
    const bool trunc = more || n > K || __any_sync(kFull, dropped);
    const int m = min(n, K);
    const float M = nan0 ? __uint_as_float(0x7FC00000u) : mx;
    int P = 1;
    while (P < m) P <<= 1;
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
    const bool fb = ncand == 0;  // sampler.c:145-149
    int nfin = 0;
    float mass = 0.0f;
    uint64_t st[2] = {0ull, 0ull};
    if (lane == 0) {
        st[0] = a.rng[2 * (size_t)row];
        st[1] = a.rng[2 * (size_t)row + 1];
    }
    auto w = [&](int i) -> float { return fb ? 1.0f : __uint_as_float((uint32_t)(sk[i] >> 32)); };
    /* the running sums go where the gathered keys were (no longer read) */
    const TailOut t = warp_tail(fb ? 1 : ncand, more_c, a.top_k, a.top_p, st, w, reinterpret_cast<float *>(ukey));
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

}  // namespace noel
