/*
 * The pipeline's sibling sampler on the GPU: the reference's
 * aether_postreq_apply_penalties, aether_postreq_grammar_mask and
 * aether_postreq_sample (Sain-Kai/noel src/pipeline_stages.c:64-189), one
 * CTA per row, each row modified in place as the reference modifies its
 * buffer.
 *
 * aether_postreq_sample (pipeline_stages.c:103-189), per row:
 *   greedy (T <= 1e-4)   the first strictly largest logit (NaN at id 0: 0);
 *                        the row is left as it is;
 *   otherwise            s = x * (1 / T); m = the first strictly largest s
 *                        (NaN if s[0] is); e = expf(s - m); sum = e summed in
 *                        id order in fp32 (one lane adds every element, in
 *                        order, from shared-memory tiles the block fills
 *                        ahead of it); p = e * (1 / sum) (0 when sum is not
 *                        > 0), written back over the row; the top
 *                        min(top_k, 256) of p by (p desc, id asc) (top_k <= 0
 *                        or > V: V), found by a block radix select on p's
 *                        bits and sorted; the first of them whose running sum
 *                        reaches top_p; renormalised by 1 / that sum; and the
 *                        draw: the first whose renormalised running sum
 *                        reaches the row's uniform r (the last otherwise; -1
 *                        when no probability is a number).
 *
 * expf is CUDA's single-precision expf (within 2 units in the last place of
 * the C library's): probabilities within 1e-5 relative of the reference's,
 * token ids equal except where a probability or the uniform lies within that
 * rounding of a top-k, top-p or draw boundary.
 */
#pragma once

#include "sampler_kernels.cuh"
#include "sampler_warp.cuh"

namespace noel {

constexpr int kPostThreads = 128;              // small CTAs: more rows (and sum chains) per SM
constexpr int kPostTile = 2048;                // elements per summed tile
constexpr int kPostMaxK = 256;                // pipeline_stages.c:148
constexpr int kPostBins = 2048;               // radix select: 11 bits per level
constexpr int kPostU = 8;                     // elements a thread loads before using them

struct PostArgs {
    float *logits;        // [B][ld] fp32, modified in place
    int64_t ld;
    int batch, vocab;
    float temperature, top_p;
    int top_k;
    const float *uniform;  // [B]: rand() / RAND_MAX per row
    int32_t *ids;          // [B]
    ExpTable et;
};

/* CUDA's single-precision expf: within 2 units in the last place of the C
 * library's, so probabilities stay within 1e-5 relative of the reference's
 * (the double-precision path the sampler uses for its bit-exact draw would
 * put 2V fp64 exponentials per row on B200's narrow fp64 pipe) */
__device__ __forceinline__ float post_expf(float d, const ExpTable &) { return expf(d); }

/* order-preserving key of a probability (0 for NaN: never selected) */
__device__ __forceinline__ uint32_t post_key(float p) { return p == p ? ord_key(p) : 0u; }

template <int NT>
__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t *s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t q = __shfl_xor_sync(kFull, v, o);
        v = q > v ? q : v;
    }
    __syncthreads();
    if (lane == 0) s[warp] = v;
    __syncthreads();
    uint64_t r = 0ull;
    for (int w = 0; w < NT / 32; ++w) r = s[w] > r ? s[w] : r;
    __syncthreads();
    return r;
}

template <int NT>
__device__ __forceinline__ int post_block_sum(int v, int *s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    __syncthreads();
    if (lane == 0) s[warp] = v;
    __syncthreads();
    int r = 0;
    for (int w = 0; w < NT / 32; ++w) r += s[w];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kPostThreads) postreq_sample_kernel(const __grid_constant__ PostArgs a) {
    constexpr int NT = kPostThreads, NW = NT / 32;
    __shared__ __align__(16) float tile[2][kPostTile];
    __shared__ uint32_t hist[kPostBins];
    __shared__ uint64_t cand[kPostMaxK];
    __shared__ uint64_t s_u64[NW];
    __shared__ int s_int[NW];
    __shared__ float s_sum;
    __shared__ int s_bin, s_above, s_ncand, s_eq;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row = blockIdx.x, V = a.vocab;
    float *x = a.logits + (size_t)row * (size_t)a.ld;

    if (a.temperature <= 1e-4f) {  // pipeline_stages.c:105-115
        uint64_t best = 0ull;
        for (int v = tid; v < V; v += NT) {
            const float xv = x[v];
            if (xv == xv) {
                const uint64_t k = comp_key(ord_key(xv), (uint32_t)v);
                best = k > best ? k : best;
            }
        }
        best = block_max_u64<NT>(best, s_u64);
        if (tid == 0) {
            const float x0 = x[0];
            a.ids[row] = (x0 != x0 || best == 0ull) ? 0 : (int)(0xFFFFFFFFu - (uint32_t)best);
        }
        return;
    }

    /* s = x * inv_temp and its first strict maximum (pipeline_stages.c:118-127) */
    const float inv_t = __fdiv_rn(1.0f, a.temperature);
    /* every pass over the row loads kPostU elements per thread before
     * using them, so their latencies overlap */
    auto load_u = [&](int base, float (&xv)[kPostU]) {
#pragma unroll
        for (int u = 0; u < kPostU; ++u) {
            const int v = base + u * NT + tid;
            xv[u] = v < V ? x[v] : 0.0f;
        }
    };
    uint64_t mk = 0ull;
    for (int base = 0; base < V; base += NT * kPostU) {
        float xv[kPostU];
        load_u(base, xv);
#pragma unroll
        for (int u = 0; u < kPostU; ++u) {
            const float s = __fmul_rn(xv[u], inv_t);
            if (base + u * NT + tid < V && s == s) {
                const uint32_t k = ord_key(s);
                mk = (uint64_t)k > mk ? (uint64_t)k : mk;
            }
        }
    }
    mk = block_max_u64<NT>(mk, s_u64);
    const float s0 = __fmul_rn(x[0], inv_t);
    const float m = s0 != s0 ? s0 : (mk ? key_float((uint32_t)mk) : -INFINITY);

    /* e = expf(s - m), summed in id order (pipeline_stages.c:128-132): the
     * block fills tile t + 1 while lane 0 of warp 0 adds tile t */
    /* tile t's e values by threads [t0, t0 + nt) of the block */
    auto fill = [&](int t, float *dst, int t0, int nt) {
        const int base = t * kPostTile;
        for (int i0 = threadIdx.x - t0; i0 < kPostTile; i0 += nt * kPostU) {
            float xv[kPostU];
#pragma unroll
            for (int u = 0; u < kPostU; ++u) {
                const int i = i0 + u * nt, v = base + i;
                xv[u] = i < kPostTile && v < V ? x[v] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kPostU; ++u) {
                const int i = i0 + u * nt, v = base + i;
                if (i < kPostTile) dst[i] = v < V ? post_expf(__fsub_rn(__fmul_rn(xv[u], inv_t), m), a.et) : 0.0f;
            }
        }
    };
    const int ntile = (V + kPostTile - 1) / kPostTile;
    float sum = 0.0f;  // lane 0 of warp 0
    fill(0, tile[0], 0, NT);
    __syncthreads();
    for (int t = 0; t < ntile; ++t) {
        if (warp == 0) {
            if (lane == 0) {
                const float *src = tile[t & 1];
                const int n = min(kPostTile, V - t * kPostTile);
                int i = 0;
                if (n >= 8) {
                    /* the next eight values load while the current eight add */
                    float4 q0 = *reinterpret_cast<const float4 *>(src);
                    float4 q1 = *reinterpret_cast<const float4 *>(src + 4);
                    for (; i + 8 <= n; i += 8) {
                        float4 n0 = q0, n1 = q1;
                        if (i + 16 <= n) {
                            n0 = *reinterpret_cast<const float4 *>(src + i + 8);
                            n1 = *reinterpret_cast<const float4 *>(src + i + 12);
                        }
                        sum = __fadd_rn(sum, q0.x);
                        sum = __fadd_rn(sum, q0.y);
                        sum = __fadd_rn(sum, q0.z);
                        sum = __fadd_rn(sum, q0.w);
                        sum = __fadd_rn(sum, q1.x);
                        sum = __fadd_rn(sum, q1.y);
                        sum = __fadd_rn(sum, q1.z);
                        sum = __fadd_rn(sum, q1.w);
                        q0 = n0;
                        q1 = n1;
                    }
                }
                for (; i < n; ++i) sum = __fadd_rn(sum, src[i]);
            }
            __syncwarp();
        } else if (t + 1 < ntile) {
            fill(t + 1, tile[(t + 1) & 1], 32, NT - 32);  // warps 1.. fill the next tile (warp 0 is adding)
        }
        __syncthreads();
    }
    if (tid == 0) s_sum = sum;
    __syncthreads();
    sum = s_sum;
    const float inv_sum = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;

    /* p = e * inv_sum written over the row (pipeline_stages.c:133-136); the
     * first radix level counts its top 11 key bits */
    for (int i = tid; i < kPostBins; i += NT) hist[i] = 0u;
    __syncthreads();
    /* histogram adds: lanes of a warp with the same bin add once (most
     * probabilities of a row share their top bits) */
    auto hist_add = [&](bool ok, uint32_t bin) {
        const uint32_t peers = __match_any_sync(kFull, ok ? bin : 0xFFFFFFFFu);
        if (ok && (peers & lanemask_lt()) == 0u) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
    };
    for (int base = 0; base < V; base += NT * kPostU) {
        float xv[kPostU];
        load_u(base, xv);
#pragma unroll
        for (int u = 0; u < kPostU; ++u) {
            const int v = base + u * NT + tid;
            uint32_t k = 0u;
            if (v < V) {
                const float p = __fmul_rn(post_expf(__fsub_rn(__fmul_rn(xv[u], inv_t), m), a.et), inv_sum);
                x[v] = p;
                k = post_key(p);
            }
            hist_add(k != 0u, k >> 21);
        }
    }
    __syncthreads();

    /* the K-th largest key T by levels of 11, 11 and 10 bits: keys above the
     * chosen bin are taken whole; a bin holding just the keys still needed
     * ends the search (pipeline_stages.c:138-158, by (p desc, id asc)) */
    int K = a.top_k;
    if (K <= 0 || K > V) K = V;
    if (K > kPostMaxK) K = kPostMaxK;
    uint32_t prefix = 0u;  // bits fixed so far
    int shift = 21, above = 0, need = K;
    bool whole = true;     // take every key at or above prefix << shift
    const int total = (int)post_block_sum<NT>([&] {
        int c = 0;
        for (int i = tid; i < kPostBins; i += NT) c += (int)hist[i];
        return c;
    }(), s_int);
    if (total < need) need = total;
    for (int level = 0; need > 0; ++level) {
        if (level > 0) {
            /* histogram of the next bits of the keys matching the prefix */
            const int nb = shift == 0 ? 1024 : 2048;
            for (int i = tid; i < kPostBins; i += NT) hist[i] = 0u;
            __syncthreads();
            for (int base = 0; base < V; base += NT * kPostU) {
                float xv[kPostU];
                load_u(base, xv);
#pragma unroll
                for (int u = 0; u < kPostU; ++u) {
                    const uint32_t k = base + u * NT + tid < V ? post_key(xv[u]) : 0u;
                    hist_add(k && (k >> (shift + (shift == 0 ? 10 : 11))) == prefix, (k >> shift) & (nb - 1));
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            int acc = 0, b = (shift == 0 ? 1024 : 2048) - 1;
            for (; b >= 0; --b) {
                if (acc + (int)hist[b] >= need) break;
                acc += (int)hist[b];
            }
            s_bin = b;
            s_above = acc;
        }
        __syncthreads();
        const int b = s_bin, acc = s_above;
        above += acc;
        need -= acc;
        prefix = (prefix << (shift == 0 ? 10 : 11)) | (uint32_t)b;
        if ((int)hist[b] == need || shift == 0) {
            whole = (int)hist[b] == need;
            break;
        }
        shift = shift == 21 ? 10 : 0;
        __syncthreads();
    }
    /* collect: keys above the bin (their prefix beats it), and the bin's keys
     * -- all of them, or (a bin of equal keys) the lowest ids first */
    if (tid == 0) {
        s_ncand = 0;
        s_eq = 0;
    }
    __syncthreads();
    const int pbits = shift == 21 ? 11 : (shift == 10 ? 22 : 32);
    const int K2 = above + need;  // = min(K, numbers in the row)
    if (K2 > 0) {
        for (int base = 0; base < V; base += NT * kPostU) {
            float xv[kPostU];
            load_u(base, xv);
#pragma unroll
            for (int u = 0; u < kPostU; ++u) {
                const int v = base + u * NT + tid;
                const uint32_t k = v < V ? post_key(xv[u]) : 0u;
                if (!k) continue;
                const uint32_t kp = pbits == 32 ? k : (k >> (32 - pbits));
                if (kp > prefix || (whole && kp == prefix)) cand[atomicAdd(&s_ncand, 1)] = comp_key(k, (uint32_t)v);
            }
        }
        __syncthreads();
        if (!whole) {
            /* the first `need` elements equal to the full key, in id order */
            for (int base = 0; base < V; base += NT) {
                const int v = base + tid;
                const bool eq = v < V && post_key(x[v]) == prefix;
                const uint32_t bal = __ballot_sync(kFull, eq);
                if (lane == 0) s_int[warp] = __popc(bal);
                __syncthreads();
                int before = 0, tot = 0;
                for (int w = 0; w < NW; ++w) {
                    before += w < warp ? s_int[w] : 0;
                    tot += s_int[w];
                }
                const int pos = s_eq + before + __popc(bal & lanemask_lt());
                if (eq && pos < need) cand[above + pos] = comp_key(prefix, (uint32_t)v);
                __syncthreads();
                if (tid == 0) s_eq += tot;
                __syncthreads();
                if (s_eq >= need) break;
            }
        }
    }
    __syncthreads();
    /* sort the K2 candidates by (p desc, id asc) */
    int P = 1;
    while (P < K2) P <<= 1;
    for (int i = K2 + tid; i < P; i += NT) cand[i] = 0ull;
    __syncthreads();
    for (int kk = 2; kk <= P; kk <<= 1)
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P; i += NT) {
                const int l = i ^ j;
                if (l > i) {
                    const bool desc = (i & kk) == 0;
                    const uint64_t u = cand[i], w = cand[l];
                    if (desc ? (u < w) : (u > w)) {
                        cand[i] = w;
                        cand[l] = u;
                    }
                }
            }
            __syncthreads();
        }

    /* top-p, renormalisation and the draw (pipeline_stages.c:160-189) */
    if (tid == 0) {
        float cum = 0.0f;
        int n = 0;
        for (int i = 0; i < K2; ++i) {
            cum = __fadd_rn(cum, key_float((uint32_t)(cand[i] >> 32)));
            ++n;
            if (cum >= a.top_p) break;
        }
        const float inv_cum = __fdiv_rn(1.0f, cum);
        const float r = a.uniform[row];
        float run = 0.0f;
        int id = K2 > 0 ? (int)(0xFFFFFFFFu - (uint32_t)cand[0]) : -1;
        for (int i = 0; i < n; ++i) {
            run = __fadd_rn(run, __fmul_rn(key_float((uint32_t)(cand[i] >> 32)), inv_cum));
            if (r <= run || i == n - 1) {
                id = (int)(0xFFFFFFFFu - (uint32_t)cand[i]);
                break;
            }
        }
        a.ids[row] = id;
    }
}

/* aether_postreq_apply_penalties (pipeline_stages.c:64-79) on row blockIdx.x:
 * each distinct history id of the window gets its penalty once per
 * occurrence (a shared (id, count) table; repeating the same operation on
 * one element is what the reference's per-occurrence loop does). */
__global__ void __launch_bounds__(kPostThreads) postreq_penalty_kernel(float *logits, int64_t ld, int V,
                                                                      const int32_t *hist, int64_t hld, int H,
                                                                      int start, float pen, int cap) {
    extern __shared__ uint32_t ptab[];  // keys [cap] (id + 1), counts [cap]
    uint32_t *key = ptab, *cnt = ptab + cap;
    const int row = blockIdx.x;
    for (int i = threadIdx.x; i < 2 * cap; i += blockDim.x) ptab[i] = 0u;
    __syncthreads();
    const int32_t *h = hist + (size_t)row * (size_t)hld;
    const int bits = __ffs(cap) - 1;
    for (int i = start + threadIdx.x; i < H; i += blockDim.x) {
        const int t = h[i];
        if (t < 0 || t >= V) continue;  // pipeline_stages.c:72
        uint32_t p = hs_hash((uint32_t)t) >> (32 - bits);
        for (int probe = 0; probe < cap; ++probe) {
            const uint32_t prev = atomicCAS(&key[p], 0u, (uint32_t)t + 1u);
            if (prev == 0u || prev == (uint32_t)t + 1u) {
                atomicAdd(&cnt[p], 1u);
                break;
            }
            p = (p + 1) & (uint32_t)(cap - 1);
        }
    }
    __syncthreads();
    float *x = logits + (size_t)row * (size_t)ld;
    for (int s = threadIdx.x; s < cap; s += blockDim.x)
        if (key[s]) x[key[s] - 1] = apply_penalty(x[key[s] - 1], cnt[s], pen);
}

/* aether_postreq_grammar_mask (pipeline_stages.c:81-94): rows whose state is
 * 0 keep only '{' (id 123); every other id becomes -1e9 */
__global__ void postreq_grammar_kernel(float *logits, int64_t ld, int B, int V, const int32_t *state, int state0) {
    const size_t n = (size_t)B * (size_t)V;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int b = (int)(i / (size_t)V), v = (int)(i % (size_t)V);
        const int st = state ? state[b] : state0;
        if (st == 0 && v != '{') logits[(size_t)b * (size_t)ld + v] = -1e9f;
    }
}

}  // namespace noel
