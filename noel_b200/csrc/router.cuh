/*
 * MoE top-k router for a batch of tokens: the reference's
 * aether_route_top_k (Sain-Kai/noel src/sparsity.c:46-79), one warp per
 * token.
 *
 * Selection (sparsity.c:47-65): the reference inserts each expert in id
 * order into a list of top_k slots initialised to (-1, -1e9) and moves an
 * entry down only for a strictly larger value, so the list holds the top_k
 * values strictly above -1e9 by (value desc, id asc) -- NaN never enters --
 * followed by (-1, -1e9) slots.  Each lane holds its experts' composite keys
 * (ord_key(value), ~id) in registers and the warp takes the largest top_k
 * times.
 *
 * Up to 16 slots, one thread per token (moe_route_thread_kernel) keeps the
 * reference's sorted slots in registers and inserts each expert where the
 * reference does (after every slot it does not strictly beat); an expert that
 * does not beat the last slot costs one comparison.
 *
 * Weights (sparsity.c:67-78): expf(w - max) with max the first slot's value,
 * summed in slot order in fp32, times 1/sum (0 when the sum is not > 0).
 * expf is CUDA's single-precision expf, within 2 units in the last place of
 * the C library's.
 */
#pragma once

#include "sampler_device.cuh"

namespace noel {

constexpr int kRouterMaxExperts = 256;  // 8 per lane
constexpr int kRouterMaxTopK = 64;
constexpr int kRouterWarps = 4;

struct RouterArgs {
    const float *logits;  // [tokens][ld]
    int64_t ld;
    int tokens, experts, top_k;
    uint2 *out;           // [tokens][top_k] (expert id, weight bits)
    ExpTable et;
};

/* CUDA's single-precision expf: within 2 units in the last place of the C
 * library's (weights within 1e-5 relative) at a fraction of the cost of the
 * sampler's bit-exact double-precision path on B200's fp64 pipe */
__device__ __forceinline__ float router_expf(float d, const ExpTable &) { return expf(d); }

constexpr int kRouterThreads = 128;

/* One token per thread: slots w / id sorted by (value desc, id asc), the
 * reference's insertion (sparsity.c:53-65) unrolled over KMAX registers. */
template <int KMAX>
__global__ void __launch_bounds__(kRouterThreads) moe_route_thread_kernel(const __grid_constant__ RouterArgs a) {
    const int t = blockIdx.x * kRouterThreads + threadIdx.x;
    if (t >= a.tokens) return;
    const float *x = a.logits + (size_t)t * (size_t)a.ld;
    float w[KMAX];
    int32_t id[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        w[k] = -1e9f;
        id[k] = -1;
    }
    auto insert = [&](float v, int e) {
        if (!(v > w[a.top_k - 1])) return;  // the common case once the slots fill (NaN never enters)
#pragma unroll
        for (int k = KMAX - 1; k >= 0; --k) {
            if (k >= a.top_k) continue;
            if (k > 0 && v > w[k - 1]) {  // slot k takes the entry above (v goes higher)
                w[k] = w[k - 1];
                id[k] = id[k - 1];
            } else if (v > w[k]) {  // the first slot v strictly beats
                w[k] = v;
                id[k] = e;
            }
        }
    };
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (a.experts % 4 == 0);
    if (vec) {
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (int e4 = 0; e4 < a.experts / 4; e4 += 4) {
            float4 q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (e4 + u < a.experts / 4) q[u] = __ldg(x4 + e4 + u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (e4 + u >= a.experts / 4) break;
                const int e = 4 * (e4 + u);
                insert(q[u].x, e);
                insert(q[u].y, e + 1);
                insert(q[u].z, e + 2);
                insert(q[u].w, e + 3);
            }
        }
    } else {
        for (int e = 0; e < a.experts; ++e) insert(__ldg(x + e), e);
    }
    /* sparsity.c:67-78, in slot order */
    const float mx = w[0];
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        if (k >= a.top_k) break;
        w[k] = router_expf(__fsub_rn(w[k], mx), a.et);
        sum = __fadd_rn(sum, w[k]);
    }
    const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
    uint2 *o = a.out + (size_t)t * a.top_k;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        if (k >= a.top_k) break;
        o[k] = make_uint2((uint32_t)id[k], __float_as_uint(__fmul_rn(w[k], inv)));
    }
}

__global__ void __launch_bounds__(32 * kRouterWarps) moe_route_kernel(const __grid_constant__ RouterArgs a) {
    constexpr int R = kRouterMaxExperts / 32;
    __shared__ uint2 sel[kRouterWarps][kRouterMaxTopK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x * kRouterWarps + warp;
    if (t >= a.tokens) return;  // whole warps; no block barrier below
    const float *x = a.logits + (size_t)t * (size_t)a.ld;
    uint64_t k[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int e = r * 32 + lane;
        k[r] = 0ull;
        if (e < a.experts) {
            const float v = x[e];
            if (v > -1e9f) k[r] = comp_key(ord_key(v), (uint32_t)e);  // sparsity.c:58 (NaN fails)
        }
    }
    /* the top_k largest composite keys, in order */
    for (int s = 0; s < a.top_k; ++s) {
        uint64_t m = 0ull;
#pragma unroll
        for (int r = 0; r < R; ++r) m = k[r] > m ? k[r] : m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t q = __shfl_xor_sync(kFull, m, o);
            m = q > m ? q : m;
        }
        if (m) {
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (k[r] == m) k[r] = 0ull;  // composite keys are unique: one lane holds it
        }
        if (lane == 0)
            sel[warp][s] = m ? make_uint2(0xFFFFFFFFu - (uint32_t)m, __float_as_uint(key_float((uint32_t)(m >> 32))))
                             : make_uint2(0xFFFFFFFFu, __float_as_uint(-1e9f));
    }
    __syncwarp();
    if (lane == 0) {
        /* sparsity.c:67-78, in slot order */
        const float mx = __uint_as_float(sel[warp][0].y);
        float sum = 0.0f;
        for (int s = 0; s < a.top_k; ++s) {
            const float w = router_expf(__fsub_rn(__uint_as_float(sel[warp][s].y), mx), a.et);
            sel[warp][s].y = __float_as_uint(w);
            sum = __fadd_rn(sum, w);
        }
        const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
        for (int s = 0; s < a.top_k; ++s)
            sel[warp][s].y = __float_as_uint(__fmul_rn(__uint_as_float(sel[warp][s].y), inv));
    }
    __syncwarp();
    for (int s = lane; s < a.top_k; s += 32) a.out[(size_t)t * a.top_k + s] = sel[warp][s];
}

}  // namespace noel
