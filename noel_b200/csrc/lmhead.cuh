/*
 * The LM head feeding the sampler: logits y[b][r] = W[r] . x[b] for the
 * reference's unquantised row formats (F32, F16, BF16), the projection of
 * Sain-Kai/noel src/engine.c:377-384 through noel_gemv_quantized
 * (src/dequant.c:412-470), in its summation order so the logits equal the
 * reference's bit for bit: eight fused multiply-add accumulators over
 * blocks of eight columns, combined as ((a0 + a4) + (a1 + a5)) +
 * ((a2 + a6) + (a3 + a7)).  Columns must be a multiple of 8 (the reference's
 * scalar tail for other widths is left to its compiler's scheduling).
 *
 * A CTA owns 128 rows of W and up to eight tokens per pass; the rows stream
 * through a cp.async pipeline of shared-memory tiles (128 bytes of every
 * row per tile, so each warp load covers four rows x 128 contiguous bytes),
 * and each thread runs its row's eight accumulators in the reference's
 * order.  The row-major weights are read once per pass; the kernel is bound
 * by HBM.  The logits (B x V fp32) are written for
 * the sampler, which runs next on the same stream while they sit in L2.
 */
#pragma once

#include "sampler_device.cuh"

#include <cuda_fp16.h>

namespace noel {

constexpr int kHeadThreads = 128;
constexpr int kHeadTokens = 8;  // tokens per pass

enum HeadType { kHeadF32 = 0, kHeadF16 = 1, kHeadBF16 = 30 };  // the reference's GGML type ids

struct HeadArgs {
    const void *w;   // [rows][ldw]
    int64_t ldw;
    const float *x;  // [tokens][ldx]
    int64_t ldx;
    int rows, cols;
    float *y;        // [tokens][ldy]
    int64_t ldy;
};

/* eight consecutive elements of a row as floats (exact conversions) */
template <int WT>
__device__ __forceinline__ void head_block(const void *row, int j, float (&w)[8]) {
    if (WT == kHeadF32) {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(row) + j);
        const float4 a = p[0], b = p[1];
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else {
        const uint4 q = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(row) + j);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint16_t lo = (uint16_t)(u[e] & 0xFFFFu), hi = (uint16_t)(u[e] >> 16);
            if (WT == kHeadBF16) {
                w[2 * e] = __uint_as_float((uint32_t)lo << 16);
                w[2 * e + 1] = __uint_as_float((uint32_t)hi << 16);
            } else {
                w[2 * e] = __half2float(__ushort_as_half(lo));
                w[2 * e + 1] = __half2float(__ushort_as_half(hi));
            }
        }
    }
}

constexpr int kHeadRowBytes = 128;   // bytes of every row a tile holds (one cache line)
constexpr int kHeadPitch = kHeadRowBytes + 16;  // shared-memory row pitch: conflict-free 16-byte reads
constexpr int kHeadStages = 4;        // tiles in flight
constexpr int kHeadXMax = 8 * 64;     // hidden values per tile for up to eight tokens

__host__ __device__ constexpr size_t head_smem_bytes() {
    return (size_t)kHeadStages * (kHeadThreads * kHeadPitch + kHeadXMax * 4);
}

/* The CTA's 128 rows stream through shared memory in tiles of 128 bytes of
 * every row (64 columns of a 2-byte type, 32 of F32): each warp load covers
 * four rows x 128 contiguous bytes, kHeadStages tiles are in flight, and the
 * thread of each row then runs that row's eight accumulators over the tile
 * in the reference's order. */
template <int WT, int NB>
__global__ void __launch_bounds__(kHeadThreads) lmhead_gemv_kernel(const __grid_constant__ HeadArgs a) {
    extern __shared__ __align__(16) unsigned char head_smem[];
    constexpr int ES = WT == kHeadF32 ? 4 : 2;
    constexpr int TC = kHeadRowBytes / ES;  // columns per tile
    constexpr int CH = kHeadRowBytes / 16;  // 16-byte chunks per row and tile
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * kHeadThreads;
    const int r = r0 + tid;
    const int ntile = (a.cols + TC - 1) / TC;
    auto stage_w = [&](int st) { return head_smem + (size_t)st * (kHeadThreads * kHeadPitch + kHeadXMax * 4); };
    auto stage_x = [&](int st) { return reinterpret_cast<float *>(stage_w(st) + kHeadThreads * kHeadPitch); };
    /* issue tile t into stage t mod kHeadStages (one commit group per tile) */
    auto issue = [&](int t) {
        if (t < ntile) {
            unsigned char *sw = stage_w(t % kHeadStages);
            float *sx = stage_x(t % kHeadStages);
            const int c0 = t * TC;
            const int cn = min(TC, a.cols - c0);
            const int nch = cn * ES / 16;  // chunks present in this tile (cols are a multiple of 8)
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                const int q = i * kHeadThreads + tid;  // chunk q: row q / CH, chunk q % CH
                const int rr = q / CH, ch = q % CH;
                if (r0 + rr < a.rows && ch < nch)
                    cp_async16(sw + rr * kHeadPitch + ch * 16,
                               static_cast<const char *>(a.w) + ((size_t)(r0 + rr) * (size_t)a.ldw + c0) * ES + ch * 16);
            }
            for (int q = tid; q < NB * (cn / 4); q += kHeadThreads) {
                const int b = q / (cn / 4), c4 = q % (cn / 4);
                cp_async16(sx + b * TC + c4 * 4, a.x + (size_t)b * (size_t)a.ldx + c0 + c4 * 4);
            }
        }
        cp_async_commit();
    };
    float acc[NB][8];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[b][k] = 0.0f;
#pragma unroll
    for (int t = 0; t < kHeadStages - 1; ++t) issue(t);
    for (int t = 0; t < ntile; ++t) {
        cp_async_wait<kHeadStages - 2>();
        __syncthreads();  // tile t landed for every thread; tile t - 1's stage is free
        issue(t + kHeadStages - 1);
        if (r < a.rows) {
            const unsigned char *sw = stage_w(t % kHeadStages) + tid * kHeadPitch;
            const float *sx = stage_x(t % kHeadStages);
            const int cn = min(TC, a.cols - t * TC);
            for (int j = 0; j < cn; j += 8) {
                float w[8];
                head_block<WT>(sw, j, w);  // from shared memory
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(sx + b * TC + j);
                    const float4 x1 = *reinterpret_cast<const float4 *>(sx + b * TC + j + 4);
                    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc[b][k] = __fmaf_rn(w[k], xv[k], acc[b][k]);  // dequant.c:440-444
                }
            }
        }
    }
    cp_async_wait<0>();
    if (r >= a.rows) return;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        /* dequant.c:447-452: lo + hi, then two horizontal adds */
        const float s0 = __fadd_rn(acc[b][0], acc[b][4]), s1 = __fadd_rn(acc[b][1], acc[b][5]);
        const float s2 = __fadd_rn(acc[b][2], acc[b][6]), s3 = __fadd_rn(acc[b][3], acc[b][7]);
        a.y[(size_t)b * (size_t)a.ldy + r] = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
    }
}

}  // namespace noel
