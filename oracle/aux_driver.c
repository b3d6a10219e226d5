/*
 * Batch driver around the reference's router (Sain-Kai/noel src/sparsity.c,
 * compiled from the reference sources by oracle/Makefile into
 * oracle/_ref/libaux_ref.so).  TEST INFRASTRUCTURE ONLY: it times the
 * reference as the CPU baseline; the shipped library never loads it.
 */
#include <stddef.h>
#include <stdint.h>

#include "sparsity.h"
#ifdef _OPENMP
#include <omp.h>
#endif

/* aether_route_top_k on tokens [0, T) (logits row t at logits + t * ld),
 * tokens split across nthreads OpenMP threads (0: all) */
void ref_route_batch(const float *logits, int T, int E, size_t ld, int top_k, moe_routing_t *out, int nthreads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : omp_get_max_threads())
#endif
    for (int t = 0; t < T; ++t) aether_route_top_k(logits + (size_t)t * ld, E, top_k, out + (size_t)t * top_k);
}
