/*
 * exp of the sampler's scaled differences, bit-identical to glibc's expf.
 *
 * The reference builds each candidate's weight as expf(diff) with glibc's
 * expf (Sain-Kai/noel src/sampler.c:140), for diff in (-15, 0].  Candidate
 * order, top-k membership and every prefix sum depend on those exact bits,
 * so the kernels reproduce them in two steps:
 *
 *   1. cr_expf(x): the correctly rounded single-precision exp.  exp((double)x)
 *      is within 1 ulp of double precision, so rounding it to float is correct
 *      unless it lies within a few double ulps of a float rounding midpoint;
 *      those rare inputs (about 1 in 4 million) are recomputed in
 *      double-double arithmetic (range reduction by ln 2, Taylor series on
 *      |s| < 2^-11, ten squarings) and rounded from there.  exp of a non-zero
 *      float is transcendental, so it never lies on a midpoint exactly.
 *   2. glibc's expf is not correctly rounded everywhere; the inputs of
 *      (-15, 0] where it differs from cr_expf are listed in a table generated
 *      at build time by calling glibc's expf (gen_expf_table.cc), and the
 *      glibc result is taken from there.
 *
 * This header is shared by host code (the table generator) and device code.
 */
#ifndef NOEL_REF_EXPF_H
#define NOEL_REF_EXPF_H

#include <stdint.h>
#include <math.h>
#include <string.h>

#if defined(__CUDACC__)
#define NOEL_HD __host__ __device__ __forceinline__
#define NOEL_HD_COLD __host__ __device__ __noinline__ /* the rare path: one copy of its code */
#else
#define NOEL_HD static inline
#define NOEL_HD_COLD static
#endif

/* Domain of the table: float bit patterns [-0.0, -15.0). */
#define NOEL_EXPF_DOMAIN_FIRST 0x80000000u
#define NOEL_EXPF_DOMAIN_END 0xC1700000u
#define NOEL_EXPF_BUCKET_SHIFT 17
#define NOEL_EXPF_NBUCKETS (((NOEL_EXPF_DOMAIN_END - NOEL_EXPF_DOMAIN_FIRST) >> NOEL_EXPF_BUCKET_SHIFT) + 1)

NOEL_HD uint64_t noel_d2u(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    memcpy(&u, &d, 8);
    return u;
#endif
}
NOEL_HD double noel_u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d;
    memcpy(&d, &u, 8);
    return d;
#endif
}
NOEL_HD uint32_t noel_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}
NOEL_HD float noel_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

/* ---- double-double arithmetic (Dekker / Knuth error-free transforms) ---- */
typedef struct { double hi, lo; } noel_dd;

NOEL_HD noel_dd noel_dd_two_sum(double a, double b) {
    noel_dd r;
    r.hi = a + b;
    double bb = r.hi - a;
    r.lo = (a - (r.hi - bb)) + (b - bb);
    return r;
}
NOEL_HD noel_dd noel_dd_fast_two_sum(double a, double b) { /* |a| >= |b| */
    noel_dd r;
    r.hi = a + b;
    r.lo = b - (r.hi - a);
    return r;
}
NOEL_HD noel_dd noel_dd_add(noel_dd a, noel_dd b) {
    noel_dd s = noel_dd_two_sum(a.hi, b.hi);
    noel_dd t = noel_dd_two_sum(a.lo, b.lo);
    s.lo += t.hi;
    s = noel_dd_fast_two_sum(s.hi, s.lo);
    s.lo += t.lo;
    return noel_dd_fast_two_sum(s.hi, s.lo);
}
NOEL_HD noel_dd noel_dd_mul(noel_dd a, noel_dd b) {
    noel_dd p;
    p.hi = a.hi * b.hi;
    p.lo = fma(a.hi, b.hi, -p.hi);          /* exact product error */
    p.lo += a.hi * b.lo + a.lo * b.hi;
    return noel_dd_fast_two_sum(p.hi, p.lo);
}
NOEL_HD noel_dd noel_dd_mul_d(noel_dd a, double b) {
    noel_dd p;
    p.hi = a.hi * b;
    p.lo = fma(a.hi, b, -p.hi);
    p.lo += a.lo * b;
    return noel_dd_fast_two_sum(p.hi, p.lo);
}
NOEL_HD noel_dd noel_dd_div_d(noel_dd a, double b) {
    double q1 = a.hi / b;
    noel_dd p = noel_dd_mul_d(noel_dd{q1, 0.0}, b);    /* q1*b exactly */
    noel_dd r = noel_dd_add(a, noel_dd{-p.hi, -p.lo});
    double q2 = r.hi / b;
    return noel_dd_fast_two_sum(q1, q2);
}

/*
 * exp(x) for a float x with exp(x) a normal float, as a double-double
 * accurate to well beyond 2^-90 relative.  ln 2 is split as the double
 * nearest to it plus the double nearest to the remainder.
 */
NOEL_HD_COLD noel_dd noel_dd_exp(float xf) {
    const noel_dd ln2 = {0.6931471805599453094172321, 2.319046813846299558417771e-17};
    const double x = (double)xf;
    const double k = nearbyint(x * 1.4426950408889634073599247);
    /* r = x - k ln2 (k has at most 8 bits, so k*ln2.hi is exact in two parts) */
    noel_dd kl = noel_dd_mul_d(ln2, k);
    noel_dd r = noel_dd_add(noel_dd{x, 0.0}, noel_dd{-kl.hi, -kl.lo});
    /* s = r / 2^10, |s| <= 3.4e-4 */
    noel_dd s = {r.hi * (1.0 / 1024.0), r.lo * (1.0 / 1024.0)};
    /* Taylor series by Horner: 1 + s(1 + s/2(1 + s/3(...))) */
    noel_dd p = {1.0, 0.0};
    for (int i = 10; i >= 1; --i) {
        p = noel_dd_div_d(noel_dd_mul(p, s), (double)i);
        p = noel_dd_add(noel_dd{1.0, 0.0}, p);
    }
    for (int i = 0; i < 10; ++i) p = noel_dd_mul(p, p);
    /* times 2^k: exact scaling of both parts */
    const int ki = (int)k;
    p.hi = ldexp(p.hi, ki);
    p.lo = ldexp(p.lo, ki);
    return p;
}

/* Correct float rounding of a positive double-double. */
NOEL_HD float noel_dd_to_float(noel_dd v) {
    const uint64_t b = noel_d2u(v.hi);
    const uint64_t low = b & 0x1FFFFFFFull;
    if (low == 0x10000000ull && v.lo != 0.0) {
        /* hi sits exactly on a float midpoint: lo decides */
        const uint64_t below = b & ~0x1FFFFFFFull;       /* float just below */
        const float fb = (float)noel_u2d(below);
        if (v.lo < 0.0) return fb;
        return noel_u2f(noel_f2u(fb) + 1u);
    }
    return (float)v.hi;
}

/* Correctly rounded expf for x with exp(x) a normal float (x in (-87, 88)). */
NOEL_HD float noel_cr_expf(float x) {
    const double d = exp((double)x);
    const uint64_t low = noel_d2u(d) & 0x1FFFFFFFull;
    const int64_t dist = (int64_t)low - 0x10000000ll;
    if (dist > -64 && dist < 64) return noel_dd_to_float(noel_dd_exp(x));
    return (float)d;
}

/*
 * glibc-identical expf on (-15, 0]: the correctly rounded value unless x is
 * in the exception table (keys sorted; bucket b holds keys
 * [offs[b], offs[b+1]) whose (bits - DOMAIN_FIRST) >> BUCKET_SHIFT == b).
 * near: every exception has exp((double)x) within near double ulps of a float
 * rounding midpoint (established by the table generator over all inputs);
 * inputs farther away (with a margin for a 1-ulp difference between double
 * exp implementations) skip the lookup.
 */
NOEL_HD float noel_ref_expf(float x, const uint32_t *keys, const uint32_t *vals,
                            const uint32_t *offs, long long near = 0x10000000ll) {
    const double d = exp((double)x);
    const long long low = (long long)(noel_d2u(d) & 0x1FFFFFFFull) - 0x10000000ll;
    const long long dist = low < 0 ? -low : low;
    const float y = (dist < 64) ? noel_dd_to_float(noel_dd_exp(x)) : (float)d;
    if (dist > near + 64) return y;
    const uint32_t k = noel_f2u(x) - NOEL_EXPF_DOMAIN_FIRST;
    if (keys && k < (NOEL_EXPF_DOMAIN_END - NOEL_EXPF_DOMAIN_FIRST)) {
        const uint32_t bkt = k >> NOEL_EXPF_BUCKET_SHIFT;
        uint32_t lo = offs[bkt], hi = offs[bkt + 1];
        const uint32_t key = noel_f2u(x);
        while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            const uint32_t km = keys[mid];
            if (km == key) return noel_u2f(vals[mid]);
            if (km < key) lo = mid + 1; else hi = mid;
        }
    }
    return y;
}

#endif /* NOEL_REF_EXPF_H */
