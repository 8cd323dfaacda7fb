// crmath.h — correctly rounded fp32 log2 / exp2 for the packed step.
//
// The reference computes the Adam denominator as exp2(p * log2(v + eps))
// (concord/packed_b.py:557) and the shared-exponent scales as exp2(+-e)
// (packed_b.py:491-492).  Parity with the reference's outputs is pinned to
// correctly rounded exp2/log2, so both functions here return the fp32 value
// nearest to the exact result, with the same bits on the host and the GPU:
//   fast path:  double-precision evaluation (relative error < 2^-49) plus a
//               rounding test (Ziv): if x + err and x - err round to the same
//               float, that float is the correctly rounded result;
//   slow path:  (about 1 call in 2^22) double-double evaluation with error
//               below 2^-100, rounded to fp32 through round-to-odd.
// Only IEEE double add/mul/div and explicit fma are used; compile host code
// with -ffp-contract=off and device code with -fmad=false so that nothing
// is contracted behind the code's back.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define CR_HD __host__ __device__ __forceinline__
#define CR_SLOW static __host__ __device__ __noinline__
#define CR_TABLE static __device__ const
#define CR_ALIGN16 __align__(16)
#else
#define CR_ALIGN16 alignas(16)
#define CR_HD static inline
#define CR_SLOW static
#define CR_TABLE static const
#endif

#include "crmath_tables.h"

namespace crmath {

CR_HD double u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d; memcpy(&d, &u, 8); return d;
#endif
}
CR_HD uint64_t d2u(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u; memcpy(&u, &d, 8); return u;
#endif
}
CR_HD uint32_t f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}
CR_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f; memcpy(&f, &u, 4); return f;
#endif
}

// table read (read-only data cache on the GPU)
CR_HD double tab(const double* t, int i) {
#if defined(__CUDA_ARCH__)
    return __ldg(t + i);
#else
    return t[i];
#endif
}

// 2^n as a double, n in [-1022, 1023]
CR_HD double pow2d(int n) { return u2d((uint64_t)(int64_t)(n + 1023) << 52); }

// ---- double-double arithmetic (value = hi + lo, |lo| <= ulp(hi)/2) ----
struct dd { double hi, lo; };

// (hi, lo) pair i of a table of double-doubles, in one 16-byte load
CR_HD dd tab2(const double* t, int i) {
#if defined(__CUDA_ARCH__)
    const double2 v = __ldg(reinterpret_cast<const double2*>(t) + i);
    return dd{v.x, v.y};
#else
    return dd{t[2 * i], t[2 * i + 1]};
#endif
}

CR_HD dd quick_two_sum(double a, double b) { double s = a + b; return {s, b - (s - a)}; }
CR_HD dd two_sum(double a, double b) {
    double s = a + b, bb = s - a;
    return {s, (a - (s - bb)) + (b - bb)};
}
CR_HD dd two_prod(double a, double b) { double p = a * b; return {p, fma(a, b, -p)}; }
CR_HD dd dd_add(dd a, dd b) {
    dd s = two_sum(a.hi, b.hi), t = two_sum(a.lo, b.lo);
    s.lo += t.hi;
    s = quick_two_sum(s.hi, s.lo);
    s.lo += t.lo;
    return quick_two_sum(s.hi, s.lo);
}
CR_HD dd dd_mul(dd a, dd b) {
    dd p = two_prod(a.hi, b.hi);
    p.lo += a.hi * b.lo + a.lo * b.hi;
    return quick_two_sum(p.hi, p.lo);
}
CR_HD dd dd_mul_d(dd a, double b) {
    dd p = two_prod(a.hi, b);
    p.lo += a.lo * b;
    return quick_two_sum(p.hi, p.lo);
}
CR_HD dd dd_div_d(dd a, double b) {  // a / b, b a double
    double q1 = a.hi / b;
    dd r = dd_add(a, dd{-q1 * b, -fma(q1, b, -q1 * b)});
    double q2 = r.hi / b;
    r = dd_add(r, dd{-q2 * b, -fma(q2, b, -q2 * b)});
    double q3 = r.hi / b;
    dd q = quick_two_sum(q1, q2);
    return dd_add(q, dd{q3, 0.0});
}
CR_HD dd dd_div(dd a, dd b) {
    double q1 = a.hi / b.hi;
    dd r = dd_add(a, dd_mul_d(b, -q1));
    double q2 = r.hi / b.hi;
    r = dd_add(r, dd_mul_d(b, -q2));
    double q3 = r.hi / b.hi;
    dd q = quick_two_sum(q1, q2);
    return dd_add(q, dd{q3, 0.0});
}

// Round hi+lo to fp32 (nearest-even) via round-to-odd at 53 bits.
CR_HD float dd_to_float(dd v) {
    if (v.lo == 0.0 || v.hi != v.hi) return (float)v.hi;
    uint64_t u = d2u(v.hi);
    if ((v.lo > 0.0) != (v.hi > 0.0)) u -= 1;  // truncate toward zero
    u |= 1;                                     // sticky bit
    return (float)u2d(u);
}

// ---- constants ----
// 1/ln2 and ln2 as double-double (hi = nearest double, lo = remainder)
#define CR_INVLN2_HI 1.4426950408889634
#define CR_INVLN2_LO 2.0355273740931033e-17
#define CR_LN2_HI 0.6931471805599453
#define CR_LN2_LO 2.3190468138462996e-17

// Decompose finite x > 0 as m * 2^e with m in [sqrt(1/2), sqrt(2)).
CR_HD void log_reduce(float x, float* m_out, int* e_out) {
    uint32_t b = f2u(x);
    int e = 0;
    if (b < 0x00800000u) {  // subnormal: scale by 2^24 (exact)
        x = x * 16777216.0f;
        b = f2u(x);
        e = -24;
    }
    e += (int)((b >> 23) & 0xffu) - 127;
    float m = u2f((b & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421353816986083984375f) { m = m * 0.5f; e += 1; }
    *m_out = m;
    *e_out = e;
}

// log(m) = 2 s (1 + z/3 + z^2/5 + ...), s = (m-1)/(m+1), z = s^2, |z| < 0.0295
CR_SLOW float log2f_slow(float m, int e) {
    double md = (double)m;
    double num = md - 1.0, den = md + 1.0;  // exact
    double sh = num / den;
    dd s = quick_two_sum(sh, fma(-sh, den, num) / den);
    dd z = dd_mul(s, s);
    dd p = dd{1.0 / 43.0, fma(-(1.0 / 43.0), 43.0, 1.0) / 43.0};
    for (int k = 20; k >= 0; --k) {
        double c = (double)(2 * k + 1);
        double ch = 1.0 / c;
        p = dd_add(dd_mul(p, z), dd{ch, fma(-ch, c, 1.0) / c});
    }
    dd lnm = dd_mul(s, p);
    lnm.hi *= 2.0; lnm.lo *= 2.0;
    dd l2 = dd_mul(lnm, dd{CR_INVLN2_HI, CR_INVLN2_LO});
    dd L = dd_add(dd{(double)e, 0.0}, l2);
    return dd_to_float(L);
}

// Full-range log2 (zero, negative, NaN, inf, subnormals) with a float-compare
// rounding test; reached from cr_log2f only for special inputs or when the
// fast path cannot decide the rounding.
template <bool FORCE_SLOW>
CR_SLOW float log2f_careful(float x) {
    if (!(x > 0.0f)) {
        if (x == 0.0f) return -INFINITY;
        return NAN;  // negative or NaN
    }
    if (x == INFINITY) return INFINITY;
    // x = 2^k * z, z in [0.699, 1.398); sub-interval i of z has center 1/invc
    uint32_t ix = f2u(x);
    int kadj = 0;
    if (ix < 0x00800000u) {  // subnormal: scale by 2^23 (exact)
        ix = f2u(x * 8388608.0f);
        kadj = -23;
    }
    const uint32_t tmp = ix - CR_LOG_OFF;
    const int i = (int)((tmp >> 16) & 127u);
    const int k = ((int32_t)tmp >> 23) + kadj;
    const float z = u2f(ix - (tmp & 0xff800000u));
    const double r = (double)z * tab(cr_log_invc, i) - 1.0;  // exact
    // log2(1+r), |r| < 2^-7, degree 9 (relative error < 2^-60)
    double p = CR_LOG_C8;
    p = fma(p, r, CR_LOG_C7);
    p = fma(p, r, CR_LOG_C6);
    p = fma(p, r, CR_LOG_C5);
    p = fma(p, r, CR_LOG_C4);
    p = fma(p, r, CR_LOG_C3);
    p = fma(p, r, CR_LOG_C2);
    p = fma(p, r, CR_LOG_C1);
    p = fma(p, r, CR_LOG_C0);
    const dd lc = tab2(cr_log_logc, i);
    const double L = ((double)k + lc.hi) + fma(p, r, lc.lo);
    const double err = fabs(L) * 0x1p-46;
    const float a = (float)(L + err), b = (float)(L - err);
    if (!FORCE_SLOW && a == b) return a;
    float m; int e;
    log_reduce(x, &m, &e);
    return log2f_slow(m, e);
}

// 2^f for -1/128 <= f < 1 in double-double: exp(t), t = f ln2, Taylor to t^30/30!
CR_HD dd exp2_frac_dd(double f) {
    dd t = dd_mul_d(dd{CR_LN2_HI, CR_LN2_LO}, f);
    dd sum = dd{1.0, 0.0}, term = dd{1.0, 0.0};
    for (int k = 1; k <= 30; ++k) {
        term = dd_div_d(dd_mul(term, t), (double)k);
        sum = dd_add(sum, term);
    }
    return sum;
}

CR_SLOW float exp2f_slow(double f, double sc) {
    dd v = exp2_frac_dd(f);
    v.hi *= sc; v.lo *= sc;  // exact scaling by a power of two
    return dd_to_float(v);
}

template <bool FORCE_SLOW>
CR_SLOW float exp2f_careful(float y) {
    if (y != y) return y;
    if (y >= 128.0f) return INFINITY;
    if (y < -150.0f) return 0.0f;
    // y = n + j/64 + f, |f| <= 1/128; 2^y = 2^n * 2^(j/64) * 2^f
    const float k64 = rintf(y * 64.0f);        // exact scaling, integer result
    const int k = (int)k64;
    const int j = k & 63, n = k >> 6;
    const double f = (double)y - (double)k64 * 0.015625;  // exact
    if (f == 0.0 && j == 0) return (float)pow2d(n);     // exact power of two
    double p = CR_EXP_C7;
    p = fma(p, f, CR_EXP_C6);
    p = fma(p, f, CR_EXP_C5);
    p = fma(p, f, CR_EXP_C4);
    p = fma(p, f, CR_EXP_C3);
    p = fma(p, f, CR_EXP_C2);
    p = fma(p, f, CR_EXP_C1);
    const double t = tab(cr_exp2_tab_hi, j);
    const double sc = pow2d(n);
    const double rr = fma(t * f, p, t) * sc;  // t * (1 + f p)
    const double err = rr * 0x1p-46;
    const float a = (float)(rr + err), b = (float)(rr - err);
    if (!FORCE_SLOW && a == b) return a;
    return exp2f_slow((double)y - (double)n, sc);
}

// True when the double v lies within 2^8 double ulps of a midpoint between
// two adjacent floats (only meaningful when (float)v is a normal float).
CR_HD bool near_float_midpoint(double v) {
    const uint32_t t = (uint32_t)d2u(v) & 0x1FFFFFFFu;   // the 29 bits below float precision
    return (uint32_t)(t - 0x10000000u + 0x100u) <= 0x200u;
}

// Correctly rounded log2 of an fp32 value.  Hot path: normal positive x,
// x = 2^k z, z*invc - 1 = r exact, log2(1+r) by a degree-7 polynomial in
// double (relative error < 2^-50); the bits test sends the rare ambiguous
// roundings (and every special input) to log2f_careful.
template <bool FORCE_SLOW = false>
CR_HD float cr_log2f(float x) {
    const uint32_t ix = f2u(x);
    if (FORCE_SLOW || ix - 0x00800000u >= 0x7F000000u) return log2f_careful<FORCE_SLOW>(x);
    const uint32_t tmp = ix - CR_LOG_OFF;
    const int i = (int)((tmp >> 16) & 127u);
    const int k = (int32_t)tmp >> 23;
    const float z = u2f(ix - (tmp & 0xff800000u));
    const double r = (double)z * tab(cr_log_invc, i) - 1.0;  // exact
    double p = CR_PL(6);
    p = fma(p, r, CR_PL(5));
    p = fma(p, r, CR_PL(4));
    p = fma(p, r, CR_PL(3));
    p = fma(p, r, CR_PL(2));
    p = fma(p, r, CR_PL(1));
    p = fma(p, r, CR_PL(0));
    const dd lc = tab2(cr_log_logc, i);
    const double L = ((double)k + lc.hi) + fma(p, r, lc.lo);
    if (near_float_midpoint(L)) return log2f_careful<false>(x);
    return (float)L;
}

// Correctly rounded 2^y for fp32 y.  Hot path: -126 <= y < 128 (normal
// result): y = (n*64 + j)/64 + f, |f| <= 1/128, 2^y = 2^n 2^(j/64) (1 + q(f)),
// q of degree 6 (relative error < 2^-50); 2^n enters the exponent field.
template <bool FORCE_SLOW = false>
CR_HD float cr_exp2f(float y) {
    if (FORCE_SLOW || !(y >= -126.0f && y < 128.0f)) return exp2f_careful<FORCE_SLOW>(y);
    const float t = y * 64.0f + 12582912.0f;          // 1.5 * 2^23: rounds y*64 to an integer
    const int k = (int)(f2u(t) - 0x4B400000u);
    const float k64 = t - 12582912.0f;
    const float f = y - k64 * 0.015625f;               // exact, |f| <= 1/128
    const int j = k & 63, n = k >> 6;
    const double fd = (double)f;
    double q = CR_PE(6);
    q = fma(q, fd, CR_PE(5));
    q = fma(q, fd, CR_PE(4));
    q = fma(q, fd, CR_PE(3));
    q = fma(q, fd, CR_PE(2));
    q = fma(q, fd, CR_PE(1));
    q = q * fd;
    const double T = tab(cr_exp2_tab_hi, j);
    double rr = fma(T, q, T);
    rr = u2d(d2u(rr) + ((uint64_t)(int64_t)n << 52));  // * 2^n
    if (near_float_midpoint(rr)) return exp2f_careful<false>(y);
    return (float)rr;
}

// Lockstep form for W values: out[j] = CR(2^(CR(p * CR(log2 x[j])))), the
// Adam denominator exp2(p*log2(x)).  Evaluating the W values side by side
// gives the scheduler independent double-precision chains, and one branch
// per stage sends only the rare hard cases to the careful paths.
template <int W>
CR_HD void cr_pow2log2(const float (&x)[W], float p, float (&out)[W]) {
    bool bad = false;
    double r[W], acc[W], L[W];
    int k[W];
    dd lc[W];
    float Lf[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
        const uint32_t ix = f2u(x[j]);
        bad |= (ix - 0x00800000u >= 0x7F000000u);
        const uint32_t tmp = ix - CR_LOG_OFF;
        const int i = (int)((tmp >> 16) & 127u);
        k[j] = (int32_t)tmp >> 23;
        const float z = u2f(ix - (tmp & 0xff800000u));
        r[j] = fma((double)z, tab(cr_log_invc, i), -1.0);  // exact
        lc[j] = tab2(cr_log_logc, i);
        acc[j] = CR_PL(6);
    }
#pragma unroll
    for (int c = 5; c >= 0; --c) {
#pragma unroll
        for (int j = 0; j < W; ++j) acc[j] = fma(acc[j], r[j], CR_PL(c));
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
        L[j] = ((double)k[j] + lc[j].hi) + fma(acc[j], r[j], lc[j].lo);
        bad |= near_float_midpoint(L[j]);
        Lf[j] = (float)L[j];
    }
    if (bad) {
#pragma unroll
        for (int j = 0; j < W; ++j) Lf[j] = cr_log2f<false>(x[j]);
    }
    // 2^y, y = p * L
    bad = false;
    double q[W], T[W];
    float y[W];
    int n[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
        y[j] = p * Lf[j];
        bad |= !(y[j] >= -126.0f && y[j] < 128.0f);
        const float t = y[j] * 64.0f + 12582912.0f;
        const int kk = (int)(f2u(t) - 0x4B400000u);
        const float f = y[j] - (t - 12582912.0f) * 0.015625f;
        n[j] = kk >> 6;
        T[j] = tab(cr_exp2_tab_hi, kk & 63);
        r[j] = (double)f;
        q[j] = CR_PE(6);
    }
#pragma unroll
    for (int c = 5; c >= 1; --c) {
#pragma unroll
        for (int j = 0; j < W; ++j) q[j] = fma(q[j], r[j], CR_PE(c));
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
        double rr = fma(T[j], q[j] * r[j], T[j]);
        rr = u2d(d2u(rr) + ((uint64_t)(int64_t)n[j] << 52));
        bad |= near_float_midpoint(rr);
        out[j] = (float)rr;
    }
    if (bad) {
#pragma unroll
        for (int j = 0; j < W; ++j) out[j] = cr_exp2f<false>(y[j]);
    }
}

}  // namespace crmath
