// SPDX-License-Identifier: MIT
//
// libm_fit.c -- exhaustive comparisons of candidate single-precision exp and
// log evaluations against the HOST C library's expf/logf, used by fit.py to
// determine the constants of qwen.haiku_b200/csrc/qh_libm.cuh.
//
// TEST / BUILD-TIME INFRASTRUCTURE, NOT PRODUCT CODE. The reference model
// calls expf/logf from the host C library (glibc on Linux: slm/qwen.c:464-470,
// slm/model.c:943, slm/tensor.c:315/491/1086, simd/simd.c:264-277,
// slm/chunked.c:324-498, slm/sampler.c:105). glibc (2.28 and later) evaluates
// both with the table-driven method of ARM's optimized-routines:
//   expf: k = round(x * 32/ln2), r = x * 32/ln2 - k,
//         exp(x) = 2^(k/32) * p(r), 2^(k/32) from a 32-entry table of 2^(i/32)
//         with the exponent added in, p a cubic, all in double precision;
//   logf: x = 2^k * z with z in [0x3f330000, 0x3f330000 + 2^23) (bit
//         patterns), z in one of 16 subintervals i with a table pair
//         (invc_i ~ 1/c_i, logc_i ~ log c_i), r = z * invc_i - 1,
//         log(x) = logc_i + k ln2 + r + r^2 q(r), q a quadratic.
// Only the structure is taken from that published method. The values that
// make the result bit-identical (the polynomial coefficients, the log table)
// are measured here: fit.py starts from textbook values and moves them, by
// linear programs over the inputs this file reports as mismatching, until
// the candidate equals the host library on every input. The 2^(i/32) table
// is computed from its definition. x86-64 glibc selects its FMA-compiled
// variant on CPUs with FMA, so every multiply-add below is a fused fma().
//
// Build: gcc -O2 -fopenmp -ffp-contract=off -fPIC -shared (fit.py does it).

#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint32_t asu(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float asf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint64_t asu64(double f) { uint64_t u; memcpy(&u, &f, 8); return u; }
static inline double asd(uint64_t u) { double f; memcpy(&f, &u, 8); return f; }

// ---- expf ---------------------------------------------------------------
// p[0..2] = C0, C1, C2 of p(r) = 1 + C2 r + C1 r^2 + C0 r^3 (r scaled by 32);
// tab[32] = bits of 2^(i/32) minus i << 47.
static inline void exp_reduce(float x, const uint64_t *tab, double *r, double *s) {
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
    double xd = x;
    double kd = fma(inv_ln2_n, xd, shift);
    uint64_t ki = asu64(kd);
    kd -= shift;
    *r = fma(inv_ln2_n, xd, -kd);
    *s = asd(tab[ki % 32] + (ki << 47));
}

float cand_expf(float x, const double *p, const uint64_t *tab) {
    uint32_t ix = asu(x);
    if (ix == 0xff800000u) return 0.0f;          // -inf
    if ((ix & 0x7f800000u) == 0x7f800000u) return x + x;  // +inf, nan
    if (x > 89.0f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    double r, s;
    exp_reduce(x, tab, &r, &s);
    double z = fma(p[0], r, p[1]);
    double r2 = r * r;
    double y = fma(p[2], r, 1.0);
    y = fma(z, r2, y);
    return (float)(y * s);
}

// Mismatching inputs in the normal range (-104, 89) as linear constraints on
// (dC0, dC1, dC2): L <= dC2 r + dC1 r^2 + dC0 r^3 <= U, in units of 2^-60.
int64_t exp_rows(const double *p, const uint64_t *tab, double *R, double *L, double *U, int64_t maxn,
                 int64_t *nrows) {
    int64_t mis = 0, cnt = 0;
#pragma omp parallel for reduction(+ : mis) schedule(dynamic, 1)
    for (int64_t hi = 0; hi < (1 << 16); hi++) {
        for (int64_t lo = 0; lo < (1 << 16); lo++) {
            float x = asf((uint32_t)((hi << 16) | lo));
            if (!(x > -104.0f && x < 89.0f)) continue;
            float g = expf(x);
            if (asu(g) == asu(cand_expf(x, p, tab))) continue;
            mis++;
            double r, s;
            exp_reduce(x, tab, &r, &s);
            if (r == 0) continue;
            long double gm = nextafterf(g, -INFINITY), gp = nextafterf(g, INFINITY);
            long double lo_ = ((long double)g + gm) / 2, hi_ = ((long double)g + gp) / 2;
            long double rr = r;
            long double t = (long double)p[2] * rr + (long double)p[1] * rr * rr + (long double)p[0] * rr * rr * rr;
            int64_t k;
#pragma omp atomic capture
            k = cnt++;
            if (k < maxn) {
                R[k] = r;
                L[k] = (double)((lo_ / (long double)s - 1.0L - t) * 0x1p60L);
                U[k] = (double)((hi_ / (long double)s - 1.0L - t) * 0x1p60L);
            }
        }
    }
    *nrows = cnt;
    return mis;
}

// ---- logf ---------------------------------------------------------------
// th[0..15] invc, th[16..31] logc, th[32..34] A0, A1, A2 with
// q(r) = A2 + A1 r + A0 r^2, th[35] ln 2.
#define LOG_OFF 0x3f330000u
static inline int log_split(uint32_t ix, int *i, int *k, double *z) {
    if (ix - 0x00800000u >= 0x7f800000u - 0x00800000u) {
        if ((ix & 0x80000000u) || ix * 2u == 0 || ix * 2u >= 0xff000000u) return 0;
        ix = asu(asf(ix) * 0x1p23f);  // subnormal: normalize
        ix -= 23u << 23;
    }
    uint32_t tmp = ix - LOG_OFF;
    *i = (int)((tmp >> 19) % 16);
    *k = (int32_t)tmp >> 23;
    *z = (double)asf(ix - (tmp & 0xff800000u));
    return 1;
}

static double log_eval(uint32_t ix, const double *th) {
    int i, k;
    double z;
    log_split(ix, &i, &k, &z);
    double r = fma(z, th[i], -1.0);
    double y0 = fma((double)k, th[35], th[16 + i]);
    double r2 = r * r;
    double y = fma(th[33], r, th[34]);
    y = fma(th[32], r2, y);
    return fma(y, r2, y0 + r);
}

// Inputs where the fitted evaluation rounds the other way than the host
// library, with the host's results (sorted by input bits); see fit.py.
static const uint32_t *g_exc_in, *g_exc_out;
static int g_exc_n;
void set_log_exceptions(const uint32_t *in, const uint32_t *out, int n) {
    g_exc_in = in;
    g_exc_out = out;
    g_exc_n = n;
}

float cand_logf(float x, const double *th) {
    uint32_t ix = asu(x);
    for (int lo = 0, hi = g_exc_n; lo < hi;) {
        int mid = (lo + hi) / 2;
        if (g_exc_in[mid] == ix) return asf(g_exc_out[mid]);
        if (g_exc_in[mid] < ix) lo = mid + 1; else hi = mid;
    }
    if (ix == 0x3f800000u) return 0.0f;
    if (ix - 0x00800000u >= 0x7f800000u - 0x00800000u) {
        if (ix * 2u == 0) return -INFINITY;
        if (ix == 0x7f800000u) return x;
        if ((ix & 0x80000000u) || ix * 2u >= 0xff000000u) return (x - x) / (x - x);
    }
    int i, k;
    double z;
    log_split(ix, &i, &k, &z);
    double r = fma(z, th[i], -1.0);
    double y0 = fma((double)k, th[35], th[16 + i]);
    double r2 = r * r;
    double y = fma(th[33], r, th[34]);
    y = fma(th[32], r2, y);
    y = fma(y, r2, y0 + r);
    return (float)y;
}

// Mismatching positive finite inputs whose subinterval is in `mask`; with
// margin > 0 also the matching ones whose unrounded candidate lies within
// margin ulps of a rounding boundary (the constraints a small parameter
// change could break).
int64_t log_rows_near(const double *th, unsigned mask, double margin, int *I, int *K, double *Z, float *G,
                      int64_t maxn, int64_t *nrows);
int64_t log_rows(const double *th, unsigned mask, int *I, int *K, double *Z, float *G, int64_t maxn,
                 int64_t *nrows) {
    return log_rows_near(th, mask, 0.0, I, K, Z, G, maxn, nrows);
}

int64_t log_rows_near(const double *th, unsigned mask, double margin, int *I, int *K, double *Z, float *G,
                      int64_t maxn, int64_t *nrows) {
    int64_t mis = 0, cnt = 0;
#pragma omp parallel for reduction(+ : mis) schedule(dynamic, 1)
    for (int64_t hi = 0; hi < (1 << 15); hi++) {
        for (int64_t lo = 0; lo < (1 << 16); lo++) {
            uint32_t ix = (uint32_t)((hi << 16) | lo);
            if (ix == 0 || ix >= 0x7f800000u || ix == 0x3f800000u) continue;
            int i, k;
            double z;
            log_split(ix, &i, &k, &z);
            if (!((mask >> i) & 1)) continue;
            float g = logf(asf(ix));
            if (asu(g) == asu(cand_logf(asf(ix), th))) {
                if (margin <= 0) continue;
                double y = log_eval(ix, th);
                float f = (float)y;
                double up = nextafterf(f, INFINITY), dn = nextafterf(f, -INFINITY);
                double ulp = up - (double)f;
                double dist = fmin(fabs(y - ((double)f + up) / 2), fabs(y - ((double)f + dn) / 2));
                if (dist > margin * ulp) continue;
            } else {
                mis++;
            }
            int64_t n;
#pragma omp atomic capture
            n = cnt++;
            if (n < maxn) { I[n] = i; K[n] = k; Z[n] = z; G[n] = g; }
        }
    }
    *nrows = cnt;
    return mis;
}

// ---- whole-range checks -----------------------------------------------
static int same(float a, float b) { return asu(a) == asu(b) || (a != a && b != b); }

// Inputs (all 2^32 bit patterns) where the candidate differs from the host
// library; NaN results compare equal to any NaN.
int64_t exp_count_all(const double *p, const uint64_t *tab) {
    int64_t mis = 0;
#pragma omp parallel for reduction(+ : mis) schedule(static)
    for (int64_t u = 0; u < (1ll << 32); u++) {
        float x = asf((uint32_t)u);
        mis += !same(expf(x), cand_expf(x, p, tab));
    }
    return mis;
}

int64_t log_count_all(const double *th) {
    int64_t mis = 0;
#pragma omp parallel for reduction(+ : mis) schedule(static)
    for (int64_t u = 0; u < (1ll << 32); u++) {
        float x = asf((uint32_t)u);
        mis += !same(logf(x), cand_logf(x, th));
    }
    return mis;
}
