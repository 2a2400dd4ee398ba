/*
 * gk_oracle.c -- scalar CPU restatement of gemmkit's i8 / requant / half GEMM semantics.
 *
 * TEST INFRASTRUCTURE ONLY (see gk_oracle.h). Built with -O2 -fno-fast-math
 * -ffp-contract=off so every f64 operation is one IEEE-754 operation under the default
 * round-to-nearest-even mode, as in the Rust reference.
 */
#include "gk_oracle.h"

#include <math.h>
#include <string.h>

/* gemmkit/src/kernel/epilogue.rs:886-897: for |x| < 2^52 adding then subtracting 2^52
 * rounds to the nearest integer, ties to even; NaN and |x| >= 2^52 pass through. */
double gko_round_ne_f64(double x) {
    const double C = 4503599627370496.0; /* 2^52 */
    if (isnan(x) || x >= C || x <= -C) return x;
    if (x >= 0.0) {
        volatile double t = x + C;
        return t - C;
    } else {
        volatile double t = x - C;
        return t + C;
    }
}

/* Rust `f64 as i64`: saturating, NaN -> 0. */
static int64_t f64_as_i64(double x) {
    if (isnan(x)) return 0;
    if (x >= 9223372036854775808.0) return INT64_MAX;
    if (x <= -9223372036854775808.0) return INT64_MIN;
    return (int64_t)x;
}

static int64_t i64_saturating_add(int64_t a, int64_t b) {
    if (b > 0 && a > INT64_MAX - b) return INT64_MAX;
    if (b < 0 && a < INT64_MIN - b) return INT64_MIN;
    return a + b;
}

static int32_t wrap_add_i32(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static int32_t wrap_mul_i32(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }

/* KRequantize::apply, gemmkit/src/kernel/epilogue.rs:810-830:
 *   scaled = round_ne_f64(f64(v.wrapping_add(b)) * f64(scale))
 *   q      = (scaled as i64).saturating_add(zp)
 *   out    = clamp(q, LO, HI)
 * ReLU (an extension; the reference epilogue has none) is max(out, clamp(zp, LO, HI)),
 * which equals requant(max(v + b, 0)) because scale > 0 and every step is monotone. */
int32_t gko_requant_apply(int32_t v, int32_t bias, float scale, int32_t zp, int32_t lo,
                          int32_t hi, int32_t relu) {
    double prod = (double)wrap_add_i32(v, bias) * (double)scale;
    double scaled = gko_round_ne_f64(prod);
    int64_t q = i64_saturating_add(f64_as_i64(scaled), (int64_t)zp);
    if (q < lo) q = lo;
    if (q > hi) q = hi;
    if (relu) {
        int64_t floor_ = zp < lo ? lo : (zp > hi ? hi : zp);
        if (q < floor_) q = floor_;
    }
    return (int32_t)q;
}

void gko_acc_i8(size_t m, size_t k, size_t n, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, int32_t *acc) {
    for (size_t i = 0; i < m; ++i) {
        for (size_t j = 0; j < n; ++j) {
            uint32_t s = 0;
            for (size_t p = 0; p < k; ++p) {
                int32_t av = a[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa];
                int32_t bv = b[(ptrdiff_t)p * rsb + (ptrdiff_t)j * csb];
                s += (uint32_t)(av * bv);
            }
            acc[i * n + j] = (int32_t)s;
        }
    }
}

/* gemmkit/src/dispatch/int.rs:131-163 (execute_int, scale_c_int) and
 * gemmkit/src/kernel/int.rs:36-120 (int32_epilogue: beta*C + alpha*AB, wrapping). */
void gko_gemm_i8(size_t m, size_t k, size_t n, int32_t alpha, const int8_t *a, ptrdiff_t rsa,
                 ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, int32_t beta,
                 int32_t *c, ptrdiff_t rsc, ptrdiff_t csc) {
    if (m == 0 || n == 0) return;
    if (k == 0 || alpha == 0) {
        for (size_t j = 0; j < n; ++j)
            for (size_t i = 0; i < m; ++i) {
                int32_t *p = c + (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
                if (beta == 0)
                    *p = 0;
                else if (beta != 1)
                    *p = wrap_mul_i32(beta, *p);
            }
        return;
    }
    for (size_t i = 0; i < m; ++i) {
        for (size_t j = 0; j < n; ++j) {
            uint32_t s = 0;
            for (size_t p = 0; p < k; ++p) {
                int32_t av = a[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa];
                int32_t bv = b[(ptrdiff_t)p * rsb + (ptrdiff_t)j * csb];
                s += (uint32_t)(av * bv);
            }
            int32_t v = wrap_mul_i32(alpha, (int32_t)s);
            int32_t *cp = c + (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            *cp = beta == 0 ? v : wrap_add_i32(wrap_mul_i32(beta, *cp), v);
        }
    }
}

/* gemmkit/src/dispatch/int.rs:672-752 (execute_int_requant, requant_degenerate: k == 0
 * applies the map to a zero accumulator) with the lookups of KRequantize::apply. */
void gko_gemm_i8_requant(size_t m, size_t k, size_t n, const int8_t *a, ptrdiff_t rsa,
                         ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb,
                         const gko_requant *q, void *c, ptrdiff_t rsc, ptrdiff_t csc) {
    if (m == 0 || n == 0) return;
    const int32_t lo = q->out_u8 ? 0 : -128, hi = q->out_u8 ? 255 : 127;
    for (size_t i = 0; i < m; ++i) {
        for (size_t j = 0; j < n; ++j) {
            uint32_t s = 0;
            for (size_t p = 0; p < k; ++p) {
                int32_t av = a[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa];
                int32_t bv = b[(ptrdiff_t)p * rsb + (ptrdiff_t)j * csb];
                s += (uint32_t)(av * bv);
            }
            int32_t bb = q->bias_axis == GKO_AXIS_ROW ? q->bias[i]
                         : q->bias_axis == GKO_AXIS_COL ? q->bias[j]
                                                        : 0;
            float sc = q->scale_axis == GKO_AXIS_ROW ? q->scales[i]
                       : q->scale_axis == GKO_AXIS_COL ? q->scales[j]
                                                       : q->scale;
            int32_t r = gko_requant_apply((int32_t)s, bb, sc, q->zp, lo, hi, q->relu);
            ptrdiff_t off = (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
            if (q->out_u8)
                ((uint8_t *)c)[off] = (uint8_t)r;
            else
                ((int8_t *)c)[off] = (int8_t)r;
        }
    }
}

float gko_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16 -> binary32, exact (normal, subnormal, inf, NaN). */
float gko_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0x1f) {
        u = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        u = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        u = sign;
    } else {
        /* subnormal: value = man * 2^-24 */
        int e = -1;
        do {
            man <<= 1;
            ++e;
        } while ((man & 0x400u) == 0);
        man &= 0x3ffu;
        u = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* f32 -> bf16, round to nearest even on the dropped 16 bits; NaN stays NaN (quiet bit
 * forced on). */
uint16_t gko_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

void gko_gemm_half_f64(int is_f16, size_t m, size_t k, size_t n, double alpha,
                       const uint16_t *a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t *b,
                       ptrdiff_t rsb, ptrdiff_t csb, double beta, const float *c_in,
                       ptrdiff_t rsc, ptrdiff_t csc, double *out) {
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            double s = 0.0;
            for (size_t p = 0; p < k; ++p) {
                uint16_t av = a[(ptrdiff_t)i * rsa + (ptrdiff_t)p * csa];
                uint16_t bv = b[(ptrdiff_t)p * rsb + (ptrdiff_t)j * csb];
                double x = is_f16 ? gko_f16_to_f32(av) : gko_bf16_to_f32(av);
                double y = is_f16 ? gko_f16_to_f32(bv) : gko_bf16_to_f32(bv);
                s += x * y;
            }
            double r = alpha * s;
            if (beta != 0.0) r += beta * (double)c_in[(ptrdiff_t)i * rsc + (ptrdiff_t)j * csc];
            out[i * n + j] = r;
        }
}
