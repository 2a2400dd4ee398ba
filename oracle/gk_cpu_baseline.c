/*
 * gk_cpu_baseline.c -- timed CPU baseline: a C restatement of gemmkit's multithreaded
 * AVX-512 VNNI integer path and its AVX-512 BF16 dot path.
 *
 * TEST INFRASTRUCTURE ONLY (see gk_oracle.h): bench.py times this beside the CUDA engine
 * ("C restatement of gemmkit's VNNI path"; gemmkit itself is Rust and cannot be built
 * here). It follows, in order:
 *   - RHS pack: k-quad interleave, NR = 12 columns per panel, zero pad
 *     (gemmkit/src/pack.rs:117-200, gemmkit/src/api/packed.rs:372-453, kc = k);
 *   - LHS pack: k-quad interleave of A + 128, MR = 32 rows per panel, pad 128
 *     (gemmkit/src/kernel/int.rs:362-386 vnni_a_xform);
 *   - microkernel: 32 x 12 i32 tile, vpdpbusd per k-quad, then minus 128 * colsum(B)
 *     (gemmkit/src/simd/avx512.rs:483-550);
 *   - requant store: widen to f64, multiply, round-to-nearest-even, + zp, clamp, truncate
 *     (gemmkit/src/simd/avx512.rs:274-324); scalar KRequantize::apply otherwise;
 *   - jobs: (row block x column-panel chunk) spread over worker threads
 *     (gemmkit/src/driver.rs:779-910).
 * Every output is bit-identical to gk_oracle.c (tests/test_oracle.py checks it).
 */
#include <immintrin.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include "gk_oracle.h"

#define MR 32
#define NR 12
#define JCHUNK 16 /* column panels per job */

int gko_threads(int threads) {
    int t = threads > 0 ? threads : omp_get_max_threads();
    return t < 1 ? 1 : t;
}

int gko_cpu_has_vnni(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512vnni");
}

static int cpu_has_avx512bf16(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bf16");
}

static size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

int gko_vnni_prepack(const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, size_t k, size_t n,
                     gko_packed_rhs *out) {
    memset(out, 0, sizeof(*out));
    out->k = k;
    out->n = n;
    out->k_pad = round_up(k, 4);
    out->n_pad = round_up(n, NR);
    size_t total = out->k_pad * out->n_pad;
    out->buf = (int8_t *)aligned_alloc(64, round_up(total ? total : 64, 64));
    out->colsum = (int32_t *)calloc(out->n_pad ? out->n_pad : 1, sizeof(int32_t));
    if (!out->buf || !out->colsum) return -1;
    size_t nq = out->k_pad / 4;
#pragma omp parallel for schedule(static)
    for (size_t jp = 0; jp < out->n_pad / NR; ++jp) {
        int8_t *panel = out->buf + jp * NR * out->k_pad;
        for (size_t qd = 0; qd < nq; ++qd)
            for (size_t j = 0; j < NR; ++j)
                for (size_t t = 0; t < 4; ++t) {
                    size_t col = jp * NR + j, p = qd * 4 + t;
                    int8_t v = 0;
                    if (col < n && p < k) v = b[(ptrdiff_t)p * rsb + (ptrdiff_t)col * csb];
                    panel[qd * NR * 4 + j * 4 + t] = v;
                }
        for (size_t j = 0; j < NR; ++j) {
            int32_t s = 0;
            size_t col = jp * NR + j;
            if (col < n)
                for (size_t p = 0; p < k; ++p) s += b[(ptrdiff_t)p * rsb + (ptrdiff_t)col * csb];
            out->colsum[col] = s;
        }
    }
    return 0;
}

void gko_vnni_packed_free(gko_packed_rhs *p) {
    free(p->buf);
    free(p->colsum);
    memset(p, 0, sizeof(*p));
}

/* A row block of MR rows, k-quad interleaved, +128 (pad 128). */
static void pack_a_block(int8_t *dst, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                         size_t m, size_t k, size_t k_pad, size_t i0) {
    size_t nq = k_pad / 4;
    for (size_t qd = 0; qd < nq; ++qd)
        for (size_t i = 0; i < MR; ++i)
            for (size_t t = 0; t < 4; ++t) {
                size_t row = i0 + i, p = qd * 4 + t;
                int v = 0;
                if (row < m && p < k) v = a[(ptrdiff_t)row * rsa + (ptrdiff_t)p * csa];
                dst[qd * MR * 4 + i * 4 + t] = (int8_t)(uint8_t)(v + 128);
            }
}

/* 32 x 12 i32 tile (column-major, out[j*MR + i]) = sum_k A*B, VNNI form. */
__attribute__((target("avx512f,avx512bw,avx512vnni"))) static void
micro_vnni(size_t nq, const int8_t *pa, const int8_t *pb, const int32_t *colsum, int32_t *out) {
    __m512i acc[NR][2];
    for (int j = 0; j < NR; ++j) acc[j][0] = acc[j][1] = _mm512_setzero_si512();
    for (size_t qd = 0; qd < nq; ++qd) {
        __m512i a0 = _mm512_loadu_si512((const void *)(pa + qd * MR * 4));
        __m512i a1 = _mm512_loadu_si512((const void *)(pa + qd * MR * 4 + 64));
        const int8_t *bq = pb + qd * NR * 4;
        for (int j = 0; j < NR; ++j) {
            int32_t bw;
            memcpy(&bw, bq + j * 4, 4);
            __m512i bj = _mm512_set1_epi32(bw);
            acc[j][0] = _mm512_dpbusd_epi32(acc[j][0], a0, bj);
            acc[j][1] = _mm512_dpbusd_epi32(acc[j][1], a1, bj);
        }
    }
    for (int j = 0; j < NR; ++j) {
        __m512i corr = _mm512_set1_epi32((int32_t)(128u * (uint32_t)colsum[j]));
        _mm512_storeu_si512((void *)(out + j * MR), _mm512_sub_epi32(acc[j][0], corr));
        _mm512_storeu_si512((void *)(out + j * MR + 16), _mm512_sub_epi32(acc[j][1], corr));
    }
}

/* Portable fallback with the same blocking (u8 x s8 products, then the same correction). */
static void micro_portable(size_t nq, const int8_t *pa, const int8_t *pb, const int32_t *colsum,
                           int32_t *out) {
    int32_t acc[NR][MR];
    memset(acc, 0, sizeof(acc));
    for (size_t qd = 0; qd < nq; ++qd)
        for (int j = 0; j < NR; ++j)
            for (int i = 0; i < MR; ++i) {
                int32_t s = 0;
                for (int t = 0; t < 4; ++t)
                    s += (int32_t)(uint8_t)pa[qd * MR * 4 + i * 4 + t] *
                         (int32_t)pb[qd * NR * 4 + j * 4 + t];
                acc[j][i] = (int32_t)((uint32_t)acc[j][i] + (uint32_t)s);
            }
    for (int j = 0; j < NR; ++j)
        for (int i = 0; i < MR; ++i)
            out[j * MR + i] = (int32_t)((uint32_t)acc[j][i] - 128u * (uint32_t)colsum[j]);
}

/* 16-lane requant store, the f64 sequence of requant_half_avx512f. */
__attribute__((target("avx512f,avx512bw"))) static void
requant_store16(void *dst, __m512i v, double scale, int32_t zp, int32_t lo, int32_t hi) {
    __m512d sc = _mm512_set1_pd(scale), z = _mm512_set1_pd((double)zp);
    __m512d l = _mm512_set1_pd((double)lo), h = _mm512_set1_pd((double)hi);
    __m256i halves[2] = {_mm512_castsi512_si256(v), _mm512_extracti64x4_epi64(v, 1)};
    __m256i r[2];
    for (int s = 0; s < 2; ++s) {
        __m512d t = _mm512_mul_pd(_mm512_cvtepi32_pd(halves[s]), sc);
        t = _mm512_roundscale_pd(t, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
        t = _mm512_add_pd(t, z);
        t = _mm512_min_pd(_mm512_max_pd(t, l), h);
        r[s] = _mm512_cvtpd_epi32(t);
    }
    __m512i comb = _mm512_inserti64x4(_mm512_castsi256_si512(r[0]), r[1], 1);
    _mm_storeu_si128((__m128i *)dst, _mm512_cvtepi32_epi8(comb));
}

/* 16 consecutive rows of one tile column: + bias, then the vector requant store. */
__attribute__((target("avx512f,avx512bw"))) static void
requant_run16(const int32_t *src, int32_t bias, void *dst, double scale, int32_t zp, int32_t lo,
              int32_t hi) {
    __m512i v = _mm512_loadu_si512((const void *)src);
    v = _mm512_add_epi32(v, _mm512_set1_epi32(bias));
    requant_store16(dst, v, scale, zp, lo, hi);
}

typedef void (*micro_fn)(size_t, const int8_t *, const int8_t *, const int32_t *, int32_t *);

static void store_requant_tile(const int32_t *tile, size_t i0, size_t j0, size_t mr_eff,
                               size_t nr_eff, const gko_requant *q, void *c, ptrdiff_t rsc,
                               ptrdiff_t csc, int vec) {
    const int32_t lo0 = q->out_u8 ? 0 : -128, hi = q->out_u8 ? 255 : 127;
    int32_t lo = lo0;
    if (q->relu) {
        int32_t f = q->zp < lo0 ? lo0 : (q->zp > hi ? hi : q->zp);
        if (f > lo) lo = f;
    }
    for (size_t j = 0; j < nr_eff; ++j) {
        size_t col = j0 + j;
        /* vector run: unit row stride, full 16-row halves, scale constant along the run */
        if (vec && rsc == 1 && q->scale_axis != GKO_AXIS_ROW && q->bias_axis != GKO_AXIS_ROW) {
            double sc = q->scale_axis == GKO_AXIS_COL ? (double)q->scales[col] : (double)q->scale;
            int32_t bb = q->bias_axis == GKO_AXIS_COL ? q->bias[col] : 0;
            size_t i = 0;
            for (; i + 16 <= mr_eff; i += 16) {
                char *dst = (char *)c + ((ptrdiff_t)(i0 + i) + (ptrdiff_t)col * csc);
                requant_run16(tile + j * MR + i, bb, dst, sc, q->zp, lo, hi);
            }
            for (; i < mr_eff; ++i) {
                int32_t r = gko_requant_apply(tile[j * MR + i], bb, (float)sc, q->zp, lo0, hi,
                                              q->relu);
                ptrdiff_t off = (ptrdiff_t)(i0 + i) + (ptrdiff_t)col * csc;
                ((int8_t *)c)[off] = (int8_t)r;
            }
            continue;
        }
        for (size_t i = 0; i < mr_eff; ++i) {
            size_t row = i0 + i;
            int32_t bb = q->bias_axis == GKO_AXIS_ROW ? q->bias[row]
                         : q->bias_axis == GKO_AXIS_COL ? q->bias[col]
                                                        : 0;
            float sc = q->scale_axis == GKO_AXIS_ROW ? q->scales[row]
                       : q->scale_axis == GKO_AXIS_COL ? q->scales[col]
                                                       : q->scale;
            int32_t r = gko_requant_apply(tile[j * MR + i], bb, sc, q->zp, lo0, hi, q->relu);
            ((int8_t *)c)[(ptrdiff_t)row * rsc + (ptrdiff_t)col * csc] = (int8_t)r;
        }
    }
}

static void store_i32_tile(const int32_t *tile, size_t i0, size_t j0, size_t mr_eff,
                           size_t nr_eff, int32_t alpha, int32_t beta, int32_t *c, ptrdiff_t rsc,
                           ptrdiff_t csc) {
    for (size_t j = 0; j < nr_eff; ++j)
        for (size_t i = 0; i < mr_eff; ++i) {
            int32_t v = (int32_t)((uint32_t)alpha * (uint32_t)tile[j * MR + i]);
            int32_t *cp = c + (ptrdiff_t)(i0 + i) * rsc + (ptrdiff_t)(j0 + j) * csc;
            *cp = beta == 0 ? v : (int32_t)((uint32_t)beta * (uint32_t)*cp + (uint32_t)v);
        }
}

static void run_blocked(size_t m, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                        const gko_packed_rhs *pb, const gko_requant *q, int32_t alpha,
                        int32_t beta, void *c, ptrdiff_t rsc, ptrdiff_t csc, int threads) {
    size_t k = pb->k, n = pb->n;
    if (m == 0 || n == 0) return;
    size_t k_pad = pb->k_pad, nq = k_pad / 4;
    size_t mblocks = (m + MR - 1) / MR, npanels = pb->n_pad / NR;
    size_t jchunks = (npanels + JCHUNK - 1) / JCHUNK;
    int vnni = gko_cpu_has_vnni();
    micro_fn micro = vnni ? micro_vnni : micro_portable;
    int nt = gko_threads(threads);
    /* Shared A pre-pack (gemmkit/src/driver.rs:763), then the job loop. */
    int8_t *pa = (int8_t *)aligned_alloc(64, round_up(mblocks * MR * k_pad + 64, 64));
#pragma omp parallel for num_threads(nt) schedule(static)
    for (size_t ib = 0; ib < mblocks; ++ib)
        pack_a_block(pa + ib * MR * k_pad, a, rsa, csa, m, k, k_pad, ib * MR);
    size_t njobs = mblocks * jchunks;
#pragma omp parallel num_threads(nt)
    {
        int32_t tile[MR * NR] __attribute__((aligned(64)));
#pragma omp for schedule(dynamic, 1)
        for (size_t job = 0; job < njobs; ++job) {
            size_t ib = job / jchunks, jc = job % jchunks;
            size_t i0 = ib * MR, mr_eff = m - i0 < MR ? m - i0 : MR;
            for (size_t jp = jc * JCHUNK; jp < npanels && jp < (jc + 1) * JCHUNK; ++jp) {
                size_t j0 = jp * NR, nr_eff = n - j0 < NR ? n - j0 : NR;
                micro(nq, pa + ib * MR * k_pad, pb->buf + jp * NR * k_pad, pb->colsum + j0, tile);
                if (q)
                    store_requant_tile(tile, i0, j0, mr_eff, nr_eff, q, c, rsc, csc, vnni);
                else
                    store_i32_tile(tile, i0, j0, mr_eff, nr_eff, alpha, beta, (int32_t *)c, rsc,
                                   csc);
            }
        }
    }
    free(pa);
}

void gko_vnni_gemm_i8_requant_packed(size_t m, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                     const gko_packed_rhs *pb, const gko_requant *q, void *c,
                                     ptrdiff_t rsc, ptrdiff_t csc, int threads) {
    if (pb->k == 0) { /* requant_degenerate: the map of a zero accumulator */
        gko_gemm_i8_requant(m, 0, pb->n, a, rsa, csa, NULL, 0, 0, q, c, rsc, csc);
        return;
    }
    run_blocked(m, a, rsa, csa, pb, q, 1, 0, c, rsc, csc, threads);
}

void gko_vnni_gemm_i8_packed(size_t m, int32_t alpha, const int8_t *a, ptrdiff_t rsa,
                             ptrdiff_t csa, const gko_packed_rhs *pb, int32_t beta, int32_t *c,
                             ptrdiff_t rsc, ptrdiff_t csc, int threads) {
    if (pb->k == 0 || alpha == 0) {
        gko_gemm_i8(m, 0, pb->n, alpha, a, rsa, csa, NULL, 0, 0, beta, c, rsc, csc);
        return;
    }
    run_blocked(m, a, rsa, csa, pb, NULL, alpha, beta, c, rsc, csc, threads);
}

/* ---- bf16 -> f32 ----------------------------------------------------------------- */

#define BMR 32
#define BNR 12

__attribute__((target("avx512f,avx512bf16"))) static void
micro_bf16(size_t npairs, const uint16_t *pa, const uint16_t *pb, float *out) {
    __m512 acc[BNR][2];
    for (int j = 0; j < BNR; ++j) acc[j][0] = acc[j][1] = _mm512_setzero_ps();
    for (size_t pr = 0; pr < npairs; ++pr) {
        __m512bh a0 = (__m512bh)_mm512_loadu_si512((const void *)(pa + pr * BMR * 2));
        __m512bh a1 = (__m512bh)_mm512_loadu_si512((const void *)(pa + pr * BMR * 2 + 32));
        for (int j = 0; j < BNR; ++j) {
            int32_t w;
            memcpy(&w, pb + pr * BNR * 2 + j * 2, 4);
            __m512bh bj = (__m512bh)_mm512_set1_epi32(w);
            acc[j][0] = _mm512_dpbf16_ps(acc[j][0], a0, bj);
            acc[j][1] = _mm512_dpbf16_ps(acc[j][1], a1, bj);
        }
    }
    for (int j = 0; j < BNR; ++j) {
        _mm512_storeu_ps(out + j * BMR, acc[j][0]);
        _mm512_storeu_ps(out + j * BMR + 16, acc[j][1]);
    }
}

static void micro_bf16_portable(size_t npairs, const uint16_t *pa, const uint16_t *pb,
                                float *out) {
    float acc[BNR][BMR];
    memset(acc, 0, sizeof(acc));
    for (size_t pr = 0; pr < npairs; ++pr)
        for (int j = 0; j < BNR; ++j)
            for (int i = 0; i < BMR; ++i)
                for (int t = 0; t < 2; ++t)
                    acc[j][i] += gko_bf16_to_f32(pa[pr * BMR * 2 + i * 2 + t]) *
                                 gko_bf16_to_f32(pb[pr * BNR * 2 + j * 2 + t]);
    for (int j = 0; j < BNR; ++j)
        for (int i = 0; i < BMR; ++i) out[j * BMR + i] = acc[j][i];
}

void gko_cpu_gemm_bf16_f32(size_t m, size_t k, size_t n, float alpha, const uint16_t *a,
                           ptrdiff_t rsa, ptrdiff_t csa, const uint16_t *b, ptrdiff_t rsb,
                           ptrdiff_t csb, float beta, float *c, ptrdiff_t rsc, ptrdiff_t csc,
                           int threads) {
    if (m == 0 || n == 0) return;
    size_t k_pad = round_up(k ? k : 2, 2), npairs = k_pad / 2;
    size_t mblocks = (m + BMR - 1) / BMR, npanels = (n + BNR - 1) / BNR;
    int nt = gko_threads(threads);
    uint16_t *pa = (uint16_t *)aligned_alloc(64, round_up(mblocks * BMR * k_pad * 2 + 64, 64));
    uint16_t *pb = (uint16_t *)aligned_alloc(64, round_up(npanels * BNR * k_pad * 2 + 64, 64));
#pragma omp parallel for num_threads(nt) schedule(static)
    for (size_t ib = 0; ib < mblocks; ++ib)
        for (size_t pr = 0; pr < npairs; ++pr)
            for (size_t i = 0; i < BMR; ++i)
                for (size_t t = 0; t < 2; ++t) {
                    size_t row = ib * BMR + i, p = pr * 2 + t;
                    pa[ib * BMR * k_pad + pr * BMR * 2 + i * 2 + t] =
                        (row < m && p < k) ? a[(ptrdiff_t)row * rsa + (ptrdiff_t)p * csa] : 0;
                }
#pragma omp parallel for num_threads(nt) schedule(static)
    for (size_t jp = 0; jp < npanels; ++jp)
        for (size_t pr = 0; pr < npairs; ++pr)
            for (size_t j = 0; j < BNR; ++j)
                for (size_t t = 0; t < 2; ++t) {
                    size_t col = jp * BNR + j, p = pr * 2 + t;
                    pb[jp * BNR * k_pad + pr * BNR * 2 + j * 2 + t] =
                        (col < n && p < k) ? b[(ptrdiff_t)p * rsb + (ptrdiff_t)col * csb] : 0;
                }
    int hw = cpu_has_avx512bf16();
    size_t jchunks = (npanels + JCHUNK - 1) / JCHUNK, njobs = mblocks * jchunks;
#pragma omp parallel num_threads(nt)
    {
        float tile[BMR * BNR] __attribute__((aligned(64)));
#pragma omp for schedule(dynamic, 1)
        for (size_t job = 0; job < njobs; ++job) {
            size_t ib = job / jchunks, jc = job % jchunks;
            size_t i0 = ib * BMR, mr_eff = m - i0 < BMR ? m - i0 : BMR;
            for (size_t jp = jc * JCHUNK; jp < npanels && jp < (jc + 1) * JCHUNK; ++jp) {
                size_t j0 = jp * BNR, nr_eff = n - j0 < BNR ? n - j0 : BNR;
                if (hw)
                    micro_bf16(npairs, pa + ib * BMR * k_pad, pb + jp * BNR * k_pad, tile);
                else
                    micro_bf16_portable(npairs, pa + ib * BMR * k_pad, pb + jp * BNR * k_pad,
                                        tile);
                for (size_t j = 0; j < nr_eff; ++j)
                    for (size_t i = 0; i < mr_eff; ++i) {
                        float *cp = c + (ptrdiff_t)(i0 + i) * rsc + (ptrdiff_t)(j0 + j) * csc;
                        float v = alpha * tile[j * BMR + i];
                        *cp = beta == 0.0f ? v : v + beta * *cp;
                    }
            }
        }
    }
    free(pa);
    free(pb);
}
