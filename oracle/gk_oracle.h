/*
 * gk_oracle.h -- CPU restatement of gemmkit's quantized-inference GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA engine in
 * gemmkit_b200/ and the timed CPU baseline of bench.py. Only tests/, the smoke check in
 * __graft_entry__.py and bench.py's CPU-baseline / reference legs may load it. The product
 * path (libgemmkit_cuda.so) never links, loads or calls anything here.
 *
 * Parity pin: gemmkit (Rust, v0.1.2) cannot be built in this environment (no Rust
 * toolchain), so this file restates its algorithm in C. The restatement is pinned against
 * the known-answer vectors the reference's own tests hard-code and against the reference
 * tests' independent round_ties_even model run on the reference tests' own xorshift*
 * inputs (tests/golden/, tests/test_oracle.py).
 *
 * Every function names the gemmkit source it follows (paths relative to the gemmkit
 * workspace root).
 */
#ifndef GK_ORACLE_H
#define GK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Axis selectors for the requant bias / scale lookups (gemmkit BiasDim / ScaleSpec,
 * gemmkit/src/kernel/epilogue.rs:205-250). */
enum { GKO_AXIS_NONE = 0, GKO_AXIS_ROW = 1, GKO_AXIS_COL = 2 };

/* Requant parameters in the user frame. scale_axis NONE means per-tensor `scale`.
 * lo/hi are the QuantOut band (i8: -128/127, u8: 0/255,
 * gemmkit/src/kernel/epilogue.rs:738-765). relu raises the lower clamp to clamp(zp). */
typedef struct gko_requant {
    float scale;
    const float *scales;
    int32_t scale_axis;
    int32_t zp;
    const int32_t *bias;
    int32_t bias_axis;
    int32_t relu;
    int32_t out_u8;
} gko_requant;

/* round_ne_f64, gemmkit/src/kernel/epilogue.rs:886-897 (the 2^52 add/subtract trick). */
double gko_round_ne_f64(double x);

/* KRequantize::apply, gemmkit/src/kernel/epilogue.rs:810-830, returning the clamped value
 * (the caller narrows to the output byte). relu: max(q, clamp(zp, lo, hi)). */
int32_t gko_requant_apply(int32_t v, int32_t bias, float scale, int32_t zp, int32_t lo,
                          int32_t hi, int32_t relu);

/* gemm_i8 semantics: execute_int + scale_c_int + int32_epilogue
 * (gemmkit/src/dispatch/int.rs:131-163, gemmkit/src/kernel/int.rs:36-120).
 * C <- alpha*A*B + beta*C with wrapping i32 arithmetic; beta == 0 never reads C. */
void gko_gemm_i8(size_t m, size_t k, size_t n, int32_t alpha, const int8_t *a, ptrdiff_t rsa,
                 ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, int32_t beta,
                 int32_t *c, ptrdiff_t rsc, ptrdiff_t csc);

/* gemm_i8_requant / gemm_i8_requant_u8 semantics with independent bias / scale axes:
 * execute_int_requant + requant_degenerate + KRequantize::apply
 * (gemmkit/src/dispatch/int.rs:672-752, gemmkit/src/kernel/epilogue.rs:810-830).
 * c points to int8_t (out_u8 == 0) or uint8_t (out_u8 == 1). */
void gko_gemm_i8_requant(size_t m, size_t k, size_t n, const int8_t *a, ptrdiff_t rsa,
                         ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb,
                         const gko_requant *q, void *c, ptrdiff_t rsc, ptrdiff_t csc);

/* The exact i32 accumulator sum_k A[i,k]*B[k,j] (wrapping), written to acc (row-major m x n). */
void gko_acc_i8(size_t m, size_t k, size_t n, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, int32_t *acc);

/* Half-precision helpers. bf16/f16 -> f32 widening is exact; f32 -> bf16 is
 * round-to-nearest-even with NaN kept quiet (the `half` 2.7.1 crate's from_f32, called at
 * gemmkit/src/scalar.rs:240-249). */
float gko_bf16_to_f32(uint16_t h);
float gko_f16_to_f32(uint16_t h);
uint16_t gko_f32_to_bf16(float f);

/* f64 reference dot for the bf16/f16 -> f32 GEMM (the accuracy oracle the reference's
 * mixed tests use, gemmkit/tests/oracle_common/mod.rs:158-219):
 * out[i*n + j] = alpha * sum_k widen(A[i,k]) * widen(B[k,j]) + beta * c_in[i,j] in f64.
 * is_f16 selects f16 inputs (else bf16). c_in may be NULL when beta == 0. */
void gko_gemm_half_f64(int is_f16, size_t m, size_t k, size_t n, double alpha,
                       const uint16_t *a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t *b,
                       ptrdiff_t rsb, ptrdiff_t csb, double beta, const float *c_in,
                       ptrdiff_t rsc, ptrdiff_t csc, double *out);

/* ---- timed CPU baseline: restatement of gemmkit's AVX-512 VNNI blocked path ---------- */

/* 1 when this host can run the VNNI restatement (avx512f+bw+vnni), else 0; the baseline
 * then runs the same blocking with a portable dot. */
int gko_cpu_has_vnni(void);

/* Prepacked RHS in gemmkit's VNNI k-quad-interleaved layout (gemmkit/src/pack.rs:117-200,
 * width NR = 12, Q = 4, pad 0), kc = k (gemmkit/src/api/packed.rs:411-419). */
typedef struct gko_packed_rhs {
    int8_t *buf;
    int32_t *colsum; /* per-column sum_k B, the +128 correction (simd/avx512.rs:483-550) */
    size_t k, n, k_pad, n_pad;
} gko_packed_rhs;

int gko_vnni_prepack(const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, size_t k, size_t n,
                     gko_packed_rhs *out);
void gko_vnni_packed_free(gko_packed_rhs *p);

/* C(i8/u8) = requant(A * packedB) over `threads` OpenMP workers (0 = all). Row-block x
 * column-panel jobs as gemmkit's driver (gemmkit/src/driver.rs:779-910); requant store in
 * f64 as requant_store_avx512f (gemmkit/src/simd/avx512.rs:274-324). */
void gko_vnni_gemm_i8_requant_packed(size_t m, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                     const gko_packed_rhs *pb, const gko_requant *q, void *c,
                                     ptrdiff_t rsc, ptrdiff_t csc, int threads);

/* C(i32) = alpha*A*packedB + beta*C, same blocking. */
void gko_vnni_gemm_i8_packed(size_t m, int32_t alpha, const int8_t *a, ptrdiff_t rsa,
                             ptrdiff_t csa, const gko_packed_rhs *pb, int32_t beta, int32_t *c,
                             ptrdiff_t rsc, ptrdiff_t csc, int threads);

/* bf16 x bf16 -> f32 blocked baseline (alpha*acc + beta*C), f32 accumulation with
 * 2-depth-step pair products as vdpbf16ps (gemmkit/src/simd/avx512.rs:554-644). */
void gko_cpu_gemm_bf16_f32(size_t m, size_t k, size_t n, float alpha, const uint16_t *a,
                           ptrdiff_t rsa, ptrdiff_t csa, const uint16_t *b, ptrdiff_t rsb,
                           ptrdiff_t csb, float beta, float *c, ptrdiff_t rsc, ptrdiff_t csc,
                           int threads);

/* Number of OpenMP threads the baseline uses for `threads` (0 = all). */
int gko_threads(int threads);

#ifdef __cplusplus
}
#endif
#endif
