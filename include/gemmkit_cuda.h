/*
 * gemmkit_cuda.h -- C ABI of the B200 (sm_100a) engine for gemmkit's quantized-inference
 * GEMM path.
 *
 * Every entry mirrors a gemmkit (Rust, v0.1.2) API function: same name after the `gk_`
 * prefix, same argument order and meaning (element strides as signed `ptrdiff_t`, `rs`/`cs`
 * views, `beta == 0` never reads C), plus a trailing CUDA stream. Pointers are DEVICE
 * pointers. Calls are asynchronous on `stream` (NULL = the legacy default stream); they
 * never unwind and return a status code. Where gemmkit panics with a `gemmkit:` message,
 * the entry returns GK_EINVAL and gk_last_error() returns the same message.
 *
 * Two tiers, as in gemmkit:
 *   - checked entries take gk_matref / gk_matmut views (a slice length plus rows, cols and
 *     strides, exactly MatRef / MatMut, gemmkit/src/api.rs:99-118) and run gemmkit's
 *     validation (gemmkit/src/api.rs:188-315, gemmkit/src/adapter.rs:190-280);
 *   - `_unchecked` entries take raw pointers and strides (negative strides allowed) and
 *     trust the caller, as gemmkit's `*_unchecked` functions do.
 *
 * Extensions beyond gemmkit (no counterpart there, see the notes on each): independent
 * bias / scale axes and ReLU in the requant descriptor, packed-B requant entries, i8
 * batched entries, and the f32-output bf16/f16 GEMM.
 */
#ifndef GEMMKIT_CUDA_H
#define GEMMKIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
    GK_OK = 0,
    GK_EINVAL = 1,   /* argument rejected (the gemmkit panic cases) */
    GK_ENOMEM = 2,   /* device allocation failed */
    GK_ECUDA = 3,    /* a CUDA runtime/driver call failed */
    GK_ETIMEOUT = 4, /* a bounded device wait gave up (see gk_device_status) */
    GK_ENODEV = 5,   /* no sm_100 device, or the kernels are not loadable */
};

typedef void *gk_stream_t; /* a cudaStream_t */

/* gemmkit::Parallelism (gemmkit/src/parallel.rs:25-39). On the device the engine always
 * uses the whole GPU; the value is accepted for API parity and otherwise ignored. */
typedef enum { GK_PAR_SERIAL = 0, GK_PAR_RAYON = 1 } gk_par_kind;
typedef struct {
    int32_t kind;    /* gk_par_kind */
    int32_t threads; /* Rayon(n): n; 0 = all */
} gk_parallelism;

/* gemmkit::Workspace (gemmkit/src/workspace.rs:53-190): reusable device scratch for the
 * operand packs a call may need. NULL selects a per-thread, per-device default. */
typedef struct gk_workspace gk_workspace;

/* gemmkit::PackedRhs<i8> (gemmkit/src/api/packed.rs:34-41): B packed once on the device
 * into the engine's K-major tile layout, read-only, shareable across streams. */
typedef struct gk_packed_rhs gk_packed_rhs;

/* Checked views: element (i, j) at data[i*rs + j*cs]; `len` is the slice length in
 * elements (gemmkit MatRef / MatMut, gemmkit/src/api.rs:99-118). */
typedef struct {
    const void *data;
    size_t len;
    size_t rows, cols;
    ptrdiff_t rs, cs;
} gk_matref;
typedef struct {
    void *data;
    size_t len;
    size_t rows, cols;
    ptrdiff_t rs, cs;
} gk_matmut;

/* Requant axis of a bias or scale vector, in the user's (row, col) frame. */
typedef enum { GK_AXIS_NONE = 0, GK_AXIS_ROW = 1, GK_AXIS_COL = 2 } gk_axis;

/* Extended requant descriptor (extension of gemmkit::Requantize,
 * gemmkit/src/api/int8.rs:185-209): gemmkit ties bias and scales to the row axis; here each
 * has its own axis (per-row, per-column, or none / per-tensor), and `relu` raises the
 * lower clamp to clamp(zero_point), which equals requantizing max(acc + bias, 0). */
typedef struct {
    float scale;           /* per-tensor scale, used when scale_axis == GK_AXIS_NONE */
    const float *scales;   /* device vector, length m (ROW) or n (COL) */
    int32_t scale_axis;    /* gk_axis */
    int32_t zero_point;    /* [-128, 127] for i8 output, [0, 255] for u8 */
    const int32_t *bias;   /* device vector, length m (ROW) or n (COL); NULL = none */
    int32_t bias_axis;     /* gk_axis */
    int32_t relu;          /* nonzero: ReLU before requantization */
    size_t scales_len;     /* checked tier only: slice lengths of scales / bias */
    size_t bias_len;
} gk_requant;

/* ---- library -------------------------------------------------------------------------- */

const char *gk_version(void);
/* Thread-local text of the last error returned by an entry on this thread. */
const char *gk_last_error(void);
/* Read (and with clear != 0 reset) the device status word of `device`: nonzero bits mean a
 * bounded in-kernel wait gave up (GK_ETIMEOUT). Synchronizes the device. */
int gk_device_status(int device, int clear, uint32_t *status);

int gk_workspace_create(gk_workspace **out);
void gk_workspace_free(gk_workspace *ws);

/* ---- i8 -> i32 ----------------------------------------------------------------------- */

/* gemm_i8_unchecked_with (gemmkit/src/api/int8.rs:136-178):
 * C(i32) <- alpha*A(i8)*B(i8) + beta*C, wrapping on overflow. */
int gk_gemm_i8_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n, int32_t alpha,
                         const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b,
                         ptrdiff_t rsb, ptrdiff_t csb, int32_t beta, int32_t *c, ptrdiff_t rsc,
                         ptrdiff_t csc, gk_parallelism par, gk_stream_t stream);

/* gemm_i8_with (gemmkit/src/api/int8.rs:38-84): validate_gemm_views, then the above. */
int gk_gemm_i8(gk_workspace *ws, int32_t alpha, gk_matref a, gk_matref b, int32_t beta,
               gk_matmut c, gk_parallelism par, gk_stream_t stream);

/* ---- i8 -> i8 / u8 requantized ------------------------------------------------------- */

/* gemm_i8_requant_unchecked_with (gemmkit/src/api/int8.rs:404-457):
 * C(i8) <- clamp(zp + round_ne(scale*(A*B + bias[i])), -128, 127), f64 scale step. */
int gk_gemm_i8_requant_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n,
                                 const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b,
                                 ptrdiff_t rsb, ptrdiff_t csb, float scale,
                                 const float *row_scales, int has_row_scales, int32_t zero_point,
                                 const int32_t *bias, int has_bias, int8_t *c, ptrdiff_t rsc,
                                 ptrdiff_t csc, gk_parallelism par, gk_stream_t stream);

/* gemm_i8_requant_u8_unchecked_with (gemmkit/src/api/int8.rs:619-672): u8 output [0, 255]. */
int gk_gemm_i8_requant_u8_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n,
                                    const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                    const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, float scale,
                                    const float *row_scales, int has_row_scales,
                                    int32_t zero_point, const int32_t *bias, int has_bias,
                                    uint8_t *c, ptrdiff_t rsc, ptrdiff_t csc, gk_parallelism par,
                                    gk_stream_t stream);

/* gemm_i8_requant_with / gemm_i8_requant_u8_with (gemmkit/src/api/int8.rs:280-338,
 * 495-552): the checked tier with gemmkit's validation and wording (per-row scales and bias
 * when the descriptor's axes are ROW; other axes are the extension). out_u8 selects the u8
 * entry. */
int gk_gemm_i8_requant(gk_workspace *ws, gk_matref a, gk_matref b, const gk_requant *req,
                       gk_matmut c, int out_u8, gk_parallelism par, gk_stream_t stream);

/* Extension: the raw tier with the extended descriptor (independent axes, ReLU). */
int gk_gemm_i8_requant_ex_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n,
                                    const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                    const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb,
                                    const gk_requant *req, void *c, ptrdiff_t rsc, ptrdiff_t csc,
                                    int out_u8, gk_parallelism par, gk_stream_t stream);

/* ---- prepacked B ------------------------------------------------------------------------ */

/* prepack_rhs_i8_unchecked (gemmkit/src/api/packed.rs:386-453): pack a k x n device B once;
 * the pack runs on `stream`. */
int gk_prepack_rhs_i8_unchecked(const int8_t *b, ptrdiff_t rsb, ptrdiff_t csb, size_t k,
                                size_t n, gk_stream_t stream, gk_packed_rhs **out);
/* prepack_rhs_i8 (gemmkit/src/api/packed.rs:372-384): check_view on B, then the above. */
int gk_prepack_rhs_i8(gk_matref b, gk_stream_t stream, gk_packed_rhs **out);
void gk_packed_rhs_free(gk_packed_rhs *p);
size_t gk_packed_rhs_rows(const gk_packed_rhs *p); /* PackedRhs::rows (k) */
/* No counterpart in gemmkit (its PackedRhs lives only in memory): store a packed B and load it
 * back, so weights are packed once and later loaded device-ready. gk_packed_rhs_serialize
 * writes a 64-byte header (magic "GKPACK01", k, n, padded dimensions, layout tag) plus the
 * packed bytes into host memory `out` of `cap` bytes (out == NULL: only set *needed).
 * gk_packed_rhs_deserialize checks the header (magic, layout, dimensions, length) and returns
 * a new handle on the current device, complete when it returns. */
int gk_packed_rhs_serialize(const gk_packed_rhs *p, void *out, size_t cap, size_t *needed);
int gk_packed_rhs_deserialize(const void *in, size_t len, gk_stream_t stream,
                              gk_packed_rhs **out);
size_t gk_packed_rhs_cols(const gk_packed_rhs *p); /* PackedRhs::cols (n) */

/* gemm_i8_packed_b_unchecked_with (gemmkit/src/api/packed.rs:609-680): C(i32) <- alpha *
 * A * packedB + beta*C. Like gemmkit, rejects a C that is not column-major-ish
 * (|csc| < |rsc|) with gemmkit's message. */
int gk_gemm_i8_packed_b_unchecked(gk_workspace *ws, int32_t alpha, size_t m, const int8_t *a,
                                  ptrdiff_t rsa, ptrdiff_t csa, const gk_packed_rhs *packed,
                                  int32_t beta, int32_t *c, ptrdiff_t rsc, ptrdiff_t csc,
                                  gk_parallelism par, gk_stream_t stream);
/* gemm_i8_packed_b_with (gemmkit/src/api/packed.rs:493-571). */
int gk_gemm_i8_packed_b(gk_workspace *ws, int32_t alpha, gk_matref a,
                        const gk_packed_rhs *packed, int32_t beta, gk_matmut c,
                        gk_parallelism par, gk_stream_t stream);

/* Extension (gemmkit has no packed requant entry; dispatch/int.rs:5): requantized product
 * with a prepacked B, any C orientation. Bit-identical to gk_gemm_i8_requant_ex_unchecked
 * on the unpacked B. Small m takes the bandwidth-bound small-M kernel shape. */
int gk_gemm_i8_packed_b_requant_unchecked(gk_workspace *ws, size_t m, const int8_t *a,
                                          ptrdiff_t rsa, ptrdiff_t csa,
                                          const gk_packed_rhs *packed, const gk_requant *req,
                                          void *c, ptrdiff_t rsc, ptrdiff_t csc, int out_u8,
                                          gk_parallelism par, gk_stream_t stream);

/* The decode-step GEMV. gemmkit reaches its small-shape route only from inside dispatch
 * (special/small_mn.rs:834-1060, gated at dispatch.rs:438-482); this entry names it:
 * C = requant(A * packedB) for 1 <= m <= 64 activation rows. When the packed side is the
 * wider one (n > m) this runs on the bandwidth-bound small-M kernel that streams the
 * prepacked weights once from HBM (unless GEMMKIT_CUDA_GEMV=0); when n <= m both sides are
 * at most 64 wide and the product goes to the general tile kernel. Arguments and results as
 * gk_gemm_i8_packed_b_requant_unchecked; m outside [1, 64] is GK_EINVAL. */
int gk_gemv_i8_requant_unchecked(gk_workspace *ws, size_t m, const int8_t *a, ptrdiff_t rsa,
                                 ptrdiff_t csa, const gk_packed_rhs *packed,
                                 const gk_requant *req, void *c, ptrdiff_t rsc, ptrdiff_t csc,
                                 int out_u8, gk_stream_t stream);

/* ---- batched (extension: gemmkit's batched entries are float-only, api/batched.rs:188) -- */

/* Strided batch of independent requantized products, shaped as gemmkit's
 * gemm_batched_unchecked_with (gemmkit/src/api/batched.rs:649): element e uses
 * A + e*a_bs, B + e*b_bs, C + e*c_bs, and the bias / scales vectors at + e*bias_bs /
 * + e*scales_bs (0 = shared by every element). */
int gk_gemm_i8_requant_batched_unchecked(gk_workspace *ws, size_t batch, size_t m, size_t k,
                                         size_t n, const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                                         ptrdiff_t a_bs, const int8_t *b, ptrdiff_t rsb,
                                         ptrdiff_t csb, ptrdiff_t b_bs, const gk_requant *req,
                                         ptrdiff_t bias_bs, ptrdiff_t scales_bs, void *c,
                                         ptrdiff_t rsc, ptrdiff_t csc, ptrdiff_t c_bs, int out_u8,
                                         gk_parallelism par, gk_stream_t stream);

/* Pointer-array batch, shaped as gemm_batched_ptr_unchecked over GemmProblem
 * (gemmkit/src/api/batched.rs:711-760, gemmkit/src/dispatch.rs:135). */
typedef struct {
    size_t m, k, n;
    const int8_t *a;
    ptrdiff_t rsa, csa;
    const int8_t *b;
    ptrdiff_t rsb, csb;
    void *c;
    ptrdiff_t rsc, csc;
    gk_requant req;
} gk_i8_requant_problem;
int gk_gemm_i8_requant_batched_ptr_unchecked(gk_workspace *ws,
                                             const gk_i8_requant_problem *problems,
                                             size_t count, int out_u8, gk_parallelism par,
                                             gk_stream_t stream);

/* ---- half -> f32 (extension: gemmkit's gemm::<bf16> writes bf16, dispatch/mixed.rs:1395;
 * its f32-output family is the internal deep-k twin, dispatch/mixed.rs:97-221) ---------- */

/* C(f32) <- alpha*A*B + beta*C with bf16 (or f16) A and B, f32 accumulation; beta == 0
 * never reads C. Argument order as gemm_unchecked (gemmkit/src/api.rs:469). */
int gk_gemm_bf16_f32_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n, float alpha,
                               const uint16_t *a, ptrdiff_t rsa, ptrdiff_t csa,
                               const uint16_t *b, ptrdiff_t rsb, ptrdiff_t csb, float beta,
                               float *c, ptrdiff_t rsc, ptrdiff_t csc, gk_parallelism par,
                               gk_stream_t stream);
int gk_gemm_f16_f32_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n, float alpha,
                              const uint16_t *a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t *b,
                              ptrdiff_t rsb, ptrdiff_t csb, float beta, float *c, ptrdiff_t rsc,
                              ptrdiff_t csc, gk_parallelism par, gk_stream_t stream);
/* Checked tier (gemm_with, gemmkit/src/api.rs:400-466 validation). is_f16 selects f16. */
int gk_gemm_half_f32(gk_workspace *ws, int is_f16, float alpha, gk_matref a, gk_matref b,
                     float beta, gk_matmut c, gk_parallelism par, gk_stream_t stream);

/* Strided batch of half -> f32 products (gemm_batched_unchecked_with shape,
 * gemmkit/src/api/batched.rs:649). */
int gk_gemm_half_f32_batched_unchecked(gk_workspace *ws, int is_f16, size_t batch, size_t m,
                                       size_t k, size_t n, float alpha, const uint16_t *a,
                                       ptrdiff_t rsa, ptrdiff_t csa, ptrdiff_t a_bs,
                                       const uint16_t *b, ptrdiff_t rsb, ptrdiff_t csb,
                                       ptrdiff_t b_bs, float beta, float *c, ptrdiff_t rsc,
                                       ptrdiff_t csc, ptrdiff_t c_bs, gk_parallelism par,
                                       gk_stream_t stream);

/* ---- fused float epilogue on the half -> f32 GEMM ------------------------------------- */

/* gemmkit's gemm_fused (gemmkit/src/api/fused.rs:149-176) computes act(alpha*A*B + beta*C +
 * bias) for f32/f64 GEMMs: the bias per row (length m) or per column (length n), then ReLU or
 * LeakyReLU(slope) (gemmkit/src/kernel/epilogue.rs:258-330). These entries give the bf16 /
 * f16 -> f32 GEMM the same fused epilogue (gemmkit has none for half inputs): the unchecked
 * tier takes gemm_fused_unchecked's (bias, bias_dim, has_bias, act) selectors, the checked
 * tier validates the views like gk_gemm_half_f32 and the bias length like gemmkit. With k == 0
 * or alpha == 0, C <- act(beta*C + bias) (gemmkit/src/dispatch/float.rs:671-676). */
enum gk_act { GK_ACT_NONE = 0, GK_ACT_RELU = 1, GK_ACT_LEAKY_RELU = 2 };
int gk_gemm_half_f32_fused_unchecked(gk_workspace *ws, int is_f16, size_t m, size_t k, size_t n,
                                     float alpha, const uint16_t *a, ptrdiff_t rsa,
                                     ptrdiff_t csa, const uint16_t *b, ptrdiff_t rsb,
                                     ptrdiff_t csb, float beta, float *c, ptrdiff_t rsc,
                                     ptrdiff_t csc, const float *bias, int bias_dim,
                                     int has_bias, int act, float leak, gk_parallelism par,
                                     gk_stream_t stream);
int gk_gemm_half_f32_fused(gk_workspace *ws, int is_f16, float alpha, gk_matref a, gk_matref b,
                           float beta, gk_matmut c, const float *bias, size_t bias_len,
                           int bias_dim, int act, float leak, gk_parallelism par,
                           gk_stream_t stream);

/* ---- fused i32 epilogue on the i8 -> i32 GEMM ------------------------------------------ */

/* The integer counterpart of gk_gemm_half_f32_fused: C = act(alpha*A*B + beta*C + bias) with
 * i8 operands and i32 C, every step wrapping mod 2^32 as gemmkit's int32_epilogue does
 * (gemmkit/src/kernel/int.rs:36-120), the i32 bias per row (length m) or per column (length
 * n), then ReLU as max(v, 0) on the signed value. gemmkit's FusedEpi (gemmkit/src/kernel/
 * epilogue.rs:258-330) composes bias-then-activation for float GEMMs only; this entry applies
 * the same composition to gemm_i8 (gemmkit/src/api/int8.rs:136-178) inside the GEMM's
 * epilogue. act is GK_ACT_NONE or GK_ACT_RELU (GK_ACT_LEAKY_RELU is GK_EINVAL: its slope is a
 * float). With k == 0 or alpha == 0, C <- act(beta*C + bias). The checked tier validates the
 * views like gk_gemm_i8 and the bias length like gk_gemm_half_f32_fused. */
int gk_gemm_i8_fused_unchecked(gk_workspace *ws, size_t m, size_t k, size_t n, int32_t alpha,
                               const int8_t *a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b,
                               ptrdiff_t rsb, ptrdiff_t csb, int32_t beta, int32_t *c,
                               ptrdiff_t rsc, ptrdiff_t csc, const int32_t *bias, int bias_dim,
                               int has_bias, int act, gk_parallelism par, gk_stream_t stream);
int gk_gemm_i8_fused(gk_workspace *ws, int32_t alpha, gk_matref a, gk_matref b, int32_t beta,
                     gk_matmut c, const int32_t *bias, size_t bias_len, int bias_dim, int act,
                     gk_parallelism par, gk_stream_t stream);

/* ---- producer step: f32 activations -> i8 (no counterpart in gemmkit) ---------------- */

/* Quantize a rows x cols f32 view (element (i, j) at x[i*rsx + j*csx]) into i8 (q[i*rsq +
 * j*csq]), the step that feeds the requantizing GEMMs: q = saturate_i8(zp +
 * round_half_even(f64(x) / f64(scale))) in f64, NaN -> zp. With row_scales == NULL one
 * per-tensor scale / zero_point (scale must be finite and > 0, zp in [-128, 127], as
 * gemmkit's requant checks them); otherwise each row gets scale_r = max |x_r| / 127 (1 for an
 * all-zero row), written to row_scales[i], with zero point 0 (symmetric, per token). */
int gk_quantize_f32_i8_unchecked(size_t rows, size_t cols, const float *x, ptrdiff_t rsx,
                                 ptrdiff_t csx, int8_t *q, ptrdiff_t rsq, ptrdiff_t csq,
                                 float scale, int32_t zero_point, float *row_scales,
                                 gk_stream_t stream);

/* ---- tuning (the gemmkit-tune profile mechanism, gemmkit/src/tuning.rs:592-621) ------- */

/* Force the tile width (N of the MMA: 16, 32, 64, 128, 192 or 256) for later calls on this
 * thread; 0 drops this thread's override, so the process-wide GEMMKIT_CUDA_BN knob applies
 * again (its default, 0, chooses the width per shape). */
int gk_set_tile_n(int bn);

/* The engine's knobs, the counterpart of gemmkit's tuning getters / setters
 * (gemmkit/src/tuning.rs:660-690): a compiled default, an environment override read once
 * (`export GEMMKIT_CUDA_...=v`, the form the tuner's profile uses) and a process-wide run-time
 * override. gk_knob_names lists them (comma-separated): GEMMKIT_CUDA_BN (0 = per shape, or 16,
 * 32, 64, 128, 192, 256), GEMMKIT_CUDA_PAIR, GEMMKIT_CUDA_GEMV, GEMMKIT_CUDA_PDL,
 * GEMMKIT_CUDA_STREAMK, GEMMKIT_CUDA_GEMV_SK, GEMMKIT_CUDA_EPI16, GEMMKIT_CUDA_MN_B,
 * GEMMKIT_CUDA_REQUANT_F32 (0 / 1),
 * GEMMKIT_CUDA_BN_SHORTK (as GEMMKIT_CUDA_BN), GEMMKIT_CUDA_STAGES (0 or 2 .. 12) and
 * GEMMKIT_CUDA_GEMV_SPLIT (0 .. 8). gk_knob_set with a negative value drops the run-time override;
 * an unknown name or an out-of-range value returns GK_EINVAL. */
const char *gk_knob_names(void);
int gk_knob_get(const char *name, int64_t *value);
int gk_knob_set(const char *name, int64_t value);

/* ---- i8 -> i32 without allocation ------------------------------------------------------ */

/* No counterpart in gemmkit. The i8 -> i32 product of gk_gemm_i8_unchecked (same arguments
 * minus the workspace and Parallelism, same result bytes) for callers that must not
 * allocate device memory: hosts that give the GPU a fixed budget through their own
 * allocator, or latency-critical loops where cudaMalloc / cudaFree could synchronise the
 * device. Operands that need packing (not K-contiguous or not 16-byte aligned) are packed
 * into one file-scope device array of GK_NOALLOC_SCRATCH_BYTES, which every GPU that loads
 * the library holds until exit; a call whose packs need more returns GK_EINVAL. The first
 * call on a device looks up that array's device address; make it before any stream capture.
 * All calls share the array: calls that overlap on the GPU race, so order them on one
 * stream. Never calls cudaMalloc, cudaFree or an allocating library routine. */
#define GK_NOALLOC_SCRATCH_BYTES (16u << 20)
int gk_gemm_i8_noalloc_unchecked(size_t m, size_t k, size_t n, int32_t alpha, const int8_t *a,
                                 ptrdiff_t rsa, ptrdiff_t csa, const int8_t *b, ptrdiff_t rsb,
                                 ptrdiff_t csb, int32_t beta, int32_t *c, ptrdiff_t rsc,
                                 ptrdiff_t csc, gk_stream_t stream);

/* ---- sharding across the GPUs of one node (no counterpart in gemmkit) ------------------ */

/* gemmkit runs in one process. For the sharded paths each GPU has its own process; a device
 * buffer of one process is exported as a CUDA IPC handle plus the pointer's offset inside its
 * allocation, and the other processes of the node map it (a plain peer mapping over NVLink).
 * gk_ipc_open reference-counts mappings of one allocation; gk_ipc_close releases one. */
typedef struct gk_ipc_handle {
    unsigned char bytes[64];
    uint64_t offset;
} gk_ipc_handle;
int gk_ipc_export(const void *dev_ptr, gk_ipc_handle *out);
int gk_ipc_open(const gk_ipc_handle *h, void **peer_ptr);
int gk_ipc_close(void *peer_ptr);

/* Mirrored outputs: the product of gk_gemm_bf16_f32_unchecked / gk_gemm_f16_f32_unchecked
 * (is_f16 selects), whose epilogue also stores every element of C at the same offset from
 * each of `mirrors[0 .. nmirror)` (nmirror <= 7; usually peer GPUs' copies of C mapped with
 * gk_ipc_open). This is the column-sharded wide GEMM with C replicated: each GPU computes
 * its block of columns and writes it into every GPU's C in the same kernel, tile by tile,
 * instead of a separate all-gather. beta reads only the local C. Needs k > 0 and
 * alpha != 0 (GK_EINVAL otherwise). The mirrors are complete once the kernel has finished
 * and the caller has synchronised with the other GPUs (for example an NCCL barrier on the
 * same stream). */
int gk_gemm_half_f32_mirrored_unchecked(gk_workspace *ws, int is_f16, size_t m, size_t k,
                                        size_t n, float alpha, const uint16_t *a, ptrdiff_t rsa,
                                        ptrdiff_t csa, const uint16_t *b, ptrdiff_t rsb,
                                        ptrdiff_t csb, float beta, float *c, ptrdiff_t rsc,
                                        ptrdiff_t csc, void *const *mirrors, int nmirror,
                                        gk_stream_t stream);
/* The same for the requantizing i8 product: gk_gemm_i8_requant_batched_unchecked's arguments
 * (batch >= 1; bias_bs / scales_bs the per-element strides of bias and scales), optionally
 * with a prepacked B instead of (b, rsb, csb, b_bs) (then batch must be 1), plus mirrors.
 * The batch-sharded path uses it to replicate each GPU's slice of a batch. */
int gk_gemm_i8_requant_mirrored_unchecked(gk_workspace *ws, size_t batch, size_t m, size_t k,
                                          size_t n, const int8_t *a, ptrdiff_t rsa,
                                          ptrdiff_t csa, ptrdiff_t a_bs, const int8_t *b,
                                          ptrdiff_t rsb, ptrdiff_t csb, ptrdiff_t b_bs,
                                          const gk_packed_rhs *packed, const gk_requant *req,
                                          ptrdiff_t bias_bs, ptrdiff_t scales_bs, void *c,
                                          ptrdiff_t rsc, ptrdiff_t csc, ptrdiff_t c_bs,
                                          int out_u8, void *const *mirrors, int nmirror,
                                          gk_stream_t stream);

/* ---- self test of the bounded-wait path ----------------------------------------------- */

/* Launch a kernel that waits on an mbarrier no one arrives on, with a `timeout_ns` bound,
 * and report the outcome: GK_ETIMEOUT (the expected result) once the wait gave up and the
 * kernel returned, leaving the context usable. */
int gk_selftest_wait_timeout(uint64_t timeout_ns, gk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
