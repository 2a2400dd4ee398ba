// gk_engine.h -- internal interface between the C ABI (gk_api.cu) and the kernels.
//
// Every product is lowered to one canonical device problem: D[Mk x Nk] = A_k[Mk x K] *
// B_k[Nk x K]^T, with both operands K-contiguous in device memory (the layout the TMA
// loads and the tcgen05 K-major shared-memory descriptors expect), and an epilogue that
// writes D(i, j) to out + e*obs + i*ldo + j*cso. The host picks the orientation (which of
// the user's m / n becomes Mk) exactly as gemmkit's orient_swap does
// (gemmkit/src/dispatch.rs:395), so that the output's contiguous axis is j.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gk {

enum class Kind : int { I8 = 0, F16 = 1, BF16 = 2 };
enum class Out : int { I32 = 0, Q8 = 1, F32 = 2, U8 = 3 };  // Q8: i8 requant, U8: u8 requant
enum Axis : int { AX_NONE = 0, AX_M = 1, AX_N = 2 };

struct EpiParams {
    void* out;
    int64_t ldo, cso, obs;  // output strides in elements (row, col, batch)
    int32_t alpha_i, beta_i;
    float alpha_f, beta_f;
    const int32_t* bias;
    int64_t bias_bs;
    int32_t bias_axis;  // Axis
    int32_t scale_axis; // Axis (AX_NONE: per-tensor `scale`)
    const float* scales;
    int64_t scale_bs;
    float scale;
    int32_t zp, lo, hi;  // lo already raised to clamp(zp) under ReLU
    int32_t relu;        // apply the raised lower clamp (the band's own clamp is a saturation)
    int32_t vec;         // cso == 1 and every row start 16-byte aligned
    // Mirrors: every output element is also stored at the same byte offset from each of
    // mirror[0 .. nmirror) (peer GPUs' copies of C, mapped into this process), so one GEMM
    // both computes its block and replicates it over NVLink.
    int32_t nmirror;
    void* mirror[7];
    // Fused float epilogue (f32 outputs; gemmkit's FusedEpi, gemmkit/src/kernel/epilogue.rs:
    // 258-330): after alpha*acc + beta*C, add fbias[row or column] then apply the activation.
    const float* fbias;
    int32_t fbias_axis;  // Axis
    int32_t act;         // FACT_*
    float leak;          // LeakyReLU slope
};

enum FusedAct : int32_t { FACT_NONE = 0, FACT_RELU = 1, FACT_LEAKY = 2 };

// Division of an unsigned n < 2^31 by a fixed d as a multiply and a shift (Granlund and
// Montgomery's round-up method): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> l. set_fast_div() computes m and l on the host.
struct FastDiv {
    uint32_t d, m, s, pad;
};
void set_fast_div(FastDiv* f, uint32_t d);

struct GemmParams {
    int64_t Mk, Nk;
    int32_t K, batch;
    int32_t tiles_m, tiles_n, tiles_per_batch, num_tiles, num_kb, group_m;
    // tile decode divisors: tiles per batch element, tiles per rasterisation band, band height
    // (group_m) and the height of the last band (tiles_m % group_m, or group_m)
    FastDiv div_tpb, div_band, div_gm, div_glast;
    int32_t a_batched, b_batched;
    // Operands held in the tiled prepacked layout (see Operand::slab) are fetched with 1-D
    // bulk copies from these bases instead of through their tensor maps (nullptr = TMA).
    const uint8_t* a_tiled;
    const uint8_t* b_tiled;
    int64_t a_slab, b_slab;  // bytes between consecutive 128-byte K blocks
    // 1: B is read MN-major (its Nk rows contiguous, K at a pitch): tile kernel, i8, BN <= 128
    int32_t b_mn;
    // Stream-K tail: tiles [0, dp_tiles) run whole, round-robin over the CTAs; the K blocks
    // of the remaining tiles are spread evenly over all CTAs. A tile cut between CTAs leaves
    // 32-bit partial accumulators in sk_part; the last CTA to finish a 32-row x WCOLS region
    // (counted in sk_ctr, tagged with sk_epoch so stale counts are ignored) sums them in slot
    // order and runs the epilogue.
    int32_t dp_tiles;
    int32_t sk_maxc;   // partial slots per stream-K tile
    int64_t sk_iters;  // (num_tiles - dp_tiles) * num_kb, 0 = no stream-K
    uint32_t* sk_part;
    uint32_t* sk_ctr;
    uint32_t sk_epoch;
    uint64_t timeout_ns;
    unsigned int* status;
    int32_t stages;
    int32_t f32q;  // 1: the pair kernel's 16-warp form may requantize items in packed f32  // ring depth cap (0: the kernel's whole ring)
    EpiParams e;
};

// One operand in the canonical frame: `rows` rows of K contiguous elements at stride `ld`
// (elements); batch element e at + e*bs (bs == 0: shared).
struct Operand {
    const void* ptr;
    int64_t rows, ld, bs;
    // slab > 0: the tiled prepacked layout. K is cut into 128-byte blocks; block kb is one
    // contiguous slab of `slab` bytes holding every (padded) row's 128 bytes at a 128-byte
    // stride, each row's 16-byte chunks already in the 128-byte-swizzle order
    // (chunk j of row r stored at j ^ (r % 8)). Any 8-row-aligned run of rows of one block is
    // then a contiguous copy that lands in shared memory exactly as the MMA reads it.
    int64_t slab;
    // mn_ld > 0: the operand is MN-major instead: element (r, p) at ptr + r + p*mn_ld (the
    // rows contiguous, K at pitch mn_ld elements; an N-contiguous right-hand side, i8 only)
    int64_t mn_ld;
};

struct TcProblem {
    Kind kind;
    Out out;
    int64_t Mk, Nk, K, batch;
    Operand a, b;
    EpiParams e;
    int bn;  // 0 = heuristic
    cudaStream_t stream;
    int pdl;  // 1: kernels that support it may overlap the previous kernel of the stream
    int stages;  // ring depth cap of the kernels (0: their whole ring)
    int epi16;   // 1: the CTA-pair kernel may take its 16-warp epilogue form (short K)
    int gemv_split;  // small-M kernel: largest cluster K split (0: up to 8)
    int f32q;        // 1: short-K requantized items may take the packed f32 path
    // Scratch for a stream-K tail (see GemmParams); nullptr = no stream-K.
    uint32_t* sk_part;
    uint32_t* sk_ctr;
    uint32_t sk_epoch;
};

// Launch geometry chosen for a problem (tile width, grid, stream-K split and the scratch it
// needs). plan_tc_gemm fills it; allow_sk = false plans without a stream-K tail.
struct TcPlan {
    int pair;  // 1: CTA-pair kernel (256-row tiles over two SMs, cluster of 2)
    int gemv;  // 1: small-M streaming kernel (Nk <= 64; bn = its MMA N)
    int split; // small-M kernel: CTAs (one cluster) sharing each tile's K blocks, 1 = none
    int gemv_sk;  // small-M kernel: stream-K over the (tile, K block) units of all CTAs
    int pdl;   // launch with programmatic stream serialization
    int bn, nepi, tiles_m, tiles_n, num_tiles, num_kb, grid;
    int dp_tiles, sk_maxc;
    int64_t sk_iters;
    int64_t part_words;  // 32-bit words of sk_part
    int64_t ctr_words;   // 32-bit words of sk_ctr
};
void plan_tc_gemm(const TcProblem& p, bool allow_sk, TcPlan* plan);
// Fills the tile decode divisors of gp from its tiles_m / tiles_n / tiles_per_batch / group_m.
void set_tile_divs(GemmParams* gp);
// allow_pair enables the CTA-pair kernel where it applies (GEMMKIT_CUDA_PAIR knob);
// allow_gemv the small-M streaming kernel (GEMMKIT_CUDA_GEMV knob).
// allow_gemv_sk lets the small-M kernel split its weight stream evenly over every SM with
// stream-K partials (the caller then provides sk_part / sk_ctr scratch, plan.sk_iters > 0).
void plan_tc_gemm2(const TcProblem& p, bool allow_sk, bool allow_pair, bool allow_gemv,
                   TcPlan* plan, bool allow_gemv_sk = false);
// The small-M streaming kernel (gk_gemv.cu): plan_gemv fills `plan` and returns true when the
// problem qualifies (batch 1, 1 <= Nk <= 64, no tile-width override, activations not tiled).
bool plan_gemv(const TcProblem& p, TcPlan* plan, bool allow_sk = false);
int launch_gemv(const TcProblem& pr, const TcPlan& plan, char* err, size_t errlen);
struct GemmParams;
int launch_pair(const TcProblem& pr, const TcPlan& plan, const GemmParams& gp, char* err,
                size_t errlen);
int launch_tc_gemm_planned(const TcProblem& p, const TcPlan& plan, char* err, size_t errlen);

// Launch the tcgen05 GEMM for `p` (all operands already TMA-compatible). Returns a GK_*
// status and fills `err` on failure.
int launch_tc_gemm(const TcProblem& p, char* err, size_t errlen);

// Device status word for the current device (bounded-wait give-ups are or-ed into it).
unsigned int* device_status_ptr();

int sm_count();

// Auxiliary kernels (gk_aux.cu).
// The tiled prepacked layout (Operand::slab) of a rows x K operand whose element (r, p) is at
// src[r*srs + p*scs]; rows_pad / k_pad are multiples of 256 / 128 and the padding is zero.
int launch_pack_tiled(uint8_t* dst, int64_t rows_pad, int64_t k_pad, const int8_t* src,
                      int64_t srs, int64_t scs, int64_t rows, int64_t K, cudaStream_t s);
// dst[e][r][k] = src[e*sbs + r*srs + k*scs] for k < K, 0 for K <= k < ld (element size es).
int launch_pack_kmajor(void* dst, int64_t dld, int64_t dbs, const void* src, int64_t srs,
                       int64_t scs, int64_t sbs, int64_t rows, int64_t K, int64_t batch, int es,
                       cudaStream_t s);
// k == 0 / alpha == 0: C <- beta*C (wrapping); beta == 0 writes zeros.
int launch_scale_c_i32(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int32_t beta,
                       cudaStream_t s);
int launch_scale_c_f32(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int64_t cbs,
                       int64_t batch, float beta, cudaStream_t s);
// Fused float epilogue with a vanishing product: C <- act(beta*C + bias) (user frame; the
// bias axis of `e` is in the user frame too).
int launch_fused_fill_f32(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, float beta,
                          const EpiParams& e, cudaStream_t s);
// The i32 counterpart (fused i32 epilogue): C <- act(beta*C + bias), wrapping, user frame.
int launch_fused_fill_i32(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                          int32_t beta, const EpiParams& e, cudaStream_t s);
// k == 0 requant fill: the map of a zero accumulator (user frame: i = row, j = col).
int launch_requant_fill(void* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int64_t cbs,
                        int64_t batch, const EpiParams& e, cudaStream_t s);
int launch_selftest_timeout(uint64_t timeout_ns, cudaStream_t s);
// f32 -> i8 quantize of a rows x cols view (per-tensor `scale`/`zp`, or per-row scales written
// to `scales` when it is not null).
int launch_quantize_rows(const float* x, int64_t rsx, int64_t csx, int64_t rows, int64_t cols,
                         int8_t* q, int64_t rsq, int64_t csq, float scale, int32_t zp,
                         float* scales, cudaStream_t s);

// Sets this thread's gk_last_error() text (gk_api.cu); returns `code`.
int set_last_error(int code, const char* text);

}  // namespace gk
