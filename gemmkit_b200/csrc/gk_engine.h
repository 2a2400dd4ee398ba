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
enum class Out : int { I32 = 0, Q8 = 1, F32 = 2 };
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
    int32_t vec;         // cso == 1 and every row start 16-byte aligned
};

struct GemmParams {
    int64_t Mk, Nk;
    int32_t K, batch;
    int32_t tiles_m, tiles_n, tiles_per_batch, num_tiles, num_kb, group_m;
    int32_t a_batched, b_batched;
    // Operands held in the tiled prepacked layout (see Operand::slab) are fetched with 1-D
    // bulk copies from these bases instead of through their tensor maps (nullptr = TMA).
    const uint8_t* a_tiled;
    const uint8_t* b_tiled;
    int64_t a_slab, b_slab;  // bytes between consecutive 128-byte K blocks
    uint64_t timeout_ns;
    unsigned int* status;
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
};

struct TcProblem {
    Kind kind;
    Out out;
    int64_t Mk, Nk, K, batch;
    Operand a, b;
    EpiParams e;
    int bn;  // 0 = heuristic
    cudaStream_t stream;
};

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
// k == 0 requant fill: the map of a zero accumulator (user frame: i = row, j = col).
int launch_requant_fill(void* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int64_t cbs,
                        int64_t batch, const EpiParams& e, cudaStream_t s);
int launch_selftest_timeout(uint64_t timeout_ns, cudaStream_t s);

// Sets this thread's gk_last_error() text (gk_api.cu); returns `code`.
int set_last_error(int code, const char* text);

}  // namespace gk
