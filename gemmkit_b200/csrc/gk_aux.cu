// gk_aux.cu -- the engine's memory-bound helper kernels:
//   * pack_kmajor: gather any strided (even negative-stride) operand into the K-contiguous,
//     16-byte-aligned rows the TMA loads need (gemmkit's pack step, gemmkit/src/pack.rs,
//     re-targeted at the tensor-core tile layout); a 32 x 32 shared-memory tile keeps both
//     the read and the write side coalesced whichever of the source strides is 1;
//   * the degenerate fills of gemmkit's k == 0 / alpha == 0 paths
//     (gemmkit/src/dispatch/int.rs:150-163 scale_c_int, :735-752 requant_degenerate);
//   * the bounded-wait self test.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gk_engine.h"
#include "gk_sm100.cuh"
#include "gk_tc_common.cuh"

namespace gk {

template <typename T>
__global__ void pack_kmajor_kernel(T* __restrict__ dst, int64_t dld, int64_t dbs,
                                   const T* __restrict__ src, int64_t srs, int64_t scs,
                                   int64_t sbs, int64_t rows, int64_t K) {
    __shared__ T tile[32][33];
    const int64_t e = blockIdx.z;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    const T* s = src + e * sbs;
    T* d = dst + e * dbs;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const bool k_fast = (scs == 1) || (srs != 1 && scs <= srs);
    // read: consecutive threads walk the source's unit-stride axis
    for (int i = ty; i < 32; i += 8) {
        int64_t r, k;
        if (k_fast) {
            r = r0 + i;
            k = k0 + tx;
        } else {
            r = r0 + tx;
            k = k0 + i;
        }
        T v = T(0);
        if (r < rows && k < K) v = s[r * srs + k * scs];
        if (k_fast)
            tile[i][tx] = v;
        else
            tile[tx][i] = v;
    }
    __syncthreads();
    // write: consecutive threads walk K (row-major destination), zero in the K padding
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, k = k0 + tx;
        if (r < rows && k < dld) d[r * dld + k] = tile[i][tx];
    }
}

int launch_pack_kmajor(void* dst, int64_t dld, int64_t dbs, const void* src, int64_t srs,
                       int64_t scs, int64_t sbs, int64_t rows, int64_t K, int64_t batch, int es,
                       cudaStream_t st) {
    if (rows == 0 || dld == 0 || batch == 0) return 0;
    dim3 block(32, 8);
    dim3 grid(static_cast<unsigned>((dld + 31) / 32), static_cast<unsigned>((rows + 31) / 32),
              static_cast<unsigned>(batch));
    if (grid.y > 65535u || grid.z > 65535u) return 1;
    if (es == 1)
        pack_kmajor_kernel<int8_t><<<grid, block, 0, st>>>(
            static_cast<int8_t*>(dst), dld, dbs, static_cast<const int8_t*>(src), srs, scs, sbs,
            rows, K);
    else
        pack_kmajor_kernel<uint16_t><<<grid, block, 0, st>>>(
            static_cast<uint16_t*>(dst), dld, dbs, static_cast<const uint16_t*>(src), srs, scs,
            sbs, rows, K);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// The tiled prepacked layout (gk_engine.h, Operand::slab): byte (r, p) of the rows x K operand
// goes to block p / 128, row r, 16-byte chunk ((p % 128) / 16) ^ (r % 8). One 32-row x 32-byte
// tile per block of 32 x 8 threads, read and written coalesced through shared memory.
__global__ void pack_tiled_kernel(uint8_t* __restrict__ dst, int64_t rows_pad,
                                  const int8_t* __restrict__ src, int64_t srs, int64_t scs,
                                  int64_t rows, int64_t K) {
    __shared__ int8_t tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;
    const bool k_fast = (scs == 1) || (srs != 1 && (scs < 0 ? -scs : scs) <= (srs < 0 ? -srs : srs));
    for (int i = ty; i < 32; i += 8) {
        int64_t r, k;
        if (k_fast) {
            r = r0 + i;
            k = k0 + tx;
        } else {
            r = r0 + tx;
            k = k0 + i;
        }
        int8_t v = 0;
        if (r < rows && k < K) v = src[r * srs + k * scs];
        if (k_fast)
            tile[i][tx] = v;
        else
            tile[tx][i] = v;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, k = k0 + tx;  // always inside [rows_pad, k_pad)
        const int64_t kb = k >> 7, c = k & 127;
        const int64_t off = kb * rows_pad * 128 + r * 128 + ((((c >> 4) ^ (r & 7)) << 4) | (c & 15));
        dst[off] = static_cast<uint8_t>(tile[i][tx]);
    }
}

int launch_pack_tiled(uint8_t* dst, int64_t rows_pad, int64_t k_pad, const int8_t* src,
                      int64_t srs, int64_t scs, int64_t rows, int64_t K, cudaStream_t st) {
    if (rows_pad == 0 || k_pad == 0) return 0;
    if ((rows_pad % 32) || (k_pad % 128)) return 1;
    dim3 block(32, 8);
    dim3 grid(static_cast<unsigned>(k_pad / 32), static_cast<unsigned>(rows_pad / 32));
    if (grid.y > 65535u) return 1;
    pack_tiled_kernel<<<grid, block, 0, st>>>(dst, rows_pad, src, srs, scs, rows, K);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

__global__ void scale_c_i32_kernel(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                                   int32_t beta) {
    const int64_t total = m * n;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = idx / m, i = idx - j * m;
        int32_t* p = c + i * rsc + j * csc;
        if (beta == 0)
            *p = 0;
        else
            *p = static_cast<int32_t>(static_cast<uint32_t>(beta) * static_cast<uint32_t>(*p));
    }
}

int launch_scale_c_i32(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int32_t beta,
                       cudaStream_t st) {
    if (m == 0 || n == 0 || beta == 1) return 0;
    int64_t blocks = (m * n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    scale_c_i32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(c, m, n, rsc, csc, beta);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

__global__ void scale_c_f32_kernel(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                                   int64_t cbs, int64_t batch, float beta) {
    const int64_t per = m * n, total = per * batch;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = idx / per, r = idx - e * per;
        const int64_t j = r / m, i = r - j * m;
        float* p = c + e * cbs + i * rsc + j * csc;
        *p = beta == 0.0f ? 0.0f : beta * *p;
    }
}

int launch_scale_c_f32(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int64_t cbs,
                       int64_t batch, float beta, cudaStream_t st) {
    if (m == 0 || n == 0 || batch == 0 || beta == 1.0f) return 0;
    int64_t blocks = (m * n * batch + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    scale_c_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(c, m, n, rsc, csc, cbs,
                                                                      batch, beta);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// The fused float epilogue with a vanishing product (k == 0 or alpha == 0): C <- act(beta*C +
// bias), gemmkit's fused degenerate rule (gemmkit/src/dispatch/float.rs:671-676); beta == 0
// does not read C. User frame: i = row, j = column.
__global__ void fused_fill_f32_kernel(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                                      float beta, EpiParams e) {
    const int64_t total = m * n;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = idx / m, i = idx - j * m;
        float* p = c + i * rsc + j * csc;
        const float x = beta == 0.0f ? 0.0f : __fmul_rn(beta, *p);
        float bias = 0.0f;
        if (e.fbias_axis == AX_M) bias = e.fbias[i];
        if (e.fbias_axis == AX_N) bias = e.fbias[j];
        *p = fused_apply(e, x, bias);
    }
}

int launch_fused_fill_f32(float* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, float beta,
                          const EpiParams& e, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    int64_t blocks = (m * n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    fused_fill_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(c, m, n, rsc, csc, beta,
                                                                         e);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// Fused i32 epilogue with a vanishing product (k == 0 or alpha == 0): C <- act(beta*C + bias),
// wrapping, in the user frame (AX_M = per row i, AX_N = per column j).
__global__ void fused_fill_i32_kernel(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                                      int32_t beta, EpiParams e) {
    const int64_t total = m * n;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = idx / m, i = idx - j * m;
        int32_t* p = c + i * rsc + j * csc;
        const uint32_t x = beta == 0 ? 0u : static_cast<uint32_t>(beta) * static_cast<uint32_t>(*p);
        uint32_t bias = 0u;
        if (e.bias_axis == AX_M) bias = static_cast<uint32_t>(e.bias[i]);
        if (e.bias_axis == AX_N) bias = static_cast<uint32_t>(e.bias[j]);
        *p = static_cast<int32_t>(fused_apply_i32(e, x, bias));
    }
}

int launch_fused_fill_i32(int32_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                          int32_t beta, const EpiParams& e, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    int64_t blocks = (m * n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    fused_fill_i32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(c, m, n, rsc, csc, beta,
                                                                         e);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// k == 0: every element is KRequantize::apply(0, i, j), computed with the reference's own
// sequence in f64 (this path is not hot).
__global__ void requant_fill_kernel(uint8_t* c, int64_t m, int64_t n, int64_t rsc, int64_t csc,
                                    int64_t cbs, int64_t batch, EpiParams e) {
    const int64_t per = m * n, total = per * batch;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = idx / per, r = idx - b * per;
        const int64_t j = r / m, i = r - j * m;
        int32_t bias = 0;
        if (e.bias_axis == AX_M) bias = e.bias[b * e.bias_bs + i];
        if (e.bias_axis == AX_N) bias = e.bias[b * e.bias_bs + j];
        float s = e.scale;
        if (e.scale_axis == AX_M) s = e.scales[b * e.scale_bs + i];
        if (e.scale_axis == AX_N) s = e.scales[b * e.scale_bs + j];
        const double x = __dmul_rn(static_cast<double>(bias), static_cast<double>(s));
        // round half to even, saturating like `as i64` (|x| stays below 2^31 * 3.4e38)
        long long qv = __double2ll_rn(x);
        if (qv > (1LL << 40)) qv = 1LL << 40;
        if (qv < -(1LL << 40)) qv = -(1LL << 40);
        long long q = qv + e.zp;
        if (q < e.lo) q = e.lo;
        if (q > e.hi) q = e.hi;
        c[b * cbs + i * rsc + j * csc] = static_cast<uint8_t>(q);
    }
}

int launch_requant_fill(void* c, int64_t m, int64_t n, int64_t rsc, int64_t csc, int64_t cbs,
                        int64_t batch, const EpiParams& e, cudaStream_t st) {
    if (m == 0 || n == 0 || batch == 0) return 0;
    int64_t blocks = (m * n * batch + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    requant_fill_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<uint8_t*>(c), m, n, rsc, csc, cbs, batch, e);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// ---- producer step: f32 activations -> i8 ------------------------------------------------
// q = saturate_i8(zp + rne(f64(x) / f64(scale))) with a correctly rounded f64 division and
// round-half-even to integer, in the f64 arithmetic of gemmkit's requant step (NaN -> zp).
// Per-tensor: one scale; dynamic per-row: scale_r = max_j |x_rj| / 127 (f32 division; 1 for an
// all-zero row), written to `scales`, zp = 0. One CTA of 256 threads per row.
__device__ __forceinline__ int8_t quant_one(float x, float scale, int32_t zp) {
    double q = __ddiv_rn(static_cast<double>(x), static_cast<double>(scale));
    long long r = isnan(q) ? 0 : __double2ll_rn(q);  // saturating for |q| beyond 2^63
    if (r > (1LL << 40)) r = 1LL << 40;
    if (r < -(1LL << 40)) r = -(1LL << 40);
    long long v = r + zp;
    v = v < -128 ? -128 : (v > 127 ? 127 : v);
    return static_cast<int8_t>(v);
}

__global__ void quantize_rows_kernel(const float* __restrict__ x, int64_t rsx, int64_t csx,
                                     int64_t cols, int8_t* __restrict__ q, int64_t rsq,
                                     int64_t csq, float scale, int32_t zp, float* scales) {
    const int64_t r = blockIdx.x;
    const float* xr = x + r * rsx;
    int8_t* qr = q + r * rsq;
    float s = scale;
    if (scales) {  // dynamic: the row's absolute maximum
        __shared__ float red[8];
        float mx = 0.0f;
        for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) mx = fmaxf(mx, fabsf(xr[j * csx]));
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
            for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (threadIdx.x == 0) red[0] = v;
        }
        __syncthreads();
        const float amax = red[0];
        s = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
        if (threadIdx.x == 0) scales[r] = s;
    }
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) qr[j * csq] = quant_one(xr[j * csx], s, zp);
}

int launch_quantize_rows(const float* x, int64_t rsx, int64_t csx, int64_t rows, int64_t cols,
                         int8_t* q, int64_t rsq, int64_t csq, float scale, int32_t zp,
                         float* scales, cudaStream_t st) {
    if (rows == 0 || cols == 0) return 0;
    if (rows > 0x7fffffffLL) return 1;
    quantize_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, st>>>(x, rsx, csx, cols, q, rsq,
                                                                      csq, scale, zp, scales);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// Waits on an mbarrier that nothing arrives on; the bounded wait gives up after timeout_ns,
// records GK_DEV_TIMEOUT_SELFTEST and the kernel returns normally.
__global__ void selftest_timeout_kernel(uint64_t timeout_ns, unsigned int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        mbar_wait(&bar, 0, &abort_flag, status, GK_DEV_TIMEOUT_SELFTEST, timeout_ns);
    __syncthreads();
}

int launch_selftest_timeout(uint64_t timeout_ns, cudaStream_t st) {
    selftest_timeout_kernel<<<1, 32, 0, st>>>(timeout_ns, device_status_ptr());
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace gk
