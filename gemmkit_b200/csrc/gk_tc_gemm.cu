// gk_tc_gemm.cu -- the engine's tensor-core GEMM for sm_100a.
//
// One persistent, warp-specialised kernel template serves every product of the path:
//   kind::i8 (s8 x s8 -> s32) with an i32 (alpha/beta) or a requantizing i8/u8 epilogue,
//   kind::f16 (bf16 or f16 -> f32) with an f32 (alpha/beta) epilogue.
//
// Per CTA (one per SM, 192 threads):
//   warp 0  TMA producer: 128-byte-swizzled K-major boxes of A (128 rows) and B (BN rows),
//           128 bytes of K per stage, into a STAGES-deep shared-memory ring;
//   warp 1  owns the TMEM allocation and issues tcgen05.mma (M = 128, N = BN, 32 bytes of K
//           per instruction) into one of two TMEM accumulators, committing each stage back
//           to the producer and each finished tile to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32 TMEM lanes, the fused epilogue in
//           registers, and direct vector stores -- while the MMA warp already accumulates the
//           next tile into the other TMEM buffer.
// Every wait is bounded (globaltimer); a give-up raises a CTA abort flag, records the role in
// the device status word, drains in-flight copies and MMAs, frees TMEM and returns.
//
// The requant arithmetic reproduces gemmkit's KRequantize::apply bit for bit
// (gemmkit/src/kernel/epilogue.rs:810-830): q = clamp(zp + rne(fl64(f64(acc + bias) *
// f64(scale))), LO, HI). See requant_one() for the exact-arithmetic argument.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "gk_engine.h"
#include "gk_sm100.cuh"

namespace gk {

constexpr int BM = 128;        // MMA M (TMEM lanes)
constexpr int BKB = 128;       // bytes of K per stage and row (one 128-byte swizzle atom)
constexpr int MMA_KB = 32;     // bytes of K per tcgen05.mma (kind::i8 K=32, kind::f16 K=16)
constexpr int NTHREADS = 192;  // 6 warps
constexpr int SMEM_LIMIT = 232448;

template <Out OUT, int BN>
struct TileCfg {
    static constexpr int A_BYTES = BM * BKB;
    static constexpr int B_BYTES = BN * BKB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int CP_BYTES = (OUT == Out::Q8) ? 2 * BN * 32 : 0;  // column params x2
    static constexpr int BAR_BYTES = 256;
    static constexpr int RAW_STAGES = (SMEM_LIMIT - 1024 - BAR_BYTES - CP_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = RAW_STAGES > 10 ? 10 : RAW_STAGES;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + CP_BYTES;
    static constexpr int TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
    static constexpr int CH = BN < 32 ? BN : 32;  // TMEM columns per tcgen05.ld
    static_assert(STAGES >= 2, "shared memory too small");
    static_assert(SMEM <= SMEM_LIMIT, "shared memory budget");
};

// Per-scale constants of the exact requant (see requant_one).
struct alignas(16) ColParam {
    double se;    // min(scale, 2048), exact
    double nms;   // -(2^52 + 2^31) * se, exact (22-bit x 24-bit significands)
    int32_t vlo;  // accumulator clamp [vlo, vhi] that keeps every result while bounding |p|
    int32_t vhi;
    int32_t bias;
    int32_t pad;
};

__device__ __forceinline__ void make_scale_param(float s, double& se, double& nms, int& vlo,
                                                 int& vhi) {
    const double s64 = static_cast<double>(s);
    se = s64 < 2048.0 ? s64 : 2048.0;
    nms = -(4503601774854144.0 * se);
    const double vs = ceil(2048.0 / se) + 1.0;
    vhi = vs >= 2147483647.0 ? 2147483647 : static_cast<int>(vs);
    vlo = vhi == 2147483647 ? (-2147483647 - 1) : -vhi - 1;
}

// clamp(zp + rne(fl64(f64(v) * f64(scale))), lo, hi) for v = acc +wrap bias, exactly:
//  1. v is clamped to [vlo, vhi]. The map is monotone in v (scale > 0), and |v| beyond
//     vhi ~ 2048/scale already drives |v*scale| >= 2048, past any clamp band, so the clamp
//     changes no result; it bounds |v*se| <= 2048 + 3*se <= 8192. For scale > 2048 the
//     band is v in [-3, 2] with se = 2048 and every v != 0 still saturates, as with scale.
//  2. d = 2^52 + 2^31 + v is exact (built from bits); fma(d, se, -(2^52 + 2^31)*se) has the
//     exact value v*se and rounds once: it is the reference's f64 product fl64(v*scale).
//  3. p + 1.5*2^52 rounds p to the nearest integer, ties to even (the reference's 2^52
//     trick, gemmkit/src/kernel/epilogue.rs:886-897); |p| <= 8192 leaves the integer in the
//     low word. zp joins after rounding, in integer, then the clamp.
__device__ __forceinline__ int requant_one(int32_t acc, int32_t bias, double se, double nms,
                                           int vlo, int vhi, int zp, int lo, int hi) {
    int v = static_cast<int>(static_cast<uint32_t>(acc) + static_cast<uint32_t>(bias));
    v = min(max(v, vlo), vhi);
    const double d = __hiloint2double(0x43300000, v ^ static_cast<int>(0x80000000u));
    const double p = __fma_rn(d, se, nms);
    const double y = __dadd_rn(p, 6755399441055744.0);
    const int q = __double2loint(y) + zp;
    return min(max(q, lo), hi);
}

__device__ __forceinline__ void decode_tile(int t, const GemmParams& p, int& b, int& tm,
                                            int& tn) {
    b = t / p.tiles_per_batch;
    const int r = t - b * p.tiles_per_batch;
    const int band_tiles = p.group_m * p.tiles_n;
    const int band = r / band_tiles;
    const int first_m = band * p.group_m;
    const int gsize = min(p.tiles_m - first_m, p.group_m);
    const int rr = r - band * band_tiles;
    tm = first_m + rr % gsize;
    tn = rr / gsize;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int* status, unsigned int where,
                                          uint64_t timeout) {
    const bool ok = mbar_wait(bar, parity, abort_flag, status, where, timeout);
    return !__any_sync(0xffffffffu, !ok);
}

template <Kind KIND, Out OUT, int BN>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using C = TileCfg<OUT, BN>;
    constexpr int STAGES = C::STAGES;
    constexpr int CH = C::CH;
    constexpr int NCHUNK = BN / CH;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    constexpr int BKE = BKB / ES;  // K elements per stage

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* pready = tfull + 4;
    uint64_t* drain = tfull + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 7);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    ColParam* cparams = reinterpret_cast<ColParam*>(smem + STAGES * C::STAGE_BYTES + C::BAR_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint64_t tmo = p.timeout_ns;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
            mbar_init(&pready[a], 128);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        if (!p.a_tiled) prefetch_tmap(&tmA);
        if (!p.b_tiled) prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                int b, tm, tn;
                decode_tile(t, p, b, tm, tn);
                const int za = p.a_batched ? b : 0, zb = p.b_batched ? b : 0;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                                   GK_DEV_TIMEOUT_PRODUCER, tmo)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    if (p.a_tiled)
                        bulk_load(sA + stage * C::A_BYTES,
                                  p.a_tiled + kb * p.a_slab + static_cast<int64_t>(tm) * BM * BKB,
                                  C::A_BYTES, &full[stage]);
                    else
                        tma_load_3d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BKE,
                                    tm * BM, za);
                    if (p.b_tiled)
                        bulk_load(sB + stage * C::B_BYTES,
                                  p.b_tiled + kb * p.b_slab + static_cast<int64_t>(tn) * BN * BKB,
                                  C::B_BYTES, &full[stage]);
                    else
                        tma_load_3d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BKE,
                                    tn * BN, zb);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: every issued copy has landed before the CTA may exit.
            int dummy = 0;
            for (int s = 0; s < STAGES; ++s)
                if (issued & (1u << s))
                    mbar_wait(&full[s], (last_par >> s) & 1u, &dummy, p.status,
                              GK_DEV_TIMEOUT_DRAIN, tmo);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t idesc;
            if constexpr (KIND == Kind::I8)
                idesc = idesc_i8(BM, BN);
            else
                idesc = idesc_f16(BM, BN, KIND == Kind::BF16);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int local = 0;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, p.status, GK_DEV_TIMEOUT_MMA,
                               tmo)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.status, GK_DEV_TIMEOUT_MMA,
                                   tmo)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
                    for (int ks = 0; ks < BKB / MMA_KB; ++ks) {
                        const uint64_t ad = sdesc_kmajor_sw128(a0 + ks * MMA_KB);
                        const uint64_t bd = sdesc_kmajor_sw128(b0 + ks * MMA_KB);
                        const uint32_t accum = (kb | ks) != 0 ? 1u : 0u;
                        if constexpr (KIND == Kind::I8)
                            mma_i8(d, ad, bd, idesc, accum);
                        else
                            mma_f16(d, ad, bd, idesc, accum);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);
            }
            // Drain: every issued MMA has finished before TMEM is freed.
            mma_commit(drain);
            int dummy = 0;
            mbar_wait(drain, 0, &dummy, p.status, GK_DEV_TIMEOUT_DRAIN, tmo);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;           // TMEM lane quarter this warp may access
        const int et = threadIdx.x - 64;  // 0..127
        const EpiParams& e = p.e;
        int local = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
            int b, tm, tn;
            decode_tile(t, p, b, tm, tn);
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int row = q * 32 + lane;
            const int64_t grow = static_cast<int64_t>(tm) * BM + row;
            const int64_t gcol0 = static_cast<int64_t>(tn) * BN;
            const bool row_ok = grow < p.Mk;

            // Requant parameters: per-row values in registers, per-column values shared
            // through shared memory (double-buffered by accumulator, published by pready).
            double r_se = 0.0, r_nms = 0.0;
            int r_vlo = 0, r_vhi = 0, r_bias = 0;
            ColParam* cp = cparams + acc * BN;
            if constexpr (OUT == Out::Q8) {
                if (e.scale_axis != AX_N) {
                    float s = e.scale;
                    if (e.scale_axis == AX_M)
                        s = row_ok ? e.scales[b * e.scale_bs + grow] : 1.0f;
                    make_scale_param(s, r_se, r_nms, r_vlo, r_vhi);
                }
                if (e.bias_axis == AX_M && row_ok) r_bias = e.bias[b * e.bias_bs + grow];
                if (e.scale_axis == AX_N || e.bias_axis == AX_N) {
                    for (int j = et; j < BN; j += 128) {
                        const int64_t gc = gcol0 + j;
                        const bool cok = gc < p.Nk;
                        ColParam c;
                        if (e.scale_axis == AX_N) {
                            make_scale_param(cok ? e.scales[b * e.scale_bs + gc] : 1.0f, c.se,
                                             c.nms, c.vlo, c.vhi);
                        } else {  // the scale lives in each thread's registers
                            c.se = 0.0;
                            c.nms = 0.0;
                            c.vlo = 0;
                            c.vhi = 0;
                        }
                        c.bias = (e.bias_axis == AX_N && cok) ? e.bias[b * e.bias_bs + gc] : 0;
                        c.pad = 0;
                        cp[j] = c;
                    }
                    mbar_arrive(&pready[acc]);
                    if (!warp_wait(&pready[acc], aph, abort_flag, p.status,
                                   GK_DEV_TIMEOUT_EPILOGUE, tmo))
                        break;
                }
            }

            if (!warp_wait(&tfull[acc], aph, abort_flag, p.status, GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            tc_fence_after();

            const int64_t obase = static_cast<int64_t>(b) * e.obs + grow * e.ldo;
#pragma unroll 1
            for (int c = 0; c < NCHUNK; ++c) {
                uint32_t v[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                       static_cast<uint32_t>(acc * BN + c * CH);
                if constexpr (CH == 32)
                    tmem_ld_x32(taddr, v);
                else
                    tmem_ld_x16(taddr, v);
                tmem_wait_ld();
                if (c == NCHUNK - 1) {
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                if (!row_ok) continue;
                const int64_t gc = gcol0 + c * CH;
                const bool full_chunk = gc + CH <= p.Nk;

                if constexpr (OUT == Out::Q8) {
                    int r[CH];
                    if (e.scale_axis == AX_N) {
                        // per-column scale (and a per-column or per-row bias)
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            const ColParam& pc = cp[c * CH + i];
                            const int bias = e.bias_axis == AX_N ? pc.bias : r_bias;
                            r[i] = requant_one(static_cast<int32_t>(v[i]), bias, pc.se, pc.nms,
                                               pc.vlo, pc.vhi, e.zp, e.lo, e.hi);
                        }
                    } else if (e.bias_axis == AX_N) {
                        // per-row (or per-tensor) scale in registers, per-column bias
#pragma unroll
                        for (int i = 0; i < CH; ++i)
                            r[i] = requant_one(static_cast<int32_t>(v[i]), cp[c * CH + i].bias,
                                               r_se, r_nms, r_vlo, r_vhi, e.zp, e.lo, e.hi);
                    } else {
#pragma unroll
                        for (int i = 0; i < CH; ++i)
                            r[i] = requant_one(static_cast<int32_t>(v[i]), r_bias, r_se, r_nms,
                                               r_vlo, r_vhi, e.zp, e.lo, e.hi);
                    }
                    uint8_t* out = static_cast<uint8_t*>(e.out);
                    if (e.vec && full_chunk) {
                        uint8_t* dst = out + obase + gc;
#pragma unroll
                        for (int g = 0; g < CH / 16; ++g) {
                            uint32_t w[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int* x = r + g * 16 + u * 4;
                                w[u] = (static_cast<uint32_t>(x[0]) & 0xFFu) |
                                       ((static_cast<uint32_t>(x[1]) & 0xFFu) << 8) |
                                       ((static_cast<uint32_t>(x[2]) & 0xFFu) << 16) |
                                       ((static_cast<uint32_t>(x[3]) & 0xFFu) << 24);
                            }
                            st_global_v4(dst + g * 16, w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < CH; ++i)
                            if (gc + i < p.Nk)
                                out[obase + (gc + i) * e.cso] = static_cast<uint8_t>(r[i]);
                    }
                } else if constexpr (OUT == Out::I32) {
                    int32_t* out = static_cast<int32_t*>(e.out);
                    uint32_t r[CH];
                    const uint32_t al = static_cast<uint32_t>(e.alpha_i);
                    const uint32_t be = static_cast<uint32_t>(e.beta_i);
                    if (e.vec && full_chunk) {
                        int32_t* dst = out + obase + gc;
                        if (be != 0u) {
#pragma unroll
                            for (int g = 0; g < CH / 4; ++g) {
                                const uint4 cv = ld_global_v4(dst + g * 4);
                                r[g * 4 + 0] = be * cv.x + al * v[g * 4 + 0];
                                r[g * 4 + 1] = be * cv.y + al * v[g * 4 + 1];
                                r[g * 4 + 2] = be * cv.z + al * v[g * 4 + 2];
                                r[g * 4 + 3] = be * cv.w + al * v[g * 4 + 3];
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < CH; ++i) r[i] = al * v[i];
                        }
#pragma unroll
                        for (int g = 0; g < CH / 4; ++g)
                            st_global_v4(dst + g * 4, r[g * 4], r[g * 4 + 1], r[g * 4 + 2],
                                         r[g * 4 + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            if (gc + i >= p.Nk) continue;
                            int32_t* cptr = out + obase + (gc + i) * e.cso;
                            uint32_t o = al * v[i];
                            if (be != 0u) o += be * static_cast<uint32_t>(*cptr);
                            *cptr = static_cast<int32_t>(o);
                        }
                    }
                } else {  // F32
                    float* out = static_cast<float*>(e.out);
                    const float al = e.alpha_f, be = e.beta_f;
                    if (e.vec && full_chunk) {
                        float* dst = out + obase + gc;
#pragma unroll
                        for (int g = 0; g < CH / 4; ++g) {
                            float x0 = al * __uint_as_float(v[g * 4 + 0]);
                            float x1 = al * __uint_as_float(v[g * 4 + 1]);
                            float x2 = al * __uint_as_float(v[g * 4 + 2]);
                            float x3 = al * __uint_as_float(v[g * 4 + 3]);
                            if (be != 0.0f) {
                                const uint4 cv = ld_global_v4(dst + g * 4);
                                x0 = __fmaf_rn(be, __uint_as_float(cv.x), x0);
                                x1 = __fmaf_rn(be, __uint_as_float(cv.y), x1);
                                x2 = __fmaf_rn(be, __uint_as_float(cv.z), x2);
                                x3 = __fmaf_rn(be, __uint_as_float(cv.w), x3);
                            }
                            st_global_v4(dst + g * 4, __float_as_uint(x0), __float_as_uint(x1),
                                         __float_as_uint(x2), __float_as_uint(x3));
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            if (gc + i >= p.Nk) continue;
                            float* cptr = out + obase + (gc + i) * e.cso;
                            float x = al * __uint_as_float(v[i]);
                            if (be != 0.0f) x = __fmaf_rn(be, *cptr, x);
                            *cptr = x;
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------

typedef CUresult (*PFN_tmapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                         const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                         const cuuint32_t*, CUtensorMapInterleave,
                                         CUtensorMapSwizzle, CUtensorMapL2promotion,
                                         CUtensorMapFloatOOBfill);

static PFN_tmapEncodeTiled get_encode() {
    static PFN_tmapEncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_tmapEncodeTiled>(f);
    });
    return fn;
}

static __device__ unsigned int g_status[64];

unsigned int* device_status_ptr() {
    int dev = 0;
    cudaGetDevice(&dev);
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
    return static_cast<unsigned int*>(p) + (dev & 63);
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

static int encode_operand(CUtensorMap* map, const Operand& op, int64_t K, int64_t batch, int es,
                          int box_rows, char* err, size_t errlen) {
    PFN_tmapEncodeTiled enc = get_encode();
    if (!enc) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled is unavailable (driver too old?)");
        return 5;
    }
    const int64_t ldb = op.ld * es;
    if ((reinterpret_cast<uintptr_t>(op.ptr) & 15) || (ldb & 15) || ldb <= 0 ||
        (batch > 1 && op.bs != 0 && ((op.bs * es) & 15))) {
        snprintf(err, errlen, "gemmkit: internal error: operand not TMA-aligned");
        return 1;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(op.rows),
                          static_cast<cuuint64_t>(op.bs != 0 ? batch : 1)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldb),
                             static_cast<cuuint64_t>(op.bs != 0 ? op.bs * es
                                                               : ((ldb * op.rows + 15) & ~15LL))};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(BKB / es), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, es == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                     3, const_cast<void*>(op.ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
        return 3;
    }
    return 0;
}

template <Kind KIND, Out OUT, int BN>
static int launch_one(const TcProblem& pr, GemmParams gp, char* err, size_t errlen) {
    using C = TileCfg<OUT, BN>;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    CUtensorMap ta, tb;
    memset(&ta, 0, sizeof(ta));
    memset(&tb, 0, sizeof(tb));
    int rc = 0;
    if (pr.a.slab == 0 && (rc = encode_operand(&ta, pr.a, pr.K, pr.batch, ES, BM, err, errlen)))
        return rc;
    if (pr.b.slab == 0 && (rc = encode_operand(&tb, pr.b, pr.K, pr.batch, ES, BN, err, errlen)))
        return rc;
    if (pr.b.slab && (pr.b.rows % BN)) {
        snprintf(err, errlen, "gemmkit: internal error: tiled operand rows not padded to %d", BN);
        return 1;
    }
    gp.a_tiled = pr.a.slab ? static_cast<const uint8_t*>(pr.a.ptr) : nullptr;
    gp.b_tiled = pr.b.slab ? static_cast<const uint8_t*>(pr.b.ptr) : nullptr;
    gp.a_slab = pr.a.slab;
    gp.b_slab = pr.b.slab;
    auto kern = tc_gemm_kernel<KIND, OUT, BN>;
    static int attr_done[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) {
            snprintf(err, errlen, "gemmkit: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? 5 : 3;
        }
        attr_done[dev & 63] = 1;
    }
    gp.tiles_n = static_cast<int>((pr.Nk + BN - 1) / BN);
    gp.tiles_per_batch = gp.tiles_m * gp.tiles_n;
    gp.num_tiles = gp.tiles_per_batch * gp.batch;
    const int grid = gp.num_tiles < sm_count() ? gp.num_tiles : sm_count();
    kern<<<grid, NTHREADS, C::SMEM, pr.stream>>>(ta, tb, gp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(err, errlen, "gemmkit: kernel launch failed: %s", cudaGetErrorString(e));
        return e == cudaErrorNoDevice || e == cudaErrorNoKernelImageForDevice ||
                       e == cudaErrorInsufficientDriver
                   ? 5
                   : 3;
    }
    return 0;
}

static int pick_bn(const TcProblem& p) {
    if (p.bn) return p.bn;
    // Small output side: one MMA N that covers it (the small-M / GEMV shape).
    if (p.Nk <= 16) return 16;
    if (p.Nk <= 32) return 32;
    if (p.Nk <= 64) return 64;
    const int64_t tm = (p.Mk + BM - 1) / BM;
    const int sms = sm_count();
    for (int bn : {256, 128}) {
        const int64_t tiles = tm * ((p.Nk + bn - 1) / bn) * p.batch;
        if (tiles >= sms) return bn;
    }
    return 64;
}

template <Kind KIND, Out OUT>
static int dispatch_bn(const TcProblem& pr, const GemmParams& gp, int bn, char* err,
                       size_t errlen) {
    switch (bn) {
        case 16: return launch_one<KIND, OUT, 16>(pr, gp, err, errlen);
        case 32: return launch_one<KIND, OUT, 32>(pr, gp, err, errlen);
        case 64: return launch_one<KIND, OUT, 64>(pr, gp, err, errlen);
        case 128: return launch_one<KIND, OUT, 128>(pr, gp, err, errlen);
        case 256: return launch_one<KIND, OUT, 256>(pr, gp, err, errlen);
        default:
            snprintf(err, errlen, "gemmkit: unsupported tile width %d", bn);
            return 1;
    }
}

int launch_tc_gemm(const TcProblem& pr, char* err, size_t errlen) {
    GemmParams gp;
    memset(&gp, 0, sizeof(gp));
    gp.Mk = pr.Mk;
    gp.Nk = pr.Nk;
    gp.K = static_cast<int32_t>(pr.K);
    gp.batch = static_cast<int32_t>(pr.batch);
    gp.tiles_m = static_cast<int>((pr.Mk + BM - 1) / BM);
    const int es = pr.kind == Kind::I8 ? 1 : 2;
    gp.num_kb = static_cast<int>((pr.K * es + BKB - 1) / BKB);
    gp.group_m = 16;
    gp.a_batched = pr.a.bs != 0 && pr.batch > 1;
    gp.b_batched = pr.b.bs != 0 && pr.batch > 1;
    gp.timeout_ns = 4000000000ull;
    gp.status = device_status_ptr();
    gp.e = pr.e;
    const int bn = pick_bn(pr);
    if (pr.kind == Kind::I8) {
        if (pr.out == Out::I32) return dispatch_bn<Kind::I8, Out::I32>(pr, gp, bn, err, errlen);
        if (pr.out == Out::Q8) return dispatch_bn<Kind::I8, Out::Q8>(pr, gp, bn, err, errlen);
    } else if (pr.out == Out::F32) {
        if (pr.kind == Kind::BF16) return dispatch_bn<Kind::BF16, Out::F32>(pr, gp, bn, err, errlen);
        return dispatch_bn<Kind::F16, Out::F32>(pr, gp, bn, err, errlen);
    }
    snprintf(err, errlen, "gemmkit: internal error: unsupported kernel combination");
    return 1;
}

}  // namespace gk
