// gk_tc_gemm.cu -- the engine's tensor-core GEMM for sm_100a.
//
// One persistent, warp-specialised kernel template serves every product of the path:
//   kind::i8 (s8 x s8 -> s32) with an i32 (alpha/beta) or a requantizing i8/u8 epilogue,
//   kind::f16 (bf16 or f16 -> f32) with an f32 (alpha/beta) epilogue.
//
// Per CTA (one per SM; 64 + 32 * NEPI threads):
//   warp 0  TMA producer: 128-byte-swizzled K-major boxes of A (128 rows) and B (BN rows),
//           128 bytes of K per stage, into a STAGES-deep shared-memory ring (1-D bulk copies
//           for operands in the tiled prepacked layout);
//   warp 1  owns the TMEM allocation and issues tcgen05.mma (M = 128, N = BN, 32 bytes of K
//           per instruction) into one of two TMEM accumulators, committing each stage back
//           to the producer and each finished tile to the epilogue;
//   warps 2 .. 1 + NEPI  epilogue (4 warps, or 8 for BN >= 64 with two column halves):
//           tcgen05.ld of their 32 TMEM lanes, the fused epilogue in registers, and direct
//           vector stores -- while the MMA warp already accumulates the next tile into the
//           other TMEM buffer.
// Every wait is bounded (globaltimer); a give-up raises a CTA abort flag, records the role in
// the device status word, drains in-flight copies and MMAs, frees TMEM and returns.
// Launched with programmatic stream serialization: operands, parameters, outputs and scratch
// are touched only after griddep_wait(), and each CTA releases the next kernel of the stream
// once its producer has issued its last copy.
//
// The requant arithmetic reproduces gemmkit's KRequantize::apply bit for bit
// (gemmkit/src/kernel/epilogue.rs:810-830): q = clamp(zp + rne(fl64(f64(acc + bias) *
// f64(scale))), LO, HI). See requant_q() (gk_tc_common.cuh) for the exact-arithmetic argument.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "gk_engine.h"
#include "gk_sm100.cuh"
#include "gk_tc_common.cuh"

namespace gk {

template <Out OUT, int BN>
struct TileCfg {
    static constexpr int NEPI = BN >= 64 ? 8 : 4;      // epilogue warps
    static constexpr int THREADS = 64 + 32 * NEPI;     // + producer warp + MMA warp
    static constexpr int WCOLS = BN / (NEPI / 4);      // accumulator columns per epilogue warp
    static constexpr int CH = WCOLS < 32 ? WCOLS : 32;  // TMEM columns per tcgen05.ld
    static constexpr int NCH = WCOLS / CH;
    static constexpr int A_BYTES = BM * BKB;
    static constexpr int B_BYTES = BN * BKB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr bool QUANT = (OUT == Out::Q8 || OUT == Out::U8);
    static constexpr int CP_BYTES = QUANT ? 2 * BN * (32 + 4) : 0;  // column params, x2 buffers
    static constexpr int BAR_BYTES = 256;
    static constexpr int RAW_STAGES = (SMEM_LIMIT - 1024 - BAR_BYTES - CP_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = RAW_STAGES > 12 ? 12 : RAW_STAGES;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES + CP_BYTES;
    static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                     : (2 * BN <= 256) ? 256 : 512;  // a power of two
    static_assert(STAGES >= 2, "shared memory too small");
    static_assert(SMEM + static_cast<int>(sizeof(EpiParams)) <= SMEM_LIMIT, "shared memory budget");
    static_assert(2 * STAGES + 7 <= BAR_BYTES / 8 - 1, "barrier area");
};

template <Kind KIND, Out OUT, int BN>
__global__ void __launch_bounds__(TileCfg<OUT, BN>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using C = TileCfg<OUT, BN>;
    constexpr int STAGES = C::STAGES;
    // ring depth in use: the run-time cap (GEMMKIT_CUDA_STAGES) or the whole ring
    const int nst = (p.stages > 0 && p.stages < STAGES) ? p.stages : STAGES;
    constexpr int CH = C::CH;
    constexpr int NCH = C::NCH;
    constexpr int NEPI_T = 32 * C::NEPI;  // epilogue threads
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    constexpr int BKE = BKB / ES;  // K elements per stage

    extern __shared__ uint8_t smem_raw[];
    // aligned by offsetting the shared array itself (not through an integer cast), so that
    // every access through smem stays a shared-memory access for the compiler
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
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
    uint32_t* cbias = reinterpret_cast<uint32_t*>(cparams + 2 * BN);

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
            mbar_init(&tempty[a], NEPI_T);
            mbar_init(&pready[a], NEPI_T);
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
    // The epilogue's parameters in shared memory, copied while the CTA starts (first reads
    // of the parameter space after the accumulator wait put constant-cache misses on the
    // critical path of a CTA's only tile).
    __shared__ EpiParams s_epi;
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(EpiParams) / 4); i += blockDim.x)
        reinterpret_cast<uint32_t*>(&s_epi)[i] = reinterpret_cast<const uint32_t*>(&p.e)[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            griddep_wait();  // operands may be written by the previous kernel of the stream
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            Sched sch(p);
            Work w;
            while (ok && sch.next(p, w)) {
                int b, tm, tn;
                decode_tile(w.tile, p, b, tm, tn);
                const int za = p.a_batched ? b : 0, zb = p.b_batched ? b : 0;
                for (int kb = w.k0; kb < w.k1; ++kb) {
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
                    else if (p.b_mn)  // 128 K-rows x BN bytes of the N-contiguous B
                        tma_load_3d(sB + stage * C::B_BYTES, &tmB, &full[stage], tn * BN,
                                    kb * BKE, 0);
                    else
                        tma_load_3d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BKE,
                                    tn * BN, zb);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == nst) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // all copies issued: the next kernel of the stream may start placing its CTAs
            griddep_launch_dependents();
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
            if (p.b_mn) idesc |= 1u << 16;  // B is MN-major
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int local = 0;
            Sched sch(p);
            Work w;
            for (; ok && sch.next(p, w); ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, p.status, GK_DEV_TIMEOUT_MMA,
                               tmo)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = w.k0; kb < w.k1; ++kb) {
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
                        // MN-major B: each MMA reads the next 32 K-rows of BN bytes
                        const uint64_t bd = p.b_mn ? sdesc_mnmajor(b0 + ks * MMA_KB * BN, BN)
                                                   : sdesc_kmajor_sw128(b0 + ks * MMA_KB);
                        const uint32_t accum = (kb != w.k0 || ks != 0) ? 1u : 0u;
                        if constexpr (KIND == Kind::I8)
                            mma_i8(d, ad, bd, idesc, accum);
                        else
                            mma_f16(d, ad, bd, idesc, accum);
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == nst) {
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
        // ---------------- epilogue (warps 2 .. 2 + NEPI) ----------------
        const int q = warp & 3;                             // TMEM lane quarter it may read
        const int col_base = ((warp - 2) >> 2) * C::WCOLS;  // its share of the tile's columns
        const int et = threadIdx.x - 64;                    // < NEPI_T, and BN <= NEPI_T
        const EpiParams& e = s_epi;
        const int row = q * 32 + lane;
        const bool col_params = C::QUANT && (e.scale_axis == AX_N || e.bias_axis == AX_N);

        // Requant parameters of a tile: this thread's row scale / bias (registers) and the
        // tile's per-column values (column `et`, shared through shared memory). The global
        // loads of tile t + 1 are issued before tile t is processed, so their latency hides
        // behind its epilogue; they are turned into ColParams after it.
        struct Raw {
            float rscale, cscale;
            int32_t rbias, cbias;
        };
        auto load_raw = [&](int t, Raw& r) {
            int b, tm, tn;
            decode_tile(t, p, b, tm, tn);
            const int64_t grow = static_cast<int64_t>(tm) * BM + row;
            const int64_t gc = static_cast<int64_t>(tn) * BN + et;
            const bool rok = grow < p.Mk, cok = et < BN && gc < p.Nk;
            r.rscale = e.scale;
            r.cscale = 1.0f;
            r.rbias = 0;
            r.cbias = 0;
            if (e.scale_axis == AX_M && rok) r.rscale = e.scales[b * e.scale_bs + grow];
            if (e.bias_axis == AX_M && rok) r.rbias = e.bias[b * e.bias_bs + grow];
            if (e.scale_axis == AX_N && cok) r.cscale = e.scales[b * e.scale_bs + gc];
            if (e.bias_axis == AX_N && cok) r.cbias = e.bias[b * e.bias_bs + gc];
        };
        double r_se = 0.0, r_nms = 0.0;
        uint32_t r_ulo = 0, r_uhi = 0, r_bp = 0x80000000u;
        auto commit = [&](const Raw& r, int buf) {
            if (e.scale_axis != AX_N) make_scale_param(r.rscale, r_se, r_nms, r_ulo, r_uhi);
            r_bp = static_cast<uint32_t>(r.rbias) + 0x80000000u;
            if (col_params) {
                if (et < BN) {
                    ColParam c;
                    if (e.scale_axis == AX_N) {
                        make_scale_param(r.cscale, c.se, c.nms, c.ulo, c.uhi);
                    } else {  // the scale lives in each thread's registers
                        c.se = 0.0;
                        c.nms = 0.0;
                        c.ulo = 0;
                        c.uhi = 0;
                    }
                    c.bias_plus = static_cast<uint32_t>(r.cbias) + 0x80000000u;
                    c.pad = 0;
                    cparams[buf * BN + et] = c;
                    cbias[buf * BN + et] = c.bias_plus;
                }
                mbar_arrive(&pready[buf]);
            }
        };

        griddep_wait();  // parameters, outputs and stream-K scratch follow the previous kernel
        Sched sch(p);
        Work w, wn;
        bool has = sch.next(p, w);
        Raw raw;
        if (C::QUANT && has) {
            load_raw(w.tile, raw);
            commit(raw, 0);
        }
        for (int local = 0; has; ++local) {
            const bool has_n = sch.next(p, wn);
            int b, tm, tn;
            decode_tile(w.tile, p, b, tm, tn);
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int64_t grow = static_cast<int64_t>(tm) * BM + row;
            const int64_t gcol0 = static_cast<int64_t>(tn) * BN;
            const bool row_ok = grow < p.Mk;
            const ColParam* cp = cparams + acc * BN;
            const float r_fb = (OUT == Out::F32 && e.fbias_axis == AX_M && row_ok)
                                   ? e.fbias[grow] : 0.0f;
            if constexpr (OUT == Out::I32)  // the fused i32 epilogue's per-row bias
                r_bp = (e.bias_axis == AX_M && row_ok) ? static_cast<uint32_t>(e.bias[grow]) : 0u;

            if (col_params && !warp_wait(&pready[acc], aph, abort_flag, p.status,
                                         GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            if (!warp_wait(&tfull[acc], aph, abort_flag, p.status, GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            tc_fence_after();

            Raw raw_next;
            if (C::QUANT && has_n) load_raw(wn.tile, raw_next);

            const int64_t obase = static_cast<int64_t>(b) * e.obs + grow * e.ldo;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + col_base);
            const bool partial = w.nctr > 1;
            // stream-K partials of this warp's 32 x WCOLS region: slot j at + j * BM * BN
            uint32_t* part = nullptr;
            if (partial)
                part = p.sk_part +
                       static_cast<int64_t>(w.tile - p.dp_tiles) * p.sk_maxc * (BM * BN) +
                       static_cast<int64_t>((warp - 2) * 32 + lane) * C::WCOLS;
            // The requantize path for this tile's rows, then the chunk loop compiled for it.
            // Double-buffered TMEM reads: chunk c + 1 is in flight while chunk c is processed.
            int qm = QM_GENERAL;
            if constexpr (C::QUANT) qm = pick_quant_mode(e, r_se);
            auto chunks = [&](auto qm_tag) {
                constexpr int QM = decltype(qm_tag)::value;
                uint32_t va[32], vb[32];
                tmem_ld_chunk<CH>(tbase, va);
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    uint32_t(&cur)[32] = (c & 1) ? vb : va;
                    uint32_t(&nxt)[32] = (c & 1) ? va : vb;
                    tmem_wait_ld();
                    reg_fence<CH>(cur);
                    if (c + 1 < NCH) {
                        tmem_ld_chunk<CH>(tbase + (c + 1) * CH, nxt);
                    } else {
                        tc_fence_before();
                        mbar_arrive(&tempty[acc]);
                    }
                    if (partial) {
                        uint32_t* dst = part + static_cast<int64_t>(w.slot) * (BM * BN) + c * CH;
#pragma unroll
                        for (int g = 0; g < CH / 4; ++g)
                            st_global_v4(dst + 4 * g, cur[4 * g], cur[4 * g + 1], cur[4 * g + 2],
                                         cur[4 * g + 3]);
                    } else if (row_ok) {
                        epilogue_chunk<OUT, CH, QM>(cur, p.Nk, e, obase, gcol0 + col_base + c * CH,
                                                    cp + col_base + c * CH,
                                                    cbias + acc * BN + col_base + c * CH, r_se,
                                                    r_nms, r_ulo, r_uhi, r_bp, r_fb);
                    }
                }
            };
            with_quant_mode<C::QUANT>(qm, chunks);
            if (partial) {
                // Publish this slot, then count it; the last contributor of the region sums
                // every slot in slot order (exact for integers, fixed order for floats).
                __threadfence();
                __syncwarp();
                uint32_t last = 0;
                if (lane == 0) {
                    uint32_t* ctr = p.sk_ctr + static_cast<int64_t>(w.tile - p.dp_tiles) *
                                                   C::NEPI + (warp - 2);
                    uint32_t old = atomicAdd(ctr, 0u);
                    while (true) {
                        const uint32_t nv =
                            (old >> 8) == p.sk_epoch ? old + 1u : ((p.sk_epoch << 8) | 1u);
                        const uint32_t prev = atomicCAS(ctr, old, nv);
                        if (prev == old) {
                            last = (nv & 0xFFu) == static_cast<uint32_t>(w.nctr) ? 1u : 0u;
                            break;
                        }
                        old = prev;
                    }
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
#pragma unroll 1
                    for (int c = 0; c < NCH; ++c) {
                        uint32_t sum[32];
#pragma unroll
                        for (int i = 0; i < CH; ++i) sum[i] = 0u;
                        for (int j = 0; j < w.nctr; ++j) {
                            const uint32_t* src = part + static_cast<int64_t>(j) * (BM * BN) + c * CH;
#pragma unroll
                            for (int g = 0; g < CH / 4; ++g) {
                                const uint4 x = __ldcg(reinterpret_cast<const uint4*>(src) + g);
                                if constexpr (KIND == Kind::I8) {
                                    sum[4 * g + 0] += x.x;
                                    sum[4 * g + 1] += x.y;
                                    sum[4 * g + 2] += x.z;
                                    sum[4 * g + 3] += x.w;
                                } else {
                                    sum[4 * g + 0] = __float_as_uint(__uint_as_float(sum[4 * g + 0]) + __uint_as_float(x.x));
                                    sum[4 * g + 1] = __float_as_uint(__uint_as_float(sum[4 * g + 1]) + __uint_as_float(x.y));
                                    sum[4 * g + 2] = __float_as_uint(__uint_as_float(sum[4 * g + 2]) + __uint_as_float(x.z));
                                    sum[4 * g + 3] = __float_as_uint(__uint_as_float(sum[4 * g + 3]) + __uint_as_float(x.w));
                                }
                            }
                        }
                        if (row_ok)
                            epilogue_chunk<OUT, CH>(sum, p.Nk, e, obase, gcol0 + col_base + c * CH,
                                                    cp + col_base + c * CH,
                                                    cbias + acc * BN + col_base + c * CH, r_se,
                                                    r_nms, r_ulo, r_uhi, r_bp, r_fb);
                    }
                }
            }
            if (C::QUANT && has_n) commit(raw_next, acc ^ 1);
            w = wn;
            has = has_n;
        }
    }

    // mirrored outputs went to peer GPUs: make them visible system-wide before exiting
    if (s_epi.nmirror > 0 && warp >= 2) __threadfence_system();
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

void set_fast_div(FastDiv* f, uint32_t d) {
    if (d == 0) d = 1;
    uint32_t l = 0;
    while (l < 31 && (1u << l) < d) ++l;
    f->d = d;
    f->s = l;
    f->m = static_cast<uint32_t>(((static_cast<uint64_t>(1) << 32) *
                                  ((static_cast<uint64_t>(1) << l) - d)) / d + 1);
    f->pad = 0;
}

void set_tile_divs(GemmParams* gp) {
    const uint32_t gm = gp->group_m > 0 ? static_cast<uint32_t>(gp->group_m) : 1u;
    const uint32_t tm = gp->tiles_m > 0 ? static_cast<uint32_t>(gp->tiles_m) : 1u;
    set_fast_div(&gp->div_tpb, static_cast<uint32_t>(gp->tiles_per_batch));
    set_fast_div(&gp->div_band, gm * static_cast<uint32_t>(gp->tiles_n));
    set_fast_div(&gp->div_gm, gm);
    set_fast_div(&gp->div_glast, tm % gm ? tm % gm : gm);
}

static __device__ unsigned int g_status[64];

unsigned int* device_status_ptr() {
    static unsigned int* cache[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!cache[dev & 63]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
        cache[dev & 63] = static_cast<unsigned int*>(p) + (dev & 63);
    }
    return cache[dev & 63];
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

// A small per-thread cache of encoded tensor maps: serving loops call the same shapes over
// the same buffers, and encoding costs about a microsecond per operand.
struct TmapKey {
    const void* ptr;
    int64_t K, rows, ld, bs, batch;
    int es, box_rows;
    bool operator==(const TmapKey& o) const {
        return ptr == o.ptr && K == o.K && rows == o.rows && ld == o.ld && bs == o.bs &&
               batch == o.batch && es == o.es && box_rows == o.box_rows;
    }
};
struct TmapEntry {
    TmapKey key;
    CUtensorMap map;
    int dev;
};
constexpr int TMAP_CACHE = 16;
thread_local TmapEntry g_tmap_cache[TMAP_CACHE];
thread_local int g_tmap_used = 0, g_tmap_next = 0;

static int encode_operand_uncached(CUtensorMap* map, const Operand& op, int64_t K, int64_t batch,
                                   int es, int box_rows, char* err, size_t errlen);

int encode_operand(CUtensorMap* map, const Operand& op, int64_t K, int64_t batch, int es,
                   int box_rows, char* err, size_t errlen) {
    int dev = 0;
    cudaGetDevice(&dev);
    const TmapKey key{op.ptr, K, op.rows, op.ld, op.bs, batch, es, box_rows};
    for (int i = 0; i < g_tmap_used; ++i)
        if (g_tmap_cache[i].dev == dev && g_tmap_cache[i].key == key) {
            *map = g_tmap_cache[i].map;
            return 0;
        }
    int rc = encode_operand_uncached(map, op, K, batch, es, box_rows, err, errlen);
    if (rc) return rc;
    TmapEntry& e = g_tmap_cache[g_tmap_next];
    e.key = key;
    e.map = *map;
    e.dev = dev;
    g_tmap_next = (g_tmap_next + 1) % TMAP_CACHE;
    if (g_tmap_used < TMAP_CACHE) ++g_tmap_used;
    return 0;
}

int encode_output_u8(CUtensorMap* map, void* out, int64_t cols, int64_t rows, int64_t batch,
                     int64_t ldo, int64_t obs, int box_cols, int box_rows, char* err,
                     size_t errlen) {
    int dev = 0;
    cudaGetDevice(&dev);
    // cached with the operand maps; a negative element size marks an output map
    const TmapKey key{out, cols, rows, ldo, batch > 1 ? obs : 0, batch, -box_cols, box_rows};
    for (int i = 0; i < g_tmap_used; ++i)
        if (g_tmap_cache[i].dev == dev && g_tmap_cache[i].key == key) {
            *map = g_tmap_cache[i].map;
            return 0;
        }
    PFN_tmapEncodeTiled enc = get_encode();
    if (!enc) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled is unavailable (driver too old?)");
        return 5;
    }
    if ((reinterpret_cast<uintptr_t>(out) & 15) || (ldo & 15) || ldo <= 0 ||
        (batch > 1 && (obs & 15)) || (box_cols != 32 && box_cols != 64 && box_cols != 128)) {
        snprintf(err, errlen, "gemmkit: internal error: output not TMA-aligned");
        return 1;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(batch > 1 ? batch : 1)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldo),
                             static_cast<cuuint64_t>(batch > 1 ? obs : ldo * rows)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = box_cols == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, out, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled (output) failed (%d)",
                 static_cast<int>(r));
        return 3;
    }
    TmapEntry& e = g_tmap_cache[g_tmap_next];
    e.key = key;
    e.map = *map;
    e.dev = dev;
    g_tmap_next = (g_tmap_next + 1) % TMAP_CACHE;
    if (g_tmap_used < TMAP_CACHE) ++g_tmap_used;
    return 0;
}

int encode_mn_operand(CUtensorMap* map, const Operand& op, int64_t K, int box_cols, char* err,
                      size_t errlen) {
    int dev = 0;
    cudaGetDevice(&dev);
    // cached with the operand maps; element size -1000 - box_cols marks an MN-major map
    const TmapKey key{op.ptr, K, op.rows, op.mn_ld, 0, 1, -1000 - box_cols, 128};
    for (int i = 0; i < g_tmap_used; ++i)
        if (g_tmap_cache[i].dev == dev && g_tmap_cache[i].key == key) {
            *map = g_tmap_cache[i].map;
            return 0;
        }
    PFN_tmapEncodeTiled enc = get_encode();
    if (!enc) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled is unavailable (driver too old?)");
        return 5;
    }
    if ((reinterpret_cast<uintptr_t>(op.ptr) & 15) || (op.mn_ld & 15) || op.mn_ld < op.rows) {
        snprintf(err, errlen, "gemmkit: internal error: MN-major operand not TMA-aligned");
        return 1;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(op.rows), static_cast<cuuint64_t>(K), 1};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(op.mn_ld),
                             static_cast<cuuint64_t>(op.mn_ld) * static_cast<cuuint64_t>(K)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = box_cols == 32   ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                   : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(op.ptr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled (MN-major) failed (%d)",
                 static_cast<int>(r));
        return 3;
    }
    TmapEntry& e = g_tmap_cache[g_tmap_next];
    e.key = key;
    e.map = *map;
    e.dev = dev;
    g_tmap_next = (g_tmap_next + 1) % TMAP_CACHE;
    if (g_tmap_used < TMAP_CACHE) ++g_tmap_used;
    return 0;
}

int encode_tiled_operand(CUtensorMap* map, const Operand& op, int64_t K, int box_rows, char* err,
                         size_t errlen) {
    PFN_tmapEncodeTiled enc = get_encode();
    if (!enc) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled is unavailable (driver too old?)");
        return 5;
    }
    const int64_t nkb = (K + BKB - 1) / BKB;
    if ((reinterpret_cast<uintptr_t>(op.ptr) & 15) || op.slab != op.rows * BKB) {
        snprintf(err, errlen, "gemmkit: internal error: tiled operand geometry");
        return 1;
    }
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(BKB), static_cast<cuuint64_t>(op.rows),
                          static_cast<cuuint64_t>(nkb)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(BKB), static_cast<cuuint64_t>(op.slab)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(BKB), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(op.ptr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "gemmkit: cuTensorMapEncodeTiled (tiled) failed (%d)",
                 static_cast<int>(r));
        return 3;
    }
    return 0;
}

static int encode_operand_uncached(CUtensorMap* map, const Operand& op, int64_t K, int64_t batch,
                                   int es, int box_rows, char* err, size_t errlen) {
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
static int launch_one(const TcProblem& pr, const TcPlan& plan, GemmParams gp, char* err,
                      size_t errlen) {
    using C = TileCfg<OUT, BN>;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    CUtensorMap ta, tb;
    memset(&ta, 0, sizeof(ta));
    memset(&tb, 0, sizeof(tb));
    int rc = 0;
    if (pr.a.slab == 0 && (rc = encode_operand(&ta, pr.a, pr.K, pr.batch, ES, BM, err, errlen)))
        return rc;
    if (pr.b.mn_ld > 0) {
        if (ES != 1 || (BN != 32 && BN != 64 && BN != 128)) {
            snprintf(err, errlen, "gemmkit: internal error: MN-major operand for this kernel");
            return 1;
        }
        rc = encode_mn_operand(&tb, pr.b, pr.K, BN, err, errlen);
        if (rc) return rc;
        gp.b_mn = 1;
    } else if (pr.b.slab == 0 &&
               (rc = encode_operand(&tb, pr.b, pr.K, pr.batch, ES, BN, err, errlen))) {
        return rc;
    }
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
    gp.tiles_n = plan.tiles_n;
    gp.tiles_per_batch = gp.tiles_m * gp.tiles_n;
    set_tile_divs(&gp);
    gp.num_tiles = plan.num_tiles;
    gp.dp_tiles = plan.dp_tiles;
    gp.sk_iters = plan.sk_iters;
    gp.sk_maxc = plan.sk_maxc;
    if (plan.sk_iters > 0) {
        if (!pr.sk_part || !pr.sk_ctr) {
            snprintf(err, errlen, "gemmkit: internal error: stream-K plan without scratch");
            return 1;
        }
        gp.sk_part = pr.sk_part;
        gp.sk_ctr = pr.sk_ctr;
        gp.sk_epoch = pr.sk_epoch & 0xFFFFFFu;
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(plan.grid));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = pr.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pr.pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, gp);
    if (e == cudaSuccess) e = cudaGetLastError();
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

void plan_tc_gemm(const TcProblem& p, bool allow_sk, TcPlan* plan) {
    TcPlan& pl = *plan;
    memset(&pl, 0, sizeof(pl));
    pl.bn = pick_bn(p);
    if (p.b.mn_ld > 0 && pl.bn > 128) pl.bn = 128;  // an MN-major B box spans <= 128 bytes
    pl.nepi = pl.bn >= 64 ? 8 : 4;
    pl.tiles_m = static_cast<int>((p.Mk + BM - 1) / BM);
    pl.tiles_n = static_cast<int>((p.Nk + pl.bn - 1) / pl.bn);
    pl.num_tiles = pl.tiles_m * pl.tiles_n * static_cast<int>(p.batch);
    const int es = p.kind == Kind::I8 ? 1 : 2;
    pl.num_kb = static_cast<int>((p.K * es + BKB - 1) / BKB);
    const int sms = sm_count();
    pl.grid = pl.num_tiles < sms ? pl.num_tiles : sms;
    pl.dp_tiles = pl.num_tiles;
    // Stream-K tail: when the last wave of whole tiles would leave SMs idle, spread the K
    // blocks of that wave's tiles over every SM (needs >= 4 K blocks per tile to pay off).
    const int rem = pl.num_tiles % sms;
    if (allow_sk && pl.num_kb >= 4 && rem != 0) {
        const int sk_tiles = pl.num_tiles < sms ? pl.num_tiles : rem;
        const int64_t iters = static_cast<int64_t>(sk_tiles) * pl.num_kb;
        if (iters >= sms) {
            const int64_t per = iters / sms;  // >= 1
            const int64_t maxc = (pl.num_kb + per - 1) / per + 1;
            if (maxc <= 255) {
                pl.dp_tiles = pl.num_tiles - sk_tiles;
                pl.sk_iters = iters;
                pl.sk_maxc = static_cast<int>(maxc);
                pl.grid = sms;
                pl.part_words = static_cast<int64_t>(sk_tiles) * maxc * BM * pl.bn;
                pl.ctr_words = static_cast<int64_t>(sk_tiles) * pl.nepi;
            }
        }
    }
}

void plan_tc_gemm2(const TcProblem& p, bool allow_sk, bool allow_pair, bool allow_gemv,
                   TcPlan* plan, bool allow_gemv_sk) {
    if (allow_gemv && p.b.mn_ld == 0 && plan_gemv(p, plan, allow_gemv_sk)) return;
    plan_tc_gemm(p, allow_sk, plan);
    TcPlan& pl = *plan;
    if (!allow_pair || pl.bn != 256 || p.Mk < 2 * BM) return;
    const int sms = sm_count();
    const int tiles_m2 = static_cast<int>((p.Mk + 2 * BM - 1) / (2 * BM));
    const int tiles = tiles_m2 * pl.tiles_n * static_cast<int>(p.batch);
    if (tiles < sms / 2) return;
    // the pair kernel: 256 x 256 tiles, one tile per cluster of two CTAs, no stream-K tail
    pl.pair = 1;
    pl.nepi = 8;
    pl.tiles_m = tiles_m2;
    pl.num_tiles = tiles;
    pl.grid = 2 * (tiles < sms / 2 ? tiles : sms / 2);
    pl.dp_tiles = tiles;
    pl.sk_iters = 0;
    pl.sk_maxc = 0;
    pl.part_words = 0;
    pl.ctr_words = 0;
}

template <Kind KIND, Out OUT>
static int dispatch_bn(const TcProblem& pr, const TcPlan& plan, const GemmParams& gp, char* err,
                       size_t errlen) {
    switch (plan.bn) {
        case 16: return launch_one<KIND, OUT, 16>(pr, plan, gp, err, errlen);
        case 32: return launch_one<KIND, OUT, 32>(pr, plan, gp, err, errlen);
        case 64: return launch_one<KIND, OUT, 64>(pr, plan, gp, err, errlen);
        case 128: return launch_one<KIND, OUT, 128>(pr, plan, gp, err, errlen);
        case 192: return launch_one<KIND, OUT, 192>(pr, plan, gp, err, errlen);
        case 256: return launch_one<KIND, OUT, 256>(pr, plan, gp, err, errlen);
        default:
            snprintf(err, errlen, "gemmkit: unsupported tile width %d", plan.bn);
            return 1;
    }
}

int launch_tc_gemm_planned(const TcProblem& pr, const TcPlan& plan, char* err, size_t errlen) {
    GemmParams gp;
    memset(&gp, 0, sizeof(gp));
    gp.Mk = pr.Mk;
    gp.Nk = pr.Nk;
    gp.K = static_cast<int32_t>(pr.K);
    gp.batch = static_cast<int32_t>(pr.batch);
    gp.tiles_m = plan.tiles_m;
    gp.num_kb = plan.num_kb;
    gp.group_m = 16;
    gp.a_batched = pr.a.bs != 0 && pr.batch > 1;
    gp.b_batched = pr.b.bs != 0 && pr.batch > 1;
    gp.timeout_ns = 4000000000ull;
    gp.status = device_status_ptr();
    gp.stages = pr.stages;
    gp.f32q = pr.f32q;
    gp.e = pr.e;
    if (plan.gemv) return launch_gemv(pr, plan, err, errlen);
    if (plan.pair) return launch_pair(pr, plan, gp, err, errlen);
    if (pr.kind == Kind::I8) {
        if (pr.out == Out::I32) return dispatch_bn<Kind::I8, Out::I32>(pr, plan, gp, err, errlen);
        if (pr.out == Out::Q8) return dispatch_bn<Kind::I8, Out::Q8>(pr, plan, gp, err, errlen);
        if (pr.out == Out::U8) return dispatch_bn<Kind::I8, Out::U8>(pr, plan, gp, err, errlen);
    } else if (pr.out == Out::F32) {
        if (pr.kind == Kind::BF16)
            return dispatch_bn<Kind::BF16, Out::F32>(pr, plan, gp, err, errlen);
        return dispatch_bn<Kind::F16, Out::F32>(pr, plan, gp, err, errlen);
    }
    snprintf(err, errlen, "gemmkit: internal error: unsupported kernel combination");
    return 1;
}

int launch_tc_gemm(const TcProblem& pr, char* err, size_t errlen) {
    TcPlan plan;
    plan_tc_gemm(pr, false, &plan);
    return launch_tc_gemm_planned(pr, plan, err, errlen);
}

}  // namespace gk
