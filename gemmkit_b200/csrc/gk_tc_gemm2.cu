// gk_tc_gemm2.cu -- the CTA-pair form of the tensor-core GEMM (tcgen05 cta_group::2).
//
// Two CTAs of a cluster on two SMs compute one 256 x BN tile: each loads its own 128 rows of A
// and its half (BN/2 rows) of B into its shared memory; the even CTA (the leader) issues
// tcgen05.mma.cta_group::2 with M = 256, which reads A and B from both CTAs' shared memory at
// the same offsets and leaves each CTA's 128 accumulator rows in its own TMEM. Per MAC this
// moves a third less operand data into each SM than the one-CTA 128 x BN tile.
//
// Synchronisation across the pair (all waits bounded, as in the one-CTA kernel):
//   full[s]    leader's barrier; both producers arrive with their byte counts and both CTAs'
//              TMA loads complete on it (cta_group::2 loads may signal the peer's barrier);
//   empty[s]   one per CTA; the leader's MMA thread commits to both when the stage is read;
//   tfull[a]   one per CTA; the leader's MMA thread commits to both when a tile is done;
//   tempty[a]  leader's; every epilogue warp of both CTAs arrives once it has read the tile.
// A cluster barrier after set-up and before teardown keeps either CTA from touching the
// other's barriers before they exist or after it has exited.
//
// Schedule: items t = pair, pair + npairs, ... Items below dp_tiles are whole 256 x BN tiles.
// When the last wave would leave at least half the pairs idle, its tiles are cut into two
// 256 x BN/2 halves (MMA N = BN/2, each CTA reading the first BN/4 rows of its B stage), so
// the tail costs half a tile instead of a whole one.
//
// Programmatic dependent launch: operands, parameters and outputs are touched only after
// griddep_wait(); each CTA releases the next kernel of the stream once its producer has issued
// its last copy, so that kernel's CTAs launch and set up while this one drains.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include "gk_engine.h"
#include "gk_sm100.cuh"
#include "gk_tc_common.cuh"

namespace gk {

// Back-off (ns) between polls of the 16-warp form's epilogue waits: 16 warps polling at once
// take issue slots from the warps that compute (the batched config measured 2 % faster with a
// 32-400 ns back-off than with a tight poll).
constexpr int EPI_SLEEP = 32;

// EPI16: 16 epilogue warps (four column groups, 16-column TMEM chunks) instead of 8, for
// quantized outputs whose K is one or two 128-byte blocks: the mainloop is then a few MMAs
// per tile and the requantize epilogue is the whole kernel, so more warps hide its latency
// (with a long K the 8-warp form is faster: the epilogue already hides behind the MMAs).
template <Out OUT, int BN, bool EPI16 = false>
struct PairCfg {
    static constexpr int NEPI = EPI16 ? 16 : 8;     // epilogue warps per CTA
    // the 16-warp form has a parameter warp (warp 2) that prepares each item's row and column
    // parameters for the epilogue warps, which then start at warp 3
    static constexpr int EPI_W0 = EPI16 ? 3 : 2;
    static constexpr int THREADS = 32 * EPI_W0 + 32 * NEPI;
    static constexpr int NGROUPS = NEPI / 4;        // column groups (4 TMEM lane quarters each)
    static constexpr int WCOLS = BN / NGROUPS;      // accumulator columns per epilogue warp
    static constexpr int CH = EPI16 ? 16 : 32;
    static constexpr int NCH = WCOLS / CH;
    static constexpr int A_BYTES = BM * BKB;        // this CTA's 128 rows of A
    static constexpr int B_BYTES = (BN / 2) * BKB;  // this CTA's half of B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr bool QUANT = (OUT == Out::Q8 || OUT == Out::U8);
    static constexpr int CP_BYTES = QUANT ? 2 * BN * (32 + 4) : 0;  // + compact bias_plus
    static constexpr int BAR_BYTES = 256;
    // 4-byte outputs keep a 4 KB tile per epilogue warp for mirrored (peer) stores
    static constexpr bool WIDE = (OUT == Out::I32 || OUT == Out::F32);
    static constexpr int EPI_STAGE_BYTES = WIDE ? NEPI * 32 * 32 * 4 : 0;
    // The 16-warp form writes C through TMA stores: each warp stages its 32 x WCOLS output
    // block in shared memory (two buffers, so one store drains while the next block fills).
    static constexpr int STORE_BLOCK = 32 * WCOLS;
    static constexpr int STORE_BYTES = EPI16 ? NEPI * 2 * STORE_BLOCK : 0;
    static constexpr int RAW_STAGES =
        (SMEM_LIMIT - 1024 - STORE_BYTES - BAR_BYTES - CP_BYTES - EPI_STAGE_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = RAW_STAGES > 10 ? 10 : RAW_STAGES;
    // layout after the 1024-byte alignment: stages | store blocks | barriers | params | epi
    static constexpr int OFF_STORE = STAGES * STAGE_BYTES;
    static constexpr int OFF_BARS = OFF_STORE + STORE_BYTES;
    static constexpr int OFF_CP = OFF_BARS + BAR_BYTES;
    static constexpr int OFF_EPI = OFF_CP + CP_BYTES;
    static constexpr int SMEM = 1024 + OFF_EPI + EPI_STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static_assert(BN == 128 || BN == 256, "pair tile width");
    static_assert(!EPI16 || WCOLS == 64, "the store blocks use the 64-byte swizzle");
    static_assert(OFF_STORE % 1024 == 0 && STORE_BLOCK % 1024 == 0, "store block alignment");
    static_assert(STAGES >= 2 && SMEM <= SMEM_LIMIT, "shared memory budget");
    static_assert(2 * STAGES + 10 <= BAR_BYTES / 8, "barrier area");
    // The parameter warp's buffers (16-warp form, two items): per row {se, nms}, bias + 2^31
    // and clamp; per column bias + 2^31; the item's position and each lane quarter's path.
    static constexpr int PB_ROWSE = 0;                    // double2[BM]
    static constexpr int PB_ROWBP = PB_ROWSE + BM * 16;   // uint32_t[BM]
    static constexpr int PB_CLAMP = PB_ROWBP + BM * 4;    // uint2[BM]
    static constexpr int PB_COLB = PB_CLAMP + BM * 8;     // uint32_t[BN]
    static constexpr int PB_POS = PB_COLB + BN * 4;       // ItemPar
    static constexpr int PB_BYTES = (PB_POS + 64 + 127) / 128 * 128;
    static_assert(!EPI16 || 2 * PB_BYTES <= CP_BYTES, "parameter buffers");
};

// The position and per-quarter requantize path of an item (16-warp form's parameter buffer).
struct ItemPar {
    int b, tm, tn, c0, width;
    int qmode[4];
};

// Item t of the pair schedule: its tile, its first column inside the tile and its width.
template <int BN>
__device__ __forceinline__ void pair_item(int t, const GemmParams& p, int& tile, int& c0,
                                          int& width) {
    if (t < p.dp_tiles) {
        tile = t;
        c0 = 0;
        width = BN;
    } else {
        const int j = t - p.dp_tiles;
        tile = p.dp_tiles + (j >> 1);
        c0 = (j & 1) * (BN / 2);
        width = BN / 2;
    }
}

// The requantize loop of one warp's share of an item when every choice is settled before it:
// a per-row or per-tensor scale (se / nms, and the clamp ulo / uhi on the general path), the
// bias per column from the warp's shared-memory slice (BCOL) or per row (r_bp), ReLU or not,
// rows of C vector-aligned and no mirrors. Each chunk is one TMEM load, the exact requantize,
// saturating packs and 16-byte stores; of the warp's columns only the first ncol exist in C
// (a chunk that C cuts is stored byte by byte). The warp hands the accumulator back after its
// last TMEM load.
// With TMA (the 16-warp form, whole items) the chunks go instead into the warp's shared-memory
// store block sblk (32 rows of 64 bytes in the 64-byte swizzle: 16-byte piece j of row r at
// piece j ^ ((r >> 1) & 3), conflict-free) and one TMA tensor store of the block at (x, y, z)
// of tmC writes it to C; the store clips rows and columns past C. The caller has made sure the
// store that last read sblk is done.
// MODE: 0 the general requantize (requant_q with clamps), 1 the short one (requant_q_small),
// 2 the packed f32 one (requant_pair_f32: se then holds the f32 scale in both halves of its
// bits and the biases are bias + 0x4B400000).
template <int MODE, bool BCOL, bool RELU, bool U8, int CH, int NCH, bool TMA = false>
__device__ __forceinline__ void quant_rows_fast(uint32_t tbase, int nch, int64_t ncol,
                                                uint8_t* dst, bool row_ok, uint32_t bslice,
                                                double se, double nms, double magic,
                                                uint32_t r_bp, uint32_t ulo, uint32_t uhi, int zp,
                                                int lo, uint32_t tempty_caddr, int lane,
                                                uint8_t* sblk = nullptr,
                                                const CUtensorMap* tmC = nullptr, int x = 0,
                                                int y = 0, int z = 0) {
    // The next chunk's TMEM load is kept in flight while a chunk is requantized (32-column
    // chunks of the 8-warp form, and the 16-warp form's TMA path); the 16-warp form's plain
    // stores (cut items) load one chunk at a time.
    constexpr bool DB = CH == 32 || TMA;
    if constexpr (TMA) nch = NCH;  // a TMA-stored block is always the warp's whole width
    uint32_t va[32], vb[32];
    tmem_ld_chunk<CH>(tbase, va);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        if (c >= nch) break;
        uint32_t(&cur)[32] = (DB && (c & 1)) ? vb : va;
        uint32_t(&nxt)[32] = (DB && (c & 1)) ? va : vb;
        tmem_wait_ld();
        reg_fence<CH>(cur);
        if (c + 1 < nch) {
            if constexpr (DB) tmem_ld_chunk<CH>(tbase + (c + 1) * CH, nxt);
        } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(tempty_caddr);
        }
        uint32_t w[CH / 4];
#pragma unroll
        for (int g = 0; g < CH / 4; ++g) {
            uint4 bq = make_uint4(r_bp, r_bp, r_bp, r_bp);
            if constexpr (BCOL) bq = ld_shared_v4(bslice + static_cast<uint32_t>(c * CH + 4 * g) * 4u);
            const uint32_t bs[4] = {bq.x, bq.y, bq.z, bq.w};
            int qv[4];
            if constexpr (MODE == 2) {
                const uint64_t ss = static_cast<uint64_t>(__double_as_longlong(se));
                const uint32_t qoff = 0x4B400000u - static_cast<uint32_t>(zp);
                requant_pair_f32(cur[4 * g], cur[4 * g + 1], bs[0], bs[1], ss, qoff, qv[0], qv[1]);
                requant_pair_f32(cur[4 * g + 2], cur[4 * g + 3], bs[2], bs[3], ss, qoff, qv[2],
                                 qv[3]);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if constexpr (MODE == 1)
                    qv[t] = requant_q_small(cur[4 * g + t], bs[t], se, nms, magic);
                else if constexpr (MODE == 0)
                    qv[t] = requant_q(cur[4 * g + t], bs[t], se, nms, ulo, uhi, zp);
                if constexpr (RELU) qv[t] = max(qv[t], lo);
            }
            w[g] = pack4_sat<U8>(qv[0], qv[1], qv[2], qv[3]);
        }
        if constexpr (TMA) {
            static_assert(CH == 16, "one 16-byte piece per chunk and row");
            *reinterpret_cast<uint4*>(sblk + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
        } else if (row_ok) {
            if (c * CH + CH <= ncol) {
#pragma unroll
                for (int k = 0; k < CH / 16; ++k)
                    st_global_v4(dst + c * CH + 16 * k, w[4 * k], w[4 * k + 1], w[4 * k + 2],
                                 w[4 * k + 3]);
            } else {
                for (int i = 0; i < CH && c * CH + i < ncol; ++i)
                    dst[c * CH + i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
            }
        }
        if constexpr (!DB) {
            if (c + 1 < nch) tmem_ld_chunk<CH>(tbase + (c + 1) * CH, va);
        }
    }
    if constexpr (TMA) {
        fence_proxy_async_smem();  // the block's bytes, before the async proxy reads them
        __syncwarp();
        if (lane == 0) {
            tma_store_3d(tmC, sblk, x, y, z);
            bulk_commit_group();
        }
    }
}

template <Kind KIND, Out OUT, int BN, bool EPI16 = false>
__global__ void __launch_bounds__(PairCfg<OUT, BN, EPI16>::THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
    using C = PairCfg<OUT, BN, EPI16>;
    constexpr int STAGES = C::STAGES;
    // ring depth in use: the run-time cap (GEMMKIT_CUDA_STAGES) or the whole ring
    const int nst = (p.stages > 0 && p.stages < STAGES) ? p.stages : STAGES;
    constexpr int CH = C::CH;
    constexpr int NCH = C::NCH;
    constexpr int NEPI_T = 32 * C::NEPI;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    constexpr int BKE = BKB / ES;

    extern __shared__ uint8_t smem_raw[];
    // aligned by offsetting the shared array itself (not through an integer cast), so that
    // every access through smem stays a shared-memory access for the compiler
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sstore = smem + C::OFF_STORE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* pready = tfull + 4;
    uint64_t* pfree = tfull + 6;
    uint64_t* drain = tfull + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 9);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    ColParam* cparams = reinterpret_cast<ColParam*>(smem + C::OFF_CP);
    uint32_t* cbias = reinterpret_cast<uint32_t*>(cparams + 2 * BN);
    uint32_t* epi_stage = reinterpret_cast<uint32_t*>(smem + C::OFF_EPI);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int npairs = static_cast<int>(gridDim.x >> 1);
    const uint64_t tmo = p.timeout_ns;
    const int n_items = p.dp_tiles + 2 * (p.num_tiles - p.dp_tiles);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);  // the leader's producer; the peer's copies only add bytes
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * C::NEPI);  // every epilogue warp of both CTAs
            // column params of the 8-warp form (every epilogue thread), or the parameter
            // warp's item buffers of the 16-warp form (its 32 lanes; freed by the epilogue warps)
            mbar_init(&pready[a], EPI16 ? 32 : NEPI_T);
            mbar_init(&pfree[a], C::NEPI);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if constexpr (EPI16) prefetch_tmap(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // shared::cluster addresses of the barriers that cross the pair
    const uint32_t full_l = mapa_shared(smem_u32(&full[0]), 0);      // leader's full[0]
    const uint32_t tempty_l = mapa_shared(smem_u32(&tempty[0]), 0);  // leader's tempty[0]
    const uint32_t drain_own = mapa_shared(smem_u32(drain), rank);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            griddep_wait();
            int stage = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            bool ok = true;
            for (int t = pair; t < n_items && ok; t += npairs) {
                int tile, c0, width;
                pair_item<BN>(t, p, tile, c0, width);
                int b, tm, tn;
                decode_tile(tile, p, b, tm, tn);
                const int za = p.a_batched ? b : 0, zb = p.b_batched ? b : 0;
                const int arow = tm * 2 * BM + static_cast<int>(rank) * BM;
                // this CTA's width/2 rows of B; a half item loads the full box and uses its
                // first BN/4 rows
                const int brow = tn * BN + c0 + static_cast<int>(rank) * (width / 2);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                                   GK_DEV_TIMEOUT_PRODUCER, tmo)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = full_l + 8u * stage;
                    // One local arrival expecting both CTAs' bytes. The peer's copies may land
                    // first: the transaction count goes negative until this arrival, and the
                    // phase cannot complete before it. (A cluster-scope release arrival per
                    // stage from each CTA serialised the ring behind the previous copies.)
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
                    if (p.a_tiled)
                        tma_load_3d_pair(sA + stage * C::A_BYTES, &tmA, fb, 0, arow, kb);
                    else
                        tma_load_3d_pair(sA + stage * C::A_BYTES, &tmA, fb, kb * BKE, arow, za);
                    if (p.b_tiled)
                        tma_load_3d_pair(sB + stage * C::B_BYTES, &tmB, fb, 0, brow, kb);
                    else
                        tma_load_3d_pair(sB + stage * C::B_BYTES, &tmB, fb, kb * BKE, brow, zb);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == nst) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            griddep_launch_dependents();
            // Drain (leader): its full barriers count both CTAs' copies.
            if (leader) {
                int dummy = 0;
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s))
                        mbar_wait(&full[s], (last_par >> s) & 1u, &dummy, p.status,
                                  GK_DEV_TIMEOUT_DRAIN, tmo);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader) ----------------
            uint32_t idesc_w, idesc_h;  // whole tile, half tile
            if constexpr (KIND == Kind::I8) {
                idesc_w = idesc_i8(2 * BM, BN);
                idesc_h = idesc_i8(2 * BM, BN / 2);
            } else {
                idesc_w = idesc_f16(2 * BM, BN, KIND == Kind::BF16);
                idesc_h = idesc_f16(2 * BM, BN / 2, KIND == Kind::BF16);
            }
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int local = 0;
            for (int t = pair; t < n_items && ok; t += npairs, ++local) {
                const uint32_t idesc = t < p.dp_tiles ? idesc_w : idesc_h;
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
                            mma_i8_pair(d, ad, bd, idesc, accum);
                        else
                            mma_f16_pair(d, ad, bd, idesc, accum);
                    }
                    mma_commit_pair_both(smem_u32(&empty[stage]), 0x3);
                    if (++stage == nst) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair_both(smem_u32(&tfull[acc]), 0x3);
            }
            mma_commit_pair(drain_own);
            int dummy = 0;
            mbar_wait(drain, 0, &dummy, p.status, GK_DEV_TIMEOUT_DRAIN, tmo);
        }
    } else if (EPI16 && warp == 2) {
        // ---------------- parameter warp (16-warp form) ----------------
        // For each item, into parameter buffer (item parity): the item's position, each row's
        // requantize constants and each column's bias, and the path of each 32-row quarter, so
        // that the epilogue warps start on an item with a few shared-memory loads.
        const EpiParams& e = p.e;
        uint8_t* pbase = reinterpret_cast<uint8_t*>(cparams);
        // The global loads of an item are issued one item ahead, into registers, so that their
        // latency passes while the epilogue warps still work on the buffer being refilled.
        struct Loads {
            int b, tm, tn, c0, width;
            float sc[4];
            int32_t rb[4];
            int32_t cb[BN / 32];
        };
        auto fetch = [&](int t, Loads& L) {
            int tile;
            pair_item<BN>(t, p, tile, L.c0, L.width);
            decode_tile(tile, p, L.b, L.tm, L.tn);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // row lane + 32 j: lane quarter j
                const int64_t grow =
                    static_cast<int64_t>(L.tm) * 2 * BM + rank * BM + lane + 32 * j;
                L.sc[j] = e.scale;
                L.rb[j] = 0;
                if (grow < p.Mk) {
                    if (e.scale_axis == AX_M) L.sc[j] = e.scales[L.b * e.scale_bs + grow];
                    if (e.bias_axis == AX_M) L.rb[j] = e.bias[L.b * e.bias_bs + grow];
                }
            }
#pragma unroll
            for (int i = 0; i < BN / 32; ++i) {
                const int c = lane + 32 * i;
                const int64_t gc = static_cast<int64_t>(L.tn) * BN + L.c0 + c;
                L.cb[i] = (e.bias_axis == AX_N && c < L.width && gc < p.Nk)
                              ? e.bias[L.b * e.bias_bs + gc] : 0;
            }
        };
        griddep_wait();  // parameters may belong to the previous kernel
        Loads L;
        if (pair < n_items) fetch(pair, L);
        int local = 0;
        for (int t = pair; t < n_items; t += npairs, ++local) {
            const int buf = local & 1;
            const uint32_t ph = (local >> 1) & 1;
            if (!warp_wait(&pfree[buf], ph ^ 1u, abort_flag, p.status, GK_DEV_TIMEOUT_EPILOGUE,
                           tmo))
                break;
            uint8_t* pb = pbase + buf * C::PB_BYTES;
            double2* rowse = reinterpret_cast<double2*>(pb + C::PB_ROWSE);
            uint32_t* rowbp = reinterpret_cast<uint32_t*>(pb + C::PB_ROWBP);
            uint2* rowclamp = reinterpret_cast<uint2*>(pb + C::PB_CLAMP);
            uint32_t* colb = reinterpret_cast<uint32_t*>(pb + C::PB_COLB);
            ItemPar* ip = reinterpret_cast<ItemPar*>(pb + C::PB_POS);
            // The packed f32 path takes the whole item when every |acc + bias| < 2^22
            // (|acc| <= K * 2^14 for i8 operands) and every scale is below 1.
            bool f32 = false;
            if (p.f32q) {
                uint32_t mb = 0;
                bool s_ok = true;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    mb = max(mb, static_cast<uint32_t>(abs(L.rb[j])));
                    s_ok = s_ok && L.sc[j] < 1.0f;
                }
#pragma unroll
                for (int i = 0; i < BN / 32; ++i) mb = max(mb, static_cast<uint32_t>(abs(L.cb[i])));
                mb = __reduce_max_sync(0xffffffffu, mb);
                f32 = __all_sync(0xffffffffu, s_ok) &&
                      static_cast<int64_t>(p.K) * 16384 + mb < (int64_t{1} << 22) &&
                      e.zp >= -(1 << 30) && e.zp <= (1 << 30);
            }
            const uint32_t boff = f32 ? 0x4B400000u : 0x80000000u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = lane + 32 * j;
                if (f32) {
                    const uint64_t ss = (static_cast<uint64_t>(__float_as_uint(L.sc[j])) << 32) |
                                        __float_as_uint(L.sc[j]);
                    rowse[r] = make_double2(__longlong_as_double(static_cast<long long>(ss)), 0.0);
                    rowbp[r] = static_cast<uint32_t>(L.rb[j]) + boff;
                    if (lane == 0) ip->qmode[j] = QM_F32;
                    continue;
                }
                double se, nms;
                make_scale_se(L.sc[j], se, nms);
                rowse[r] = make_double2(se, nms);
                rowbp[r] = static_cast<uint32_t>(L.rb[j]) + 0x80000000u;
                const bool small = __all_sync(0xffffffffu, se <= 0x1p-9);
                int qm = QM_GENERAL;
                if (small && (e.zp & 1) == 0)
                    qm = e.bias_axis == AX_N ? QM_SMALL_COLB : QM_SMALL_ROWB;
                if (qm == QM_GENERAL) {
                    uint32_t lo, hi;
                    make_scale_clamp(se, lo, hi);
                    rowclamp[r] = make_uint2(lo, hi);
                }
                if (lane == 0) ip->qmode[j] = qm;
            }
#pragma unroll
            for (int i = 0; i < BN / 32; ++i)
                colb[lane + 32 * i] = static_cast<uint32_t>(L.cb[i]) + boff;
            if (lane == 0) {
                ip->b = L.b;
                ip->tm = L.tm;
                ip->tn = L.tn;
                ip->c0 = L.c0;
                ip->width = L.width;
            }
            __syncwarp();
            mbar_arrive(&pready[buf]);  // every lane: its own writes are released
            if (t + npairs < n_items) fetch(t + npairs, L);
        }
    } else if constexpr (EPI16) {
        // ---------------- epilogue (16-warp form: warps 3 .. 18, both CTAs) ----------------
        const int ew = warp - C::EPI_W0;  // 0 .. NEPI - 1
        const int q = warp & 3;           // TMEM lane quarter (warp id mod 4)
        const int cgroup = ew >> 2;       // column group of the item
        const int row = q * 32 + lane;
        const EpiParams& e = p.e;
        const bool bcol = e.bias_axis == AX_N;
        const bool relu = e.relu != 0;
        const double magic = 6755399441055744.0 + static_cast<double>(e.zp);
        constexpr bool U8 = OUT == Out::U8;
        const uint8_t* pbase = reinterpret_cast<const uint8_t*>(cparams);
        griddep_wait();  // outputs may belong to the previous kernel
        int local = 0;
        for (int t = pair; t < n_items; t += npairs, ++local) {
            const int buf = local & 1;
            const uint32_t ph = (local >> 1) & 1;
            const int acc = buf;
            if (!warp_wait<EPI_SLEEP>(&pready[buf], ph, abort_flag, p.status,
                                      GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            const uint8_t* pb = pbase + buf * C::PB_BYTES;
            const ItemPar* ip = reinterpret_cast<const ItemPar*>(pb + C::PB_POS);
            const int b = ip->b, tm = ip->tm, tn = ip->tn, c0 = ip->c0, width = ip->width;
            const int qm = ip->qmode[q];
            const double2 sn = reinterpret_cast<const double2*>(pb + C::PB_ROWSE)[row];
            const uint32_t r_bp = reinterpret_cast<const uint32_t*>(pb + C::PB_ROWBP)[row];
            uint32_t r_ulo = 0, r_uhi = 0;
            if (qm == QM_GENERAL) {
                const uint2 cl = reinterpret_cast<const uint2*>(pb + C::PB_CLAMP)[row];
                r_ulo = cl.x;
                r_uhi = cl.y;
            }
            const int wcols = width / C::NGROUPS;
            const int col_base = cgroup * wcols;
            const int nch = wcols / CH;
            const int64_t grow = static_cast<int64_t>(tm) * 2 * BM + rank * BM + row;
            const bool row_ok = grow < p.Mk;
            const int64_t gcol0 = static_cast<int64_t>(tn) * BN + c0;
            const uint32_t bslice = smem_u32(pb + C::PB_COLB) + static_cast<uint32_t>(col_base) * 4u;
            uint8_t* dst = static_cast<uint8_t*>(e.out) + static_cast<int64_t>(b) * e.obs +
                           grow * e.ldo + gcol0 + col_base;
            const bool tma = wcols == C::WCOLS;
            uint8_t* sblk = sstore + (ew * 2 + buf) * C::STORE_BLOCK;
            if (tma) {
                if (lane == 0) bulk_wait_group_read<1>();  // the store of two items ago
                __syncwarp();
            }
            const int ty = tm * 2 * BM + static_cast<int>(rank) * BM + q * 32;
            if (!warp_wait<EPI_SLEEP>(&tfull[acc], ph, abort_flag, p.status,
                                      GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + col_base);
            auto run = [&](auto mode_tag, auto bcol_tag, auto relu_tag) {
                constexpr int SM = decltype(mode_tag)::value;
                constexpr bool BC = decltype(bcol_tag)::value;
                constexpr bool RL = decltype(relu_tag)::value;
                if (tma)
                    quant_rows_fast<SM, BC, RL, U8, CH, NCH, true>(
                        tbase, nch, p.Nk - (gcol0 + col_base), dst, row_ok, bslice, sn.x, sn.y,
                        magic, r_bp, r_ulo, r_uhi, e.zp, e.lo, tempty_l + 8u * acc, lane, sblk,
                        &tmC, static_cast<int>(gcol0 + col_base), ty, b);
                else
                    quant_rows_fast<SM, BC, RL, U8, CH, NCH>(
                        tbase, nch, p.Nk - (gcol0 + col_base), dst, row_ok, bslice, sn.x, sn.y,
                        magic, r_bp, r_ulo, r_uhi, e.zp, e.lo, tempty_l + 8u * acc, lane);
            };
            using T = std::true_type;
            using F = std::false_type;
            auto by_axes = [&](auto mode_tag) {
                if (bcol) {
                    if (relu) run(mode_tag, T{}, T{}); else run(mode_tag, T{}, F{});
                } else {
                    if (relu) run(mode_tag, F{}, T{}); else run(mode_tag, F{}, F{});
                }
            };
            if (qm == QM_F32)
                by_axes(std::integral_constant<int, 2>{});
            else if (qm != QM_GENERAL)
                by_axes(std::integral_constant<int, 1>{});
            else
                by_axes(std::integral_constant<int, 0>{});
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfree[buf]);  // this item's parameters are read
        }
    } else {
        // ---------------- epilogue (warps 2 .. 1 + NEPI, both CTAs) ----------------
        const int q = warp & 3;
        const int cgroup = (warp - 2) >> 2;  // which column group of the item this warp drains
        const int et = threadIdx.x - 64;
        const EpiParams& e = p.e;
        const int row = q * 32 + lane;
        // A per-column scale becomes ColParams once per item for the whole CTA (shared memory,
        // the pready barrier). With a per-row or per-tensor scale the only per-column value is
        // the bias, which each warp fetches for its own columns into a private shared-memory
        // slice, so the epilogue warps never wait for one another.
        const bool col_params = C::QUANT && e.scale_axis == AX_N;
        const bool warp_bias = C::QUANT && !col_params && e.bias_axis == AX_N;
        uint32_t* wslice = reinterpret_cast<uint32_t*>(cparams) + (warp - 2) * C::WCOLS;
        constexpr int WB = C::WCOLS / 32;  // bias values a lane fetches for its warp's slice
        // The 16-warp form (short K: the epilogue is the kernel) fetches the next item's slice
        // into registers ahead of time; the 8-warp form (long K: the epilogue hides behind the
        // mainloop) loads it when the slice is written, leaving its registers to the chunks.
        constexpr int WBR = EPI16 ? WB : 1;

        struct Pos {
            int b, tm, tn, c0, width;
        };
        auto locate = [&](int t) {
            Pos ps;
            int tile;
            pair_item<BN>(t, p, tile, ps.c0, ps.width);
            decode_tile(tile, p, ps.b, ps.tm, ps.tn);
            return ps;
        };
        struct Raw {
            float rscale, cscale;
            int32_t rbias, cbias;
            int32_t wb[WBR];
        };
        // bias j of this lane's share of the warp's slice for the item at ps
        auto slice_bias = [&](const Pos& ps, int j) {
            const int wcols = ps.width / C::NGROUPS;
            const int64_t gc0 = static_cast<int64_t>(ps.tn) * BN + ps.c0 + cgroup * wcols;
            const int cj = lane + 32 * j;
            return (cj < wcols && gc0 + cj < p.Nk) ? e.bias[ps.b * e.bias_bs + gc0 + cj] : 0;
        };
        auto load_raw = [&](const Pos& ps, Raw& r) {
            const int64_t grow = static_cast<int64_t>(ps.tm) * 2 * BM + rank * BM + row;
            const bool rok = grow < p.Mk;
            r.rscale = e.scale;
            r.cscale = 1.0f;
            r.rbias = 0;
            r.cbias = 0;
            if (e.scale_axis == AX_M && rok) r.rscale = e.scales[ps.b * e.scale_bs + grow];
            if (e.bias_axis == AX_M && rok) r.rbias = e.bias[ps.b * e.bias_bs + grow];
            if (col_params) {
                const int64_t gc = static_cast<int64_t>(ps.tn) * BN + ps.c0 + et;
                const bool cok = et < ps.width && gc < p.Nk;
                if (cok) r.cscale = e.scales[ps.b * e.scale_bs + gc];
                if (e.bias_axis == AX_N && cok) r.cbias = e.bias[ps.b * e.bias_bs + gc];
            }
            if constexpr (EPI16) {
                if (warp_bias) {
#pragma unroll
                    for (int j = 0; j < WB; ++j) r.wb[j] = slice_bias(ps, j);
                }
            }
        };
        double r_se = 0.0, r_nms = 0.0;
        uint32_t r_ulo = 0, r_uhi = 0, r_bp = 0x80000000u;
        auto commit = [&](const Raw& r, const Pos& ps, int buf) {
            // the clamp of a per-row scale is computed only if the general path runs
            if (e.scale_axis != AX_N) make_scale_se(r.rscale, r_se, r_nms);
            r_bp = static_cast<uint32_t>(r.rbias) + 0x80000000u;
            if (col_params) {
                if (et < BN) {
                    ColParam c;
                    make_scale_param(r.cscale, c.se, c.nms, c.ulo, c.uhi);
                    c.bias_plus = static_cast<uint32_t>(r.cbias) + 0x80000000u;
                    c.pad = 0;
                    cparams[buf * BN + et] = c;
                    cbias[buf * BN + et] = c.bias_plus;
                }
                mbar_arrive(&pready[buf]);
            }
            if (warp_bias) {
                __syncwarp();  // every lane is done with the previous item's slice
#pragma unroll
                for (int j = 0; j < WB; ++j) {
                    int32_t v;
                    if constexpr (EPI16)
                        v = r.wb[j];
                    else
                        v = slice_bias(ps, j);
                    wslice[lane + 32 * j] = static_cast<uint32_t>(v) + 0x80000000u;
                }
                __syncwarp();
            }
        };

        griddep_wait();  // parameters and outputs may belong to the previous kernel
        Raw raw;
        Pos pos = locate(pair);
        if (C::QUANT && pair < n_items) {
            load_raw(pos, raw);
            commit(raw, pos, 0);
        }
        int local = 0;
        for (int t = pair; t < n_items; t += npairs, ++local) {
            const int b = pos.b, tm = pos.tm, tn = pos.tn, c0 = pos.c0, width = pos.width;
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int64_t grow = static_cast<int64_t>(tm) * 2 * BM + rank * BM + row;
            const int64_t gcol0 = static_cast<int64_t>(tn) * BN + c0;
            const bool row_ok = grow < p.Mk;
            const ColParam* cp = cparams + acc * BN;
            const float r_fb = (OUT == Out::F32 && e.fbias_axis == AX_M && row_ok)
                                   ? e.fbias[grow] : 0.0f;
            if constexpr (OUT == Out::I32)  // the fused i32 epilogue's per-row bias
                r_bp = (e.bias_axis == AX_M && row_ok) ? static_cast<uint32_t>(e.bias[grow]) : 0u;
            const int wcols = width / C::NGROUPS;  // columns per warp group
            const int col_base = cgroup * wcols;
            const int nch = wcols / CH;
            const uint32_t* cb = warp_bias ? wslice : cbias + acc * BN + col_base;

            if (col_params && !warp_wait(&pready[acc], aph, abort_flag, p.status,
                                         GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            if (!warp_wait(&tfull[acc], aph, abort_flag, p.status, GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            tc_fence_after();

            const int t_next = t + npairs;
            Raw raw_next;
            if (C::QUANT && t_next < n_items) load_raw(locate(t_next), raw_next);

            const int64_t obase = static_cast<int64_t>(b) * e.obs + grow * e.ldo;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + col_base);
            // the requantize path for this tile's rows, then the chunk loop compiled for it
            int qm = QM_GENERAL;
            if constexpr (C::QUANT) {
                qm = pick_quant_mode(e, r_se);
                if (qm == QM_GENERAL && e.scale_axis != AX_N) make_scale_clamp(r_se, r_ulo, r_uhi);
            }
            // the straight-line loop covers every item of the 16-warp form (the host launches
            // that form only for such problems), and the common layouts of the 8-warp form
            bool fast = false;
            if constexpr (C::QUANT) fast = EPI16 || (!col_params && e.vec && e.nmirror == 0);
            if constexpr (C::QUANT) {
                if (fast) {
                    uint8_t* dst = static_cast<uint8_t*>(e.out) + obase + gcol0 + col_base;
                    const uint32_t bslice = smem_u32(wslice);
                    const double magic = 6755399441055744.0 + static_cast<double>(e.zp);
                    constexpr bool U8 = OUT == Out::U8;
                    // 16-warp form, whole item: the warp's block goes out through a TMA store
                    // from its store block of this item's parity (the store of two items ago
                    // on that block has finished reading it)
                    const bool tma = EPI16 && wcols == C::WCOLS;
                    uint8_t* sblk = sstore + ((warp - 2) * 2 + (local & 1)) * C::STORE_BLOCK;
                    if (EPI16 && tma) {
                        if (lane == 0) bulk_wait_group_read<1>();
                        __syncwarp();
                    }
                    const int ty = tm * 2 * BM + static_cast<int>(rank) * BM + q * 32;
                    auto run = [&](auto small_tag, auto bcol_tag, auto relu_tag) {
                        constexpr bool SM = decltype(small_tag)::value;
                        constexpr bool BC = decltype(bcol_tag)::value;
                        constexpr bool RL = decltype(relu_tag)::value;
                        if constexpr (EPI16) {
                            if (tma) {
                                quant_rows_fast<SM ? 1 : 0, BC, RL, U8, CH, NCH, true>(
                                    tbase, nch, p.Nk - (gcol0 + col_base), dst, row_ok, bslice,
                                    r_se, r_nms, magic, r_bp, r_ulo, r_uhi, e.zp, e.lo,
                                    tempty_l + 8u * acc, lane, sblk, &tmC,
                                    static_cast<int>(gcol0 + col_base), ty, b);
                                return;
                            }
                        }
                        quant_rows_fast<SM ? 1 : 0, BC, RL, U8, CH, NCH>(
                            tbase, nch, p.Nk - (gcol0 + col_base), dst, row_ok, bslice, r_se,
                            r_nms, magic, r_bp, r_ulo, r_uhi, e.zp, e.lo, tempty_l + 8u * acc,
                            lane);
                    };
                    using T = std::true_type;
                    using F = std::false_type;
                    const bool small = qm != QM_GENERAL;
                    if (small) {
                        if (warp_bias) {
                            if (e.relu) run(T{}, T{}, T{}); else run(T{}, T{}, F{});
                        } else {
                            if (e.relu) run(T{}, F{}, T{}); else run(T{}, F{}, F{});
                        }
                    } else {
                        if (warp_bias) {
                            if (e.relu) run(F{}, T{}, T{}); else run(F{}, T{}, F{});
                        } else {
                            if (e.relu) run(F{}, F{}, T{}); else run(F{}, F{}, F{});
                        }
                    }
                }
            }
            auto chunks = [&](auto qm_tag) {
                constexpr int QM = decltype(qm_tag)::value;
                uint32_t va[32], vb[32];
                tmem_ld_chunk<CH>(tbase, va);
    #pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    if (c >= nch) break;
                    uint32_t(&cur)[32] = (c & 1) ? vb : va;
                    uint32_t(&nxt)[32] = (c & 1) ? va : vb;
                    tmem_wait_ld();
                    reg_fence<CH>(cur);
                    if (c + 1 < nch) {
                        tmem_ld_chunk<CH>(tbase + (c + 1) * CH, nxt);
                    } else {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster_relaxed(tempty_l + 8u * acc);
                    }
                    const int64_t gc = gcol0 + col_base + c * CH;
                    if constexpr (C::WIDE && CH == 32) {
                        // mirrored full chunk: the whole warp stages it (conditions warp-uniform)
                        if (e.nmirror > 0 && e.vec && gc + CH <= p.Nk) {
                            epilogue_chunk_mirrored_wide<OUT>(cur, e, obase, gc, row_ok,
                                                              epi_stage + (warp - 2) * 1024, lane);
                            continue;
                        }
                    }
                    if (row_ok)
                        epilogue_chunk<OUT, CH, QM>(cur, p.Nk, e, obase, gc, cp + col_base + c * CH,
                                                    cb + c * CH, r_se, r_nms, r_ulo, r_uhi, r_bp,
                                                    r_fb);
                }
            };
            if constexpr (!EPI16) {
                if (!fast) with_quant_mode<C::QUANT>(qm, chunks);
            } else {
                (void)chunks;
            }
            // (the next item is located again rather than kept live across the chunk loop)
            if (t_next < n_items) pos = locate(t_next);
            if (C::QUANT && t_next < n_items) commit(raw_next, pos, acc ^ 1);
        }
    }

    // the epilogue's TMA stores complete before the CTA (and its shared memory) goes away
    if constexpr (EPI16) {
        if (warp >= 2 && lane == 0) bulk_wait_group_all();
    }
    // mirrored outputs went to peer GPUs: make them visible system-wide before exiting
    if (p.e.nmirror > 0 && warp >= 2) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
}

template <Kind KIND, Out OUT, int BN, bool EPI16 = false>
static int launch_pair_one(const TcProblem& pr, const TcPlan& plan, GemmParams gp, char* err,
                           size_t errlen) {
    using C = PairCfg<OUT, BN, EPI16>;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    CUtensorMap ta, tb;
    int rc;
    if (pr.a.slab)
        rc = encode_tiled_operand(&ta, pr.a, pr.K, BM, err, errlen);
    else
        rc = encode_operand(&ta, pr.a, pr.K, pr.batch, ES, BM, err, errlen);
    if (rc) return rc;
    if (pr.b.slab)
        rc = encode_tiled_operand(&tb, pr.b, pr.K, BN / 2, err, errlen);
    else
        rc = encode_operand(&tb, pr.b, pr.K, pr.batch, ES, BN / 2, err, errlen);
    if (rc) return rc;
    gp.a_tiled = pr.a.slab ? static_cast<const uint8_t*>(pr.a.ptr) : nullptr;
    gp.b_tiled = pr.b.slab ? static_cast<const uint8_t*>(pr.b.ptr) : nullptr;
    gp.a_slab = pr.a.slab;
    gp.b_slab = pr.b.slab;
    // the 16-warp form stores C through TMA (byte outputs, vector-aligned, no mirrors)
    CUtensorMap tc;
    memset(&tc, 0, sizeof(tc));
    if constexpr (EPI16) {
        rc = encode_output_u8(&tc, pr.e.out, pr.Nk, pr.Mk, pr.batch, pr.e.ldo, pr.e.obs,
                              C::WCOLS, 32, err, errlen);
        if (rc) return rc;
    }
    auto kern = tc_gemm_pair_kernel<KIND, OUT, BN, EPI16>;
    static int attr_done[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) {
            snprintf(err, errlen, "gemmkit: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return 3;
        }
        attr_done[dev & 63] = 1;
    }
    gp.tiles_n = plan.tiles_n;
    gp.tiles_per_batch = gp.tiles_m * gp.tiles_n;
    set_tile_divs(&gp);
    gp.num_tiles = plan.num_tiles;
    gp.dp_tiles = plan.num_tiles;

    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    // A persistent grid must be co-resident: GPC boundaries can leave fewer two-SM clusters
    // than SMs / 2, so ask the runtime how many clusters of this kernel fit at once.
    static int max_clusters[64] = {0};
    int grid = plan.grid;
    {
        cudaLaunchConfig_t q;
        memset(&q, 0, sizeof(q));
        q.gridDim = dim3(static_cast<unsigned>(plan.grid));
        q.blockDim = dim3(C::THREADS);
        q.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 2;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        if (!max_clusters[dev & 63]) {
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) {
                cudaGetLastError();
                n = 1;
            }
            max_clusters[dev & 63] = n;
        }
        const int tiles = plan.num_tiles;
        const int pairs = tiles < max_clusters[dev & 63] ? tiles : max_clusters[dev & 63];
        grid = 2 * pairs;
        // Tail split: a last wave that would occupy at most half the pairs runs as half tiles.
        const int rem = tiles % pairs;
        if (rem > 0 && 2 * rem <= pairs) gp.dp_tiles = tiles - rem;
    }
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = pr.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pr.pdl ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, gp);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(err, errlen, "gemmkit: pair kernel launch failed: %s", cudaGetErrorString(e));
        return 3;
    }
    return 0;
}

int launch_pair(const TcProblem& pr, const TcPlan& plan, const GemmParams& gp, char* err,
                size_t errlen) {
    // the planner runs the pair kernel with 256-wide tiles only
    if (plan.bn != 256) {
        snprintf(err, errlen, "gemmkit: internal error: pair kernel tile width %d", plan.bn);
        return 1;
    }
#define GK_PAIR_CASE(K, O) \
    if (pr.kind == K && pr.out == O) return launch_pair_one<K, O, 256>(pr, plan, gp, err, errlen);
    // quantized output with a one- or two-block K: the epilogue-bound form, whose epilogue is
    // only the straight-line requantize loop (per-row or per-tensor scale, vector-aligned C,
    // no mirrors)
    if (pr.epi16 && pr.kind == Kind::I8 && plan.bn == 256 && plan.num_kb <= 2 &&
        pr.e.scale_axis != AX_N && pr.e.vec && pr.e.nmirror == 0) {
        if (pr.out == Out::Q8)
            return launch_pair_one<Kind::I8, Out::Q8, 256, true>(pr, plan, gp, err, errlen);
        if (pr.out == Out::U8)
            return launch_pair_one<Kind::I8, Out::U8, 256, true>(pr, plan, gp, err, errlen);
    }
    GK_PAIR_CASE(Kind::I8, Out::I32)
    GK_PAIR_CASE(Kind::I8, Out::Q8)
    GK_PAIR_CASE(Kind::I8, Out::U8)
    GK_PAIR_CASE(Kind::BF16, Out::F32)
    GK_PAIR_CASE(Kind::F16, Out::F32)
#undef GK_PAIR_CASE
    snprintf(err, errlen, "gemmkit: internal error: unsupported pair kernel combination");
    return 1;
}

}  // namespace gk
