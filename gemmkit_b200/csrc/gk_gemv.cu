// gk_gemv.cu -- the bandwidth-bound small-M path: D[Mk x Nk] = W[Mk x K] * X[Nk x K]^T for
// Nk <= 64, where W is the large operand, streamed once from HBM (for a prepacked right-hand
// side it is the packed buffer in the output-channel frame that the host's orientation choice
// gives it) and X holds the few activation rows, re-read from L2 by every CTA.
//
// gemmkit has no dedicated integer gemv route: a gemv-shaped integer product goes through its
// small_mn dot kernels or the general driver (gemmkit/src/dispatch/int.rs:164-200), and the
// prepacked entry always takes the general driver (gemmkit/src/dispatch/int.rs:249-256). The
// results are the same integers on every route because i32 wrap-around sums are associative
// (gemmkit/src/dispatch/int.rs:190-193), which is also what lets this kernel cut K and still
// match bit for bit.
//
// Design. The time of one call is a fixed start (CTA set-up, then about a microsecond before
// the first weight block lands), the streaming phase, and the tail. Streaming runs at the HBM
// copy rate once roughly three quarters of the SMs each keep a deep ring of 16 KB copies in
// flight, so:
//  * with enough 128-channel tiles, each CTA streams whole tiles (persistent over the tiles,
//    two TMEM accumulators so one tile's epilogue overlaps the next tile's copies);
//  * with few tiles, the K blocks of each tile are cut between the `split` CTAs of a thread-
//    block cluster, and the partial accumulators are summed on chip: the other CTAs store
//    theirs into the leader's (by then idle) stage ring through distributed shared memory and
//    the leader adds them in rank order and runs the epilogue. Nothing goes through global
//    memory, so the reduction costs two cluster barriers instead of fenced global round trips
//    behind the streaming traffic;
//  * launched with programmatic stream serialization, a call overlaps its set-up and its first
//    ring of prepacked-weight copies with the tail of the previous kernel of the stream (each
//    CTA releases the next kernel once it has issued its last copy). The
//    weights of a prepacked handle are immutable (gk_prepack_rhs_i8 returns after the packed
//    buffer is complete), so they may be fetched before the grid dependency resolves; the
//    activations, scales, bias and every store wait for it (griddep_wait).
// Roles: warp 0 streams (one 1-D bulk copy per weight block from the tiled prepacked layout, or
// a TMA tile of a plain K-contiguous operand, plus the X block); warp 1 issues tcgen05.mma
// M=128 x N=NB; warps 2..5 drain the accumulators (one TMEM lane quarter each).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "gk_engine.h"
#include "gk_sm100.cuh"
#include "gk_tc_common.cuh"

namespace gk {

// Stream-K split of the weight stream: at most this many CTAs share one tile (the planner
// gives every CTA at least half a tile's K blocks).
constexpr int GEMV_SK_MAXC = 3;

struct GemvParams {
    int64_t Mk, Nk;
    int32_t num_kb, tiles;
    int32_t split;           // CTAs (one cluster) per tile; 1 = whole tiles, persistent
    // Stream-K (sk = 1): the tiles x num_kb (tile, K block) units are cut into gridDim.x equal
    // contiguous runs, one per CTA. A tile shared by several CTAs leaves one 32-bit partial
    // accumulator tile per CTA in `part` (slot = CTA - first CTA of the tile); the last CTA to
    // finish a 32-row quarter of it (counted in ctr, tagged with `epoch`) sums the slots in
    // slot order and runs the epilogue.
    int32_t sk;
    int64_t units;
    uint32_t* part;
    uint32_t* ctr;
    uint32_t epoch;
    int32_t early_weights;   // fetch the first ring of weights before griddep_wait
    // the activation rows (Nk of them, x_row_bytes each at a pitch of x_ld bytes), for an L2
    // prefetch hint before griddep_wait
    const uint8_t* x;
    int64_t x_ld, x_row_bytes;

    const uint8_t* w_tiled;  // tiled prepacked weights, or nullptr: load through the tensor map
    int64_t w_slab;          // bytes between consecutive K blocks of w_tiled
    uint64_t timeout_ns;
    unsigned int* status;
    int32_t stages;  // ring depth cap (0: the whole ring)
    EpiParams e;
};

template <int NB>
struct GemvCfg {
    static constexpr int W_BYTES = BM * BKB;  // one 128-channel x 128-byte weight block
    static constexpr int X_BYTES = NB * BKB;  // the NB activation rows of the same K block
    static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
    static constexpr int BAR_BYTES = 256;
    static constexpr int CP_BYTES = NB * static_cast<int>(sizeof(ColParam) + 4);
    // N = 16: a 6-stage ring (110 KB) so that two CTAs fit on an SM, one of this call and one
    // of the next, which fills its ring while this one drains. Wider N need more registers than
    // two CTAs allow and keep one CTA with 8 stages.
    static constexpr int MIN_BLOCKS = NB == 16 ? 2 : 1;
    static constexpr int STAGES_WANT = NB == 16 ? 6 : 8;
    static constexpr int STAGES_FIT = (SMEM_LIMIT - 1024 - BAR_BYTES - CP_BYTES) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT < STAGES_WANT ? STAGES_FIT : STAGES_WANT;
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int SLOT_BYTES = BM * NB * 4;  // one CTA's partial accumulator tile
    static constexpr int MAX_SPLIT_RING = RING_BYTES / SLOT_BYTES + 1;
    // Accumulators in TMEM: four, so that the epilogue of a stream-K piece (its partial store,
    // fence and counter) never holds back the MMAs of the next items.
    static constexpr int NACC = 4;
    static constexpr int TMEM_COLS = NACC * NB < 32 ? 32 : NACC * NB;
    static constexpr int THREADS = 192;  // producer, MMA, 4 epilogue warps
    static constexpr int SMEM = 1024 + RING_BYTES + BAR_BYTES + CP_BYTES;
    static constexpr int CH = NB == 16 ? 16 : 32;  // TMEM columns per load
    static constexpr int NCH = NB / CH;
    static_assert(SMEM + static_cast<int>(sizeof(EpiParams)) <= SMEM_LIMIT, "gemv stages exceed shared memory");
    static_assert((STAGE_BYTES % 1024) == 0, "stages must keep the 1024-byte swizzle alignment");
    static_assert((2 * STAGES + 2 * NACC + 1) * 8 + 8 <= BAR_BYTES, "barrier area");
};

// One work item of a CTA: K blocks [k0, k1) of `tile`. In stream-K mode a tile shared by
// nctr CTAs (consecutive in blockIdx) is finished by the highest-numbered of them, its
// finisher; the others are writers and publish 32-bit partial accumulators in slot
// (CTA - first CTA of the tile). role: GEMV_WHOLE, GEMV_WRITER or GEMV_FINISHER.
enum : int { GEMV_WHOLE = 0, GEMV_WRITER = 1, GEMV_FINISHER = 2 };
struct GemvItem {
    int tile, k0, k1, slot, nctr, role;
};

// The CTA's work items, identical for every role.
//  * split > 1: K blocks [r*num_kb/split, (r+1)*num_kb/split) of tile blockIdx.x / split,
//    r = blockIdx.x % split (the CTA's rank in its cluster);
//  * sk: the CTA's run [s, e) of the units. Its run ends inside a tile it shares with the next
//    CTAs (it writes that tile's first K blocks: a writer piece) and starts inside a tile it
//    shares with the previous CTAs (it holds that tile's last K blocks: the finisher piece).
//    Order: the writer piece first, the whole tiles, the finisher piece last. A finisher
//    therefore waits only on lower-numbered CTAs, which have long finished their first item,
//    and it collects their partials while its own last MMAs run, so no reduction sits at the
//    end of the call;
//  * otherwise whole tiles blockIdx.x, blockIdx.x + gridDim.x, ...
struct GemvSched {
    int w_lo, w_cnt;
    bool has_wr, has_fin;
    GemvItem wr, fin;

    __device__ __forceinline__ static int64_t start(const GemvParams& p, int c) {
        return static_cast<int64_t>(c) * p.units / static_cast<int64_t>(gridDim.x);
    }
    // the CTA whose run holds unit T: the largest c with start(c) <= T
    __device__ __forceinline__ static int owner(const GemvParams& p, int64_t T) {
        const int64_t G = gridDim.x;
        const int64_t c = ((T + 1) * G + p.units - 1) / p.units - 1;
        return static_cast<int>(c < 0 ? 0 : (c >= G ? G - 1 : c));
    }
    __device__ __forceinline__ static GemvItem piece(const GemvParams& p, int tile, int k0, int k1,
                                                     int role) {
        const int64_t t0 = static_cast<int64_t>(tile) * p.num_kb;
        const int cf = owner(p, t0), cl = owner(p, t0 + p.num_kb - 1);
        return GemvItem{tile, k0, k1, static_cast<int>(blockIdx.x) - cf, cl - cf + 1, role};
    }
    __device__ __forceinline__ explicit GemvSched(const GemvParams& p) {
        w_lo = 0;
        w_cnt = 0;
        has_wr = has_fin = false;
        wr = fin = GemvItem{0, 0, 0, 0, 1, GEMV_WHOLE};
        if (!p.sk) return;
        const int nkb = p.num_kb;
        const int64_t s = start(p, blockIdx.x), e = start(p, blockIdx.x + 1);
        if (e <= s) return;
        const int tA = static_cast<int>(s / nkb), tB = static_cast<int>((e - 1) / nkb);
        const int sA = static_cast<int>(s - static_cast<int64_t>(tA) * nkb);
        const int eB = static_cast<int>(e - static_cast<int64_t>(tB) * nkb);  // 1 .. nkb
        if (tA == tB) {
            // the run lies inside one tile: [sA, eB)
            if (eB < nkb) {
                has_wr = true;
                wr = piece(p, tA, sA, eB, GEMV_WRITER);
            } else if (sA > 0) {
                has_fin = true;
                fin = piece(p, tA, sA, nkb, GEMV_FINISHER);
            }
        } else {
            if (sA > 0) {
                has_fin = true;
                fin = piece(p, tA, sA, nkb, GEMV_FINISHER);
            }
            if (eB < nkb) {
                has_wr = true;
                wr = piece(p, tB, 0, eB, GEMV_WRITER);
            }
        }
        w_lo = static_cast<int>((s + nkb - 1) / nkb);
        const int w_hi = static_cast<int>(e / nkb) - 1;
        w_cnt = w_hi >= w_lo ? w_hi - w_lo + 1 : 0;
    }
    __device__ __forceinline__ bool get(const GemvParams& p, int idx, GemvItem& it) const {
        if (p.sk) {
            if (has_wr) {
                if (idx == 0) {
                    it = wr;
                    return true;
                }
                --idx;
            }
            if (idx < w_cnt) {
                it = GemvItem{w_lo + idx, 0, p.num_kb, 0, 1, GEMV_WHOLE};
                return true;
            }
            if (has_fin && idx == w_cnt) {
                it = fin;
                return true;
            }
            return false;
        }
        if (p.split > 1) {
            if (idx > 0) return false;
            const int tile = static_cast<int>(blockIdx.x) / p.split;
            const int r = static_cast<int>(blockIdx.x) - tile * p.split;
            it = GemvItem{tile, static_cast<int>(static_cast<int64_t>(r) * p.num_kb / p.split),
                          static_cast<int>(static_cast<int64_t>(r + 1) * p.num_kb / p.split), 0,
                          1, GEMV_WHOLE};
            return true;
        }
        const int tile = static_cast<int>(blockIdx.x) + idx * static_cast<int>(gridDim.x);
        if (tile >= p.tiles) return false;
        it = GemvItem{tile, 0, p.num_kb, 0, 1, GEMV_WHOLE};
        return true;
    }
};

// The CTA's stages in streaming order, the same for the producer and the MMA issuer: item
// by item (whole tiles, cluster split), or in stream-K mode K block by K block across the
// CTA's items (at most GemvCfg::NACC), so that at any moment every CTA reads the same K-block
// slab of the weights (the slabs are contiguous in the tiled prepacked layout) and each item
// accumulates in its own TMEM accumulator.
struct GemvStage {
    int item, tile, kb, k0, k1;
};
struct GemvStages {
    int item, kb, nitems;
    __device__ __forceinline__ GemvStages(const GemvParams& p, const GemvSched& sch) {
        item = 0;
        kb = -1;
        nitems = p.sk ? (sch.has_wr ? 1 : 0) + sch.w_cnt + (sch.has_fin ? 1 : 0) : 0;
    }
    __device__ __forceinline__ bool next(const GemvParams& p, const GemvSched& sch, GemvStage& st) {
        GemvItem it;
        if (!p.sk) {
            while (true) {
                if (!sch.get(p, item, it)) return false;
                kb = kb < 0 ? it.k0 : kb + 1;
                if (kb < it.k1) {
                    st = GemvStage{item, it.tile, kb, it.k0, it.k1};
                    return true;
                }
                ++item;
                kb = -1;
            }
        }
        if (kb < 0) {
            kb = 0;
            item = 0;
        }
        while (kb < p.num_kb) {
            while (item < nitems) {
                const int j = item++;
                sch.get(p, j, it);
                if (it.k0 <= kb && kb < it.k1) {
                    st = GemvStage{j, it.tile, kb, it.k0, it.k1};
                    return true;
                }
            }
            item = 0;
            ++kb;
        }
        return false;
    }
};

__device__ __forceinline__ void epi_bar_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <Kind KIND, Out OUT, int NB>
__global__ void __launch_bounds__(192, GemvCfg<NB>::MIN_BLOCKS)
    gemv_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const GemvParams p) {
    using C = GemvCfg<NB>;
    constexpr int STAGES = C::STAGES;
    // The ring depth is the kernel's whole ring: the single-thread producer and MMA loops are
    // on the critical path of the streaming (each stage's turnaround bounds the bytes in
    // flight), and a run-time modulus measured slower; GEMMKIT_CUDA_STAGES does not apply.
    constexpr int nst = STAGES;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    constexpr int BKE = BKB / ES;
    constexpr bool QUANT = OUT == Out::Q8 || OUT == Out::U8;
    constexpr int CH = C::CH, NCH = C::NCH;

    extern __shared__ uint8_t smem_raw[];
    // aligned by offsetting the shared array itself (not through an integer cast), so that
    // every access through smem stays a shared-memory access for the compiler
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW = smem;
    uint8_t* sX = smem + STAGES * C::W_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::RING_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = tfull + C::NACC;
    uint64_t* drain = tfull + 2 * C::NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    ColParam* cp = reinterpret_cast<ColParam*>(smem + C::RING_BYTES + C::BAR_BYTES);
    uint32_t* cbias = reinterpret_cast<uint32_t*>(cp + NB);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint64_t tmo = p.timeout_ns;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < C::NACC; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    // The epilogue's parameters, copied to shared memory while the CTA starts: read from the
    // kernel's parameter space for the first time after the last accumulator is ready, each
    // field's constant-cache miss lands on the call's tail (about a microsecond in all).
    __shared__ EpiParams s_epi;
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(EpiParams) / 4); i += blockDim.x)
        reinterpret_cast<uint32_t*>(&s_epi)[i] = reinterpret_cast<const uint32_t*>(&p.e)[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // the epilogue's accumulator rows, kept past the loop for the cluster reduction
    uint32_t v[NCH][32];
    int64_t grow = 0;
    bool have = false;
    double r_se = 0.0, r_nms = 0.0;
    uint32_t r_ulo = 0, r_uhi = 0, r_bp = 0x80000000u;
    float r_fb = 0.0f;
    const int q = warp & 3;  // the TMEM lane quarter an epilogue warp may read
    const int row = q * 32 + lane;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer ----------------
            if (!p.w_tiled) prefetch_tmap(&tmW);
            prefetch_tmap(&tmX);
            auto issue_w = [&](int stage, int tile, int kb) {
                uint8_t* dw = sW + stage * C::W_BYTES;
                if (p.w_tiled)
                    bulk_load(dw,
                              p.w_tiled + static_cast<int64_t>(kb) * p.w_slab +
                                  static_cast<int64_t>(tile) * C::W_BYTES,
                              C::W_BYTES, &full[stage]);
                else
                    tma_load_3d(dw, &tmW, &full[stage], kb * BKE, tile * BM, 0);
            };
            // The first ring of weight blocks, ahead of the grid dependency (prepacked only).
            const GemvSched sch(p);
            GemvStage sg;
            int pre = 0;
            if (p.early_weights && p.w_tiled) {
                GemvStages it0(p, sch);
                for (; pre < nst && it0.next(p, sch, sg); ++pre) {
                    mbar_arrive_expect_tx(&full[pre], C::STAGE_BYTES);
                    issue_w(pre, sg.tile, sg.kb);
                }
            }
            griddep_wait();
            int stage = 0, idx = 0;
            uint32_t phase = 0, issued = 0, last_par = 0;
            if (!p.sk) {
                // item by item (kept as plain loops: this thread's per-stage turnaround is on
                // the streaming's critical path)
                GemvItem wi;
                bool ok = true;
                for (int n = 0; ok && sch.get(p, n, wi); ++n) {
                    const int tile = wi.tile;
                    for (int kb = wi.k0; kb < wi.k1; ++kb, ++idx) {
                        if (idx >= pre) {
                            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                                           GK_DEV_TIMEOUT_PRODUCER, tmo)) {
                                ok = false;
                                break;
                            }
                            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                            issue_w(stage, tile, kb);
                        }
                        tma_load_3d(sX + stage * C::X_BYTES, &tmX, &full[stage], kb * BKE, 0, 0);
                        issued |= 1u << stage;
                        last_par = (last_par & ~(1u << stage)) | (phase << stage);
                        if (++stage == nst) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            } else {
                auto one = [&](int tile, int kb) {
                    if (idx >= pre) {
                        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                                       GK_DEV_TIMEOUT_PRODUCER, tmo))
                            return false;
                        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                        issue_w(stage, tile, kb);
                    }
                    tma_load_3d(sX + stage * C::X_BYTES, &tmX, &full[stage], kb * BKE, 0, 0);
                    issued |= 1u << stage;
                    last_par = (last_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == nst) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    ++idx;
                    return true;
                };
                // stream-K: K block by K block across the items (writer, whole tiles, finisher)
                bool ok = true;
                for (int kb = 0; kb < p.num_kb && ok; ++kb) {
                    if (sch.has_wr && kb >= sch.wr.k0 && kb < sch.wr.k1) ok = one(sch.wr.tile, kb);
                    for (int j = 0; j < sch.w_cnt && ok; ++j) ok = one(sch.w_lo + j, kb);
                    if (ok && sch.has_fin && kb >= sch.fin.k0) ok = one(sch.fin.tile, kb);
                }
            }
            // This CTA has asked for all its data: the next kernel of the stream may start
            // placing its CTAs, so that their first copies queue up behind this call's last
            // ones (triggering any earlier was measured slower: the next call's copies then
            // compete with this call's streaming instead of filling the gap after it).
            griddep_launch_dependents();
            // Copies land in this CTA's shared memory: wait for the last one of every stage
            // before the CTA may exit (they have all landed already unless a wait gave up).
            int dummy = 0;
            for (int st = 0; st < STAGES; ++st)
                if (issued & (1u << st))
                    mbar_wait(&full[st], (last_par >> st) & 1u, &dummy, p.status,
                              GK_DEV_TIMEOUT_DRAIN, tmo);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t idesc;
            if constexpr (KIND == Kind::I8)
                idesc = idesc_i8(BM, NB);
            else
                idesc = idesc_f16(BM, NB, KIND == Kind::BF16);
            const GemvSched sch(p);
            int stage = 0;
            uint32_t phase = 0;
            if (!p.sk) {
                // item by item, the items taking turns on the accumulators (plain loops: this
                // thread's per-stage turnaround is on the streaming's critical path)
                GemvItem wi;
                int local = 0;
                bool ok = true;
                for (int n = 0; ok && sch.get(p, n, wi); ++n) {
                    const int k0 = wi.k0, k1 = wi.k1;
                    const int acc = local % C::NACC;
                    const uint32_t aph = (local / C::NACC) & 1u;
                    ++local;
                    if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, p.status,
                                   GK_DEV_TIMEOUT_MMA, tmo)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * NB);
                    for (int kb = k0; kb < k1; ++kb) {
                        if (!mbar_wait(&full[stage], phase, abort_flag, p.status,
                                       GK_DEV_TIMEOUT_MMA, tmo)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sW + stage * C::W_BYTES);
                        const uint32_t b0 = smem_u32(sX + stage * C::X_BYTES);
#pragma unroll
                        for (int ks = 0; ks < BKB / MMA_KB; ++ks) {
                            const uint64_t ad = sdesc_kmajor_sw128(a0 + ks * MMA_KB);
                            const uint64_t bd = sdesc_kmajor_sw128(b0 + ks * MMA_KB);
                            const uint32_t accum = (kb != k0 || ks != 0) ? 1u : 0u;
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
            } else {
                // stream-K: K block by K block, every item in its own accumulator (item order:
                // writer, whole tiles, finisher; the planner keeps them within NACC)
                int acc = 0;
                auto mma_stage = [&](int kb, int k0, int k1) {
                    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * NB);
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.status, GK_DEV_TIMEOUT_MMA,
                                   tmo))
                        return false;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sW + stage * C::W_BYTES);
                    const uint32_t b0 = smem_u32(sX + stage * C::X_BYTES);
#pragma unroll
                    for (int ks = 0; ks < BKB / MMA_KB; ++ks) {
                        const uint64_t ad = sdesc_kmajor_sw128(a0 + ks * MMA_KB);
                        const uint64_t bd = sdesc_kmajor_sw128(b0 + ks * MMA_KB);
                        const uint32_t accum = (kb != k0 || ks != 0) ? 1u : 0u;
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
                    if (kb == k1 - 1) mma_commit(&tfull[acc]);
                    return true;
                };
                const int nitems = (sch.has_wr ? 1 : 0) + sch.w_cnt + (sch.has_fin ? 1 : 0);
                bool ok = nitems <= C::NACC;
                if (!ok) {
                    *abort_flag = 1;
                    atomicOr(p.status, GK_DEV_TIMEOUT_MMA);
                }
                const int w0 = sch.has_wr ? 1 : 0;
                for (int kb = 0; kb < p.num_kb && ok; ++kb) {
                    if (sch.has_wr && kb >= sch.wr.k0 && kb < sch.wr.k1) {
                        acc = 0;
                        ok = mma_stage(kb, sch.wr.k0, sch.wr.k1);
                    }
                    for (int j = 0; j < sch.w_cnt && ok; ++j) {
                        acc = w0 + j;
                        ok = mma_stage(kb, 0, p.num_kb);
                    }
                    if (ok && sch.has_fin && kb >= sch.fin.k0) {
                        acc = nitems - 1;
                        ok = mma_stage(kb, sch.fin.k0, p.num_kb);
                    }
                }
            }
            // every MMA this CTA issued has finished before TMEM is released
            mma_commit(drain);
            int dummy = 0;
            mbar_wait(drain, 0, &dummy, p.status, GK_DEV_TIMEOUT_DRAIN, tmo);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int et = threadIdx.x - 64;
        const EpiParams& e = s_epi;
        // Hint the activation rows into L2 (128-byte lines spread over the grid's epilogue
        // threads): their first TMA loads after the dependency wait start the call's MMAs. A
        // hint only; the loads read whatever the previous kernel wrote.
        if (p.early_weights) {
            const int64_t lines_per_row = (p.x_row_bytes + 127) / 128;
            const int64_t lines = lines_per_row * p.Nk;
            for (int64_t l = static_cast<int64_t>(blockIdx.x) * 128 + et; l < lines;
                 l += static_cast<int64_t>(gridDim.x) * 128) {
                const int64_t r = l / lines_per_row, c = (l - r * lines_per_row) * 128;
                prefetch_l2(p.x + r * p.x_ld + c);
            }
        }
        griddep_wait();  // scales, bias and the output may belong to the previous kernel
        if (QUANT && (e.scale_axis == AX_N || e.bias_axis == AX_N)) {
            if (et < NB) {
                ColParam c;
                const bool ok = et < p.Nk;
                const float cs = (e.scale_axis == AX_N && ok) ? e.scales[et] : 1.0f;
                make_scale_param(cs, c.se, c.nms, c.ulo, c.uhi);
                const int32_t cb = (e.bias_axis == AX_N && ok) ? e.bias[et] : 0;
                c.bias_plus = static_cast<uint32_t>(cb) + 0x80000000u;
                c.pad = 0;
                cp[et] = c;
                cbias[et] = c.bias_plus;
            }
            epi_bar_sync();
        }

        const GemvSched sch(p);
        GemvItem wi;
        int local = 0;
        for (int n = 0; sch.get(p, n, wi); ++n) {
            const int tile = wi.tile;
            // stream-K: item n's own accumulator, used once; otherwise the items take turns
            const int acc = p.sk ? n : local % C::NACC;
            const uint32_t aph = p.sk ? 0u : (local / C::NACC) & 1u;
            ++local;
            if (p.sk && n >= C::NACC) break;
            grow = static_cast<int64_t>(tile) * BM + row;
            const bool row_ok = grow < p.Mk;
            // this row's requant constants, fetched while the MMAs run (loads issued before the
            // accumulator wait: with one item per CTA their latency is otherwise the call's tail)
            if constexpr (OUT == Out::F32)
                r_fb = (e.fbias_axis == AX_M && row_ok)
                           ? __uint_as_float(ld_global_issue_u32(e.fbias + grow)) : 0.0f;
            if constexpr (OUT == Out::I32)  // the fused i32 epilogue's per-row bias
                r_bp = (e.bias_axis == AX_M && row_ok) ? ld_global_issue_u32(e.bias + grow) : 0u;
            if constexpr (QUANT) {
                float rs = e.scale;
                uint32_t rb = 0;
                if (row_ok) {
                    if (e.scale_axis == AX_M)
                        rs = __uint_as_float(ld_global_issue_u32(e.scales + grow));
                    if (e.bias_axis == AX_M) rb = ld_global_issue_u32(e.bias + grow);
                }
                if (e.scale_axis != AX_N) make_scale_param(rs, r_se, r_nms, r_ulo, r_uhi);
                r_bp = rb + 0x80000000u;
                // the constants are computed here, not after the accumulator wait
                asm volatile("" ::"d"(r_se), "d"(r_nms), "r"(r_ulo), "r"(r_uhi), "r"(r_bp));
            }
            // A finisher gathers the writers' partials of its 32 rows while its own last MMAs
            // run: it waits (bounded) until the tile's writers have counted in, then sums their
            // slots in slot order (exact for integers, a fixed order for floats).
            uint32_t pre[NCH][CH];
            if (wi.role == GEMV_FINISHER) {
                uint32_t ok = 1;
                if (lane == 0) {
                    const volatile uint32_t* ctr = p.ctr + static_cast<int64_t>(tile) * 4 + q;
                    const uint32_t want = (p.epoch << 8) | static_cast<uint32_t>(wi.nctr - 1);
                    if (*ctr != want) {
                        const uint64_t t0 = globaltimer_ns();
                        while (*ctr != want) {
                            if (*abort_flag || globaltimer_ns() - t0 > tmo) {
                                if (!*abort_flag) {
                                    *abort_flag = 1;
                                    atomicOr(p.status, GK_DEV_TIMEOUT_EPILOGUE);
                                }
                                ok = 0;
                                break;
                            }
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) break;
                __threadfence();
                const uint32_t* base = p.part +
                                       static_cast<int64_t>(tile) * GEMV_SK_MAXC * (BM * NB) +
                                       static_cast<int64_t>(row) * NB;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
#pragma unroll
                    for (int i = 0; i < CH; ++i) pre[c][i] = 0u;
                for (int j = 0; j + 1 < wi.nctr; ++j) {
                    const uint4* src =
                        reinterpret_cast<const uint4*>(base + static_cast<int64_t>(j) * (BM * NB));
#pragma unroll
                    for (int c = 0; c < NCH; ++c)
#pragma unroll
                        for (int g = 0; g < CH / 4; ++g) {
                            const uint4 x = __ldcg(src + (c * CH) / 4 + g);
                            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                uint32_t& d = pre[c][4 * g + t];
                                if constexpr (KIND == Kind::I8)
                                    d += xs[t];
                                else
                                    d = __float_as_uint(__fadd_rn(__uint_as_float(d),
                                                                  __uint_as_float(xs[t])));
                            }
                        }
                }
            }
            if (!warp_wait(&tfull[acc], aph, abort_flag, p.status, GK_DEV_TIMEOUT_EPILOGUE, tmo))
                break;
            tc_fence_after();
            const uint32_t taddr =
                tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * NB);
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                if constexpr (CH == 16)
                    tmem_ld_x16(taddr + c * CH, v[c]);
                else
                    tmem_ld_x32(taddr + c * CH, v[c]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            have = true;
            if (p.split > 1) break;  // one item; summed across the cluster below
            if (wi.role == GEMV_WRITER) {
                // publish this CTA's partial rows in its slot, then count this warp's quarter
                uint32_t* mine = p.part + static_cast<int64_t>(tile) * GEMV_SK_MAXC * (BM * NB) +
                                 static_cast<int64_t>(wi.slot) * (BM * NB) +
                                 static_cast<int64_t>(row) * NB;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
#pragma unroll
                    for (int g = 0; g < CH / 4; ++g)
                        st_global_v4(mine + c * CH + 4 * g, v[c][4 * g], v[c][4 * g + 1],
                                     v[c][4 * g + 2], v[c][4 * g + 3]);
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    uint32_t* ctr = p.ctr + static_cast<int64_t>(tile) * 4 + q;
                    uint32_t old = atomicAdd(ctr, 0u);
                    while (true) {
                        const uint32_t nv =
                            (old >> 8) == p.epoch ? old + 1u : ((p.epoch << 8) | 1u);
                        const uint32_t prev = atomicCAS(ctr, old, nv);
                        if (prev == old) break;
                        old = prev;
                    }
                }
                continue;
            }
            if (wi.role == GEMV_FINISHER) {
#pragma unroll
                for (int c = 0; c < NCH; ++c)
#pragma unroll
                    for (int i = 0; i < CH; ++i) {
                        if constexpr (KIND == Kind::I8)
                            v[c][i] += pre[c][i];
                        else
                            v[c][i] = __float_as_uint(
                                __fadd_rn(__uint_as_float(pre[c][i]), __uint_as_float(v[c][i])));
                    }
            }
            int qm = QM_GENERAL;
            if constexpr (QUANT) qm = pick_quant_mode(e, r_se);
            with_quant_mode<QUANT>(qm, [&](auto qm_tag) {
                constexpr int QM = decltype(qm_tag)::value;
                if (row_ok) {
#pragma unroll
                    for (int c = 0; c < NCH; ++c)
                        epilogue_chunk<OUT, CH, QM>(v[c], p.Nk, e, grow * e.ldo, c * CH,
                                                    cp + c * CH, cbias + c * CH, r_se, r_nms,
                                                    r_ulo, r_uhi, r_bp, r_fb);
                }
            });
        }
    }

    tc_fence_before();
    __syncthreads();

    if (p.split > 1) {
        // Every CTA of the cluster is past its MMAs, so the leader's stage ring is idle: the
        // others store their accumulator rows into it (slot rank - 1), then the leader sums
        // them in rank order.
        const uint32_t rank = cluster_ctarank();
        cluster_sync();
        if (warp >= 2 && rank != 0 && have) {
            const uint32_t dst = mapa_shared(smem_u32(sW), 0) +
                                 (rank - 1) * C::SLOT_BYTES + static_cast<uint32_t>(row * NB * 4);
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
                for (int g = 0; g < CH / 4; ++g)
                    st_cluster_v4(dst + (c * CH + 4 * g) * 4, v[c][4 * g], v[c][4 * g + 1],
                                  v[c][4 * g + 2], v[c][4 * g + 3]);
        }
        cluster_sync();
        int qm = QM_GENERAL;
        if (QUANT && warp >= 2 && rank == 0 && have) qm = pick_quant_mode(s_epi, r_se);
        if (warp >= 2 && rank == 0 && have && grow < p.Mk) {
            for (int j = 1; j < p.split; ++j) {
                const uint32_t* src = reinterpret_cast<const uint32_t*>(
                    sW + (j - 1) * C::SLOT_BYTES + row * NB * 4);
#pragma unroll
                for (int c = 0; c < NCH; ++c)
#pragma unroll
                    for (int i = 0; i < CH; ++i) {
                        if constexpr (KIND == Kind::I8)
                            v[c][i] += src[c * CH + i];
                        else
                            v[c][i] = __float_as_uint(
                                __fadd_rn(__uint_as_float(v[c][i]), __uint_as_float(src[c * CH + i])));
                    }
            }
            with_quant_mode<QUANT>(qm, [&](auto qm_tag) {
                constexpr int QM = decltype(qm_tag)::value;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
                    epilogue_chunk<OUT, CH, QM>(v[c], p.Nk, s_epi, grow * s_epi.ldo, c * CH,
                                                cp + c * CH, cbias + c * CH, r_se, r_nms, r_ulo,
                                                r_uhi, r_bp, r_fb);
            });
        }
    }

    // mirrored outputs went to peer GPUs: make them visible system-wide before exiting
    if (s_epi.nmirror > 0 && warp >= 2) __threadfence_system();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Largest cluster count that can be resident at once for `split` (cached per kernel/split).
template <Kind KIND, Out OUT, int NB>
static int max_clusters(int split) {
    static int cache[64][17];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    int& c = cache[dev & 63][split];
    if (c == 0) {
        using C = GemvCfg<NB>;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(split * 64), 1, 1);
        cfg.blockDim = dim3(C::THREADS, 1, 1);
        cfg.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = static_cast<unsigned>(split);
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemv_kernel<KIND, OUT, NB>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = -1;
        }
        c = n > 0 ? n : -1;
    }
    return c;
}

template <Kind KIND, Out OUT, int NB>
static int launch_gemv_nb(const TcProblem& pr, const TcPlan& plan, GemvParams gp, char* err,
                          size_t errlen) {
    using C = GemvCfg<NB>;
    constexpr int ES = (KIND == Kind::I8) ? 1 : 2;
    CUtensorMap tw, tx;
    memset(&tw, 0, sizeof(tw));
    memset(&tx, 0, sizeof(tx));
    int rc = 0;
    if (pr.a.slab == 0 && (rc = encode_operand(&tw, pr.a, pr.K, 1, ES, BM, err, errlen)))
        return rc;
    if ((rc = encode_operand(&tx, pr.b, pr.K, 1, ES, NB, err, errlen))) return rc;
    if (pr.a.slab && (pr.a.rows % BM)) {
        snprintf(err, errlen, "gemmkit: internal error: tiled operand rows not padded to %d", BM);
        return 1;
    }
    gp.w_tiled = pr.a.slab ? static_cast<const uint8_t*>(pr.a.ptr) : nullptr;
    gp.w_slab = pr.a.slab;
    gp.x = static_cast<const uint8_t*>(pr.b.ptr);
    gp.x_ld = pr.b.ld * ES;
    gp.x_row_bytes = pr.K * ES;

    auto kern = gemv_kernel<KIND, OUT, NB>;
    static int attr_done[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM);
        if (e != cudaSuccess) {
            snprintf(err, errlen, "gemmkit: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? 5 : 3;
        }
        attr_done[dev & 63] = 1;
    }
    // The K split: bounded by the partial slots the leader's ring holds, and lowered until
    // every tile's cluster can be resident at once.
    int split = plan.split;
    if (split > C::MAX_SPLIT_RING) split = C::MAX_SPLIT_RING;
    while (split > 1) {
        const int mc = max_clusters<KIND, OUT, NB>(split);
        if (mc >= plan.tiles_m) break;
        --split;
    }
    if (split < 1) split = 1;
    gp.split = split;
    int grid = split > 1 ? plan.tiles_m * split
                         : (plan.tiles_m < sm_count() ? plan.tiles_m : sm_count());
    if (plan.gemv_sk) {
        if (!pr.sk_part || !pr.sk_ctr) {
            snprintf(err, errlen, "gemmkit: internal error: small-M stream-K without scratch");
            return 1;
        }
        gp.sk = 1;
        gp.split = 1;
        gp.units = plan.sk_iters;
        gp.part = pr.sk_part;
        gp.ctr = pr.sk_ctr;
        gp.epoch = pr.sk_epoch;
        grid = plan.grid;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = pr.stream;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (plan.pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (split > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = static_cast<unsigned>(split);
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, gp);
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

template <Kind KIND, Out OUT>
static int dispatch_gemv(const TcProblem& pr, const TcPlan& plan, const GemvParams& gp,
                         char* err, size_t errlen) {
    switch (plan.bn) {
        case 16: return launch_gemv_nb<KIND, OUT, 16>(pr, plan, gp, err, errlen);
        case 32: return launch_gemv_nb<KIND, OUT, 32>(pr, plan, gp, err, errlen);
        case 64: return launch_gemv_nb<KIND, OUT, 64>(pr, plan, gp, err, errlen);
        default:
            snprintf(err, errlen, "gemmkit: unsupported small-M width %d", plan.bn);
            return 1;
    }
}

bool plan_gemv(const TcProblem& p, TcPlan* plan, bool allow_sk) {
    // the activation side comes through a tensor map; a tiled operand there (a prepacked
    // right-hand side with <= 64 columns) stays with the general kernel
    if (p.batch != 1 || p.Nk > 64 || p.Nk < 1 || p.bn != 0 || p.b.slab != 0) return false;
    TcPlan pl;
    memset(&pl, 0, sizeof(pl));
    pl.gemv = 1;
    pl.pdl = p.pdl ? 1 : 0;
    pl.bn = p.Nk <= 16 ? 16 : (p.Nk <= 32 ? 32 : 64);
    pl.nepi = 4;
    pl.tiles_m = static_cast<int>((p.Mk + BM - 1) / BM);
    pl.tiles_n = 1;
    pl.num_tiles = pl.tiles_m;
    const int es = p.kind == Kind::I8 ? 1 : 2;
    pl.num_kb = static_cast<int>((p.K * es + BKB - 1) / BKB);
    const int sms = sm_count();
    // Whole tiles once about three quarters of the SMs have one; else cut K inside clusters
    // of up to 8 (portable cluster size) so that tiles * split approaches the SM count.
    int split = 1;
    const int max_split = p.gemv_split > 0 ? p.gemv_split : 8;
    if (static_cast<int64_t>(pl.tiles_m) * 4 < static_cast<int64_t>(sms) * 3) {
        split = sms / pl.tiles_m;
        if (split > max_split) split = max_split;
        if (split > pl.num_kb) split = pl.num_kb;
        if (split < 1) split = 1;
    }
    pl.split = split;
    pl.grid = split > 1 ? pl.tiles_m * split : (pl.tiles_m < sms ? pl.tiles_m : sms);
    // Stream-K over the weight stream when whole tiles would leave SMs idle or unevenly loaded
    // (tiles not a multiple of the SM count) and every SM still gets at least half a tile of
    // K blocks (so at most GEMV_SK_MAXC CTAs share a tile): the bytes each SM streams, which
    // bound a call, are then the same on every SM.
    const int64_t units = static_cast<int64_t>(pl.tiles_m) * pl.num_kb;
    // (a run of at most 2*num_kb + 1 units touches at most four tiles: one accumulator each)
    if (allow_sk && split == 1 && pl.num_kb >= 2 && pl.tiles_m % sms != 0 &&
        units / sms >= (pl.num_kb + 1) / 2 && units / sms <= 2 * pl.num_kb) {
        pl.gemv_sk = 1;
        pl.grid = sms;
        pl.sk_iters = units;
        pl.sk_maxc = GEMV_SK_MAXC;
        pl.ctr_words = static_cast<int64_t>(pl.tiles_m) * 4;
        pl.part_words = static_cast<int64_t>(pl.tiles_m) * GEMV_SK_MAXC * BM * pl.bn;
    }
    pl.dp_tiles = pl.num_tiles;
    *plan = pl;
    return true;
}

int launch_gemv(const TcProblem& pr, const TcPlan& plan, char* err, size_t errlen) {
    GemvParams gp;
    memset(&gp, 0, sizeof(gp));
    gp.Mk = pr.Mk;
    gp.Nk = pr.Nk;
    gp.num_kb = plan.num_kb;
    gp.tiles = plan.tiles_m;
    gp.early_weights = plan.pdl;
    gp.timeout_ns = 4000000000ull;
    gp.stages = pr.stages;
    gp.status = device_status_ptr();
    gp.e = pr.e;
    if (pr.kind == Kind::I8) {
        if (pr.out == Out::I32) return dispatch_gemv<Kind::I8, Out::I32>(pr, plan, gp, err, errlen);
        if (pr.out == Out::Q8) return dispatch_gemv<Kind::I8, Out::Q8>(pr, plan, gp, err, errlen);
        if (pr.out == Out::U8) return dispatch_gemv<Kind::I8, Out::U8>(pr, plan, gp, err, errlen);
    } else if (pr.out == Out::F32) {
        if (pr.kind == Kind::BF16)
            return dispatch_gemv<Kind::BF16, Out::F32>(pr, plan, gp, err, errlen);
        return dispatch_gemv<Kind::F16, Out::F32>(pr, plan, gp, err, errlen);
    }
    snprintf(err, errlen, "gemmkit: internal error: unsupported kernel combination");
    return 1;
}

}  // namespace gk
