// gk_tc_common.cuh -- device pieces shared by the one-CTA and the CTA-pair tensor-core GEMM
// kernels: tile constants, the exact requant arithmetic, saturating packs, the tile order,
// the work schedule, and the per-chunk epilogue.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "gk_engine.h"
#include "gk_sm100.cuh"

namespace gk {

constexpr int BM = 128;     // MMA M (TMEM lanes)
constexpr int BKB = 128;    // bytes of K per stage and row (one 128-byte swizzle atom)
constexpr int MMA_KB = 32;  // bytes of K per tcgen05.mma (kind::i8 K=32, kind::f16 K=16)
constexpr int SMEM_LIMIT = 232448;

// Per-scale constants of the exact requant (see requant_q).
struct alignas(16) ColParam {
    double se;           // min(scale, 2048), exact
    double nms;          // -(2^52 + 2^31) * se, exact (22-bit x 24-bit significands)
    uint32_t ulo, uhi;   // accumulator clamp [vlo, vhi], offset by 2^31 (unsigned domain)
    uint32_t bias_plus;  // bias + 2^31 (mod 2^32)
    uint32_t pad;
};

// The two parts of a scale's constants: se / nms (every requantize path), and the
// accumulator clamp (only the general path; it costs an f64 division).
__device__ __forceinline__ void make_scale_se(float s, double& se, double& nms) {
    const double s64 = static_cast<double>(s);
    se = s64 < 2048.0 ? s64 : 2048.0;
    nms = -(4503601774854144.0 * se);
}
__device__ __forceinline__ void make_scale_clamp(double se, uint32_t& ulo, uint32_t& uhi) {
    const double vs = ceil(2048.0 / se) + 1.0;
    const int vhi = vs >= 2147483647.0 ? 2147483647 : static_cast<int>(vs);
    const int vlo = vhi == 2147483647 ? (-2147483647 - 1) : -vhi - 1;
    ulo = static_cast<uint32_t>(vlo) + 0x80000000u;
    uhi = static_cast<uint32_t>(vhi) + 0x80000000u;
}
__device__ __forceinline__ void make_scale_param(float s, double& se, double& nms, uint32_t& ulo,
                                                 uint32_t& uhi) {
    make_scale_se(s, se, nms);
    make_scale_clamp(se, ulo, uhi);
}

// zp + rne(fl64(f64(v) * f64(scale))) for v = acc +wrap bias, exactly (the caller clamps to
// the output band). gemmkit's KRequantize::apply (gemmkit/src/kernel/epilogue.rs:810-830):
//  1. u = acc + bias + 2^31 (mod 2^32) is v + 2^31 as an unsigned number, so the unsigned clamp
//     to [vlo, vhi] + 2^31 is the signed clamp of v. The map is monotone in v (scale > 0), and
//     |v| beyond vhi ~ 2048/scale already drives |v*scale| >= 2048, past any clamp band, so the
//     clamp changes no result; it bounds |v*se| <= 2048 + 3*se <= 8192. For scale > 2048 the
//     band is v in [-3, 2] with se = 2048 and every v != 0 still saturates, as with scale.
//  2. d = 2^52 + u = 2^52 + 2^31 + v is exact (built from bits); fma(d, se, -(2^52+2^31)*se)
//     has the exact value v*se and rounds once: the reference's f64 product fl64(v*scale).
//  3. p + 1.5*2^52 rounds p to the nearest integer, ties to even (the reference's 2^52 trick,
//     gemmkit/src/kernel/epilogue.rs:886-897); |p| <= 8192 leaves the integer in the low word.
//     zp joins after rounding, in integer.
__device__ __forceinline__ int requant_q(uint32_t acc, uint32_t bias_plus, double se, double nms,
                                         uint32_t ulo, uint32_t uhi, int zp) {
    uint32_t u = acc + bias_plus;
    u = min(max(u, ulo), uhi);
    const double d = __hiloint2double(0x43300000, static_cast<int>(u));
    const double p = __fma_rn(d, se, nms);
    const double y = __dadd_rn(p, 6755399441055744.0);
    return __double2loint(y) + zp;
}

// requant_q without the clamp and with zp inside the rounding constant (magic = 1.5*2^52 + zp),
// exact when the scale is at most 2^-9 and zp is even: |v| <= 2^31 then bounds |p| by 2^22, so
// the rounded integer plus zp sits in the low word, and a tie of p + zp goes to the even
// neighbour of p shifted by the even zp, the same integer as rne(p) + zp.
// (Written as one PTX sequence: the 64-bit operand is assembled from the sum and the
// exponent word in place, which keeps the per-element instruction count at its minimum.)
__device__ __forceinline__ int requant_q_small(uint32_t acc, uint32_t bias_plus, double se,
                                               double nms, double magic) {
    int q;
    asm("{\n\t.reg .b32 u, h;\n\t.reg .f64 d, p;\n\t"
        "add.u32 u, %1, %2;\n\t"
        "mov.b32 h, 0x43300000;\n\t"
        "mov.b64 d, {u, h};\n\t"
        "fma.rn.f64 p, d, %3, %4;\n\t"
        "add.rn.f64 p, p, %5;\n\t"
        "mov.b64 {%0, h}, p;\n\t}"
        : "=r"(q)
        : "r"(acc), "r"(bias_plus), "d"(se), "d"(nms), "d"(magic));
    return q;
}

// The same requantize for two elements in packed f32x2 arithmetic, for items whose values
// v = acc + bias all satisfy |v| < 2^22 and whose scale s (f32) is below 1. Then fl64(v * s) is
// v * s exactly (22 + 24 significant bits), |v * s| < 2^22, and one f32 FMA gives it rounded
// half-even: fma(v, s, 1.5 * 2^23) lies in [2^23, 2^24), where the f32 spacing is 1, so the
// single rounding of the exact sum is 1.5 * 2^23 + rne(v * s) (1.5 * 2^23 is even: ties keep
// their parity). v enters as f32 through its bit pattern: bias_f carries bias + 0x4B400000, so
// acc + bias_f is the pattern of 1.5 * 2^23 + v and subtracting 1.5 * 2^23 leaves v exactly.
// The result's pattern minus qoff = 0x4B400000 - zp is rne(v * s) + zp for any zero point
// with |zp| <= 2^30. ss holds s in both halves. Per pair: two adds, one add.f32x2, one
// fma.f32x2, two subtracts.
__device__ __forceinline__ void requant_pair_f32(uint32_t acc0, uint32_t acc1, uint32_t bias0,
                                                 uint32_t bias1, uint64_t ss, uint32_t qoff,
                                                 int& q0, int& q1) {
    asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 e, y;\n\t"
        "add.u32 a, %2, %4;\n\t"
        "add.u32 b, %3, %5;\n\t"
        "mov.b64 e, {a, b};\n\t"
        "add.rn.f32x2 e, e, %6;\n\t"
        "fma.rn.f32x2 y, e, %7, %8;\n\t"
        "mov.b64 {a, b}, y;\n\t"
        "sub.u32 %0, a, %9;\n\t"
        "sub.u32 %1, b, %9;\n\t}"
        : "=r"(q0), "=r"(q1)
        : "r"(acc0), "r"(acc1), "r"(bias0), "r"(bias1), "l"(0xCB400000CB400000ull), "l"(ss),
          "l"(0x4B4000004B400000ull), "r"(qoff));
}

// Four values saturated to the output band and packed little-endian (x0 in the low byte).
template <bool U8>
__device__ __forceinline__ uint32_t pack4_sat(int x0, int x1, int x2, int x3) {
    uint32_t t, d;
    if constexpr (U8) {
        asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(x3), "r"(x2), "r"(0));
        asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x1), "r"(x0), "r"(t));
    } else {
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(x3), "r"(x2), "r"(0));
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x1), "r"(x0), "r"(t));
    }
    return d;
}

__device__ __forceinline__ uint32_t fast_div(const FastDiv& f, uint32_t n) {
    return (__umulhi(n, f.m) + n) >> f.s;
}

// Tile t -> (batch element b, tile row tm, tile column tn): batch-major, then bands of group_m
// tile rows, column by column inside a band (so a wave of CTAs shares A rows and B columns in
// L2). Divisions by the fixed divisors of the launch use their multiply-shift forms.
__device__ __forceinline__ void decode_tile(int t, const GemmParams& p, int& b, int& tm,
                                            int& tn) {
    const uint32_t ut = static_cast<uint32_t>(t);
    const uint32_t ub = fast_div(p.div_tpb, ut);
    const uint32_t r = ut - ub * p.div_tpb.d;
    const uint32_t band = fast_div(p.div_band, r);
    const uint32_t first_m = band * static_cast<uint32_t>(p.group_m);
    const uint32_t rr = r - band * p.div_band.d;
    const FastDiv& g =
        static_cast<uint32_t>(p.tiles_m) - first_m < static_cast<uint32_t>(p.group_m) ? p.div_glast
                                                                                    : p.div_gm;
    const uint32_t q = fast_div(g, rr);
    b = static_cast<int>(ub);
    tn = static_cast<int>(q);
    tm = static_cast<int>(first_m + (rr - q * g.d));
}

// One unit of a CTA's work: K blocks [k0, k1) of `tile`. nctr > 1 marks a stream-K tile cut
// between nctr CTAs; this CTA holds partial slot `slot` of it.
struct Work {
    int tile, k0, k1, slot, nctr;
};

// The CTA's sequence of work items, computed identically by every role: first the whole tiles
// blockIdx.x, blockIdx.x + grid, ... below dp_tiles, then this CTA's contiguous share
// [start(c), start(c + 1)) of the stream-K iterations (sk_iters >= grid, so every share is
// non-empty and a tile's contributors are consecutive CTAs).
struct Sched {
    int cta, G, dp_next;
    int64_t it, it_end;

    __device__ __forceinline__ explicit Sched(const GemmParams& p) {
        cta = blockIdx.x;
        G = gridDim.x;
        dp_next = cta;
        it = p.sk_iters > 0 ? start(p, cta) : 0;
        it_end = p.sk_iters > 0 ? start(p, cta + 1) : 0;
    }
    __device__ __forceinline__ int64_t start(const GemmParams& p, int c) const {
        return (static_cast<int64_t>(c) * p.sk_iters) / G;
    }
    // the CTA whose share holds iteration T: the largest c with start(c) <= T
    __device__ __forceinline__ int owner(const GemmParams& p, int64_t T) const {
        const int64_t c = ((T + 1) * G + p.sk_iters - 1) / p.sk_iters - 1;
        return static_cast<int>(c < 0 ? 0 : (c >= G ? G - 1 : c));
    }
    __device__ __forceinline__ bool next(const GemmParams& p, Work& w) {
        if (dp_next < p.dp_tiles) {
            w = Work{dp_next, 0, p.num_kb, 0, 1};
            dp_next += G;
            return true;
        }
        if (it < it_end) {
            const int skt = static_cast<int>(it / p.num_kb);
            const int k0 = static_cast<int>(it - static_cast<int64_t>(skt) * p.num_kb);
            const int64_t left = it_end - it;
            const int k1 = left < p.num_kb - k0 ? k0 + static_cast<int>(left) : p.num_kb;
            const int64_t T0 = static_cast<int64_t>(skt) * p.num_kb;
            const int cf = owner(p, T0), cl = owner(p, T0 + p.num_kb - 1);
            w = Work{p.dp_tiles + skt, k0, k1, cta - cf, cl - cf + 1};
            it += k1 - k0;
            return true;
        }
        return false;
    }
};

template <int SLEEP_NS = 0>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int* status, unsigned int where,
                                          uint64_t timeout) {
    const bool ok = mbar_wait<SLEEP_NS>(bar, parity, abort_flag, status, where, timeout);
    return !__any_sync(0xffffffffu, !ok);
}

// gemmkit's FusedEpi::apply (gemmkit/src/kernel/epilogue.rs:300-330): bias, then ReLU
// (v > 0 ? v : 0, so NaN -> 0) or LeakyReLU composed as max-part + slope * min-part (NaN -> 0,
// -0 -> +0), each step rounded in f32 like the reference's scalar expression.
__device__ __forceinline__ float fused_apply(const EpiParams& e, float v, float bias) {
    if (e.fbias_axis != AX_NONE) v = __fadd_rn(v, bias);
    if (e.act == FACT_RELU) return v > 0.0f ? v : 0.0f;
    if (e.act == FACT_LEAKY) {
        const float hi = v > 0.0f ? v : 0.0f;
        const float lo = v < 0.0f ? v : 0.0f;
        return __fadd_rn(hi, __fmul_rn(e.leak, lo));
    }
    return v;
}

// The integer counterpart of fused_apply for i32 outputs (an extension: gemmkit's FusedEpi is
// float-only, gemmkit/src/kernel/epilogue.rs:258-330): after alpha*acc + beta*C (wrapping, as
// int32_epilogue, gemmkit/src/kernel/int.rs:36-120) add the bias with wrap-around, then ReLU
// as max(v, 0) on the signed value. Only the i32 entry with a fused epilogue sets
// e.bias / e.act for an i32 output.
__device__ __forceinline__ uint32_t fused_apply_i32(const EpiParams& e, uint32_t v, uint32_t bias) {
    if (e.bias_axis != AX_NONE) v += bias;
    if (e.act == FACT_RELU) v = static_cast<uint32_t>(max(static_cast<int32_t>(v), 0));
    return v;
}

// Output stores: the local C and every mirror (same byte offset).
__device__ __forceinline__ void out_v4(const EpiParams& e, int64_t byte_off, uint32_t a,
                                       uint32_t b, uint32_t c, uint32_t d) {
    st_global_v4(static_cast<uint8_t*>(e.out) + byte_off, a, b, c, d);
    for (int i = 0; i < e.nmirror; ++i)
        st_global_v4(static_cast<uint8_t*>(e.mirror[i]) + byte_off, a, b, c, d);
}
template <typename T>
__device__ __forceinline__ void out_1(const EpiParams& e, int64_t elem_off, T v) {
    static_cast<T*>(e.out)[elem_off] = v;
    for (int i = 0; i < e.nmirror; ++i) static_cast<T*>(e.mirror[i])[elem_off] = v;
}

// Requantize paths an epilogue picks once per tile (uniform across the warp), so that the chunk
// loop is straight-line code: the general path takes every axis, zero point and scale; the two
// short ones take a per-row (or per-tensor) scale of at most 2^-9 with an even zero point
// (requant_q_small), with the bias per column (compact array) or per row / none (register).
// QM_F32 (the CTA-pair kernel's 16-warp form only) takes items whose |acc + bias| < 2^22 and
// whose scales are below 1 through requant_pair_f32.
enum QuantMode { QM_GENERAL = 0, QM_SMALL_COLB = 1, QM_SMALL_ROWB = 2, QM_F32 = 3 };

// The quant mode of this warp's rows for the current tile; every lane of the warp calls it.
__device__ __forceinline__ int pick_quant_mode(const EpiParams& e, double r_se) {
    const bool small = __all_sync(0xffffffffu, r_se <= 0x1p-9);
    if (e.scale_axis == AX_N || (e.zp & 1) != 0 || !small) return QM_GENERAL;
    return e.bias_axis == AX_N ? QM_SMALL_COLB : QM_SMALL_ROWB;
}

// Calls f(std::integral_constant<int, QM>) for the runtime mode qm (quantized outputs only;
// the other outputs take the general path), so that each mode's chunk loop is its own code.
template <bool QUANT, typename F>
__device__ __forceinline__ void with_quant_mode(int qm, F&& f) {
    if constexpr (QUANT) {
        if (qm == QM_SMALL_COLB)
            f(std::integral_constant<int, QM_SMALL_COLB>{});
        else if (qm == QM_SMALL_ROWB)
            f(std::integral_constant<int, QM_SMALL_ROWB>{});
        else
            f(std::integral_constant<int, QM_GENERAL>{});
    } else {
        f(std::integral_constant<int, QM_GENERAL>{});
    }
}

// The epilogue of one chunk of CH accumulator columns held by this thread (its row), starting
// at column gc of the output; columns at or past Nk are not written. For quantized outputs cp
// holds the chunk's per-column ColParams (per-column scale) and cb the chunk's per-column
// bias + 2^31 (per-column bias), both in shared memory; r_* are this row's values.
template <Out OUT, int CH, int QM = QM_GENERAL>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&v)[32], int64_t Nk,
                                               const EpiParams& e, int64_t obase, int64_t gc,
                                               const ColParam* cp, const uint32_t* cb,
                                               double r_se, double r_nms, uint32_t r_ulo,
                                               uint32_t r_uhi, uint32_t r_bp,
                                               float r_fbias = 0.0f) {
    const bool full_chunk = gc + CH <= Nk;
    if constexpr ((OUT == Out::Q8 || OUT == Out::U8) && QM != QM_GENERAL) {
        constexpr bool U8 = OUT == Out::U8;
        const double magic = 6755399441055744.0 + static_cast<double>(e.zp);
        int q[CH];
        if constexpr (QM == QM_SMALL_COLB) {
#pragma unroll
            for (int g = 0; g < CH / 4; ++g) {
                const uint4 bq = reinterpret_cast<const uint4*>(cb)[g];
                q[4 * g + 0] = requant_q_small(v[4 * g + 0], bq.x, r_se, r_nms, magic);
                q[4 * g + 1] = requant_q_small(v[4 * g + 1], bq.y, r_se, r_nms, magic);
                q[4 * g + 2] = requant_q_small(v[4 * g + 2], bq.z, r_se, r_nms, magic);
                q[4 * g + 3] = requant_q_small(v[4 * g + 3], bq.w, r_se, r_nms, magic);
            }
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) q[i] = requant_q_small(v[i], r_bp, r_se, r_nms, magic);
        }
        if (e.relu) {
#pragma unroll
            for (int i = 0; i < CH; ++i) q[i] = max(q[i], e.lo);
        }
        uint32_t w[CH / 4];
#pragma unroll
        for (int g = 0; g < CH / 4; ++g)
            w[g] = pack4_sat<U8>(q[4 * g], q[4 * g + 1], q[4 * g + 2], q[4 * g + 3]);
        if (e.vec && full_chunk) {
#pragma unroll
            for (int g = 0; g < CH / 16; ++g)
                out_v4(e, obase + gc + g * 16, w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i)
                if (gc + i < Nk)
                    out_1<uint8_t>(e, obase + (gc + i) * e.cso,
                                   static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3))));
        }
    } else if constexpr (OUT == Out::Q8 || OUT == Out::U8) {
        constexpr bool U8 = OUT == Out::U8;
        int q[CH];
        if (e.scale_axis == AX_N) {
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                const ColParam& pc = cp[i];
                const uint32_t bp = e.bias_axis == AX_N ? pc.bias_plus : r_bp;
                q[i] = requant_q(v[i], bp, pc.se, pc.nms, pc.ulo, pc.uhi, e.zp);
            }
        } else if (e.bias_axis == AX_N) {
#pragma unroll
            for (int i = 0; i < CH; ++i)
                q[i] = requant_q(v[i], cb[i], r_se, r_nms, r_ulo, r_uhi, e.zp);
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i)
                q[i] = requant_q(v[i], r_bp, r_se, r_nms, r_ulo, r_uhi, e.zp);
        }
        if (e.relu) {
#pragma unroll
            for (int i = 0; i < CH; ++i) q[i] = max(q[i], e.lo);
        }
        uint32_t w[CH / 4];
#pragma unroll
        for (int g = 0; g < CH / 4; ++g)
            w[g] = pack4_sat<U8>(q[4 * g], q[4 * g + 1], q[4 * g + 2], q[4 * g + 3]);
        if (e.vec && full_chunk) {
#pragma unroll
            for (int g = 0; g < CH / 16; ++g)
                out_v4(e, obase + gc + g * 16, w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i)
                if (gc + i < Nk)
                    out_1<uint8_t>(e, obase + (gc + i) * e.cso,
                                   static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3))));
        }
    } else if constexpr (OUT == Out::I32) {
        // r_bp carries this row's i32 bias (fused i32 epilogue with a per-row bias); a
        // per-column bias is read from e.bias (the fused i32 entry is not batched)
        int32_t* out = static_cast<int32_t*>(e.out);
        uint32_t r[CH];
        const uint32_t al = static_cast<uint32_t>(e.alpha_i);
        const uint32_t be = static_cast<uint32_t>(e.beta_i);
        const bool fused = e.bias_axis != AX_NONE || e.act != FACT_NONE;
        const bool colb = e.bias_axis == AX_N;
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
            if (fused) {
#pragma unroll
                for (int i = 0; i < CH; ++i)
                    r[i] = fused_apply_i32(e, r[i],
                                           colb ? static_cast<uint32_t>(__ldg(e.bias + gc + i))
                                                : r_bp);
            }
#pragma unroll
            for (int g = 0; g < CH / 4; ++g)
                out_v4(e, (obase + gc + g * 4) * 4, r[g * 4], r[g * 4 + 1], r[g * 4 + 2],
                       r[g * 4 + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                if (gc + i >= Nk) continue;
                const int64_t off = obase + (gc + i) * e.cso;
                uint32_t o = al * v[i];
                if (be != 0u) o += be * static_cast<uint32_t>(out[off]);
                if (fused)
                    o = fused_apply_i32(e, o,
                                        colb ? static_cast<uint32_t>(__ldg(e.bias + gc + i)) : r_bp);
                out_1<int32_t>(e, off, static_cast<int32_t>(o));
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
                if (e.act != FACT_NONE || e.fbias_axis != AX_NONE) {
                    const bool colb = e.fbias_axis == AX_N;
                    const float* fb = e.fbias + gc + g * 4;
                    x0 = fused_apply(e, x0, colb ? fb[0] : r_fbias);
                    x1 = fused_apply(e, x1, colb ? fb[1] : r_fbias);
                    x2 = fused_apply(e, x2, colb ? fb[2] : r_fbias);
                    x3 = fused_apply(e, x3, colb ? fb[3] : r_fbias);
                }
                out_v4(e, (obase + gc + g * 4) * 4, __float_as_uint(x0), __float_as_uint(x1),
                       __float_as_uint(x2), __float_as_uint(x3));
            }
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                if (gc + i >= Nk) continue;
                const int64_t off = obase + (gc + i) * e.cso;
                float x = al * __uint_as_float(v[i]);
                if (be != 0.0f) x = __fmaf_rn(be, out[off], x);
                if (e.act != FACT_NONE || e.fbias_axis != AX_NONE)
                    x = fused_apply(e, x, e.fbias_axis == AX_N ? e.fbias[gc + i] : r_fbias);
                out_1<float>(e, off, x);
            }
        }
    }
}

// A full 32-column chunk of 4-byte outputs (i32 or f32) with mirrored copies, the whole warp
// together (the caller checks e.vec, e.nmirror > 0 and that the chunk is inside Nk, all
// uniform across the warp; rows past Mk pass row_ok = false). The local C gets each lane's
// 128 bytes directly. For the mirrors (peer GPUs over NVLink) the warp's 32 x 32 block goes
// through a 4 KB shared-memory tile (16-byte pieces XOR-swizzled by row, conflict-free on both
// sides), so that every store instruction writes four whole 128-byte lines instead of 32
// separate 16-byte pieces.
template <Out OUT>
__device__ __forceinline__ void epilogue_chunk_mirrored_wide(const uint32_t (&v)[32],
                                                             const EpiParams& e, int64_t obase,
                                                             int64_t gc, bool row_ok,
                                                             uint32_t* stage, int lane) {
    static_assert(OUT == Out::I32 || OUT == Out::F32, "4-byte outputs only");
    uint32_t r[32];
    const int64_t off = obase + gc;  // element offset of this lane's 32 outputs
    if constexpr (OUT == Out::I32) {
        const uint32_t al = static_cast<uint32_t>(e.alpha_i);
        const uint32_t be = static_cast<uint32_t>(e.beta_i);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            uint4 cv = make_uint4(0u, 0u, 0u, 0u);
            if (be != 0u && row_ok) cv = ld_global_v4(static_cast<int32_t*>(e.out) + off + 4 * g);
            r[4 * g + 0] = be * cv.x + al * v[4 * g + 0];
            r[4 * g + 1] = be * cv.y + al * v[4 * g + 1];
            r[4 * g + 2] = be * cv.z + al * v[4 * g + 2];
            r[4 * g + 3] = be * cv.w + al * v[4 * g + 3];
        }
    } else {
        const float al = e.alpha_f, be = e.beta_f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            float x[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) x[t] = al * __uint_as_float(v[4 * g + t]);
            if (be != 0.0f && row_ok) {
                const uint4 cv = ld_global_v4(static_cast<float*>(e.out) + off + 4 * g);
                x[0] = __fmaf_rn(be, __uint_as_float(cv.x), x[0]);
                x[1] = __fmaf_rn(be, __uint_as_float(cv.y), x[1]);
                x[2] = __fmaf_rn(be, __uint_as_float(cv.z), x[2]);
                x[3] = __fmaf_rn(be, __uint_as_float(cv.w), x[3]);
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) r[4 * g + t] = __float_as_uint(x[t]);
        }
    }
    uint8_t* local = static_cast<uint8_t*>(e.out) + off * 4;
    const int sw = lane & 7;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        if (row_ok) st_global_v4(local + g * 16, r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
        *reinterpret_cast<uint4*>(stage + (lane * 8 + (g ^ sw)) * 4) =
            make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
    }
    __syncwarp();
    const int piece = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int src = 4 * i + (lane >> 3);  // the row whose piece this lane stores
        const long long soff = __shfl_sync(0xffffffffu, static_cast<long long>(off), src);
        const int sok = __shfl_sync(0xffffffffu, row_ok ? 1 : 0, src);
        const uint4 x = *reinterpret_cast<const uint4*>(stage + (src * 8 + (piece ^ (src & 7))) * 4);
        if (sok) {
            const int64_t boff = static_cast<int64_t>(soff) * 4 + piece * 16;
            for (int mi = 0; mi < e.nmirror; ++mi)
                st_global_v4(static_cast<uint8_t*>(e.mirror[mi]) + boff, x.x, x.y, x.z, x.w);
        }
    }
    __syncwarp();  // the tile is reused by the next chunk
}

// Host helpers shared by the launchers (gk_tc_gemm.cu).
int encode_operand(CUtensorMap* map, const Operand& op, int64_t K, int64_t batch, int es,
                   int box_rows, char* err, size_t errlen);
// Tensor map for TMA stores of a byte output: element (e, i, j) at out + e*obs + i*ldo + j,
// cols x rows x batch, box box_cols x box_rows x 1 with the swizzle of its box_cols-byte rows
// (32, 64 or 128).
int encode_output_u8(CUtensorMap* map, void* out, int64_t cols, int64_t rows, int64_t batch,
                     int64_t ldo, int64_t obs, int box_cols, int box_rows, char* err,
                     size_t errlen);
// Tensor map over an MN-major i8 operand (Operand::mn_ld): box box_cols (32/64/128) of its
// contiguous rows x 128 K-rows, swizzled by box_cols bytes.
int encode_mn_operand(CUtensorMap* map, const Operand& op, int64_t K, int box_cols, char* err,
                      size_t errlen);
// Tensor map over the tiled prepacked layout (Operand::slab): 128-byte rows already in
// swizzled order, so the map itself does not swizzle; box = box_rows rows of one K block.
int encode_tiled_operand(CUtensorMap* map, const Operand& op, int64_t K, int box_rows, char* err,
                         size_t errlen);

}  // namespace gk
