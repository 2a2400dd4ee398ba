// gk_api.cu -- the C ABI (include/gemmkit_cuda.h): gemmkit's validation with its wording,
// the degenerate-shape rules, the orientation choice, operand packing into the workspace,
// and the lowering of every entry to one canonical tensor-core problem (gk_engine.h).
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "gemmkit_cuda.h"
#include "gk_engine.h"

using gk::AX_M;
using gk::AX_N;
using gk::AX_NONE;

struct gk_workspace {
    int device;
    void* ptr;  // operand packs + stream-K partial accumulators
    size_t cap;
    uint32_t* ctr;  // stream-K arrival counters: zeroed when allocated, epoch-tagged after
    size_t ctr_cap;
    uint32_t epoch;
};

struct gk_packed_rhs {
    int device;
    uint8_t* buf;  // B^T in the tiled layout (gk_engine.h, Operand::slab), zero padded
    size_t k, n, k_pad, n_pad;  // k_pad: multiple of 128; n_pad: multiple of 256
};

namespace {

thread_local char g_err[1024] = "";
thread_local int g_tile_n = -1;

int set_err(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_err(cudaError_t e, const char* what) {
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ||
        e == cudaErrorNoKernelImageForDevice)
        return set_err(GK_ENODEV, "gemmkit: %s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorMemoryAllocation)
        return set_err(GK_ENOMEM, "gemmkit: %s: %s", what, cudaGetErrorString(e));
    return set_err(GK_ECUDA, "gemmkit: %s: %s", what, cudaGetErrorString(e));
}

// The engine runs only on sm_100 devices; anything else fails loudly (no fallback).
int check_device(int* dev_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_err(e, "no CUDA device");
    static int ok[64] = {0};
    if (dev < 0 || dev >= 64) return set_err(GK_ENODEV, "gemmkit: device index out of range");
    if (ok[dev] == 0) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        ok[dev] = (major == 10 && minor == 0) ? 1 : 2;
    }
    if (ok[dev] != 1)
        return set_err(GK_ENODEV, "gemmkit: the CUDA engine needs an sm_100 (B200) device");
    if (dev_out) *dev_out = dev;
    return GK_OK;
}

// ---- runtime knobs ---------------------------------------------------------------------
// gemmkit's tuning module (gemmkit/src/tuning.rs:585-690): every knob has a compiled default,
// an environment override read once, and a process-wide override set at run time
// (gk_knob_set, the counterpart of its set_* functions). The tuner sweeps them and writes a
// profile of `export GEMMKIT_CUDA_*=...` lines.
//   GEMMKIT_CUDA_BN       tile width (MMA N) of the tile kernels; 0 = chosen per shape
//   GEMMKIT_CUDA_PAIR     1 = CTA-pair (cta_group::2) kernel for 256-wide tiles
//   GEMMKIT_CUDA_GEMV     1 = streaming small-M kernel for Nk <= 64
//   GEMMKIT_CUDA_PDL      1 = programmatic dependent launch (overlap with the previous kernel)
//   GEMMKIT_CUDA_STREAMK  1 = stream-K tail for the last wave of the one-CTA kernel
//   GEMMKIT_CUDA_GEMV_SK  1 = the small-M kernel splits its weight stream evenly over all SMs
//                         (stream-K partials in the workspace) when whole tiles would not;
//                         off by default (measured slower than whole tiles on config 5)
//   GEMMKIT_CUDA_BN_SHORTK tile width for products whose K is at most 256 bytes (one or two
//                         128-byte blocks: epilogue-bound); 0 = the GEMMKIT_CUDA_BN rule
//   GEMMKIT_CUDA_EPI16    1 = the CTA-pair kernel takes its 16-warp epilogue form for short K
//   GEMMKIT_CUDA_STAGES   shared-memory ring depth cap of the kernels (0 = their whole ring,
//                         else 2 .. 12)
//   GEMMKIT_CUDA_GEMV_SPLIT largest cluster K split of the small-M kernel (0 = up to 8)
//   GEMMKIT_CUDA_MN_B     1 = an N-contiguous i8 B is read MN-major by the tile kernel (no
//                         transpose pack; tiles at most 128 wide); 0 = packed K-major first
//   GEMMKIT_CUDA_REQUANT_F32 1 = the 16-warp form requantizes an item in packed f32 when its
//                         |acc + bias| < 2^22 and its scales are below 1 (exact there)
enum KnobId {
    K_BN = 0, K_PAIR, K_GEMV, K_PDL, K_STREAMK, K_GEMVSK, K_BNSHORTK, K_EPI16, K_STAGES,
    K_GEMVSPLIT, K_MNB, K_F32Q, K_COUNT
};
const char* const kKnobEnv[K_COUNT] = {
    "GEMMKIT_CUDA_BN",       "GEMMKIT_CUDA_PAIR",      "GEMMKIT_CUDA_GEMV",
    "GEMMKIT_CUDA_PDL",      "GEMMKIT_CUDA_STREAMK",   "GEMMKIT_CUDA_GEMV_SK",
    "GEMMKIT_CUDA_BN_SHORTK", "GEMMKIT_CUDA_EPI16",    "GEMMKIT_CUDA_STAGES",
    "GEMMKIT_CUDA_GEMV_SPLIT", "GEMMKIT_CUDA_MN_B", "GEMMKIT_CUDA_REQUANT_F32"};
const int64_t kKnobDefault[K_COUNT] = {0, 1, 1, 1, 0, 0, 0, 1, 0, 0, 1, 1};
std::atomic<int64_t> g_knob_set[K_COUNT];  // value + 1; 0 = no run-time override

bool knob_valid(int id, int64_t v) {
    if (id == K_BN || id == K_BNSHORTK)
        return v == 0 || v == 16 || v == 32 || v == 64 || v == 128 || v == 192 || v == 256;
    if (id == K_STAGES) return v == 0 || (v >= 2 && v <= 12);
    if (id == K_GEMVSPLIT) return v >= 0 && v <= 8;
    return v == 0 || v == 1;
}

int64_t knob_env(int id) {
    static int64_t cache[K_COUNT];
    static std::once_flag once[K_COUNT];
    std::call_once(once[id], [id] {
        int64_t v = kKnobDefault[id];
        const char* s = getenv(kKnobEnv[id]);
        if (s && *s) {
            char* end = nullptr;
            const long long x = strtoll(s, &end, 10);
            if (end && *end == '\0' && knob_valid(id, x)) v = x;
        }
        cache[id] = v;
    });
    return cache[id];
}

int64_t knob(int id) {
    const int64_t s = g_knob_set[id].load(std::memory_order_relaxed);
    return s ? s - 1 : knob_env(id);
}

int knob_id(const char* name) {
    if (!name) return -1;
    for (int i = 0; i < K_COUNT; ++i)
        if (strcmp(name, kKnobEnv[i]) == 0) return i;
    return -1;
}

bool streamk_enabled() { return knob(K_STREAMK) == 1; }
bool pair_enabled() { return knob(K_PAIR) == 1; }
bool gemv_enabled() { return knob(K_GEMV) == 1; }
bool pdl_enabled() { return knob(K_PDL) == 1; }
bool gemv_sk_enabled() { return knob(K_GEMVSK) == 1; }
bool mn_major_enabled() { return knob(K_MNB) == 1; }

int tile_n_override(int64_t k_bytes = -1) {
    if (g_tile_n >= 0) return g_tile_n;
    if (k_bytes >= 0 && k_bytes <= 256) {
        const int64_t v = knob(K_BNSHORTK);
        if (v) return static_cast<int>(v);
    }
    return static_cast<int>(knob(K_BN));
}

// ---- gemmkit's checked-tier validation (gemmkit/src/api.rs:188-315) -----------------------

// extent (gemmkit/src/api.rs:188-210): highest offset (exclusive) reached, or false when a
// stride paired with a dimension > 1 is negative or the arithmetic overflows.
bool extent(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, size_t* need) {
    if (rows == 0 || cols == 0) {
        *need = 0;
        return true;
    }
    __int128 lo = 0, hi = 0;
    const size_t dims[2] = {rows, cols};
    const ptrdiff_t strides[2] = {rs, cs};
    for (int i = 0; i < 2; ++i) {
        if (dims[i] > static_cast<size_t>(PTRDIFF_MAX)) return false;
        __int128 e = static_cast<__int128>(dims[i] - 1) * strides[i];
        if (e > PTRDIFF_MAX || e < PTRDIFF_MIN) return false;
        if (e < 0)
            lo += e;
        else
            hi += e;
        if (hi > PTRDIFF_MAX || lo < PTRDIFF_MIN) return false;
    }
    if (lo < 0) return false;
    *need = static_cast<size_t>(hi) + 1;
    return true;
}

int check_view(size_t len, size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs, const char* name) {
    size_t need = 0;
    if (!extent(rows, cols, rs, cs, &need))
        return set_err(GK_EINVAL,
                       "gemmkit: %s view has negative strides or is too large to address; use "
                       "gemm_unchecked",
                       name);
    if (need > len)
        return set_err(GK_EINVAL,
                       "gemmkit: %s view of %zux%zu (strides %td,%td) needs %zu elements but slice "
                       "has %zu",
                       name, rows, cols, rs, cs, need, len);
    return GK_OK;
}

// self_aliases (gemmkit/src/api.rs:236-255)
bool self_aliases(size_t rows, size_t cols, ptrdiff_t rs, ptrdiff_t cs) {
    if (rows == 0 || cols == 0) return false;
    const bool hr = rows > 1, hc = cols > 1;
    const size_t ars = static_cast<size_t>(rs < 0 ? -rs : rs);
    const size_t acs = static_cast<size_t>(cs < 0 ? -cs : cs);
    if (!hr && !hc) return false;
    if (hr && !hc) return ars == 0;
    if (!hr && hc) return acs == 0;
    size_t sm_s, sm_d, big;
    if (ars <= acs) {
        sm_s = ars;
        sm_d = rows;
        big = acs;
    } else {
        sm_s = acs;
        sm_d = cols;
        big = ars;
    }
    unsigned __int128 span = static_cast<unsigned __int128>(sm_s) * sm_d;
    return sm_s == 0 || static_cast<unsigned __int128>(big) < span;
}

// overlaps_bytes (gemmkit/src/api.rs:519-532)
bool overlaps_bytes(const void* pa, size_t na, size_t sa, const void* pb, size_t nb, size_t sb) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(pa), a1 = a0 + na * sa;
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(pb), b1 = b0 + nb * sb;
    return a0 < b1 && b0 < a1;
}

// validate_gemm_views (gemmkit/src/api.rs:270-315)
int validate_gemm_views(const gk_matref& a, const gk_matref& b, const gk_matmut& c, size_t si,
                        size_t so) {
    if (a.cols != b.rows)
        return set_err(GK_EINVAL, "gemmkit: A.cols (%zu) != B.rows (%zu)", a.cols, b.rows);
    if (a.rows != c.rows)
        return set_err(GK_EINVAL, "gemmkit: A.rows (%zu) != C.rows (%zu)", a.rows, c.rows);
    if (b.cols != c.cols)
        return set_err(GK_EINVAL, "gemmkit: B.cols (%zu) != C.cols (%zu)", b.cols, c.cols);
    int rc;
    if ((rc = check_view(a.len, a.rows, a.cols, a.rs, a.cs, "A"))) return rc;
    if ((rc = check_view(b.len, b.rows, b.cols, b.rs, b.cs, "B"))) return rc;
    if ((rc = check_view(c.len, c.rows, c.cols, c.rs, c.cs, "C"))) return rc;
    if (self_aliases(c.rows, c.cols, c.rs, c.cs))
        return set_err(GK_EINVAL,
                       "gemmkit: C view aliases itself (strides %td,%td map distinct elements to "
                       "the same memory); C must address each (i,j) uniquely",
                       c.rs, c.cs);
    if (overlaps_bytes(c.data, c.len, so, a.data, a.len, si) ||
        overlaps_bytes(c.data, c.len, so, b.data, b.len, si))
        return set_err(GK_EINVAL, "gemmkit: C aliases A or B");
    return GK_OK;
}

// Rust's `{}` formatting of an f32, as the reference's messages print it: shortest
// round-trip digits, never an exponent, "NaN" / "inf" / "-inf".
std::string rust_f32(float x) {
    if (isnan(x)) return "NaN";
    if (isinf(x)) return x > 0 ? "inf" : "-inf";
    char buf[64];
    int prec = 1;
    for (; prec <= 9; ++prec) {
        snprintf(buf, sizeof(buf), "%.*e", prec - 1, static_cast<double>(x));
        if (strtof(buf, nullptr) == x) break;
    }
    // buf = d.ddddde[+-]XX; expand to positional notation
    std::string s(buf);
    const size_t epos = s.find('e');
    int exp10 = atoi(s.c_str() + epos + 1);
    std::string mant = s.substr(0, epos);
    bool neg = false;
    if (mant[0] == '-') {
        neg = true;
        mant = mant.substr(1);
    }
    std::string digits;
    for (char ch : mant)
        if (ch != '.') digits.push_back(ch);
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    std::string out;
    const int point = 1 + exp10;  // digits before the decimal point
    if (point <= 0) {
        out = "0." + std::string(-point, '0') + digits;
    } else if (point >= static_cast<int>(digits.size())) {
        out = digits + std::string(point - digits.size(), '0');
    } else {
        out = digits.substr(0, point) + "." + digits.substr(point);
    }
    if (out == "0") neg = neg && true;
    return (neg ? "-" : "") + out;
}

// ---- workspace -------------------------------------------------------------------------

gk_workspace* default_ws(int dev) {
    thread_local gk_workspace* tls[64] = {nullptr};
    if (!tls[dev & 63]) {
        tls[dev & 63] = new gk_workspace{dev, nullptr, 0, nullptr, 0, 0};
    }
    return tls[dev & 63];
}

int ws_ensure(gk_workspace* ws, size_t bytes, void** out) {
    if (bytes == 0) {
        *out = nullptr;
        return GK_OK;
    }
    if (ws->cap < bytes) {
        if (ws->ptr) {
            cudaDeviceSynchronize();  // the old buffer may still be read by queued kernels
            cudaFree(ws->ptr);
            ws->ptr = nullptr;
            ws->cap = 0;
        }
        size_t cap = (bytes + (1 << 20) - 1) & ~static_cast<size_t>((1 << 20) - 1);
        cudaError_t e = cudaMalloc(&ws->ptr, cap);
        if (e != cudaSuccess) {
            cudaGetLastError();
            ws->ptr = nullptr;
            return cuda_err(e, "workspace allocation");
        }
        ws->cap = cap;
    }
    *out = ws->ptr;
    return GK_OK;
}

// Stream-K counters: `words` zero-initialised 32-bit words, and the epoch of the next launch
// (1 .. 2^24 - 1; on wrap-around the counters are cleared again on `st`).
int ctr_ensure(gk_workspace* ws, size_t words, cudaStream_t st, uint32_t* epoch) {
    const size_t bytes = words * sizeof(uint32_t);
    if (ws->ctr_cap < bytes) {
        if (ws->ctr) {
            cudaDeviceSynchronize();
            cudaFree(ws->ctr);
            ws->ctr = nullptr;
            ws->ctr_cap = 0;
        }
        size_t cap = (bytes + 4095) & ~static_cast<size_t>(4095);
        cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&ws->ctr), cap);
        if (e == cudaSuccess) e = cudaMemset(ws->ctr, 0, cap);
        if (e != cudaSuccess) {
            cudaGetLastError();
            if (ws->ctr) cudaFree(ws->ctr);
            ws->ctr = nullptr;
            return cuda_err(e, "workspace counter allocation");
        }
        ws->ctr_cap = cap;
        ws->epoch = 0;
    }
    ws->epoch = ws->epoch >= 0xFFFFFFu ? 1u : ws->epoch + 1u;
    if (ws->epoch == 1u && ws->ctr_cap) {
        cudaError_t e = cudaMemsetAsync(ws->ctr, 0, ws->ctr_cap, st);
        if (e != cudaSuccess) return cuda_err(e, "workspace counter reset");
    }
    *epoch = ws->epoch;
    return GK_OK;
}

// ---- lowering --------------------------------------------------------------------------

struct Side {  // a user operand view with its batch stride (elements)
    const void* p;
    int64_t rs, cs, bs;
};

struct Job {
    gk::Kind kind;
    gk::Out out;
    int64_t m, k, n, batch;
    Side a, b;
    const gk_packed_rhs* packed;
    void* c;
    int64_t rsc, csc, cbs;
    int32_t alpha_i, beta_i;
    float alpha_f, beta_f;
    const int32_t* bias;
    int bias_axis;  // gk_axis (user frame)
    int64_t bias_bs;
    const float* scales;
    int scale_axis;  // gk_axis (user frame)
    float scale;
    int64_t scale_bs;
    int32_t zp, lo, hi;
    cudaStream_t stream;
    gk_workspace* ws;
    int nmirror;  // copies of C that receive every output element (see EpiParams::mirror)
    void* mirror[7];
    const float* fbias;  // fused float epilogue (f32 outputs)
    int fbias_axis;      // gk_axis (user frame)
    int act;             // gk_act
    float leak;
};

struct KOp {  // an operand in the canonical frame: rows x K, element (r, p) at r*rs + p*ks
    const void* p;
    int64_t rows, rs, ks, bs;
    int64_t slab;  // > 0: the tiled prepacked layout (already device-ready)
};

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

bool tma_ready(const KOp& o, int64_t K, int64_t batch, int es) {
    if (o.ks != 1 && K > 1) return false;
    if (reinterpret_cast<uintptr_t>(o.p) & 15) return false;
    if (o.rows > 1 && (o.rs <= 0 || (o.rs * es) % 16 != 0 || o.rs < 1)) return false;
    if (batch > 1 && o.bs != 0 && (o.bs < 0 || (o.bs * es) % 16 != 0)) return false;
    return true;
}

int map_axis(int user_axis, bool swap) {
    if (user_axis == GK_AXIS_ROW) return swap ? AX_N : AX_M;
    if (user_axis == GK_AXIS_COL) return swap ? AX_M : AX_N;
    return AX_NONE;
}

int execute(const Job& j) {
    if (j.m == 0 || j.n == 0 || j.batch == 0) return GK_OK;
    int dev = 0;
    int rc = check_device(&dev);
    if (rc) return rc;
    if (j.m > INT32_MAX || j.n > INT32_MAX || j.k > INT32_MAX / 2 || j.batch > INT32_MAX)
        return set_err(GK_EINVAL, "gemmkit: problem dimensions exceed the engine's limits");
    const int es = j.kind == gk::Kind::I8 ? 1 : 2;
    const int eso = j.out == gk::Out::Q8 ? 1 : 4;

    gk::EpiParams e;
    memset(&e, 0, sizeof(e));
    e.alpha_i = j.alpha_i;
    e.beta_i = j.beta_i;
    e.alpha_f = j.alpha_f;
    e.beta_f = j.beta_f;
    e.bias = j.bias;
    e.bias_bs = j.bias_bs;
    e.scales = j.scales;
    e.scale_bs = j.scale_bs;
    e.scale = j.scale;
    // The kernels add zp to the rounded product (|rne| < 2^22 on every path) in 32-bit
    // integers; the reference adds it in 64 bits with saturation. Clamping zp to +-2^30 keeps
    // the 32-bit sum exact, and any zp past that drives the output to the same band edge.
    e.zp = j.zp < -(1 << 30) ? -(1 << 30) : (j.zp > (1 << 30) ? (1 << 30) : j.zp);
    e.lo = j.lo;
    e.hi = j.hi;
    e.relu = j.out == gk::Out::Q8 && j.lo > (j.hi == 255 ? 0 : -128);

    // Degenerate products: gemmkit's scale_c_int (k == 0 or alpha == 0) and
    // requant_degenerate (k == 0).
    const bool alpha_zero = (j.out == gk::Out::I32 && j.alpha_i == 0) ||
                            (j.out == gk::Out::F32 && j.alpha_f == 0.0f);
    if ((j.k == 0 || alpha_zero) && j.nmirror > 0)
        return set_err(GK_EINVAL, "gemmkit: mirrored outputs need k > 0 and a nonzero alpha");
    if (j.k == 0 || alpha_zero) {
        if (j.out == gk::Out::I32 && (j.act != GK_ACT_NONE || j.bias)) {
            gk::EpiParams fe = e;
            fe.bias_axis = map_axis(j.bias ? j.bias_axis : GK_AXIS_NONE, false);
            fe.act = j.act;
            rc = gk::launch_fused_fill_i32(static_cast<int32_t*>(j.c), j.m, j.n, j.rsc, j.csc,
                                           j.beta_i, fe, j.stream);
            return rc ? set_err(GK_ECUDA, "gemmkit: fill kernel launch failed") : GK_OK;
        }
        if (j.out == gk::Out::I32) {
            for (int64_t b = 0; b < j.batch; ++b) {
                rc = gk::launch_scale_c_i32(static_cast<int32_t*>(j.c) + b * j.cbs, j.m, j.n,
                                            j.rsc, j.csc, j.beta_i, j.stream);
                if (rc) return set_err(GK_ECUDA, "gemmkit: fill kernel launch failed");
            }
            return GK_OK;
        }
        if (j.out == gk::Out::F32) {
            if (j.act != GK_ACT_NONE || j.fbias) {
                gk::EpiParams fe = e;
                fe.fbias = j.fbias;
                fe.fbias_axis = map_axis(j.fbias ? j.fbias_axis : GK_AXIS_NONE, false);
                fe.act = j.act;
                fe.leak = j.leak;
                rc = gk::launch_fused_fill_f32(static_cast<float*>(j.c), j.m, j.n, j.rsc, j.csc,
                                               j.beta_f, fe, j.stream);
            } else {
                rc = gk::launch_scale_c_f32(static_cast<float*>(j.c), j.m, j.n, j.rsc, j.csc,
                                            j.cbs, j.batch, j.beta_f, j.stream);
            }
            return rc ? set_err(GK_ECUDA, "gemmkit: fill kernel launch failed") : GK_OK;
        }
        e.bias_axis = map_axis(j.bias ? j.bias_axis : GK_AXIS_NONE, false);
        e.scale_axis = map_axis(j.scales ? j.scale_axis : GK_AXIS_NONE, false);
        rc = gk::launch_requant_fill(j.c, j.m, j.n, j.rsc, j.csc, j.cbs, j.batch, e, j.stream);
        return rc ? set_err(GK_ECUDA, "gemmkit: fill kernel launch failed") : GK_OK;
    }

    // Orientation: the output's unit-stride axis becomes the kernel's column axis, except
    // that a small side (<= 64) always goes to the MMA N so the 128 TMEM lanes stay busy.
    bool swap;
    if (j.m <= 64 && j.n > j.m)
        swap = true;
    else if (j.n <= 64 && j.m > j.n)
        swap = false;
    else if (j.csc == 1)
        swap = false;
    else if (j.rsc == 1)
        swap = true;
    else
        swap = llabs(j.csc) > llabs(j.rsc);

    KOp ua{j.a.p, j.m, j.a.rs, j.a.cs, j.a.bs, 0};
    KOp ub;
    if (j.packed)
        ub = KOp{j.packed->buf, static_cast<int64_t>(j.packed->n_pad), 128, 1, 0,
                 static_cast<int64_t>(j.packed->n_pad) * 128};
    else
        ub = KOp{j.b.p, j.n, j.b.cs, j.b.rs, j.b.bs, 0};
    KOp ka = swap ? ub : ua, kb = swap ? ua : ub;
    const int64_t Mk = swap ? j.n : j.m, Nk = swap ? j.m : j.n;

    // Operands that are not K-contiguous / 16-byte aligned are packed into the workspace.
    const int64_t ldp = round_up(j.k, 16 / es);
    int64_t need[2] = {0, 0};
    KOp* ops[2] = {&ka, &kb};
    for (int i = 0; i < 2; ++i) {
        KOp& o = *ops[i];
        if (o.slab) continue;
        if (o.rows == 1 && o.ks == 1 && !(reinterpret_cast<uintptr_t>(o.p) & 15)) o.rs = ldp;
        if (!tma_ready(o, j.k, j.batch, es)) {
            const int64_t nb = (j.batch > 1 && o.bs != 0) ? j.batch : 1;
            need[i] = round_up(o.rows * ldp * es * nb, 256);
        }
    }

    e.out = j.c;
    e.fbias = j.fbias;
    e.fbias_axis = map_axis(j.fbias ? j.fbias_axis : GK_AXIS_NONE, swap);
    e.act = j.act;
    e.leak = j.leak;
    e.nmirror = j.nmirror;
    for (int i = 0; i < j.nmirror; ++i) e.mirror[i] = j.mirror[i];
    e.ldo = swap ? j.csc : j.rsc;
    e.cso = swap ? j.rsc : j.csc;
    e.obs = j.cbs;
    e.bias_axis = map_axis(j.bias ? j.bias_axis : GK_AXIS_NONE, swap);
    e.scale_axis = map_axis(j.scales ? j.scale_axis : GK_AXIS_NONE, swap);
    e.vec = (e.cso == 1) && !(reinterpret_cast<uintptr_t>(j.c) & 15) &&
            ((e.ldo * eso) % 16 == 0 || Mk == 1) && (j.batch <= 1 || (j.cbs * eso) % 16 == 0);

    gk::TcProblem pr;
    memset(&pr, 0, sizeof(pr));
    pr.kind = j.kind;
    pr.out = (j.out == gk::Out::Q8 && j.hi == 255) ? gk::Out::U8 : j.out;
    pr.Mk = Mk;
    pr.Nk = Nk;
    pr.K = j.k;
    pr.batch = j.batch;
    pr.e = e;
    pr.bn = tile_n_override(j.k * es);
    pr.stream = j.stream;
    pr.pdl = pdl_enabled() ? 1 : 0;
    pr.stages = static_cast<int>(knob(K_STAGES));
    pr.epi16 = static_cast<int>(knob(K_EPI16));
    pr.gemv_split = static_cast<int>(knob(K_GEMVSPLIT));
    pr.f32q = static_cast<int>(knob(K_F32Q));
    // An N-contiguous i8 right-hand side (row-major B of C = A*B) is read MN-major by the
    // tile kernel's TMA, with no transpose pack: rows contiguous, K at a 16-byte pitch.
    if (need[1] && j.kind == gk::Kind::I8 && j.batch == 1 && kb.rs == 1 && kb.ks >= kb.rows &&
        kb.ks % 16 == 0 && !(reinterpret_cast<uintptr_t>(kb.p) & 15) && Nk > 64 &&
        (pr.bn == 0 || pr.bn >= 32) && pr.bn != 16 && mn_major_enabled()) {
        need[1] = 0;
        pr.b.mn_ld = kb.ks;
        if (pr.bn == 192 || pr.bn == 256) pr.bn = 128;
    }
    // the planners look at which operand is in the tiled prepacked layout; the operands
    // themselves are filled in below, once any packing has its scratch
    pr.a.slab = ka.slab;
    pr.b.slab = kb.slab;
    gk::TcPlan plan;
    gk::plan_tc_gemm2(pr, streamk_enabled(), pair_enabled(), gemv_enabled(), &plan,
                      gemv_sk_enabled());
    const int64_t part_bytes = round_up(plan.part_words * 4, 256);

    gk_workspace* ws = j.ws ? j.ws : default_ws(dev);
    char* base = nullptr;
    if (need[0] + need[1] + part_bytes) {
        void* vb = nullptr;
        rc = ws_ensure(ws, static_cast<size_t>(need[0] + need[1] + part_bytes), &vb);
        if (rc) return rc;
        base = static_cast<char*>(vb);
    }
    if (plan.sk_iters > 0) {
        rc = ctr_ensure(ws, static_cast<size_t>(plan.ctr_words), j.stream, &pr.sk_epoch);
        if (rc) return rc;
        pr.sk_ctr = ws->ctr;
        pr.sk_part = reinterpret_cast<uint32_t*>(base + need[0] + need[1]);
    }
    char* cur = base;
    for (int i = 0; i < 2; ++i) {
        if (!need[i]) continue;
        KOp& o = *ops[i];
        const int64_t nb = (j.batch > 1 && o.bs != 0) ? j.batch : 1;
        const int64_t dbs = o.rows * ldp;
        if (gk::launch_pack_kmajor(cur, ldp, dbs, o.p, o.rs, o.ks, o.bs, o.rows, j.k, nb, es,
                                   j.stream))
            return set_err(GK_ECUDA, "gemmkit: pack kernel launch failed");
        o = KOp{cur, o.rows, ldp, 1, nb > 1 ? dbs : 0, 0};
        cur += need[i];
    }
    pr.a = gk::Operand{ka.p, ka.rows, ka.rs, ka.bs, ka.slab};
    const int64_t mn_ld = pr.b.mn_ld;
    pr.b = gk::Operand{kb.p, kb.rows, kb.rs, kb.bs, kb.slab, mn_ld};
    char err[512] = "";
    rc = gk::launch_tc_gemm_planned(pr, plan, err, sizeof(err));
    if (rc) return set_err(rc, "%s", err);
    return GK_OK;
}

gk_parallelism par_ignored(gk_parallelism p) { return p; }

// Requant descriptor -> job fields, with the output band of the entry.
void fill_requant(Job& j, const gk_requant* q, bool out_u8) {
    j.out = gk::Out::Q8;
    j.bias = q->bias;
    j.bias_axis = q->bias ? q->bias_axis : GK_AXIS_NONE;
    j.scales = q->scale_axis != GK_AXIS_NONE ? q->scales : nullptr;
    j.scale_axis = q->scale_axis;
    j.scale = q->scale;
    j.zp = q->zero_point;
    j.lo = out_u8 ? 0 : -128;
    j.hi = out_u8 ? 255 : 127;
    if (q->relu) {
        int f = q->zero_point < j.lo ? j.lo : (q->zero_point > j.hi ? j.hi : q->zero_point);
        if (f > j.lo) j.lo = f;
    }
}

Job base_job(gk_workspace* ws, gk_stream_t stream) {
    Job j;
    memset(&j, 0, sizeof(j));
    j.batch = 1;
    j.ws = ws;
    j.stream = static_cast<cudaStream_t>(stream);
    j.alpha_i = 1;
    j.alpha_f = 1.0f;
    return j;
}

int check_scale_value(float s) {
    if (!(isfinite(s) && s > 0.0f))
        return set_err(GK_EINVAL, "gemmkit: requantize scale (%s) must be finite and > 0",
                       rust_f32(s).c_str());
    return GK_OK;
}

}  // namespace

namespace gk {
// Records `text` as this thread's gk_last_error() message (for entries in other files).
int set_last_error(int code, const char* text) { return set_err(code, "%s", text); }
}  // namespace gk

// ==========================================================================================
// C ABI
// ==========================================================================================

extern "C" {

const char* gk_version(void) { return "gemmkit-cuda 0.1.0 (sm_100a)"; }

const char* gk_last_error(void) { return g_err; }

int gk_device_status(int device, int clear, uint32_t* status) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return set_err(GK_ENODEV, "gemmkit: bad device");
    cudaError_t e = cudaDeviceSynchronize();
    unsigned int* p = gk::device_status_ptr();
    unsigned int v = 0;
    if (e == cudaSuccess && p) e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear && p) e = cudaMemset(p, 0, sizeof(v));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_err(e, "device status");
    if (status) *status = v;
    return GK_OK;
}

int gk_workspace_create(gk_workspace** out) {
    if (!out) return set_err(GK_EINVAL, "gemmkit: null output pointer");
    int dev = 0;
    cudaGetDevice(&dev);
    *out = new gk_workspace{dev, nullptr, 0, nullptr, 0, 0};
    return GK_OK;
}

void gk_workspace_free(gk_workspace* ws) {
    if (!ws) return;
    if (ws->ptr || ws->ctr) cudaDeviceSynchronize();
    if (ws->ptr) cudaFree(ws->ptr);
    if (ws->ctr) cudaFree(ws->ctr);
    delete ws;
}

const char* gk_knob_names(void) {
    return "GEMMKIT_CUDA_BN,GEMMKIT_CUDA_PAIR,GEMMKIT_CUDA_GEMV,GEMMKIT_CUDA_PDL,"
           "GEMMKIT_CUDA_STREAMK,GEMMKIT_CUDA_GEMV_SK,GEMMKIT_CUDA_BN_SHORTK,GEMMKIT_CUDA_EPI16,"
           "GEMMKIT_CUDA_STAGES,GEMMKIT_CUDA_GEMV_SPLIT,GEMMKIT_CUDA_MN_B,"
           "GEMMKIT_CUDA_REQUANT_F32";
}

int gk_knob_get(const char* name, int64_t* value) {
    const int id = knob_id(name);
    if (id < 0) return set_err(GK_EINVAL, "gemmkit: unknown knob %s", name ? name : "(null)");
    if (!value) return set_err(GK_EINVAL, "gemmkit: null output pointer");
    *value = knob(id);
    return GK_OK;
}

int gk_knob_set(const char* name, int64_t value) {
    const int id = knob_id(name);
    if (id < 0) return set_err(GK_EINVAL, "gemmkit: unknown knob %s", name ? name : "(null)");
    if (value < 0) {
        g_knob_set[id].store(0, std::memory_order_relaxed);
        return GK_OK;
    }
    if (!knob_valid(id, value))
        return set_err(GK_EINVAL, "gemmkit: %s cannot be %lld", kKnobEnv[id],
                       static_cast<long long>(value));
    g_knob_set[id].store(value + 1, std::memory_order_relaxed);
    return GK_OK;
}

int gk_set_tile_n(int bn) {
    if (!(bn == 0 || bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 192 || bn == 256))
        return set_err(GK_EINVAL, "gemmkit: tile width must be 0, 16, 32, 64, 128, 192 or 256");
    g_tile_n = bn == 0 ? -1 : bn;  // 0: no thread override, the GEMMKIT_CUDA_BN knob decides
    return GK_OK;
}

// ---- i8 -> i32 ----------------------------------------------------------------------------

int gk_gemm_i8_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n, int32_t alpha,
                         const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b,
                         ptrdiff_t rsb, ptrdiff_t csb, int32_t beta, int32_t* c, ptrdiff_t rsc,
                         ptrdiff_t csc, gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    if (m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && n && k && alpha && (!a || !b)) return set_err(GK_EINVAL, "gemmkit: null A or B");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.out = gk::Out::I32;
    j.m = m;
    j.k = k;
    j.n = n;
    j.a = Side{a, rsa, csa, 0};
    j.b = Side{b, rsb, csb, 0};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.alpha_i = alpha;
    j.beta_i = beta;
    return execute(j);
}

int gk_gemm_i8(gk_workspace* ws, int32_t alpha, gk_matref a, gk_matref b, int32_t beta,
               gk_matmut c, gk_parallelism par, gk_stream_t stream) {
    gk_matmut cc = c;
    int rc = validate_gemm_views(a, b, cc, 1, 4);
    if (rc) return rc;
    return gk_gemm_i8_unchecked(ws, a.rows, a.cols, b.cols, alpha,
                                static_cast<const int8_t*>(a.data), a.rs, a.cs,
                                static_cast<const int8_t*>(b.data), b.rs, b.cs, beta,
                                static_cast<int32_t*>(c.data), c.rs, c.cs, par, stream);
}

// ---- fused i32 epilogue (extension: gemmkit's gemm_fused is float-only) ---------------------

static int i8_fused(gk_workspace* ws, size_t m, size_t k, size_t n, int32_t alpha,
                    const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b, ptrdiff_t rsb,
                    ptrdiff_t csb, int32_t beta, int32_t* c, ptrdiff_t rsc, ptrdiff_t csc,
                    const int32_t* bias, int bias_dim, int has_bias, int act,
                    gk_stream_t stream) {
    if (m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && n && k && alpha && (!a || !b)) return set_err(GK_EINVAL, "gemmkit: null A or B");
    if (act == GK_ACT_LEAKY_RELU)
        return set_err(GK_EINVAL,
                       "gemmkit: the i32 fused epilogue has no LeakyReLU (its slope is a float)");
    if (act != GK_ACT_NONE && act != GK_ACT_RELU)
        return set_err(GK_EINVAL, "gemmkit: unknown activation %d", act);
    if (has_bias && bias_dim != GK_AXIS_ROW && bias_dim != GK_AXIS_COL)
        return set_err(GK_EINVAL, "gemmkit: bias dimension must be row or column");
    if (has_bias && m && n && !bias) return set_err(GK_EINVAL, "gemmkit: null bias");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.out = gk::Out::I32;
    j.m = m;
    j.k = k;
    j.n = n;
    j.a = Side{a, rsa, csa, 0};
    j.b = Side{b, rsb, csb, 0};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.alpha_i = alpha;
    j.beta_i = beta;
    j.bias = has_bias ? bias : nullptr;
    j.bias_axis = has_bias ? bias_dim : GK_AXIS_NONE;
    j.act = act;
    return execute(j);
}

int gk_gemm_i8_fused_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n, int32_t alpha,
                               const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b,
                               ptrdiff_t rsb, ptrdiff_t csb, int32_t beta, int32_t* c,
                               ptrdiff_t rsc, ptrdiff_t csc, const int32_t* bias, int bias_dim,
                               int has_bias, int act, gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    return i8_fused(ws, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, bias,
                    bias_dim, has_bias, act, stream);
}

int gk_gemm_i8_fused(gk_workspace* ws, int32_t alpha, gk_matref a, gk_matref b, int32_t beta,
                     gk_matmut c, const int32_t* bias, size_t bias_len, int bias_dim, int act,
                     gk_parallelism par, gk_stream_t stream) {
    int rc = validate_gemm_views(a, b, c, 1, 4);
    if (rc) return rc;
    if (bias) {
        // the bias check of gemmkit's gemm_fused (gemmkit/src/api.rs:318-330)
        const size_t want = bias_dim == GK_AXIS_COL ? b.cols : a.rows;
        if (bias_dim != GK_AXIS_ROW && bias_dim != GK_AXIS_COL)
            return set_err(GK_EINVAL, "gemmkit: bias dimension must be row or column");
        if (bias_len != want)
            return set_err(GK_EINVAL, "gemmkit: %s bias length %zu does not match %s = %zu",
                           bias_dim == GK_AXIS_COL ? "per-column" : "per-row", bias_len,
                           bias_dim == GK_AXIS_COL ? "n" : "m", want);
    }
    (void)par_ignored(par);
    return i8_fused(ws, a.rows, a.cols, b.cols, alpha, static_cast<const int8_t*>(a.data), a.rs,
                    a.cs, static_cast<const int8_t*>(b.data), b.rs, b.cs, beta,
                    static_cast<int32_t*>(c.data), c.rs, c.cs, bias, bias_dim, bias != nullptr,
                    act, stream);
}

// ---- requant ------------------------------------------------------------------------------

int gk_gemm_i8_requant_ex_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n,
                                    const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                                    const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb,
                                    const gk_requant* req, void* c, ptrdiff_t rsc, ptrdiff_t csc,
                                    int out_u8, gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    if (!req) return set_err(GK_EINVAL, "gemmkit: null requant descriptor");
    if (m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && n && k && (!a || !b)) return set_err(GK_EINVAL, "gemmkit: null A or B");
    if (req->scale_axis != GK_AXIS_NONE && !req->scales)
        return set_err(GK_EINVAL, "gemmkit: null requantize scales");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.m = m;
    j.k = k;
    j.n = n;
    j.a = Side{a, rsa, csa, 0};
    j.b = Side{b, rsb, csb, 0};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    fill_requant(j, req, out_u8 != 0);
    return execute(j);
}

static int requant_plain(gk_workspace* ws, size_t m, size_t k, size_t n, const int8_t* a,
                         ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b, ptrdiff_t rsb,
                         ptrdiff_t csb, float scale, const float* row_scales, int has_row_scales,
                         int32_t zp, const int32_t* bias, int has_bias, void* c, ptrdiff_t rsc,
                         ptrdiff_t csc, int out_u8, gk_parallelism par, gk_stream_t stream) {
    gk_requant q;
    memset(&q, 0, sizeof(q));
    q.scale = scale;
    q.scales = has_row_scales ? row_scales : nullptr;
    q.scale_axis = has_row_scales ? GK_AXIS_ROW : GK_AXIS_NONE;
    q.zero_point = zp;
    q.bias = has_bias ? bias : nullptr;
    q.bias_axis = has_bias ? GK_AXIS_ROW : GK_AXIS_NONE;
    return gk_gemm_i8_requant_ex_unchecked(ws, m, k, n, a, rsa, csa, b, rsb, csb, &q, c, rsc, csc,
                                           out_u8, par, stream);
}

int gk_gemm_i8_requant_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n, const int8_t* a,
                                 ptrdiff_t rsa, ptrdiff_t csa, const int8_t* b, ptrdiff_t rsb,
                                 ptrdiff_t csb, float scale, const float* row_scales,
                                 int has_row_scales, int32_t zero_point, const int32_t* bias,
                                 int has_bias, int8_t* c, ptrdiff_t rsc, ptrdiff_t csc,
                                 gk_parallelism par, gk_stream_t stream) {
    return requant_plain(ws, m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales, has_row_scales,
                         zero_point, bias, has_bias, c, rsc, csc, 0, par, stream);
}

int gk_gemm_i8_requant_u8_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n,
                                    const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                                    const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb, float scale,
                                    const float* row_scales, int has_row_scales,
                                    int32_t zero_point, const int32_t* bias, int has_bias,
                                    uint8_t* c, ptrdiff_t rsc, ptrdiff_t csc, gk_parallelism par,
                                    gk_stream_t stream) {
    return requant_plain(ws, m, k, n, a, rsa, csa, b, rsb, csb, scale, row_scales, has_row_scales,
                         zero_point, bias, has_bias, c, rsc, csc, 1, par, stream);
}

// requant_scale / requant_bias (gemmkit/src/adapter.rs:190-280) over C's backing slice as a
// unit-stride footprint, in gemmkit's order: views, scale, zero-point, bias.
static int validate_requant(const gk_requant* q, size_t m, size_t n, const gk_matmut& c,
                            int out_u8, cudaStream_t st) {
    const size_t c_bytes = c.len;  // 1-byte output
    auto axis_len = [&](int axis) { return axis == GK_AXIS_COL ? n : m; };
    const char* axis_dim = nullptr;
    if (q->scale_axis == GK_AXIS_NONE) {
        int rc = check_scale_value(q->scale);
        if (rc) return rc;
    } else {
        const size_t want = axis_len(q->scale_axis);
        axis_dim = q->scale_axis == GK_AXIS_COL ? "B.cols" : "A.rows";
        if (q->scales_len != want)
            return set_err(GK_EINVAL, "gemmkit: requantize scales length (%zu) != %s (%zu)",
                           q->scales_len, axis_dim, want);
        if (c_bytes && q->scales_len &&
            overlaps_bytes(c.data, c_bytes, 1, q->scales, q->scales_len, 4))
            return set_err(GK_EINVAL, "gemmkit: requantize scales overlap C");
        if (q->scales_len) {
            float* host = static_cast<float*>(malloc(q->scales_len * sizeof(float)));
            if (!host) return set_err(GK_ENOMEM, "gemmkit: host allocation failed");
            cudaError_t e = cudaMemcpyAsync(host, q->scales, q->scales_len * sizeof(float),
                                            cudaMemcpyDeviceToHost, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) {
                free(host);
                return cuda_err(e, "reading requantize scales");
            }
            for (size_t i = 0; i < q->scales_len; ++i) {
                int rc = check_scale_value(host[i]);
                if (rc) {
                    free(host);
                    return rc;
                }
            }
            free(host);
        }
    }
    if (out_u8) {
        if (q->zero_point < 0 || q->zero_point > 255)
            return set_err(GK_EINVAL,
                           "gemmkit: requantize zero_point (%d) out of u8 range [0, 255]",
                           q->zero_point);
    } else if (q->zero_point < -128 || q->zero_point > 127) {
        return set_err(GK_EINVAL, "gemmkit: requantize zero_point (%d) out of i8 range [-128, 127]",
                       q->zero_point);
    }
    if (q->bias) {
        const size_t want = axis_len(q->bias_axis);
        const char* dim = q->bias_axis == GK_AXIS_COL ? "B.cols" : "A.rows";
        if (q->bias_len != want)
            return set_err(GK_EINVAL, "gemmkit: requantize bias length (%zu) != %s (%zu)",
                           q->bias_len, dim, want);
        if (c_bytes && q->bias_len && overlaps_bytes(c.data, c_bytes, 1, q->bias, q->bias_len, 4))
            return set_err(GK_EINVAL, "gemmkit: requantize bias overlaps C");
    }
    return GK_OK;
}

int gk_gemm_i8_requant(gk_workspace* ws, gk_matref a, gk_matref b, const gk_requant* req,
                       gk_matmut c, int out_u8, gk_parallelism par, gk_stream_t stream) {
    if (!req) return set_err(GK_EINVAL, "gemmkit: null requant descriptor");
    int rc = validate_gemm_views(a, b, c, 1, 1);
    if (rc) return rc;
    rc = validate_requant(req, a.rows, b.cols, c, out_u8, static_cast<cudaStream_t>(stream));
    if (rc) return rc;
    return gk_gemm_i8_requant_ex_unchecked(
        ws, a.rows, a.cols, b.cols, static_cast<const int8_t*>(a.data), a.rs, a.cs,
        static_cast<const int8_t*>(b.data), b.rs, b.cs, req, c.data, c.rs, c.cs, out_u8, par,
        stream);
}

// ---- prepacked B --------------------------------------------------------------------------

int gk_prepack_rhs_i8_unchecked(const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb, size_t k, size_t n,
                                gk_stream_t stream, gk_packed_rhs** out) {
    if (!out) return set_err(GK_EINVAL, "gemmkit: null output pointer");
    *out = nullptr;
    int dev = 0;
    int rc = check_device(&dev);
    if (rc) return rc;
    if (k > static_cast<size_t>(INT32_MAX / 2) || n > static_cast<size_t>(INT32_MAX))
        return set_err(GK_EINVAL,
                       "gemmkit: prepacked RHS of %zux%zu is too large; the pack buffer size "
                       "overflows usize",
                       k, n);
    gk_packed_rhs* p = new gk_packed_rhs{dev, nullptr, k, n, 0, 0};
    p->k_pad = static_cast<size_t>(round_up(static_cast<int64_t>(k), 128));
    p->n_pad = static_cast<size_t>(round_up(static_cast<int64_t>(n), 256));
    const size_t bytes = (k && n) ? p->k_pad * p->n_pad : 0;
    if (bytes) {
        if (!b) {
            delete p;
            return set_err(GK_EINVAL, "gemmkit: null B");
        }
        cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&p->buf), bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            delete p;
            return cuda_err(e, "prepack allocation");
        }
        // B^T rows (one per column j of B): element (j, p) = b[p*rsb + j*csb]
        if (gk::launch_pack_tiled(p->buf, p->n_pad, p->k_pad, b, csb, rsb, n, k,
                                  static_cast<cudaStream_t>(stream))) {
            cudaFree(p->buf);
            delete p;
            return set_err(GK_ECUDA, "gemmkit: pack kernel launch failed");
        }
        // The handle is immutable from here on, like gemmkit's packed buffer: the pack is
        // complete before it is returned, so kernels may read it ahead of their stream order.
        e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) {
            cudaGetLastError();
            cudaFree(p->buf);
            delete p;
            return cuda_err(e, "prepack");
        }
    }
    *out = p;
    return GK_OK;
}

int gk_prepack_rhs_i8(gk_matref b, gk_stream_t stream, gk_packed_rhs** out) {
    int rc = check_view(b.len, b.rows, b.cols, b.rs, b.cs, "B");
    if (rc) return rc;
    return gk_prepack_rhs_i8_unchecked(static_cast<const int8_t*>(b.data), b.rs, b.cs, b.rows,
                                       b.cols, stream, out);
}

void gk_packed_rhs_free(gk_packed_rhs* p) {
    if (!p) return;
    if (p->buf) {
        cudaDeviceSynchronize();
        cudaFree(p->buf);
    }
    delete p;
}

// Serialized form: a 64-byte little-endian header (magic "GKPACK01", k, n, k_pad, n_pad,
// layout tag, payload bytes, zero padding) followed by the tiled buffer as it lies on the
// device. The layout tag names the tiled layout, so a future layout change is refused on load.
namespace {
constexpr char kPackMagic[8] = {'G', 'K', 'P', 'A', 'C', 'K', '0', '1'};
constexpr uint64_t kPackLayoutTiled128 = 1;  // 128-byte K blocks, rows 16-byte-chunk swizzled
struct PackHeader {
    char magic[8];
    uint64_t k, n, k_pad, n_pad, layout, payload;
    uint64_t pad[1];
};
static_assert(sizeof(PackHeader) == 64, "header size");
}  // namespace

int gk_packed_rhs_serialize(const gk_packed_rhs* p, void* out, size_t cap, size_t* needed) {
    if (!p || !needed) return set_err(GK_EINVAL, "gemmkit: null packed handle or size pointer");
    const size_t payload = (p->k && p->n) ? p->k_pad * p->n_pad : 0;
    *needed = sizeof(PackHeader) + payload;
    if (!out) return GK_OK;  // size query
    if (cap < *needed)
        return set_err(GK_EINVAL, "gemmkit: serialization buffer of %zu bytes, %zu needed", cap,
                       *needed);
    PackHeader h;
    memset(&h, 0, sizeof(h));
    memcpy(h.magic, kPackMagic, 8);
    h.k = p->k;
    h.n = p->n;
    h.k_pad = p->k_pad;
    h.n_pad = p->n_pad;
    h.layout = kPackLayoutTiled128;
    h.payload = payload;
    memcpy(out, &h, sizeof(h));
    if (payload) {
        cudaError_t e = cudaMemcpy(static_cast<char*>(out) + sizeof(h), p->buf, payload,
                                   cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return cuda_err(e, "packed serialization copy");
        }
    }
    return GK_OK;
}

int gk_packed_rhs_deserialize(const void* in, size_t len, gk_stream_t stream,
                              gk_packed_rhs** out) {
    if (!out || !in) return set_err(GK_EINVAL, "gemmkit: null input or output pointer");
    *out = nullptr;
    PackHeader h;
    if (len < sizeof(h)) return set_err(GK_EINVAL, "gemmkit: serialized packed B is truncated");
    memcpy(&h, in, sizeof(h));
    if (memcmp(h.magic, kPackMagic, 8) != 0)
        return set_err(GK_EINVAL, "gemmkit: not a serialized packed B (bad magic)");
    if (h.layout != kPackLayoutTiled128)
        return set_err(GK_EINVAL, "gemmkit: serialized packed B has unknown layout %llu",
                       static_cast<unsigned long long>(h.layout));
    const uint64_t want_kp = (h.k + 127) / 128 * 128, want_np = (h.n + 255) / 256 * 256;
    const uint64_t want_payload = (h.k && h.n) ? want_kp * want_np : 0;
    if (h.k_pad != want_kp || h.n_pad != want_np || h.payload != want_payload ||
        h.k > static_cast<uint64_t>(INT32_MAX / 2) || h.n > static_cast<uint64_t>(INT32_MAX))
        return set_err(GK_EINVAL, "gemmkit: serialized packed B has inconsistent dimensions");
    if (len < sizeof(h) + h.payload)
        return set_err(GK_EINVAL, "gemmkit: serialized packed B is truncated");
    int dev = 0;
    int rc = check_device(&dev);
    if (rc) return rc;
    gk_packed_rhs* p = new gk_packed_rhs{dev, nullptr, h.k, h.n, h.k_pad, h.n_pad};
    if (h.payload) {
        cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&p->buf), h.payload);
        if (e != cudaSuccess) {
            cudaGetLastError();
            delete p;
            return cuda_err(e, "packed deserialization allocation");
        }
        e = cudaMemcpyAsync(p->buf, static_cast<const char*>(in) + sizeof(h), h.payload,
                            cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
        if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) {  // complete before returning, like gk_prepack_rhs_i8
            cudaGetLastError();
            cudaFree(p->buf);
            delete p;
            return cuda_err(e, "packed deserialization copy");
        }
    }
    *out = p;
    return GK_OK;
}

size_t gk_packed_rhs_rows(const gk_packed_rhs* p) { return p ? p->k : 0; }
size_t gk_packed_rhs_cols(const gk_packed_rhs* p) { return p ? p->n : 0; }

int gk_gemm_i8_packed_b_unchecked(gk_workspace* ws, int32_t alpha, size_t m, const int8_t* a,
                                  ptrdiff_t rsa, ptrdiff_t csa, const gk_packed_rhs* packed,
                                  int32_t beta, int32_t* c, ptrdiff_t rsc, ptrdiff_t csc,
                                  gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    if (!packed) return set_err(GK_EINVAL, "gemmkit: null packed RHS");
    // gemmkit/src/api/packed.rs:626-631
    if (llabs(csc) < llabs(rsc))
        return set_err(GK_EINVAL,
                       "gemmkit: gemm_packed_b requires column-major-ish C (|csc| >= |rsc|); a "
                       "row-major C would swap A/B and invalidate the prepacked RHS \xe2\x80\x94 "
                       "use gemm() for that layout");
    if (m && packed->n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && packed->n && packed->k && alpha && !a) return set_err(GK_EINVAL, "gemmkit: null A");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.out = gk::Out::I32;
    j.m = m;
    j.k = packed->k;
    j.n = packed->n;
    j.a = Side{a, rsa, csa, 0};
    j.packed = packed;
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.alpha_i = alpha;
    j.beta_i = beta;
    return execute(j);
}

int gk_gemm_i8_packed_b(gk_workspace* ws, int32_t alpha, gk_matref a, const gk_packed_rhs* packed,
                        int32_t beta, gk_matmut c, gk_parallelism par, gk_stream_t stream) {
    if (!packed) return set_err(GK_EINVAL, "gemmkit: null packed RHS");
    // gemmkit/src/api/packed.rs:503-553
    if (a.cols != packed->k)
        return set_err(GK_EINVAL, "gemmkit: A.cols (%zu) != packed B.rows (%zu)", a.cols,
                       packed->k);
    if (packed->n != c.cols)
        return set_err(GK_EINVAL, "gemmkit: packed B.cols (%zu) != C.cols (%zu)", packed->n,
                       c.cols);
    if (a.rows != c.rows)
        return set_err(GK_EINVAL, "gemmkit: A.rows (%zu) != C.rows (%zu)", a.rows, c.rows);
    int rc;
    if ((rc = check_view(a.len, a.rows, a.cols, a.rs, a.cs, "A"))) return rc;
    if ((rc = check_view(c.len, c.rows, c.cols, c.rs, c.cs, "C"))) return rc;
    if (self_aliases(c.rows, c.cols, c.rs, c.cs))
        return set_err(GK_EINVAL,
                       "gemmkit: C view aliases itself (strides %td,%td map distinct elements to "
                       "the same memory); C must address each (i,j) uniquely",
                       c.rs, c.cs);
    if (overlaps_bytes(c.data, c.len, 4, a.data, a.len, 1))
        return set_err(GK_EINVAL, "gemmkit: C aliases A");
    return gk_gemm_i8_packed_b_unchecked(ws, alpha, a.rows, static_cast<const int8_t*>(a.data),
                                         a.rs, a.cs, packed, beta, static_cast<int32_t*>(c.data),
                                         c.rs, c.cs, par, stream);
}

int gk_gemm_i8_packed_b_requant_unchecked(gk_workspace* ws, size_t m, const int8_t* a,
                                          ptrdiff_t rsa, ptrdiff_t csa,
                                          const gk_packed_rhs* packed, const gk_requant* req,
                                          void* c, ptrdiff_t rsc, ptrdiff_t csc, int out_u8,
                                          gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    if (!packed) return set_err(GK_EINVAL, "gemmkit: null packed RHS");
    if (!req) return set_err(GK_EINVAL, "gemmkit: null requant descriptor");
    if (m && packed->n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && packed->n && packed->k && !a) return set_err(GK_EINVAL, "gemmkit: null A");
    if (req->scale_axis != GK_AXIS_NONE && !req->scales)
        return set_err(GK_EINVAL, "gemmkit: null requantize scales");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.m = m;
    j.k = packed->k;
    j.n = packed->n;
    j.a = Side{a, rsa, csa, 0};
    j.packed = packed;
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    fill_requant(j, req, out_u8 != 0);
    return execute(j);
}

int gk_gemv_i8_requant_unchecked(gk_workspace* ws, size_t m, const int8_t* a, ptrdiff_t rsa,
                                 ptrdiff_t csa, const gk_packed_rhs* packed,
                                 const gk_requant* req, void* c, ptrdiff_t rsc, ptrdiff_t csc,
                                 int out_u8, gk_stream_t stream) {
    if (m < 1 || m > 64)
        return set_err(GK_EINVAL, "gemmkit: gemv takes 1 to 64 activation rows (m = %zu)", m);
    const gk_parallelism par{0, 0};
    return gk_gemm_i8_packed_b_requant_unchecked(ws, m, a, rsa, csa, packed, req, c, rsc, csc,
                                                 out_u8, par, stream);
}

// ---- batched ------------------------------------------------------------------------------

int gk_gemm_i8_requant_batched_unchecked(gk_workspace* ws, size_t batch, size_t m, size_t k,
                                         size_t n, const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                                         ptrdiff_t a_bs, const int8_t* b, ptrdiff_t rsb,
                                         ptrdiff_t csb, ptrdiff_t b_bs, const gk_requant* req,
                                         ptrdiff_t bias_bs, ptrdiff_t scales_bs, void* c,
                                         ptrdiff_t rsc, ptrdiff_t csc, ptrdiff_t c_bs, int out_u8,
                                         gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    if (!req) return set_err(GK_EINVAL, "gemmkit: null requant descriptor");
    if (batch && m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (batch && m && n && k && (!a || !b)) return set_err(GK_EINVAL, "gemmkit: null A or B");
    if (req->scale_axis != GK_AXIS_NONE && !req->scales)
        return set_err(GK_EINVAL, "gemmkit: null requantize scales");
    Job j = base_job(ws, stream);
    j.kind = gk::Kind::I8;
    j.m = m;
    j.k = k;
    j.n = n;
    j.batch = batch;
    j.a = Side{a, rsa, csa, a_bs};
    j.b = Side{b, rsb, csb, b_bs};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.cbs = c_bs;
    fill_requant(j, req, out_u8 != 0);
    j.bias_bs = bias_bs;
    j.scale_bs = scales_bs;
    if (batch > 1 && c_bs == 0 && m && n)
        return set_err(GK_EINVAL, "gemmkit: batched C elements must not alias (c_bs == 0)");
    return execute(j);
}

int gk_gemm_i8_requant_batched_ptr_unchecked(gk_workspace* ws,
                                             const gk_i8_requant_problem* problems, size_t count,
                                             int out_u8, gk_parallelism par, gk_stream_t stream) {
    if (count && !problems) return set_err(GK_EINVAL, "gemmkit: null problem list");
    for (size_t i = 0; i < count; ++i) {
        const gk_i8_requant_problem& p = problems[i];
        int rc = gk_gemm_i8_requant_ex_unchecked(ws, p.m, p.k, p.n, p.a, p.rsa, p.csa, p.b, p.rsb,
                                                 p.csb, &p.req, p.c, p.rsc, p.csc, out_u8, par,
                                                 stream);
        if (rc) return rc;
    }
    return GK_OK;
}

// ---- half -> f32 ---------------------------------------------------------------------------

static int half_f32(gk_workspace* ws, bool f16, size_t batch, size_t m, size_t k, size_t n,
                    float alpha, const uint16_t* a, ptrdiff_t rsa, ptrdiff_t csa, ptrdiff_t a_bs,
                    const uint16_t* b, ptrdiff_t rsb, ptrdiff_t csb, ptrdiff_t b_bs, float beta,
                    float* c, ptrdiff_t rsc, ptrdiff_t csc, ptrdiff_t c_bs, gk_stream_t stream) {
    if (batch && m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (batch && m && n && k && alpha != 0.0f && (!a || !b))
        return set_err(GK_EINVAL, "gemmkit: null A or B");
    Job j = base_job(ws, stream);
    j.kind = f16 ? gk::Kind::F16 : gk::Kind::BF16;
    j.out = gk::Out::F32;
    j.m = m;
    j.k = k;
    j.n = n;
    j.batch = batch;
    j.a = Side{a, rsa, csa, a_bs};
    j.b = Side{b, rsb, csb, b_bs};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.cbs = c_bs;
    j.alpha_f = alpha;
    j.beta_f = beta;
    if (batch > 1 && c_bs == 0 && m && n)
        return set_err(GK_EINVAL, "gemmkit: batched C elements must not alias (c_bs == 0)");
    return execute(j);
}

int gk_gemm_bf16_f32_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n, float alpha,
                               const uint16_t* a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t* b,
                               ptrdiff_t rsb, ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc,
                               ptrdiff_t csc, gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    return half_f32(ws, false, 1, m, k, n, alpha, a, rsa, csa, 0, b, rsb, csb, 0, beta, c, rsc,
                    csc, 0, stream);
}

int gk_gemm_f16_f32_unchecked(gk_workspace* ws, size_t m, size_t k, size_t n, float alpha,
                              const uint16_t* a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t* b,
                              ptrdiff_t rsb, ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc,
                              ptrdiff_t csc, gk_parallelism par, gk_stream_t stream) {
    (void)par_ignored(par);
    return half_f32(ws, true, 1, m, k, n, alpha, a, rsa, csa, 0, b, rsb, csb, 0, beta, c, rsc,
                    csc, 0, stream);
}

int gk_gemm_half_f32(gk_workspace* ws, int is_f16, float alpha, gk_matref a, gk_matref b,
                     float beta, gk_matmut c, gk_parallelism par, gk_stream_t stream) {
    int rc = validate_gemm_views(a, b, c, 2, 4);
    if (rc) return rc;
    (void)par_ignored(par);
    return half_f32(ws, is_f16 != 0, 1, a.rows, a.cols, b.cols, alpha,
                    static_cast<const uint16_t*>(a.data), a.rs, a.cs, 0,
                    static_cast<const uint16_t*>(b.data), b.rs, b.cs, 0, beta,
                    static_cast<float*>(c.data), c.rs, c.cs, 0, stream);
}

int gk_gemm_half_f32_batched_unchecked(gk_workspace* ws, int is_f16, size_t batch, size_t m,
                                       size_t k, size_t n, float alpha, const uint16_t* a,
                                       ptrdiff_t rsa, ptrdiff_t csa, ptrdiff_t a_bs,
                                       const uint16_t* b, ptrdiff_t rsb, ptrdiff_t csb,
                                       ptrdiff_t b_bs, float beta, float* c, ptrdiff_t rsc,
                                       ptrdiff_t csc, ptrdiff_t c_bs, gk_parallelism par,
                                       gk_stream_t stream) {
    (void)par_ignored(par);
    return half_f32(ws, is_f16 != 0, batch, m, k, n, alpha, a, rsa, csa, a_bs, b, rsb, csb, b_bs,
                    beta, c, rsc, csc, c_bs, stream);
}

// ---- fused float epilogue (gemm_fused on the half -> f32 GEMM) -------------------------------

static int half_fused(gk_workspace* ws, bool f16, size_t m, size_t k, size_t n, float alpha,
                      const uint16_t* a, ptrdiff_t rsa, ptrdiff_t csa, const uint16_t* b,
                      ptrdiff_t rsb, ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc,
                      ptrdiff_t csc, const float* bias, int bias_dim, int has_bias, int act,
                      float leak, gk_stream_t stream) {
    if (m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && n && k && alpha != 0.0f && (!a || !b))
        return set_err(GK_EINVAL, "gemmkit: null A or B");
    if (act != GK_ACT_NONE && act != GK_ACT_RELU && act != GK_ACT_LEAKY_RELU)
        return set_err(GK_EINVAL, "gemmkit: unknown activation %d", act);
    if (has_bias && bias_dim != GK_AXIS_ROW && bias_dim != GK_AXIS_COL)
        return set_err(GK_EINVAL, "gemmkit: bias dimension must be row or column");
    if (has_bias && m && n && !bias) return set_err(GK_EINVAL, "gemmkit: null bias");
    Job j = base_job(ws, stream);
    j.kind = f16 ? gk::Kind::F16 : gk::Kind::BF16;
    j.out = gk::Out::F32;
    j.m = m;
    j.k = k;
    j.n = n;
    j.a = Side{a, rsa, csa, 0};
    j.b = Side{b, rsb, csb, 0};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.alpha_f = alpha;
    j.beta_f = beta;
    j.fbias = has_bias ? bias : nullptr;
    j.fbias_axis = has_bias ? bias_dim : GK_AXIS_NONE;
    j.act = act;
    j.leak = act == GK_ACT_LEAKY_RELU ? leak : 0.0f;
    return execute(j);
}

int gk_gemm_half_f32_fused_unchecked(gk_workspace* ws, int is_f16, size_t m, size_t k, size_t n,
                                     float alpha, const uint16_t* a, ptrdiff_t rsa,
                                     ptrdiff_t csa, const uint16_t* b, ptrdiff_t rsb,
                                     ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc,
                                     ptrdiff_t csc, const float* bias, int bias_dim,
                                     int has_bias, int act, float leak, gk_parallelism par,
                                     gk_stream_t stream) {
    (void)par_ignored(par);
    return half_fused(ws, is_f16 != 0, m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc,
                      csc, bias, bias_dim, has_bias, act, leak, stream);
}

int gk_gemm_half_f32_fused(gk_workspace* ws, int is_f16, float alpha, gk_matref a, gk_matref b,
                           float beta, gk_matmut c, const float* bias, size_t bias_len,
                           int bias_dim, int act, float leak, gk_parallelism par,
                           gk_stream_t stream) {
    int rc = validate_gemm_views(a, b, c, 2, 4);
    if (rc) return rc;
    if (bias) {
        // gemmkit's bias check (gemmkit/src/api.rs:318-330): the length follows its dimension
        const size_t want = bias_dim == GK_AXIS_COL ? b.cols : a.rows;
        if (bias_dim != GK_AXIS_ROW && bias_dim != GK_AXIS_COL)
            return set_err(GK_EINVAL, "gemmkit: bias dimension must be row or column");
        if (bias_len != want)
            return set_err(GK_EINVAL, "gemmkit: %s bias length %zu does not match %s = %zu",
                           bias_dim == GK_AXIS_COL ? "per-column" : "per-row", bias_len,
                           bias_dim == GK_AXIS_COL ? "n" : "m", want);
    }
    (void)par_ignored(par);
    return half_fused(ws, is_f16 != 0, a.rows, a.cols, b.cols, alpha,
                      static_cast<const uint16_t*>(a.data), a.rs, a.cs,
                      static_cast<const uint16_t*>(b.data), b.rs, b.cs, beta,
                      static_cast<float*>(c.data), c.rs, c.cs, bias, bias_dim, bias != nullptr,
                      act, leak, stream);
}

// ---- producer step: quantize f32 activations (extension) -----------------------------------

int gk_quantize_f32_i8_unchecked(size_t rows, size_t cols, const float* x, ptrdiff_t rsx,
                                 ptrdiff_t csx, int8_t* q, ptrdiff_t rsq, ptrdiff_t csq,
                                 float scale, int32_t zero_point, float* row_scales,
                                 gk_stream_t stream) {
    if (rows == 0 || cols == 0) return GK_OK;
    if (!x || !q) return set_err(GK_EINVAL, "gemmkit: null input or output");
    if (!row_scales) {
        int rc = check_scale_value(scale);
        if (rc) return rc;
        if (zero_point < -128 || zero_point > 127)
            return set_err(GK_EINVAL, "gemmkit: i8 zero point %d out of range", zero_point);
    }
    int dev = 0;
    int rc = check_device(&dev);
    if (rc) return rc;
    if (gk::launch_quantize_rows(x, rsx, csx, static_cast<int64_t>(rows),
                                 static_cast<int64_t>(cols), q, rsq, csq, scale,
                                 row_scales ? 0 : zero_point, row_scales,
                                 static_cast<cudaStream_t>(stream)))
        return set_err(GK_ECUDA, "gemmkit: quantize kernel launch failed");
    return GK_OK;
}

// ---- mirrored outputs (extension) ----------------------------------------------------------

static int set_mirrors(Job& j, void* const* mirrors, int nmirror) {
    if (nmirror < 0 || nmirror > 7)
        return set_err(GK_EINVAL, "gemmkit: at most 7 mirrored outputs (got %d)", nmirror);
    if (nmirror && !mirrors) return set_err(GK_EINVAL, "gemmkit: null mirror list");
    for (int i = 0; i < nmirror; ++i) {
        if (!mirrors[i]) return set_err(GK_EINVAL, "gemmkit: null mirrored output %d", i);
        j.mirror[i] = mirrors[i];
    }
    j.nmirror = nmirror;
    return GK_OK;
}

int gk_gemm_half_f32_mirrored_unchecked(gk_workspace* ws, int is_f16, size_t m, size_t k,
                                        size_t n, float alpha, const uint16_t* a, ptrdiff_t rsa,
                                        ptrdiff_t csa, const uint16_t* b, ptrdiff_t rsb,
                                        ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc,
                                        ptrdiff_t csc, void* const* mirrors, int nmirror,
                                        gk_stream_t stream) {
    if (m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (m && n && k && (!a || !b)) return set_err(GK_EINVAL, "gemmkit: null A or B");
    Job j = base_job(ws, stream);
    int rc = set_mirrors(j, mirrors, nmirror);
    if (rc) return rc;
    j.kind = is_f16 ? gk::Kind::F16 : gk::Kind::BF16;
    j.out = gk::Out::F32;
    j.m = m;
    j.k = k;
    j.n = n;
    j.a = Side{a, rsa, csa, 0};
    j.b = Side{b, rsb, csb, 0};
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.alpha_f = alpha;
    j.beta_f = beta;
    return execute(j);
}

int gk_gemm_i8_requant_mirrored_unchecked(gk_workspace* ws, size_t batch, size_t m, size_t k,
                                          size_t n, const int8_t* a, ptrdiff_t rsa,
                                          ptrdiff_t csa, ptrdiff_t a_bs, const int8_t* b,
                                          ptrdiff_t rsb, ptrdiff_t csb, ptrdiff_t b_bs,
                                          const gk_packed_rhs* packed, const gk_requant* req,
                                          ptrdiff_t bias_bs, ptrdiff_t scales_bs, void* c,
                                          ptrdiff_t rsc, ptrdiff_t csc, ptrdiff_t c_bs,
                                          int out_u8, void* const* mirrors, int nmirror,
                                          gk_stream_t stream) {
    if (!req) return set_err(GK_EINVAL, "gemmkit: null requant descriptor");
    if (batch && m && n && !c) return set_err(GK_EINVAL, "gemmkit: null C");
    if (batch && m && n && k && (!a || (!b && !packed)))
        return set_err(GK_EINVAL, "gemmkit: null A or B");
    if (req->scale_axis != GK_AXIS_NONE && !req->scales)
        return set_err(GK_EINVAL, "gemmkit: null requantize scales");
    if (packed && (batch > 1 || packed->k != k || packed->n != n))
        return set_err(GK_EINVAL, "gemmkit: prepacked B geometry does not match (k, n) or batch > 1");
    Job j = base_job(ws, stream);
    int rc = set_mirrors(j, mirrors, nmirror);
    if (rc) return rc;
    j.kind = gk::Kind::I8;
    j.m = m;
    j.k = k;
    j.n = n;
    j.batch = batch;
    j.a = Side{a, rsa, csa, a_bs};
    j.b = Side{b, rsb, csb, b_bs};
    j.packed = packed;
    j.c = c;
    j.rsc = rsc;
    j.csc = csc;
    j.cbs = c_bs;
    fill_requant(j, req, out_u8 != 0);
    j.bias_bs = bias_bs;
    j.scale_bs = scales_bs;
    if (batch > 1 && c_bs == 0 && m && n)
        return set_err(GK_EINVAL, "gemmkit: batched C elements must not alias (c_bs == 0)");
    return execute(j);
}

// ---- self test -----------------------------------------------------------------------------

int gk_selftest_wait_timeout(uint64_t timeout_ns, gk_stream_t stream) {
    int dev = 0;
    int rc = check_device(&dev);
    if (rc) return rc;
    uint32_t before = 0;
    rc = gk_device_status(dev, 1, &before);
    if (rc) return rc;
    if (gk::launch_selftest_timeout(timeout_ns, static_cast<cudaStream_t>(stream)))
        return set_err(GK_ECUDA, "gemmkit: self-test launch failed");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "self-test");
    uint32_t st = 0;
    rc = gk_device_status(dev, 1, &st);
    if (rc) return rc;
    if (st & 0x10u)
        return set_err(GK_ETIMEOUT, "gemmkit: device wait gave up after %llu ns (status 0x%x)",
                       static_cast<unsigned long long>(timeout_ns), st);
    return GK_OK;
}

}  // extern "C"
