// gk_noalloc.cu -- gk_gemm_i8_noalloc_unchecked: the i8 -> i32 product for callers that must
// not allocate device memory.
//
// gk_gemm_i8_unchecked gathers an operand that is not K-contiguous and 16-byte aligned (a
// row-major B, a column-major A, a negative or odd stride) into a workspace, and the default
// workspace grows with cudaMalloc. Some callers cannot allow that: a host that hands the GPU
// a fixed memory budget through its own allocator, or a latency-critical serving loop, where
// cudaMalloc / cudaFree may synchronise the device and stall every other stream. This entry
// takes the same arguments and gives the same bytes, but its operand packs go to a
// file-scope device array of fixed size instead of a workspace, so it never calls cudaMalloc,
// cudaFree or any allocating library routine.
//
// Limits and rules:
//  - The array holds GK_NOALLOC_SCRATCH_BYTES (16 MiB). Every GPU that loads this library
//    holds it until the process exits. A call whose packs need more returns GK_EINVAL.
//  - The first call on a device looks up the array's device address (cudaGetSymbolAddress,
//    with that device current); make that first call before any stream capture.
//  - Every call shares the one array and it keeps the last call's contents. Calls that overlap
//    on the GPU (different streams, or host threads without ordering) race on it; order them
//    on one stream. Each call writes every scratch byte it later reads (zero K padding
//    included), so nothing needs to start at zero.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "gemmkit_cuda.h"
#include "gk_engine.h"

namespace {

// The scratch itself. In host code `g_noalloc_scratch` is only a stand-in symbol, never a
// device address: a kernel given it would fault or, where the GPU can reach host memory,
// silently use the wrong memory. Host code uses the address from noalloc_scratch_addr().
__device__ __align__(256) unsigned char g_noalloc_scratch[GK_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void* g_addr[64] = {nullptr};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return gk::set_last_error(code, buf);
}

// Device address of the scratch on `dev` (which must be current), looked up once per device.
int noalloc_scratch_addr(int dev, void** out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return fail(GK_ECUDA, "gemmkit: cannot resolve the no-alloc scratch on device %d: %s",
                        dev, cudaGetErrorString(e));
        }
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return GK_OK;
}

struct Op {  // canonical-frame operand: rows x K, element (r, p) at r*rs + p*ks
    const void* p;
    int64_t rows, rs, ks;
};

bool tma_ready(const Op& o, int64_t K) {
    if (o.ks != 1 && K > 1) return false;
    if (reinterpret_cast<uintptr_t>(o.p) & 15) return false;
    if (o.rows > 1 && (o.rs <= 0 || o.rs % 16 != 0)) return false;
    return true;
}

}  // namespace

extern "C" int gk_gemm_i8_noalloc_unchecked(size_t m, size_t k, size_t n, int32_t alpha,
                                            const int8_t* a, ptrdiff_t rsa, ptrdiff_t csa,
                                            const int8_t* b, ptrdiff_t rsb, ptrdiff_t csb,
                                            int32_t beta, int32_t* c, ptrdiff_t rsc,
                                            ptrdiff_t csc, gk_stream_t stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (m == 0 || n == 0) return GK_OK;
    if (!c) return fail(GK_EINVAL, "gemmkit: null C");
    if (k && alpha && (!a || !b)) return fail(GK_EINVAL, "gemmkit: null A or B");
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess || dev < 0 || dev >= 64)
        return fail(GK_ENODEV, "gemmkit: no CUDA device");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
        return fail(GK_ENODEV, "gemmkit: the CUDA engine needs an sm_100 (B200) device");
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX / 2)
        return fail(GK_EINVAL, "gemmkit: problem dimensions exceed the engine's limits");
    void* scratch = nullptr;
    int rc = noalloc_scratch_addr(dev, &scratch);
    if (rc) return rc;

    // gemmkit's degenerate rule (execute_int, gemmkit/src/dispatch/int.rs:131-163)
    if (k == 0 || alpha == 0) {
        if (gk::launch_scale_c_i32(c, m, n, rsc, csc, beta, st))
            return fail(GK_ECUDA, "gemmkit: fill kernel launch failed");
        return GK_OK;
    }

    // the orientation rule of the allocating entry
    bool swap;
    if (m <= 64 && n > m)
        swap = true;
    else if (n <= 64 && m > n)
        swap = false;
    else if (csc == 1)
        swap = false;
    else if (rsc == 1)
        swap = true;
    else
        swap = llabs(csc) > llabs(rsc);
    const Op ua{a, static_cast<int64_t>(m), rsa, csa};
    const Op ub{b, static_cast<int64_t>(n), csb, rsb};
    Op ops[2] = {swap ? ub : ua, swap ? ua : ub};
    const int64_t Mk = swap ? n : m, Nk = swap ? m : n;
    const int64_t K = static_cast<int64_t>(k);
    const int64_t ldp = (K + 15) / 16 * 16;

    int64_t need[2] = {0, 0};
    for (int i = 0; i < 2; ++i) {
        if (ops[i].rows == 1 && ops[i].ks == 1 && !(reinterpret_cast<uintptr_t>(ops[i].p) & 15))
            ops[i].rs = ldp;
        if (!tma_ready(ops[i], K)) need[i] = (ops[i].rows * ldp + 255) / 256 * 256;
    }
    const int64_t total = need[0] + need[1];
    if (total > static_cast<int64_t>(GK_NOALLOC_SCRATCH_BYTES))
        return fail(GK_EINVAL,
                    "gemmkit: gk_gemm_i8_noalloc_unchecked needs %lld bytes of scratch to pack its "
                    "operands but its fixed scratch holds %u bytes; pass K-contiguous, 16-byte "
                    "aligned operands or use gk_gemm_i8_unchecked",
                    static_cast<long long>(total), static_cast<unsigned>(GK_NOALLOC_SCRATCH_BYTES));
    char* cur = static_cast<char*>(scratch);
    for (int i = 0; i < 2; ++i) {
        if (!need[i]) continue;
        if (gk::launch_pack_kmajor(cur, ldp, 0, ops[i].p, ops[i].rs, ops[i].ks, 0, ops[i].rows, K,
                                   1, 1, st))
            return fail(GK_ECUDA, "gemmkit: pack kernel launch failed");
        ops[i] = Op{cur, ops[i].rows, ldp, 1};
        cur += need[i];
    }

    gk::EpiParams e;
    memset(&e, 0, sizeof(e));
    e.out = c;
    e.ldo = swap ? csc : rsc;
    e.cso = swap ? rsc : csc;
    e.alpha_i = alpha;
    e.beta_i = beta;
    e.vec = (e.cso == 1) && !(reinterpret_cast<uintptr_t>(c) & 15) &&
            ((e.ldo * 4) % 16 == 0 || Mk == 1);
    gk::TcProblem pr;
    memset(&pr, 0, sizeof(pr));  // no stream-K scratch (sk_* null), no launch overlap
    pr.pdl = 0;
    pr.kind = gk::Kind::I8;
    pr.out = gk::Out::I32;
    pr.Mk = Mk;
    pr.Nk = Nk;
    pr.K = K;
    pr.batch = 1;
    pr.a = gk::Operand{ops[0].p, ops[0].rows, ops[0].rs, 0};
    pr.b = gk::Operand{ops[1].p, ops[1].rows, ops[1].rs, 0};
    pr.e = e;
    pr.bn = 0;
    pr.stream = st;
    char err[512] = "";
    rc = gk::launch_tc_gemm(pr, err, sizeof(err));
    if (rc) return gk::set_last_error(rc, err);
    return GK_OK;
}
