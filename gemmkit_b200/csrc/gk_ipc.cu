// gk_ipc.cu -- peer-memory plumbing for the sharded paths (no counterpart in gemmkit, which
// is single-process): a device buffer of one process is exported as a CUDA IPC handle plus
// the offset of the pointer inside its allocation, and other processes on the same node map
// it. The mapping is a plain peer mapping over NVLink (cudaIpcOpenMemHandle), never a
// multicast object. Opened allocations are reference-counted, so two pointers into one
// allocation share one mapping.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>

#include "gemmkit_cuda.h"
#include "gk_engine.h"

namespace {

typedef CUresult (*PFN_memGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_memGetAddressRange get_range_fn() {
    static PFN_memGetAddressRange fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_memGetAddressRange>(f);
    });
    return fn;
}

struct Mapping {
    void* base;
    int refs;
};

std::mutex g_mu;
std::map<std::string, Mapping> g_by_handle;  // handle bytes -> mapped base
std::map<void*, std::string> g_by_ptr;      // pointer handed out -> handle bytes
std::map<void*, int> g_ptr_refs;            // pointer handed out -> open count

int fail(int code, const char* what, cudaError_t e) {
    std::string s = std::string("gemmkit: ") + what;
    if (e != cudaSuccess) s += std::string(": ") + cudaGetErrorString(e);
    return gk::set_last_error(code, s.c_str());
}

}  // namespace

extern "C" int gk_ipc_export(const void* dev_ptr, gk_ipc_handle* out) {
    if (!dev_ptr || !out) return fail(GK_EINVAL, "null pointer passed to gk_ipc_export", cudaSuccess);
    PFN_memGetAddressRange range = get_range_fn();
    if (!range) return fail(GK_ENODEV, "cuMemGetAddressRange is unavailable", cudaSuccess);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(GK_EINVAL, "gk_ipc_export: not a device allocation", cudaSuccess);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(GK_ECUDA, "cudaIpcGetMemHandle", e);
    }
    static_assert(sizeof(h) <= sizeof(out->bytes), "IPC handle size");
    memset(out, 0, sizeof(*out));
    memcpy(out->bytes, &h, sizeof(h));
    out->offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(dev_ptr) - base);
    return GK_OK;
}

extern "C" int gk_ipc_open(const gk_ipc_handle* h, void** peer_ptr) {
    if (!h || !peer_ptr) return fail(GK_EINVAL, "null pointer passed to gk_ipc_open", cudaSuccess);
    *peer_ptr = nullptr;
    cudaIpcMemHandle_t mh;
    memcpy(&mh, h->bytes, sizeof(mh));
    const std::string key(reinterpret_cast<const char*>(h->bytes), sizeof(mh));
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_by_handle.find(key);
    void* base = nullptr;
    if (it != g_by_handle.end()) {
        base = it->second.base;
        it->second.refs++;
    } else {
        cudaError_t e = cudaIpcOpenMemHandle(&base, mh, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(GK_ECUDA, "cudaIpcOpenMemHandle", e);
        }
        g_by_handle[key] = Mapping{base, 1};
    }
    void* p = static_cast<char*>(base) + h->offset;
    g_by_ptr[p] = key;
    g_ptr_refs[p]++;
    *peer_ptr = p;
    return GK_OK;
}

extern "C" int gk_ipc_close(void* peer_ptr) {
    if (!peer_ptr) return GK_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    auto pi = g_by_ptr.find(peer_ptr);
    if (pi == g_by_ptr.end())
        return fail(GK_EINVAL, "gk_ipc_close: pointer was not opened by gk_ipc_open", cudaSuccess);
    const std::string key = pi->second;
    if (--g_ptr_refs[peer_ptr] == 0) {
        g_ptr_refs.erase(peer_ptr);
        g_by_ptr.erase(pi);
    }
    auto it = g_by_handle.find(key);
    if (it != g_by_handle.end() && --it->second.refs == 0) {
        cudaError_t e = cudaIpcCloseMemHandle(it->second.base);
        g_by_handle.erase(it);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(GK_ECUDA, "cudaIpcCloseMemHandle", e);
        }
    }
    return GK_OK;
}
