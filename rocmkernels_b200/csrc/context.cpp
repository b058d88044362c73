// Identity of the CUDA context a cached per-device value belongs to.
//
// The library caches two things per device: the kernels' dynamic shared-memory attribute (set
// once with cudaFuncSetAttribute) and the device address of its static delta array
// (cudaGetSymbolAddress). Both belong to one context: cudaDeviceReset (ROCmKernels::ResetDevice,
// or any other code in the process) destroys the primary context, unloads the library's module
// and frees its device memory, and the next runtime call creates a new context where the
// attribute is unset and the array may sit at another address. A cache entry therefore records
// the context it was made in, and is trusted only while that context is current.
#include "context.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

namespace rk {

namespace {

using CtxGetCurrent = CUresult (*)(CUcontext *);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long *);

std::atomic<unsigned long long> g_generation{1};

struct DriverCalls {
    CtxGetCurrent get_current = nullptr;
    CtxGetId get_id = nullptr;
};

const DriverCalls &driver_calls() {
    static DriverCalls calls;
    static std::once_flag once;
    std::call_once(once, [] {
        void *pointer = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &pointer, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            calls.get_current = reinterpret_cast<CtxGetCurrent>(pointer);
        pointer = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &pointer, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            calls.get_id = reinterpret_cast<CtxGetId>(pointer);
    });
    return calls;
}

}  // namespace

unsigned long long current_context_id() {
    const DriverCalls &calls = driver_calls();
    if (calls.get_current == nullptr || calls.get_id == nullptr) return 0;
    CUcontext context = nullptr;
    if (calls.get_current(&context) != CUDA_SUCCESS || context == nullptr) return 0;
    unsigned long long id = 0;
    if (calls.get_id(context, &id) != CUDA_SUCCESS) return 0;
    return id;
}

unsigned long long context_generation() { return g_generation.load(std::memory_order_acquire); }

void invalidate_context_caches() { g_generation.fetch_add(1, std::memory_order_acq_rel); }

unsigned long long context_key() {
    const unsigned long long id = current_context_id();
    if (id == 0) return 0;
    // 40 bits of context id, 24 bits of reset generation: distinct keys for every context the
    // process creates and every library-initiated reset.
    return (id << 24) ^ (context_generation() & 0xFFFFFFull);
}

}  // namespace rk
