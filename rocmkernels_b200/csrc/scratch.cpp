// Per-device, stream-ordered scratch pool of the library (scratch.h).
//
// One cudaMemPool_t per device, created on first use with that device current. A pool belongs to
// the CUDA context it was made in: cudaDeviceReset destroys it with the context, so each entry
// records the context key (context.h) and a new pool is made when another context is current.
#include "scratch.h"

#include <cstdint>
#include <mutex>

#include "context.h"

namespace rk {

namespace {

constexpr int kDevices = 64;

struct PoolSlot {
    cudaMemPool_t pool = nullptr;
    unsigned long long key = 0;
};

std::mutex g_lock;
PoolSlot g_pools[kDevices];

// The pool of the current device and context, created if needed.
cudaError_t current_pool(cudaMemPool_t *pool, bool create) {
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return status;
    if (device < 0 || device >= kDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(g_lock);
    PoolSlot &slot = g_pools[device];
    unsigned long long key = context_key();
    if (slot.pool != nullptr && key != 0 && slot.key == key) {
        *pool = slot.pool;
        return cudaSuccess;
    }
    *pool = nullptr;
    if (!create) return cudaSuccess;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t created = nullptr;
    status = cudaMemPoolCreate(&created, &props);  // creates the context if none is current yet
    if (status != cudaSuccess) return status;
    uint64_t keep = kScratchKeepBytes;
    status = cudaMemPoolSetAttribute(created, cudaMemPoolAttrReleaseThreshold, &keep);
    if (status != cudaSuccess) {
        cudaMemPoolDestroy(created);
        return status;
    }
    // A pool left from an earlier context died with it (its handle must not be used again).
    slot.pool = created;
    slot.key = context_key();
    *pool = created;
    return cudaSuccess;
}

}  // namespace

cudaError_t scratch_acquire(void **pointer, size_t bytes, cudaStream_t stream) {
    *pointer = nullptr;
    cudaMemPool_t pool = nullptr;
    cudaError_t status = current_pool(&pool, true);
    if (status != cudaSuccess) return status;
    status = cudaMallocFromPoolAsync(pointer, bytes, pool, stream);
    if (status != cudaSuccess) *pointer = nullptr;
    return status;
}

cudaError_t scratch_release(void *pointer, cudaStream_t stream) {
    return pointer == nullptr ? cudaSuccess : cudaFreeAsync(pointer, stream);
}

cudaError_t scratch_trim() {
    cudaMemPool_t pool = nullptr;
    const cudaError_t status = current_pool(&pool, false);
    if (status != cudaSuccess || pool == nullptr) return status;
    return cudaMemPoolTrimTo(pool, 0);
}

}  // namespace rk
