// Device scratch memory that the library allocates for itself (implemented in scratch.cpp).
//
// The reference's entry points take no workspace argument, yet the d = 32 flash forward needs one
// (the split K/V operands its pre-pass writes). It comes from a stream-ordered memory pool that the
// library creates per device: acquiring and releasing are enqueued on the caller's stream like the
// kernels, so calls on different streams never share memory that is in use, and no call waits for
// the device.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace rk {

// Allocates `bytes` on the current device, ordered on `stream` (cudaMallocFromPoolAsync from the
// library's pool for that device and context). Returns the CUDA status; on failure *pointer is null
// and nothing is enqueued.
cudaError_t scratch_acquire(void **pointer, size_t bytes, cudaStream_t stream);

// Gives memory from scratch_acquire back to the pool, ordered on `stream` after the work enqueued
// before it (cudaFreeAsync).
cudaError_t scratch_release(void *pointer, cudaStream_t stream);

// Returns the current device's pooled memory that no call is using to the system
// (cudaMemPoolTrimTo(pool, 0)); a no-op when the library has no pool on that device.
cudaError_t scratch_trim();

// The pool keeps up to this many bytes across synchronisations (its release threshold), so that
// calls of a repeated shape do not map memory again (mapping the 806 MB of a B64 H12 S4096 forward
// inside a timed loop cost about as much as its kernels saved); memory above it returns to the
// system at the next synchronisation, and rocmkernels_attention_release_scratch returns the rest.
constexpr size_t kScratchKeepBytes = size_t(4) << 30;

}  // namespace rk
