// Keys for per-device caches that must not outlive the CUDA context they were made in
// (implemented in context.cpp).
#pragma once

namespace rk {

// Unique id of the CUDA context current on the calling thread (cuCtxGetId: unique for the life
// of the process, so a context that cudaDeviceReset destroyed and the runtime created again has
// a new id), or 0 when no context is current yet or the driver cannot say.
unsigned long long current_context_id();

// Counter bumped by ROCmKernels::ResetDevice after it reset a device.
unsigned long long context_generation();
void invalidate_context_caches();

// Cache key of the current context: nonzero, and different for every context and every reset
// the library made; 0 when no context is current (the caller then does the work uncached, which
// creates the context, and asks again).
unsigned long long context_key();

}  // namespace rk
