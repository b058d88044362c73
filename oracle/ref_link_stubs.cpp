// Link-time stand-ins for the reference's CPU shims (libref_attention.so, libref_positional.so).
// TEST INFRASTRUCTURE ONLY.
//
// The shims include the reference's test files to reach their CPU functions (ReferenceAttention,
// ReferenceRotary, RandomValues). Those files also hold TEST_CASEs that name the attention entry
// points and a few CUDA runtime calls (through DeviceBuffer and the HIP header). The shims never
// run a TEST_CASE, so every such name is defined here as a function that does nothing and
// reports failure. The shims therefore load neither librocmkernels_attention.so nor a CUDA
// runtime: timing the reference's CPU code never maps the product library. The linker version
// script (ref_exports.map) keeps these definitions local, so they can never stand in for the
// real functions of another library loaded into the same process.
#include <cuda_runtime_api.h>
#include <rocmkernels_attention.h>

extern "C" {

int attention_fp32_forward(const float *, const float *, const float *, const bool *, float *, float *, int, int, int, int,
                           int, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                           RocmKernelsStream) {
    return 1;
}

int attention_fp32_forward_tiled(const float *, const float *, const float *, const bool *, float *, float *, int, int, int,
                                 int, int, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                                 RocmKernelsStream) {
    return 1;
}

int attention_fp32_forward_flash(const float *, const float *, const float *, const bool *, float *, float *, int, int, int,
                                 int, int, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                                 RocmKernelsStream) {
    return 1;
}

int attention_fp32_forward_flash_tuned(const float *, const float *, const float *, const bool *, float *, float *, int, int,
                                       int, int, int, int, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                                       RocmKernelsStrides, RocmKernelsStream) {
    return 1;
}

int attention64_fp32_forward(const float *, const float *, const float *, const bool *, float *, float *, int, int, int, int,
                             int, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                             RocmKernelsStream) {
    return 1;
}

int attention_fp32_backward(const float *, const float *, const float *, const bool *, const float *, const float *,
                            const float *, float *, float *, float *, float *, int, int, int, int, int, RocmKernelsStrides,
                            RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStream) {
    return 1;
}

int attention_fp32_backward_tiled(const float *, const float *, const float *, const bool *, const float *, const float *,
                                  const float *, float *, float *, float *, float *, int, int, int, int, int,
                                  RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                                  RocmKernelsStrides, RocmKernelsStream) {
    return 1;
}

int attention64_fp32_backward(const float *, const float *, const float *, const bool *, const float *, const float *,
                              const float *, float *, float *, float *, float *, int, int, int, int, int, RocmKernelsStrides,
                              RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides,
                              RocmKernelsStream) {
    return 1;
}

int rotary_fp32(const float *, const float *, const float *, const float *, float *, float *, int, int, int, int,
                RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStrides, RocmKernelsStream) {
    return 1;
}

cudaError_t cudaMalloc(void **pointer, size_t) {
    if (pointer) *pointer = nullptr;
    return cudaErrorNotSupported;
}
cudaError_t cudaFree(void *) { return cudaErrorNotSupported; }
cudaError_t cudaMemcpy(void *, const void *, size_t, cudaMemcpyKind) { return cudaErrorNotSupported; }
cudaError_t cudaDeviceSynchronize(void) { return cudaErrorNotSupported; }
const char *cudaGetErrorString(cudaError_t) { return "not available in the reference's CPU shim"; }

}  // extern "C"
