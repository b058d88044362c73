// Exposes the reference's own CPU rotary embedding to the oracle checks.
// TEST INFRASTRUCTURE: compiled into oracle/_ref/libref_positional.so by oracle/Makefile, only
// when the reference tree is present; never committed, never part of the product.
//
// The reference file is included, not copied: ROCMKERNELS_REFERENCE_POSITIONAL names
// ROCmKernels.Tests/PositionalTests.cpp where it lies, so its ReferenceRotary (:18-50) lives in
// this translation unit. The file's TEST_CASEs reference the library's rotary entry point,
// which oracle/ref_link_stubs.cpp defines as a local stand-in: nothing here calls it, and the
// shim loads neither the product library nor a CUDA runtime.
#include <cstddef>
#include <vector>

#include ROCMKERNELS_REFERENCE_POSITIONAL

extern "C" void ref_rotary(const float *input, const float *cosine, const float *sine, float *output, int batch, int heads,
                           int length, int backward) {
    const std::size_t elements = static_cast<std::size_t>(batch) * heads * length * kHeadWidth;
    const std::size_t table = static_cast<std::size_t>(batch) * length * kHeadWidth;
    const std::vector<float> in(input, input + elements), c(cosine, cosine + table), s(sine, sine + table);
    std::vector<float> out(elements);
    ReferenceRotary(in, c, s, out, batch, heads, length, backward != 0);
    std::copy(out.begin(), out.end(), output);
}
