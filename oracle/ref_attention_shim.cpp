// Exposes the reference's own CPU attention and input generator to the oracle checks.
// TEST INFRASTRUCTURE: compiled into oracle/_ref/libref_attention.so by oracle/Makefile, only
// when the reference tree is present; never committed, never part of the product.
//
// The reference file is included, not copied: ROCMKERNELS_REFERENCE_TESTS names
// ROCmKernels.Tests/AttentionTests.cpp where it lies. Its ReferenceAttention (:28-125) and
// TestSupport.hpp's RandomValues (:11-21) live in this translation unit, so the extern "C"
// functions below can call them. The file's TEST_CASE references the library's entry points,
// which oracle/ref_link_stubs.cpp defines as local stand-ins: nothing here calls them, and the
// shim loads neither the product library nor a CUDA runtime.
#include <cstddef>
#include <cstdint>
#include <vector>

#include ROCMKERNELS_REFERENCE_TESTS

extern "C" int ref_attention(const float *q, const float *k, const float *v, const std::uint8_t *mask,
                             const float *upstream, int head_width, int batch, int heads, int queries, int keys,
                             int radius, float *output, float *lse, float *grad_q, float *grad_k, float *grad_v) {
    const std::size_t qn = static_cast<std::size_t>(batch) * heads * queries * head_width;
    const std::size_t kn = static_cast<std::size_t>(batch) * heads * keys * head_width;
    const std::vector<float> vq(q, q + qn), vk(k, k + kn), vv(v, v + kn), vu(upstream, upstream + qn);
    const std::vector<std::uint8_t> vm(mask, mask + static_cast<std::size_t>(batch) * keys);
    const Reference r = ReferenceAttention(vq, vk, vv, vm, vu, head_width, batch, heads, queries, keys, radius);
    std::copy(r.output.begin(), r.output.end(), output);
    std::copy(r.lse.begin(), r.lse.end(), lse);
    std::copy(r.gradientQ.begin(), r.gradientQ.end(), grad_q);
    std::copy(r.gradientK.begin(), r.gradientK.end(), grad_k);
    std::copy(r.gradientV.begin(), r.gradientV.end(), grad_v);
    return 0;
}

extern "C" void ref_random_values(float *out, std::size_t count, unsigned int seed, float low, float high) {
    const std::vector<float> values = ROCmKernels::Tests::RandomValues<float>(count, seed, low, high);
    std::copy(values.begin(), values.end(), out);
}
