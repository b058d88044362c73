// tcgen05 / TMEM tensor-core flash forward (sm_100a). Interface used by the entry points.
#pragma once

#include "attention_common.cuh"

namespace rk {
namespace tc {

// launch_flash_forward's return value when the tensor maps cannot describe the tensors; the
// caller then runs the SIMT kernel instead.
constexpr int kNotEligible = -1;

// True when the tensor-core kernel accepts the problem (head width 32, TMA-addressable tensors).
bool flash_supported(const AttentionParams &p);
// Launches the tensor-core flash forward; returns a cudaError_t value.
int launch_flash_forward(const AttentionParams &p, cudaStream_t stream);
// Static description of the build (architecture and kernel families).
const char *build_info();
// Reads (and optionally clears) the device status word set by a failed bounded wait;
// synchronizes with the device. 0 = no failure recorded.
unsigned int read_device_status(bool clear);
// Name of the tensor-core flash kernel (for benchmarks and profiles).
const char *kernel_name();

}  // namespace tc
}  // namespace rk
