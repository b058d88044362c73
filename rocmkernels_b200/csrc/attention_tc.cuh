// tcgen05 / TMEM tensor-core flash forward and backward (sm_100a). Interface used by the entry points.
#pragma once

#include "attention_common.cuh"

namespace rk {
namespace tc {

// launch_flash_forward's return value when the tensor maps cannot describe the tensors; the
// caller then runs the SIMT kernel instead.
constexpr int kNotEligible = -1;

// True when the tensor-core flash forward accepts the tensors (TMA-addressable K and V, 16-byte
// addressable Q rows).
bool flash_supported(const AttentionParams &p);
// Launches the tensor-core flash forward for head width 32 or 64 (16: the 32-wide kernel over
// zero-filled features 16-31); returns a cudaError_t value or kNotEligible. Head width 32 with a
// workspace (prepared_forward_bytes, 128-byte aligned; nullptr for none) runs, where it pays, the
// prepared-operand forward (an operand pre-pass into the workspace, then the forward), else the
// forward with in-kernel split warps.
int launch_flash_forward(const AttentionParams &p, int head_width, void *workspace, cudaStream_t stream);
// Workspace bytes of the prepared d = 32 forward: a 16 KB stage image and a 16-byte header per
// 64-key tile of each (batch, head).
long long prepared_forward_bytes(int batch, int heads, int keys);
// The flash forward for head width 32 with the rotary prologue (q and k rotated by the tables in
// p.rot_*, which must be 16-byte aligned with strides of 4 floats), with an optional workspace as
// launch_flash_forward; cudaError_t or kNotEligible.
int launch_flash_forward_rotary(const AttentionParams &p, void *workspace, cudaStream_t stream);

// Statistics only ({row max, sum} per query, no V and no output): the split-FP16 flash forward
// without the P.V products; the row sums are taken in FP32 by the softmax threads. Eligible when
// K is TMA-addressable and Q rows 16-byte addressable; cudaError_t or kNotEligible.
bool statistics_supported(const AttentionParams &p);
int launch_statistics(const AttentionParams &p, cudaStream_t stream);
// True when the FP16-storage tensor-core forward accepts the tensors (TMA-addressable K and V,
// 16-byte addressable Q rows).
bool half_flash_supported(const AttentionParams &p);
// Launches the FP16-storage tensor-core forward (the generic forward's DType::Float16) for head
// width 16, 32 or 64; returns a cudaError_t value or kNotEligible.
int launch_half_flash_forward(const AttentionParams &p, int head_width, cudaStream_t stream);
// False when the driver rejects the tensor maps the tensor-core forward would use for these
// tensors (the launch then falls back to SIMT); true when it accepts them or no driver is loaded.
bool tensor_maps_encodable(const AttentionParams &p, int head_width, bool half);
// Name of the FP16-storage tensor-core kernel for a head width.
const char *half_kernel_name(int head_width);
// Static description of the build (architecture and kernel families).
const char *build_info();
// Reads (and optionally clears) the device status word set by a failed bounded wait;
// synchronizes with the device. 0 = no failure recorded.
unsigned int read_device_status(bool clear);
// Name of the tensor-core flash kernel that a problem of these sizes runs at this head width, with
// or without a workspace (for benchmarks and profiles); "-prepared" marks the d = 32 path of an
// operand pre-pass and the forward.
const char *kernel_name(const AttentionParams &p, int head_width, bool workspace);

// True when the tensor-core backward accepts the tensors (TMA-addressable q, k, v, dO; 16-byte
// addressable O and gradients).
bool backward_supported(const AttentionParams &p);
// Launches the tensor-core backward for head width 32 or 64: delta and dQ (query-major), then
// dK and dV (key-major), ordered on `stream`; returns a cudaError_t value or kNotEligible.
int launch_backward(const AttentionParams &p, int head_width, cudaStream_t stream);
// Workspace bytes of the fused backward for batch * heads heads of `queries` queries: the split
// scale Q and dO rows (128 bytes per query, queries padded to 64 per head) and one 528-byte record
// per 64-query tile.
long long fused_backward_workspace_bytes(long long batch_heads, long long queries);
// Launches the fused single-pass backward for head width 32 (a column pre-pass writing delta,
// zeroing dQ and filling the workspace, then one key-major kernel: dK and dV per key row, dQ added
// per query tile with FP32 atomics); returns a cudaError_t value or kNotEligible (also for a
// workspace that is not 128-byte aligned). Same tensors as launch_backward; `workspace` holds
// fused_backward_workspace_bytes bytes.
int launch_fused_backward(const AttentionParams &p, void *workspace, cudaStream_t stream);
// Device status word of the backward kernels (as read_device_status).
unsigned int read_backward_status(bool clear);

}  // namespace tc
}  // namespace rk
