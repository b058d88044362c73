// tcgen05 / TMEM tensor-core flash forward for sm_100a (placeholder until the kernel lands).
#include "attention_tc.cuh"

namespace rk {
namespace tc {

bool flash_supported(const AttentionParams &) { return false; }

int launch_flash_forward(const AttentionParams &, cudaStream_t) { return cudaErrorNotSupported; }

const char *kernel_name() { return "tcgen05-3xtf32-flash-d32"; }

const char *build_info() { return "sm_100a; simt-fp32 d32/d64 forward+backward"; }

}  // namespace tc
}  // namespace rk
