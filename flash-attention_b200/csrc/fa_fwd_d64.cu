// Instantiates the sm_100a forward kernel for head_dim = 64 (f16/bf16 x causal/non-causal).
#include "fa_launch.h"

namespace fa {
cudaError_t launch_d64(const LaunchSpec& s) { return launch_for_dim<64>(s); }
}  // namespace fa
