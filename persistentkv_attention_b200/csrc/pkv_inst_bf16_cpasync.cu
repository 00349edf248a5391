// pkv_inst_bf16_cpasync.cu -- decode-kernel instantiations: bf16 pools, 16-byte cp.async gather;
// box rows 16 (page sizes that are multiples of 16) and 8, G = 1, 2, 4, 8.
#include "pkv_launch.cuh"

namespace pkv_internal {
PKV_DEFINE_LAUNCH_G(__nv_bfloat16, 16, pkv::kLoadCpAsync, false)
PKV_DEFINE_LAUNCH_G(__nv_bfloat16, 8, pkv::kLoadCpAsync, false)
}  // namespace pkv_internal
