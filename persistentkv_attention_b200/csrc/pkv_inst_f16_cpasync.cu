// pkv_inst_f16_cpasync.cu -- decode-kernel instantiations: fp16 pools, 16-byte cp.async gather;
// box rows 16 (page sizes that are multiples of 16) and 8, G = 1, 2, 4, 8.
#include "pkv_launch.cuh"

namespace pkv_internal {
PKV_DEFINE_LAUNCH_G(__half, 16, pkv::kLoadCpAsync, false)
PKV_DEFINE_LAUNCH_G(__half, 8, pkv::kLoadCpAsync, false)
}  // namespace pkv_internal
