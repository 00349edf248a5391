// pkv_inst_e4m3.cu -- decode-kernel instantiations: e4m3 pools (fp16 q / output), 16-byte cp.async gather;
// box rows 16 (page sizes that are multiples of 16) and 8, G = 1, 2, 4, 8.
#include "pkv_launch.cuh"

namespace pkv_internal {
PKV_DEFINE_LAUNCH_G(__half, 16, pkv::kLoadCpAsync, true)
PKV_DEFINE_LAUNCH_G(__half, 8, pkv::kLoadCpAsync, true)
}  // namespace pkv_internal
