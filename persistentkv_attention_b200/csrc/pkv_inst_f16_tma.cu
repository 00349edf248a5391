// pkv_inst_f16_tma.cu -- decode-kernel instantiations: fp16 pools, TMA (cp.async.bulk.tensor) gather;
// box rows 16 (page sizes that are multiples of 16) and 8, G = 1, 2, 4, 8.
#include "pkv_launch.cuh"

namespace pkv_internal {
PKV_DEFINE_LAUNCH_G(__half, 16, pkv::kLoadTma, false)
PKV_DEFINE_LAUNCH_G(__half, 8, pkv::kLoadTma, false)
}  // namespace pkv_internal
