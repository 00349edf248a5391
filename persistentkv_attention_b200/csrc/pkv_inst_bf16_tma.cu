// pkv_inst_bf16_tma.cu -- decode-kernel instantiations: bf16 pools, TMA (cp.async.bulk.tensor) gather;
// box rows 16 (page sizes that are multiples of 16) and 8, G = 1, 2, 4, 8.
#include "pkv_launch.cuh"

namespace pkv_internal {
PKV_DEFINE_LAUNCH_G(__nv_bfloat16, 16, pkv::kLoadTma, false)
PKV_DEFINE_LAUNCH_G(__nv_bfloat16, 8, pkv::kLoadTma, false)
}  // namespace pkv_internal
