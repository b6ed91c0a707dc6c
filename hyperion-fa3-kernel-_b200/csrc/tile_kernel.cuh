// tile_kernel.cuh -- 128-row tcgen05 tile kernel (prefill path).
#pragma once

#include "common.cuh"

namespace hyp {
namespace tile {

inline int setup(int& ctas, int& smem) {
  ctas = 0;
  smem = 0;
  return HYPERION_ERR_UNSUPPORTED;
}

inline int launch(const FwdParams&, int, int, int, cudaStream_t, int*) { return HYPERION_ERR_UNSUPPORTED; }

}  // namespace tile
}  // namespace hyp
