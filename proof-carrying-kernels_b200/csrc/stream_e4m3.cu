// Streaming kernel instantiations for E4M3 weights (vectors of 16).
#include "stream_launch.cuh"

namespace pck {

cudaError_t launch_stream_e4m3(const Plan& plan, int nv, int bg, bool tma, unsigned grid,
                               size_t smem, cudaStream_t stream) {
  return launch_format<kWeightsE4m3>(plan, nv, bg, tma, grid, smem, stream);
}

PCK_STATUS_READER(status_stream_e4m3)

}  // namespace pck
