// Streaming kernel instantiations for bfloat16 weights (vectors of 8).
#include "stream_launch.cuh"

namespace pck {

cudaError_t launch_stream_bf16(const Plan& plan, int nv, int bg, bool tma, unsigned grid,
                               size_t smem, cudaStream_t stream) {
  return launch_format<kWeightsBf16>(plan, nv, bg, tma, grid, smem, stream);
}

PCK_STATUS_READER(status_stream_bf16)

}  // namespace pck
