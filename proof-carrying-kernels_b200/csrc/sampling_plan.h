// Arguments of the top-k / top-p set-check kernel (sampling_kernel.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace pck {

constexpr int kSamplingThreads = 512;
constexpr int kSamplingMaxCluster = 8;     // CTAs per row (portable cluster size)
constexpr size_t kSamplingSmemCap = 200 * 1024;  // bitmap of a slice plus the partials

struct SamplingArgs {
  const float* logits;      // (rows, vocab)
  const int64_t* selected;  // (rows, max_len)
  const int64_t* lengths;   // (rows,)
  int64_t rows;
  int64_t vocab;
  int64_t max_len;
  int64_t k;                // top-k: the selection length required
  int64_t slice;            // logits per CTA (a multiple of 32)
  int32_t top_p;
  int32_t reserved;
  double p;
  double temperature;
  double slack;
  uint8_t* passed;
  float* min_selected;
  float* max_rejected;
  double* mass;
  double* without;
};

size_t sampling_smem_bytes(int64_t slice);
cudaError_t launch_sampling_check(const SamplingArgs& args, int cluster, cudaStream_t stream);

}  // namespace pck
