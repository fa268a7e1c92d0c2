// Arguments of the membership-check kernel (member_kernel.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace pck {

constexpr int kLogitsF32 = 0;
constexpr int kLogitsBf16 = 1;
constexpr int kLogitsF16 = 2;

constexpr int kMemberThreads = 1024;     // one CTA per row
constexpr int kMemberCandidates = 8192;  // logits >= tau kept in shared memory

struct MemberArgs {
  const void* logits;     // (rows, row_stride) of dtype
  int64_t rows;
  int64_t vocab;
  int64_t row_stride;     // elements
  int32_t dtype;
  int32_t reserved;
  const int64_t* tokens;  // (rows,)
  const int64_t* top_k;   // (rows,) or NULL (no top-k)
  const double* top_p;    // (rows,) or NULL (no top-p)
  const uint8_t* greedy;  // (rows,) or NULL
  double slack;           // next_up(tol + member_eps32(vocab)), from the caller
  uint8_t* ok;
  int64_t* above;
  double* mass_above;
};

size_t member_smem_bytes();
cudaError_t launch_member_check(const MemberArgs& args, cudaStream_t stream);

}  // namespace pck
