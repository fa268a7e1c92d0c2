// Launch plan of the wide-batch bank kernel (bank_batch_kernel.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pck {

constexpr int kBankBatchJobs = 16;
constexpr int64_t kBankBatchSegment = 512;  // bank columns per segment the kernel aims for

struct BankBatchJob {
  const float* c;       // (checks, nb, n)
  const uint16_t* a;    // (nb, n) bfloat16
  const uint16_t* X;    // (batch, n) bfloat16
  double* partial_cx;   // (batch, checks, nb, seg_alloc)
  double* partial_s;    // (batch, nb, seg_alloc)
  int64_t n;
  int64_t seg_len;
  int32_t nb;
  int32_t checks;
  int32_t batch;
  int32_t seg_alloc;
  int32_t segs;
  int32_t tile_begin;   // first row tile: ceil(checks*nb / 32) c tiles, then ceil(nb / 32) a tiles
  int32_t c_tiles;
  int32_t a_tiles;
};

struct BankBatchPlan {
  BankBatchJob jobs[kBankBatchJobs];
  int32_t njobs;
  int32_t total_tiles;
};

// Segments of a bank row of n columns for this kernel: about kBankBatchSegment columns each,
// at most `segments` (the scratch's count) of them.
inline int32_t bank_batch_segments(int64_t n, int64_t segments, int64_t* seg_len) {
  int64_t want = (n + kBankBatchSegment - 1) / kBankBatchSegment;
  if (want > segments) want = segments;
  *seg_len = (n + want - 1) / want;
  return static_cast<int32_t>((n + *seg_len - 1) / *seg_len);
}

cudaError_t launch_bank_batch(const BankBatchPlan& plan, int col_groups, int max_segs, cudaStream_t stream);

}  // namespace pck
