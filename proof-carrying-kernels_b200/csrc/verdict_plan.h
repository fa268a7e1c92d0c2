// Launch plan of the verdict kernel (host and device view).
//
// The streaming kernel leaves, for every checked GEMV output, the binary64 partial sums of
// c . x_b and a . |x_b| per row block and column segment. The verdict kernel turns them
// into the decision of every (column b, check k, row block beta): one warp per triple,
// reading y as stored in memory after the producing kernels have finished.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace pck {

constexpr int kMaxVerdictJobs = 16;
constexpr int kVerdictThreads = 128;

struct VerdictJob {
  const float* y;             // (batch, num_blocks * block)
  const int8_t* r;            // (checks, num_blocks, block)
  const double* partial_cx;   // (batch, checks, num_blocks, seg_alloc)
  const double* partial_s;    // (batch, num_blocks, seg_alloc)
  uint8_t* passed;            // (batch, checks, num_blocks)
  double* rho;
  double* tau;
  int64_t task_begin;         // first task (warp) of this job
  int64_t tasks;              // batch * checks * num_blocks
  int32_t block;
  int32_t num_blocks;
  int32_t checks;
  int32_t segs;               // segments holding partial sums
  int32_t seg_alloc;          // segment stride of the partial-sum arrays
  int32_t batch;
  double coef;
  double geps;
  double tau_floor;
};

struct VerdictPlan {
  VerdictJob jobs[kMaxVerdictJobs];
  int32_t njobs;
};

cudaError_t launch_verdicts(const VerdictPlan& plan, int64_t tasks, cudaStream_t stream);

// Column segments of a bank row of n columns when the caller's scratch holds `segments`:
// about `target` columns each, a multiple of 8, at most `segments` of them. The streaming
// kernel writes exactly these partial sums and the verdict kernel reads them.
inline void segment_split(int64_t n, int64_t segments, int64_t target, int64_t* seg_len, int32_t* segs) {
  const int64_t want = segments < (n + target - 1) / target ? segments : (n + target - 1) / target;
  int64_t len = (n + want - 1) / want;
  len = (len + 7) / 8 * 8;
  *seg_len = len;
  *segs = static_cast<int32_t>((n + len - 1) / len);
}

}  // namespace pck
