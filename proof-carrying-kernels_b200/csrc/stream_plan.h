// Launch plan of the persistent streaming kernel (host and device view).
//
// A launch processes up to kMaxPlanJobs jobs. A job is a GEMV over W (m, n) with
// activations X (batch, n) and outputs Y (batch, m), or the bank part of a check of one
// GEMV output (a checked GEMV is planned as one job of each kind, over the same X). Its work
// is a sequence of "units", each a contiguous byte range that the CTA's consumer warps
// reduce against the activations together:
//   - R consecutive W rows                         -> y[b, row] for every column b
//   - a segment of a checksum row c[k, beta, :]    -> partial c . x_b (binary64)
//   - a segment of a bound row a[beta, :]          -> partial a . |x_b| (binary64, up)
// For a check the units of row block beta are laid out contiguously:
//   [checks x segs c-units] [segs a-units]
// (the layout also admits a block's row units in front of them, which the host no longer
// plans). The segment units leave binary64 partial sums; the verdict kernel
// (verdict_plan.h) turns them, with y as stored, into the block decisions once this kernel
// has finished — or the next streaming launch does, as its `prior` verdicts: the CTAs from
// verdict_cta_begin on stream nothing; after griddepcontrol.wait (the previous kernels
// complete) their warps decide the prior launch's blocks while the other CTAs stream.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "verdict_plan.h"

namespace pck {

constexpr int kMaxJobs = 16;                 // GEMVs or checks a caller passes to one launch
constexpr int kMaxPlanJobs = 2 * kMaxJobs;   // a checked GEMV is planned as two jobs
constexpr int kConsumerWarps = 16;
constexpr int kTmaThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kPlainThreads = kConsumerWarps * 32;
constexpr int kMaxStages = 32;
constexpr int kSmemCap = 232448;  // 227 KB: the opt-in dynamic shared memory per CTA
constexpr int kMaxBatch = 16;
constexpr int kSegBatch = 4;  // staged path: batch columns of a checked job (more: plain path)
// Staged path: ring slots a warp fills before waiting for the producers. Deeper prefetch keeps
// HBM busy through the previous launch's tail but delays this launch's activation loads; it
// pays where the previous launch ends raggedly (launches with checks, whose bank and verdict
// CTAs finish early), so the host picks per launch (Plan::pre_slots).
constexpr int kPreSlotsPlain = 1;
constexpr int kPreSlotsChecked = 2;
constexpr int kWeightsBf16 = 0;
constexpr int kWeightsE4m3 = 1;

// Accumulators per batch column of a warp reducing a row: NV chains per lane.
__host__ __device__ constexpr int warp_accumulators(int /*wfmt*/, int nv) { return nv; }

struct JobPlan {
  // GEMV part (has_w): W (m, n); units of R rows.
  const void* W;
  const uint16_t* X;  // (batch, n) bfloat16 bits
  float* Y;           // (batch, m)
  int64_t m;
  int64_t n;
  int64_t row_bytes;  // n * element size
  int32_t batch;
  int32_t has_w;
  int32_t rows;       // R, rows per row unit
  int32_t row_units;  // row units per block (checked) or in total (unchecked)
  int32_t w_exp_min;  // smallest exponent field of a nonzero weight (1 for subnormals); 0 = unknown
  int32_t w_exp_max;  // largest exponent field of a weight; 0 = unknown
  // check part (has_check)
  int32_t has_check;
  int32_t block;
  int32_t num_blocks;
  int32_t checks;
  int32_t seg_alloc;  // segment stride of the scratch arrays
  int32_t segs;       // effective segments (seg_len-aligned)
  int32_t bank_settled;  // PCK_CHECK_BANK_SETTLED: bank pieces may be requested before the producer wait
  int64_t seg_len;    // columns per segment (multiple of 8)
  const float* c;
  const uint16_t* a;
  double* partial_cx;  // (batch, checks, num_blocks, seg_alloc)
  double* partial_s;   // (batch, num_blocks, seg_alloc)
  // partition
  int64_t units;         // total units
  int64_t period_units;  // units per row block (checked) or 1 (unchecked)
  int64_t period_bytes;  // bytes per period (checked)
  int64_t total_bytes;
  int32_t cta_begin;  // the job's CTAs (host bookkeeping; the kernel reads Plan::cta_units)
  int32_t cta_count;
};

constexpr int kMaxCtas = 320;  // grid limit of a streaming launch (2 per SM without staging)

__host__ __device__ __forceinline__ int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// First unit whose starting byte is >= target; units are partitioned between the CTAs of
// a job by their starting byte (the host fills Plan::cta_units with these boundaries).
__host__ __device__ __forceinline__ int64_t first_unit_at(const JobPlan& jb, int64_t target) {
  if (target <= 0) return 0;
  if (target >= jb.total_bytes) return jb.units;
  const int64_t unit_bytes = jb.rows * jb.row_bytes;
  if (!jb.has_check) return ceil_div64(target, unit_bytes);
  const int64_t beta = target / jb.period_bytes;
  int64_t rem = target - beta * jb.period_bytes;
  const int64_t base = beta * jb.period_units;
  if (rem == 0) return base;
  const int64_t ru = jb.has_w ? jb.row_units : 0;
  const int64_t wbytes = jb.has_w ? jb.block * jb.row_bytes : 0;
  if (rem <= wbytes) return base + ceil_div64(rem, unit_bytes);
  rem -= wbytes;
  const int64_t crow = 4 * jb.n;
  const int64_t cbytes = jb.checks * crow;
  if (rem <= cbytes) {
    const int64_t k = rem / crow;
    const int64_t r3 = rem - k * crow;
    return base + ru + k * jb.segs + ceil_div64(r3, 4 * jb.seg_len);
  }
  rem -= cbytes;
  return base + ru + static_cast<int64_t>(jb.checks) * jb.segs + ceil_div64(rem, 2 * jb.seg_len);
}

// A GEMV job of the launch that follows, whose first weight pieces this launch prefetches.
constexpr int kMaxPrefetchJobs = 16;
struct PrefetchJob {
  const uint8_t* W;
  int64_t row_bytes;
  int32_t bytes;  // prefetched from the start of each row (up to two row pieces)
  int32_t pad;
};

struct Plan {
  JobPlan jobs[kMaxPlanJobs];
  int32_t njobs;
  int32_t stages;       // staged path: ring slots per warp
  int32_t stage_bytes;  // staged path: bytes per slot
  int32_t x_bytes;
  int32_t threads;      // tree parameter T (all W jobs share it)
  int32_t sum_bytes;    // staged path: bytes per row piece (whole vector iterations)
  int32_t pre_slots;    // staged path: ring slots a warp fills before the producer wait
  int32_t verdict_cta_begin;  // CTAs [verdict_cta_begin, + verdict_ctas) decide `prior`
  int32_t verdict_ctas;       // (the grid's last CTAs; 0 and grid size: none)
  int64_t prior_tasks;        // verdict tasks of `prior`
  VerdictPlan prior;          // checks of an earlier launch decided by this one
  int2 cta_units[kMaxCtas];   // CTA c reduces units [x, y) of job cta_job[c]
  uint8_t cta_job[kMaxCtas];
  // The next launch's first pieces: CTA c of this launch, as its warps finish, prefetches into
  // L2 the first pieces of rows next_units[c].x + w (w = the warp) of next_jobs[next_job[c]],
  // the rows the next launch's CTA c starts with (255: nothing).
  int32_t next_ctas;
  PrefetchJob next_jobs[kMaxPrefetchJobs];
  int2 next_units[kMaxCtas];
  uint8_t next_job[kMaxCtas];
};

// Host-side launch of one instantiation family (stream_bf16.cu, stream_e4m3.cu). nv is
// threads / 32, bg the batch columns reduced together, tma the staged path.
cudaError_t launch_stream_bf16(const Plan& plan, int nv, int bg, bool tma, unsigned grid,
                               size_t smem, cudaStream_t stream);
cudaError_t launch_stream_e4m3(const Plan& plan, int nv, int bg, bool tma, unsigned grid,
                               size_t smem, cudaStream_t stream);

}  // namespace pck
