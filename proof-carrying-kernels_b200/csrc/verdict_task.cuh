// One block verdict: the decision rule of the reference checker
// (src/pck/cuda/csrc/checker_kernel.cu:146-184) evaluated by one warp from the partial sums
// the streaming kernel left, for (column b, check k, row block beta):
//   rho = cx - r . y_b[beta]                      cx = sum of the c . x_b segment partials
//   s   = sum of the a . |x_b| segment partials   (rounded up)
//   tau = coef*s + geps*((1+u32) s + sum |y_b[beta]|) + tau_floor   (rounded up)
//   passed = every y of the block finite && tau finite && |rho| <= tau
// Beyond the binary32 range of s the checked kernel's rounding model (no overflow) cannot
// hold, so tau is +inf and the block fails closed.
//
// The warp first issues every load it needs (y and r of the block, the segment partials) and
// only then adds, so a verdict costs one round trip to L2; the additions run in a fixed
// order: lane-strided per lane, then a shuffle tree for the y sums, and the segment
// partials in index order. Used by the verdict kernel and, for the checks of the previous
// launch, by the streaming kernel.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "verdict_plan.h"

namespace pck {
namespace verdict {

constexpr int kYPerLane = 8;  // y values (and signs) a lane holds per round: blocks of 256

__device__ __forceinline__ double shfl_sum_rn(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_down_sync(kFullMask, v, o));
  return v;
}

__device__ __forceinline__ double shfl_sum_ru(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_ru(v, __shfl_down_sync(kFullMask, v, o));
  return v;
}

// Adds the 32 values the lanes hold, in lane order, to `total` (every lane returns it).
template <bool kUp>
__device__ __forceinline__ double add_in_order(double total, double mine, int here) {
  for (int i = 0; i < here; ++i) {
    const double v = __shfl_sync(kFullMask, mine, i);
    total = kUp ? __dadd_ru(total, v) : __dadd_rn(total, v);
  }
  return total;
}

// Task t (in [0, vj.tasks)) of a verdict job, by a whole warp; y and the partial sums must
// be complete and visible (the caller has waited for the kernels that wrote them).
static __device__ __forceinline__ void run_task(const VerdictJob& vj, int64_t t, int lane) {
  const int64_t nb = vj.num_blocks;
  const int blk = vj.block;
  const int64_t beta = t % nb;
  const int k = static_cast<int>((t / nb) % vj.checks);
  const int b = static_cast<int>(t / (nb * vj.checks));
  const float* yb = vj.y + static_cast<int64_t>(b) * nb * blk + beta * blk;
  const int8_t* rk = vj.r + (static_cast<int64_t>(k) * nb + beta) * blk;
  const double* ps = vj.partial_s + (static_cast<int64_t>(b) * nb + beta) * vj.seg_alloc;
  const double* pcx = vj.partial_cx + ((static_cast<int64_t>(b) * vj.checks + k) * nb + beta) * vj.seg_alloc;

  double yabs = 0.0, ry = 0.0;
  bool bad = false;
  double s_mine = 0.0, cx_mine = 0.0;
  for (int base = 0; base < blk; base += kYPerLane * kWarp) {
    float yv[kYPerLane];
    int8_t rv[kYPerLane];
#pragma unroll
    for (int q = 0; q < kYPerLane; ++q) {
      const int i = base + q * kWarp + lane;
      yv[q] = i < blk ? __ldcg(yb + i) : 0.0f;
      rv[q] = i < blk ? __ldg(rk + i) : static_cast<int8_t>(1);
    }
    if (base == 0) {  // the first segment partials travel with the first round of y
      s_mine = lane < vj.segs ? __ldcg(ps + lane) : 0.0;
      cx_mine = lane < vj.segs ? __ldcg(pcx + lane) : 0.0;
    }
#pragma unroll
    for (int q = 0; q < kYPerLane; ++q) {
      if (base + q * kWarp + lane < blk) {
        const double v = static_cast<double>(yv[q]);
        bad |= !isfinite(yv[q]);
        yabs = __dadd_ru(yabs, fabs(v));
        ry = __dadd_rn(ry, rv[q] > 0 ? v : -v);
      }
    }
  }
  yabs = shfl_sum_ru(yabs);
  ry = shfl_sum_rn(ry);
  bad = __any_sync(kFullMask, bad);
  double s_total = add_in_order<true>(0.0, s_mine, min(kWarp, vj.segs));
  double cx = add_in_order<false>(0.0, cx_mine, min(kWarp, vj.segs));
  for (int s0 = kWarp; s0 < vj.segs; s0 += kWarp) {  // more than 32 segments
    const int here = min(kWarp, vj.segs - s0);
    s_total = add_in_order<true>(s_total, s0 + lane < vj.segs ? __ldcg(ps + s0 + lane) : 0.0, here);
    cx = add_in_order<false>(cx, s0 + lane < vj.segs ? __ldcg(pcx + s0 + lane) : 0.0, here);
  }

  if (lane == 0) {
    constexpr double kOnePlusU32 = 1.0 + 0x1p-24;
    constexpr double kFloatMax = 3.4028234663852886e38;
    const double rho = __dsub_rn(cx, ry);
    const double cabs = __dmul_ru(kOnePlusU32, s_total);
    const double eps = __dmul_ru(vj.geps, __dadd_ru(cabs, yabs));
    double tau = __dadd_ru(__dadd_ru(__dmul_ru(vj.coef, s_total), eps), vj.tau_floor);
    if (!(s_total <= kFloatMax)) tau = __longlong_as_double(0x7ff0000000000000LL);
    const int64_t o = (static_cast<int64_t>(b) * vj.checks + k) * nb + beta;
    vj.passed[o] = (!bad && isfinite(tau) && fabs(rho) <= tau) ? 1 : 0;
    vj.rho[o] = rho;
    vj.tau[o] = tau;
  }
}

// The job of plan task `task` (tasks numbered over the jobs in order), or -1 past the end.
__device__ __forceinline__ int job_of(const VerdictPlan& plan, int64_t task) {
  int j = 0;
  while (j + 1 < plan.njobs && task >= plan.jobs[j + 1].task_begin) ++j;
  const int64_t t = task - plan.jobs[j].task_begin;
  return t >= 0 && t < plan.jobs[j].tasks ? j : -1;
}

}  // namespace verdict
}  // namespace pck
