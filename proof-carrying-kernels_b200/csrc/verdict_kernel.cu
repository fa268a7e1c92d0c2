// The verdict kernel: one warp per (column b, check k, row block beta), each running
// verdict::run_task (verdict_task.cuh, the decision rule of the reference checker,
// src/pck/cuda/csrc/checker_kernel.cu:146-184) once the producing kernels have finished.
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "verdict_plan.h"
#include "verdict_task.cuh"

namespace pck {
namespace {

constexpr int kWarpsPerCta = kVerdictThreads / kWarp;

__global__ void __launch_bounds__(kVerdictThreads) verdict_kernel(const __grid_constant__ VerdictPlan plan) {
  allow_dependents();
  const int lane = static_cast<int>(threadIdx.x) % kWarp;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + threadIdx.x / kWarp;
  const int j = verdict::job_of(plan, task);
  wait_for_producers();  // y and the partial sums come from the kernels before this one
  if (j < 0) return;     // uniform per warp
  verdict::run_task(plan.jobs[j], task - plan.jobs[j].task_begin, lane);
}

}  // namespace

cudaError_t launch_verdicts(const VerdictPlan& plan, int64_t tasks, cudaStream_t stream) {
  const int64_t blocks = (tasks + kWarpsPerCta - 1) / kWarpsPerCta;
  if (blocks < 1 || blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kVerdictThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, verdict_kernel, plan);
}

}  // namespace pck
