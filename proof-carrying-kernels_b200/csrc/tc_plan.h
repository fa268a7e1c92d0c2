// Launch plan of the tensor-core batched GEMV (tc_kernel.cu): Y (batch, m) = X (batch, n) W^T
// for bfloat16 W and X, binary32 accumulation in tensor memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace pck {

constexpr int kTcMaxJobs = 8;
constexpr int kTcTileM = 128;     // W rows per tile (the MMA's M)
constexpr int kTcTileK = 64;      // bfloat16 columns per pipeline stage (one 128-byte swizzle row)
constexpr int kTcThreads = 192;   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kTcMaxBatch = 256;  // the MMA's largest N

struct TcJob {
  CUtensorMap w_map;  // W (m, n), box (64, 128), 128-byte swizzle
  CUtensorMap x_map;  // X (batch, n), box (64, n_pad), 128-byte swizzle
  float* Y;           // (batch, m)
  int64_t m;
  int64_t n;
  int32_t tile_begin;  // first tile of this job in the launch's tile sequence
  int32_t tiles;
};

struct alignas(64) TcPlan {
  TcJob jobs[kTcMaxJobs];
  int32_t njobs;
  int32_t total_tiles;
  int32_t batch;   // columns of X and Y
  int32_t n_pad;   // batch rounded up to a multiple of 16 (the MMA's N)
  int32_t stages;      // shared-memory pipeline depth
  int32_t acc_stride;  // persistent form: tensor-memory columns per accumulator (n_pad up to 32s)
  int32_t tmem_cols;   // allocated columns: a power of two >= 2 * acc_stride (persistent) or n_pad
};

constexpr int kTcMaxSplits = 8;  // CTAs of a tile's cluster (K ranges), the portable cluster size

// splits == 1: the persistent kernel; else total_tiles * splits CTAs in clusters of `splits`
cudaError_t launch_tc(const TcPlan& plan, int splits, size_t smem, cudaStream_t stream);
size_t tc_stage_bytes(int n_pad);
cudaError_t tc_status(unsigned int* value, bool clear);

}  // namespace pck
