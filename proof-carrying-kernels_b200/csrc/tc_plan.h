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
constexpr int kTcThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue, 6-9 bank
constexpr int kTcMaxChecks = 8;   // sign draws of a fused check
constexpr int kTcBankBytes = (kTcMaxChecks + 1) * kTcTileK * 8;  // a stage's bank rows in binary64
constexpr int kTcMaxBatch = 256;  // the MMA's largest N

struct TcJob {
  CUtensorMap w_map;  // W (m, n), box (64, 128), 128-byte swizzle
  CUtensorMap x_map;  // X (batch, n), box (64, n_pad), 128-byte swizzle
  float* Y;           // (batch, m)
  int64_t m;
  int64_t n;
  int32_t tile_begin;  // first tile of this job in the launch's tile sequence
  int32_t tiles;
  // fused check (has_check): a 128-row tile is one checker block; the bank rows of the block
  // are reduced against the staged X tiles into segment 0 of the partial sums
  const float* c;       // (checks, tiles, n)
  const uint16_t* a;    // (tiles, n) bfloat16
  double* partial_cx;   // (batch, checks, tiles, seg_alloc)
  double* partial_s;    // (batch, tiles, seg_alloc)
  int32_t has_check;
  int32_t checks;
  int32_t seg_alloc;
  int32_t reserved;
};

struct alignas(64) TcPlan {
  TcJob jobs[kTcMaxJobs];
  int32_t njobs;
  int32_t total_tiles;
  int32_t batch;   // columns of X and Y
  int32_t n_pad;   // batch rounded up to a multiple of 16 (the MMA's N)
  int32_t stages;      // shared-memory pipeline depth
  int32_t acc_stride;  // tensor-memory columns per accumulator: n_pad rounded up to 32
  int32_t tmem_cols;   // allocated columns: a power of two >= 2 * acc_stride
};

cudaError_t launch_tc(const TcPlan& plan, unsigned grid, size_t smem, cudaStream_t stream);
size_t tc_stage_bytes(int n_pad);
cudaError_t tc_status(unsigned int* value, bool clear);

}  // namespace pck
