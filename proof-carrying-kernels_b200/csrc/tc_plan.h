// Launch plan of the tensor-core batched GEMV (tc_kernel.cu): Y (batch, m) = X (batch, n) W^T
// for bfloat16 X, bfloat16 or E4M3 W (E4M3 widened to bfloat16 in shared memory, exactly),
// binary32 accumulation in tensor memory, and optionally the binary64 checksum-bank sums of
// each job's blocked check reduced against the same staged X tiles.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace pck {

constexpr int kTcMaxJobs = 8;
constexpr int kTcTileM = 128;     // W rows per MMA (the MMA's M); one checker block when fused
constexpr int kTcTileK = 64;      // columns per pipeline stage (one 128-byte swizzle row of bfloat16)
constexpr int kTcMaxBatch = 256;  // the MMA's largest N
constexpr int kTcMaxUnitTiles = 2;  // 128-row tiles sharing one staged X tile (persistent form)
constexpr int kTcBankWarps = 8;     // binary64 bank warps, two per SM sub-partition (also widen E4M3)
constexpr int kTcThreads = 32 * (6 + kTcBankWarps);  // warp 0 TMA, 1 MMA, 2-5 epilogue, 6-13 bank
constexpr int kTcMaxChecks = 2;   // checks per job reduced inside the kernel (more: bank kernel)
constexpr int kTcFuseMaxBatch = 128;  // batches reduced inside the kernel (wider: bank kernel)
constexpr int kTcMaxSplits = 8;   // CTAs of a tile's cluster (K ranges), the portable cluster size
// Shared memory of the bank warps beyond the stages: per warp, the binary64 widening of the
// bank values its columns need in a stage (also, at the end of a work item, the area where the
// chunk groups' sums are combined).
constexpr int kTcBankWarpStage = kTcMaxUnitTiles * (kTcMaxChecks + 1) * 32;  // doubles per bank warp
constexpr int kTcCombDoubles = kTcMaxUnitTiles * (kTcMaxChecks + 1) * 2 * 32 * kTcBankWarps;
constexpr int kTcBankSmemBytes =
    8 * (kTcBankWarps * kTcBankWarpStage > kTcCombDoubles ? kTcBankWarps * kTcBankWarpStage : kTcCombDoubles);
constexpr int kTcWeightsBf16 = 0;
constexpr int kTcWeightsE4m3 = 1;

struct TcJob {
  CUtensorMap w_map;  // W (m, n): box (64, unit rows) of bfloat16 (128-byte swizzle) or E4M3 (none)
  CUtensorMap x_map;  // X (batch, n): box (64, n_pad), 128-byte swizzle
  float* Y;           // (batch, m)
  // fused check (fused != 0): bank rows of block beta = row / 128
  const float* c;     // (checks, nb, n) binary32
  const double* c64;  // the same widened to binary64, or NULL (then the bank warps widen c)
  const uint16_t* a;  // (nb, n) bfloat16, rounded up
  double* partial_cx;  // (batch, checks, nb, seg_alloc)
  double* partial_s;   // (batch, nb, seg_alloc)
  int64_t m;
  int64_t n;
  int32_t tile_begin;  // first 128-row tile of this job in the launch's tile sequence
  int32_t tiles;
  int32_t unit_begin;  // strided order: first unit of this job in the launch's unit sequence
  int32_t units;       // ceil(tiles / unit_tiles)
  int32_t fused;
  int32_t checks;
  int32_t nb;
  int32_t seg_alloc;
};

struct alignas(64) TcPlan {
  TcJob jobs[kTcMaxJobs];
  int32_t njobs;
  int32_t total_tiles;
  int32_t batch;       // columns of X and Y
  int32_t n_pad;       // batch rounded up to a multiple of 16 (the MMA's N)
  int32_t stages;      // shared-memory pipeline depth
  int32_t stage_bytes;  // W region + X region + bank region (+ raw E4M3 region), 1024-aligned
  int32_t w_bytes;      // bfloat16 W region of a stage: unit tiles * 16 KB
  int32_t x_bytes;      // X region: n_pad * 128
  int32_t bank_bytes;   // bank region: unit tiles * tile_bank_bytes (0 when nothing is fused)
  int32_t tile_bank_bytes;  // per tile: checks * 512 (c, binary64) or * 256 (binary32), + 128 (a)
  int32_t raw_bytes;    // E4M3 only: the raw weight bytes of a stage (unit tiles * 8 KB)
  int32_t acc_stride;   // tensor-memory columns per accumulator (n_pad up to 32s)
  int32_t acc_bufs;     // accumulator sets (1 or 2): the epilogue of one unit overlaps the next
  int32_t tmem_cols;    // allocated columns: a power of two >= acc_bufs * unit_tiles * acc_stride
  int32_t unit_tiles;   // persistent form: 128-row tiles per unit (1 or 2)
  int32_t any_fused;    // bank warps take part in the stages
  int32_t max_checks;   // largest `checks` of a fused job
  int32_t weights;      // kTcWeightsBf16 or kTcWeightsE4m3
  int32_t strided;      // persistent form: CTA c takes units c, c + grid, ... (else a contiguous
                        // range of tiles [c * total / grid, (c + 1) * total / grid), paired)
  int32_t total_units;
  int32_t settled;      // every job's W was written before the preceding kernel began: the
                        // first stages' W tiles are requested before the producer wait
};

// splits == 1: the persistent kernel over `grid` CTAs; else `grid` = total_units * splits CTAs
// in clusters of `splits` (K ranges of one unit of unit_tiles 128-row tiles).
cudaError_t launch_tc(const TcPlan& plan, int splits, int grid, size_t smem, cudaStream_t stream);
cudaError_t tc_status(unsigned int* value, bool clear);
// How many clusters of `splits` CTAs of the split form can run at once on the current device
// (0 if unknown): a split launch of more clusters would run in waves.
int tc_max_clusters(int splits);

}  // namespace pck
