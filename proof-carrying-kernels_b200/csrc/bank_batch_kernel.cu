// Checksum-bank partial sums for a wide decode batch (the checks of the tensor-core GEMV):
// for every bank row (c[k, beta, :] or a[beta, :]), column b of X and column segment s,
//   partial_cx[b, k, beta, s] = sum over the segment of c[k, beta, j] x[b, j]    (binary64)
//   partial_s [b, beta, s]    = sum over the segment of a[beta, j] |x[b, j]|     (rounded up)
// with exact products (binary32 x bfloat16 and bfloat16 x bfloat16 are exact in binary64).
//
// This is a small binary64 matrix product, bank rows x batch columns, done on the CUDA cores:
// a CTA takes 32 bank rows of one kind, 32 batch columns and one segment, and widens 32
// columns j of the rows and of X to binary64 in shared memory at a time (the global loads of
// the next round are in flight meanwhile). Its 256 threads form four groups of 64; group g
// takes the columns j = 8g .. 8g+7 of every round, and each thread accumulates 4 rows x 4
// batch columns (rows 4ty + i, columns tx + 8q) over them, j ascending: 8 shared loads per 16
// binary64 FMAs. At the end the four group sums of every output are added in group order
// (rounded up for bound rows), a fixed order like the rest; the binary64 bound holds for any
// split of a segment no deeper than its serial sum. The verdict kernel (verdict_kernel.cu)
// adds the segments and decides the blocks.
//
// It is launched as a programmatic dependent of the tensor-core kernel, whose outputs it
// does not read (its inputs, X and the bank, were final before that kernel started), so its
// CTAs may run beside it on free SMs. Every CTA waits for that kernel before it exits: the
// bank grid completes only after the GEMV, so the verdict kernel's wait covers both.
#include <cuda_runtime.h>

#include <cstdint>

#include "bank_batch_plan.h"
#include "pck_common.cuh"

namespace pck {
namespace {

constexpr int kRows = 32;   // bank rows per CTA
constexpr int kCols = 32;   // batch columns per CTA
constexpr int kChunk = 32;  // columns of the bank (j) per shared-memory round
constexpr int kGroups = 4;  // thread groups splitting a round's columns
constexpr int kPerGroup = kChunk / kGroups;

// One round's raw values: each thread fetches 4 bank values (rows t/32 + 8i, column t%32)
// and 4 activations (batch columns t/32 + 8i), fetched a round ahead of their use.
struct Round {
  uint32_t row[4];
  uint16_t x[4];
};

__device__ __forceinline__ void fetch_round(const BankBatchJob& jb, bool bound, int64_t nrows, int64_t row0,
                                            int b0, int64_t jc, int64_t j1, int t, Round& rd) {
  const int jj = t % kChunk;
  const int64_t col = jc + jj;
  const bool in = col < j1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + t / kChunk + 8 * i;
    rd.row[i] = 0u;
    if (in && row < nrows) {
      rd.row[i] = bound ? static_cast<uint32_t>(__ldg(jb.a + row * jb.n + col))
                        : __float_as_uint(__ldg(jb.c + row * jb.n + col));
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int b = b0 + t / kChunk + 8 * i;
    rd.x[i] = (in && b < jb.batch) ? __ldg(jb.X + static_cast<int64_t>(b) * jb.n + col) : static_cast<uint16_t>(0);
  }
}

__global__ void __launch_bounds__(256) bank_batch_kernel(const __grid_constant__ BankBatchPlan plan) {
  // one padding word per line: the 32 lanes of a warp store one bank column j each
  __shared__ double rows_s[kChunk][kRows + 1];
  __shared__ double x_s[kChunk][kCols + 1];
  __shared__ double red[kGroups - 1][kRows][kCols + 1];  // sums of groups 1..3
  int j = 0;
  while (j + 1 < plan.njobs && static_cast<int>(blockIdx.x) >= plan.jobs[j + 1].tile_begin) ++j;
  const BankBatchJob& jb = plan.jobs[j];
  const int tile = static_cast<int>(blockIdx.x) - jb.tile_begin;
  const int seg = static_cast<int>(blockIdx.z);
  if (seg >= jb.segs) {  // uniform
    wait_for_producers();
    return;
  }
  const bool bound = tile >= jb.c_tiles;  // a rows: |x|, rounded up
  const int64_t nrows = bound ? jb.nb : static_cast<int64_t>(jb.checks) * jb.nb;
  const int64_t row0 = static_cast<int64_t>(bound ? tile - jb.c_tiles : tile) * kRows;
  const int b0 = static_cast<int>(blockIdx.y) * kCols;
  if (b0 >= jb.batch) {
    wait_for_producers();
    return;
  }
  const int64_t j0 = static_cast<int64_t>(seg) * jb.seg_len;
  const int64_t j1 = min(jb.n, j0 + jb.seg_len);
  const int t = static_cast<int>(threadIdx.x);
  const int grp = t / 64, u = t % 64;
  const int ty = u / 8, tx = u % 8;  // rows 4ty + i, columns tx + 8q (i, q < 4)
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[i][q] = 0.0;
  }
  Round rd;
  fetch_round(jb, bound, nrows, row0, b0, j0, j1, t, rd);
  for (int64_t jc = j0; jc < j1; jc += kChunk) {
    const int jj = t % kChunk;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rows_s[jj][t / kChunk + 8 * i] = bound ? static_cast<double>(bf16_bits_to_float(static_cast<uint16_t>(rd.row[i])))
                                             : static_cast<double>(__uint_as_float(rd.row[i]));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const double xv = static_cast<double>(bf16_bits_to_float(rd.x[i]));
      x_s[jj][t / kChunk + 8 * i] = bound ? fabs(xv) : xv;
    }
    __syncthreads();
    if (jc + kChunk < j1) fetch_round(jb, bound, nrows, row0, b0, jc + kChunk, j1, t, rd);  // next round in flight
#pragma unroll
    for (int kk = 0; kk < kPerGroup; ++kk) {
      const int k = grp * kPerGroup + kk;
      double rv[4], xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rv[i] = rows_s[k][4 * ty + i];
#pragma unroll
      for (int q = 0; q < 4; ++q) xv[q] = x_s[k][tx + 8 * q];
      if (bound) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[i][q] = __fma_ru(rv[i], xv[q], acc[i][q]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[i][q] = __fma_rn(rv[i], xv[q], acc[i][q]);
        }
      }
    }
    __syncthreads();
  }
  // Groups 1..3 hand their sums to group 0, which adds them in group order.
  if (grp > 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int q = 0; q < 4; ++q) red[grp - 1][4 * ty + i][tx + 8 * q] = acc[i][q];
    }
  }
  __syncthreads();
  if (grp > 0) {
    wait_for_producers();
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + 4 * ty + i;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      double v = acc[i][q];
#pragma unroll
      for (int g = 0; g < kGroups - 1; ++g) {
        v = bound ? __dadd_ru(v, red[g][4 * ty + i][tx + 8 * q]) : __dadd_rn(v, red[g][4 * ty + i][tx + 8 * q]);
      }
      const int b = b0 + tx + 8 * q;
      if (row >= nrows || b >= jb.batch) continue;
      if (bound) {
        jb.partial_s[(static_cast<int64_t>(b) * jb.nb + row) * jb.seg_alloc + seg] = v;
      } else {
        // row = k * nb + beta, and partial_cx is (batch, checks, nb, seg_alloc)
        jb.partial_cx[(static_cast<int64_t>(b) * jb.checks * jb.nb + row) * jb.seg_alloc + seg] = v;
      }
    }
  }
  wait_for_producers();
}

}  // namespace

cudaError_t launch_bank_batch(const BankBatchPlan& plan, int col_groups, int max_segs, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(plan.total_tiles), static_cast<unsigned>(col_groups),
                  static_cast<unsigned>(max_segs));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, bank_batch_kernel, plan);
}

}  // namespace pck
