// Tensor-core batched GEMV for decode batches: Y (batch, m) = X (batch, n) W^T with bfloat16 W
// and X and binary32 accumulation in tensor memory (tcgen05), for the batched decode path.
//
// The summation order is the tensor core's, not the reference's coalesced tree, so the result
// is not bit-exact to it; its checker uses the declared height of this accumulation (see
// pck.cuda.gemv.tc_height): each tcgen05.mma adds 16 exact products to the accumulator, at most
// n/16 of them in sequence per output.
//
// A 128-row tile of W is one thread-block cluster of `splits` CTAs (splits <= 8, chosen by
// the host so that small matrices still fill the GPU); CTA r of the cluster accumulates the
// r-th range of the tile's K blocks:
//   warp 0      one thread issues the TMA loads of a 128 x 64 tile of W and the n_pad x 64 tile
//               of X per stage (128-byte swizzle, the canonical K-major layout of the MMA);
//   warp 1      allocates the tensor memory, and one thread issues four 128 x n_pad x 16 MMAs
//               per stage, committing each stage back to the producer and the last to the
//               epilogue;
//   warps 2..5  copy the accumulator out of tensor memory (warp w reads lanes 32 (w % 4) ...)
//               into shared memory. After a cluster barrier, CTA r adds rows r*128/splits ...
//               of all the cluster's partial accumulators, in rank order (distributed shared
//               memory), and stores them as columns of Y.
// Every mbarrier wait is bounded; a wait that gives up records the status bit and the roles
// stop issuing work.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "tc_plan.h"

namespace cg = cooperative_groups;

namespace pck {
namespace {

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle: rows of 128 bytes,
// 8-row groups 1024 bytes apart (stride byte offset), version 1, layout type 2 (128B swizzle).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor: D binary32, A and B bfloat16, both K-major, N = n_pad, M = 128.
__device__ __forceinline__ uint32_t instr_desc(int n_pad) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n_pad >> 3) << 17) |
         (static_cast<uint32_t>(kTcTileM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ int job_of(const TcPlan& plan, int tile) {
  int j = 0;
  while (j + 1 < plan.njobs && tile >= plan.jobs[j + 1].tile_begin) ++j;
  return j;
}

// The persistent form (splits == 1 and many tiles): a CTA per SM walks the tiles with two
// tensor-memory accumulators, so the epilogue of one tile overlaps the main loop of the next.
__global__ void __launch_bounds__(kTcThreads, 1) tc_persistent_kernel(const __grid_constant__ TcPlan plan) {
  // The bank kernel that follows (launched as a programmatic dependent) reads nothing this
  // kernel writes, so it may start on the SMs this grid leaves free.
  allow_dependents();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const int stages = plan.stages;
  const uint32_t a_bytes = kTcTileM * 128u;
  const uint32_t b_bytes = static_cast<uint32_t>(plan.n_pad) * 128u;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = static_cast<int>(threadIdx.x) / kWarp;
  const int lane = static_cast<int>(threadIdx.x) % kWarp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      const uint64_t stream_policy = policy_evict_first();
      const uint64_t keep_policy = policy_evict_last();
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < plan.total_tiles; tile += gridDim.x) {
        const TcJob& jb = plan.jobs[job_of(plan, tile)];
        const int row0 = (tile - jb.tile_begin) * kTcTileM;
        const int kblocks = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % stages);
          if (!mbar_wait(empty + s, ((it / stages) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + static_cast<size_t>(s) * stage_bytes;
          mbar_arrive_expect_tx(full + s, stage_bytes);
          tma_load_2d(a_dst, &jb.w_map, full + s, kb * kTcTileK, row0, stream_policy);
          tma_load_2d(a_dst + a_bytes, &jb.x_map, full + s, kb * kTcTileK, 0, keep_policy);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = instr_desc(plan.n_pad);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < plan.total_tiles; tile += gridDim.x, ++local) {
        const TcJob& jb = plan.jobs[job_of(plan, tile)];
        const int kblocks = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
        const uint32_t acc = local & 1u;
        if (!mbar_wait(tempty + acc, ((local >> 1) & 1u) ^ 1u)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * static_cast<uint32_t>(plan.acc_stride);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = static_cast<int>(it % stages);
          if (!mbar_wait(full + s, (it / stages) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + static_cast<size_t>(s) * stage_bytes);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc = sw128_desc(a_addr + a_bytes);
#pragma unroll
          for (int k = 0; k < kTcTileK / 16; ++k) {  // 16 bfloat16 = 32 bytes = 2 descriptor units
            umma_bf16(d, adesc + 2u * k, bdesc + 2u * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty + s);  // the stage is free once these MMAs have read it
        }
        if (ok) umma_commit(tfull + acc);
      }
    }
  } else {  // epilogue warps 2..5
    const int quarter = warp % 4;
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < plan.total_tiles; tile += gridDim.x, ++local) {
      const TcJob& jb = plan.jobs[job_of(plan, tile)];
      const uint32_t acc = local & 1u;
      if (!mbar_wait(tfull + acc, (local >> 1) & 1u)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tile - jb.tile_begin) * kTcTileM + quarter * 32 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * static_cast<uint32_t>(plan.acc_stride);
      for (int c0 = 0; c0 < plan.n_pad; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(base + static_cast<uint32_t>(c0), v);
        if (row < jb.m) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (c0 + i < plan.batch) jb.Y[static_cast<int64_t>(c0 + i) * jb.m + row] = __uint_as_float(v[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
  }
}

// The split form: one tile per cluster of `splits` CTAs, each a range of the tile's K blocks.
__global__ void __launch_bounds__(kTcThreads, 1) tc_split_kernel(const __grid_constant__ TcPlan plan) {
  allow_dependents();  // as in tc_persistent_kernel
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  cg::cluster_group cluster = cg::this_cluster();
  const int splits = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int stages = plan.stages;
  const uint32_t a_bytes = kTcTileM * 128u;
  const uint32_t b_bytes = static_cast<uint32_t>(plan.n_pad) * 128u;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * stage_bytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  // After the main loop the stages hold the partial accumulator: 128 rows of n_pad + 1 words
  // (the extra word keeps the rows of a warp in different banks).
  float* part = reinterpret_cast<float*>(smem);
  const int pstride = plan.n_pad + 1;
  const int warp = static_cast<int>(threadIdx.x) / kWarp;
  const int lane = static_cast<int>(threadIdx.x) % kWarp;

  const int tile = static_cast<int>(blockIdx.x) / splits;
  const TcJob& jb = plan.jobs[job_of(plan, tile)];
  const int row0 = (tile - jb.tile_begin) * kTcTileM;
  const int kblocks = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
  const int kper = (kblocks + splits - 1) / splits;
  const int kb0 = min(kblocks, rank * kper);
  const int kb1 = min(kblocks, kb0 + kper);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(tfull, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      const uint64_t stream_policy = policy_evict_first();
      const uint64_t keep_policy = policy_evict_last();
      uint32_t it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = static_cast<int>(it % stages);
        if (!mbar_wait(empty + s, ((it / stages) & 1u) ^ 1u)) break;
        uint8_t* a_dst = smem + static_cast<size_t>(s) * stage_bytes;
        mbar_arrive_expect_tx(full + s, stage_bytes);
        tma_load_2d(a_dst, &jb.w_map, full + s, kb * kTcTileK, row0, stream_policy);
        tma_load_2d(a_dst + a_bytes, &jb.x_map, full + s, kb * kTcTileK, 0, keep_policy);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = instr_desc(plan.n_pad);
      uint32_t it = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = static_cast<int>(it % stages);
        if (!mbar_wait(full + s, (it / stages) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_addr(smem + static_cast<size_t>(s) * stage_bytes);
        const uint64_t adesc = sw128_desc(a_addr);
        const uint64_t bdesc = sw128_desc(a_addr + a_bytes);
#pragma unroll
        for (int k = 0; k < kTcTileK / 16; ++k) {  // 16 bfloat16 = 32 bytes = 2 descriptor units
          umma_bf16(tmem, adesc + 2u * k, bdesc + 2u * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(empty + s);  // the stage is free once these MMAs have read it
      }
      if (ok && kb1 > kb0) umma_commit(tfull);
    }
  } else {  // epilogue warps 2..5: the partial accumulator into shared memory
    const int quarter = warp % 4;
    const int lrow = quarter * 32 + lane;
    const bool have = __all_sync(kFullMask, kb1 > kb0 && mbar_wait(tfull, 0));  // uniform per warp
    tc_fence_after();
    for (int c0 = 0; c0 < plan.n_pad; c0 += 32) {
      uint32_t v[32];
      if (have) tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c0), v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (c0 + i < plan.n_pad) part[lrow * pstride + c0 + i] = have ? __uint_as_float(v[i]) : 0.0f;
      }
    }
  }
  __syncwarp();  // the roles' lane 0 rejoins its warp before the cluster barrier
  tc_fence_before();
  cluster.sync();  // every CTA's partial is in its shared memory

  if (warp >= 2) {  // rows [rank * R, (rank + 1) * R) of the tile, summed over the cluster
    const int R = kTcTileM / splits;
    const int t = static_cast<int>(threadIdx.x) - 2 * kWarp;  // 0..127
    for (int idx = t; idx < R * plan.batch; idx += 4 * kWarp) {
      const int r = rank * R + idx % R;
      const int col = idx / R;
      float sum = 0.0f;
      for (int c = 0; c < splits; ++c) {
        const float* peer = cluster.map_shared_rank(part, c);
        const float v = peer[r * pstride + col];
        sum = c == 0 ? v : __fadd_rn(sum, v);
      }
      const int64_t row = static_cast<int64_t>(row0) + r;
      if (row < jb.m) jb.Y[static_cast<int64_t>(col) * jb.m + row] = sum;
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its partial
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
  }
}

}  // namespace

PCK_STATUS_READER(tc_status)

size_t tc_stage_bytes(int n_pad) { return static_cast<size_t>(kTcTileM) * 128 + static_cast<size_t>(n_pad) * 128; }

cudaError_t launch_tc(const TcPlan& plan, int splits, size_t smem, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    for (auto* fn : {tc_persistent_kernel, tc_split_kernel}) {
      const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      if (err != cudaSuccess) return err;
    }
    configured[dev] = 1;
  }
  if (splits <= 1) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const unsigned grid = static_cast<unsigned>(plan.total_tiles < sms ? plan.total_tiles : sms);
    tc_persistent_kernel<<<grid, kTcThreads, smem, stream>>>(plan);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.total_tiles) * static_cast<unsigned>(splits));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tc_split_kernel, plan);
}

}  // namespace pck
