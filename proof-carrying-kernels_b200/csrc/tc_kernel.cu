// Tensor-core batched GEMV for decode batches: Y (batch, m) = X (batch, n) W^T with bfloat16 X,
// bfloat16 or E4M3 W (E4M3 widened exactly to bfloat16 in shared memory) and binary32
// accumulation in tensor memory (tcgen05), with the binary64 checksum-bank sums of each job's
// blocked check reduced in the same pass over the staged X tiles.
//
// The summation order is the tensor core's, not the reference's coalesced tree, so the result
// is not bit-exact to it; its checker uses the declared height of this accumulation (see
// pck.cuda.gemv.tc_height): each tcgen05.mma adds 16 exact products to the accumulator, at most
// n/16 of them in sequence per output.
//
// Work is a sequence of 128-row tiles of W (one checker block each when the check is fused).
// Two forms share the kernel body:
//   persistent  a CTA per SM takes a contiguous range of the launch's tiles and walks it in
//               units of up to two tiles of one job, which share every staged X tile (two
//               MMAs per K step, two accumulators): X crosses L2 once per 256 rows of W;
//   split       a unit of one or two tiles per cluster of `splits` CTAs (2 to 8); CTA r
//               accumulates the r-th of `splits` near-equal ranges of the K blocks, and the
//               partial accumulators are added in rank order through distributed shared
//               memory (for launches with few tiles).
// Roles (14 warps):
//   warp 0      one thread issues, per stage, the TMA loads of the unit's W tiles (128 rows x
//               64 columns each; bfloat16 with 128-byte swizzle, or raw E4M3 bytes) and of the
//               n_pad x 64 X tile, and the bulk copies of the fused checks' bank rows;
//   warp 1      allocates tensor memory; one thread issues four 128 x n_pad x 16 MMAs per tile
//               and stage and commits each stage back to the producer, each unit to the epilogue;
//   warps 2..5  copy the accumulators out of tensor memory (warp w reads lanes 32 (w % 4) ...)
//               into Y (persistent) or into shared memory for the cluster sum (split);
//   warps 6..13 the bank warps: widen E4M3 tiles to bfloat16 for the MMA, and for fused checks
//               reduce the stage's bank rows against the stage's X tile — c . x in binary64
//               rounded to nearest (binary32 x bfloat16 products are exact in binary64),
//               a . |x| in binary32 rounded up (bfloat16 x bfloat16 products are exact in
//               binary32) — into the checks' partial sums: one segment per tile (persistent)
//               or per K range (split).
// A stage is released to the producer once the MMAs have read it (tcgen05.commit) and every
// bank warp is done with it. Every mbarrier wait is bounded; a wait that gives up records the
// status bit and the roles stop issuing work.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "tc_plan.h"

namespace cg = cooperative_groups;

namespace pck {
namespace {

constexpr uint32_t kTileBf16Bytes = kTcTileM * 128u;  // one 128 x 64 bfloat16 tile
constexpr uint32_t kTileE4m3Bytes = kTcTileM * 64u;   // one 128 x 64 E4M3 tile
constexpr int kBankThreads = 32 * kTcBankWarps;

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

// Shared-memory writes of this thread become visible to the tensor core (the async proxy).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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

// The address of the same shared-memory location in the CTA of rank `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void lds_f64x2(uint32_t addr, double& a, double& b) {
  asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(a), "=d"(b) : "r"(addr));
}

__device__ __forceinline__ void lds_f64x2_one(uint32_t addr, double& a) {
  asm volatile("ld.shared.f64 %0, [%1];" : "=d"(a) : "r"(addr));
}

__device__ __forceinline__ void sts_f64(uint32_t addr, double v) {
  asm volatile("st.shared.f64 [%0], %1;" ::"r"(addr), "d"(v) : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Two E4M3 values (low byte first) to two bfloat16 in one word, exactly: E4M3 -> binary16 is
// exact, binary16 -> binary32 is exact, and a value of at most 4 significant bits in the
// E4M3 range rounds to itself in bfloat16.
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t pair) {
  uint32_t h2, out;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(pair)));
  asm("{\n\t.reg .b16 l, h;\n\t.reg .f32 fl, fh;\n\tmov.b32 {l, h}, %1;\n\tcvt.f32.f16 fl, l;\n\t"
      "cvt.f32.f16 fh, h;\n\tcvt.rn.bf16x2.f32 %0, fh, fl;\n\t}"
      : "=r"(out)
      : "r"(h2));
  return out;
}

__device__ __forceinline__ int job_of(const TcPlan& plan, int tile) {
  int j = 0;
  while (j + 1 < plan.njobs && tile >= plan.jobs[j + 1].tile_begin) ++j;
  return j;
}

// One item of a CTA's work: `ntiles` consecutive 128-row tiles of one job (from job-local
// tile `tile`), over the K blocks [kb0, kb1); its bank sums go to segment `seg`.
struct Work {
  int job;
  int tile;
  int ntiles;
  int kb0;
  int kb1;
  int seg;
};

// A role's position in the stage ring: slot and the parity of its current pass, stepped
// without divisions (the stage count is a launch parameter).
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// The work sequence of a CTA; every role walks the same one.
struct WorkWalk {
  int cur;
  int end;
  bool split;
};

__device__ __forceinline__ WorkWalk work_start(const TcPlan& plan, bool split) {
  WorkWalk w;
  w.split = split;
  if (split) {
    w.cur = 0;
    w.end = 1;
  } else if (plan.strided) {
    w.cur = static_cast<int>(blockIdx.x);  // a unit index, stepping by the grid
    w.end = plan.total_units;
  } else {
    const int64_t total = plan.total_tiles, g = gridDim.x, c = blockIdx.x;
    w.cur = static_cast<int>(c * total / g);
    w.end = static_cast<int>((c + 1) * total / g);
  }
  return w;
}

__device__ __forceinline__ bool work_next(const TcPlan& plan, WorkWalk& w, Work& out) {
  if (w.cur >= w.end) return false;
  if (w.split) {
    // cluster u takes unit u (up to unit_tiles tiles of one job); its CTA of rank r takes the
    // r-th of `splits` near-equal ranges of the K blocks
    cg::cluster_group cluster = cg::this_cluster();
    const int splits = static_cast<int>(cluster.num_blocks());
    const int rank = static_cast<int>(cluster.block_rank());
    const int unit = static_cast<int>(blockIdx.x) / splits;
    int j = 0;
    while (j + 1 < plan.njobs && unit >= plan.jobs[j + 1].unit_begin) ++j;
    const TcJob& jb = plan.jobs[j];
    out.job = j;
    out.tile = (unit - jb.unit_begin) * plan.unit_tiles;
    out.ntiles = min(plan.unit_tiles, jb.tiles - out.tile);
    const int kblocks = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
    out.kb0 = rank * kblocks / splits;
    out.kb1 = (rank + 1) * kblocks / splits;
    out.seg = rank;
    w.cur = 1;
    return true;
  }
  if (plan.strided) {
    int j = 0;
    while (j + 1 < plan.njobs && w.cur >= plan.jobs[j + 1].unit_begin) ++j;
    const TcJob& jb = plan.jobs[j];
    out.job = j;
    out.tile = (w.cur - jb.unit_begin) * plan.unit_tiles;
    out.ntiles = min(plan.unit_tiles, jb.tiles - out.tile);
    out.kb0 = 0;
    out.kb1 = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
    out.seg = 0;
    w.cur += static_cast<int>(gridDim.x);
    return true;
  }
  out.job = job_of(plan, w.cur);
  const TcJob& jb = plan.jobs[out.job];
  out.tile = w.cur - jb.tile_begin;
  out.ntiles = (plan.unit_tiles > 1 && w.cur + 1 < w.end && out.tile + 1 < jb.tiles) ? 2 : 1;
  out.kb0 = 0;
  out.kb1 = static_cast<int>((jb.n + kTcTileK - 1) / kTcTileK);
  out.seg = 0;
  w.cur += out.ntiles;
  return true;
}


// ---------------------------------------------------------------------------------------------
// Bank warps

// Which batch columns and which 16-byte chunks of a stage's X rows a bank thread reduces. The
// 256 bank threads form `nsplit` groups of `group` threads, group g taking chunks
// [8g / nsplit, 8(g + 1) / nsplit) of every column. Up to 32 columns: one column per thread
// (group 32, 8 groups); more: two columns c and c + group per thread (group = the batch
// rounded up to 64, 128 or 256, halved), so each widened bank value serves two columns. A
// group is whole warps, so the chunks of a warp are uniform. The group sums are added in
// group order at the end of a work item.
struct BankLanes {
  int col[2];  // batch columns, -1 for none
  int ch0;
  int ch1;
  int split;
  int nsplit;
  int group;
};

__device__ __forceinline__ BankLanes bank_lanes(int batch, int bt) {
  BankLanes L;
  if (batch <= 32) {
    L.group = 32;
    L.col[0] = bt % 32 < batch ? bt % 32 : -1;
    L.col[1] = -1;
  } else {
    L.group = (batch <= 64 ? 64 : batch <= 128 ? 128 : 256) / 2;
    const int c = bt % L.group;
    L.col[0] = c < batch ? c : -1;
    L.col[1] = c + L.group < batch ? c + L.group : -1;
  }
  L.nsplit = kBankThreads / L.group;
  L.split = bt / L.group;
  const int per = 8 / L.nsplit;
  L.ch0 = L.split * per;
  L.ch1 = L.ch0 + per;
  return L;
}

// The stage's raw E4M3 tiles widened to bfloat16 in the 128-byte-swizzled K-major layout the
// MMA reads (16-byte chunk c of row r at chunk c ^ (r % 8) of the row), then made visible to
// the tensor core.
__device__ __forceinline__ void widen_stage(const TcPlan& plan, int ntiles, uint8_t* stage, int bt) {
  const uint32_t raw = smem_addr(stage + plan.w_bytes + plan.x_bytes + plan.bank_bytes);
  const uint32_t wbase = smem_addr(stage);
  const int items = ntiles * kTcTileM * 8;  // 8 bytes of one row each
  for (int i = bt; i < items; i += kBankThreads) {
    const int t = i >> 10, r = (i >> 3) & (kTcTileM - 1), ch = i & 7;
    const uint2 q = lds64(raw + static_cast<uint32_t>(t) * kTileE4m3Bytes + static_cast<uint32_t>(r * 64 + ch * 8));
    uint4 o;
    o.x = e4m3x2_to_bf16x2(q.x & 0xFFFFu);
    o.y = e4m3x2_to_bf16x2(q.x >> 16);
    o.z = e4m3x2_to_bf16x2(q.y & 0xFFFFu);
    o.w = e4m3x2_to_bf16x2(q.y >> 16);
    sts128(wbase + static_cast<uint32_t>(t) * kTileBf16Bytes + static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4)), o);
  }
  fence_proxy_async();
}

// Running sums of a bank thread over a work item, per column: c . x per (tile, check) in
// binary64 rounded to nearest, a . |x| per tile in binary32 rounded up, each as kPartials
// interleaved partial sums (column j to partial j % kPartials), added in order at the end.
// The bound sum needs no binary64: a (bfloat16) times |x| (bfloat16) is exact in binary32,
// and a sum of non-negative terms rounded up at every step is never below the exact sum, so
// it is an upper bound as the verdict rule requires (inflated by at most a relative
// (1 + 2^-23)^h - 1 for a chain of h additions; an overflow gives +inf and fails the block).
// Both bounds hold for any split of a sum.
constexpr int kPartials = 2;
template <int kK>  // checks per job reduced by the bank warps (1 or 2)
struct BankSums {
  double cx[2][kTcMaxUnitTiles][kK][kPartials];
  float sx[2][kTcMaxUnitTiles][kPartials];
};

template <int kK>
__device__ __forceinline__ void bank_zero(BankSums<kK>& a) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
#pragma unroll
    for (int t = 0; t < kTcMaxUnitTiles; ++t) {
#pragma unroll
      for (int p = 0; p < kPartials; ++p) {
        a.sx[c][t][p] = 0.0f;
#pragma unroll
        for (int k = 0; k < kK; ++k) a.cx[c][t][k][p] = 0.0;
      }
    }
  }
}

// What the bank warps need of a work item, read from the launch parameters once per item.
struct BankItem {
  int fused;
  int checks;
  int ntiles;
  int c64;           // binary64 checksums staged by the producer: no widening
  int cstride;       // bytes per checksum row of a stage's bank region
  int tile_bytes;    // bank bytes per tile of a stage
  int last_kb;       // the row's last K block, and its columns (a multiple of 8)
  int last_cols;
  uint32_t x_off;    // the X tile and the bank region within a stage
  uint32_t bank_off;
};

__device__ __forceinline__ BankItem bank_item(const TcPlan& plan, const TcJob& jb, const Work& wk) {
  BankItem it;
  it.fused = jb.fused;
  it.checks = jb.checks;
  it.ntiles = wk.ntiles;
  it.c64 = jb.c64 != nullptr;
  it.cstride = it.c64 ? 512 : 256;
  it.tile_bytes = plan.tile_bank_bytes;
  it.last_kb = static_cast<int>((jb.n - 1) / kTcTileK);
  it.last_cols = static_cast<int>(jb.n - static_cast<int64_t>(it.last_kb) * kTcTileK);
  it.x_off = static_cast<uint32_t>(plan.w_bytes);
  it.bank_off = static_cast<uint32_t>(plan.w_bytes + plan.x_bytes);
  return it;
}

// One stage of the fused check for one bank warp (`jmax` columns of the stage are valid).
// Without binary64 checksums in the stage, the warp widens to binary64 the checksum values its
// chunks need (rows c[k] of each tile of the unit, zeros past the end of the row) into its own
// staging buffer at shared address `wstg` ([tile][check][32 columns j]). Then each thread,
// chunk by chunk: its columns' 8 activations (binary64 for c . x, binary32 |x| for the bound),
// and per tile 4 two-value shared loads per check serving 8 binary64 FMAs per column, and one
// 16-byte load of 8 bound values serving 8 binary32 FMAs per column. Only the warp
// synchronizes; every access names the shared space.
template <int kK>
__device__ __forceinline__ void bank_stage(const BankItem& item, int jmax, const uint8_t* stage, uint32_t wstg,
                                           const BankLanes& L, int lane, BankSums<kK>& acc) {
  const int K = item.checks;
  const int ntiles = item.ntiles;
  const uint32_t bank = smem_addr(stage) + item.bank_off;
  const int j0 = L.ch0 * 8, jn = (L.ch1 - L.ch0) * 8;  // at most 32 columns j
  const bool c64 = item.c64 != 0;
  const int cstride = item.cstride;
  __syncwarp();  // the previous stage's reads of the buffer are done
  if (!c64 && lane < jn) {  // lane jj widens column j0 + jj of every checksum row of the unit
    const int j = j0 + lane;
#pragma unroll
    for (int t = 0; t < kTcMaxUnitTiles; ++t) {
      if (t >= ntiles) break;
      const uint32_t tb = bank + static_cast<uint32_t>(t * item.tile_bytes);
      const uint32_t dst = wstg + static_cast<uint32_t>((t * kTcMaxChecks * 32 + lane) * 8);
#pragma unroll
      for (int r = 0; r < kTcMaxChecks; ++r) {
        if (r >= K) break;
        const double v = j < jmax ? static_cast<double>(__uint_as_float(lds32(tb + static_cast<uint32_t>(r * 256 + j * 4))))
                                  : 0.0;
        sts_f64(dst + static_cast<uint32_t>(r * 32 * 8), v);
      }
    }
  }
  __syncwarp();
  if (L.col[0] < 0) return;
  const uint32_t xs = smem_addr(stage) + item.x_off;
  const bool two = L.col[1] >= 0;
  const uint32_t rstride = c64 ? 512u : 256u;  // bytes between checksum rows of a chunk
  // tiles whose checksum loads are issued together (as many as the registers hold)
  constexpr int kPre = kK == 1 ? kTcMaxUnitTiles : 1;
  for (int ch = L.ch0; ch < L.ch1 && ch * 8 < jmax; ++ch) {  // jmax is a multiple of 8
    // The shared-memory loads first (the tensor core and TMA keep shared memory busy, so each
    // round trip is long): the columns' 8 activations, and per tile the 8 binary64 checksums
    // of each check (in the stage itself, or in the warp's widened copy) and the 8 bfloat16
    // bound values.
    uint4 xq[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int b = (c == 0 || two) ? L.col[c] : L.col[0];
      xq[c] = lds128(xs + static_cast<uint32_t>(b * 128 + ((ch ^ (b & 7)) << 4)));
    }
#pragma unroll
    for (int t0 = 0; t0 < kTcMaxUnitTiles; t0 += kPre) {
      if (t0 >= ntiles) break;
      double cv[kPre][kK][8];
      uint4 aq[kPre];
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int t = t0 + u;
        if (t >= ntiles) break;
        const uint32_t row0 = c64 ? bank + static_cast<uint32_t>(t * item.tile_bytes + ch * 64)
                                  : wstg + static_cast<uint32_t>((t * kTcMaxChecks * 32 + (ch - L.ch0) * 8) * 8);
#pragma unroll
        for (int k = 0; k < kK; ++k) {
          if (k >= K) break;
#pragma unroll
          for (int h = 0; h < 8; h += 2) {
            lds_f64x2(row0 + static_cast<uint32_t>(k) * rstride + static_cast<uint32_t>(h * 8), cv[u][k][h],
                      cv[u][k][h + 1]);
          }
        }
        aq[u] = lds128(bank + static_cast<uint32_t>(t * item.tile_bytes + K * cstride + ch * 16));
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c == 1 && !two) break;
        const uint32_t w[4] = {xq[c].x, xq[c].y, xq[c].z, xq[c].w};
        double xv[8];
        float ax[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float f = (h & 1) ? bf16_hi(w[h >> 1]) : bf16_lo(w[h >> 1]);
          xv[h] = static_cast<double>(f);
          ax[h] = fabsf(f);
        }
#pragma unroll
        for (int u = 0; u < kPre; ++u) {
          const int t = t0 + u;
          if (t >= ntiles) break;
#pragma unroll
          for (int k = 0; k < kK; ++k) {
            if (k >= K) break;
#pragma unroll
            for (int h = 0; h < 8; ++h) {
              acc.cx[c][t][k][h % kPartials] = __fma_rn(cv[u][k][h], xv[h], acc.cx[c][t][k][h % kPartials]);
            }
          }
          const uint32_t aw[4] = {aq[u].x, aq[u].y, aq[u].z, aq[u].w};
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const float a = (h & 1) ? bf16_hi(aw[h >> 1]) : bf16_lo(aw[h >> 1]);
            acc.sx[c][t][h % kPartials] = __fmaf_ru(a, ax[h], acc.sx[c][t][h % kPartials]);
          }
        }
      }
    }
  }
}

// The end of a work item: each thread's partial sums added in order, then the chunk groups'
// sums added in group order through `comb` (the bank warps' staging area, at its shared
// address; barrier `ready` three times: every warp is done with its staging, every sum is in
// place, every sum is read) and stored as segment `seg` of the checks' partial sums.
// `phase` counts the barrier's completions. False if a barrier wait gave up.
template <int kK>
__device__ __forceinline__ bool bank_finish(const TcJob& jb, const Work& wk, uint32_t comb, uint64_t* ready,
                                            uint32_t& phase, const BankLanes& L, int bt, const BankSums<kK>& acc) {
  const int K = jb.checks;
  double cx[2][kTcMaxUnitTiles][kK], sx[2][kTcMaxUnitTiles];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
#pragma unroll
    for (int t = 0; t < kTcMaxUnitTiles; ++t) {
      float sf = acc.sx[c][t][0];
#pragma unroll
      for (int p = 1; p < kPartials; ++p) sf = __fadd_ru(sf, acc.sx[c][t][p]);
      sx[c][t] = static_cast<double>(sf);  // exact
#pragma unroll
      for (int k = 0; k < kK; ++k) {
        cx[c][t][k] = acc.cx[c][t][k][0];
#pragma unroll
        for (int p = 1; p < kPartials; ++p) cx[c][t][k] = __dadd_rn(cx[c][t][k], acc.cx[c][t][k][p]);
      }
    }
  }
  auto sync = [&]() {
    mbar_arrive(ready);
    const bool ok = mbar_wait(ready, phase & 1u);
    ++phase;
    return ok;
  };
  auto at = [&](int t, int r, int c, int thread) {
    return comb + static_cast<uint32_t>((((t * (kTcMaxChecks + 1) + r) * 2 + c) * kBankThreads + thread) * 8);
  };
  if (L.nsplit > 1) {
    if (!sync()) return false;  // the staging buffers are free
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
      for (int t = 0; t < kTcMaxUnitTiles; ++t) {
        if (t >= wk.ntiles) break;
#pragma unroll
        for (int k = 0; k < kK; ++k) {
          if (k < K) sts_f64(at(t, k, c, bt), cx[c][t][k]);
        }
        sts_f64(at(t, kTcMaxChecks, c, bt), sx[c][t]);
      }
    }
    if (!sync()) return false;  // every group's sums are in place
    if (L.split == 0) {
      for (int g = 1; g < L.nsplit; ++g) {
        const int src = bt + g * L.group;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int t = 0; t < kTcMaxUnitTiles; ++t) {
            if (t >= wk.ntiles) break;
            double other;
#pragma unroll
            for (int k = 0; k < kK; ++k) {
              if (k < K) {
                lds_f64x2_one(at(t, k, c, src), other);
                cx[c][t][k] = __dadd_rn(cx[c][t][k], other);
              }
            }
            lds_f64x2_one(at(t, kTcMaxChecks, c, src), other);
            sx[c][t] = __dadd_ru(sx[c][t], other);
          }
        }
      }
    }
    if (!sync()) return false;  // the area is free for the next stage's staging
    if (L.split != 0) return true;
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int b = L.col[c];
    if (b < 0) continue;
#pragma unroll
    for (int t = 0; t < kTcMaxUnitTiles; ++t) {
      if (t >= wk.ntiles) break;
      const int64_t beta = wk.tile + t;
#pragma unroll
      for (int k = 0; k < kK; ++k) {
        if (k < K) jb.partial_cx[((static_cast<int64_t>(b) * K + k) * jb.nb + beta) * jb.seg_alloc + wk.seg] = cx[c][t][k];
      }
      jb.partial_s[(static_cast<int64_t>(b) * jb.nb + beta) * jb.seg_alloc + wk.seg] = sx[c][t];
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// The kernel (kSplit: the cluster form; kK: checks per job reduced by the bank warps, 1 or 2)

template <bool kSplit, int kK>
__global__ void __launch_bounds__(kTcThreads, 1) tc_kernel(const __grid_constant__ TcPlan plan) {
  // A kernel launched after this one as its programmatic dependent reads nothing it writes
  // (the bank kernel for unfused checks), so it may start on the SMs this grid leaves free.
  allow_dependents();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const int stages = plan.stages;
  const uint32_t stage_bytes = static_cast<uint32_t>(plan.stage_bytes);
  uint8_t* bank_area = smem + static_cast<size_t>(stages) * stage_bytes;  // kTcBankSmemBytes
  uint64_t* full = reinterpret_cast<uint64_t*>(bank_area + kTcBankSmemBytes);
  uint64_t* empty = full + stages;
  uint64_t* wready = empty + stages;  // E4M3: the stage's W widened
  uint64_t* tfull = wready + stages;  // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* comb_ready = tempty + 2;  // the bank threads' barrier at the end of a work item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(comb_ready + 1);
  const bool e4m3 = plan.weights == kTcWeightsE4m3;
  const bool bank_role = plan.any_fused != 0 || e4m3;
  const int warp = static_cast<int>(threadIdx.x) / kWarp;
  const int lane = static_cast<int>(threadIdx.x) % kWarp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1 + (bank_role ? kTcBankWarps : 0));
      mbar_init(wready + s, kTcBankWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 4);
    }
    mbar_init(comb_ready, kBankThreads);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  if constexpr (kSplit) {
    cg::this_cluster().sync();  // every CTA's barriers are initialised before any peer access
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tile_w_bytes = e4m3 ? kTileE4m3Bytes : kTileBf16Bytes;
  // Launched as the programmatic dependent of the kernel before it: every thread but the
  // producer (which may first request settled weights) waits for that kernel here.
  if (!(warp == 0 && lane == 0)) wait_for_producers();
  [[maybe_unused]] Work last{};  // the split form's one item, for its epilogue
  [[maybe_unused]] uint32_t last_it = 0;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      const uint64_t stream_policy = policy_evict_first();
      const uint64_t keep_policy = policy_evict_last();
      // The stage's bytes (W tiles, X tile, the fused checks' bank rows) and its W tiles.
      auto stage_bytes_of = [&](const TcJob& jb, const Work& wk, int kb) {
        const int64_t col = static_cast<int64_t>(kb) * kTcTileK;
        const uint32_t jmax = static_cast<uint32_t>(min(static_cast<int64_t>(kTcTileK), jb.n - col));
        uint32_t bytes = static_cast<uint32_t>(wk.ntiles) * tile_w_bytes + static_cast<uint32_t>(plan.x_bytes);
        const uint32_t csize = jb.c64 ? 8u : 4u;  // bytes of a checksum value in the bank rows
        if (jb.fused) bytes += static_cast<uint32_t>(wk.ntiles) * (static_cast<uint32_t>(jb.checks) * jmax * csize + jmax * 2u);
        return bytes;
      };
      auto load_w = [&](const TcJob& jb, const Work& wk, int kb, uint8_t* st, uint64_t* bar) {
        uint8_t* wdst = e4m3 ? st + plan.w_bytes + plan.x_bytes + plan.bank_bytes : st;
        for (int t = 0; t < wk.ntiles; ++t) {
          tma_load_2d(wdst + static_cast<size_t>(t) * tile_w_bytes, &jb.w_map, bar, kb * kTcTileK,
                      (wk.tile + t) * kTcTileM, stream_policy);
        }
      };
      // Settled weights: the first `stages` stages' W tiles before the producer wait (the ring
      // starts empty), so they stream while the previous kernel finishes.
      int pre = 0;
      if (plan.settled) {
        WorkWalk walk = work_start(plan, kSplit);
        Work wk;
        Ring ring;
        while (pre < stages && work_next(plan, walk, wk)) {
          const TcJob& jb = plan.jobs[wk.job];
          for (int kb = wk.kb0; kb < wk.kb1 && pre < stages; ++kb, ++pre, ring.next(stages)) {
            uint8_t* st = smem + static_cast<size_t>(ring.slot) * stage_bytes;
            mbar_arrive_expect_tx(full + ring.slot, stage_bytes_of(jb, wk, kb));
            load_w(jb, wk, kb, st, full + ring.slot);
          }
        }
      }
      wait_for_producers();  // X, the bank rows and the outputs belong to the kernels before
      WorkWalk walk = work_start(plan, kSplit);
      Work wk;
      Ring ring;
      bool ok = true;
      int issued = 0;
      while (ok && work_next(plan, walk, wk)) {
        const TcJob& jb = plan.jobs[wk.job];
        for (int kb = wk.kb0; kb < wk.kb1; ++kb, ring.next(stages), ++issued) {
          const int s = ring.slot;
          if (!mbar_wait_sleep(empty + s, ring.phase ^ 1u)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + static_cast<size_t>(s) * stage_bytes;
          const int64_t col = static_cast<int64_t>(kb) * kTcTileK;
          const uint32_t jmax = static_cast<uint32_t>(min(static_cast<int64_t>(kTcTileK), jb.n - col));
          if (issued >= pre) {
            mbar_arrive_expect_tx(full + s, stage_bytes_of(jb, wk, kb));
            load_w(jb, wk, kb, st, full + s);
          }
          tma_load_2d(st + plan.w_bytes, &jb.x_map, full + s, kb * kTcTileK, 0, keep_policy);
          if (jb.fused) {
            for (int t = 0; t < wk.ntiles; ++t) {
              const int64_t beta = wk.tile + t;
              uint8_t* tb = st + plan.w_bytes + plan.x_bytes + t * plan.tile_bank_bytes;
              const int cstride = jb.c64 ? 512 : 256;
              for (int k = 0; k < jb.checks; ++k) {
                const int64_t off = (static_cast<int64_t>(k) * jb.nb + beta) * jb.n + col;
                if (jb.c64) {
                  bulk_load(tb + k * cstride, jb.c64 + off, jmax * 8u, full + s, stream_policy);
                } else {
                  bulk_load(tb + k * cstride, jb.c + off, jmax * 4u, full + s, stream_policy);
                }
              }
              bulk_load(tb + jb.checks * cstride, jb.a + beta * jb.n + col, jmax * 2u, full + s, stream_policy);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = instr_desc(plan.n_pad);
      WorkWalk walk = work_start(plan, kSplit);
      Work wk;
      Ring ring;
      uint32_t local = 0;
      bool ok = true;
      while (ok && work_next(plan, walk, wk)) {
        const uint32_t ab = kSplit ? 0u : local % static_cast<uint32_t>(plan.acc_bufs);
        const uint32_t use = kSplit ? 0u : local / static_cast<uint32_t>(plan.acc_bufs);
        if (!mbar_wait_sleep(tempty + ab, (use & 1u) ^ 1u)) break;
        tc_fence_after();
        for (int kb = wk.kb0; kb < wk.kb1; ++kb, ring.next(stages)) {
          const int s = ring.slot;
          const uint32_t parity = ring.phase;
          if (!mbar_wait_sleep(full + s, parity) || (e4m3 && !mbar_wait_sleep(wready + s, parity))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_addr(smem + static_cast<size_t>(s) * stage_bytes);
          const uint64_t bdesc = sw128_desc(st + static_cast<uint32_t>(plan.w_bytes));
          for (int t = 0; t < wk.ntiles; ++t) {
            const uint32_t d = tmem + (ab * static_cast<uint32_t>(plan.unit_tiles) + static_cast<uint32_t>(t)) *
                                          static_cast<uint32_t>(plan.acc_stride);
            const uint64_t adesc = sw128_desc(st + static_cast<uint32_t>(t) * kTileBf16Bytes);
#pragma unroll
            for (int k = 0; k < kTcTileK / 16; ++k) {  // 16 bfloat16 = 32 bytes = 2 descriptor units
              umma_bf16(d, adesc + 2u * k, bdesc + 2u * k, idesc, (kb > wk.kb0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit(empty + s);  // the stage is free once these MMAs (and the bank warps) are done
        }
        if (ok && wk.kb1 > wk.kb0) umma_commit(tfull + ab);
        ++local;
      }
    }
  } else if (warp < 6) {  // epilogue warps 2..5
    const int quarter = warp % 4;
    if constexpr (!kSplit) {
      WorkWalk walk = work_start(plan, false);
      Work wk;
      uint32_t local = 0;
      while (work_next(plan, walk, wk)) {
        const TcJob& jb = plan.jobs[wk.job];
        const uint32_t ab = local % static_cast<uint32_t>(plan.acc_bufs);
        const uint32_t use = local / static_cast<uint32_t>(plan.acc_bufs);
        if (!mbar_wait_sleep(tfull + ab, use & 1u)) break;
        tc_fence_after();
        for (int t = 0; t < wk.ntiles; ++t) {
          const int64_t row = static_cast<int64_t>(wk.tile + t) * kTcTileM + quarter * 32 + lane;
          const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                                (ab * static_cast<uint32_t>(plan.unit_tiles) + static_cast<uint32_t>(t)) *
                                    static_cast<uint32_t>(plan.acc_stride);
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
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + ab);
        ++local;
      }
    } else {
      WorkWalk walk = work_start(plan, true);
      work_next(plan, walk, last);
      last_it = static_cast<uint32_t>(last.kb1 - last.kb0);
    }
  } else if (bank_role) {  // bank warps 6..13
    const int bt = static_cast<int>(threadIdx.x) - 6 * kWarp;
    const BankLanes L = bank_lanes(plan.batch, bt);
    const uint32_t wstg = smem_addr(bank_area) + static_cast<uint32_t>((warp - 6) * kTcBankWarpStage * 8);
    WorkWalk walk = work_start(plan, kSplit);
    Work wk;
    Ring ring;
    uint32_t phase = 0;
    bool ok = true;
    BankSums<kK> acc;
    while (ok && work_next(plan, walk, wk)) {
      const TcJob& jb = plan.jobs[wk.job];
      const BankItem item = bank_item(plan, jb, wk);
      bank_zero(acc);
      for (int kb = wk.kb0; kb < wk.kb1; ++kb, ring.next(stages)) {
        const int s = ring.slot;
        if (!mbar_wait(full + s, ring.phase)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + static_cast<size_t>(s) * stage_bytes;
        if (e4m3) {
          widen_stage(plan, wk.ntiles, st, bt);
          __syncwarp();
          if (lane == 0) mbar_arrive(wready + s);
        }
        if (item.fused) bank_stage(item, kb == item.last_kb ? item.last_cols : kTcTileK, st, wstg, L, lane, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);
      }
      if (ok && jb.fused && wk.kb1 > wk.kb0) ok = bank_finish(jb, wk, smem_addr(bank_area), comb_ready, phase, L, bt, acc);
    }
  }

  if constexpr (kSplit) {
    // The partial accumulators into shared memory (over the stages, once every stage is done
    // with: the last stage's release covers the MMAs and the bank warps), column-major per
    // tile, part[(t * n_pad + col) * 128 + row], so a warp's 32 rows of one column are one
    // conflict-free line; then the cluster sum in rank order by every thread of the CTA, four
    // rows at a time (one 16-byte load per peer), rank r taking row groups
    // [32 r / splits, 32 (r + 1) / splits) of every column.
    float* part = reinterpret_cast<float*>(smem);
    const int n_pad = plan.n_pad;
    if (warp >= 2 && warp < 6) {
      const int quarter = warp % 4;
      const int lrow = quarter * 32 + lane;
      bool have = last_it > 0;
      if (have) {
        const uint32_t i = last_it - 1;
        have = mbar_wait_sleep(tfull, 0) && mbar_wait_sleep(empty + i % stages, (i / stages) & 1u);
      }
      have = __all_sync(kFullMask, have);
      tc_fence_after();
      for (int t = 0; t < last.ntiles; ++t) {
        for (int c0 = 0; c0 < n_pad; c0 += 32) {
          uint32_t v[32];
          if (have) {
            tmem_ld32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                          static_cast<uint32_t>(t * plan.acc_stride + c0), v);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (c0 + i < n_pad) part[(t * n_pad + c0 + i) * kTcTileM + lrow] = have ? __uint_as_float(v[i]) : 0.0f;
          }
        }
      }
    }
    __syncwarp();  // the roles' lane 0 rejoins its warp before the cluster barrier
    tc_fence_before();
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's partial is in its shared memory
    {
      Work unit;  // the cluster's unit, for every thread (only the epilogue warps hold `last`)
      {
        WorkWalk walk = work_start(plan, true);
        work_next(plan, walk, unit);
      }
      const int splits = static_cast<int>(cluster.num_blocks());
      const int rank = static_cast<int>(cluster.block_rank());
      const TcJob& jb = plan.jobs[unit.job];
      constexpr int kGroups = kTcTileM / 4;
      const int g0 = rank * kGroups / splits;
      const int ng = (rank + 1) * kGroups / splits - g0;
      const int items = unit.ntiles * plan.batch * ng;
      const uint32_t local = smem_addr(part);
      uint32_t peer[kTcMaxSplits];
#pragma unroll
      for (int c = 0; c < kTcMaxSplits; ++c) peer[c] = c < splits ? mapa_shared(local, static_cast<uint32_t>(c)) : 0u;
      for (int it0 = static_cast<int>(threadIdx.x); it0 < items; it0 += 2 * kTcThreads) {
        float4 sum[2];
        int64_t row[2];
        int colb[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int item = it0 + h * kTcThreads;
          row[h] = -1;
          if (item >= items) continue;
          const int g = g0 + item % ng;
          const int rest = item / ng;  // t * batch + column
          const int t = rest / plan.batch;
          colb[h] = rest - t * plan.batch;
          row[h] = static_cast<int64_t>(unit.tile + t) * kTcTileM + 4 * g;
          const uint32_t off = static_cast<uint32_t>(((t * n_pad + colb[h]) * kTcTileM + 4 * g) * 4);
          float4 v[kTcMaxSplits];
#pragma unroll
          for (int c = 0; c < kTcMaxSplits; ++c) {
            if (c < splits) v[c] = ld_dsmem_f4(peer[c] + off);
          }
          sum[h] = v[0];
#pragma unroll
          for (int c = 1; c < kTcMaxSplits; ++c) {
            if (c < splits) {
              sum[h].x = __fadd_rn(sum[h].x, v[c].x);
              sum[h].y = __fadd_rn(sum[h].y, v[c].y);
              sum[h].z = __fadd_rn(sum[h].z, v[c].z);
              sum[h].w = __fadd_rn(sum[h].w, v[c].w);
            }
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (row[h] < 0) continue;
          float* dst = jb.Y + static_cast<int64_t>(colb[h]) * jb.m + row[h];
          if (row[h] + 3 < jb.m && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            *reinterpret_cast<float4*>(dst) = sum[h];
          } else {
            const float e[4] = {sum[h].x, sum[h].y, sum[h].z, sum[h].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (row[h] + k < jb.m) dst[k] = e[k];
            }
          }
        }
      }
    }
    cluster.sync();  // no CTA leaves while a peer may still read its partial
  } else {
    __syncwarp();
    tc_fence_before();
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(static_cast<uint32_t>(plan.tmem_cols))
                 : "memory");
  }
}

}  // namespace

PCK_STATUS_READER(tc_status)

namespace {

constexpr int kTcSmemMax = 232448;

// Opts both forms into the largest dynamic shared memory, once per device.
cudaError_t configure(int* dev_out) {
  static int configured[64] = {0};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    for (auto* fn : {tc_kernel<false, 1>, tc_kernel<true, 1>, tc_kernel<false, 2>, tc_kernel<true, 2>}) {
      const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemMax);
      if (err != cudaSuccess) return err;
    }
    configured[dev] = 1;
  }
  *dev_out = dev;
  return cudaSuccess;
}

}  // namespace

int tc_max_clusters(int splits) {
  static int cache[64][kTcMaxSplits + 1] = {};
  int dev = -1;
  if (splits < 2 || splits > kTcMaxSplits || configure(&dev) != cudaSuccess) return 0;
  if (cache[dev][splits] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(splits));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmemMax;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_kernel<true, 1>, &cfg) != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = -1;  // unknown: never chosen
    }
    cache[dev][splits] = n;
  }
  return cache[dev][splits] > 0 ? cache[dev][splits] : 0;
}

cudaError_t launch_tc(const TcPlan& plan, int splits, int grid, size_t smem, cudaStream_t stream) {
  int dev = -1;
  if (const cudaError_t err = configure(&dev); err != cudaSuccess) return err;
  const bool two = plan.max_checks > 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));  // split: a cluster of `splits` CTAs per unit
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // starts during the kernel before
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  if (splits <= 1) {
    return two ? cudaLaunchKernelEx(&cfg, tc_kernel<false, 2>, plan) : cudaLaunchKernelEx(&cfg, tc_kernel<false, 1>, plan);
  }
  return two ? cudaLaunchKernelEx(&cfg, tc_kernel<true, 2>, plan) : cudaLaunchKernelEx(&cfg, tc_kernel<true, 1>, plan);
}

}  // namespace pck
