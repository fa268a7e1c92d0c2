// The persistent streaming kernel: GEMV rows, checksum-bank segments and the block
// verdicts of the trusted checker, for every job of a launch plan (stream_plan.h).
//
// Staged path (kTma): one producer warp streams each unit's bytes from HBM into a ring of
// shared-memory stages with cp.async.bulk (completion counted as transaction bytes on a
// per-stage "full" mbarrier); the activations X of the CTA's job are copied to shared
// memory once. All eight consumer warps work on every stage, in order: each takes its
// share of the unit, publishes a partial result in the stage's scratch and takes a ticket
// (a shared-memory atomic); the warp with the last ticket finishes the unit (final
// reduction, store) and every warp hands the stage back through its "empty" mbarrier
// (eight arrivals). Because every warp consumes every stage in order, a warp waiting for
// use u of a stage has itself consumed use u - 1, so the mbarrier parity waits are exact.
// Plain path (unaligned pointers, n not a multiple of the vector width): each warp takes
// whole units and reads global memory directly; the arithmetic is the same.
//
// GEMV row arithmetic (bit-exact with the reference's model of its coalesced kernel,
// src/pck/gemv.py:71-101 / src/pck/cuda/csrc/gemv_kernel.cu:139-178): with T = 32*NV
// chains, chain t = 32*g + l (group g, lane l) owns vectors t, t + T, ... of V columns
// (V = 8 bfloat16 or 16 E4M3 weights per 16-byte vector) and adds its products in order
// (binary32 product, then binary32 sum — or one FMA where the product is provably exact).
// Each group of 32 chains is reduced by halving across lanes (l += l + 16, ..., l += l + 1)
// and the NV group sums by halving again (g += g + NV/2, ..., g += g + 1).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "stream_plan.h"

namespace pck {

template <int WFMT>
struct Format;
template <>
struct Format<kWeightsBf16> {
  static constexpr int kVec = 8;
  static constexpr int kBytes = 2;
};
template <>
struct Format<kWeightsE4m3> {
  static constexpr int kVec = 16;
  static constexpr int kBytes = 1;
};

enum UnitKind : int { kUnitRow = 0, kUnitC = 1, kUnitA = 2 };

struct Unit {
  int kind;
  int k;
  int s;
  int rows;      // kUnitRow: rows in this unit
  int64_t row;   // kUnitRow: first row
  int64_t beta;  // row block (checked jobs)
  int64_t col0;  // first column (segments)
  int64_t len;   // columns (segments)
  const void* src;
  uint32_t bytes;
};

__host__ __device__ __forceinline__ int64_t ceil_div64(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

__device__ __forceinline__ Unit decode_unit(const JobPlan& jb, int64_t u) {
  Unit x{};
  if (!jb.has_check) {
    x.kind = kUnitRow;
    x.row = u * jb.rows;
    x.rows = static_cast<int>(min(static_cast<int64_t>(jb.rows), jb.m - x.row));
    x.src = static_cast<const uint8_t*>(jb.W) + x.row * jb.row_bytes;
    x.bytes = static_cast<uint32_t>(x.rows * jb.row_bytes);
    return x;
  }
  const int64_t beta = u / jb.period_units;
  int64_t o = u - beta * jb.period_units;
  x.beta = beta;
  const int64_t ru = jb.has_w ? jb.row_units : 0;
  if (o < ru) {
    x.kind = kUnitRow;
    const int64_t first = o * jb.rows;
    x.row = beta * jb.block + first;
    x.rows = static_cast<int>(min(static_cast<int64_t>(jb.rows), jb.block - first));
    x.src = static_cast<const uint8_t*>(jb.W) + x.row * jb.row_bytes;
    x.bytes = static_cast<uint32_t>(x.rows * jb.row_bytes);
    return x;
  }
  o -= ru;
  const int64_t cs = static_cast<int64_t>(jb.checks) * jb.segs;
  if (o < cs) {
    x.kind = kUnitC;
    x.k = static_cast<int>(o / jb.segs);
    x.s = static_cast<int>(o - static_cast<int64_t>(x.k) * jb.segs);
    x.col0 = x.s * jb.seg_len;
    x.len = min(jb.seg_len, jb.n - x.col0);
    x.src = jb.c + (static_cast<int64_t>(x.k) * jb.num_blocks + beta) * jb.n + x.col0;
    x.bytes = static_cast<uint32_t>(x.len * 4);
    return x;
  }
  x.kind = kUnitA;
  x.s = static_cast<int>(o - cs);
  x.col0 = x.s * jb.seg_len;
  x.len = min(jb.seg_len, jb.n - x.col0);
  x.src = jb.a + beta * jb.n + x.col0;
  x.bytes = static_cast<uint32_t>(x.len * 2);
  return x;
}

// First unit whose starting byte is >= target; units are partitioned between the CTAs of
// a job by their starting byte, so every CTA finds the same boundaries.
__device__ __forceinline__ int64_t first_unit_at(const JobPlan& jb, int64_t target) {
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

// ---------------------------------------------------------------------------------------
// Reduction of a row's chains.

// Level LVL (offset 16 >> LVL) of the halving tree over the 32 lanes, for the live slots.
template <int NV, int LVL>
struct HalveLanes {
  static __device__ __forceinline__ void run(float (&a)[NV], int lane) {
    constexpr int kOff = 16 >> LVL;
    constexpr int kLive = (NV >> LVL) > 0 ? (NV >> LVL) : 1;
    const bool upper = (lane & kOff) != 0;
    if constexpr (kLive >= 2) {
      // Partners l and l ^ kOff hold the same chain groups for tree positions l and
      // l ^ kOff. The lower lane keeps the first half of the groups, the upper lane the
      // second half; each adds the partner's value for the groups it keeps.
      constexpr int kHalf = kLive / 2;
#pragma unroll
      for (int j = 0; j < kHalf; ++j) {
        const float send = upper ? a[j] : a[kHalf + j];
        const float recv = __shfl_xor_sync(kFullMask, send, kOff);
        a[j] = __fadd_rn(upper ? a[kHalf + j] : a[j], recv);
      }
    } else {
      a[0] = __fadd_rn(a[0], __shfl_xor_sync(kFullMask, a[0], kOff));
    }
    HalveLanes<NV, LVL + 1>::run(a, lane);
  }
};
template <int NV>
struct HalveLanes<NV, 5> {
  static __device__ __forceinline__ void run(float (&)[NV], int) {}
};

// Lane that holds the sum of chain group g after HalveLanes: group bits from the most
// significant one map to lane bits 16, 8, 4, ...
template <int NV>
__device__ __forceinline__ int group_lane(int g) {
  int lane = 0;
  int bit = NV >> 1;
  int off = 16;
  while (bit > 0) {
    if (g & bit) lane |= off;
    bit >>= 1;
    off >>= 1;
  }
  return lane;
}

// Row value from the per-lane chain sums a[g] = chain 32*g + lane. Every lane returns it.
template <int NV>
__device__ __forceinline__ float halve_groups(float (&a)[NV], int lane) {
  HalveLanes<NV, 0>::run(a, lane);
  float g[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) g[i] = __shfl_sync(kFullMask, a[0], group_lane<NV>(i));
#pragma unroll
  for (int h = NV / 2; h >= 1; h /= 2) {
#pragma unroll
    for (int i = 0; i < h; ++i) g[i] = __fadd_rn(g[i], g[i + h]);
  }
  return g[0];
}

// ---------------------------------------------------------------------------------------
// Products of one vector, added to a chain.

__device__ __forceinline__ void chain_bf16(float& acc, const uint4 w, const uint4 x) {
  acc = __fadd_rn(acc, __fmul_rn(bf16_lo(w.x), bf16_lo(x.x)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_hi(w.x), bf16_hi(x.x)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_lo(w.y), bf16_lo(x.y)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_hi(w.y), bf16_hi(x.y)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_lo(w.z), bf16_lo(x.z)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_hi(w.z), bf16_hi(x.z)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_lo(w.w), bf16_lo(x.w)));
  acc = __fadd_rn(acc, __fmul_rn(bf16_hi(w.w), bf16_hi(x.w)));
}

template <bool kFma>
__device__ __forceinline__ void chain_pair(float& acc, float w, float x) {
  if constexpr (kFma) {
    acc = __fmaf_rn(w, x, acc);  // the product is exact: same as product then sum
  } else {
    acc = __fadd_rn(acc, __fmul_rn(w, x));
  }
}

template <bool kFma>
__device__ __forceinline__ void chain_e4m3_word(float& acc, uint32_t w4, uint32_t xa, uint32_t xb) {
  const float2 w01 = e4m3x2_to_float2(static_cast<uint16_t>(w4 & 0xffffu));
  const float2 w23 = e4m3x2_to_float2(static_cast<uint16_t>(w4 >> 16));
  chain_pair<kFma>(acc, w01.x, bf16_lo(xa));
  chain_pair<kFma>(acc, w01.y, bf16_hi(xa));
  chain_pair<kFma>(acc, w23.x, bf16_lo(xb));
  chain_pair<kFma>(acc, w23.y, bf16_hi(xb));
}

template <bool kFma>
__device__ __forceinline__ void chain_e4m3(float& acc, const uint4 w, const uint4 xa,
                                           const uint4 xb) {
  chain_e4m3_word<kFma>(acc, w.x, xa.x, xa.y);
  chain_e4m3_word<kFma>(acc, w.y, xa.z, xa.w);
  chain_e4m3_word<kFma>(acc, w.z, xb.x, xb.y);
  chain_e4m3_word<kFma>(acc, w.w, xb.z, xb.w);
}

template <int WFMT>
__device__ __forceinline__ float load_weight(const uint8_t* w, int64_t j) {
  if constexpr (WFMT == kWeightsBf16) {
    return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(w)[j]);
  } else {
    return e4m3_to_float(w[j]);
  }
}

// One W row against X: writes Y[b*ldy + row] for every column b (lane 0 stores).
// kFast: 16-byte aligned row and X, n a multiple of the vector width.
template <int WFMT, int NV, int BG, bool kFast, bool kFma>
__device__ __forceinline__ void gemv_row(const uint8_t* __restrict__ wrow,
                                         const uint16_t* __restrict__ X, int64_t n, int batch,
                                         float* __restrict__ Y, int64_t ldy, int64_t row,
                                         int lane) {
  constexpr int V = Format<WFMT>::kVec;
  constexpr int T = NV * kWarp;
  const int64_t per_thread = ceil_div64(ceil_div64(n, V), T);
  for (int g0 = 0; g0 < batch; g0 += BG) {
    float acc[BG][NV];
#pragma unroll
    for (int b = 0; b < BG; ++b) {
#pragma unroll
      for (int w = 0; w < NV; ++w) acc[b][w] = -0.0f;  // -0 + p == p for every p
    }
    const uint16_t* xcol[BG];
#pragma unroll
    for (int b = 0; b < BG; ++b) xcol[b] = X + static_cast<int64_t>(min(g0 + b, batch - 1)) * n;

    for (int64_t v = 0; v < per_thread; ++v) {
#pragma unroll
      for (int w = 0; w < NV; ++w) {
        const int64_t q = v * T + w * kWarp + lane;
        const int64_t col0 = q * V;
        if constexpr (kFast) {
          if (col0 < n) {
            const uint4 wv = *reinterpret_cast<const uint4*>(wrow + col0 * Format<WFMT>::kBytes);
#pragma unroll
            for (int b = 0; b < BG; ++b) {
              const uint4* xp = reinterpret_cast<const uint4*>(xcol[b] + col0);
              if constexpr (WFMT == kWeightsBf16) {
                chain_bf16(acc[b][w], wv, xp[0]);
              } else {
                chain_e4m3<kFma>(acc[b][w], wv, xp[0], xp[1]);
              }
            }
          } else {
#pragma unroll
            for (int b = 0; b < BG; ++b) acc[b][w] = __fadd_rn(acc[b][w], 0.0f);
          }
        } else {
#pragma unroll 1
          for (int e = 0; e < V; ++e) {
            const int64_t j = col0 + e;
            const bool in = j < n;
            const float wj = in ? load_weight<WFMT>(wrow, j) : 0.0f;
#pragma unroll
            for (int b = 0; b < BG; ++b) {
              const float xj = in ? bf16_bits_to_float(xcol[b][j]) : 0.0f;
              const float p = in ? __fmul_rn(wj, xj) : 0.0f;
              acc[b][w] = __fadd_rn(acc[b][w], p);
            }
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < BG; ++b) {
      const float yv = halve_groups<NV>(acc[b], lane);
      if (lane == 0 && g0 + b < batch) Y[static_cast<int64_t>(g0 + b) * ldy + row] = yv;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Checksum-bank segments (binary64; bfloat16 x binary32 and bfloat16 x bfloat16 products
// are exact in binary64, so every step is one rounding of an exact value).

__device__ __forceinline__ double warp_sum_rn(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_down_sync(kFullMask, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_ru(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_ru(v, __shfl_down_sync(kFullMask, v, o));
  return v;
}

// c-segment: partial c . x_b for every column b; lane 0 stores it.
template <bool kFast>
__device__ __forceinline__ void c_segment(const float* __restrict__ cs,
                                          const uint16_t* __restrict__ X, int64_t n, int batch,
                                          int64_t col0, int64_t len, double* __restrict__ out,
                                          int64_t out_stride, int lane) {
  for (int b = 0; b < batch; ++b) {
    const uint16_t* xb = X + static_cast<int64_t>(b) * n + col0;
    double acc = 0.0;
    if constexpr (kFast) {
      for (int64_t j = lane * 4; j < len; j += 4 * kWarp) {
        const float4 cv = *reinterpret_cast<const float4*>(cs + j);
        const uint2 xv = *reinterpret_cast<const uint2*>(xb + j);
        acc = __fma_rn(static_cast<double>(cv.x), static_cast<double>(bf16_lo(xv.x)), acc);
        acc = __fma_rn(static_cast<double>(cv.y), static_cast<double>(bf16_hi(xv.x)), acc);
        acc = __fma_rn(static_cast<double>(cv.z), static_cast<double>(bf16_lo(xv.y)), acc);
        acc = __fma_rn(static_cast<double>(cv.w), static_cast<double>(bf16_hi(xv.y)), acc);
      }
    } else {
      for (int64_t j = lane; j < len; j += kWarp) {
        acc = __fma_rn(static_cast<double>(cs[j]), static_cast<double>(bf16_bits_to_float(xb[j])),
                       acc);
      }
    }
    acc = warp_sum_rn(acc);
    if (lane == 0) out[b * out_stride] = acc;
  }
}

// a-segment: upper bound of a . |x_b| for every column b; lane 0 stores it.
template <bool kFast>
__device__ __forceinline__ void a_segment(const uint16_t* __restrict__ as,
                                          const uint16_t* __restrict__ X, int64_t n, int batch,
                                          int64_t col0, int64_t len, double* __restrict__ out,
                                          int64_t out_stride, int lane) {
  for (int b = 0; b < batch; ++b) {
    const uint16_t* xb = X + static_cast<int64_t>(b) * n + col0;
    double acc = 0.0;
    if constexpr (kFast) {
      for (int64_t j = lane * 4; j < len; j += 4 * kWarp) {
        const uint2 av = *reinterpret_cast<const uint2*>(as + j);
        const uint2 xv = *reinterpret_cast<const uint2*>(xb + j);
        acc = __fma_ru(static_cast<double>(bf16_lo(av.x)), fabs(static_cast<double>(bf16_lo(xv.x))), acc);
        acc = __fma_ru(static_cast<double>(bf16_hi(av.x)), fabs(static_cast<double>(bf16_hi(xv.x))), acc);
        acc = __fma_ru(static_cast<double>(bf16_lo(av.y)), fabs(static_cast<double>(bf16_lo(xv.y))), acc);
        acc = __fma_ru(static_cast<double>(bf16_hi(av.y)), fabs(static_cast<double>(bf16_hi(xv.y))), acc);
      }
    } else {
      for (int64_t j = lane; j < len; j += kWarp) {
        acc = __fma_ru(static_cast<double>(bf16_bits_to_float(as[j])),
                       fabs(static_cast<double>(bf16_bits_to_float(xb[j]))), acc);
      }
    }
    acc = warp_sum_ru(acc);
    if (lane == 0) out[b * out_stride] = acc;
  }
}

// ---------------------------------------------------------------------------------------
// Verdict of row block beta: runs in the warp that completed the block's last unit, after
// every other unit's results were published (fence, then ticket). Reads y from memory.
// Decision rule of the reference checker (src/pck/cuda/csrc/checker_kernel.cu:146-184).

static __device__ __noinline__ void merge_block(const JobPlan& jb, int64_t beta, int lane) {
  __threadfence();
  const int blk = jb.block;
  const int64_t nb = jb.num_blocks;
  const int64_t ldy = jb.m;
  constexpr double kOnePlusU32 = 1.0 + 0x1p-24;
  constexpr double kFloatMax = 3.4028234663852886e38;
  for (int col = 0; col < jb.batch; ++col) {
    const float* yb = jb.y_check + col * ldy + beta * blk;
    double yabs = 0.0;
    bool bad = false;
    for (int i = lane; i < blk; i += kWarp) {
      const float v = __ldcg(yb + i);
      bad |= !isfinite(v);
      yabs = __dadd_ru(yabs, fabs(static_cast<double>(v)));
    }
    yabs = warp_sum_ru(yabs);
    bad = __any_sync(kFullMask, bad);
    double s_total = 0.0;
    if (lane == 0) {
      const double* ps = jb.partial_s + (col * nb + beta) * jb.seg_alloc;
      for (int s = 0; s < jb.segs; ++s) s_total = __dadd_ru(s_total, __ldcg(ps + s));
    }
    for (int k = 0; k < jb.checks; ++k) {
      const int8_t* rk = jb.r + (static_cast<int64_t>(k) * nb + beta) * blk;
      double ry = 0.0;
      for (int i = lane; i < blk; i += kWarp) {
        const double v = static_cast<double>(__ldcg(yb + i));
        ry = __dadd_rn(ry, __ldg(rk + i) > 0 ? v : -v);
      }
      ry = warp_sum_rn(ry);
      if (lane == 0) {
        const double* pc =
            jb.partial_cx + ((static_cast<int64_t>(col) * jb.checks + k) * nb + beta) * jb.seg_alloc;
        double cx = 0.0;
        for (int s = 0; s < jb.segs; ++s) cx = __dadd_rn(cx, __ldcg(pc + s));
        const double rho = __dsub_rn(cx, ry);
        const double cabs = __dmul_ru(kOnePlusU32, s_total);
        const double eps = __dmul_ru(jb.geps, __dadd_ru(cabs, yabs));
        double tau = __dadd_ru(__dadd_ru(__dmul_ru(jb.coef, s_total), eps), jb.tau_floor);
        // Beyond the binary32 range of a.|x| the checked kernel's rounding model (no
        // overflow) cannot hold: the threshold is unbounded and the block fails closed.
        if (!(s_total <= kFloatMax)) tau = __longlong_as_double(0x7ff0000000000000LL);
        const int64_t o = (static_cast<int64_t>(col) * jb.checks + k) * nb + beta;
        jb.passed[o] = (!bad && isfinite(tau) && fabs(rho) <= tau) ? 1 : 0;
        jb.rho[o] = rho;
        jb.tau[o] = tau;
      }
    }
  }
  if (lane == 0) jb.counters[beta] = 0;  // ready for the next call
}

// Publishes `count` finished units of block beta; the warp that finishes the block
// computes its verdict.
__device__ __forceinline__ void credit_block(const JobPlan& jb, int64_t beta, uint32_t count,
                                             int lane) {
  __syncwarp();
  uint32_t before = 0;
  if (lane == 0) {
    __threadfence();
    before = atomicAdd(jb.counters + beta, count);
  }
  before = __shfl_sync(kFullMask, before, 0);
  const uint32_t total = static_cast<uint32_t>(jb.period_units);
  if (before + count == total) merge_block(jb, beta, lane);
}

// ---------------------------------------------------------------------------------------
// Plain path: one warp per unit, global memory.

template <int WFMT, int NV, int BG>
__device__ __forceinline__ void plain_unit(const JobPlan& jb, const Unit& un, const uint16_t* X,
                                           int lane) {
  if (un.kind == kUnitRow) {
    for (int r = 0; r < un.rows; ++r) {
      const uint8_t* wrow = static_cast<const uint8_t*>(un.src) + r * jb.row_bytes;
      gemv_row<WFMT, NV, BG, false, false>(wrow, X, jb.n, jb.batch, jb.Y, jb.m, un.row + r, lane);
    }
  } else if (un.kind == kUnitC) {
    const int64_t nb = jb.num_blocks;
    double* out = jb.partial_cx + (static_cast<int64_t>(un.k) * nb + un.beta) * jb.seg_alloc + un.s;
    const int64_t stride = static_cast<int64_t>(jb.checks) * nb * jb.seg_alloc;
    c_segment<false>(static_cast<const float*>(un.src), X, jb.n, jb.batch, un.col0, un.len, out,
                     stride, lane);
  } else {
    const int64_t nb = jb.num_blocks;
    double* out = jb.partial_s + un.beta * jb.seg_alloc + un.s;
    a_segment<false>(static_cast<const uint16_t*>(un.src), X, jb.n, jb.batch, un.col0, un.len, out,
                     nb * jb.seg_alloc, lane);
  }
}

// ---------------------------------------------------------------------------------------
// Staged path: all consumer warps share each unit.

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// Which chains and rows of a row unit a consumer warp owns. Pairs (row r, group g) are
// dealt to the eight warps: with NV >= 8 groups, warp w takes groups w, w + 8, ... for
// every row; with fewer, warp w takes group w % NV for rows w / NV, w / NV + 8 / NV, ...
// A warp loads each activation vector once and uses it for all its rows.
template <int WFMT, int NV>
struct Share {
  static constexpr int kRows = unit_rows(WFMT, NV);                    // rows per unit, max
  static constexpr int kGroups = NV >= kConsumerWarps ? NV / kConsumerWarps : 1;
  static constexpr int kRowsPerWarp = NV >= kConsumerWarps ? kRows : kRows * NV / kConsumerWarps;
  static __device__ __forceinline__ int group(int warp, int j) {
    return NV >= kConsumerWarps ? warp + kConsumerWarps * j : warp % NV;
  }
  static __device__ __forceinline__ int row(int warp, int k) {
    return NV >= kConsumerWarps ? k : warp / NV + (kConsumerWarps / NV) * k;
  }
};

__device__ __forceinline__ float lane_halving(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(kFullMask, v, o));
  return v;
}

// This warp's share of a row unit at stage address `stage` (rows of row_bytes), against
// the activations at `xs` (batch rows of n bfloat16). Publishes the group sums
// sums[(r * NV + g) * batch + b] for its (row, group) pairs.
template <int WFMT, int NV, int BG, bool kFma>
__device__ __forceinline__ void rows_share(const JobPlan& jb, uint32_t stage, uint32_t xs, float* sums,
                                           int rows_here, int warp, int lane) {
  using S = Share<WFMT, NV>;
  constexpr int V = Format<WFMT>::kVec;
  constexpr int T = NV * kWarp;
  constexpr uint32_t kWV = 16;          // bytes of one weight vector
  constexpr uint32_t kXV = V * 2;       // bytes of one activation vector (16 or 32)
  const int nvec = static_cast<int>(jb.n / V);  // n % V == 0 on this path
  const int full = nvec / T;
  const bool tail = full * T != nvec;
  const uint32_t row_bytes = static_cast<uint32_t>(jb.row_bytes);
  const uint32_t xcol = static_cast<uint32_t>(jb.n * 2);
  const int batch = jb.batch;
  for (int g0 = 0; g0 < batch; g0 += BG) {
    float acc[S::kRowsPerWarp][S::kGroups][BG];
#pragma unroll
    for (int k = 0; k < S::kRowsPerWarp; ++k)
#pragma unroll
      for (int j = 0; j < S::kGroups; ++j)
#pragma unroll
        for (int b = 0; b < BG; ++b) acc[k][j][b] = -0.0f;  // -0 + p == p for every p

    const int iters = full + (tail ? 1 : 0);
    for (int v = 0; v < iters; ++v) {
#pragma unroll
      for (int j = 0; j < S::kGroups; ++j) {
        const int q = v * T + S::group(warp, j) * kWarp + lane;
        if (v == full && q >= nvec) {  // padding past n: +0 terms
#pragma unroll
          for (int k = 0; k < S::kRowsPerWarp; ++k)
#pragma unroll
            for (int b = 0; b < BG; ++b) acc[k][j][b] = __fadd_rn(acc[k][j][b], 0.0f);
          continue;
        }
        uint4 xa[BG], xb[BG];
#pragma unroll
        for (int b = 0; b < BG; ++b) {
          const uint32_t xaddr = xs + static_cast<uint32_t>(min(g0 + b, batch - 1)) * xcol + q * kXV;
          xa[b] = lds128(xaddr);
          if constexpr (WFMT == kWeightsE4m3) xb[b] = lds128(xaddr + 16);
        }
#pragma unroll
        for (int k = 0; k < S::kRowsPerWarp; ++k) {
          const int r = S::row(warp, k);
          if (r < rows_here) {
            const uint4 wv = lds128(stage + r * row_bytes + q * kWV);
#pragma unroll
            for (int b = 0; b < BG; ++b) {
              if constexpr (WFMT == kWeightsBf16) {
                if constexpr (kFma) {
                  chain_pair<true>(acc[k][j][b], bf16_lo(wv.x), bf16_lo(xa[b].x));
                  chain_pair<true>(acc[k][j][b], bf16_hi(wv.x), bf16_hi(xa[b].x));
                  chain_pair<true>(acc[k][j][b], bf16_lo(wv.y), bf16_lo(xa[b].y));
                  chain_pair<true>(acc[k][j][b], bf16_hi(wv.y), bf16_hi(xa[b].y));
                  chain_pair<true>(acc[k][j][b], bf16_lo(wv.z), bf16_lo(xa[b].z));
                  chain_pair<true>(acc[k][j][b], bf16_hi(wv.z), bf16_hi(xa[b].z));
                  chain_pair<true>(acc[k][j][b], bf16_lo(wv.w), bf16_lo(xa[b].w));
                  chain_pair<true>(acc[k][j][b], bf16_hi(wv.w), bf16_hi(xa[b].w));
                } else {
                  chain_bf16(acc[k][j][b], wv, xa[b]);
                }
              } else {
                chain_e4m3<kFma>(acc[k][j][b], wv, xa[b], xb[b]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < S::kRowsPerWarp; ++k) {
      const int r = S::row(warp, k);
#pragma unroll
      for (int j = 0; j < S::kGroups; ++j) {
#pragma unroll
        for (int b = 0; b < BG; ++b) {
          const float s = lane_halving(acc[k][j][b]);
          if (lane == 0 && r < rows_here && g0 + b < batch) {
            sums[(r * NV + S::group(warp, j)) * batch + g0 + b] = s;
          }
        }
      }
    }
  }
}

// Last warp of a row unit: halving over the NV group sums of every (row, column).
template <int NV>
__device__ __forceinline__ void rows_finish(const JobPlan& jb, const float* sums, int64_t row0,
                                            int rows_here, int lane) {
  const int batch = jb.batch;
  for (int o = lane; o < rows_here * batch; o += kWarp) {
    const int r = o / batch;
    const int b = o - r * batch;
    float g[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) g[i] = sums[(r * NV + i) * batch + b];
#pragma unroll
    for (int h = NV / 2; h >= 1; h /= 2) {
#pragma unroll
      for (int i = 0; i < h; ++i) g[i] = __fadd_rn(g[i], g[i + h]);
    }
    jb.Y[static_cast<int64_t>(b) * jb.m + row0 + r] = g[0];
  }
}

// This warp's share of a c- or a-segment: elements (4 at a time) warp*32 + lane, + 256, ...
// Publishes dsums[warp * batch + b].
template <bool kAbs>
__device__ __forceinline__ void segment_share(const JobPlan& jb, const Unit& un, uint32_t stage,
                                              uint32_t xs, double* dsums, int warp, int lane) {
  const int batch = jb.batch;
  const uint32_t xcol = static_cast<uint32_t>(jb.n * 2);
  const int len = static_cast<int>(un.len);
  for (int b = 0; b < batch; ++b) {
    const uint32_t xb = xs + static_cast<uint32_t>(b) * xcol + static_cast<uint32_t>(un.col0) * 2;
    double acc = 0.0;
    for (int e = (warp * kWarp + lane) * 4; e < len; e += kConsumerWarps * kWarp * 4) {
      const uint2 xv = lds64(xb + e * 2);
      if constexpr (kAbs) {
        const uint2 av = lds64(stage + e * 2);
        acc = __fma_ru(static_cast<double>(bf16_lo(av.x)), fabs(static_cast<double>(bf16_lo(xv.x))), acc);
        acc = __fma_ru(static_cast<double>(bf16_hi(av.x)), fabs(static_cast<double>(bf16_hi(xv.x))), acc);
        acc = __fma_ru(static_cast<double>(bf16_lo(av.y)), fabs(static_cast<double>(bf16_lo(xv.y))), acc);
        acc = __fma_ru(static_cast<double>(bf16_hi(av.y)), fabs(static_cast<double>(bf16_hi(xv.y))), acc);
      } else {
        const uint4 cv = lds128(stage + e * 4);
        acc = __fma_rn(static_cast<double>(__uint_as_float(cv.x)), static_cast<double>(bf16_lo(xv.x)), acc);
        acc = __fma_rn(static_cast<double>(__uint_as_float(cv.y)), static_cast<double>(bf16_hi(xv.x)), acc);
        acc = __fma_rn(static_cast<double>(__uint_as_float(cv.z)), static_cast<double>(bf16_lo(xv.y)), acc);
        acc = __fma_rn(static_cast<double>(__uint_as_float(cv.w)), static_cast<double>(bf16_hi(xv.y)), acc);
      }
    }
    acc = kAbs ? warp_sum_ru(acc) : warp_sum_rn(acc);
    if (lane == 0) dsums[warp * batch + b] = acc;
  }
}

// Last warp of a segment: the warp partials in warp order, stored to the block's scratch.
__device__ __forceinline__ void segment_finish(const JobPlan& jb, const Unit& un, const double* dsums,
                                               int lane) {
  const int batch = jb.batch;
  const int64_t nb = jb.num_blocks;
  for (int b = lane; b < batch; b += kWarp) {
    double total = 0.0;
    if (un.kind == kUnitC) {
      for (int w = 0; w < kConsumerWarps; ++w) total = __dadd_rn(total, dsums[w * batch + b]);
      jb.partial_cx[((static_cast<int64_t>(b) * jb.checks + un.k) * nb + un.beta) * jb.seg_alloc + un.s] = total;
    } else {
      for (int w = 0; w < kConsumerWarps; ++w) total = __dadd_ru(total, dsums[w * batch + b]);
      jb.partial_s[(static_cast<int64_t>(b) * nb + un.beta) * jb.seg_alloc + un.s] = total;
    }
  }
}

// Exponent fields (bfloat16 bits 7-14) of the activations: smallest over nonzero values
// (subnormals count as 1) and largest over all.
__device__ __forceinline__ void x_exponents(const uint16_t* X, int64_t count, int first, int step,
                                            unsigned* lo, unsigned* hi) {
  unsigned mn = 1000, mx = 0;
  for (int64_t j = first; j < count; j += step) {
    const unsigned mag = X[j] & 0x7fffu;
    const unsigned e = mag >> 7;
    mx = max(mx, e);
    if (mag) mn = min(mn, max(e, 1u));
  }
  atomicMin(lo, mn);
  atomicMax(hi, mx);
}

// Whether one FMA equals the product-then-sum for every weight x activation pair.
// E4M3 x bfloat16: the product is always exact (<= 12 significant bits, lowest bit >=
// 2^-142) unless it overflows, which needs an activation exponent field >= 246.
// bfloat16 x bfloat16: exact iff no product falls below 2^-126 with bits under 2^-149 and
// none overflows: e_w + e_x >= 119 for the smallest nonzero exponent fields, and
// e_w + e_x <= 380 for the largest (the weights' range comes with the job, 0 = unknown).
template <int WFMT>
__device__ __forceinline__ bool fma_is_exact(const JobPlan& jb, unsigned x_lo, unsigned x_hi) {
  if constexpr (WFMT == kWeightsE4m3) {
    return x_hi <= 245u;
  } else {
    if (jb.w_exp_min <= 0 || jb.w_exp_max <= 0) return false;
    const bool low_ok = x_lo >= 1000u || static_cast<int>(x_lo) + jb.w_exp_min >= 119;
    const bool high_ok = static_cast<int>(x_hi) + jb.w_exp_max <= 380;
    return low_ok && high_ok;
  }
}

template <int WFMT, int NV, int BG, bool kTma>
__global__ void __launch_bounds__(kTma ? kTmaThreads : kPlainThreads, 1)
    stream_kernel(const __grid_constant__ Plan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  int j = 0;
  while (j + 1 < plan.njobs && static_cast<int>(blockIdx.x) >= plan.jobs[j + 1].cta_begin) ++j;
  const JobPlan& jb = plan.jobs[j];
  const int64_t local = static_cast<int64_t>(blockIdx.x) - jb.cta_begin;
  if (local >= jb.cta_count) return;
  const int64_t u0 = first_unit_at(jb, local * jb.total_bytes / jb.cta_count);
  const int64_t u1 = first_unit_at(jb, (local + 1) * jb.total_bytes / jb.cta_count);
  const int64_t count = u1 - u0;
  if (count <= 0) return;  // uniform for the whole CTA
  const int warp = static_cast<int>(threadIdx.x) / kWarp;
  const int lane = static_cast<int>(threadIdx.x) % kWarp;

  if constexpr (kTma) {
    const int stages = plan.stages;
    const int sum_bytes = plan.sum_bytes;
    uint8_t* xs = smem;
    uint8_t* ring = smem + plan.x_bytes;
    uint8_t* scratch = ring + static_cast<int64_t>(stages) * plan.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(scratch + static_cast<int64_t>(stages) * sum_bytes);
    uint64_t* empty = full + stages;
    uint64_t* xbar = empty + stages;
    uint32_t* tickets = reinterpret_cast<uint32_t*>(xbar + 1);
    uint32_t* xexp = tickets + stages;  // [0] smallest, [1] largest exponent field of x
    if (threadIdx.x == 0) {
      for (int s = 0; s < stages; ++s) {
        mbar_init(full + s, 1);
        mbar_init(empty + s, kConsumerWarps);
        tickets[s] = 0;
      }
      mbar_init(xbar, 1);
      xexp[0] = 1000;
      xexp[1] = 0;
      fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {  // producer
      if (lane == 0) {
        const uint64_t keep = policy_evict_last();
        const uint64_t once = policy_evict_first();
        const uint32_t xbytes = static_cast<uint32_t>(static_cast<int64_t>(jb.batch) * jb.n * 2);
        mbar_arrive_expect_tx(xbar, xbytes);
        bulk_load(xs, jb.X, xbytes, xbar, keep);
        int64_t issued = 0;
        for (int64_t i = 0; i < count; ++i) {
          const int st = static_cast<int>(i % stages);
          if (i >= stages && !mbar_wait(empty + st, static_cast<uint32_t>((i / stages - 1) & 1))) break;
          const Unit un = decode_unit(jb, u0 + i);
          mbar_arrive_expect_tx(full + st, un.bytes);
          bulk_load(ring + static_cast<int64_t>(st) * plan.stage_bytes, un.src, un.bytes, full + st, once);
          ++issued;
        }
        // Leave only after every copy into this CTA's shared memory has landed.
        for (int64_t i = issued > stages ? issued - stages : 0; i < issued; ++i) {
          mbar_wait(full + i % stages, static_cast<uint32_t>((i / stages) & 1));
        }
        mbar_wait(xbar, 0);
      }
      return;
    }

    // consumers
    const uint16_t* X = reinterpret_cast<const uint16_t*>(xs);
    const bool have_x = mbar_wait(xbar, 0);
    if (have_x && jb.has_w) {
      x_exponents(X, static_cast<int64_t>(jb.batch) * jb.n, static_cast<int>(threadIdx.x), kPlainThreads,
                  xexp, xexp + 1);
    }
    named_barrier(1, kPlainThreads);
    if (!have_x) return;
    const bool fma = jb.has_w && fma_is_exact<WFMT>(jb, xexp[0], xexp[1]);
    const uint32_t xs_addr = smem_addr(xs);
    const uint32_t ring_addr = smem_addr(ring);

    int64_t cur_beta = -1;
    uint32_t pending = 0;
    for (int64_t i = 0; i < count; ++i) {
      const int st = static_cast<int>(i % stages);
      if (!mbar_wait(full + st, static_cast<uint32_t>((i / stages) & 1))) return;
      const Unit un = decode_unit(jb, u0 + i);
      const uint32_t stage = ring_addr + static_cast<uint32_t>(st) * static_cast<uint32_t>(plan.stage_bytes);
      uint8_t* sums = scratch + static_cast<int64_t>(st) * sum_bytes;
      if (un.kind == kUnitRow) {
        if (fma) {
          rows_share<WFMT, NV, BG, true>(jb, stage, xs_addr, reinterpret_cast<float*>(sums), un.rows, warp, lane);
        } else {
          rows_share<WFMT, NV, BG, false>(jb, stage, xs_addr, reinterpret_cast<float*>(sums), un.rows, warp, lane);
        }
      } else if (un.kind == kUnitC) {
        segment_share<false>(jb, un, stage, xs_addr, reinterpret_cast<double*>(sums), warp, lane);
      } else {
        segment_share<true>(jb, un, stage, xs_addr, reinterpret_cast<double*>(sums), warp, lane);
      }
      __syncwarp();
      uint32_t ticket = 0;
      if (lane == 0) {
        __threadfence_block();
        ticket = atomicAdd(tickets + st, 1u);
      }
      ticket = __shfl_sync(kFullMask, ticket, 0);
      const bool last = ticket == kConsumerWarps - 1;
      if (last) {
        __threadfence_block();
        if (un.kind == kUnitRow) {
          rows_finish<NV>(jb, reinterpret_cast<const float*>(sums), un.row, un.rows, lane);
        } else {
          segment_finish(jb, un, reinterpret_cast<const double*>(sums), lane);
        }
        __syncwarp();
        if (lane == 0) tickets[st] = 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);
      if (last && jb.has_check) {
        if (un.beta != cur_beta && pending) {
          credit_block(jb, cur_beta, pending, lane);
          pending = 0;
        }
        cur_beta = un.beta;
        ++pending;
      }
    }
    if (pending) credit_block(jb, cur_beta, pending, lane);
  } else {
    // Plain path: every warp takes whole units and reads global memory directly, one
    // element at a time (product, then sum: the same values as the staged path's).
    const uint16_t* X = jb.X;
    int64_t cur_beta = -1;
    uint32_t pending = 0;
    for (int64_t i = warp; i < count; i += kConsumerWarps) {
      const Unit un = decode_unit(jb, u0 + i);
      plain_unit<WFMT, NV, BG>(jb, un, X, lane);
      if (jb.has_check) {
        if (un.beta != cur_beta && pending) {
          credit_block(jb, cur_beta, pending, lane);
          pending = 0;
        }
        cur_beta = un.beta;
        ++pending;
      }
    }
    if (pending) credit_block(jb, cur_beta, pending, lane);
  }
}

}  // namespace pck
