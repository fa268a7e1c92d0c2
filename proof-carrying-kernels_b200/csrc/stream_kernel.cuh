// The persistent streaming kernel: GEMV rows, checksum-bank segments and the block
// verdicts of the trusted checker, for every job of a launch plan (stream_plan.h).
//
// Data path (kTma): one producer warp streams each unit's bytes from HBM into a ring of
// shared-memory stages with cp.async.bulk (completion counted on a per-stage mbarrier);
// the activations X of the CTA's job are copied to shared memory once. C consumer warps
// (C <= 8, the stage count a multiple of C) take the units in turn: warp w reduces units
// w, w + C, ... of the CTA's range and hands each stage back through its "empty" mbarrier.
// Unit i uses stage i mod stages, so every use of a stage belongs to the same warp: a
// warp waiting for use u of its stage has itself consumed use u - 1, which keeps the
// mbarrier's phase within one of the awaited one and the parity wait exact. Without kTma (unaligned pointers,
// n not a multiple of the vector width) the consumer warps read global memory directly
// with scalar loads; the arithmetic is identical.
//
// GEMV row arithmetic (bit-exact with the reference's model of its coalesced kernel,
// src/pck/gemv.py:71-101 / src/pck/cuda/csrc/gemv_kernel.cu:139-178): with T = 32*NV
// chains, chain t = 32*w + l owns vectors t, t + T, ... of V columns (V = 8 bfloat16 or
// 16 E4M3 weights per 16-byte vector). Lane l of the warp holds the NV chains
// l, 32 + l, ..., 32*(NV-1) + l of the row in registers and adds each chain's products in
// order (binary32 product, then binary32 sum; an E4M3 x bfloat16 product is exact, so
// when no product can overflow the pair is one FMA). The chains of each group of 32 are
// combined by the halving tree (i += i + 16, ..., i += i + 1) and the NV group sums by
// halving again; the exchange scheme in `halve_groups` evaluates exactly those additions
// while moving only half of the live values at each level.
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
  int64_t row;   // kUnitRow
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
    x.row = u;
    x.src = static_cast<const uint8_t*>(jb.W) + u * jb.row_bytes;
    x.bytes = static_cast<uint32_t>(jb.row_bytes);
    return x;
  }
  const int64_t beta = u / jb.period_units;
  int64_t o = u - beta * jb.period_units;
  x.beta = beta;
  const int64_t bw = jb.has_w ? jb.block : 0;
  if (o < bw) {
    x.kind = kUnitRow;
    x.row = beta * jb.block + o;
    x.src = static_cast<const uint8_t*>(jb.W) + x.row * jb.row_bytes;
    x.bytes = static_cast<uint32_t>(jb.row_bytes);
    return x;
  }
  o -= bw;
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
  if (!jb.has_check) return ceil_div64(target, jb.row_bytes);
  const int64_t beta = target / jb.period_bytes;
  int64_t rem = target - beta * jb.period_bytes;
  const int64_t base = beta * jb.period_units;
  if (rem == 0) return base;
  const int64_t bw = jb.has_w ? jb.block : 0;
  const int64_t wbytes = bw * jb.row_bytes;
  if (rem <= wbytes) return base + ceil_div64(rem, jb.row_bytes);
  rem -= wbytes;
  const int64_t crow = 4 * jb.n;
  const int64_t cbytes = jb.checks * crow;
  if (rem <= cbytes) {
    const int64_t k = rem / crow;
    const int64_t r3 = rem - k * crow;
    return base + bw + k * jb.segs + ceil_div64(r3, 4 * jb.seg_len);
  }
  rem -= cbytes;
  return base + bw + static_cast<int64_t>(jb.checks) * jb.segs + ceil_div64(rem, 2 * jb.seg_len);
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

// One unit: reduce it and store its result.
template <int WFMT, int NV, int BG, bool kFast, bool kFma>
__device__ __forceinline__ void run_unit(const JobPlan& jb, const Unit& un, const uint8_t* data,
                                         const uint16_t* X, int lane) {
  if (un.kind == kUnitRow) {
    gemv_row<WFMT, NV, BG, kFast, kFma>(data, X, jb.n, jb.batch, jb.Y, jb.m, un.row, lane);
  } else if (un.kind == kUnitC) {
    const int64_t nb = jb.num_blocks;
    double* out = jb.partial_cx + (static_cast<int64_t>(un.k) * nb + un.beta) * jb.seg_alloc + un.s;
    const int64_t stride = static_cast<int64_t>(jb.checks) * nb * jb.seg_alloc;
    c_segment<kFast>(reinterpret_cast<const float*>(data), X, jb.n, jb.batch, un.col0, un.len, out,
                     stride, lane);
  } else {
    const int64_t nb = jb.num_blocks;
    double* out = jb.partial_s + un.beta * jb.seg_alloc + un.s;
    a_segment<kFast>(reinterpret_cast<const uint16_t*>(data), X, jb.n, jb.batch, un.col0, un.len,
                     out, nb * jb.seg_alloc, lane);
  }
}

// E4M3 x bfloat16 products are exact; an FMA equals product-then-sum unless a product
// overflows, which needs |x| >= 2^128 / 448. True when every |x| < 2^119 and finite.
__device__ __forceinline__ bool x_allows_fma(const uint16_t* X, int64_t count, int first, int step) {
  bool ok = true;
  for (int64_t j = first; j < count; j += step) ok &= (X[j] & 0x7fffu) < 0x7b00u;
  return ok;
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
  const bool e4m3 = WFMT == kWeightsE4m3 && jb.has_w;

  if constexpr (kTma) {
    const int stages = plan.stages;
    uint8_t* xs = smem;
    uint8_t* ring = smem + plan.x_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<int64_t>(stages) * plan.stage_bytes);
    uint64_t* empty = full + stages;
    uint64_t* xbar = empty + stages;
    uint32_t* flag = reinterpret_cast<uint32_t*>(xbar + 1);
    if (threadIdx.x == 0) {
      for (int s = 0; s < stages; ++s) {
        mbar_init(full + s, 1);
        mbar_init(empty + s, 1);
      }
      mbar_init(xbar, 1);
      *flag = 0;
      fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {  // producer
      if (lane == 0) {
        const uint64_t keep = policy_evict_last();
        const uint64_t stream = policy_evict_first();
        const uint32_t xbytes = static_cast<uint32_t>(static_cast<int64_t>(jb.batch) * jb.n * 2);
        mbar_arrive_expect_tx(xbar, xbytes);
        bulk_load(xs, jb.X, xbytes, xbar, keep);
        int64_t issued = 0;
        for (int64_t i = 0; i < count; ++i) {
          const int st = static_cast<int>(i % stages);
          if (i >= stages && !mbar_wait(empty + st, static_cast<uint32_t>((i / stages - 1) & 1))) break;
          const Unit un = decode_unit(jb, u0 + i);
          mbar_arrive_expect_tx(full + st, un.bytes);
          bulk_load(ring + static_cast<int64_t>(st) * plan.stage_bytes, un.src, un.bytes, full + st,
                    stream);
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
    const int consumers = plan.consumers;
    if (warp >= consumers) return;  // idle warp (stages too large for eight)
    const uint16_t* X = reinterpret_cast<const uint16_t*>(xs);
    const bool have_x = mbar_wait(xbar, 0);
    if (e4m3) {
      if (have_x && !x_allows_fma(X, static_cast<int64_t>(jb.batch) * jb.n,
                                  static_cast<int>(threadIdx.x), consumers * kWarp)) {
        atomicOr(flag, 1u);
      }
      named_barrier(1, consumers * kWarp);
    }
    if (!have_x) return;
    const bool fma = e4m3 && *flag == 0;

    int64_t cur_beta = -1;
    uint32_t pending = 0;
    for (int64_t i = warp; i < count; i += consumers) {
      const int st = static_cast<int>(i % stages);
      if (!mbar_wait(full + st, static_cast<uint32_t>((i / stages) & 1))) return;
      const Unit un = decode_unit(jb, u0 + i);
      const uint8_t* data = ring + static_cast<int64_t>(st) * plan.stage_bytes;
      if (fma) {
        run_unit<WFMT, NV, BG, true, true>(jb, un, data, X, lane);
      } else {
        run_unit<WFMT, NV, BG, true, false>(jb, un, data, X, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);
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
  } else {
    // Plain path: every warp is a consumer and reads global memory directly, one element
    // at a time (product, then sum: the same values as the fast path's).
    (void)e4m3;
    const uint16_t* X = jb.X;
    int64_t cur_beta = -1;
    uint32_t pending = 0;
    for (int64_t i = warp; i < count; i += kConsumerWarps) {
      const Unit un = decode_unit(jb, u0 + i);
      run_unit<WFMT, NV, BG, false, false>(jb, un, static_cast<const uint8_t*>(un.src), X, lane);
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
