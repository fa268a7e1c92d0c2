// The persistent streaming kernel: GEMV rows and the checksum-bank segments of the trusted
// checker, for every job of a launch plan (stream_plan.h). The block verdicts follow in the
// verdict kernel (verdict_kernel.cu), or in the next streaming launch (Plan::prior: a few
// CTAs of that launch, past the streaming ones, decide the earlier launch's blocks while the
// others stream; the streaming warps run no verdict code).
//
// Staged path (kTma): each of the 16 consumer warps of a CTA owns the units w, w + 16, ... of the
// CTA's range and streams them through its own ring of `slots` shared-memory pieces with
// cp.async.bulk: lane 0 arms the piece's mbarrier with the expected bytes and issues the
// copy; the warp waits for the barrier's phase, reduces the piece, and refills the same
// slot with its next piece. Each slot is used by one warp in order, so every parity wait
// is exact. Rows longer than a piece are split at vector-iteration boundaries and their
// chains carry over in registers. The activations X of the CTA's job are copied to shared
// memory once, after the weight prefetch. Plain path (unaligned pointers, n not a multiple of the vector width): the
// same units read straight from global memory with scalar loads; the arithmetic is the
// same.
//
// GEMV row arithmetic (bit-exact with the reference's model of its coalesced kernel,
// src/pck/gemv.py:71-101 / src/pck/cuda/csrc/gemv_kernel.cu:139-178): with T = 32*NV
// chains, chain t = 32*g + l (group g, lane l) owns vectors t, t + T, ... of V columns
// (V = 8 bfloat16 or 16 E4M3 weights per 16-byte vector) and adds its products in order
// (binary32 product, then binary32 sum — or one FMA where the product is provably exact).
// Lane l holds the NV chains l, 32 + l, ... of the row; each group of 32 chains is reduced
// by halving across lanes (l += l + 16, ..., l += l + 1) and the NV group sums by halving
// again (g += g + NV/2, ..., g += g + 1); `halve_groups` evaluates exactly those additions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"
#include "stream_plan.h"
#include "verdict_task.cuh"

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


// Unit o of row block beta of a checked job.
__device__ __forceinline__ Unit decode_checked(const JobPlan& jb, int64_t beta, int64_t o) {
  Unit x{};
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
  const int oc = static_cast<int>(o - ru);
  const int cs = jb.checks * jb.segs;
  if (oc < cs) {
    x.kind = kUnitC;
    x.k = oc / jb.segs;
    x.s = oc - x.k * jb.segs;
    x.col0 = x.s * jb.seg_len;
    x.len = min(jb.seg_len, jb.n - x.col0);
    x.src = jb.c + (static_cast<int64_t>(x.k) * jb.num_blocks + beta) * jb.n + x.col0;
    x.bytes = static_cast<uint32_t>(x.len * 4);
    return x;
  }
  x.kind = kUnitA;
  x.s = oc - cs;
  x.col0 = x.s * jb.seg_len;
  x.len = min(jb.seg_len, jb.n - x.col0);
  x.src = jb.a + beta * jb.n + x.col0;
  x.bytes = static_cast<uint32_t>(x.len * 2);
  return x;
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

// One vector of 16 E4M3 weights against 16 binary16 activations (xa: columns 0-7, xb: 8-15),
// each product added with one mixed-precision FMA. Used only when every activation is
// exactly a binary16 value: an E4M3 x binary16 product then has at most 12 significant bits
// and lies in [2^-33, 2^25], so it is exact in binary32 and the FMA equals product-then-sum.
__device__ __forceinline__ void chain_e4m3_half(float& acc, const uint4 w, const uint4 xa, const uint4 xb) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  const uint32_t xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    asm("{\n\t.reg .b16 p0, p1, w0, w1, w2, w3, x0, x1, x2, x3;\n\t.reg .b32 h01, h23;\n\t"
        "mov.b32 {p0, p1}, %1;\n\t"
        "cvt.rn.f16x2.e4m3x2 h01, p0;\n\tcvt.rn.f16x2.e4m3x2 h23, p1;\n\t"
        "mov.b32 {w0, w1}, h01;\n\tmov.b32 {w2, w3}, h23;\n\t"
        "mov.b32 {x0, x1}, %2;\n\tmov.b32 {x2, x3}, %3;\n\t"
        "fma.rn.f32.f16 %0, w0, x0, %0;\n\tfma.rn.f32.f16 %0, w1, x1, %0;\n\t"
        "fma.rn.f32.f16 %0, w2, x2, %0;\n\tfma.rn.f32.f16 %0, w3, x3, %0;\n\t}"
        : "+f"(acc)
        : "r"(ws[i]), "r"(xs[2 * i]), "r"(xs[2 * i + 1]));
  }
}

// kMode: 0 product then sum, 1 one FMA per product (exact products), 2 the E4M3 weights
// against binary16 activations (chain_e4m3_half).
template <int kMode>
__device__ __forceinline__ void chain_e4m3_mode(float& acc, const uint4 w, const uint4 xa, const uint4 xb) {
  if constexpr (kMode == 2) {
    chain_e4m3_half(acc, w, xa, xb);
  } else {
    chain_e4m3<kMode != 0>(acc, w, xa, xb);
  }
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
    } else {  // the same element order as above: lane l takes 4l..4l+3, then + 128
      for (int64_t j = lane * 4; j < len; j += 4 * kWarp) {
        for (int64_t e = j; e < j + 4 && e < len; ++e) {
          acc = __fma_rn(static_cast<double>(cs[e]), static_cast<double>(bf16_bits_to_float(xb[e])), acc);
        }
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
    } else {  // the same element order as above
      for (int64_t j = lane * 4; j < len; j += 4 * kWarp) {
        for (int64_t e = j; e < j + 4 && e < len; ++e) {
          acc = __fma_ru(static_cast<double>(bf16_bits_to_float(as[e])),
                         fabs(static_cast<double>(bf16_bits_to_float(xb[e]))), acc);
        }
      }
    }
    acc = warp_sum_ru(acc);
    if (lane == 0) out[b * out_stride] = acc;
  }
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
// Staged path: every warp streams its own units through a private ring of pieces.

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

// Orders this thread's earlier shared-memory reads before a later bulk copy into the same
// bytes (generic proxy, then async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Row accumulators of one warp: NV chains per lane for each of BG batch columns.
template <int WFMT, int NV, int BG>
struct RowState {
  float acc[BG][NV];
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int b = 0; b < BG; ++b)
#pragma unroll
      for (int g = 0; g < NV; ++g) acc[b][g] = -0.0f;  // -0 + p == p for every p
  }
};

// Eight bfloat16 weights w (one 16-byte vector) times eight bfloat16 activations x, added
// to a chain in element order with the mixed-precision multiply-add of sm_100
// (fma.rn.f32.bf16: the exact product plus the binary32 chain, rounded once). kFma: one
// instruction per term — equal to product-then-sum because the product is exact.
// Otherwise the product is rounded first (fma with -0 addend, which is RN(w*x) for every
// input, signed zeros included) and added with its own rounding, as the reference does.
template <bool kFma>
__device__ __forceinline__ void chain8_bf16(float& acc, const uint4 w, const uint4 x) {
  if constexpr (kFma) {
    asm("{\n\t.reg .b16 w0, w1, x0, x1;\n\t"
        "mov.b32 {w0, w1}, %1;\n\tmov.b32 {x0, x1}, %5;\n\t"
        "fma.rn.f32.bf16 %0, w0, x0, %0;\n\tfma.rn.f32.bf16 %0, w1, x1, %0;\n\t"
        "mov.b32 {w0, w1}, %2;\n\tmov.b32 {x0, x1}, %6;\n\t"
        "fma.rn.f32.bf16 %0, w0, x0, %0;\n\tfma.rn.f32.bf16 %0, w1, x1, %0;\n\t"
        "mov.b32 {w0, w1}, %3;\n\tmov.b32 {x0, x1}, %7;\n\t"
        "fma.rn.f32.bf16 %0, w0, x0, %0;\n\tfma.rn.f32.bf16 %0, w1, x1, %0;\n\t"
        "mov.b32 {w0, w1}, %4;\n\tmov.b32 {x0, x1}, %8;\n\t"
        "fma.rn.f32.bf16 %0, w0, x0, %0;\n\tfma.rn.f32.bf16 %0, w1, x1, %0;\n\t}"
        : "+f"(acc)
        : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
  } else {
    asm("{\n\t.reg .b16 w0, w1, x0, x1;\n\t.reg .f32 p;\n\t"
        "mov.b32 {w0, w1}, %1;\n\tmov.b32 {x0, x1}, %5;\n\t"
        "fma.rn.f32.bf16 p, w0, x0, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "fma.rn.f32.bf16 p, w1, x1, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "mov.b32 {w0, w1}, %2;\n\tmov.b32 {x0, x1}, %6;\n\t"
        "fma.rn.f32.bf16 p, w0, x0, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "fma.rn.f32.bf16 p, w1, x1, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "mov.b32 {w0, w1}, %3;\n\tmov.b32 {x0, x1}, %7;\n\t"
        "fma.rn.f32.bf16 p, w0, x0, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "fma.rn.f32.bf16 p, w1, x1, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "mov.b32 {w0, w1}, %4;\n\tmov.b32 {x0, x1}, %8;\n\t"
        "fma.rn.f32.bf16 p, w0, x0, %9;\n\tadd.rn.f32 %0, %0, p;\n\t"
        "fma.rn.f32.bf16 p, w1, x1, %9;\n\tadd.rn.f32 %0, %0, p;\n\t}"
        : "+f"(acc)
        : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w),
          "f"(-0.0f));
  }
}

// One bfloat16 x bfloat16 term, element `hi` (0 = low half) of the words w and x.
template <bool kFma, int kHi>
__device__ __forceinline__ void term_bf16(float& acc, uint32_t w, uint32_t x) {
  if constexpr (kFma) {
    if constexpr (kHi) {
      asm("{\n\t.reg .b16 a, b, c, d;\n\tmov.b32 {a, b}, %1;\n\tmov.b32 {c, d}, %2;\n\t"
          "fma.rn.f32.bf16 %0, b, d, %0;\n\t}" : "+f"(acc) : "r"(w), "r"(x));
    } else {
      asm("{\n\t.reg .b16 a, b, c, d;\n\tmov.b32 {a, b}, %1;\n\tmov.b32 {c, d}, %2;\n\t"
          "fma.rn.f32.bf16 %0, a, c, %0;\n\t}" : "+f"(acc) : "r"(w), "r"(x));
    }
  } else {
    acc = __fadd_rn(acc, __fmul_rn(kHi ? bf16_hi(w) : bf16_lo(w), kHi ? bf16_hi(x) : bf16_lo(x)));
  }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// The vector iterations [v_lo, v_hi) of a row against columns [g0, g0 + BG) of X. The piece
// holds the row bytes from vector v_lo * T on; vector q of the row is at
// piece + (q - v_lo * T) * 16. nvec = n / V (n % V == 0 on this path). The shared-memory
// loads of an iteration are issued together, before its arithmetic.
template <int WFMT, int NV, int BG, int kMode>
__device__ __forceinline__ void reduce_row_piece(RowState<WFMT, NV, BG>& st, uint32_t piece, uint32_t xs,
                                                 uint32_t xcol, int g0, int batch, int v_lo, int v_hi,
                                                 int nvec, int lane) {
  constexpr int T = NV * kWarp;
  // bytes between the activations of consecutive vectors: bfloat16 rows keep columns in
  // order (16 bytes a vector); E4M3 rows keep each column in halves (load_activations), the
  // second half xcol / 2 bytes after the first
  constexpr uint32_t kXV = 16;
  const uint32_t xhalf = xcol / 2;
  uint32_t xcol_addr[BG];
#pragma unroll
  for (int b = 0; b < BG; ++b) xcol_addr[b] = xs + static_cast<uint32_t>(min(g0 + b, batch - 1)) * xcol;
  for (int v = v_lo; v < v_hi; ++v) {
    const uint32_t wbase = piece + static_cast<uint32_t>((v - v_lo) * T + lane) * 16u;
    const uint32_t xoff = static_cast<uint32_t>(v * T + lane) * kXV;
    // Vectors of this iteration inside the row (all T but in the last one). Chains past the
    // row's end add +0. A partial iteration whose valid vectors fill whole blocks of kStep
    // groups (the 14336-column E4M3 rows: 4 of 8 groups) takes the grouped path below.
    constexpr int kStep = NV < 4 ? NV : 4;
    const int valid = nvec - v * T;
    if (valid < T && valid % (kStep * kWarp) != 0) {  // a ragged last iteration, lane by lane
      const int qbase = v * T + lane;
#pragma unroll
      for (int g = 0; g < NV; ++g) {
        const bool in = qbase + g * kWarp < nvec;
        const uint4 wv = in ? lds128(wbase + g * (kWarp * 16u)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int b = 0; b < BG; ++b) {
          if (!in) {
            st.acc[b][g] = __fadd_rn(st.acc[b][g], 0.0f);
            continue;
          }
          const uint32_t xaddr = xcol_addr[b] + xoff + g * (kWarp * kXV);
          if constexpr (WFMT == kWeightsBf16) {
            chain8_bf16<kMode != 0>(st.acc[b][g], wv, lds128(xaddr));
          } else {
            chain_e4m3_mode<kMode>(st.acc[b][g], wv, lds128(xaddr), lds128(xaddr + xhalf));
          }
        }
      }
      continue;
    }
    // chain groups four at a time: their loads together, then their terms interleaved
#pragma unroll
    for (int g0w = 0; g0w < NV; g0w += kStep) {
      if (g0w * kWarp >= valid) {  // past the row's end (uniform for the warp)
#pragma unroll
        for (int b = 0; b < BG; ++b)
#pragma unroll
          for (int g = 0; g < kStep; ++g) st.acc[b][g0w + g] = __fadd_rn(st.acc[b][g0w + g], 0.0f);
        continue;
      }
      uint4 wv[kStep];
#pragma unroll
      for (int g = 0; g < kStep; ++g) wv[g] = lds128(wbase + (g0w + g) * (kWarp * 16u));
#pragma unroll
      for (int b = 0; b < BG; ++b) {
        if constexpr (WFMT == kWeightsBf16) {
          uint4 xv[kStep];
#pragma unroll
          for (int g = 0; g < kStep; ++g) xv[g] = lds128(xcol_addr[b] + xoff + (g0w + g) * (kWarp * kXV));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int g = 0; g < kStep; ++g) term_bf16<kMode != 0, 0>(st.acc[b][g0w + g], word(wv[g], i), word(xv[g], i));
#pragma unroll
            for (int g = 0; g < kStep; ++g) term_bf16<kMode != 0, 1>(st.acc[b][g0w + g], word(wv[g], i), word(xv[g], i));
          }
        } else {
          uint4 xa[kStep], xb[kStep];
#pragma unroll
          for (int g = 0; g < kStep; ++g) {
            xa[g] = lds128(xcol_addr[b] + xoff + (g0w + g) * (kWarp * kXV));
            xb[g] = lds128(xcol_addr[b] + xoff + (g0w + g) * (kWarp * kXV) + xhalf);
          }
#pragma unroll
          for (int g = 0; g < kStep; ++g) chain_e4m3_mode<kMode>(st.acc[b][g0w + g], wv[g], xa[g], xb[g]);
        }
      }
    }
  }
}

// Elements [e_lo, e_hi) of a c- or a-segment (element e of the piece at piece + e * size):
// lane l adds elements 4l..4l+3, then + 128, ..., in order — the same order as the plain
// path's c_segment / a_segment over the whole segment when e_lo is a multiple of 128.
template <bool kAbs>
__device__ __forceinline__ void segment_piece(double* acc, uint32_t piece, uint32_t xs, uint32_t xcol,
                                              int64_t col0, int batch, int e_lo, int e_hi, int lane) {
  for (int e = e_lo + lane * 4; e < e_hi; e += 4 * kWarp) {
    const uint32_t off = static_cast<uint32_t>(e - e_lo);
    uint4 cv;
    uint2 av;
    if constexpr (kAbs) {
      av = lds64(piece + off * 2);
    } else {
      cv = lds128(piece + off * 4);
    }
#pragma unroll
    for (int b = 0; b < kSegBatch; ++b) {
      if (b >= batch) break;
      const uint2 xv = lds64(xs + static_cast<uint32_t>(b) * xcol + static_cast<uint32_t>(col0 + e) * 2);
      double a = acc[b];
      if constexpr (kAbs) {
        a = __fma_ru(static_cast<double>(bf16_lo(av.x)), fabs(static_cast<double>(bf16_lo(xv.x))), a);
        a = __fma_ru(static_cast<double>(bf16_hi(av.x)), fabs(static_cast<double>(bf16_hi(xv.x))), a);
        a = __fma_ru(static_cast<double>(bf16_lo(av.y)), fabs(static_cast<double>(bf16_lo(xv.y))), a);
        a = __fma_ru(static_cast<double>(bf16_hi(av.y)), fabs(static_cast<double>(bf16_hi(xv.y))), a);
      } else {
        a = __fma_rn(static_cast<double>(__uint_as_float(cv.x)), static_cast<double>(bf16_lo(xv.x)), a);
        a = __fma_rn(static_cast<double>(__uint_as_float(cv.y)), static_cast<double>(bf16_hi(xv.x)), a);
        a = __fma_rn(static_cast<double>(__uint_as_float(cv.z)), static_cast<double>(bf16_lo(xv.y)), a);
        a = __fma_rn(static_cast<double>(__uint_as_float(cv.w)), static_cast<double>(bf16_hi(xv.y)), a);
      }
      acc[b] = a;
    }
  }
}

// Copies the activations X (batch * n bfloat16, a multiple of 16 bytes, 16-byte aligned)
// into shared memory with one 16-byte load per thread and step, through L2 (X may have been
// written by the kernel this one waited for), and merges the smallest nonzero (subnormals
// counted as 1) and the largest exponent field into xexp[0..1].
// E4M3 rows (16 weights, 32 bytes of activations per vector) keep each column in halves:
// the first 16 bytes of every vector, then the second 16 bytes (n bytes on), so a warp's
// 16-byte loads of one half are contiguous and free of bank conflicts.
template <int WFMT>
__device__ __forceinline__ void load_activations(const JobPlan& jb, uint8_t* xs, uint32_t* xexp, int tid,
                                                 int lane) {
  const int64_t words = static_cast<int64_t>(jb.batch) * jb.n / 8;
  const uint4* src = reinterpret_cast<const uint4*>(jb.X);
  uint4* dst = reinterpret_cast<uint4*>(xs);
  const bool split = WFMT == kWeightsE4m3 && jb.has_w;  // n % 16 == 0 on the staged path
  const uint32_t cw = static_cast<uint32_t>(jb.n / 8);  // 16-byte words per column
  unsigned mn = 1000, mx = 0;
  // Up to kXLoads loads of a thread in flight before any store: the activations come after
  // the producer wait, while HBM traffic makes every L2 round trip long.
  constexpr int kXLoads = 4;
  for (int64_t base = tid; base < words; base += kXLoads * kPlainThreads) {
    uint4 vs[kXLoads];
#pragma unroll
    for (int u = 0; u < kXLoads; ++u) {
      const int64_t i = base + static_cast<int64_t>(u) * kPlainThreads;
      if (i < words) vs[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < kXLoads; ++u) {
      const int64_t i = base + static_cast<int64_t>(u) * kPlainThreads;
      if (i >= words) break;
      const uint4 v = vs[u];
      if (split) {
        const uint32_t b = static_cast<uint32_t>(i) / cw, w = static_cast<uint32_t>(i) - b * cw;
        dst[b * cw + (w & 1u) * (cw / 2) + (w >> 1)] = v;
      } else {
        dst[i] = v;
      }
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const unsigned mag = (h & 1 ? w[h / 2] >> 16 : w[h / 2]) & 0x7fffu;
        const unsigned e = mag >> 7;
        mx = max(mx, e);
        if (mag) mn = min(mn, max(e, 1u));
      }
    }
  }
  if (jb.has_w) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = min(mn, __shfl_xor_sync(kFullMask, mn, o));
      mx = max(mx, __shfl_xor_sync(kFullMask, mx, o));
    }
    if (lane == 0) {
      atomicMin(xexp, mn);
      atomicMax(xexp + 1, mx);
    }
  }
}

// Rewrites the bfloat16 activations in shared memory as binary16 (each value exact: the
// caller has checked every exponent field is in [110, 142]; zeros stay zeros).
__device__ __forceinline__ void activations_to_half(const JobPlan& jb, uint8_t* xs, int tid) {
  const int64_t words = static_cast<int64_t>(jb.batch) * jb.n / 8;
  uint4* p = reinterpret_cast<uint4*>(xs);
  for (int64_t i = tid; i < words; i += kPlainThreads) {
    uint4 v = p[i];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float lo = __uint_as_float(w[h] << 16);
      const float hi = __uint_as_float(w[h] & 0xffff0000u);
      const __half2 pair = __floats2half2_rn(lo, hi);
      w[h] = *reinterpret_cast<const uint32_t*>(&pair);
    }
    p[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
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

// A warp's walk over its pieces: units warp, warp + 8, ... of the CTA's range, each cut
// into pieces.
// Rows are cut into pieces of row_piece bytes (whole vector iterations), checksum-bank
// segments into pieces of seg_piece bytes (a multiple of 512, so every piece starts at a
// multiple of 128 elements and the lanes add the elements in one fixed order).
struct PieceWalk {
  int64_t unit;   // CTA-local unit index
  int64_t beta;   // checked jobs: row block of `unit` ...
  int64_t o;      // ... and its index within the block
  int piece;
  int pieces;     // pieces of `unit` (0: the walk is over)
  uint32_t size;  // piece size of `unit`
};

// The unit a walk stands on (decoded again where needed: cheaper than keeping it).
__device__ __forceinline__ Unit walk_unit(const PieceWalk& w, const JobPlan& jb, int64_t u0) {
  return jb.has_check ? decode_checked(jb, w.beta, w.o) : decode_unit(jb, u0 + w.unit);
}

__device__ __forceinline__ void walk_load(PieceWalk& w, const JobPlan& jb, int64_t u0, int64_t count,
                                          uint32_t row_piece, uint32_t seg_piece) {
  w.piece = 0;
  if (w.unit < count) {
    const Unit un = walk_unit(w, jb, u0);
    w.size = un.kind == kUnitRow ? row_piece : seg_piece;
    w.pieces = static_cast<int>((un.bytes + w.size - 1) / w.size);
  } else {
    w.pieces = 0;
  }
}

// Start at CTA-local unit `local` (one division, at the start only).
__device__ __forceinline__ void walk_to(PieceWalk& w, const JobPlan& jb, int64_t u0, int64_t local,
                                        int64_t count, uint32_t row_piece, uint32_t seg_piece) {
  w.unit = local;
  if (jb.has_check) {
    w.beta = (u0 + local) / jb.period_units;
    w.o = u0 + local - w.beta * jb.period_units;
  }
  walk_load(w, jb, u0, count, row_piece, seg_piece);
}

// Next piece; after the last piece of a unit, the unit kConsumerWarps further on.
__device__ __forceinline__ void walk_next(PieceWalk& w, const JobPlan& jb, int64_t u0, int64_t count,
                                          uint32_t row_piece, uint32_t seg_piece) {
  if (++w.piece < w.pieces) return;
  w.unit += kConsumerWarps;
  if (jb.has_check) {
    w.o += kConsumerWarps;
    while (w.o >= jb.period_units) {
      w.o -= jb.period_units;
      ++w.beta;
    }
  }
  walk_load(w, jb, u0, count, row_piece, seg_piece);
}

// The consuming half of staged_warp (see there); `issue` and `issued` continue the walk
// that primed the ring.
template <int WFMT, int NV, int BG, int kMode>
__device__ __forceinline__ void staged_consume(const JobPlan& jb, int64_t u0, int64_t count, int slots,
                                               uint32_t slot_bytes, uint32_t row_piece, uint8_t* ring,
                                               uint64_t* full, uint32_t xs, int warp, int lane,
                                               PieceWalk issue, int64_t issued) {
  constexpr int V = Format<WFMT>::kVec;
  constexpr int T = NV * kWarp;
  const uint64_t once = policy_evict_first();
  const uint32_t ring_addr = smem_addr(ring);
  const uint32_t xcol = static_cast<uint32_t>(jb.n * 2);
  const int nvec = static_cast<int>(jb.n / V);
  const int vtotal = (nvec + T - 1) / T;
  const uint32_t seg_piece = slot_bytes / 512u * 512u;
  PieceWalk take;
  walk_to(take, jb, u0, warp, count, row_piece, seg_piece);
  int64_t taken = 0;
  auto issue_one = [&](int slot) {  // into `slot`, the one just consumed
    if (lane == 0) {
      const Unit iu = walk_unit(issue, jb, u0);
      const uint32_t off = static_cast<uint32_t>(issue.piece) * issue.size;
      const uint32_t bytes = min(issue.size, iu.bytes - off);
      mbar_arrive_expect_tx(full + slot, bytes);
      bulk_load(ring + static_cast<int64_t>(slot) * slot_bytes, static_cast<const uint8_t*>(iu.src) + off,
                bytes, full + slot, once);
    }
    ++issued;
    walk_next(issue, jb, u0, count, row_piece, seg_piece);
  };

  RowState<WFMT, NV, BG> row;
  double dacc[kSegBatch];  // indexed only by unrolled loops: registers
  int slot = 0;  // the slot of piece `taken`, and its phase parity
  uint32_t phase = 0;
  while (take.pieces > 0) {
    if (!mbar_wait(full + slot, phase)) break;
    const uint32_t piece = ring_addr + static_cast<uint32_t>(slot) * slot_bytes;
    const Unit un = walk_unit(take, jb, u0);
    const bool first = take.piece == 0;
    const bool last = take.piece + 1 == take.pieces;
    if (un.kind == kUnitRow) {
      // one piece per column group when the batch exceeds BG (the host keeps such rows whole)
      // vector iterations in this piece (pieces of a multi-piece row are whole iterations)
      const uint32_t off = static_cast<uint32_t>(take.piece) * take.size;
      const uint32_t bytes = min(take.size, un.bytes - off);
      const int v_lo = static_cast<int>(off / (T * 16u));
      const int v_hi = min(static_cast<int>((off + bytes + T * 16u - 1) / (T * 16u)), vtotal);
      for (int g0 = 0; g0 < jb.batch; g0 += BG) {
        if (first) row.reset();
        reduce_row_piece<WFMT, NV, BG, kMode>(row, piece, xs, xcol, g0, jb.batch, v_lo, v_hi, nvec, lane);
        if (last) {
#pragma unroll
          for (int b = 0; b < BG; ++b) {
            const float yv = halve_groups<NV>(row.acc[b], lane);
            if (lane == 0 && g0 + b < jb.batch) jb.Y[static_cast<int64_t>(g0 + b) * jb.m + un.row] = yv;
          }
        }
      }
    } else {
      if (first) {
#pragma unroll
        for (int b = 0; b < kSegBatch; ++b) dacc[b] = 0.0;
      }
      const int esz = un.kind == kUnitC ? 4 : 2;
      const int e_lo = static_cast<int>(static_cast<int64_t>(take.piece) * take.size / esz);
      const int e_hi = static_cast<int>(min(static_cast<int64_t>(e_lo) + take.size / esz, un.len));
      if (un.kind == kUnitC) {
        segment_piece<false>(dacc, piece, xs, xcol, un.col0, jb.batch, e_lo, e_hi, lane);
      } else {
        segment_piece<true>(dacc, piece, xs, xcol, un.col0, jb.batch, e_lo, e_hi, lane);
      }
      if (last) {
        const int64_t nb = jb.num_blocks;
#pragma unroll
        for (int b = 0; b < kSegBatch; ++b) {
          if (b >= jb.batch) break;
          if (un.kind == kUnitC) {
            const double t = warp_sum_rn(dacc[b]);
            if (lane == 0) {
              jb.partial_cx[((static_cast<int64_t>(b) * jb.checks + un.k) * nb + un.beta) * jb.seg_alloc + un.s] = t;
            }
          } else {
            const double t = warp_sum_ru(dacc[b]);
            if (lane == 0) jb.partial_s[(static_cast<int64_t>(b) * nb + un.beta) * jb.seg_alloc + un.s] = t;
          }
        }
      }
    }
    __syncwarp();
    ++taken;
    if (issue.pieces > 0) {  // refill the slot just consumed
      if (lane == 0) fence_proxy_async_smem();
      issue_one(slot);
    }
    if (++slot == slots) {
      slot = 0;
      phase ^= 1u;
    }
    walk_next(take, jb, u0, count, row_piece, seg_piece);
  }
  // Leave only after every copy into this warp's slots has landed.
  for (int64_t i = taken; i < issued; ++i) mbar_wait(full + i % slots, static_cast<uint32_t>((i / slots) & 1));
}

// ---------------------------------------------------------------------------------------
// Bank CTAs: the staged path of a check-only job, with its own lean walk. A warp's units are
// u0 + warp, + 16, ...; a cursor keeps the unit it stands on decoded and steps to the next
// without divisions, so a piece costs its arithmetic and little else. Same pieces, same
// element order and the same partial sums as the generic walk.
struct BankCursor {
  int64_t beta;        // row block of the unit
  int o;               // unit within the block: [checks x segs c-units][segs a-units]
  int piece;
  int pieces;          // 0: the walk is over
  int64_t left;        // units of this warp still to visit, this one included
  int kind;            // kUnitC or kUnitA
  int k;               // c-units: check
  int s;               // segment
  int col0;
  int len;             // columns of the segment
  const uint8_t* src;  // the unit's bytes
  uint32_t bytes;
};

__device__ __forceinline__ void bank_load(BankCursor& c, const JobPlan& jb, uint32_t piece_bytes) {
  c.piece = 0;
  if (c.left <= 0) {
    c.pieces = 0;
    return;
  }
  const int segs = jb.segs;
  const int cs = jb.checks * segs;
  int o = c.o;
  if (o < cs) {
    c.kind = kUnitC;
    c.k = 0;
    while (o >= segs) {  // checks is small
      o -= segs;
      ++c.k;
    }
    c.s = o;
  } else {
    c.kind = kUnitA;
    c.s = o - cs;
  }
  c.col0 = c.s * static_cast<int>(jb.seg_len);
  c.len = static_cast<int>(min(jb.seg_len, jb.n - c.col0));
  if (c.kind == kUnitC) {
    c.src = reinterpret_cast<const uint8_t*>(jb.c + (static_cast<int64_t>(c.k) * jb.num_blocks + c.beta) * jb.n + c.col0);
    c.bytes = static_cast<uint32_t>(c.len) * 4u;
  } else {
    c.src = reinterpret_cast<const uint8_t*>(jb.a + c.beta * jb.n + c.col0);
    c.bytes = static_cast<uint32_t>(c.len) * 2u;
  }
  c.pieces = static_cast<int>((c.bytes + piece_bytes - 1) / piece_bytes);
}

__device__ __forceinline__ void bank_start(BankCursor& c, const JobPlan& jb, int64_t u0, int64_t count, int warp,
                                           uint32_t piece_bytes) {
  const int64_t u = u0 + warp;
  c.beta = u / jb.period_units;
  c.o = static_cast<int>(u - c.beta * jb.period_units);
  c.left = warp < count ? (count - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
  bank_load(c, jb, piece_bytes);
}

__device__ __forceinline__ void bank_next(BankCursor& c, const JobPlan& jb, uint32_t piece_bytes) {
  if (++c.piece < c.pieces) return;
  --c.left;
  c.o += kConsumerWarps;
  const int period = static_cast<int>(jb.period_units);
  while (c.o >= period) {
    c.o -= period;
    ++c.beta;
  }
  bank_load(c, jb, piece_bytes);
}

// The bank warp: primes its ring, calls `before_inputs` (producer wait and activations; a
// negative return means leave), fills the ring, then reduces its units piece by piece.
template <typename Inputs>
__device__ __forceinline__ void bank_warp(const JobPlan& jb, int64_t u0, int64_t count, int slots, int pre_slots,
                                          uint32_t slot_bytes, uint8_t* ring, uint64_t* full, uint32_t xs,
                                          int warp, int lane, Inputs before_inputs) {
  const uint64_t once = policy_evict_first();
  const uint32_t piece_bytes = slot_bytes / 512u * 512u;  // a multiple of 128 elements
  const uint32_t ring_addr = smem_addr(ring);
  const uint32_t xcol = static_cast<uint32_t>(jb.n * 2);
  BankCursor issue, take;
  bank_start(issue, jb, u0, count, warp, piece_bytes);
  take = issue;
  int64_t issued = 0, taken = 0;
  auto issue_one = [&](int slot) {
    if (lane == 0) {
      const uint32_t off = static_cast<uint32_t>(issue.piece) * piece_bytes;
      const uint32_t bytes = min(piece_bytes, issue.bytes - off);
      mbar_arrive_expect_tx(full + slot, bytes);
      bulk_load(ring + static_cast<int64_t>(slot) * slot_bytes, issue.src + off, bytes, full + slot, once);
    }
    ++issued;
    bank_next(issue, jb, piece_bytes);
  };
  while (issued < min(slots, pre_slots) && issue.pieces > 0) issue_one(static_cast<int>(issued));
  const int mode = before_inputs();
  while (issued < slots && issue.pieces > 0) issue_one(static_cast<int>(issued));
  if (mode < 0) {
    for (int64_t i = 0; i < issued; ++i) mbar_wait(full + i, 0);
    return;
  }
  double dacc[kSegBatch];  // indexed only by unrolled loops: registers
  const int64_t nb = jb.num_blocks;
  int slot = 0;  // the slot of piece `taken`, and its phase parity
  uint32_t phase = 0;
  while (take.pieces > 0) {
    if (!mbar_wait(full + slot, phase)) break;
    const uint32_t piece = ring_addr + static_cast<uint32_t>(slot) * slot_bytes;
    if (take.piece == 0) {
#pragma unroll
      for (int b = 0; b < kSegBatch; ++b) dacc[b] = 0.0;
    }
    const bool is_c = take.kind == kUnitC;
    const int per_piece = static_cast<int>(piece_bytes >> (is_c ? 2 : 1));
    const int e_lo = take.piece * per_piece;
    const int e_hi = min(e_lo + per_piece, take.len);
    if (is_c) {
      segment_piece<false>(dacc, piece, xs, xcol, take.col0, jb.batch, e_lo, e_hi, lane);
    } else {
      segment_piece<true>(dacc, piece, xs, xcol, take.col0, jb.batch, e_lo, e_hi, lane);
    }
    if (take.piece + 1 == take.pieces) {
#pragma unroll
      for (int b = 0; b < kSegBatch; ++b) {
        if (b >= jb.batch) break;
        if (is_c) {
          const double t = warp_sum_rn(dacc[b]);
          if (lane == 0) {
            jb.partial_cx[((static_cast<int64_t>(b) * jb.checks + take.k) * nb + take.beta) * jb.seg_alloc + take.s] = t;
          }
        } else {
          const double t = warp_sum_ru(dacc[b]);
          if (lane == 0) jb.partial_s[(static_cast<int64_t>(b) * nb + take.beta) * jb.seg_alloc + take.s] = t;
        }
      }
    }
    __syncwarp();
    ++taken;
    if (issue.pieces > 0) {  // refill the slot just consumed
      if (lane == 0) fence_proxy_async_smem();
      issue_one(slot);
    }
    if (++slot == slots) {
      slot = 0;
      phase ^= 1u;
    }
    bank_next(take, jb, piece_bytes);
  }
  // Leave only after every copy into this warp's slots has landed.
  for (int64_t i = taken; i < issued; ++i) mbar_wait(full + i % slots, static_cast<uint32_t>((i / slots) & 1));
}

// ---------------------------------------------------------------------------------------
// Row CTAs: the staged path of a GEMV job without checks (one row per unit), with a lean walk.
// A warp's rows are u0 + warp, + 16, ...; every row is `ppr` pieces of row_piece bytes (the
// last one shorter), so a piece costs its arithmetic plus a few additions. Same pieces, same
// vector iterations per piece and the same chains as the generic walk.
struct RowCursor {
  int64_t row;
  int piece;
  int64_t left;  // rows of this warp still to visit, this one included
};

__device__ __forceinline__ void row_next(RowCursor& c, int ppr) {
  if (++c.piece < ppr) return;
  c.piece = 0;
  c.row += kConsumerWarps;
  --c.left;
}

// row_consume for E4M3 rows of exactly one vector iteration (n = 16 * T: the 4096-column
// projections at 256 threads), batch 1, binary16 activations, one piece per row: chain g of a
// lane always meets the same 16 activations (vector 32g + lane), so the lane keeps them in
// registers for all its rows and a row costs one shared load per vector. The terms and their
// order are those of reduce_row_piece's single iteration.
template <int NV>
__device__ __forceinline__ void row_consume_e4m3_xreg(const JobPlan& jb, int slots, uint32_t slot_bytes,
                                                      uint8_t* ring, uint64_t* full, uint32_t xs, int lane,
                                                      RowCursor issue, RowCursor take, int64_t issued) {
  const uint64_t once = policy_evict_first();
  const uint32_t ring_addr = smem_addr(ring);
  const uint32_t xhalf = static_cast<uint32_t>(jb.n);  // second halves, n bytes on (load_activations)
  const uint32_t row_bytes = static_cast<uint32_t>(jb.row_bytes);
  const uint8_t* W = static_cast<const uint8_t*>(jb.W);
  uint4 xa[NV], xb[NV];
#pragma unroll
  for (int g = 0; g < NV; ++g) {
    const uint32_t q = static_cast<uint32_t>(g * kWarp + lane) * 16u;
    xa[g] = lds128(xs + q);
    xb[g] = lds128(xs + xhalf + q);
  }
  int64_t taken = 0;
  int slot = 0;  // the slot of piece `taken`, and its phase parity
  uint32_t phase = 0;
  while (take.left > 0) {
    if (!mbar_wait(full + slot, phase)) break;
    const uint32_t piece = ring_addr + static_cast<uint32_t>(slot) * slot_bytes;
    float acc[NV];
#pragma unroll
    for (int g = 0; g < NV; ++g) acc[g] = -0.0f;  // -0 + p == p for every p
    constexpr int kStep = NV < 4 ? NV : 4;
#pragma unroll
    for (int g0 = 0; g0 < NV; g0 += kStep) {
      uint4 wv[kStep];
#pragma unroll
      for (int g = 0; g < kStep; ++g) wv[g] = lds128(piece + static_cast<uint32_t>((g0 + g) * kWarp + lane) * 16u);
#pragma unroll
      for (int g = 0; g < kStep; ++g) chain_e4m3_half(acc[g0 + g], wv[g], xa[g0 + g], xb[g0 + g]);
    }
    const float yv = halve_groups<NV>(acc, lane);
    if (lane == 0) jb.Y[take.row] = yv;
    __syncwarp();
    ++taken;
    if (issue.left > 0) {  // refill the slot just consumed
      if (lane == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(full + slot, row_bytes);
        bulk_load(ring + static_cast<int64_t>(slot) * slot_bytes, W + issue.row * jb.row_bytes, row_bytes,
                  full + slot, once);
      }
      ++issued;
      row_next(issue, 1);
    }
    if (++slot == slots) {
      slot = 0;
      phase ^= 1u;
    }
    row_next(take, 1);
  }
  // Leave only after every copy into this warp's slots has landed.
  for (int64_t i = taken; i < issued; ++i) mbar_wait(full + i % slots, static_cast<uint32_t>((i / slots) & 1));
}

template <int WFMT, int NV, int BG, int kMode>
__device__ __forceinline__ void row_consume(const JobPlan& jb, int slots, uint32_t slot_bytes, uint32_t row_piece,
                                            int ppr, uint8_t* ring, uint64_t* full, uint32_t xs, int lane,
                                            RowCursor issue, RowCursor take, int64_t issued) {
  constexpr int V = Format<WFMT>::kVec;
  constexpr int T = NV * kWarp;
  const uint64_t once = policy_evict_first();
  const uint32_t ring_addr = smem_addr(ring);
  const uint32_t xcol = static_cast<uint32_t>(jb.n * 2);
  const uint32_t row_bytes = static_cast<uint32_t>(jb.row_bytes);
  const int nvec = static_cast<int>(jb.n / V);
  const int vtotal = (nvec + T - 1) / T;
  const uint8_t* W = static_cast<const uint8_t*>(jb.W);
  RowState<WFMT, NV, BG> st;
  int64_t taken = 0;
  int slot = 0;  // the slot of piece `taken`, and its phase parity
  uint32_t phase = 0;
  while (take.left > 0) {
    if (!mbar_wait(full + slot, phase)) break;
    const uint32_t piece = ring_addr + static_cast<uint32_t>(slot) * slot_bytes;
    const uint32_t off = static_cast<uint32_t>(take.piece) * row_piece;
    const uint32_t bytes = min(row_piece, row_bytes - off);
    const int v_lo = static_cast<int>(off / (T * 16u));
    const int v_hi = min(static_cast<int>((off + bytes + T * 16u - 1) / (T * 16u)), vtotal);
    const bool first = take.piece == 0;
    const bool last = take.piece + 1 == ppr;
    for (int g0 = 0; g0 < jb.batch; g0 += BG) {
      if (first) st.reset();
      reduce_row_piece<WFMT, NV, BG, kMode>(st, piece, xs, xcol, g0, jb.batch, v_lo, v_hi, nvec, lane);
      if (last) {
#pragma unroll
        for (int b = 0; b < BG; ++b) {
          const float yv = halve_groups<NV>(st.acc[b], lane);
          if (lane == 0 && g0 + b < jb.batch) jb.Y[static_cast<int64_t>(g0 + b) * jb.m + take.row] = yv;
        }
      }
    }
    __syncwarp();
    ++taken;
    if (issue.left > 0) {  // refill the slot just consumed
      if (lane == 0) {
        fence_proxy_async_smem();
        const uint32_t ioff = static_cast<uint32_t>(issue.piece) * row_piece;
        const uint32_t ibytes = min(row_piece, row_bytes - ioff);
        mbar_arrive_expect_tx(full + slot, ibytes);
        bulk_load(ring + static_cast<int64_t>(slot) * slot_bytes, W + issue.row * jb.row_bytes + ioff, ibytes,
                  full + slot, once);
      }
      ++issued;
      row_next(issue, ppr);
    }
    if (++slot == slots) {
      slot = 0;
      phase ^= 1u;
    }
    row_next(take, ppr);
  }
  // Leave only after every copy into this warp's slots has landed.
  for (int64_t i = taken; i < issued; ++i) mbar_wait(full + i % slots, static_cast<uint32_t>((i / slots) & 1));
}

// The row warp: primes its ring (pre_slots pieces), calls `before_inputs` (producer wait and
// activations; it returns the arithmetic mode, or -1 to leave), fills the ring, then reduces.
template <int WFMT, int NV, int BG, typename Inputs>
__device__ __forceinline__ void row_warp(const JobPlan& jb, int64_t u0, int64_t count, int slots, int pre_slots,
                                         uint32_t slot_bytes, uint32_t row_piece, uint8_t* ring, uint64_t* full,
                                         uint32_t xs, int warp, int lane, Inputs before_inputs) {
  const uint64_t once = policy_evict_first();
  const int ppr = static_cast<int>((jb.row_bytes + row_piece - 1) / row_piece);
  const uint8_t* W = static_cast<const uint8_t*>(jb.W);
  RowCursor issue{u0 + warp, 0, warp < count ? (count - warp + kConsumerWarps - 1) / kConsumerWarps : 0};
  const RowCursor take = issue;
  int64_t issued = 0;
  auto prime = [&](int upto) {
    for (; issued < upto && issue.left > 0; ++issued) {
      const int s = static_cast<int>(issued);
      if (lane == 0) {
        const uint32_t off = static_cast<uint32_t>(issue.piece) * row_piece;
        const uint32_t bytes = min(row_piece, static_cast<uint32_t>(jb.row_bytes) - off);
        mbar_arrive_expect_tx(full + s, bytes);
        bulk_load(ring + static_cast<int64_t>(s) * slot_bytes, W + issue.row * jb.row_bytes + off, bytes, full + s,
                  once);
      }
      row_next(issue, ppr);
    }
  };
  prime(min(slots, pre_slots));
  const int mode = before_inputs();
  prime(slots);
  if (mode < 0) {  // leave only after the copies into this warp's slots have landed
    for (int64_t i = 0; i < issued; ++i) mbar_wait(full + i, 0);
    return;
  }
  if constexpr (WFMT == kWeightsE4m3) {
    if (mode == 2) {
      if (jb.batch == 1 && ppr == 1 && jb.n == 16 * NV * kWarp) {
        row_consume_e4m3_xreg<NV>(jb, slots, slot_bytes, ring, full, xs, lane, issue, take, issued);
      } else {
        row_consume<WFMT, NV, BG, 2>(jb, slots, slot_bytes, row_piece, ppr, ring, full, xs, lane, issue, take, issued);
      }
      return;
    }
  }
  if (mode) {
    row_consume<WFMT, NV, BG, 1>(jb, slots, slot_bytes, row_piece, ppr, ring, full, xs, lane, issue, take, issued);
  } else {
    row_consume<WFMT, NV, BG, 0>(jb, slots, slot_bytes, row_piece, ppr, ring, full, xs, lane, issue, take, issued);
  }
}

// This warp's share of the prior launch's verdict tasks, on the launch's last
// plan.verdict_ctas CTAs (which stream nothing): task t goes to verdict CTA t % C, warp
// (t / C) % 16. The caller has waited for the producing kernels.
__device__ __forceinline__ void prior_verdicts(const Plan& plan, int warp, int lane) {
  const int64_t ctas = plan.verdict_ctas;
  const int64_t first = static_cast<int64_t>(blockIdx.x) - plan.verdict_cta_begin + ctas * warp;
  for (int64_t t = first; t < plan.prior_tasks; t += ctas * kConsumerWarps) {
    const int j = verdict::job_of(plan.prior, t);
    if (j >= 0) verdict::run_task(plan.prior.jobs[j], t - plan.prior.jobs[j].task_begin, lane);
  }
}

// A warp's stream: primes its ring with up to pre_slots weight pieces (settled weights only,
// which the previous kernel does not write, so this may overlap it), then calls
// `before_inputs` (which waits for the producers and brings in the activations; it returns
// -1 if that failed, else the arithmetic mode: 0 product then sum, 1 one FMA per exact
// product, 2 E4M3 weights against binary16 activations), then reduces its units.
template <int WFMT, int NV, int BG, typename Inputs>
__device__ __forceinline__ void staged_warp(const JobPlan& jb, int64_t u0, int64_t count, int slots, int pre_slots,
                                            uint32_t slot_bytes, uint32_t row_piece, uint8_t* ring,
                                            uint64_t* full, uint32_t xs, int warp, int lane,
                                            Inputs before_inputs) {
  const uint64_t once = policy_evict_first();
  const uint32_t seg_piece = slot_bytes / 512u * 512u;
  PieceWalk issue;
  walk_to(issue, jb, u0, warp, count, row_piece, seg_piece);
  int64_t issued = 0;
  auto prime = [&](int upto) {
    for (; issued < upto && issue.pieces > 0; ++issued) {
      const int s = static_cast<int>(issued);
      if (lane == 0) {
        const Unit iu = walk_unit(issue, jb, u0);
        const uint32_t off = static_cast<uint32_t>(issue.piece) * issue.size;
        const uint32_t bytes = min(issue.size, iu.bytes - off);
        mbar_arrive_expect_tx(full + s, bytes);
        bulk_load(ring + static_cast<int64_t>(s) * slot_bytes, static_cast<const uint8_t*>(iu.src) + off, bytes,
                  full + s, once);
      }
      walk_next(issue, jb, u0, count, row_piece, seg_piece);
    }
  };
  // pre_slots slots before the producers are waited for (only settled weights, which the
  // preceding kernel does not write); the rest after the activations, whose loads would
  // otherwise queue behind the whole ring's worth of weight requests.
  prime(min(slots, pre_slots));
  const int fma_mode = before_inputs();
  prime(slots);
  if (fma_mode < 0) {  // leave only after the copies into this warp's slots have landed
    for (int64_t i = 0; i < issued; ++i) mbar_wait(full + i, 0);
    return;
  }
  if constexpr (WFMT == kWeightsE4m3) {
    if (fma_mode == 2) {
      staged_consume<WFMT, NV, BG, 2>(jb, u0, count, slots, slot_bytes, row_piece, ring, full, xs, warp, lane,
                                      issue, issued);
      return;
    }
  }
  if (fma_mode) {
    staged_consume<WFMT, NV, BG, 1>(jb, u0, count, slots, slot_bytes, row_piece, ring, full, xs, warp, lane,
                                    issue, issued);
  } else {
    staged_consume<WFMT, NV, BG, 0>(jb, u0, count, slots, slot_bytes, row_piece, ring, full, xs, warp, lane,
                                    issue, issued);
  }
}

// Once this warp has finished its units: the first pieces of row (next_units[c].x + warp) of
// the next launch's CTA c (same index), into L2, so the next launch starts from L2 while this
// one's last CTAs still stream (the launch boundary keeps HBM busy).
__device__ __forceinline__ void prefetch_next(const Plan& plan, int warp, int lane) {
  const int c = static_cast<int>(blockIdx.x);
  if (lane != 0 || c >= plan.next_ctas) return;
  const int j = plan.next_job[c];
  if (j == 255) return;
  const int2 r = plan.next_units[c];
  const int64_t row = static_cast<int64_t>(r.x) + warp;
  if (row >= r.y) return;
  const PrefetchJob& pj = plan.next_jobs[j];
  if (pj.bytes <= 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pj.W + row * pj.row_bytes), "r"(pj.bytes)
               : "memory");
}

template <int WFMT, int NV, int BG, bool kTma>
__global__ void __launch_bounds__(kPlainThreads, 1) stream_kernel(const __grid_constant__ Plan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  if (static_cast<int>(blockIdx.x) >= plan.verdict_cta_begin) {  // a CTA of the prior verdicts
    allow_dependents();
    wait_for_producers();
    prior_verdicts(plan, static_cast<int>(threadIdx.x) / kWarp, static_cast<int>(threadIdx.x) % kWarp);
    prefetch_next(plan, static_cast<int>(threadIdx.x) / kWarp, static_cast<int>(threadIdx.x) % kWarp);
    return;
  }
  // The CTA's job and unit range come precomputed (one parameter read, no divisions).
  const int2 range = plan.cta_units[blockIdx.x];
  const JobPlan& jb = plan.jobs[plan.cta_job[blockIdx.x]];
  const int64_t u0 = range.x;
  const int64_t count = range.y - range.x;
  const int warp = static_cast<int>(threadIdx.x) / kWarp;
  const int lane = static_cast<int>(threadIdx.x) % kWarp;
  if (count <= 0) {  // uniform for the whole CTA
    if constexpr (kTma) prefetch_next(plan, warp, lane);
    return;
  }

  if constexpr (kTma) {
    const int slots = plan.stages;  // per warp
    const uint32_t slot_bytes = static_cast<uint32_t>(plan.stage_bytes);
    const uint32_t row_piece = static_cast<uint32_t>(plan.sum_bytes);
    uint8_t* xs = smem;
    uint8_t* rings = smem + plan.x_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(rings + static_cast<int64_t>(kConsumerWarps) * slots * slot_bytes);
    uint32_t* xexp = reinterpret_cast<uint32_t*>(bars + kConsumerWarps * slots);  // [0] smallest, [1] largest exponent of x
    if (lane == 0) {  // each warp its own ring's barriers
      for (int s = 0; s < slots; ++s) mbar_init(bars + warp * slots + s, 1);
      if (warp == 0) {
        xexp[0] = 1000;
        xexp[1] = 0;
      }
      fence_barrier_init();
    }
    __syncthreads();
    allow_dependents();
    uint8_t* ring = rings + static_cast<int64_t>(warp) * slots * slot_bytes;
    uint64_t* full = bars + warp * slots;
    const uint32_t xs_addr = smem_addr(xs);
    // After the weight prefetch: wait for the kernels this one depends on, then bring in the
    // activations with 16-byte loads of every thread (not bulk copies, which would queue
    // behind the weight pieces already requested) and take their exponent range.
    auto inputs = [&]() -> int {
      wait_for_producers();
      load_activations<WFMT>(jb, xs, xexp, static_cast<int>(threadIdx.x), lane);
      __syncthreads();
      if constexpr (WFMT == kWeightsE4m3) {
        // Every nonzero activation with an exponent field in [110, 142] is exactly a binary16
        // value: convert the copy in shared memory once and take the binary16 FMA form.
        if (jb.has_w && xexp[0] >= 110u && xexp[1] <= 142u) {
          activations_to_half(jb, xs, static_cast<int>(threadIdx.x));
          __syncthreads();
          return 2;
        }
      }
      return jb.has_w && fma_is_exact<WFMT>(jb, xexp[0], xexp[1]) ? 1 : 0;
    };
    if (jb.has_check && !jb.has_w) {  // a bank CTA (uniform for the CTA)
      // Bank pieces before the producer wait only for a settled bank: otherwise c and a may
      // come from the kernel just before (pck_bank_build), whose writes are visible only
      // after griddepcontrol.wait.
      bank_warp(jb, u0, count, slots, jb.bank_settled ? plan.pre_slots : 0, slot_bytes, ring, full, xs_addr, warp,
                lane, inputs);
    } else if (!jb.has_check && jb.rows == 1) {  // a row CTA
      row_warp<WFMT, NV, BG>(jb, u0, count, slots, plan.pre_slots, slot_bytes, row_piece, ring, full, xs_addr, warp,
                             lane, inputs);
    } else {
      staged_warp<WFMT, NV, BG>(jb, u0, count, slots, jb.has_check ? 0 : plan.pre_slots, slot_bytes, row_piece,
                                ring, full, xs_addr,
                                warp, lane, inputs);
    }
    prefetch_next(plan, warp, lane);
  } else {
    // Plain path: every warp takes whole units and reads global memory directly, one
    // element at a time (product, then sum: the same values as the staged path's).
    allow_dependents();
    wait_for_producers();
    const uint16_t* X = jb.X;
    for (int64_t i = warp; i < count; i += kConsumerWarps) {
      plain_unit<WFMT, NV, BG>(jb, decode_unit(jb, u0 + i), X, lane);
    }
  }
}

}  // namespace pck
