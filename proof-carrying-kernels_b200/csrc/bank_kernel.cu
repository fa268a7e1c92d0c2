// On-device construction of a checker's bank from bfloat16 W and its signs r
// (the weight-load arithmetic of the reference's src/pck/cuda/checker.py:94-107):
//   c[k, beta, j] = fl32( sum_i r[k, beta, i] * W[beta*b + i, j] )   binary64 sum, i in order
//   a[beta, j]    = round_up_bf16( next_up( fl64(sum_i |W[beta*b + i, j]|) * sum_up_factor ) )
// where round_up_bf16 (checker.py:29-43) rounds a non-negative binary64 value up to binary32,
// then up to bfloat16 by carrying into bit 16 when any of the low 16 bits is set.
// The products r * W are exact (+-W); one thread owns one column j of one row block.
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"

namespace pck {
namespace {

constexpr int kBankThreads = 256;
constexpr int kBankChecks = 8;  // checksums accumulated per pass over the block

__device__ __forceinline__ uint16_t round_up_bf16_bits(double v) {
  float f = __double2float_rn(v);
  if (static_cast<double>(f) < v) f = nextafterf(f, __int_as_float(0x7f800000));
  uint32_t bits = __float_as_uint(f);
  if (bits & 0xffffu) bits = (bits + 0x10000u) & 0xffff0000u;
  return static_cast<uint16_t>(bits >> 16);
}

__global__ void __launch_bounds__(kBankThreads)
    bank_kernel(const uint16_t* __restrict__ W, const int8_t* __restrict__ r, float* __restrict__ c,
                uint16_t* __restrict__ a, int64_t n, int block, int num_blocks, int checks,
                double factor) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * kBankThreads + threadIdx.x;
  const int64_t beta = blockIdx.y;
  if (j >= n) return;
  const uint16_t* wcol = W + beta * block * n + j;
  double abs_sum = 0.0;
  for (int i = 0; i < block; ++i) {
    abs_sum = __dadd_rn(abs_sum, fabs(static_cast<double>(bf16_bits_to_float(wcol[static_cast<int64_t>(i) * n]))));
  }
  const double bound = nextafter(__dmul_rn(abs_sum, factor), __longlong_as_double(0x7ff0000000000000LL));
  a[beta * n + j] = round_up_bf16_bits(bound);
  for (int k0 = 0; k0 < checks; k0 += kBankChecks) {
    double acc[kBankChecks];
#pragma unroll
    for (int q = 0; q < kBankChecks; ++q) acc[q] = 0.0;
    for (int i = 0; i < block; ++i) {
      const double w = static_cast<double>(bf16_bits_to_float(wcol[static_cast<int64_t>(i) * n]));
#pragma unroll
      for (int q = 0; q < kBankChecks; ++q) {
        if (k0 + q < checks) {
          const int8_t s = __ldg(r + (static_cast<int64_t>(k0 + q) * num_blocks + beta) * block + i);
          acc[q] = __dadd_rn(acc[q], s > 0 ? w : -w);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kBankChecks; ++q) {
      if (k0 + q < checks) c[(static_cast<int64_t>(k0 + q) * num_blocks + beta) * n + j] = __double2float_rn(acc[q]);
    }
  }
}

}  // namespace

cudaError_t launch_bank_build(const void* W, const int8_t* r, float* c, void* a, int64_t n,
                              int block, int num_blocks, int checks, double factor,
                              cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((n + kBankThreads - 1) / kBankThreads),
                  static_cast<unsigned>(num_blocks));
  bank_kernel<<<grid, kBankThreads, 0, stream>>>(static_cast<const uint16_t*>(W), r, c,
                                                  static_cast<uint16_t*>(a), n, block, num_blocks,
                                                  checks, factor);
  return cudaGetLastError();
}

}  // namespace pck
