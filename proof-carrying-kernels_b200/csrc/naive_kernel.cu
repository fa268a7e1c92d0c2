// The naive GEMV tree (API parity with the reference's `gemv_naive`), bit-exact with the
// reference model `emulate_gemv` (src/pck/gemv.py:14-57; kernel gemv_kernel.cu:27-55):
// thread t of `threads` sums the contiguous columns [t*chunk, (t+1)*chunk), chunk =
// ceil(n / threads), in order (columns past n add +0), then a pairwise tree combines the
// partials: stride 1, 2, 4, ..., partial[t] += partial[t + stride] for t % (2 stride) == 0.
// One CTA of `threads` threads per row, rows grid-strided.
#include <cuda_runtime.h>

#include <cstdint>

#include "pck_common.cuh"

namespace pck {
namespace {

__global__ void gemv_naive_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ x,
                                  float* __restrict__ y, int64_t m, int64_t n, int64_t chunk) {
  extern __shared__ float partial[];
  const int t = static_cast<int>(threadIdx.x);
  const int threads = static_cast<int>(blockDim.x);
  for (int64_t row = blockIdx.x; row < m; row += gridDim.x) {
    const uint16_t* w = W + row * n;
    const int64_t begin = static_cast<int64_t>(t) * chunk;
    float acc = -0.0f;  // -0 + p == p: the chain starts with its first term
    for (int64_t j = begin; j < begin + chunk; ++j) {
      const float p = j < n ? __fmul_rn(bf16_bits_to_float(w[j]), bf16_bits_to_float(x[j])) : 0.0f;
      acc = __fadd_rn(acc, p);
    }
    partial[t] = acc;
    __syncthreads();
    for (int stride = 1; stride < threads; stride *= 2) {
      if (t % (2 * stride) == 0) partial[t] = __fadd_rn(partial[t], partial[t + stride]);
      __syncthreads();
    }
    if (t == 0) y[row] = partial[0];
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_gemv_naive(const void* W, const void* x, float* y, int64_t m, int64_t n,
                              int threads, int sms, cudaStream_t stream) {
  const int64_t chunk = (n + threads - 1) / threads;
  const int64_t grid = m < 64LL * sms ? m : 64LL * sms;
  gemv_naive_kernel<<<static_cast<unsigned>(grid), threads, static_cast<size_t>(threads) * sizeof(float),
                      stream>>>(static_cast<const uint16_t*>(W), static_cast<const uint16_t*>(x), y,
                                m, n, chunk);
  return cudaGetLastError();
}

}  // namespace pck
