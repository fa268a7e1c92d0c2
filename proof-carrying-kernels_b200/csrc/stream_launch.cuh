// Instantiation and launch of the streaming kernel for one weight format (included by
// stream_bf16.cu and stream_e4m3.cu, which nvcc compiles in parallel).
#pragma once

#include "stream_kernel.cuh"

namespace pck {

inline int current_device() {
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess ? dev : -1;
}

template <int WFMT, int NV, int BG, bool kTma>
cudaError_t launch_variant(const Plan& plan, unsigned grid, size_t smem, cudaStream_t stream) {
  auto* fn = stream_kernel<WFMT, NV, BG, kTma>;
  if (kTma) {
    // The opt-in shared-memory size is a per-device function attribute: set it once per
    // device to the largest size this library ever asks for.
    static int configured[64] = {0};
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
      const cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
      if (err != cudaSuccess) return err;
      configured[dev] = 1;
    }
  }
  // Programmatic dependent launch: this kernel may start while the previous kernel of the
  // stream finishes; it prefetches only weights before griddepcontrol.wait.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPlainThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, plan);
}

template <int WFMT, int NV>
cudaError_t launch_nv(const Plan& plan, int bg, bool tma, unsigned grid, size_t smem,
                      cudaStream_t stream) {
  if (!tma) return launch_variant<WFMT, NV, 1, false>(plan, grid, smem, stream);
  constexpr int kAcc = warp_accumulators(WFMT, NV);
  switch (bg) {
    case 1: return launch_variant<WFMT, NV, 1, true>(plan, grid, smem, stream);
    case 2: return launch_variant<WFMT, NV, (2 * kAcc <= 64 ? 2 : 1), true>(plan, grid, smem, stream);
    case 4: return launch_variant<WFMT, NV, (4 * kAcc <= 64 ? 4 : 1), true>(plan, grid, smem, stream);
    case 8: return launch_variant<WFMT, NV, (8 * kAcc <= 64 ? 8 : 1), true>(plan, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int WFMT>
cudaError_t launch_format(const Plan& plan, int nv, int bg, bool tma, unsigned grid, size_t smem,
                          cudaStream_t stream) {
  switch (nv) {
    case 1: return launch_nv<WFMT, 1>(plan, bg, tma, grid, smem, stream);
    case 2: return launch_nv<WFMT, 2>(plan, bg, tma, grid, smem, stream);
    case 4: return launch_nv<WFMT, 4>(plan, bg, tma, grid, smem, stream);
    case 8: return launch_nv<WFMT, 8>(plan, bg, tma, grid, smem, stream);
    case 16: return launch_nv<WFMT, 16>(plan, bg, tma, grid, smem, stream);
    case 32: return launch_nv<WFMT, 32>(plan, bg, tma, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pck
