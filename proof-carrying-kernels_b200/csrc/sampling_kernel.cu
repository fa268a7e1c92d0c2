// Trusted top-k / top-p set check (the GPU form of src/pck/sampling.py:90-122, the behaviour
// of the reference's sampling_check, src/pck/cuda/csrc/sampling_kernel.cu): for row b with
// selection sel[b, :len[b]] over V logits,
//   top-k passes iff the selection is well formed (len in [1, max_len], len <= V, distinct
//     in-range ids, len == k), no logit is NaN and min(selected) >= max(rejected);
//   top-p also needs mass >= p - slack and mass_without_smallest < p + slack, the masses
//     from terms e^((l - M) / T) (M the row maximum) in binary32 expf on an exact split
//     argument, summed in binary64.
//
// One launch, no scratch memory: row b is one thread-block cluster of C CTAs, CTA c owning
// the logits [c*L, (c+1)*L). Each CTA marks the selected ids of its slice in a shared-memory
// bitmap (a duplicate or out-of-range id marks the row malformed), scans its slice once for
// NaN, the maximum, min(selected) and max(rejected), and the cluster exchanges these partials
// through distributed shared memory. Every CTA then knows the row maximum M, so the top-p
// terms are taken against M directly (no per-segment rescaling), and CTA 0 adds the C
// partial sums in rank order and decides.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "pck_common.cuh"
#include "sampling_plan.h"

namespace cg = cooperative_groups;

namespace pck {
namespace {

constexpr int kWarpsPerCta = kSamplingThreads / kWarp;

struct SlicePartial {
  float min_sel;
  float max_rej;
  float max_all;
  int nan;
  int malformed;
  int pad;
  double z;
  double z_sel;
};

struct SamplingShared {
  SlicePartial part;
  float f[3][kWarpsPerCta];
  double d[2][kWarpsPerCta];
};

__device__ __forceinline__ void block_minmax3(float& mn, float& mx_rej, float& mx_all, SamplingShared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(kFullMask, mn, o));
    mx_rej = fmaxf(mx_rej, __shfl_xor_sync(kFullMask, mx_rej, o));
    mx_all = fmaxf(mx_all, __shfl_xor_sync(kFullMask, mx_all, o));
  }
  if (lane == 0) {
    sh.f[0][warp] = mn;
    sh.f[1][warp] = mx_rej;
    sh.f[2][warp] = mx_all;
  }
  __syncthreads();
  mn = INFINITY;
  mx_rej = -INFINITY;
  mx_all = -INFINITY;
  for (int w = 0; w < kWarpsPerCta; ++w) {
    mn = fminf(mn, sh.f[0][w]);
    mx_rej = fmaxf(mx_rej, sh.f[1][w]);
    mx_all = fmaxf(mx_all, sh.f[2][w]);
  }
  __syncthreads();
}

__device__ __forceinline__ void block_sum2(double& z, double& zs, SamplingShared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    z = __dadd_rn(z, __shfl_xor_sync(kFullMask, z, o));
    zs = __dadd_rn(zs, __shfl_xor_sync(kFullMask, zs, o));
  }
  if (lane == 0) {
    sh.d[0][warp] = z;
    sh.d[1][warp] = zs;
  }
  __syncthreads();
  z = 0.0;
  zs = 0.0;
  for (int w = 0; w < kWarpsPerCta; ++w) {
    z = __dadd_rn(z, sh.d[0][w]);
    zs = __dadd_rn(zs, sh.d[1][w]);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSamplingThreads) sampling_kernel(const __grid_constant__ SamplingArgs a) {
  extern __shared__ __align__(16) uint8_t dyn[];
  SamplingShared& sh = *reinterpret_cast<SamplingShared*>(dyn);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(dyn + sizeof(SamplingShared));
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int csize = static_cast<int>(cluster.num_blocks());
  const int tid = static_cast<int>(threadIdx.x);
  const int64_t row = blockIdx.y;
  const int64_t vocab = a.vocab;
  const int64_t j0 = min(vocab, static_cast<int64_t>(rank) * a.slice);
  const int64_t j1 = min(vocab, j0 + a.slice);
  const float* l = a.logits + row * vocab;

  // Bitmap of the selected ids in this slice.
  const int64_t words = (j1 - j0 + 31) / 32;
  for (int64_t w = tid; w < words; w += kSamplingThreads) bitmap[w] = 0u;
  __syncthreads();
  const int64_t len = a.lengths[row];
  const int64_t n_ins = min(len, a.max_len);
  bool bad = false;
  for (int64_t i = tid; i < n_ins; i += kSamplingThreads) {
    const int64_t idx = a.selected[row * a.max_len + i];
    if (idx < 0 || idx >= vocab) {
      bad = true;
    } else if (idx >= j0 && idx < j1) {
      const uint32_t bit = 1u << ((idx - j0) & 31);
      if (atomicOr(&bitmap[(idx - j0) >> 5], bit) & bit) bad = true;
    }
  }
  bad = __syncthreads_or(bad);

  // One pass over the slice.
  float mn = INFINITY, mx_rej = -INFINITY, mx_all = -INFINITY;
  bool nan = false;
  auto take = [&](int64_t j, float x) {
    nan |= isnan(x);
    mx_all = fmaxf(mx_all, x);
    const int64_t o = j - j0;
    if (bitmap[o >> 5] & (1u << (o & 31))) {
      mn = fminf(mn, x);
    } else {
      mx_rej = fmaxf(mx_rej, x);
    }
  };
  constexpr int kAhead = 4;  // loads in flight per thread
  int64_t j = j0 + tid;
  for (; j + (kAhead - 1) * kSamplingThreads < j1; j += kAhead * kSamplingThreads) {
    float xs[kAhead];
#pragma unroll
    for (int u = 0; u < kAhead; ++u) xs[u] = __ldg(l + j + u * kSamplingThreads);
#pragma unroll
    for (int u = 0; u < kAhead; ++u) take(j + u * kSamplingThreads, xs[u]);
  }
  for (; j < j1; j += kSamplingThreads) take(j, __ldg(l + j));
  nan = __syncthreads_or(nan);
  block_minmax3(mn, mx_rej, mx_all, sh);
  if (tid == 0) sh.part = SlicePartial{mn, mx_rej, mx_all, nan ? 1 : 0, bad ? 1 : 0, 0, 0.0, 0.0};
  cluster.sync();

  // Every CTA merges the slices' partials in rank order (the same values everywhere).
  float min_sel = INFINITY, max_rej = -INFINITY, big_m = -INFINITY;
  bool any_nan = false, malformed = false;
  for (int c = 0; c < csize; ++c) {
    const SlicePartial* p = cluster.map_shared_rank(&sh.part, c);
    min_sel = fminf(min_sel, p->min_sel);
    max_rej = fmaxf(max_rej, p->max_rej);
    big_m = fmaxf(big_m, p->max_all);
    any_nan |= p->nan != 0;
    malformed |= p->malformed != 0;
  }
  const bool well_formed = !malformed && len >= 1 && len <= a.max_len && len <= vocab && (a.top_p || len == a.k);
  bool ok = well_formed && !any_nan && min_sel >= max_rej;  // -inf when nothing is rejected
  double mass = 0.0, without = 0.0;
  if (a.top_p && ok) {  // uniform over the cluster
    const double m = static_cast<double>(big_m);
    const double inv_t = 1.0 / a.temperature;
    double z = 0.0, zs = 0.0;
    for (int64_t j = j0 + tid; j < j1; j += kSamplingThreads) {
      const float x = __ldg(l + j);
      const double d = __dmul_rn(__dsub_rn(static_cast<double>(x), m), inv_t);
      const float hi = __double2float_rn(d);
      const float lo = __double2float_rn(__dsub_rn(d, static_cast<double>(hi)));
      const float eh = expf(hi);
      // Terms below e^-128 (masked -inf logits among them) are left out; -inf would
      // otherwise turn lo into NaN.
      const double e = d >= -128.0 ? static_cast<double>(__fmaf_rn(eh, lo, eh)) : 0.0;
      z = __dadd_rn(z, e);
      const int64_t o = j - j0;
      if (bitmap[o >> 5] & (1u << (o & 31))) zs = __dadd_rn(zs, e);
    }
    block_sum2(z, zs, sh);
    if (tid == 0) {
      sh.part.z = z;
      sh.part.z_sel = zs;
    }
    cluster.sync();
    if (rank == 0 && tid == 0) {
      double big_z = 0.0, big_zs = 0.0;
      for (int c = 0; c < csize; ++c) {
        const SlicePartial* p = cluster.map_shared_rank(&sh.part, c);
        big_z = __dadd_rn(big_z, p->z);
        big_zs = __dadd_rn(big_zs, p->z_sel);
      }
      const double e_min = exp(__dmul_rn(__dsub_rn(static_cast<double>(min_sel), m), inv_t));
      mass = __ddiv_rn(big_zs, big_z);
      without = __ddiv_rn(__dsub_rn(big_zs, e_min), big_z);
      ok = mass >= __dsub_rn(a.p, a.slack) && without < __dadd_rn(a.p, a.slack);
    }
  }
  if (rank == 0 && tid == 0) {
    a.passed[row] = ok ? 1 : 0;
    a.min_selected[row] = min_sel;
    a.max_rejected[row] = max_rej;
    a.mass[row] = mass;
    a.without[row] = without;
  }
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace

cudaError_t launch_sampling_check(const SamplingArgs& args, int cluster, cudaStream_t stream) {
  const int64_t words = (args.slice + 31) / 32;
  const size_t smem = sizeof(SamplingShared) + static_cast<size_t>(words) * 4;
  static int configured[64] = {0};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t err = cudaFuncSetAttribute(sampling_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kSamplingSmemCap));
    if (err != cudaSuccess) return err;
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster), static_cast<unsigned>(args.rows));
  cfg.blockDim = dim3(kSamplingThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sampling_kernel, args);
}

size_t sampling_smem_bytes(int64_t slice) { return sizeof(SamplingShared) + static_cast<size_t>((slice + 31) / 32) * 4; }

}  // namespace pck
