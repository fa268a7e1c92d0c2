// Sampled-token membership check (the batched check of src/pck/member.py:118-197), one CTA
// per row of logits:
//   above  = #{j : l_j > l_t}                      (t clamped into [0, V) for the gather)
//   ok     = no NaN in the row && 0 <= t < V && above < (greedy ? 1 : k)
//   top-p (rows with p < 1): kept = {j : l_j >= k-th largest} (all when k = V), m = max,
//     e_j = binary32 e^(l_j - m) from the exact TwoSum split (src/pck/member.py:105-115),
//     Z = sum of kept e_j, A = sum of kept e_j with l_j > l_t (binary64), r = A / Z,
//     ok &= p >= 1 || greedy || r < nextafter(p + slack, +inf);  mass_above = r (p < 1) else 0.
//
// Pass 1 reads the row once from HBM: NaN flag, `above`, the row maximum and every thread's
// own maximum. When a k-th largest value is needed (top-p with k < V), the k-th largest of
// the thread maxima is a value tau with at least k logits >= tau, so the k-th largest logit
// is >= tau: pass 2 (from L2) copies every logit >= tau into shared memory (for random
// logits a few times k of them), an exact radix select over those finds the k-th largest,
// and the masses are summed from shared memory. Rows whose candidates do not fit (heavy
// ties, k above the thread count) fall back to a radix select over the whole row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "member_plan.h"
#include "pck_common.cuh"

namespace pck {
namespace {

constexpr int kWarpsPerRow = kMemberThreads / kWarp;

// Monotone map of binary32 values (not NaN) to unsigned keys; -0 and +0 share a key.
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// binary32 e^(x - m) as src/pck/member.py:105-115 computes it: x - m = hi + lo exactly
// (TwoSum), term = expf(hi) + expf(hi) * lo, 0 where hi < -128 (or NaN).
__device__ __forceinline__ float member_term(float x, float nm) {
  const float hi = __fadd_rn(x, nm);
  const float bv = __fsub_rn(hi, x);
  const float lo = __fadd_rn(__fsub_rn(x, __fsub_rn(hi, bv)), __fsub_rn(nm, bv));
  const float eh = expf(hi);
  return hi >= -128.0f ? __fadd_rn(eh, __fmul_rn(eh, lo)) : 0.0f;
}

template <int DT>
__device__ __forceinline__ float logit_at(const void* row, int64_t j) {
  if constexpr (DT == kLogitsF32) {
    return __ldg(static_cast<const float*>(row) + j);
  } else if constexpr (DT == kLogitsBf16) {
    return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(row) + j)) << 16);
  } else {
    return __half2float(__ldg(static_cast<const __half*>(row) + j));
  }
}

// Calls fn(value) for every logit of the row, each thread a strided share, with 16-byte
// loads (four in flight per thread) when the row start allows.
template <int DT, typename Fn>
__device__ __forceinline__ void for_each_logit(const void* row, int64_t vocab, Fn fn) {
  constexpr int kPer = DT == kLogitsF32 ? 4 : 8;  // logits per 16 bytes
  const int tid = static_cast<int>(threadIdx.x);
  int64_t head = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
    const int64_t vecs = vocab / kPer;
    const uint4* v4 = static_cast<const uint4*>(row);
    auto take = [&](const uint4 q) {
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      if constexpr (DT == kLogitsF32) {
#pragma unroll
        for (int h = 0; h < 4; ++h) fn(__uint_as_float(w[h]));
      } else {
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const uint32_t bits = h & 1 ? w[h / 2] >> 16 : w[h / 2] & 0xffffu;
          if constexpr (DT == kLogitsBf16) {
            fn(__uint_as_float(bits << 16));
          } else {
            fn(__half2float(__ushort_as_half(static_cast<unsigned short>(bits))));
          }
        }
      }
    };
    // four 16-byte loads in flight per thread, then their values
    constexpr int kAhead = 4;
    int64_t i = tid;
    for (; i + (kAhead - 1) * kMemberThreads < vecs; i += kAhead * kMemberThreads) {
      uint4 q[kAhead];
#pragma unroll
      for (int u = 0; u < kAhead; ++u) q[u] = __ldg(v4 + i + u * kMemberThreads);
#pragma unroll
      for (int u = 0; u < kAhead; ++u) take(q[u]);
    }
    for (; i < vecs; i += kMemberThreads) take(__ldg(v4 + i));
    head = vecs * kPer;
  }
  for (int64_t j = head + tid; j < vocab; j += kMemberThreads) fn(logit_at<DT>(row, j));
}

struct Shared {
  uint32_t hist[256];
  uint32_t keys[kMemberThreads];  // thread maxima (as keys)
  double dsum[2][kWarpsPerRow];
  int64_t isum[kWarpsPerRow];
  float fmax[kWarpsPerRow];
  uint32_t count;
  uint32_t pick;
  uint32_t need;
  int flag;
};

__device__ __forceinline__ int64_t block_sum(int64_t v, Shared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  if (lane == 0) sh.isum[warp] = v;
  __syncthreads();
  int64_t t = 0;
  for (int w = 0; w < kWarpsPerRow; ++w) t += sh.isum[w];
  __syncthreads();
  return t;
}

__device__ __forceinline__ float block_max(float v, Shared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  if (lane == 0) sh.fmax[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < kWarpsPerRow; ++w) t = fmaxf(t, sh.fmax[w]);
  __syncthreads();
  return t;
}

// (Z, A) summed over the block in a fixed order (warps in order, lanes by a fixed tree).
__device__ __forceinline__ void block_sum2(double& z, double& a, Shared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    z = __dadd_rn(z, __shfl_xor_sync(kFullMask, z, o));
    a = __dadd_rn(a, __shfl_xor_sync(kFullMask, a, o));
  }
  if (lane == 0) {
    sh.dsum[0][warp] = z;
    sh.dsum[1][warp] = a;
  }
  __syncthreads();
  z = 0.0;
  a = 0.0;
  for (int w = 0; w < kWarpsPerRow; ++w) {
    z = __dadd_rn(z, sh.dsum[0][w]);
    a = __dadd_rn(a, sh.dsum[1][w]);
  }
  __syncthreads();
}

// Key of the need-th largest (1-based) of n keys, by four 8-bit digit passes; key(i) gives
// the i-th key. Every thread returns it.
template <typename KeyAt>
__device__ uint32_t radix_kth(KeyAt key, int64_t n, uint32_t need, Shared& sh) {
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += kMemberThreads) sh.hist[b] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += kMemberThreads) {
      const uint32_t k = key(i);
      if ((k & mask) == prefix) atomicAdd(&sh.hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < kWarp) {
      // Lane l owns digits 255 - 8l ... 248 - 8l (from the top); an exclusive scan of the
      // lane totals from lane 0 gives the count above each lane's digits.
      const int lane = threadIdx.x;
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c[q] = sh.hist[255 - 8 * lane - q];
        tot += c[q];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const uint32_t v = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += v;
      }
      uint32_t above = incl - tot;
      const uint32_t want = need;
      if (above < want && want <= incl) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (above < want && want <= above + c[q]) {
            sh.pick = 255u - 8u * lane - q;
            sh.need = want - above;
          }
          above += c[q];
        }
      }
    }
    __syncthreads();
    prefix |= sh.pick << shift;
    mask |= 255u << shift;
    need = sh.need;
    __syncthreads();
  }
  return prefix;
}

template <int DT>
__global__ void __launch_bounds__(kMemberThreads, 1) member_kernel(const __grid_constant__ MemberArgs args) {
  extern __shared__ __align__(16) uint8_t dyn[];
  Shared& sh = *reinterpret_cast<Shared*>(dyn);
  uint32_t* cands = reinterpret_cast<uint32_t*>(dyn + sizeof(Shared));
  const int64_t row_i = blockIdx.x;
  const int64_t vocab = args.vocab;
  const void* row = static_cast<const uint8_t*>(args.logits) +
                    row_i * args.row_stride * (DT == kLogitsF32 ? 4 : 2);
  const int64_t tok = args.tokens[row_i];
  const bool in_range = tok >= 0 && tok < vocab;
  const float lt = logit_at<DT>(row, tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok));
  const int64_t k = args.top_k ? min(max(args.top_k[row_i], static_cast<int64_t>(1)), vocab) : vocab;
  const bool greedy = args.greedy ? args.greedy[row_i] != 0 : false;
  const double p = args.top_p ? args.top_p[row_i] : 1.0;

  // Pass 1: NaN, above, maxima.
  bool nan = false;
  int64_t gt = 0;
  float tmax = -INFINITY;
  for_each_logit<DT>(row, vocab, [&](float v) {
    nan |= isnan(v);
    gt += v > lt;
    tmax = fmaxf(tmax, v);
  });
  nan = __syncthreads_or(nan);
  const int64_t above = block_sum(gt, sh);
  const float m = block_max(tmax, sh);
  bool ok = !nan && in_range && above < (greedy ? 1 : k);

  double r = 0.0;
  const bool need_r = args.top_p != nullptr && p < 1.0;
  if (need_r && nan) {
    r = __longlong_as_double(0x7ff8000000000000LL);
  } else if (need_r) {
    const float nm = -m;
    double z = 0.0, a = 0.0;
    if (k >= vocab) {  // every logit is kept
      for_each_logit<DT>(row, vocab, [&](float v) {
        const float t = member_term(v, nm);
        z = __dadd_rn(z, static_cast<double>(t));
        if (v > lt) a = __dadd_rn(a, static_cast<double>(t));
      });
    } else {
      bool fits = false;
      uint32_t kth = 0;
      if (k <= kMemberThreads) {
        sh.keys[threadIdx.x] = order_key(tmax);
        if (threadIdx.x == 0) sh.count = 0;
        __syncthreads();
        const uint32_t tau = radix_kth([&](int64_t i) { return sh.keys[i]; }, kMemberThreads,
                                       static_cast<uint32_t>(k), sh);
        // Pass 2: every logit >= tau into shared memory (a warp reserves its slots at once).
        for_each_logit<DT>(row, vocab, [&](float v) {
          const uint32_t key = order_key(v);
          const bool take = key >= tau;
          const unsigned bal = __ballot_sync(__activemask(), take);
          if (bal) {
            const int lane = threadIdx.x % kWarp;
            const int leader = __ffs(bal) - 1;
            uint32_t base = 0;
            if (lane == leader) base = atomicAdd(&sh.count, static_cast<uint32_t>(__popc(bal)));
            base = __shfl_sync(__activemask(), base, leader);
            const uint32_t at = base + __popc(bal & ((1u << lane) - 1u));
            if (take && at < kMemberCandidates) cands[at] = key;
          }
        });
        __syncthreads();
        const uint32_t nc = sh.count;
        fits = nc <= kMemberCandidates;
        if (fits) {
          kth = radix_kth([&](int64_t i) { return cands[i]; }, nc, static_cast<uint32_t>(k), sh);
          for (uint32_t i = threadIdx.x; i < nc; i += kMemberThreads) {
            const uint32_t key = cands[i];
            if (key >= kth) {
              const float v = key_value(key);
              const float t = member_term(v, nm);
              z = __dadd_rn(z, static_cast<double>(t));
              if (v > lt) a = __dadd_rn(a, static_cast<double>(t));
            }
          }
        }
      }
      if (!fits) {  // exact select over the whole row, then one more pass for the masses
        kth = radix_kth([&](int64_t i) { return order_key(logit_at<DT>(row, i)); }, vocab,
                        static_cast<uint32_t>(k), sh);
        const float kv = key_value(kth);
        for_each_logit<DT>(row, vocab, [&](float v) {
          if (v >= kv) {
            const float t = member_term(v, nm);
            z = __dadd_rn(z, static_cast<double>(t));
            if (v > lt) a = __dadd_rn(a, static_cast<double>(t));
          }
        });
      }
    }
    block_sum2(z, a, sh);
    r = __ddiv_rn(a, z);
  }
  if (args.top_p != nullptr) {
    const double high = nextafter(__dadd_rn(p, args.slack), __longlong_as_double(0x7ff0000000000000LL));
    ok = ok && (p >= 1.0 || greedy || r < high);
  }
  if (threadIdx.x == 0) {
    args.ok[row_i] = ok ? 1 : 0;
    args.above[row_i] = above;
    args.mass_above[row_i] = need_r ? r : 0.0;
  }
}

}  // namespace

size_t member_smem_bytes() { return sizeof(Shared) + sizeof(uint32_t) * kMemberCandidates; }

cudaError_t launch_member_check(const MemberArgs& args, cudaStream_t stream) {
  const size_t smem = member_smem_bytes();
  auto launch = [&](auto kernel) -> cudaError_t {
    static int configured[64] = {0};
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
      const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      configured[dev] = 1;
    }
    kernel<<<static_cast<unsigned>(args.rows), kMemberThreads, smem, stream>>>(args);
    return cudaGetLastError();
  };
  switch (args.dtype) {
    case kLogitsF32: return launch(member_kernel<kLogitsF32>);
    case kLogitsBf16: return launch(member_kernel<kLogitsBf16>);
    case kLogitsF16: return launch(member_kernel<kLogitsF16>);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pck
