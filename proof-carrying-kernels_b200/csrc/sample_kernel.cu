// An untrusted top-k / top-p sampler over binary32 logits (B, V), one CTA per row: the
// sampling step of the checked LM head, whose every token the trusted
// membership kernel checks afterwards. It is not part of the trusted path; a wrong token
// here is a caught fault, not a wrong verdict.
//
// Per row, with l = logits / temperature:
//   1. one pass over the row (HBM): every thread's largest value, and the row's smallest
//      value at its lowest index (the argmin, for the planted faults);
//   2. tau = the k-th largest of the 1024 thread maxima: at least k logits are >= tau, so the
//      k-th largest logit is >= tau; a second pass (L2) copies the logits >= tau with their
//      indices into shared memory (a few times k of them for spread-out logits), and an
//      exact radix select there gives the k-th largest value;
//   3. exactly k of them (ties at the k-th value by position), sorted descending; binary32
//      softmax over them, the shortest prefix whose probability mass before it stays below
//      p (the nucleus), and an inverse-CDF draw from that prefix with the row's uniform draw;
//   4. with probability fault_rate (the row's fault draw) the token is replaced by the argmin
//      (the fault the reference's vLLM plugin plants).
// Rows whose candidates overflow shared memory (heavy ties) take a radix select over the
// whole row and a third pass.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "pck_b200.h"
#include "pck_common.cuh"

namespace pck {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / kWarp;
constexpr int kSampleCandidates = 6144;  // (key, index) pairs in shared memory
constexpr int kSampleMaxK = 1024;

struct SampleArgs {
  const float* logits;
  int64_t vocab;
  int64_t row_stride;
  int64_t k;
  float p;
  float inv_t;
  const float* draws;
  const float* fault_draws;
  float fault_rate;
  int64_t* tokens;
  uint8_t* injected;
};

// Monotone map of binary32 values (not NaN) to unsigned keys; -0 and +0 share a key.
__device__ __forceinline__ uint32_t skey(float v) {
  const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float skey_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleShared {
  uint32_t hist[256];
  uint32_t keys[kSampleThreads];
  float wmin[kSampleWarps];
  int64_t wimin[kSampleWarps];
  uint32_t count;
  uint32_t nsel;
  uint32_t ties;
  uint32_t pick;
  uint32_t need;
  uint32_t sel_key[kSampleMaxK];
  int64_t sel_idx[kSampleMaxK];
};

// Calls fn(value, index) for every element of the row, each thread a strided share, with
// 16-byte loads when the row start allows.
template <typename Fn>
__device__ __forceinline__ void each_logit(const float* row, int64_t vocab, Fn fn) {
  const int tid = static_cast<int>(threadIdx.x);
  int64_t head = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
    const int64_t vecs = vocab / 4;
    const float4* v4 = reinterpret_cast<const float4*>(row);
    int64_t i = tid;
    for (; i + 3 * kSampleThreads < vecs; i += 4 * kSampleThreads) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldg(v4 + i + u * kSampleThreads);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = 4 * (i + u * kSampleThreads);
        fn(q[u].x, j);
        fn(q[u].y, j + 1);
        fn(q[u].z, j + 2);
        fn(q[u].w, j + 3);
      }
    }
    for (; i < vecs; i += kSampleThreads) {
      const float4 q = __ldg(v4 + i);
      fn(q.x, 4 * i);
      fn(q.y, 4 * i + 1);
      fn(q.z, 4 * i + 2);
      fn(q.w, 4 * i + 3);
    }
    head = vecs * 4;
  }
  for (int64_t j = head + tid; j < vocab; j += kSampleThreads) fn(__ldg(row + j), j);
}

// Key of the need-th largest (1-based) of n keys by four 8-bit digit passes; key(i) gives the
// i-th key. Every thread returns it.
template <typename KeyAt>
__device__ uint32_t select_kth(KeyAt key, int64_t n, uint32_t need, SampleShared& sh) {
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += kSampleThreads) sh.hist[b] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += kSampleThreads) {
      const uint32_t k = key(i);
      if ((k & mask) == prefix) atomicAdd(&sh.hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // digits from the top until the running count reaches `need`
      uint32_t above = 0;
      for (int d = 255; d >= 0; --d) {
        const uint32_t c = sh.hist[d];
        if (above + c >= need) {
          sh.pick = static_cast<uint32_t>(d);
          sh.need = need - above;
          break;
        }
        above += c;
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

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(const __grid_constant__ SampleArgs args) {
  extern __shared__ __align__(16) uint8_t dyn[];
  SampleShared& sh = *reinterpret_cast<SampleShared*>(dyn);
  uint32_t* cand_key = reinterpret_cast<uint32_t*>(dyn + sizeof(SampleShared));
  uint32_t* cand_idx = cand_key + kSampleCandidates;
  const int64_t row_i = blockIdx.x;
  const int64_t vocab = args.vocab;
  const float* row = args.logits + row_i * args.row_stride;
  const uint32_t k = static_cast<uint32_t>(args.k);
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;

  // Pass 1: thread maxima; the row minimum at its lowest index.
  float tmax = -INFINITY, tmin = INFINITY;
  int64_t imin = INT64_MAX;
  each_logit(row, vocab, [&](float v, int64_t j) {
    tmax = fmaxf(tmax, v);
    if (v < tmin || (v == tmin && j < imin)) {
      tmin = v;
      imin = j;
    }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(kFullMask, tmin, o);
    const int64_t oi = __shfl_xor_sync(kFullMask, imin, o);
    if (ov < tmin || (ov == tmin && oi < imin)) {
      tmin = ov;
      imin = oi;
    }
  }
  if (lane == 0) {
    sh.wmin[warp] = tmin;
    sh.wimin[warp] = imin;
  }
  sh.keys[threadIdx.x] = skey(tmax);
  if (threadIdx.x == 0) {
    sh.count = 0;
    sh.nsel = 0;
    sh.ties = 0;
  }
  __syncthreads();

  // The k-th largest value: candidates >= tau in shared memory, or the whole row.
  const uint32_t tau = select_kth([&](int64_t i) { return sh.keys[i]; }, kSampleThreads, k, sh);
  each_logit(row, vocab, [&](float v, int64_t j) {
    const uint32_t key = skey(v);
    const bool take = key >= tau;
    const unsigned bal = __ballot_sync(__activemask(), take);
    if (bal) {
      const int leader = __ffs(bal) - 1;
      uint32_t base = 0;
      if (lane == leader) base = atomicAdd(&sh.count, static_cast<uint32_t>(__popc(bal)));
      base = __shfl_sync(__activemask(), base, leader);
      const uint32_t at = base + __popc(bal & ((1u << lane) - 1u));
      if (take && at < kSampleCandidates) {
        cand_key[at] = key;
        cand_idx[at] = static_cast<uint32_t>(j);
      }
    }
  });
  __syncthreads();
  const uint32_t nc = sh.count;
  const bool fits = nc <= kSampleCandidates;
  uint32_t kth;
  if (fits) {
    kth = select_kth([&](int64_t i) { return cand_key[i]; }, nc, k, sh);
  } else {
    kth = select_kth([&](int64_t i) { return skey(__ldg(row + i)); }, vocab, k, sh);
  }
  // The number of values strictly above the k-th: the rest of the k are ties at it.
  // Select exactly k: every key > kth, and the first (k - above) ties by arrival.
  auto offer = [&](uint32_t key, int64_t j) {
    if (key > kth) {
      const uint32_t at = atomicAdd(&sh.nsel, 1u);
      if (at < k) {
        sh.sel_key[at] = key;
        sh.sel_idx[at] = j;
      }
    } else if (key == kth) {
      const uint32_t t = atomicAdd(&sh.ties, 1u);
      if (t < k) {  // stored from the top down; trimmed below
        sh.sel_key[k - 1 - t] = key;
        sh.sel_idx[k - 1 - t] = j;
      }
    }
  };
  if (fits) {
    for (uint32_t i = threadIdx.x; i < nc; i += kSampleThreads) offer(cand_key[i], cand_idx[i]);
  } else {
    each_logit(row, vocab, [&](float v, int64_t j) { offer(skey(v), j); });
  }
  __syncthreads();
  // sel[0, above) holds the keys above the k-th, sel[above, k) ties (the ties that landed
  // below `above` were overwritten by larger keys, which is fine: any k-subset of ties is a
  // top-k set). Sort the k keys descending, indices along (bitonic, padded to a power of 2).
  uint32_t P = 1;
  while (P < k) P <<= 1;
  for (uint32_t i = threadIdx.x + k; i < P; i += kSampleThreads) {
    sh.sel_key[i] = 0u;  // below every key of a real value
    sh.sel_idx[i] = -1;
  }
  __syncthreads();
  for (uint32_t size = 2; size <= P; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = threadIdx.x; i < P; i += kSampleThreads) {
        const uint32_t jx = i ^ stride;
        if (jx > i) {
          const bool desc = (i & size) == 0;
          const uint32_t a = sh.sel_key[i], b = sh.sel_key[jx];
          if (desc ? a < b : a > b) {
            sh.sel_key[i] = b;
            sh.sel_key[jx] = a;
            const int64_t t = sh.sel_idx[i];
            sh.sel_idx[i] = sh.sel_idx[jx];
            sh.sel_idx[jx] = t;
          }
        }
      }
      __syncthreads();
    }
  }

  // Softmax over the k, nucleus, draw: one warp, the k values in lane-strided chunks.
  if (warp == 0) {
    const float m = skey_value(sh.sel_key[0]) * args.inv_t;
    // total mass of the k, then the nucleus: positions whose mass before them is below p
    float z = 0.0f;
    for (uint32_t i = lane; i < k; i += kWarp) z += expf(skey_value(sh.sel_key[i]) * args.inv_t - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(kFullMask, z, o);
    const float target_p = args.p * z;
    // prefix sums in chunks of 32: kept = positions with mass before < p * z
    float before = 0.0f, kept_mass = 0.0f;
    uint32_t kept = 0;
    for (uint32_t c0 = 0; c0 < k; c0 += kWarp) {
      const uint32_t i = c0 + lane;
      const float e = i < k ? expf(skey_value(sh.sel_key[i]) * args.inv_t - m) : 0.0f;
      float incl = e;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const float v = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += v;
      }
      const float excl = before + incl - e;
      const bool in = i < k && excl < target_p;
      const unsigned bal = __ballot_sync(kFullMask, in);
      kept += __popc(bal);
      const float chunk_kept = __shfl_sync(kFullMask, in ? excl + e : 0.0f, bal ? 31 - __clz(bal) : 0);
      if (bal) kept_mass = chunk_kept;
      before += __shfl_sync(kFullMask, incl, kWarp - 1);
      if (__popc(bal) < kWarp) break;  // the nucleus ended in this chunk
    }
    kept = kept < 1 ? 1 : kept;
    // inverse CDF over the kept prefix
    const float u = args.draws[row_i];
    const float target = u * kept_mass;
    uint32_t pick = kept - 1;
    float run = 0.0f;
    for (uint32_t c0 = 0; c0 < kept; c0 += kWarp) {
      const uint32_t i = c0 + lane;
      const float e = i < kept ? expf(skey_value(sh.sel_key[i]) * args.inv_t - m) : 0.0f;
      float incl = e;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const float v = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned bal = __ballot_sync(kFullMask, i < kept && run + incl > target);
      if (bal) {
        pick = c0 + static_cast<uint32_t>(__ffs(bal) - 1);
        break;
      }
      run += __shfl_sync(kFullMask, incl, kWarp - 1);
    }
    if (lane == 0) {
      int64_t token = sh.sel_idx[pick];
      bool planted = false;
      if (args.fault_draws != nullptr && args.fault_draws[row_i] < args.fault_rate) {
        float bm = sh.wmin[0];
        int64_t bi = sh.wimin[0];
        for (int w = 1; w < kSampleWarps; ++w) {
          if (sh.wmin[w] < bm || (sh.wmin[w] == bm && sh.wimin[w] < bi)) {
            bm = sh.wmin[w];
            bi = sh.wimin[w];
          }
        }
        token = bi;
        planted = true;
      }
      args.tokens[row_i] = token;
      if (args.injected) args.injected[row_i] = planted ? 1 : 0;
    }
  }
}

}  // namespace

size_t sample_smem_bytes() {
  return sizeof(SampleShared) + 2 * sizeof(uint32_t) * static_cast<size_t>(kSampleCandidates);
}

cudaError_t launch_sample(const float* logits, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k, float p,
                          float inv_t, const float* draws, const float* fault_draws, float fault_rate,
                          int64_t* tokens, uint8_t* injected, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const size_t smem = sample_smem_bytes();
  if (!configured[dev]) {
    const cudaError_t err =
        cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    configured[dev] = 1;
  }
  SampleArgs a{logits, vocab, row_stride, k, p, inv_t, draws, fault_draws, fault_rate, tokens, injected};
  sample_kernel<<<static_cast<unsigned>(rows), kSampleThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace pck

namespace pck {
int report_error(int code, const char* message);
}  // namespace pck

extern "C" int pck_sample_topk_topp(const float* logits, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k,
                                    double p, double temperature, const float* draws, const float* fault_draws,
                                    double fault_rate, int64_t* tokens, uint8_t* injected, void* stream) {
  if (rows < 0 || vocab < 1 || row_stride < vocab) {
    return pck::report_error(PCK_ERR_ARGUMENT, "sampler: need rows >= 0, vocab >= 1 and row_stride >= vocab");
  }
  if (k < 1 || k > vocab || k > 1024) return pck::report_error(PCK_ERR_ARGUMENT, "sampler: k must be in [1, min(vocab, 1024)]");
  if (!(p > 0.0 && p <= 1.0) || !(temperature > 0.0)) {
    return pck::report_error(PCK_ERR_ARGUMENT, "sampler: need 0 < p <= 1 and temperature > 0");
  }
  if (vocab > 0xffffffffLL) return pck::report_error(PCK_ERR_UNSUPPORTED, "sampler: vocab too large");
  if (rows == 0) return PCK_OK;
  if (!logits || !draws || !tokens) return pck::report_error(PCK_ERR_ARGUMENT, "sampler: NULL logits, draws or tokens");
  const cudaError_t err = pck::launch_sample(logits, rows, vocab, row_stride, k, static_cast<float>(p),
                                             static_cast<float>(1.0 / temperature), draws, fault_draws,
                                             static_cast<float>(fault_rate), tokens, injected,
                                             static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) {
    char msg[160];
    snprintf(msg, sizeof msg, "sampler kernel: %s", cudaGetErrorString(err));
    return pck::report_error(PCK_ERR_CUDA, msg);
  }
  return PCK_OK;
}
