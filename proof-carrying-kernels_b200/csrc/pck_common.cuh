// Shared device helpers for the sm_100a kernels: mbarriers, bulk async copies, bounded
// waits and the library's device-side error status.
//
// Every spin on an mbarrier is bounded by wall time (the %globaltimer register): a wait
// that has not completed after kWaitLimitNs records PCK_DEV_TIMEOUT in the status word and
// gives up, so a kernel never hangs the GPU even if a copy were lost.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace pck {

constexpr int kWarp = 32;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr unsigned long long kWaitLimitNs = 4000000000ull;  // 4 s

// Device status bits (read with pck_device_status).
constexpr unsigned kDevTimeout = 1u;

// Device status word. Without relocatable device code every translation unit has its own
// copy (internal linkage); each unit exposes a reader (PCK_STATUS_READER) and
// pck_device_status() ORs them together.
static __device__ unsigned int g_device_status = 0;

#define PCK_STATUS_READER(fn)                                                         \
  cudaError_t fn(unsigned int* value, bool clear) {                                   \
    cudaError_t err = cudaMemcpyFromSymbol(value, g_device_status, sizeof(unsigned)); \
    if (err != cudaSuccess || !clear) return err;                                     \
    const unsigned int zero = 0;                                                      \
    return cudaMemcpyToSymbol(g_device_status, &zero, sizeof zero);                   \
  }

__device__ __forceinline__ void report(unsigned bits) { atomicOr(&g_device_status, bits); }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits until the phase with the given parity of `bar` has completed. Returns false (and
// records a timeout) if that takes longer than kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      if (mbar_test(bar, parity)) return true;
    }
    if (global_ns() - start > kWaitLimitNs) {
      report(kDevTimeout);
      return false;
    }
  }
}

// mbar_wait for waits that usually last long (a whole tile of work): each try suspends the
// thread in hardware for up to `hint_ns` or until the phase completes, instead of spinning,
// so waiting warps leave the issue slots to the warps that compute. Bounded like mbar_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 20000) {
  const unsigned long long start = global_ns();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    if (done) return true;
    if (global_ns() - start > kWaitLimitNs) {
      report(kDevTimeout);
      return false;
    }
  }
}

// L2 policy for data read exactly once (weights, bank rows).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 policy for data every CTA reads (activations).
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to
// this CTA's shared memory, completing as transaction bytes on `bar`. No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: let the next kernel of the stream start its prologue
// now, and wait until the previous kernel's writes are visible (a no-op when this kernel
// was launched without the programmatic attribute or the previous one has finished).
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_for_producers() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// bfloat16 halves of a 32-bit word as binary32 (exact): low half first in memory.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Two E4M3 values (low byte first) to binary32, exactly: E4M3 -> f16x2 is exact.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t pair) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(pair));
  float lo, hi;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "r"(h2));
  return make_float2(lo, hi);
}

__device__ __forceinline__ float e4m3_to_float(uint8_t b) {
  return e4m3x2_to_float2(static_cast<uint16_t>(b)).x;
}

}  // namespace pck
