// pck_gemv_checked_static: the fused checked GEMV of pck_gemv_checked for callers that
// cannot allocate device memory.
//
// A check needs scratch beside its inputs and outputs: the binary64 partial sums of the
// checksum and bound rows, per row block and column segment. pck_gemv_checked takes that
// scratch from the caller. Some callers have none to give: a serving engine that reserved
// almost all of HBM for its own pool up front (a cudaMalloc beside it can fail, and is
// invisible to its memory accounting), or a host runtime that reaches this library through
// a plain C FFI with only the device pointers the engine handed it, and no allocator of its
// own. This entry point serves them from one array of PCK_STATIC_SCRATCH_BYTES that lives in
// this library's device code, so it allocates no device memory at all.
//
// The array is shared by every call on a device and keeps what the last call left in it.
// Nothing in it has to start at zero: every partial sum is written by the streaming kernel
// before the verdict kernel of the same call reads it. Two calls whose work overlaps on the GPU (other streams, other host threads) race on the
// array and may produce wrong verdicts; keep the calls of one device on one stream, or
// order them.
//
// The address of the array on a device is looked up by the first call made while that
// device is current, and cached together with the device's current context; that first call
// should come before any stream capture. A call that finds another context current on the
// device (after cudaDeviceReset, or under a context of the driver API) looks it up again.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "pck_b200.h"

namespace pck {
int report_error(int code, const char* message);
}  // namespace pck

// The scratch of pck_gemv_checked_static on each device: the checks' partial sums, every
// region aligned to 256 bytes.
static __device__ __align__(256) unsigned char g_static_scratch[PCK_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kRegionAlign = 256;
constexpr int64_t kLimit = PCK_STATIC_SCRATCH_BYTES;
constexpr int64_t kSaturated = INT64_MAX / 4;

// Per device: the context the address was looked up in, and the address.
struct Cached {
  CUcontext ctx;
  unsigned char* base;
};
std::mutex g_setup;
Cached g_cache[kMaxDevices];

// cuCtxGetCurrent from the driver, through the runtime (no link against libcuda).
using CtxGetCurrent = CUresult (*)(CUcontext*);
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      return reinterpret_cast<CtxGetCurrent>(p);
    }
    return static_cast<CtxGetCurrent>(nullptr);
  }();
  return fn;
}

__attribute__((format(printf, 2, 3))) int reject(int code, const char* fmt, ...) {
  char msg[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof msg, fmt, ap);
  va_end(ap);
  return pck::report_error(code, msg);
}

// Address of the array on the current device, looked up once per device and context.
int scratch_base(unsigned char** base) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return reject(PCK_ERR_CUDA, "static scratch set-up failed: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) {
    return reject(PCK_ERR_UNSUPPORTED, "device %d is beyond the %d devices served", dev, kMaxDevices);
  }
  const CtxGetCurrent current = ctx_get_current();
  if (!current) return reject(PCK_ERR_CUDA, "static scratch set-up failed: cuCtxGetCurrent is unavailable");
  CUcontext ctx = nullptr;  // NULL until the runtime has made a context current on this thread
  if (current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_setup);
  Cached& entry = g_cache[dev];
  if (!ctx || !entry.base || entry.ctx != ctx) {
    void* addr = nullptr;
    err = cudaGetSymbolAddress(&addr, g_static_scratch);  // makes the primary context current if none is
    if (err != cudaSuccess || !addr) {
      return reject(PCK_ERR_CUDA, "static scratch set-up failed: %s",
                    err != cudaSuccess ? cudaGetErrorString(err) : "no address");
    }
    if (current(&ctx) != CUDA_SUCCESS || !ctx) {
      return reject(PCK_ERR_CUDA, "static scratch set-up failed: no current context");
    }
    entry.ctx = ctx;
    entry.base = static_cast<unsigned char*>(addr);
  }
  *base = entry.base;
  return PCK_OK;
}

// a * b for non-negative operands, saturated far above the limit.
int64_t mul_sat(int64_t a, int64_t b) {
  if (a == 0 || b == 0) return 0;
  return a > kSaturated / b ? kSaturated : a * b;
}

int64_t region(int64_t bytes) {
  return bytes >= kSaturated ? kSaturated : (bytes + kRegionAlign - 1) / kRegionAlign * kRegionAlign;
}

// Whether the sizes of `d` are ones pck_gemv_checked accepts (others are left for its own
// argument checks to report, with no scratch reserved).
bool sized(const pck_check_desc* d) {
  return d->batch >= 1 && d->batch <= 16 && d->checks >= 1 && d->num_blocks >= 1 && d->n >= 1 &&
         d->segments >= 1 && d->segments <= d->n;
}

}  // namespace

extern "C" int pck_gemv_checked_static(const pck_gemv_job* jobs, int count, void* stream) {
  if (count < 1 || count > PCK_MAX_JOBS || !jobs) return pck_gemv_checked(jobs, count, stream);

  pck_gemv_job local[PCK_MAX_JOBS];
  pck_check_desc descs[PCK_MAX_JOBS];
  int64_t cx_at[PCK_MAX_JOBS], s_at[PCK_MAX_JOBS];

  // Layout: each check's c . x partials, then its a . |x| partials.
  int64_t used = 0;
  for (int i = 0; i < count; ++i) {
    local[i] = jobs[i];
    cx_at[i] = s_at[i] = 0;
    if (!jobs[i].check) continue;
    descs[i] = *jobs[i].check;
    local[i].check = &descs[i];
    if (!sized(&descs[i])) continue;
    const pck_check_desc& d = descs[i];
    const int64_t cells = mul_sat(mul_sat(d.batch, d.num_blocks), d.segments);
    cx_at[i] = used;
    used += region(mul_sat(mul_sat(cells, d.checks), 8));
    s_at[i] = used;
    used += region(mul_sat(cells, 8));
    if (used > kLimit) break;
  }
  if (used > kLimit) {
    if (used >= kSaturated) {
      return reject(PCK_ERR_ARGUMENT, "the checks need more scratch than the static limit of %lld bytes",
                    static_cast<long long>(kLimit));
    }
    return reject(PCK_ERR_ARGUMENT,
                  "the checks need %lld bytes of scratch, more than the static limit of %lld bytes",
                  static_cast<long long>(used), static_cast<long long>(kLimit));
  }

  unsigned char* base = nullptr;
  if (int rc = scratch_base(&base)) return rc;
  for (int i = 0; i < count; ++i) {
    if (!jobs[i].check) continue;
    descs[i].counters = nullptr;
    descs[i].partial_cx = reinterpret_cast<double*>(base + cx_at[i]);
    descs[i].partial_s = reinterpret_cast<double*>(base + s_at[i]);
  }
  return pck_gemv_checked(local, count, stream);
}
