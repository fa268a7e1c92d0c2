// The all-gather of the row-sharded outputs over peer memory (NVLink / NVSwitch), in one
// kernel per call, in one of two forms chosen by the slice size (the same on every rank):
//
//   flagged  (slices up to kFlaggedMaxSlice; the decode layer's outputs) every 8 bytes of
//            payload travel as 16 with the call number beside each 4-byte word, in one
//            16-byte store; the receiving threads poll their words until every word carries
//            this call's number. No fence and no counter: the latency is one NVLink store.
//   counted  (larger slices, e.g. the LM head's logits) the slice is stored as is; each CTA
//            then fences at system scope and raises one counter per peer, and the receivers
//            wait until every peer's CTAs have raised theirs.
// Both then leave the assembled slices in `gathered`.
//
// Exchange buffer of each rank (allocated here, mapped into the peers with CUDA IPC):
//   two receive regions      used by calls of odd and even number: a rank writes call e's
//                            slice into region e & 1 of every rank, so it never overwrites
//                            what a slower rank still reads from the previous call (a rank
//                            starts call e + 2 only after every peer has sent its part of
//                            call e + 1, which it sends after finishing call e);
//   counters                 (counted form) one 32-bit counter per source rank (own 128-byte
//                            line), raised once per CTA of that rank per call, never reset:
//                            after call e it holds e * grid;
//   epochs                   the number of calls so far, one per CTA of this rank (each CTA
//                            reads and writes only its own).
// A call needs the previous one on this rank complete (stream order), and every rank to
// make the same sequence of calls with the same slice size, as NCCL collectives do. Each
// wait gives up after kWaitLimitNs with the device timeout bit set, so a rank that never
// arrives cannot hang the others. No multicast and no TMA: plain 16-byte stores to peer
// memory and system-scope atomics.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

#include "pck_b200.h"
#include "pck_common.cuh"

namespace pck {
int report_error(int code, const char* message);

namespace {

constexpr int kPeerThreads = 256;
constexpr int kPeerMaxCtas = 128;
constexpr int64_t kCounterStride = 128;  // bytes: one counter per cache line
constexpr int64_t kFlaggedMaxSlice = 1 << 20;  // bytes of a slice sent in the flagged form

struct PeerParams {
  uint8_t* buffers[PCK_PEER_MAX_RANKS];
  const uint4* local;
  uint4* gathered;
  int64_t slice_words;  // 16-byte words of one rank's slice
  int32_t rank;
  int32_t world;
};

__host__ __device__ constexpr bool flagged_form(int64_t slice_bytes) { return slice_bytes <= kFlaggedMaxSlice; }

// Bytes of one receive region: every rank's slice, twice as large in the flagged form.
__host__ __device__ constexpr int64_t region_bytes(int64_t slice_bytes, int world) {
  return static_cast<int64_t>(world) * slice_bytes * (flagged_form(slice_bytes) ? 2 : 1);
}

__host__ __device__ constexpr int64_t flags_offset(int64_t slice_bytes, int world) {
  return 2 * region_bytes(slice_bytes, world);
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_v4(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_v4_volatile(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// The flagged form. Payload word w (16 bytes) of a slice travels as two 16-byte units
// {d0, e, d1, e} and {d2, e, d3, e} (e = the call number, never 0), at units 2w and 2w + 1 of
// the sender's part of the receive region; each 8-byte half is written in one piece, so a
// receiver that sees e beside a data word sees that word of this call. Sends and receives
// are spread over the (rank, word) pairs, one pair per thread where the grid allows, so the
// polls of different words and peers overlap.
__global__ void __launch_bounds__(kPeerThreads) peer_gather_flagged(const __grid_constant__ PeerParams p) {
  const int64_t slice_bytes = p.slice_words * 16;
  const int64_t region = region_bytes(slice_bytes, p.world);
  uint8_t* self = p.buffers[p.rank];
  unsigned int* epochs = reinterpret_cast<unsigned int*>(self + flags_offset(slice_bytes, p.world) +
                                                         PCK_PEER_MAX_RANKS * kCounterStride);
  __shared__ unsigned int s_epoch;
  // Launched as the programmatic dependent of the kernel that wrote `local`: the next kernel
  // may start now (it waits for this one before it writes anything), and this one waits for
  // the previous before it reads.
  allow_dependents();
  wait_for_producers();
  if (threadIdx.x == 0) s_epoch = epochs[blockIdx.x] + 1;
  __syncthreads();
  const unsigned int e = s_epoch;
  const int64_t base = static_cast<int64_t>(e & 1u) * region;
  const int64_t part = 2 * slice_bytes;  // bytes of one sender's part of a region
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kPeerThreads;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kPeerThreads + threadIdx.x;
  const int64_t pairs = static_cast<int64_t>(p.world) * p.slice_words;
  // send: pair (r, w) stores word w of this rank's slice, flagged, into rank r (its own part
  // of `gathered` directly)
  for (int64_t i = first; i < pairs; i += stride) {
    const int r = static_cast<int>(i / p.slice_words);
    const int64_t w = i - static_cast<int64_t>(r) * p.slice_words;
    const uint4 v = p.local[w];
    if (r == p.rank) {
      p.gathered[p.rank * p.slice_words + w] = v;
      continue;
    }
    uint4* dst = reinterpret_cast<uint4*>(p.buffers[r] + base + p.rank * part) + 2 * w;
    st_v4(dst, make_uint4(v.x, e, v.y, e));
    st_v4(dst + 1, make_uint4(v.z, e, v.w, e));
  }
  // receive: pair (r, w) polls rank r's word w until its flags carry this call's number
  bool ok = true;
  const unsigned long long start = global_ns();
  for (int64_t i = first; i < pairs && ok; i += stride) {
    const int r = static_cast<int>(i / p.slice_words);
    if (r == p.rank) continue;
    const int64_t w = i - static_cast<int64_t>(r) * p.slice_words;
    const uint4* src = reinterpret_cast<const uint4*>(self + base + r * part) + 2 * w;
    uint4 u0, u1;
    int spins = 0;
    while (true) {
      u0 = ld_v4_volatile(src);
      u1 = ld_v4_volatile(src + 1);
      if (u0.y == e && u0.w == e && u1.y == e && u1.w == e) break;
      if (++spins % 64 == 0 && global_ns() - start > kWaitLimitNs) {
        report(kDevTimeout);
        ok = false;
        break;
      }
    }
    if (ok) p.gathered[r * p.slice_words + w] = make_uint4(u0.x, u0.z, u1.x, u1.z);
  }
  __syncthreads();
  if (threadIdx.x == 0) epochs[blockIdx.x] = e;
}

__global__ void __launch_bounds__(kPeerThreads) peer_gather_kernel(const __grid_constant__ PeerParams p) {
  const int64_t slice_bytes = p.slice_words * 16;
  const int64_t flags = flags_offset(slice_bytes, p.world);
  uint8_t* self = p.buffers[p.rank];
  unsigned int* epochs = reinterpret_cast<unsigned int*>(self + flags + PCK_PEER_MAX_RANKS * kCounterStride);
  __shared__ unsigned int s_epoch;
  __shared__ int s_ok;
  allow_dependents();
  wait_for_producers();
  if (threadIdx.x == 0) {
    s_epoch = epochs[blockIdx.x] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned int epoch = s_epoch;
  const int64_t region = static_cast<int64_t>(epoch & 1u) * region_bytes(slice_bytes, p.world);

  // 1. this rank's slice into region `epoch & 1` of every rank (its own included)
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kPeerThreads;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * kPeerThreads + threadIdx.x; w < p.slice_words; w += stride) {
    const uint4 v = p.local[w];
    for (int r = 0; r < p.world; ++r) {
      reinterpret_cast<uint4*>(p.buffers[r] + region + p.rank * slice_bytes)[w] = v;
    }
  }
  // 2. the stores reach every rank before its counter for this rank moves
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world && threadIdx.x != p.rank) {
    unsigned int* counter = reinterpret_cast<unsigned int*>(p.buffers[threadIdx.x] + flags + p.rank * kCounterStride);
    atomicAdd_system(counter, 1u);
  }
  // 3. every peer's CTAs of this call have stored their slices here
  if (threadIdx.x < p.world && threadIdx.x != p.rank) {
    const unsigned int* counter = reinterpret_cast<const unsigned int*>(self + flags + threadIdx.x * kCounterStride);
    const unsigned int target = epoch * gridDim.x;
    const unsigned long long start = global_ns();
    // counters only grow; the difference stays meaningful across the 32-bit wrap
    while (static_cast<int>(load_acquire_sys(counter) - target) < 0) {
      if (global_ns() - start > kWaitLimitNs) {
        report(kDevTimeout);
        s_ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  // 4. the assembled region into `gathered` (skipped if a peer never arrived)
  if (s_ok) {
    const uint4* src = reinterpret_cast<const uint4*>(self + region);
    const int64_t words = p.slice_words * p.world;
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * kPeerThreads + threadIdx.x; w < words; w += stride) {
      p.gathered[w] = src[w];
    }
  }
  if (threadIdx.x == 0) epochs[blockIdx.x] = epoch;
}

}  // namespace

PCK_STATUS_READER(peer_status)

}  // namespace pck

namespace {

int peer_fail(int code, const char* what, cudaError_t err) {
  char msg[256];
  snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(err));
  return pck::report_error(code, msg);
}

}  // namespace

extern "C" int64_t pck_peer_buffer_bytes(int64_t slice_bytes, int world) {
  if (slice_bytes < 0 || world < 1) return -1;
  return pck::flags_offset(slice_bytes, world) + PCK_PEER_MAX_RANKS * pck::kCounterStride +
         pck::kPeerMaxCtas * static_cast<int64_t>(sizeof(unsigned int));
}

extern "C" int pck_peer_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes < 1) return pck::report_error(PCK_ERR_ARGUMENT, "peer buffer: need a size and an output pointer");
  *ptr = nullptr;
  cudaError_t err = cudaMalloc(ptr, static_cast<size_t>(bytes));
  if (err != cudaSuccess) return peer_fail(PCK_ERR_CUDA, "peer buffer allocation", err);
  err = cudaMemset(*ptr, 0, static_cast<size_t>(bytes));
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return peer_fail(PCK_ERR_CUDA, "peer buffer initialisation", err);
  }
  return PCK_OK;
}

extern "C" int pck_peer_free(void* ptr) {
  const cudaError_t err = cudaFree(ptr);
  return err == cudaSuccess ? PCK_OK : peer_fail(PCK_ERR_CUDA, "peer buffer free", err);
}

extern "C" int pck_peer_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return pck::report_error(PCK_ERR_ARGUMENT, "peer export: NULL argument");
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (err != cudaSuccess) return peer_fail(PCK_ERR_CUDA, "peer export", err);
  static_assert(sizeof(h) <= PCK_PEER_HANDLE_BYTES, "IPC handle larger than the exported bytes");
  memset(handle, 0, PCK_PEER_HANDLE_BYTES);
  memcpy(handle, &h, sizeof h);
  return PCK_OK;
}

extern "C" int pck_peer_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return pck::report_error(PCK_ERR_ARGUMENT, "peer import: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  *ptr = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return err == cudaSuccess ? PCK_OK : peer_fail(PCK_ERR_CUDA, "peer import", err);
}

extern "C" int pck_peer_close(void* ptr) {
  const cudaError_t err = cudaIpcCloseMemHandle(ptr);
  return err == cudaSuccess ? PCK_OK : peer_fail(PCK_ERR_CUDA, "peer close", err);
}

extern "C" int pck_peer_all_gather(const pck_peer_gather* g, void* stream) {
  if (!g) return pck::report_error(PCK_ERR_ARGUMENT, "peer gather: NULL descriptor");
  if (g->world < 1 || g->world > PCK_PEER_MAX_RANKS || g->rank < 0 || g->rank >= g->world) {
    return pck::report_error(PCK_ERR_ARGUMENT, "peer gather: rank outside the world (at most 8 ranks)");
  }
  if (g->slice_bytes < 0 || g->slice_bytes % 16 != 0) {
    return pck::report_error(PCK_ERR_ARGUMENT, "peer gather: the slice must be a multiple of 16 bytes");
  }
  if (!g->local || !g->gathered || reinterpret_cast<uintptr_t>(g->local) % 16 ||
      reinterpret_cast<uintptr_t>(g->gathered) % 16) {
    return pck::report_error(PCK_ERR_ARGUMENT, "peer gather: local and gathered must be 16-byte aligned");
  }
  for (int r = 0; r < g->world; ++r) {
    if (!g->buffers[r] || reinterpret_cast<uintptr_t>(g->buffers[r]) % 16) {
      return pck::report_error(PCK_ERR_ARGUMENT, "peer gather: every rank's buffer must be mapped and aligned");
    }
  }
  if (g->slice_bytes == 0) return PCK_OK;
  pck::PeerParams p{};
  for (int r = 0; r < g->world; ++r) p.buffers[r] = static_cast<uint8_t*>(g->buffers[r]);
  p.local = static_cast<const uint4*>(g->local);
  p.gathered = static_cast<uint4*>(g->gathered);
  p.slice_words = g->slice_bytes / 16;
  p.rank = g->rank;
  p.world = g->world;
  // The same grid on every rank (it depends on the slice and the world only): the flagged
  // form one (rank, word) pair per thread, the counted form about 4 words a thread.
  const bool flagged = pck::flagged_form(g->slice_bytes);
  const int64_t want = flagged ? (p.world * p.slice_words + pck::kPeerThreads - 1) / pck::kPeerThreads
                               : (p.slice_words + pck::kPeerThreads * 4 - 1) / (pck::kPeerThreads * 4);
  const int grid = static_cast<int>(want < 1 ? 1 : want > pck::kPeerMaxCtas ? pck::kPeerMaxCtas : want);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(pck::kPeerThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // starts during the kernel before
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = flagged ? cudaLaunchKernelEx(&cfg, pck::peer_gather_flagged, p)
                                  : cudaLaunchKernelEx(&cfg, pck::peer_gather_kernel, p);
  return err == cudaSuccess ? PCK_OK : peer_fail(PCK_ERR_CUDA, "peer gather kernel", err);
}
