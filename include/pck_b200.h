/*
 * pck_b200 — C ABI of the B200-native checked decode path (sm_100a).
 *
 * These entry points replace the pybind11 module `pck_kernels` of the reference project
 * r7919/proof-carrying-kernels (src/pck/cuda/csrc/bindings.cpp:302-335) and its internal
 * launchers (bindings.cpp:15-38). Every function takes plain device pointers, sizes and a
 * CUDA stream (`void*` holding a cudaStream_t; NULL is the legacy default stream), launches
 * asynchronously on that stream, and returns PCK_OK or an error code; the message of the
 * last failing call on this host thread is available from pck_last_error().
 *
 * Conventions shared by all entry points:
 *   - bfloat16 and E4M3 data are passed as untyped pointers to their bit patterns;
 *   - matrices are row-major and contiguous; W (m, n) holds output rows;
 *   - inputs are only read; outputs are written; scratch buffers named as such must stay
 *     untouched by other work while a call that uses them is in flight (one stream);
 *   - a call with m == 0 (or rows == 0) launches nothing and succeeds.
 */
#ifndef PCK_B200_H
#define PCK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PCK_OK 0
#define PCK_ERR_ARGUMENT 1    /* a size, pointer, alignment or option is invalid */
#define PCK_ERR_CUDA 2        /* a CUDA runtime call failed; see pck_last_error() */
#define PCK_ERR_UNSUPPORTED 3 /* valid input this build does not handle */

#define PCK_WEIGHTS_BF16 0
#define PCK_WEIGHTS_E4M3 1
/*
 * Flag OR-ed into a job's weight_format: the weights were written before the kernel that
 * precedes this call on its stream began (e.g. loaded at start-up, followed by a
 * synchronize). The streaming and tensor-core kernels then request their first weight
 * pieces while that kernel is still running (programmatic dependent launch); without the
 * flag they wait for the preceding kernel to complete before reading any weight, as they
 * do for the checksum bank (c, a) unless its check carries PCK_CHECK_BANK_SETTLED, and
 * always for the activations. A caller that sets the flag
 * while the preceding kernel writes W can get stale weights and false alarms. (For
 * pck_gemv_tc every job of the call must carry it.)
 */
#define PCK_WEIGHTS_SETTLED 0x100
/*
 * Flag OR-ed into a job's weight_format for pck_gemv_tc: every output accumulates its whole
 * K range in one tensor-memory chain, so its value does not depend on which other rows share
 * the launch (the row shards of one matrix, each computed by its own call, concatenate bit
 * for bit to the unsharded result). Without it a launch of few tiles may split K over a
 * cluster of CTAs and add the partial sums, which is faster but rounds differently.
 */
#define PCK_TC_FULL_K 0x200

/* Message of the last failing call on this thread ("" if none). */
const char* pck_last_error(void);

/* ABI version of this library (increases when a declaration here changes): 6. */
int pck_abi_version(void);

/*
 * SHA-256 (hex) over the sources this library was compiled from (csrc/, include/ and the
 * compiler flags), as computed by the build; pck.manifest compares it with the sources on
 * disk and their pinned hashes. No counterpart in the reference, whose checker is compiled
 * at import time from the pinned sources themselves (src/pck/cuda/_ext.py:20-29).
 */
const char* pck_source_digest(void);

/*
 * Device status word shared by every kernel of the library: bit 0 = a bounded wait gave up
 * (the result of that launch is not valid). Synchronizes the current device, stores the
 * word in *status and, if `clear`, resets it.
 */
int pck_device_status(unsigned int* status, int clear);

/* ------------------------------------------------------------------------------------ */
/* GEMV: y = W x with binary32 accumulation in the reference's summation tree.           */

/*
 * Naive tree: thread t of `threads` (a power of two in [1, 1024]) sums the contiguous
 * columns [t*ceil(n/threads), ...) in order, then a pairwise tree (t += t + stride).
 * Bit-exact with the reference model `emulate_gemv` (src/pck/gemv.py:14-57).
 * Replaces bindings.cpp:73-75 / gemv_kernel.cu:204-211 (`gemv_naive`).
 */
int pck_gemv_naive(const void* W, const void* x, float* y, int64_t m, int64_t n, int threads,
                   void* stream);

/*
 * Coalesced tree: chain t (threads a power of two in [32, 1024]) owns the 8-column vectors
 * t, t + threads, ...; chains are halved within groups of 32, then across groups.
 * Bit-exact with `emulate_gemv_coalesced(W, x, threads, 8)` (src/pck/gemv.py:71-101).
 * Replaces bindings.cpp:77-79 / gemv_kernel.cu:182-191 (`gemv_coalesced`).
 */
int pck_gemv_coalesced(const void* W, const void* x, float* y, int64_t m, int64_t n,
                       int threads, void* stream);

/*
 * E4M3 weights Q (m, n), bfloat16 x: z = Q x with the coalesced tree over 16-column
 * vectors, bit-exact with `emulate_gemv_coalesced(Q, x, threads, 16)`. The per-row scales
 * of the quantisation are applied by the caller afterwards (y = s * z).
 * Replaces bindings.cpp:81-83 / gemv_kernel.cu:193-202 (`gemv_fp8`).
 */
int pck_gemv_fp8(const void* Q, const void* x, float* z, int64_t m, int64_t n, int threads,
                 void* stream);

/*
 * Batched coalesced GEMV: Y (batch, m) = X (batch, n) W^T, every column of the batch
 * bit-exact with the single-vector tree above (vec 8 for bfloat16, 16 for E4M3),
 * batch in [1, 16]. The reference has no library counterpart; its diagnostic
 * harness/csrc/batched_gemv.cu:25-82 computes the same product for batch <= 8.
 */
int pck_gemv_batched(int weight_format, const void* W, const void* X, float* Y, int64_t m,
                     int64_t n, int64_t batch, int threads, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Blocked checksum checker (the trusted check of y = W x).                               */

/*
 * One GEMV output to check, with the bank built at weight load (src/pck/cuda/checker.py:
 * 72-129). For every column b of the batch, check k and row block beta:
 *   rho = c[k,beta] . x_b - r[k,beta] . y_b[beta]             (binary64, exact products)
 *   s   = a[beta] . |x_b|                                       (binary64, rounded up)
 *   tau = coef*s + geps*((1+u32) s + sum |y_b[beta]|) + tau_floor   (rounded up)
 *   passed = every y in the block finite && tau finite && |rho| <= tau
 * (the decision rule of src/pck/cuda/csrc/checker_kernel.cu:87-185). Mirrors the
 * reference's `CheckDesc` (src/pck/cuda/csrc/checker.h:13-34), extended by a batch.
 */
typedef struct pck_check_desc {
  const float* c;       /* (checks, num_blocks, n) binary32 checksums r^T W_beta        */
  const void* a;        /* (num_blocks, n) bfloat16, rounded up                          */
  const int8_t* r;      /* (checks, num_blocks, block) signs, +-1                        */
  const void* x;        /* (batch, n) bfloat16                                            */
  const float* y;       /* (batch, num_blocks*block) binary32 output to check            */
  double* partial_cx;   /* scratch (batch, checks, num_blocks, segments)                 */
  double* partial_s;    /* scratch (batch, num_blocks, segments)                         */
  uint32_t* counters;   /* unused since ABI version 2 (may be NULL)                      */
  uint8_t* passed;      /* out (batch, checks, num_blocks), 1 = passed                   */
  double* rho;          /* out (batch, checks, num_blocks)                               */
  double* tau;          /* out (batch, checks, num_blocks)                               */
  int64_t n;
  int32_t block;
  int32_t num_blocks;
  int32_t checks;
  int32_t segments;     /* column segments per bank row, in [1, n]                        */
  int32_t batch;        /* columns of x and y, in [1, 16]                                 */
  int32_t flags;        /* 0 or PCK_CHECK_BANK_SETTLED                                    */
  double coef;          /* >= gamma_h + u32, rounded up                                   */
  double geps;          /* >= the checker's own rounding constant, rounded up             */
  double tau_floor;     /* >= n 2^-148, rounded up                                        */
  const double* c64;    /* optional: c widened to binary64, same shape (or NULL); the
                           tensor-core GEMV's fused reduction then reads it instead of c    */
} pck_check_desc;

/*
 * Check flag: c and a were written before the kernel preceding this launch on the stream
 * began (the bank is built at weight load), so the streaming kernel's bank CTAs may request
 * their first bank pieces before that kernel completes, as PCK_WEIGHTS_SETTLED lets the row
 * CTAs do for W (it takes effect in launches whose weights are all settled). A caller that
 * sets it while the preceding kernel writes the bank can get false alarms.
 */
#define PCK_CHECK_BANK_SETTLED 0x1

#define PCK_MAX_JOBS 16

/*
 * Checks up to PCK_MAX_JOBS GEMV outputs (the standalone check, run after the producing
 * kernel has finished): one launch streams the bank rows into the partial sums, a second
 * one decides every block. Replaces bindings.cpp:221-256 (`blocked_check`) and
 * checker_kernel.cu:189-196; the reference batches at most 8.
 */
int pck_blocked_check(const pck_check_desc* descs, int count, void* stream);

/*
 * One GEMV, optionally checked in the same pass over memory.
 * weight_format: PCK_WEIGHTS_BF16 (vec 8) or PCK_WEIGHTS_E4M3 (vec 16), optionally OR-ed
 * with PCK_WEIGHTS_SETTLED.
 * If `check` is not NULL, its x and y must equal this job's X and Y; the streaming kernel
 * reduces the job's bank rows against x together with W (fused production mode), and the
 * verdict of each row block is then computed from the y values as stored in memory.
 */
typedef struct pck_gemv_job {
  const void* W;                /* (m, n) weights                                         */
  const void* X;                /* (batch, n) bfloat16                                    */
  float* Y;                     /* (batch, m) binary32                                    */
  int64_t m;
  int64_t n;
  int32_t batch;                /* [1, 16]                                                */
  int32_t threads;              /* tree parameter, power of two in [32, 1024]             */
  int32_t weight_format;
  /* bfloat16 weights only, optional (0 = unknown): the smallest exponent field (bits
     7-14) of a nonzero weight, subnormals counted as 1, and the largest exponent field.
     When they and the activations prove every product exact in binary32, the kernel
     adds each product with one FMA, which is then bit-identical to product-then-sum. */
  int16_t w_exp_min;
  int16_t w_exp_max;
  const pck_check_desc* check;  /* NULL: unchecked                                        */
} pck_gemv_job;

/*
 * Up to PCK_MAX_JOBS independent GEMVs (each optionally checked) in one persistent launch
 * of the streaming kernel, e.g. the q, k, v projections of a decode layer with their checks,
 * followed by one launch of the verdict kernel for the checked jobs. No reference
 * counterpart: the reference launches each GEMV and the check separately.
 */
int pck_gemv_checked(const pck_gemv_job* jobs, int count, void* stream);

/*
 * pck_gemv_checked without the verdicts: the GEMVs and their checks' partial sums only.
 * The caller decides the blocks later with pck_check_verdicts on the same stream (before
 * reusing the checks' scratch), e.g. once for all checks of a decode layer, as the
 * reference runs one checker launch per layer. No reference counterpart.
 */
int pck_gemv_partials(const pck_gemv_job* jobs, int count, void* stream);

/*
 * pck_gemv_partials that also decides up to PCK_MAX_JOBS `prior` checks whose partial sums
 * and outputs earlier kernels on this stream produced (typically the previous
 * pck_gemv_pipelined call of a decode layer): the same decisions, bit for bit, as
 * pck_check_verdicts on those descriptors, without a launch of their own — each warp of the
 * streaming kernel decides its share of the prior blocks while its first weight copies are in
 * flight. The prior checks' y, scratch and verdict arrays must not overlap the outputs or
 * scratch of this call's jobs (rejected with PCK_ERR_ARGUMENT); nprior = 0 is
 * pck_gemv_partials. The last launch of a sequence leaves its own checks to
 * pck_check_verdicts (or to the next sequence). No reference counterpart: the reference
 * decides every layer's checks in a checker launch of their own.
 */
int pck_gemv_pipelined(const pck_gemv_job* jobs, int count, const pck_check_desc* prior, int nprior,
                       void* stream);

/*
 * pck_gemv_pipelined for a launch that is followed on the stream by a known one (`next`, the
 * jobs of that launch, e.g. the next projection group of a decode layer, which will decide
 * this call's checks): as each CTA of this launch finishes its work, it prefetches into L2
 * the first weight pieces that the same-numbered CTA of the next launch will read, so that
 * launch starts from L2 while this one's last CTAs still stream. The results are those of
 * pck_gemv_pipelined; nnext = 0 is pck_gemv_pipelined. No reference counterpart.
 */
int pck_gemv_pipelined_next(const pck_gemv_job* jobs, int count, const pck_check_desc* prior, int nprior,
                            const pck_gemv_job* next, int nnext, void* stream);

/*
 * The block verdicts of up to PCK_MAX_JOBS checks whose partial sums an earlier
 * pck_gemv_partials call on this stream computed (same descriptors), reading y as stored.
 * The decision rule of src/pck/cuda/csrc/checker_kernel.cu:146-184.
 */
int pck_check_verdicts(const pck_check_desc* descs, int count, void* stream);

/*
 * pck_gemv_checked for callers that cannot allocate device memory: a serving engine that
 * reserved nearly all of HBM for its own pool (a cudaMalloc beside it can fail and escapes
 * its accounting), or a host runtime that reaches this library through a plain C FFI holding
 * only device pointers the engine gave it. The checks' scratch (the partial sums; the
 * scratch fields of each job's descriptor are ignored and may be NULL) comes from one array
 * of PCK_STATIC_SCRATCH_BYTES inside this library, one per device. A call needs, per checked
 * job, 8*batch*checks*num_blocks*segments bytes for the c . x partials and
 * 8*batch*num_blocks*segments bytes for the a . |x| partials, each region rounded up to 256
 * bytes; a call needing more is rejected with PCK_ERR_ARGUMENT before any work. Nothing is
 * allocated: the call launches the same kernels as pck_gemv_checked, with bit-identical
 * results; nothing in the array has to start at zero, since every partial sum is written
 * before it is read. All calls on a device share the array, which keeps the last call's
 * contents: calls whose work overlaps on the GPU (different streams or host threads) race
 * and must be ordered by the caller. The first call on each device (with that device
 * current) looks up the array's address with cudaGetSymbolAddress; make that first call
 * before any stream capture. A later call that finds another context current on the device
 * (after cudaDeviceReset, or under a driver-API context) looks the address up again.
 * No counterpart in the reference.
 */
#define PCK_STATIC_SCRATCH_BYTES (4 << 20)
int pck_gemv_checked_static(const pck_gemv_job* jobs, int count, void* stream);

/*
 * Builds a checker's bank on the device from bfloat16 W (m, n) and signs r
 * (checks, m/block, block): c[k,beta,j] = fl32(sum_i r[k,beta,i] W[beta*block+i, j])
 * (binary64 sum over i in order, then rounded to nearest binary32) and
 * a[beta,j] = round_up_bf16(next_up(fl64(sum_i |W_ij|) * sum_up_factor)), where
 * `sum_up_factor` is passed by the caller. Replaces the weight-load arithmetic of
 * src/pck/cuda/checker.py:94-107 (torch einsum and `round_up_bf16`, :29-43).
 */
int pck_bank_build(const void* W, const int8_t* r, float* c, void* a, int64_t m, int64_t n,
                   int block, int checks, double sum_up_factor, void* stream);

/*
 * Batched GEMV on the tensor cores (tcgen05) for decode batches of 1 to 256: Y (batch, m) =
 * X (batch, n) W^T for up to 8 jobs sharing the batch and weight format; bfloat16 X, bfloat16
 * W (n a multiple of 8) or E4M3 W (n a multiple of 16, widened exactly to bfloat16 in shared
 * memory), W and X 16-byte aligned; binary32 outputs accumulated in tensor memory. Not
 * bit-exact to the coalesced tree: the tensor core adds 16 exact products per MMA and n/16
 * MMAs in sequence (or K ranges of them, added in rank order, unless PCK_TC_FULL_K is set),
 * so a checker of these outputs takes that accumulation's declared height
 * (pck.cuda.gemv.tc_height). `threads` and the exponent range are unused. A job's `check`
 * (optional; the job's own X, Y and shape, batch up to 256) is decided in the same call: for
 * 128-row blocks, at most 2 sign draws and batches up to 128 the GEMV kernel itself reduces
 * the bank rows against the staged X tiles in binary64 (exact products, the bound rounded
 * up); other checks take a bank launch of their own; a verdict launch follows. The reference
 * has no counterpart; its batched decode runs batch-1 GEMVs (harness/csrc/batched_gemv.cu:25-82
 * is a CUDA-core diagnostic).
 */
int pck_gemv_tc(const pck_gemv_job* jobs, int count, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Top-k / top-p set check of a sampler's selection.                                       */

/*
 * For row b of logits (rows, vocab) (binary32) and the selection selected[b, :lengths[b]]
 * (selected is (rows, max_len) int64): passed[b] = the selection is well formed (length in
 * [1, max_len], at most vocab, distinct ids in range, and equal to k when top_p is 0), no
 * logit is NaN, and min over selected >= max over rejected; when top_p is nonzero also
 * mass >= p - slack and mass_without_smallest < p + slack, masses of the softmax at
 * `temperature` from binary32 expf terms on an exact split argument summed in binary64.
 * min_selected, max_rejected, mass and without (mass less the smallest selected term) are
 * written per row (masses 0 unless computed). `segments` in [1, vocab] splits a row between
 * up to 8 CTAs (one cluster); verdicts do not depend on it. `slack` comes from the caller
 * (src/pck/cuda/sampling.py:62-90). No scratch memory. Replaces bindings.cpp:260-300
 * (`sampling_check`) and src/pck/cuda/csrc/sampling_kernel.cu:38-229.
 */
int pck_sampling_check(const float* logits, const int64_t* selected, const int64_t* lengths, int64_t rows,
                       int64_t vocab, int64_t max_len, int64_t k, int top_p, double p, double temperature,
                       double slack, int64_t segments, uint8_t* passed, float* min_selected,
                       float* max_rejected, double* mass, double* without, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Sampled-token membership check.                                                        */

#define PCK_LOGITS_F32 0
#define PCK_LOGITS_BF16 1
#define PCK_LOGITS_F16 2

/*
 * For every row b of logits (rows, vocab) (row b at logits + b*row_stride elements) and its
 * sampled token tokens[b]: above[b] = #{j : l_j > l_t} (t clamped into range for the
 * gather); ok[b] = no NaN in the row && 0 <= t < vocab && above < (greedy[b] ? 1 : k) with
 * k = top_k[b] clamped to [1, vocab] (vocab when top_k is NULL); when top_p is not NULL,
 * rows with p = top_p[b] < 1 also compute r = (mass of kept logits above l_t) / (mass of
 * kept logits), kept = logits >= the k-th largest, with binary32 terms e^(l - max) from the
 * exact TwoSum split summed in binary64, and require p >= 1 || greedy || r <
 * nextafter(p + slack, +inf); mass_above[b] = r there, else 0. `slack` is
 * next_up(tol + member_eps32(vocab)) (src/pck/member.py:84-102). greedy may be NULL.
 * Replaces the torch implementation `check_members` (src/pck/member.py:118-197), which
 * the reference runs as some 80 kernel launches; here one launch, one CTA per row.
 */
int pck_member_check(const void* logits, int logits_dtype, int64_t rows, int64_t vocab,
                     int64_t row_stride, const int64_t* tokens, const int64_t* top_k,
                     const double* top_p, const uint8_t* greedy, double slack, uint8_t* ok,
                     int64_t* above, double* mass_above, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Untrusted top-k / top-p sampler (checked afterwards by pck_member_check).              */

/*
 * For every row b of binary32 logits (rows, vocab) (row b at logits + b*row_stride): with
 * l = logits / temperature, the k largest values (1 <= k <= 1024; ties at the k-th value by
 * position), their binary32 softmax, the shortest prefix in descending order whose mass
 * before each kept position is below p, and an inverse-CDF draw from it with draws[b]
 * (uniform in [0, 1)): tokens[b]. When fault_draws is not NULL and fault_draws[b] <
 * fault_rate, tokens[b] is the row's argmin instead and injected[b] = 1 (else 0; injected
 * may be NULL). One launch, one CTA per row, no scratch memory. Not part of the trusted
 * path: the reference samples with torch (vLLM's sampler, src/pck/vllm_plugin.py, and the
 * untrusted samplers of src/pck/cuda/sampling.py:96-136), and every token is checked by the
 * membership kernel.
 */
int pck_sample_topk_topp(const float* logits, int64_t rows, int64_t vocab, int64_t row_stride, int64_t k, double p,
                         double temperature, const float* draws, const float* fault_draws, double fault_rate,
                         int64_t* tokens, uint8_t* injected, void* stream);

/* ------------------------------------------------------------------------------------ */
/* All-gather of row-sharded outputs over peer memory (one process per GPU of one node).  */

#define PCK_PEER_MAX_RANKS 8
#define PCK_PEER_HANDLE_BYTES 64

/*
 * Every rank's exchange buffer as mapped in this process (this rank's own at [rank], the
 * others from pck_peer_import), this rank's slice `local` (slice_bytes, a multiple of 16,
 * the same on every rank) and `gathered` (world * slice_bytes) for the result: slice r of
 * `gathered` is rank r's `local`. Buffers hold pck_peer_buffer_bytes(slice_bytes, world)
 * bytes each, from pck_peer_alloc.
 */
typedef struct pck_peer_gather {
  void* buffers[PCK_PEER_MAX_RANKS];
  const void* local;
  void* gathered;
  int64_t slice_bytes;
  int32_t rank;
  int32_t world;
} pck_peer_gather;

/* Bytes of an exchange buffer for slices of `slice_bytes` over `world` ranks (-1 if invalid). */
int64_t pck_peer_buffer_bytes(int64_t slice_bytes, int world);
/* A zeroed device buffer of this process (cudaMalloc; not from a caching allocator, so it can be exported). */
int pck_peer_alloc(int64_t bytes, void** ptr);
int pck_peer_free(void* ptr);
/* The buffer's CUDA IPC handle, PCK_PEER_HANDLE_BYTES bytes, for the other ranks to import. */
int pck_peer_export(const void* ptr, void* handle);
/* Maps another rank's exported buffer into this process (peer access enabled); pck_peer_close unmaps it. */
int pck_peer_import(const void* handle, void** ptr);
int pck_peer_close(void* ptr);
/*
 * The all-gather, one kernel on `stream`: this rank stores its slice into every rank's
 * buffer over NVLink, signals each peer with a system-scope atomic, waits (at most 4 s, then
 * the device timeout bit of pck_device_status and no copy) for every peer's slice, and
 * copies the assembled slices into `gathered`. Every rank makes the same sequence of calls
 * with the same slice size, each after the previous one on its stream, as for an NCCL
 * all-gather; the calls are capturable in a CUDA graph. No multicast. Replaces the north
 * star's NCCL all_gather_into_tensor of y and the verdict bits (no counterpart in the
 * reference, which runs on one GPU).
 */
int pck_peer_all_gather(const pck_peer_gather* gather, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PCK_B200_H */
