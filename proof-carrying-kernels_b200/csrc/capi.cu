// extern "C" entry points of libpck_b200.so (declared in include/pck_b200.h): argument
// validation, launch planning and dispatch. Messages of rejected calls follow the
// reference bindings' wording (src/pck/cuda/csrc/bindings.cpp) so callers can match them.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "member_plan.h"
#include "pck_b200.h"
#include "sampling_plan.h"
#include "tc_plan.h"
#include "bank_batch_plan.h"
#include "stream_plan.h"
#include "verdict_plan.h"

namespace pck {
cudaError_t launch_gemv_naive(const void* W, const void* x, float* y, int64_t m, int64_t n,
                              int threads, int sms, cudaStream_t stream);
cudaError_t status_stream_bf16(unsigned int* value, bool clear);
cudaError_t status_stream_e4m3(unsigned int* value, bool clear);
cudaError_t peer_status(unsigned int* value, bool clear);
cudaError_t launch_bank_build(const void* W, const int8_t* r, float* c, void* a, int64_t n,
                              int block, int num_blocks, int checks, double factor,
                              cudaStream_t stream);
}  // namespace pck

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int cuda_fail(const char* what, cudaError_t err) {
  return fail(PCK_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(err));
}

int ok() {
  g_error.clear();
  return PCK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool power_of_two(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v < 1) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

// One job of a streaming launch, as requested by the caller.
struct Spec {
  const void* W;
  const void* X;
  float* Y;
  int64_t m;
  int64_t n;
  int batch;
  int threads;
  int wfmt;
  bool has_w;
  bool settled;  // PCK_WEIGHTS_SETTLED: weights may be read before the producer wait
  const pck_check_desc* check;
  int w_exp_min;
  int w_exp_max;
};

int validate_check(const pck_check_desc* d) {
  if (!d) return fail(PCK_ERR_ARGUMENT, "check descriptor is NULL");
  if (!d->c || !d->a || !d->r || !d->x || !d->y || !d->partial_cx || !d->partial_s ||
      !d->passed || !d->rho || !d->tau) {
    return fail(PCK_ERR_ARGUMENT, "check descriptor has a NULL pointer");
  }
  if (d->checks < 1 || d->num_blocks < 1 || d->n < 1 || d->block < 1) {
    return fail(PCK_ERR_ARGUMENT, "empty checker");
  }
  if (d->segments < 1 || d->segments > d->n) {
    return fail(PCK_ERR_ARGUMENT, "segments must be in [1, n], got %d", d->segments);
  }
  if (d->batch < 1 || d->batch > pck::kMaxBatch) {
    return fail(PCK_ERR_ARGUMENT, "check batch must be in [1, %d], got %d", pck::kMaxBatch, d->batch);
  }
  if (!(d->coef > 0) || !(d->geps > 0) || !(d->tau_floor > 0)) {
    return fail(PCK_ERR_ARGUMENT, "coef, geps and floor must be positive");
  }
  if (d->flags & ~PCK_CHECK_BANK_SETTLED) return fail(PCK_ERR_ARGUMENT, "unknown check flags 0x%x", d->flags);
  return PCK_OK;
}

constexpr int64_t kPieceTarget = 4 * 1024;  // row piece size the staged path aims for
constexpr int kMaxSlots = 4;                // ring slots per warp
constexpr int64_t kSegmentTarget = 2048;    // columns per checksum-bank segment
// Time per byte of a bank segment (binary64 products and sums) relative to a weight row,
// for the CTA split between the jobs of a launch: bfloat16 rows, and E4M3 rows (twice the
// weights per byte, so the bank costs less against them). Measured: the CTAs of both kinds
// end together.
constexpr double kBankCostBf16 = 2.5;
constexpr double kBankCostE4m3 = 1.8;
constexpr int kMaxVerdictCtas = 8;
// Prior verdicts: a warp's tasks run one after another, each an L2 round trip while the
// launch saturates HBM. A verdict CTA ends about kVerdictBaseUs + kVerdictTaskUs per task
// after the producer wait, the rows about their bytes over the per-format streaming rate
// (bytes per microsecond) after it; a warp takes 4, 2 or 1 tasks, the most that still end
// before the rows.
constexpr double kVerdictBaseUs = 2.5;
constexpr double kVerdictTaskUs = 1.5;
constexpr double kRowBytesPerUsBf16 = 6.0e6;
constexpr double kRowBytesPerUsE4m3 = 5.0e6;

int64_t fill_verdicts(const pck_check_desc* const* descs, int count, const int32_t* fixed_segs,
                      pck::VerdictPlan& plan);
int run_verdicts(const pck_check_desc* const* descs, int count, cudaStream_t stream,
                 const int32_t* fixed_segs);

// Launch shape of a planned streaming launch.
struct StreamShape {
  bool empty = false;  // no job has work (only prior verdicts, if any)
  int wfmt = 0;
  int nv = 8;
  int bg = 1;
  bool tma = false;
  unsigned grid = 0;
  size_t smem = 0;
};

// Plans the streaming kernel for `specs` (validated by the caller) into `plan` (zeroed by the
// caller); `prior` (validated, at most kMaxVerdictJobs) are checks of earlier launches that
// this one decides.
int plan_stream(const std::vector<Spec>& specs, const std::vector<const pck_check_desc*>& prior,
                pck::Plan& plan, StreamShape& shape) {
  if (specs.empty() || specs.size() > static_cast<size_t>(pck::kMaxJobs)) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %zu", pck::kMaxJobs, specs.size());
  }
  int wfmt = -1, threads = -1, batch = -1;
  for (const Spec& s : specs) {
    if (s.has_w) {
      if (wfmt < 0) {
        wfmt = s.wfmt;
        threads = s.threads;
        batch = s.batch;
      } else if (s.wfmt != wfmt || s.threads != threads || s.batch != batch) {
        return fail(PCK_ERR_ARGUMENT, "jobs in one launch must share weight format, threads and batch");
      }
    }
  }
  if (wfmt < 0) {  // checks only: the tree parameters are unused
    wfmt = pck::kWeightsBf16;
    threads = 256;
    batch = 1;
  }
  const int nv = threads / 32;
  const int vec = wfmt == pck::kWeightsBf16 ? 8 : 16;
  const int esize = wfmt == pck::kWeightsBf16 ? 2 : 1;

  // Pass 1: which jobs have work, and whether the staged (bulk-copy) path applies.
  std::vector<const Spec*> live;
  bool tma = true;
  int max_batch = 1;
  for (const Spec& s : specs) {
    const int64_t m = s.check ? static_cast<int64_t>(s.check->num_blocks) * s.check->block : s.m;
    if (m == 0) continue;
    live.push_back(&s);
    const int64_t n = s.check ? s.check->n : s.n;
    const int b = s.check ? s.check->batch : s.batch;
    max_batch = std::max(max_batch, b);
    if (s.has_w && (!aligned16(s.W) || !aligned16(s.X) || n % vec != 0)) tma = false;
    if (s.check) {
      const pck_check_desc* d = s.check;
      if (!aligned16(d->c) || !aligned16(d->a) || !aligned16(d->x) || d->n % 8 != 0) tma = false;
      if (d->batch > pck::kSegBatch) tma = false;
    }
  }
  if (live.empty()) {  // nothing to stream: the prior verdicts alone
    shape.empty = true;
    return PCK_OK;
  }

  // Pass 2: units and bytes of every job (one row per row unit). A checked GEMV becomes two
  // jobs of the launch: its rows, and its bank rows (reduced against the same x). Their
  // partial sums meet in the verdict kernel, so the bank work need not follow the rows of
  // its block; as a job of its own it is spread over CTAs weighted by its cost.
  int64_t x_bytes = 0;
  std::vector<double> bytes;  // cost-weighted, for the CTA split
  int64_t max_row_bytes = 0;
  int nj = 0;
  for (const Spec* sp : live) {
    const Spec& s = *sp;
    if (s.has_w) {
      pck::JobPlan jb{};
      jb.W = s.W;
      jb.X = static_cast<const uint16_t*>(s.X);
      jb.Y = s.Y;
      jb.has_w = 1;
      jb.w_exp_min = s.w_exp_min;
      jb.w_exp_max = s.w_exp_max;
      jb.m = s.m;
      jb.n = s.n;
      jb.batch = s.batch;
      jb.row_bytes = jb.n * esize;
      jb.rows = 1;
      jb.row_units = static_cast<int32_t>(jb.m);
      jb.period_units = 1;
      jb.period_bytes = jb.row_bytes;
      jb.units = jb.m;
      jb.total_bytes = jb.m * jb.row_bytes;
      max_row_bytes = std::max<int64_t>(max_row_bytes, jb.row_bytes);
      x_bytes = std::max<int64_t>(x_bytes, static_cast<int64_t>(jb.batch) * jb.n * 2);
      plan.jobs[nj++] = jb;
      bytes.push_back(static_cast<double>(jb.total_bytes));
    }
    if (s.check) {
      const pck_check_desc* d = s.check;
      pck::JobPlan jb{};
      jb.X = static_cast<const uint16_t*>(d->x);
      jb.has_check = 1;
      jb.m = static_cast<int64_t>(d->num_blocks) * d->block;
      jb.n = d->n;
      jb.batch = d->batch;
      jb.row_bytes = jb.n * esize;
      jb.rows = 1;
      jb.block = d->block;
      jb.num_blocks = d->num_blocks;
      jb.checks = d->checks;
      // Bank rows are cut into segments of about kSegmentTarget columns (at most the
      // scratch's `segments`): the binary64 bound holds for any split, so the split is
      // chosen for the kernel, not taken from the caller.
      jb.seg_alloc = d->segments;
      pck::segment_split(d->n, d->segments, kSegmentTarget, &jb.seg_len, &jb.segs);
      jb.c = d->c;
      jb.a = static_cast<const uint16_t*>(d->a);
      jb.bank_settled = (d->flags & PCK_CHECK_BANK_SETTLED) ? 1 : 0;
      jb.partial_cx = d->partial_cx;
      jb.partial_s = d->partial_s;
      jb.row_units = 0;
      jb.period_units = static_cast<int64_t>(d->checks + 1) * jb.segs;
      jb.period_bytes = (4LL * d->checks + 2) * d->n;
      jb.units = jb.period_units * d->num_blocks;
      jb.total_bytes = jb.period_bytes * d->num_blocks;
      x_bytes = std::max<int64_t>(x_bytes, static_cast<int64_t>(jb.batch) * jb.n * 2);
      plan.jobs[nj++] = jb;
      bytes.push_back(static_cast<double>(jb.total_bytes) *
                      (wfmt == pck::kWeightsBf16 ? kBankCostBf16 : kBankCostE4m3));
    }
  }

  // Columns reduced together; a batch wider than that re-reads each row from its slot, so
  // such rows stay whole in one piece.
  int bg = 1;
  while (bg * 2 <= 8 && bg * 2 <= max_batch && bg * 2 * nv <= 64) bg *= 2;

  // Staged path: a row piece is whole vector iterations (T * 16 bytes) up to kPieceTarget,
  // or the whole row; every warp has `slots` slots of the largest piece.
  x_bytes = (x_bytes + 127) / 128 * 128;
  int64_t row_piece = 512, slot_bytes = 512;
  int slots = 0;
  if (tma) {
    const int64_t viter = static_cast<int64_t>(threads) * 16;
    if (max_row_bytes > 0) {
      if (max_batch > bg || max_row_bytes <= kPieceTarget) {
        row_piece = max_row_bytes;
      } else {
        row_piece = std::max<int64_t>(viter, kPieceTarget / viter * viter);
      }
    } else {
      row_piece = kPieceTarget;  // checks only: bank pieces of the usual size
    }
    slot_bytes = (std::max<int64_t>(row_piece, 512) + 127) / 128 * 128;
    const int64_t room = pck::kSmemCap - x_bytes - 8 * (pck::kConsumerWarps * kMaxSlots + 1) - 64;
    const int64_t fit = room / (pck::kConsumerWarps * slot_bytes);
    slots = static_cast<int>(std::min<int64_t>(kMaxSlots, fit));
    if (slots < 1) tma = false;
  }
  size_t smem = 0;
  if (tma) {
    smem = static_cast<size_t>(x_bytes + pck::kConsumerWarps * slots * slot_bytes +
                               8 * (pck::kConsumerWarps * slots + 1) + 16);
    plan.stages = slots;
    plan.stage_bytes = static_cast<int32_t>(slot_bytes);
    plan.x_bytes = static_cast<int32_t>(x_bytes);
    plan.sum_bytes = static_cast<int32_t>(row_piece);
    bool checked = !prior.empty();
    for (const Spec* sp : live) checked = checked || sp->check != nullptr;
    // Weight pieces before the producer wait only when every job's weights are settled; the
    // bank CTAs take as many only for checks whose bank is settled too (PCK_CHECK_BANK_SETTLED).
    bool settled = true;
    for (const Spec* sp : live) settled = settled && (!sp->has_w || sp->settled);
    plan.pre_slots = !settled ? 0 : checked ? pck::kPreSlotsChecked : pck::kPreSlotsPlain;
  }

  // CTAs: one per SM in total (two without shared-memory staging), split between the jobs
  // in proportion to their bytes, at least one each and never more than their units.
  // Prior verdicts: CTAs of their own past the streaming ones, 4, 2 or 1 tasks per warp by
  // the launch's length (kVerdictBaseUs above).
  int64_t prior_tasks = 0;
  int verdict_ctas = 0;
  if (!prior.empty()) {
    prior_tasks = fill_verdicts(prior.data(), static_cast<int>(prior.size()), nullptr, plan.prior);
    int64_t w_bytes = 0;
    for (int j = 0; j < nj; ++j) w_bytes += plan.jobs[j].has_w ? plan.jobs[j].total_bytes : 0;
    const double rows_us =
        static_cast<double>(w_bytes) / (wfmt == pck::kWeightsBf16 ? kRowBytesPerUsBf16 : kRowBytesPerUsE4m3);
    int per_warp = 1;
    for (int t : {4, 2}) {
      if (kVerdictBaseUs + kVerdictTaskUs * t <= rows_us) {
        per_warp = t;
        break;
      }
    }
    const int64_t per_cta = static_cast<int64_t>(pck::kConsumerWarps) * per_warp;
    verdict_ctas = static_cast<int>(std::min<int64_t>(kMaxVerdictCtas, (prior_tasks + per_cta - 1) / per_cta));
    verdict_ctas = std::max(verdict_ctas, 1);
  }
  const int sms = std::max(1, sm_count() - verdict_ctas);
  int64_t total_units = 0;
  double total_bytes = 0.0;
  for (int j = 0; j < nj; ++j) {
    total_units += plan.jobs[j].units;
    total_bytes += bytes[j];
  }
  const int64_t want = std::min<int64_t>(tma ? sms : 2LL * sms, total_units);
  std::vector<int64_t> cnt(nj);
  int64_t assigned = 0;
  for (int j = 0; j < nj; ++j) {
    const double share = static_cast<double>(want) * bytes[j] / total_bytes;
    cnt[j] = std::min<int64_t>(std::max<int64_t>(1, static_cast<int64_t>(share)), plan.jobs[j].units);
    assigned += cnt[j];
  }
  // Remaining CTAs go, one at a time, to the job whose CTAs carry the most bytes.
  while (assigned < want) {
    int best = -1;
    double load = -1.0;
    for (int j = 0; j < nj; ++j) {
      const double l = bytes[j] / static_cast<double>(cnt[j]);
      if (cnt[j] < plan.jobs[j].units && l > load) {
        best = j;
        load = l;
      }
    }
    if (best < 0) break;
    ++cnt[best];
    ++assigned;
  }
  // Never more CTAs than SMs on the staged path (one resident CTA each, so a dependent
  // launch cannot take an SM that this grid still needs): trim the lightest jobs' extras.
  const int64_t cap = tma ? std::max<int64_t>(sms, nj) : assigned;
  while (assigned > cap) {
    int best = -1;
    double load = 1e300;
    for (int j = 0; j < nj; ++j) {
      const double l = bytes[j] / static_cast<double>(cnt[j] - 1 > 0 ? cnt[j] - 1 : 1);
      if (cnt[j] > 1 && l < load) {
        best = j;
        load = l;
      }
    }
    if (best < 0) break;
    --cnt[best];
    --assigned;
  }
  int64_t begin = 0;
  for (int j = 0; j < nj; ++j) begin += cnt[j];
  if (begin + verdict_ctas > pck::kMaxCtas) {
    return fail(PCK_ERR_ARGUMENT, "streaming grid of %lld CTAs exceeds %d", static_cast<long long>(begin + verdict_ctas),
                pck::kMaxCtas);
  }
  // Bank jobs take the grid's first CTAs. A dependent launch's CTAs start in index order on
  // the SMs the previous launch frees, and a CTA's prologue (its share of the launch
  // parameters, read through the constant cache while HBM is saturated, then its first
  // requests) takes over a microsecond. The CTAs that start first have it done, and their
  // first pieces in flight, before the producer wait returns; the bank CTAs, whose segment
  // sums take longest after the wait, go first.
  int order[pck::kMaxPlanJobs];
  int no = 0;
  for (int j = 0; j < nj; ++j) {
    if (!plan.jobs[j].has_w) order[no++] = j;
  }
  for (int j = 0; j < nj; ++j) {
    if (plan.jobs[j].has_w) order[no++] = j;
  }
  begin = 0;
  for (int oi = 0; oi < nj; ++oi) {
    const int j = order[oi];
    pck::JobPlan& jb = plan.jobs[j];
    jb.cta_begin = static_cast<int32_t>(begin);
    jb.cta_count = static_cast<int32_t>(cnt[j]);
    if (jb.units > INT32_MAX) return fail(PCK_ERR_ARGUMENT, "a job of %lld units is too large", static_cast<long long>(jb.units));
    // Each CTA's unit range, from its share of the job's bytes.
    for (int64_t c = 0; c < cnt[j]; ++c) {
      const int64_t u0 = pck::first_unit_at(jb, c * jb.total_bytes / cnt[j]);
      const int64_t u1 = pck::first_unit_at(jb, (c + 1) * jb.total_bytes / cnt[j]);
      plan.cta_units[begin + c] = make_int2(static_cast<int>(u0), static_cast<int>(u1));
      plan.cta_job[begin + c] = static_cast<uint8_t>(j);
    }
    begin += cnt[j];
  }
  plan.njobs = nj;
  plan.threads = threads;
  plan.verdict_cta_begin = static_cast<int32_t>(begin);
  plan.verdict_ctas = verdict_ctas;
  plan.prior_tasks = prior_tasks;

  if (!tma) bg = 1;
  shape.wfmt = wfmt;
  shape.nv = nv;
  shape.bg = bg;
  shape.tma = tma;
  shape.grid = static_cast<unsigned>(begin + verdict_ctas);
  shape.smem = smem;
  return PCK_OK;
}

// The first weight pieces of the launch planned in `next` (its GEMV CTAs' first row per warp,
// up to two pieces each), as a table in `plan` that the CTAs of `plan`'s launch prefetch into
// L2 as they finish.
void fill_prefetch(pck::Plan& plan, const pck::Plan& next, const StreamShape& ns) {
  plan.next_ctas = 0;
  if (ns.empty || !ns.tma) return;
  int nj = 0;
  int8_t map[pck::kMaxPlanJobs];
  for (int j = 0; j < next.njobs; ++j) {
    map[j] = -1;
    const pck::JobPlan& jb = next.jobs[j];
    if (!jb.has_w || jb.has_check || jb.rows != 1 || nj >= pck::kMaxPrefetchJobs) continue;
    pck::PrefetchJob& pj = plan.next_jobs[nj];
    pj.W = static_cast<const uint8_t*>(jb.W);
    pj.row_bytes = jb.row_bytes;
    pj.bytes = static_cast<int32_t>(std::min<int64_t>(jb.row_bytes, 2LL * next.sum_bytes) / 16 * 16);
    map[j] = static_cast<int8_t>(nj++);
  }
  const int ctas = std::min<int>(next.verdict_cta_begin, pck::kMaxCtas);
  for (int c = 0; c < ctas; ++c) {
    const int j = next.cta_job[c];
    plan.next_job[c] = static_cast<uint8_t>(map[j] < 0 ? 255 : map[j]);
    plan.next_units[c] = next.cta_units[c];
  }
  plan.next_ctas = ctas;
}

// Plans and launches the streaming kernel for `specs`; with `next` (the jobs of the launch
// that follows on the stream, deciding `next_prior`), the CTAs also prefetch that launch's
// first weight pieces into L2 as they finish.
int run_stream(const std::vector<Spec>& specs, cudaStream_t stream,
               const std::vector<const pck_check_desc*>& prior = {}, const std::vector<Spec>* next = nullptr,
               const std::vector<const pck_check_desc*>& next_prior = {}) {
  pck::Plan plan{};
  StreamShape shape;
  if (int rc = plan_stream(specs, prior, plan, shape)) return rc;
  if (shape.empty) {
    return prior.empty() ? ok() : run_verdicts(prior.data(), static_cast<int>(prior.size()), stream, nullptr);
  }
  if (next && !next->empty() && shape.tma) {
    pck::Plan np{};
    StreamShape ns;
    if (plan_stream(*next, next_prior, np, ns) == PCK_OK) fill_prefetch(plan, np, ns);
    g_error.clear();  // a next launch that does not plan only loses its prefetch
  }
  const cudaError_t err = shape.wfmt == pck::kWeightsBf16
                              ? pck::launch_stream_bf16(plan, shape.nv, shape.bg, shape.tma, shape.grid, shape.smem, stream)
                              : pck::launch_stream_e4m3(plan, shape.nv, shape.bg, shape.tma, shape.grid, shape.smem, stream);
  if (err != cudaSuccess) return cuda_fail("streaming kernel", err);
  return ok();
}

// The verdict plan of `count` validated checks (count in [1, kMaxVerdictJobs]); returns its
// number of tasks (one warp each).
int64_t fill_verdicts(const pck_check_desc* const* descs, int count, const int32_t* fixed_segs,
                      pck::VerdictPlan& plan) {
  int64_t tasks = 0;
  for (int i = 0; i < count; ++i) {
    const pck_check_desc* d = descs[i];
    pck::VerdictJob& vj = plan.jobs[i];
    int64_t seg_len = 0;
    if (fixed_segs) {
      vj.segs = fixed_segs[i];
    } else {
      pck::segment_split(d->n, d->segments, kSegmentTarget, &seg_len, &vj.segs);
    }
    vj.y = d->y;
    vj.r = d->r;
    vj.partial_cx = d->partial_cx;
    vj.partial_s = d->partial_s;
    vj.passed = d->passed;
    vj.rho = d->rho;
    vj.tau = d->tau;
    vj.block = d->block;
    vj.num_blocks = d->num_blocks;
    vj.checks = d->checks;
    vj.seg_alloc = d->segments;
    vj.batch = d->batch;
    vj.coef = d->coef;
    vj.geps = d->geps;
    vj.tau_floor = d->tau_floor;
    vj.task_begin = tasks;
    vj.tasks = static_cast<int64_t>(d->batch) * d->checks * d->num_blocks;
    tasks += vj.tasks;
  }
  plan.njobs = count;
  return tasks;
}

// Launches the verdict kernel for `count` validated checks whose partial sums are (or will
// be, earlier on the stream) in their scratch.
int run_verdicts(const pck_check_desc* const* descs, int count, cudaStream_t stream,
                 const int32_t* fixed_segs) {
  if (count < 1 || count > pck::kMaxVerdictJobs) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %d", pck::kMaxVerdictJobs, count);
  }
  pck::VerdictPlan plan{};
  const int64_t tasks = fill_verdicts(descs, count, fixed_segs, plan);
  const cudaError_t err = pck::launch_verdicts(plan, tasks, stream);
  if (err != cudaSuccess) return cuda_fail("verdict kernel", err);
  return ok();
}

// cuTensorMapEncodeTiled from the driver, through the runtime (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  return fn;
}

// A 2-D bfloat16 tensor map over rows x cols (row-major), box 64 columns x box_rows rows,
// 128-byte swizzle, zero fill outside.
bool encode_bf16_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(pck::kTcTileK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A 2-D E4M3 tensor map over rows x cols bytes (row-major), box 64 columns x 128 rows, no
// swizzle (the kernel widens the tile to bfloat16 itself), zero fill outside.
bool encode_e4m3_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols) {
  auto encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(pck::kTcTileK), static_cast<cuuint32_t>(pck::kTcTileM)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A byte range of device memory (NULL or empty: nothing).
struct Range {
  const void* p;
  int64_t bytes;
};

bool overlaps(const Range& a, const Range& b) {
  if (!a.p || !b.p || a.bytes <= 0 || b.bytes <= 0) return false;
  const auto a0 = reinterpret_cast<uintptr_t>(a.p), b0 = reinterpret_cast<uintptr_t>(b.p);
  return a0 < b0 + static_cast<uintptr_t>(b.bytes) && b0 < a0 + static_cast<uintptr_t>(a.bytes);
}

int check_gemv_args(const void* W, const void* x, const float* y, int64_t m, int64_t n,
                    int threads, int min_threads) {
  if (m < 0 || n < 0) return fail(PCK_ERR_ARGUMENT, "expected W of shape (m, n) with m, n >= 0");
  if (threads < min_threads || threads > 1024 || !power_of_two(threads)) {
    return fail(PCK_ERR_ARGUMENT, "threads must be a power of two in [%d, 1024], got %d", min_threads, threads);
  }
  if (m > 0 && n < 1) return fail(PCK_ERR_ARGUMENT, "n must be positive");
  if (m > 0 && (!W || !x || !y)) return fail(PCK_ERR_ARGUMENT, "W, x and y must not be NULL");
  return PCK_OK;
}

}  // namespace

namespace {

// The specs of a validated job array (shared by the pipelined entry points).
int job_specs(const pck_gemv_job* jobs, int count, std::vector<Spec>& specs) {
  if (count < 1 || count > PCK_MAX_JOBS || !jobs) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %d", PCK_MAX_JOBS, count);
  }
  for (int i = 0; i < count; ++i) {
    const pck_gemv_job& jb = jobs[i];
    const int wfmt = jb.weight_format & ~PCK_WEIGHTS_SETTLED;
    if (wfmt != PCK_WEIGHTS_BF16 && wfmt != PCK_WEIGHTS_E4M3) {
      return fail(PCK_ERR_ARGUMENT, "unknown weight format %d", jb.weight_format);
    }
    if (int rc = check_gemv_args(jb.W, jb.X, jb.Y, jb.m, jb.n, jb.threads, 32)) return rc;
    if (jb.batch < 1 || jb.batch > pck::kMaxBatch) {
      return fail(PCK_ERR_ARGUMENT, "batch must be in [1, %d], got %d", pck::kMaxBatch, jb.batch);
    }
    if (jb.check) {
      const pck_check_desc* d = jb.check;
      if (int rc = validate_check(d)) return rc;
      if (d->x != jb.X || d->y != jb.Y || d->n != jb.n || d->batch != jb.batch ||
          static_cast<int64_t>(d->num_blocks) * d->block != jb.m) {
        return fail(PCK_ERR_ARGUMENT, "a fused check must cover the job's own x, y and shape");
      }
    }
    specs.push_back(Spec{jb.W, jb.X, jb.Y, jb.m, jb.n, jb.batch, jb.threads, wfmt, true,
                         (jb.weight_format & PCK_WEIGHTS_SETTLED) != 0, jb.check, jb.w_exp_min, jb.w_exp_max});
  }
  return PCK_OK;
}

// The prior checks of a pipelined call, validated against what the call's jobs write.
int prior_checks(const pck_gemv_job* jobs, int count, const pck_check_desc* prior, int nprior,
                 std::vector<const pck_check_desc*>& before) {
  if (nprior < 0 || nprior > PCK_MAX_JOBS || (nprior > 0 && !prior)) {
    return fail(PCK_ERR_ARGUMENT, "prior checks must number [0, %d], got %d", PCK_MAX_JOBS, nprior);
  }
  for (int i = 0; i < nprior; ++i) {
    const pck_check_desc* d = prior + i;
    if (int rc = validate_check(d)) return rc;
    // The prior checks' inputs must be final and their outputs untouched by this launch.
    const int64_t nb = d->num_blocks, rows = nb * d->block;
    const Range reads_writes[] = {
        {d->y, 4 * d->batch * rows},
        {d->partial_cx, 8 * d->batch * d->checks * nb * d->segments},
        {d->partial_s, 8 * d->batch * nb * d->segments},
        {d->passed, d->batch * d->checks * nb},
        {d->rho, 8 * d->batch * d->checks * nb},
        {d->tau, 8 * d->batch * d->checks * nb},
    };
    for (int j = 0; j < count; ++j) {
      const pck_gemv_job& jb = jobs[j];
      const pck_check_desc* c = jb.check;
      const Range writes[] = {
          {jb.Y, 4 * jb.batch * jb.m},
          {c ? c->partial_cx : nullptr, c ? 8LL * c->batch * c->checks * c->num_blocks * c->segments : 0},
          {c ? c->partial_s : nullptr, c ? 8LL * c->batch * c->num_blocks * c->segments : 0},
      };
      for (const Range& a : reads_writes) {
        for (const Range& b : writes) {
          if (overlaps(a, b)) {
            return fail(PCK_ERR_ARGUMENT, "prior check %d shares memory with what job %d writes", i, j);
          }
        }
      }
    }
    before.push_back(d);
  }
  return PCK_OK;
}

}  // namespace

extern "C" {

const char* pck_last_error(void) { return g_error.c_str(); }

int pck_abi_version(void) { return 6; }

int pck_device_status(unsigned int* status, int clear) {
  if (!status) return fail(PCK_ERR_ARGUMENT, "status must not be NULL");
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return cuda_fail("device synchronize", err);
  unsigned int total = 0;
  for (auto* reader : {pck::status_stream_bf16, pck::status_stream_e4m3, pck::tc_status, pck::peer_status}) {
    unsigned int v = 0;
    err = reader(&v, clear != 0);
    if (err != cudaSuccess) return cuda_fail("status read", err);
    total |= v;
  }
  *status = total;
  return ok();
}

int pck_gemv_naive(const void* W, const void* x, float* y, int64_t m, int64_t n, int threads,
                   void* stream) {
  if (int rc = check_gemv_args(W, x, y, m, n, threads, 1)) return rc;
  if (m == 0) return ok();
  const cudaError_t err = pck::launch_gemv_naive(W, x, y, m, n, threads, sm_count(),
                                                 static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail("gemv kernel", err);
  return ok();
}

int pck_gemv_batched(int weight_format, const void* W, const void* X, float* Y, int64_t m,
                     int64_t n, int64_t batch, int threads, void* stream) {
  if (weight_format != PCK_WEIGHTS_BF16 && weight_format != PCK_WEIGHTS_E4M3) {
    return fail(PCK_ERR_ARGUMENT, "unknown weight format %d", weight_format);
  }
  if (int rc = check_gemv_args(W, X, Y, m, n, threads, 32)) return rc;
  if (batch < 1 || batch > pck::kMaxBatch) {
    return fail(PCK_ERR_ARGUMENT, "batch must be in [1, %d], got %lld", pck::kMaxBatch, static_cast<long long>(batch));
  }
  if (m == 0) return ok();
  std::vector<Spec> specs{{W, X, Y, m, n, static_cast<int>(batch), threads, weight_format, true, false, nullptr, 0, 0}};
  return run_stream(specs, static_cast<cudaStream_t>(stream));
}

int pck_gemv_coalesced(const void* W, const void* x, float* y, int64_t m, int64_t n,
                       int threads, void* stream) {
  return pck_gemv_batched(PCK_WEIGHTS_BF16, W, x, y, m, n, 1, threads, stream);
}

int pck_gemv_fp8(const void* Q, const void* x, float* z, int64_t m, int64_t n, int threads,
                 void* stream) {
  return pck_gemv_batched(PCK_WEIGHTS_E4M3, Q, x, z, m, n, 1, threads, stream);
}

int pck_blocked_check(const pck_check_desc* descs, int count, void* stream) {
  if (count < 1 || count > PCK_MAX_JOBS || !descs) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %d", PCK_MAX_JOBS, count);
  }
  std::vector<Spec> specs;
  for (int i = 0; i < count; ++i) {
    if (int rc = validate_check(descs + i)) return rc;
    specs.push_back(Spec{nullptr, nullptr, nullptr, 0, descs[i].n, descs[i].batch, 256,
                         PCK_WEIGHTS_BF16, false, false, descs + i, 0, 0});
  }
  if (int rc = run_stream(specs, static_cast<cudaStream_t>(stream))) return rc;
  const pck_check_desc* checks[PCK_MAX_JOBS];
  for (int i = 0; i < count; ++i) checks[i] = descs + i;
  return run_verdicts(checks, count, static_cast<cudaStream_t>(stream), nullptr);
}

int pck_gemv_partials(const pck_gemv_job* jobs, int count, void* stream) {
  return pck_gemv_pipelined(jobs, count, nullptr, 0, stream);
}

int pck_gemv_pipelined(const pck_gemv_job* jobs, int count, const pck_check_desc* prior, int nprior,
                       void* stream) {
  return pck_gemv_pipelined_next(jobs, count, prior, nprior, nullptr, 0, stream);
}

int pck_gemv_pipelined_next(const pck_gemv_job* jobs, int count, const pck_check_desc* prior, int nprior,
                            const pck_gemv_job* next, int nnext, void* stream) {
  std::vector<Spec> specs;
  if (int rc = job_specs(jobs, count, specs)) return rc;
  std::vector<const pck_check_desc*> before;
  if (int rc = prior_checks(jobs, count, prior, nprior, before)) return rc;
  if (nnext < 0 || nnext > PCK_MAX_JOBS || (nnext > 0 && !next)) {
    return fail(PCK_ERR_ARGUMENT, "next jobs must number [0, %d], got %d", PCK_MAX_JOBS, nnext);
  }
  std::vector<Spec> next_specs;
  std::vector<const pck_check_desc*> next_prior;  // the next launch decides this call's checks
  if (nnext > 0) {
    if (int rc = job_specs(next, nnext, next_specs)) return rc;
    for (int i = 0; i < count; ++i) {
      if (jobs[i].check && jobs[i].m > 0) next_prior.push_back(jobs[i].check);
    }
  }
  return run_stream(specs, static_cast<cudaStream_t>(stream), before, nnext > 0 ? &next_specs : nullptr, next_prior);
}

int pck_check_verdicts(const pck_check_desc* descs, int count, void* stream) {
  if (count < 1 || count > PCK_MAX_JOBS || !descs) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %d", PCK_MAX_JOBS, count);
  }
  const pck_check_desc* checks[PCK_MAX_JOBS];
  for (int i = 0; i < count; ++i) {
    if (int rc = validate_check(descs + i)) return rc;
    checks[i] = descs + i;
  }
  return run_verdicts(checks, count, static_cast<cudaStream_t>(stream), nullptr);
}

int pck_gemv_checked(const pck_gemv_job* jobs, int count, void* stream) {
  if (int rc = pck_gemv_partials(jobs, count, stream)) return rc;
  const pck_check_desc* checks[PCK_MAX_JOBS];
  int n = 0;
  for (int i = 0; i < count; ++i) {
    if (jobs[i].check && jobs[i].m > 0) checks[n++] = jobs[i].check;
  }
  if (n == 0) return ok();
  return run_verdicts(checks, n, static_cast<cudaStream_t>(stream), nullptr);
}

int pck_bank_build(const void* W, const int8_t* r, float* c, void* a, int64_t m, int64_t n,
                   int block, int checks, double sum_up_factor, void* stream) {
  if (!W || !r || !c || !a) return fail(PCK_ERR_ARGUMENT, "W, r, c and a must not be NULL");
  if (block < 1 || m < 1 || m % block != 0) {
    return fail(PCK_ERR_ARGUMENT, "block=%d must be positive and divide m=%lld", block, static_cast<long long>(m));
  }
  if (checks < 1) return fail(PCK_ERR_ARGUMENT, "checks must be positive, got %d", checks);
  if (n < 1) return fail(PCK_ERR_ARGUMENT, "n must be positive");
  const int64_t nb = m / block;
  if (nb > 65535) return fail(PCK_ERR_UNSUPPORTED, "too many row blocks (%lld > 65535)", static_cast<long long>(nb));
  const cudaError_t err = pck::launch_bank_build(W, r, c, a, n, block, static_cast<int>(nb), checks,
                                                 sum_up_factor, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail("bank kernel", err);
  return ok();
}

int pck_member_check(const void* logits, int logits_dtype, int64_t rows, int64_t vocab,
                     int64_t row_stride, const int64_t* tokens, const int64_t* top_k,
                     const double* top_p, const uint8_t* greedy, double slack, uint8_t* ok_out,
                     int64_t* above, double* mass_above, void* stream) {
  if (logits_dtype != PCK_LOGITS_F32 && logits_dtype != PCK_LOGITS_BF16 && logits_dtype != PCK_LOGITS_F16) {
    return fail(PCK_ERR_ARGUMENT, "unknown logits dtype %d", logits_dtype);
  }
  if (rows < 0 || vocab < 1) return fail(PCK_ERR_ARGUMENT, "expected logits of shape (B, V) with V >= 1");
  if (row_stride < vocab) return fail(PCK_ERR_ARGUMENT, "row stride %lld is below the vocabulary %lld",
                                      static_cast<long long>(row_stride), static_cast<long long>(vocab));
  if (rows > 0x7fffffffLL) return fail(PCK_ERR_UNSUPPORTED, "too many rows (%lld)", static_cast<long long>(rows));
  if (!(slack >= 0)) return fail(PCK_ERR_ARGUMENT, "slack must be non-negative");
  if (rows == 0) return ok();
  if (!logits || !tokens || !ok_out || !above || !mass_above) {
    return fail(PCK_ERR_ARGUMENT, "logits, tokens and the outputs must not be NULL");
  }
  pck::MemberArgs args{};
  args.logits = logits;
  args.rows = rows;
  args.vocab = vocab;
  args.row_stride = row_stride;
  args.dtype = logits_dtype;
  args.tokens = tokens;
  args.top_k = top_k;
  args.top_p = top_p;
  args.greedy = greedy;
  args.slack = slack;
  args.ok = ok_out;
  args.above = above;
  args.mass_above = mass_above;
  const cudaError_t err = pck::launch_member_check(args, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail("membership kernel", err);
  return ok();
}

int pck_sampling_check(const float* logits, const int64_t* selected, const int64_t* lengths, int64_t rows,
                       int64_t vocab, int64_t max_len, int64_t k, int top_p, double p, double temperature,
                       double slack, int64_t segments, uint8_t* passed, float* min_selected,
                       float* max_rejected, double* mass, double* without, void* stream) {
  if (rows < 1 || vocab < 1 || max_len < 1) return fail(PCK_ERR_ARGUMENT, "empty input");
  if (rows > 65535) return fail(PCK_ERR_ARGUMENT, "too many rows");
  if (segments < 1 || segments > vocab) {
    return fail(PCK_ERR_ARGUMENT, "segments must be in [1, V], got %lld", static_cast<long long>(segments));
  }
  if (!(temperature > 0) || !(slack >= 0)) {
    return fail(PCK_ERR_ARGUMENT, "temperature must be positive, slack >= 0");
  }
  if (!logits || !selected || !lengths || !passed || !min_selected || !max_rejected || !mass || !without) {
    return fail(PCK_ERR_ARGUMENT, "pointers must not be NULL");
  }
  // The segments only choose how many CTAs (at most one cluster) share a row.
  const int64_t cluster = std::min<int64_t>({segments, pck::kSamplingMaxCluster, (vocab + 31) / 32});
  int64_t slice = (vocab + cluster - 1) / cluster;
  slice = (slice + 31) / 32 * 32;
  if (pck::sampling_smem_bytes(slice) > pck::kSamplingSmemCap) {
    return fail(PCK_ERR_UNSUPPORTED, "vocabulary of %lld is beyond this build's %d slices of shared memory",
                static_cast<long long>(vocab), pck::kSamplingMaxCluster);
  }
  pck::SamplingArgs args{};
  args.logits = logits;
  args.selected = selected;
  args.lengths = lengths;
  args.rows = rows;
  args.vocab = vocab;
  args.max_len = max_len;
  args.k = k;
  args.slice = slice;
  args.top_p = top_p ? 1 : 0;
  args.p = p;
  args.temperature = temperature;
  args.slack = slack;
  args.passed = passed;
  args.min_selected = min_selected;
  args.max_rejected = max_rejected;
  args.mass = mass;
  args.without = without;
  const cudaError_t err = pck::launch_sampling_check(args, static_cast<int>(cluster), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail("sampling checker", err);
  return ok();
}

int pck_gemv_tc(const pck_gemv_job* jobs, int count, void* stream) {
  if (count < 1 || count > pck::kTcMaxJobs || !jobs) {
    return fail(PCK_ERR_ARGUMENT, "batch size must be in [1, %d], got %d", pck::kTcMaxJobs, count);
  }
  pck::TcPlan plan{};
  const int batch = jobs[0].batch;
  if (batch < 1 || batch > pck::kTcMaxBatch) {
    return fail(PCK_ERR_ARGUMENT, "batch must be in [1, %d], got %d", pck::kTcMaxBatch, batch);
  }
  constexpr int kFlags = PCK_WEIGHTS_SETTLED | PCK_TC_FULL_K;
  const int wfmt = jobs[0].weight_format & ~kFlags;
  if (wfmt != PCK_WEIGHTS_BF16 && wfmt != PCK_WEIGHTS_E4M3) {
    return fail(PCK_ERR_ARGUMENT, "unknown weight format %d", jobs[0].weight_format);
  }
  const bool e4m3 = wfmt == PCK_WEIGHTS_E4M3;
  bool full_k = false, settled = true;
  const int n_pad = (batch + 15) / 16 * 16;
  int tiles = 0, nj = 0;
  const pck_check_desc* descs[pck::kTcMaxJobs] = {};
  for (int i = 0; i < count; ++i) {
    const pck_gemv_job& jb = jobs[i];
    if ((jb.weight_format & ~kFlags) != wfmt) {
      return fail(PCK_ERR_ARGUMENT, "jobs in one launch must share the weight format");
    }
    full_k = full_k || (jb.weight_format & PCK_TC_FULL_K) != 0;
    settled = settled && (jb.weight_format & PCK_WEIGHTS_SETTLED) != 0;
    if (jb.batch != batch) return fail(PCK_ERR_ARGUMENT, "jobs in one launch must share the batch");
    if (int rc = check_gemv_args(jb.W, jb.X, jb.Y, jb.m, jb.n, 256, 1)) return rc;
    if (jb.m == 0) continue;
    if (jb.n % (e4m3 ? 16 : 8) != 0 || !aligned16(jb.W) || !aligned16(jb.X)) {
      return fail(PCK_ERR_UNSUPPORTED, "the tensor-core GEMV needs n a multiple of 8 (16 for E4M3) and 16-byte "
                                       "aligned W and X");
    }
    if (jb.m > (1LL << 31) - pck::kTcTileM || jb.n > (1LL << 31)) return fail(PCK_ERR_UNSUPPORTED, "matrix too large");
    pck::TcJob& tj = plan.jobs[nj];
    const bool maps = (e4m3 ? encode_e4m3_map(&tj.w_map, jb.W, jb.m, jb.n)
                            : encode_bf16_map(&tj.w_map, jb.W, jb.m, jb.n, pck::kTcTileM)) &&
                      encode_bf16_map(&tj.x_map, jb.X, batch, jb.n, n_pad);
    if (!maps) return fail(PCK_ERR_CUDA, "tensor map encoding failed");
    tj.Y = jb.Y;
    tj.m = jb.m;
    tj.n = jb.n;
    if (jb.check) {
      const pck_check_desc* d = jb.check;
      if (!d->c || !d->a || !d->r || !d->partial_cx || !d->partial_s || !d->passed || !d->rho || !d->tau) {
        return fail(PCK_ERR_ARGUMENT, "check descriptor has a NULL pointer");
      }
      if (d->x != jb.X || d->y != jb.Y || d->n != jb.n || d->batch != batch ||
          static_cast<int64_t>(d->num_blocks) * d->block != jb.m) {
        return fail(PCK_ERR_ARGUMENT, "a fused check must cover the job's own x, y and shape");
      }
      if (d->checks < 1) return fail(PCK_ERR_ARGUMENT, "empty checker");
      if (d->segments < 1 || d->segments > d->n) {
        return fail(PCK_ERR_ARGUMENT, "segments must be in [1, n], got %d", d->segments);
      }
      if (!(d->coef > 0) || !(d->geps > 0) || !(d->tau_floor > 0)) {
        return fail(PCK_ERR_ARGUMENT, "coef, geps and floor must be positive");
      }
      descs[nj] = d;
    }
    tj.tile_begin = tiles;
    tj.tiles = static_cast<int32_t>((jb.m + pck::kTcTileM - 1) / pck::kTcTileM);
    tiles += tj.tiles;
    ++nj;
  }
  if (nj == 0) return ok();
  plan.njobs = nj;
  plan.total_tiles = tiles;
  plan.batch = batch;
  plan.n_pad = n_pad;
  plan.weights = e4m3 ? pck::kTcWeightsE4m3 : pck::kTcWeightsBf16;
  plan.settled = settled ? 1 : 0;

  // The form. Persistent: a CTA per SM over contiguous ranges of tiles, in units of two tiles
  // sharing each staged X tile. Split: a cluster of `splits` CTAs per unit of one or two
  // tiles, each CTA a near-equal range of the K blocks, for launches with few tiles. The
  // choice minimises the modelled time of the busiest CTA: its shared-memory fill (W and the
  // X tile of every stage) at a per-SM streaming rate, bounded below by the launch's weight
  // bytes at HBM rate (rates measured on B200: about 52 GB/s per SM, 6.5 TB/s in all).
  const int sms = sm_count();
  int64_t kmin = INT64_MAX, kmax = 0;
  double wtotal = 0.0;
  for (int j = 0; j < nj; ++j) {
    const int64_t kb = (plan.jobs[j].n + pck::kTcTileK - 1) / pck::kTcTileK;
    kmin = std::min(kmin, kb);
    kmax = std::max(kmax, kb);
    wtotal += static_cast<double>(plan.jobs[j].m) * static_cast<double>(plan.jobs[j].n) * (e4m3 ? 1.0 : 2.0);
  }
  const double tile_w = pck::kTcTileM * pck::kTcTileK * (e4m3 ? 1.0 : 2.0);  // W bytes of a tile per stage
  const double x_stage = n_pad * 128.0;
  constexpr double kSmRate = 52e3, kHbmRate = 6.5e6;  // bytes per microsecond
  const double floor_us = wtotal / kHbmRate;
  int splits = 1, unit_tiles = pck::kTcMaxUnitTiles;
  {
    const int64_t per = (tiles + sms - 1) / sms;  // tiles of the busiest persistent CTA
    const double fill = static_cast<double>(kmax) * (per * tile_w + ((per + 1) / 2) * x_stage);
    double best = std::max(fill / kSmRate, floor_us);
    // the split form's partial sums of a unit overlay the stages: 2 tiles fit up to batch 128
    const int max_t = full_k ? 0 : n_pad <= 128 ? 2 : 1;
    for (int t = 1; t <= max_t; ++t) {
      int64_t units = 0;
      for (int j = 0; j < nj; ++j) units += (plan.jobs[j].tiles + t - 1) / t;
      for (int sp = 2; sp <= pck::kTcMaxSplits; ++sp) {
        if (units * sp > sms || kmin < 2LL * sp) break;
        if (units > pck::tc_max_clusters(sp)) continue;  // would not run in one wave
        const double f = static_cast<double>((kmax + sp - 1) / sp) * (t * tile_w + x_stage);
        const double est = std::max(f / kSmRate, floor_us) + 0.05 * sp;  // the cluster sum grows with sp
        if (est < best) {
          best = est;
          splits = sp;
          unit_tiles = t;
        }
      }
    }
  }
  plan.unit_tiles = unit_tiles;
  plan.strided = 0;
  plan.total_units = 0;
  for (int j = 0; j < nj; ++j) {
    plan.jobs[j].unit_begin = plan.total_units;
    plan.jobs[j].units = (plan.jobs[j].tiles + plan.unit_tiles - 1) / plan.unit_tiles;
    plan.total_units += plan.jobs[j].units;
  }

  // Checks whose bank rows the kernel reduces itself: 128-row blocks (one per tile), at most
  // kTcMaxChecks sign draws, 16-byte aligned bank rows, room for one partial sum per tile (per
  // K range in the split form), and batches up to kTcFuseMaxBatch: the binary64 work per stage
  // grows with the batch while a stage's weight bytes do not, and past 128 columns the bank
  // warps fall further behind the weight stream than a separate bank launch costs (measured on
  // the decode layer: at batch 128 fused 0.27 ms against 0.35 ms with the bank launch).
  // Others take the wide-batch bank kernel.
  const int segs_fused = splits;
  int max_checks = 0;
  bool any_c64 = false;
  for (int j = 0; j < nj; ++j) {
    const pck_check_desc* d = descs[j];
    pck::TcJob& tj = plan.jobs[j];
    if (d && batch <= pck::kTcFuseMaxBatch && d->block == pck::kTcTileM && d->checks <= pck::kTcMaxChecks &&
        d->segments >= segs_fused &&
        aligned16(d->c) && aligned16(d->a)) {
      tj.fused = 1;
      tj.c = d->c;
      tj.c64 = d->c64 && aligned16(d->c64) ? d->c64 : nullptr;
      any_c64 = any_c64 || tj.c64 != nullptr;
      tj.a = static_cast<const uint16_t*>(d->a);
      tj.partial_cx = d->partial_cx;
      tj.partial_s = d->partial_s;
      tj.checks = d->checks;
      tj.nb = d->num_blocks;
      tj.seg_alloc = d->segments;
      max_checks = std::max(max_checks, d->checks);
    }
  }
  plan.any_fused = max_checks > 0;
  plan.max_checks = max_checks;

  plan.w_bytes = plan.unit_tiles * pck::kTcTileM * 128;
  plan.x_bytes = n_pad * 128;
  plan.tile_bank_bytes = plan.any_fused ? max_checks * (any_c64 ? 512 : 256) + 128 : 0;
  plan.bank_bytes = (plan.unit_tiles * plan.tile_bank_bytes + 1023) / 1024 * 1024;
  plan.raw_bytes = e4m3 ? plan.unit_tiles * pck::kTcTileM * 64 : 0;
  plan.stage_bytes = (plan.w_bytes + plan.x_bytes + plan.bank_bytes + plan.raw_bytes + 1023) / 1024 * 1024;
  // Beyond the stages: 1024 bytes of alignment slack, the bank warps' binary64 staging and
  // group sums, and the barriers.
  const size_t extra = 1024 + pck::kTcBankSmemBytes + 8 * (3 * 8 + 5) + 16;
  constexpr size_t kSmemCap = 232448;
  plan.stages = static_cast<int32_t>(std::min<size_t>(8, (kSmemCap - extra) / plan.stage_bytes));
  if (plan.stages < 2) return fail(PCK_ERR_UNSUPPORTED, "a batch of %d leaves no room for two stages", batch);
  if (splits > 1 && static_cast<size_t>(plan.stages) * plan.stage_bytes <
                        static_cast<size_t>(plan.unit_tiles) * pck::kTcTileM * n_pad * 4) {
    return fail(PCK_ERR_UNSUPPORTED, "no room for the partial accumulator of a batch of %d", batch);
  }
  plan.acc_stride = (n_pad + 31) / 32 * 32;  // every epilogue read takes 32 columns
  plan.acc_bufs = (splits == 1 && 2 * plan.unit_tiles * plan.acc_stride <= 512) ? 2 : 1;
  int cols = 32;
  while (cols < plan.acc_bufs * plan.unit_tiles * plan.acc_stride) cols *= 2;
  plan.tmem_cols = cols;
  const size_t smem = extra + static_cast<size_t>(plan.stages) * plan.stage_bytes;
  const int grid = splits == 1 ? std::min(plan.strided ? plan.total_units : tiles, sms) : plan.total_units * splits;
  cudaError_t err = pck::launch_tc(plan, splits, grid, smem, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail("tensor-core gemv kernel", err);

  // The checks: the wide-batch bank kernel for the checks the GEMV kernel did not reduce
  // (bank rows x batch columns in binary64), then the block verdicts of all of them.
  const pck_check_desc* checks[pck::kTcMaxJobs];
  int32_t segs[pck::kTcMaxJobs];
  int nc = 0, nbank = 0;
  pck::BankBatchPlan bank{};
  int max_segs = 1;
  for (int j = 0; j < nj; ++j) {
    const pck_check_desc* d = descs[j];
    if (!d) continue;
    if (plan.jobs[j].fused) {
      segs[nc] = segs_fused;
      checks[nc++] = d;
      continue;
    }
    pck::BankBatchJob& bj = bank.jobs[nbank++];
    bj.c = d->c;
    bj.a = static_cast<const uint16_t*>(d->a);
    bj.X = static_cast<const uint16_t*>(d->x);
    bj.partial_cx = d->partial_cx;
    bj.partial_s = d->partial_s;
    bj.n = d->n;
    bj.nb = d->num_blocks;
    bj.checks = d->checks;
    bj.batch = d->batch;
    bj.seg_alloc = d->segments;
    bj.segs = pck::bank_batch_segments(d->n, d->segments, &bj.seg_len);
    bj.tile_begin = bank.total_tiles;
    bj.c_tiles = static_cast<int32_t>((static_cast<int64_t>(d->checks) * d->num_blocks + 31) / 32);  // 32-row tiles
    bj.a_tiles = (d->num_blocks + 31) / 32;
    bank.total_tiles += bj.c_tiles + bj.a_tiles;
    max_segs = std::max(max_segs, bj.segs);
    segs[nc] = bj.segs;
    checks[nc++] = d;
  }
  if (nc == 0) return ok();
  if (nbank > 0) {
    bank.njobs = nbank;
    err = pck::launch_bank_batch(bank, (batch + 31) / 32, max_segs, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail("bank kernel", err);
  }
  return run_verdicts(checks, nc, static_cast<cudaStream_t>(stream), segs);
}

}  // extern "C"

namespace pck {

// Records `message` as the last error of this thread (for entry points in other files).
int report_error(int code, const char* message) { return fail(code, "%s", message); }

}  // namespace pck
