// Fused residual-add + RMSNorm (and its plain / quantised-output forms) for
// sm_100a: launch plans, argument validation, kernel dispatch and the C-ABI
// entry points.  The kernels and their arithmetic are in rms_norm_kernels.cuh.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "rms_norm_kernels.cuh"
#include "runtime.cuh"

namespace hprn {

// ---------------------------------------------------------------------------
// Launch plans.

enum Kind { kWarpRows = 0, kCtaRows = 1, kClusterRows = 2, kTwoPass = 3, kTma = 4 };

struct Plan {
  Kind kind = kWarpRows;
  int vec = 32;          // bytes per vector
  int vpt = 1;           // vectors per thread
  int tpr = 32;          // threads per CTA working on one row slice
  int cluster = 1;       // CTAs per row
  int rows_per_cta = 1;  // warp kind: rows per CTA; tma kind: ring depth (rows in flight per CTA)
  // Launch knobs (-1: the default for the plan, see default_knobs):
  int prefetch = -1;  // L2 prefetch before the programmatic-launch wait: 0 none,
                      // 1 the grid's first wave of CTAs, 2 every CTA, 3 the first
                      // wave, and every CTA also the row one wave ahead
  int early = -1;     // where dependents are triggered: 0 after the last store, 1 after
                      // the row reduction, 2 once the loads are issued (-1: by grid size)
  bool knobs_given = false;  // set by parse_plan when the string carried both knobs
  bool knobs_only = false;   // override "default:pf<p>:et<e>": the default plan, these knobs
  bool trig_loads = false;   // launch: the kernel instance that triggers once its loads are issued
};

enum Prefetch { kPrefetchNone = 0, kPrefetchFirstWave = 1, kPrefetchAll = 2, kPrefetchAhead = 3 };

// Kernel family of one call: residual or not, and the output form.
struct Variant {
  bool res = true;
  int out = kOutSame;
  // The in-place fused form (the reference's operation) carries the full set
  // of compiled plans; the other forms a reduced set.
  bool full() const { return res && out == kOutSame; }
};

const char* kind_name(Kind k) {
  switch (k) {
    case kWarpRows: return "warp";
    case kCtaRows: return "cta";
    case kClusterRows: return "cluster";
    case kTma: return "tma";
    default: return "twopass";
  }
}

std::string plan_string(const Plan& p) {
  char buf[96];
  int n = snprintf(buf, sizeof(buf), "%s:vec%d:vpt%d:tpr%d:cluster%d:rpc%d", kind_name(p.kind),
                   p.vec, p.vpt, p.tpr, p.cluster, p.rows_per_cta);
  // Knobs given explicitly (a plan override) are echoed; defaults are implied.
  if (p.knobs_given && n > 0 && n < static_cast<int>(sizeof(buf)))
    snprintf(buf + n, sizeof(buf) - n, ":pf%d:et%d", p.prefetch, p.early);
  return buf;
}

// VPT values compiled for each kind and variant (must match the dispatch
// tables below).
bool vpt_supported(Kind k, int vec, int vpt, const Variant& v) {
  if (k == kTma)
    return (vec == 16 || vec == 32) && v.out == kOutSame && (vpt == 1 || vpt == 2 || vpt == 4 || vpt == 8);
  if (!v.full()) {
    switch (k) {
      case kWarpRows: return vpt == 1 || vpt == 2 || vpt == 4;
      case kCtaRows: return vpt == 1 || vpt == 2 || vpt == 4;
      case kClusterRows: return vpt == 1 || vpt == 2 || vpt == 4;
      default: return v.out == kOutSame;
    }
  }
  switch (k) {
    case kWarpRows: return vpt >= 1 && vpt <= 4;
    case kCtaRows:
    case kClusterRows:
      if (vec == 32) return vpt == 1 || vpt == 2 || vpt == 3 || vpt == 4 || vpt == 6 || vpt == 8;
      // Eight 4-byte vectors per thread in a cluster CTA is not compiled:
      // ptxas gives that one instance a 4-byte spill (at 48 registers).
      if (vec == 4 && k == kClusterRows) return vpt == 1 || vpt == 2 || vpt == 4;
      return vpt == 1 || vpt == 2 || vpt == 4 || vpt == 8;
    default: return true;
  }
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Vectors per cluster CTA: the row split evenly, rounded up to whole groups
// (8 vectors, a multiple of every group size) for per-group fp8 output so a
// group never straddles two CTAs.
int slice_vecs_of(int nvec, int cluster, int out) {
  const int slice = (nvec + cluster - 1) / cluster;
  return out == kOutFp8Group && cluster > 1 ? (slice + 7) / 8 * 8 : slice;
}

// Launch-plan heuristic, fitted to a cold-L2 sweep of every compiled plan on
// B200 (batch 4096 bf16, hidden 1024..32768; the kernel timed as back-to-back
// CUDA-graph launches over rotating buffers).  What won everywhere:
//   * one CTA per row with as many threads as the row has 32-byte vectors
//     (one vector per thread): the most warps per SM, so the most loads in
//     flight, and the shortest serial chain per thread;
//   * rows of at most 16 vectors: one vector per lane, several rows per
//     warp; rows of 17..64 vectors: one warp per row, eight rows per CTA;
//   * rows of 1025..2048 vectors: two vectors per thread (four below ~1440
//     vectors, where 1024-thread CTAs would leave SMs a CTA short);
//   * thread-block clusters only once a row no longer fits one CTA: splitting
//     rows that do fit cost 5-15% (cluster scheduling and the cluster barrier).
// The extended forms (plain rows, quantised outputs) hold more live values per
// vector in their epilogues, or half the bytes per vector in flight (no
// residual), and the same sweep run per form (tune.py --variant) favours more
// vectors per thread in smaller CTAs as rows grow.  Vectors per thread for a
// one-CTA row of nvec vectors, or 0 for the warp-per-row kernel:
int extended_vpt(int nvec, bool residual, int out) {
  // Fused NVFP4: one vector per thread up to 768 vectors, then two, but four
  // at 1025-1280 vectors: there two vectors per thread need 544-640 threads
  // at 60 registers (one CTA per SM) and four need at most 320 at 94 (two
  // per SM); 4096 x 17408 / 20480: 72.8 / 85.0 vs 86.8 / 94.0 us.  Past 1280
  // both fit one CTA per SM and two vectors win (101.8 vs 107.4 us at
  // 22528).  -1: the fused 16-bit rule.
  if (residual)
    return out == kOutNvfp4 ? (nvec <= 768 ? 1 : (nvec > 1024 && nvec <= 1280 ? 4 : 2)) : -1;
  if (nvec <= 64) return 0;
  switch (out) {
    case kOutSame: return nvec <= 128 ? 0 : (nvec <= 256 ? 1 : 2);
    case kOutFp8Static: return nvec <= 128 ? 0 : (nvec <= 1024 ? 2 : 4);
    // fp8 with per-row or per-group scales: two vectors per thread up to 512
    // (the dynamic form then holds its products across the reduction; 4096 x
    // 6144-8192: 15.6 / 19.1 vs 16.8 / 20.2 us at four), four past it.
    case kOutFp8Dynamic:
    case kOutFp8Group: return nvec <= 128 ? 1 : (nvec <= 512 ? 2 : 4);
    // NVFP4: at 4096 x 32768, one 512-thread CTA at four vectors per thread
    // takes 62.8 us (83 us for a 4-CTA cluster).
    default: return nvec <= 128 ? 1 : (nvec <= 256 ? 2 : 4);
  }
}

// Every plan default_plan returns is compiled for the variant it is returned
// for; two passes (rows past 8 * 2048 vectors) exist for 16-bit outputs only.
Plan default_plan(int nvec, int vec, bool residual, int out, int64_t rows) {
  Plan p;
  p.vec = vec;
  if (residual && out == kOutSame && vec == 32 && rows <= 512 && nvec > 32 && nvec <= 128) {
    // Decode-sized batches of fused rows of 33..128 32-byte vectors (hidden
    // 528..2048): the GPU is not full, so what counts is one row's latency,
    // and one CTA per row with one 16-byte vector per thread (twice the
    // threads of 32-byte vectors) is the fastest plan at every batch of 1-512
    // rows (warm, back-to-back launches: 1 x 1024 in 1.15 against 1.60 us for
    // a warp per row, 512 x 1024 in 1.78 against 2.10).  From 1024 rows the
    // warp and CTA rules below win again.
    p.kind = kCtaRows;
    p.vec = 16;
    p.vpt = 1;
    p.tpr = round_up(2 * nvec, 32);
    return p;
  }
  const int ext = nvec <= 2048 ? extended_vpt(nvec, residual, out) : -1;
  if (nvec <= 64 || ext == 0) {
    p.kind = kWarpRows;
    if (nvec <= 16) {
      // Short rows (hidden <= 256 at 32-byte vectors, e.g. per-head norms):
      // one vector per lane, 32 / lanes rows per warp, 256-thread CTAs.  At
      // 131072 rows x hidden 64-256: 3.2-4.3x one warp per row, as fast as
      // torch's copy of the same bytes.
      int lanes = 1;
      while (lanes < nvec) lanes <<= 1;
      // Per-group fp8: eight lanes (a group's lanes must share one row), one
      // or two vectors each (hidden 256: 25.3 vs 28.1 us with sixteen lanes).
      if (out == kOutFp8Group) lanes = 8;
      p.vpt = (nvec + lanes - 1) / lanes;
      p.tpr = lanes;
      p.rows_per_cta = 256 / lanes;
      return p;
    }
    p.vpt = nvec <= 64 ? (nvec + 31) / 32 : 4;
    p.tpr = 32;
    // Four warp-rows (128 threads) per CTA: best or within 2% for every form
    // at hidden 1024-2048 with the programmatic-launch trigger at each
    // kernel's end (fused 6.52-6.55 vs 6.70-6.79 us with eight at 4096 x
    // 1024); plain 16-bit rows of <= 64 vectors keep eight (4.36 vs 4.50 us).
    p.rows_per_cta = (!residual && out == kOutSame && nvec <= 64) ? 8 : 4;
    return p;
  }
  if (residual && out == kOutSame && nvec <= 96) {
    // Fused rows of 65..96 vectors (hidden 1040-1536): one warp per row at
    // three vectors per lane beat one CTA per row (9.00 vs 9.38 us at 4096 x
    // 1536).
    p.kind = kWarpRows;
    p.vpt = 3;
    p.tpr = 32;
    p.rows_per_cta = 4;
    return p;
  }
  if (ext > 0) {
    p.kind = kCtaRows;
    p.vpt = ext;
    p.tpr = round_up((nvec + p.vpt - 1) / p.vpt, 32);
    return p;
  }
  if (nvec <= 1024) {
    p.kind = kCtaRows;
    p.vpt = 1;
    p.tpr = round_up(nvec, 32);
    return p;
  }
  if (nvec <= 2048) {
    p.kind = kCtaRows;
    p.vpt = nvec <= 1440 ? 4 : 2;
    p.tpr = round_up((nvec + p.vpt - 1) / p.vpt, 32);
    return p;
  }
  // Longer rows of the fused 16-bit form: always eight CTAs per row, one
  // vector per thread up to 512 vectors per CTA, else two (hidden 40960-131072
  // at batch 4096: 0.88-0.95 of the copy peak, against 0.76-0.86 for the
  // smallest cluster that fits).
  const int64_t elems = static_cast<int64_t>(nvec) * (vec / 2);
  const bool many_rows = rows >= 1024 && vec >= 16;
  if (residual && out == kOutSame && nvec > 4096 && (elems > 98304 || (elems > 65536 && many_rows))) {
    // Fused 16-bit rows past 65536 elements (past 98304 for small batches):
    // two passes, the second re-reading the row's residual from L2, beat
    // every register-resident cluster plan, reaching 1.00-1.03 of the copy
    // peak at hidden 81920-262144 x 4096 rows (1.15-1.38x the clustered
    // kernel).  Up to 98304 elements with enough rows to fill the GPU, one
    // 512-thread CTA per row; else an eight-CTA cluster per row, 128 threads
    // per CTA up to 262144 elements and 256 past it (64-1024 rows x hidden
    // 512K-1M).  At 64 rows x 81920 the register-resident cluster stays 13%
    // faster, hence the larger threshold for small batches.
    p.kind = kTwoPass;
    p.vpt = 4;
    if (elems <= 98304 && many_rows) {
      p.cluster = 1;
      p.tpr = 512;
    } else {
      p.cluster = 8;
      p.tpr = elems <= 262144 ? 128 : 256;
    }
    return p;
  }
  if (residual && out == kOutSame && nvec <= 8 * 2048) {
    const int slice = (nvec + 7) / 8;
    p.kind = kClusterRows;
    p.cluster = 8;
    p.vpt = slice <= 512 ? 1 : 2;
    p.tpr = round_up((slice + p.vpt - 1) / p.vpt, 32);
    return p;
  }
  // Other forms, re-tuned per form at hidden 40960-131072 (batch 4096): fused
  // rows with quantised outputs take eight CTAs at two vectors per thread;
  // plain rows four vectors per thread over four CTAs, or eight from 4096
  // vectors (1.1-1.6x the smallest cluster that fits, within 3% of each
  // shape's best plan).
  if (nvec <= 8 * 2048) {
    p.kind = kClusterRows;
    p.vpt = residual ? 2 : 4;
    p.cluster = residual ? 8 : (nvec < 4096 ? 4 : 8);
    const int slice = slice_vecs_of(nvec, p.cluster, out);
    p.tpr = round_up((slice + p.vpt - 1) / p.vpt, 32);
    return p;
  }
  // Past 8 * 2048 vectors: two passes, each row split over an eight-CTA
  // cluster of 256-thread CTAs (rows 64-1024 x hidden 512K-1M: 10-23% faster
  // than one 512-thread CTA per row, whose 102 registers held one CTA per SM).
  p.kind = kTwoPass;
  p.vpt = 4;
  p.tpr = 256;
  p.cluster = 8;
  return p;
}

// Fills the launch knobs a plan leaves at -1 (default_plan's plans, and
// overrides without ":pf..:et.."), from cold-L2 timings of the combinations
// (tune.py --knobs: one process per combination, three runs each) at batch
// 4096 x hidden 1024-32768 for every output form, and at 64 rows x hidden
// 4096-1M (cluster and two-pass kernels):
//   * triggering dependents after the row reduction is as fast or faster
//     than after the last store everywhere (4096 x 1024: fused 6.07 vs 6.12
//     us, plain NVFP4 3.75 vs 4.14, fused per-group fp8 6.29 vs 6.80; 64 x
//     262144: 24.8 vs 25.4), and triggering once the loads are issued is
//     faster still for grids of more than one wave (fused 4096 x 2048 / 4096
//     / 8192: 10.40 / 19.82 / 39.16 us against 11.18 / 21.22 / 40.56) but
//     slower for single-wave grids (128 x 4096 warm: 1.77 vs 1.61), so the
//     trigger point is left to the launch (-1), which picks by grid size;
//   * the L2 prefetch of the first wave's rows, with every CTA also
//     prefetching the row of the CTA one wave after it, is the fastest mode
//     for the fused forms and plain 16-bit rows of every length (fused 4096 x
//     4096 / 16384 / 32768: 20.78 / 79.15 / 156.4 us, against 21.15 / 80.2 /
//     158.6 with every CTA prefetching only its own row; plain 4096 x 4096:
//     10.66 vs 11.62), and for the plain quantised forms from 1024 vectors
//     per CTA (512 for per-row fp8);
//   * shorter plain quantised rows (their CTAs issue-bound and short-lived)
//     and the two-pass kernel do better prefetching only their own rows: in
//     every CTA while one CTA prefetches less than 64 KB (plain static fp8 at
//     4096 x 4096: 9.74 vs 10.20 with the row ahead), in the first wave past
//     that (and from 64 KB for the fused form).
void default_knobs(Plan* p, const Variant& var) {
  // The TMA-staged kernel stages rows itself and triggers at its end; CTA
  // kernels of the issue-bound plain quantised forms are built without the
  // knobs (cta_has_knobs).
  if (p->kind == kTma || ((p->kind == kCtaRows || p->kind == kClusterRows) &&
                          !cta_has_knobs(var.res, var.out, p->vpt))) {
    p->prefetch = kPrefetchNone;
    p->early = 0;
    return;
  }
  if (p->prefetch < 0) {
    // Vectors of one row a CTA holds, and the bytes its own prefetch covers.
    const int slice = p->tpr * p->vpt;
    const int threads = p->kind == kWarpRows ? p->rows_per_cta * p->tpr : p->tpr;
    const int vpt = p->kind == kTwoPass ? kTwoPassUnroll : p->vpt;  // two passes: its first chunk
    const int64_t bytes = static_cast<int64_t>(threads) * vpt * p->vec * (var.res ? 2 : 1);
    const bool plain_quant = !var.res && var.out != kOutSame;
    if (p->kind != kTwoPass &&
        (!plain_quant || slice >= (var.out == kOutFp8Dynamic ? 512 : 1024))) {
      p->prefetch = kPrefetchAhead;
    } else {
      const bool big = bytes > 65536 || (bytes == 65536 && var.full());
      p->prefetch = big ? kPrefetchFirstWave : kPrefetchAll;
    }
  }
}

bool parse_plan(const std::string& s, Plan* p);

// Test hook of the TMA-staged kernel (hprn_test_stall_bulk_copy): the row of
// each later call whose staged copy is made to stall (-1: none), and the
// per-row wait limit in nanoseconds.
std::atomic<int64_t> g_stall_row{-1};
std::atomic<uint64_t> g_stall_wait_ns{kWaitLimitNs};

// Optional plan override for benchmarking and tuning: hprn_set_plan_override,
// or the HP_RMS_NORM_PLAN environment variable (read at the first call).
// Parsed once when set; calls read it under a mutex only while one is set.
std::mutex g_override_mu;
std::atomic<bool> g_override_set{false};
Plan g_override_plan;
std::once_flag g_override_env_once;

void set_override(const Plan* p) {
  std::lock_guard<std::mutex> lock(g_override_mu);
  if (p) g_override_plan = *p;
  g_override_set.store(p != nullptr, std::memory_order_release);
}

bool override_plan(Plan* out) {
  std::call_once(g_override_env_once, [] {
    const char* env = getenv("HP_RMS_NORM_PLAN");
    Plan p;
    if (env && *env && parse_plan(env, &p)) set_override(&p);
  });
  if (!g_override_set.load(std::memory_order_acquire)) return false;
  std::lock_guard<std::mutex> lock(g_override_mu);
  if (!g_override_set.load(std::memory_order_relaxed)) return false;
  *out = g_override_plan;
  return true;
}

bool parse_plan(const std::string& s, Plan* p) {
  if (s.rfind("default:", 0) == 0) {
    int pf = -1, et = -1, end = 0;
    if (sscanf(s.c_str(), "default:pf%d:et%d%n", &pf, &et, &end) != 2 ||
        static_cast<size_t>(end) != s.size() || pf < 0 || pf > 3 || et < 0 || et > 2)
      return false;
    p->prefetch = pf;
    p->early = et;
    p->knobs_given = p->knobs_only = true;
    return true;
  }
  char kind[16] = {0};
  int vec, vpt, tpr, cluster, rpc, pf = -1, et = -1, end = 0;
  const int got = sscanf(s.c_str(), "%15[a-z]:vec%d:vpt%d:tpr%d:cluster%d:rpc%d%n:pf%d:et%d%n",
                         kind, &vec, &vpt, &tpr, &cluster, &rpc, &end, &pf, &et, &end);
  // Six fields, optionally followed by both knobs (":pf<0..3>:et<0..2>"), and nothing else.
  if ((got != 6 && got != 8) || static_cast<size_t>(end) != s.size()) return false;
  if (got == 8 && (pf < 0 || pf > 3 || et < 0 || et > 2)) return false;
  p->prefetch = got == 8 ? pf : -1;
  p->early = got == 8 ? et : -1;
  p->knobs_given = got == 8;
  std::string k(kind);
  if (k == "warp") p->kind = kWarpRows;
  else if (k == "cta") p->kind = kCtaRows;
  else if (k == "cluster") p->kind = kClusterRows;
  else if (k == "twopass") p->kind = kTwoPass;
  else if (k == "tma") p->kind = kTma;
  else return false;
  p->vec = vec;
  p->vpt = vpt;
  p->tpr = tpr;
  p->cluster = cluster;
  p->rows_per_cta = rpc;
  return true;
}

// Checks that `p` covers a row of `nvec` vectors within hardware limits.
bool plan_valid(const Plan& p, int nvec, int max_vec, const Variant& var, std::string* why) {
  if (p.vec > max_vec || (p.vec != 32 && p.vec != 16 && p.vec != 8 && p.vec != 4 && p.vec != 2)) {
    *why = "vector width not allowed by alignment / hidden size";
    return false;
  }
  if (!vpt_supported(p.kind, p.vec, p.vpt, var)) {
    *why = "vectors-per-thread value (or kernel kind) not compiled for this variant";
    return false;
  }
  switch (p.kind) {
    case kWarpRows: {
      // tpr = lanes per row (a power of two); rows_per_cta rows of tpr lanes
      // fill whole warps of a CTA of at most 256 threads.
      const bool pow2 = p.tpr >= 1 && p.tpr <= 32 && (p.tpr & (p.tpr - 1)) == 0;
      const int threads = p.rows_per_cta * p.tpr;
      if (!pow2 || p.rows_per_cta < 1 || threads % 32 || threads > 256 || p.vpt * p.tpr < nvec ||
          (var.out == kOutFp8Group && p.tpr < 8)) {
        *why = "warp plan needs tpr (lanes per row) a power of two <= 32 (>= 8 for per-group "
               "fp8), rpc * tpr a multiple of 32 up to 256, and vpt * tpr >= vectors per row";
        return false;
      }
      return true;
    }
    case kCtaRows:
    case kClusterRows: {
      const int c = p.kind == kCtaRows ? 1 : p.cluster;
      if (p.kind == kCtaRows && p.cluster != 1) {
        *why = "cta plan needs cluster 1";
        return false;
      }
      if (c < 1 || c > 8 || p.tpr < 32 || p.tpr > cta_max_threads(p.vpt) || p.tpr % 32) {
        *why = "cluster must be 1..8 and tpr a multiple of 32 within the kernel's launch bound";
        return false;
      }
      const int slice = slice_vecs_of(nvec, c, var.out);
      if (static_cast<int64_t>(p.tpr) * p.vpt < slice) {
        *why = "tpr * vpt does not cover the row slice";
        return false;
      }
      return true;
    }
    case kTma:
      if (p.cluster != 1 || p.tpr < 32 || p.tpr > cta_max_threads(p.vpt * p.vec / 16) || p.tpr % 32 ||
          static_cast<int64_t>(p.tpr) * p.vpt < nvec || p.rows_per_cta < 1 ||
          p.rows_per_cta > kTmaMaxStages) {
        *why = "tma plan needs cluster 1, tpr a multiple of 32 within the launch bound covering "
               "the row, and 1..16 stages (rpc)";
        return false;
      }
      return true;
    default:
      if (p.tpr < 32 || p.tpr > kTwoPassThreads || p.tpr % 32 ||
          (p.cluster != 1 && p.cluster != 2 && p.cluster != 4 && p.cluster != 8)) {
        *why = "twopass tpr must be a multiple of 32 in [32, 512] and cluster 1, 2, 4 or 8";
        return false;
      }
      return true;
  }
}

// ---------------------------------------------------------------------------
// Dispatch: (dtype, variant, vec, kind, vpt) -> kernel function pointer.

using KernelFn = void (*)(RmsArgs);

// The instance that triggers its dependents once its loads are issued (tl),
// or the one whose trigger point is the runtime knob.
template <typename T, int VEC, int VPT, bool RES, int OUT>
KernelFn warp_fn(bool tl) {
  return tl ? rms_norm_warp_rows<T, VEC, VPT, RES, OUT, true>
            : rms_norm_warp_rows<T, VEC, VPT, RES, OUT, false>;
}

template <typename T, int VEC, int VPT, bool CL, bool RES, int OUT>
KernelFn cta_fn(bool tl) {
  if constexpr (!cta_has_knobs(RES, OUT, VPT)) {
    return rms_norm_cta_rows<T, VEC, VPT, CL, RES, OUT, false>;
  } else {
    return tl ? rms_norm_cta_rows<T, VEC, VPT, CL, RES, OUT, true>
              : rms_norm_cta_rows<T, VEC, VPT, CL, RES, OUT, false>;
  }
}

template <typename T, int VEC, bool RES, int OUT>
KernelFn pick_warp(int vpt, bool tl) {
  if constexpr (RES && OUT == kOutSame) {
    if (vpt == 3) return warp_fn<T, VEC, 3, RES, OUT>(tl);
  }
  switch (vpt) {
    case 1: return warp_fn<T, VEC, 1, RES, OUT>(tl);
    case 2: return warp_fn<T, VEC, 2, RES, OUT>(tl);
    case 4: return warp_fn<T, VEC, 4, RES, OUT>(tl);
  }
  return nullptr;
}

template <typename T, int VEC, bool CL, bool RES, int OUT>
KernelFn pick_cta(int vpt, bool tl) {
  if constexpr (RES && OUT == kOutSame) {
    if constexpr (VEC == 32) {
      switch (vpt) {
        case 3: return cta_fn<T, VEC, 3, CL, RES, OUT>(tl);
        case 6: return cta_fn<T, VEC, 6, CL, RES, OUT>(tl);
      }
    }
    if constexpr (!(CL && VEC == 4)) {
      if (vpt == 8) return cta_fn<T, VEC, 8, CL, RES, OUT>(tl);
    }
  }
  switch (vpt) {
    case 1: return cta_fn<T, VEC, 1, CL, RES, OUT>(tl);
    case 2: return cta_fn<T, VEC, 2, CL, RES, OUT>(tl);
    case 4: return cta_fn<T, VEC, 4, CL, RES, OUT>(tl);
  }
  return nullptr;
}

template <typename T, int VEC, bool RES>
KernelFn pick_tma(int vpt) {
  switch (vpt) {
    case 1: return rms_norm_tma_rows<T, VEC, 1, RES>;
    case 2: return rms_norm_tma_rows<T, VEC, 2, RES>;
    case 4: return rms_norm_tma_rows<T, VEC, 4, RES>;
    case 8: return rms_norm_tma_rows<T, VEC, 8, RES>;
  }
  return nullptr;
}

template <typename T, int VEC, bool RES, int OUT>
KernelFn pick_kind(const Plan& p) {
  switch (p.kind) {
    case kTma:
      if constexpr ((VEC == 16 || VEC == 32) && OUT == kOutSame) return pick_tma<T, VEC, RES>(p.vpt);
      return nullptr;
    case kWarpRows: return pick_warp<T, VEC, RES, OUT>(p.vpt, p.trig_loads);
    case kCtaRows: return pick_cta<T, VEC, false, RES, OUT>(p.vpt, p.trig_loads);
    case kClusterRows: return pick_cta<T, VEC, true, RES, OUT>(p.vpt, p.trig_loads);
    default:
      if constexpr (OUT == kOutSame)
        return p.cluster > 1 ? rms_norm_two_pass<T, VEC, RES, true> : rms_norm_two_pass<T, VEC, RES, false>;
      return nullptr;
  }
}

template <typename T, bool RES, int OUT>
KernelFn pick_vec(const Plan& p) {
  if constexpr (OUT == kOutNvfp4 || OUT == kOutFp8Group) {
    return p.vec == 32 ? pick_kind<T, 32, RES, OUT>(p) : nullptr;
  } else if constexpr (OUT == kOutSame) {
    switch (p.vec) {
      case 32: return pick_kind<T, 32, RES, OUT>(p);
      case 16: return pick_kind<T, 16, RES, OUT>(p);
      case 8: return pick_kind<T, 8, RES, OUT>(p);
      case 4: return pick_kind<T, 4, RES, OUT>(p);
      default: return pick_kind<T, 2, RES, OUT>(p);
    }
  } else {
    switch (p.vec) {
      case 32: return pick_kind<T, 32, RES, OUT>(p);
      case 16: return pick_kind<T, 16, RES, OUT>(p);
      case 8: return pick_kind<T, 8, RES, OUT>(p);
      default: return nullptr;  // fp8 output needs >= 4 elements per vector
    }
  }
}

template <typename T>
KernelFn pick_variant(const Plan& p, const Variant& v) {
  if (v.res) {
    switch (v.out) {
      case kOutSame: return pick_vec<T, true, kOutSame>(p);
      case kOutFp8Static: return pick_vec<T, true, kOutFp8Static>(p);
      case kOutNvfp4: return pick_vec<T, true, kOutNvfp4>(p);
      case kOutFp8Group: return pick_vec<T, true, kOutFp8Group>(p);
      default: return pick_vec<T, true, kOutFp8Dynamic>(p);
    }
  }
  switch (v.out) {
    case kOutSame: return pick_vec<T, false, kOutSame>(p);
    case kOutFp8Static: return pick_vec<T, false, kOutFp8Static>(p);
    case kOutNvfp4: return pick_vec<T, false, kOutNvfp4>(p);
    case kOutFp8Group: return pick_vec<T, false, kOutFp8Group>(p);
    default: return pick_vec<T, false, kOutFp8Dynamic>(p);
  }
}

KernelFn pick_kernel(int dtype, const Plan& p, const Variant& v) {
  return dtype == HPRN_DTYPE_BF16 ? pick_variant<__nv_bfloat16>(p, v)
                                  : pick_variant<__half>(p, v);
}

// Max CTAs per launch in grid.x (2^31 - 1), kept a multiple of 8 for clusters.
constexpr int64_t kMaxGridX = 2147483640LL;

struct Problem {
  void* out;
  const void* x;
  const void* w;
  void* r;  // null: plain RMSNorm
  int64_t rows, hidden, os, xs, rs;
  double eps;
  int dtype;
  int out_form;
  const float* scale;
  float* row_scales;  // per-row fp8 scales, or the per-group scales
  uint8_t* block_scales;
  int64_t gs_row = 0, gs_group = 0;  // per-group scale strides (floats)
  int group_size = 0;
  int scale_pow2 = 0;
};

int out_elem_bytes(const Problem& q) { return q.out_form == kOutSame ? 2 : 1; }

bool is_fp8(const Problem& q) {
  return q.out_form == kOutFp8Static || q.out_form == kOutFp8Dynamic || q.out_form == kOutFp8Group;
}


// [first, last) byte range of `rows` rows of `hidden` elements at `stride`.
struct Span {
  const char* b;
  const char* e;
};

Span span_of(const void* p, int64_t rows, int64_t hidden, int64_t stride, int elem) {
  const char* b = static_cast<const char*>(p);
  return {b, b + elem * ((rows - 1) * stride + hidden)};
}

bool overlap(const Span& a, const Span& b) { return a.b < b.e && b.b < a.e; }

// Two strided 16-bit row sets that overlap as ranges can still share no
// element when their rows interleave (same stride, offset between rows).
bool rows_interleave(const void* p, const void* q, int64_t stride_p, int64_t stride_q,
                     int64_t hidden) {
  const char* a = static_cast<const char*>(p);
  const char* b = static_cast<const char*>(q);
  if (stride_p != stride_q || (b - a) % 2) return false;
  const int64_t d = (b - a) / 2;
  const int64_t m = ((d % stride_p) + stride_p) % stride_p;
  return m >= hidden && stride_p - m >= hidden;
}

int validate(const Problem& q) {
  if (q.dtype != HPRN_DTYPE_BF16 && q.dtype != HPRN_DTYPE_FP16)
    return fail(HPRN_ERR_UNSUPPORTED_DTYPE, "dtype must be kFloat16 or kBFloat16");
  if (q.out_form != kOutSame && q.out_form != kOutFp8Static && q.out_form != kOutFp8Dynamic &&
      q.out_form != kOutNvfp4 && q.out_form != kOutFp8Group)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "unknown output form");
  if (q.rows < 0) return fail(HPRN_ERR_INVALID_ARGUMENT, "rows must be >= 0");
  if (q.hidden < 1 || q.hidden > (static_cast<int64_t>(1) << 30))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "hidden_dim must be in [1, 2^30]");
  if (q.rows == 0) return HPRN_OK;
  if (!q.x || !q.w || !q.out) return fail(HPRN_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (q.out_form == kOutFp8Static && !q.scale)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "static fp8 output needs a scale");
  if (q.out_form == kOutFp8Dynamic && !q.row_scales)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "dynamic fp8 output needs a row_scales buffer");
  if (q.out_form == kOutNvfp4 && (!q.scale || !q.block_scales))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "NVFP4 output needs a global scale and a block_scales buffer");
  if (q.out_form == kOutFp8Group) {
    if (!q.row_scales)
      return fail(HPRN_ERR_INVALID_ARGUMENT, "per-group fp8 output needs a scales buffer");
    if (q.group_size != 32 && q.group_size != 64 && q.group_size != 128)
      return fail(HPRN_ERR_INVALID_ARGUMENT, "group_size must be 32, 64 or 128");
    if (q.hidden % q.group_size)
      return fail(HPRN_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of group_size");
    if (q.gs_row < 0 || q.gs_group < 0 || (q.rows > 1 && q.gs_row == 0) ||
        (q.hidden > q.group_size && q.gs_group == 0))
      return fail(HPRN_ERR_INVALID_ARGUMENT,
                  "scale strides must be positive (one scale slot per row and group)");
  }
  if (q.out_form == kOutNvfp4 && (q.hidden % 16 || (q.rows > 1 && q.os % 16)))
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "NVFP4 output needs hidden_dim % 16 == 0 and an output row stride that is a "
                "multiple of 16 elements");
  if (!aligned(q.x, 2) || !aligned(q.w, 2) || (q.r && !aligned(q.r, 2)) ||
      (q.out_form == kOutSame && !aligned(q.out, 2)))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "tensor pointers must be 2-byte aligned");
  if (q.rows > 1 && (q.xs < q.hidden || q.os < q.hidden || (q.r && q.rs < q.hidden)))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "row strides must be >= hidden_dim");
  const Span xs = span_of(q.x, q.rows, q.hidden, q.xs, 2);
  const Span ws = span_of(q.w, 1, q.hidden, q.hidden, 2);
  const Span os = q.out_form == kOutNvfp4
                      ? span_of(q.out, q.rows, q.hidden / 2, q.os / 2, 1)
                      : span_of(q.out, q.rows, q.hidden, q.os, out_elem_bytes(q));
  // input and residual must not share any element.
  if (q.r) {
    const Span rs = span_of(q.r, q.rows, q.hidden, q.rs, 2);
    if (overlap(xs, rs) && !rows_interleave(q.x, q.r, q.xs, q.rs, q.hidden))
      return fail(HPRN_ERR_INVALID_ARGUMENT, "input and residual must not overlap");
    if (overlap(os, rs) && !(q.out_form == kOutSame && rows_interleave(q.out, q.r, q.os, q.rs, q.hidden)))
      return fail(HPRN_ERR_INVALID_ARGUMENT, "output and residual must not overlap");
    if (overlap(ws, rs)) return fail(HPRN_ERR_INVALID_ARGUMENT, "weight must not overlap input or residual");
  }
  // The output is either exactly the input (16-bit, same strides: in place) or disjoint from it.
  const bool in_place = q.out_form == kOutSame && q.out == q.x && (q.os == q.xs || q.rows == 1);
  if (!in_place && overlap(os, xs) &&
      !(q.out_form == kOutSame && rows_interleave(q.out, q.x, q.os, q.xs, q.hidden)))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "output must be the input itself or not overlap it");
  // The weight is read through the non-coherent cache: nothing this call writes may alias it.
  if (overlap(ws, os))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "weight must not overlap input or residual");
  return HPRN_OK;
}

// Largest vector width every pointer, stride and the hidden size allow.
int choose_vec(const Problem& q) {
  if (q.out_form == kOutFp8Group) {
    const bool ok = q.hidden % 16 == 0 && aligned(q.x, 32) && aligned(q.w, 32) &&
                    (!q.r || aligned(q.r, 32)) && aligned(q.out, 16) &&
                    (q.rows <= 1 || ((q.xs * 2) % 32 == 0 && (!q.r || (q.rs * 2) % 32 == 0) &&
                                     q.os % 16 == 0));
    return ok ? 32 : 0;
  }
  if (q.out_form == kOutNvfp4) {
    const bool ok = q.hidden % 16 == 0 && aligned(q.x, 32) && aligned(q.w, 32) &&
                    (!q.r || aligned(q.r, 32)) && aligned(q.out, 8) &&
                    (q.rows <= 1 || ((q.xs * 2) % 32 == 0 && (!q.r || (q.rs * 2) % 32 == 0) &&
                                     (q.os / 2) % 8 == 0));
    return ok ? 32 : 0;
  }
  const bool fp8 = q.out_form != kOutSame;
  for (int vec : {32, 16, 8, 4}) {
    const int epv = vec / 2;
    if (q.hidden % epv) continue;
    if (!aligned(q.x, vec) || !aligned(q.w, vec) || (q.r && !aligned(q.r, vec))) continue;
    const int out_vec = fp8 ? vec / 2 : vec;
    if (!aligned(q.out, out_vec)) continue;
    if (q.rows > 1 && (((q.xs * 2) % vec) || (q.r && (q.rs * 2) % vec) ||
                       ((q.os * (fp8 ? 1 : 2)) % out_vec)))
      continue;
    return vec;
  }
  return 2;
}

int make_plan(const Problem& q, const Variant& var, Plan* plan, RmsArgs* args) {
  const int max_vec = choose_vec(q);
  if (q.out_form == kOutNvfp4 && max_vec != 32)
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "NVFP4 output needs 32-byte aligned input/weight/residual rows and 8-byte aligned "
                "output rows");
  if (q.out_form == kOutFp8Group && max_vec != 32)
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "per-group fp8 output needs 32-byte aligned input/weight/residual rows and "
                "16-byte aligned output rows");
  if (is_fp8(q) && max_vec < 8)
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "fp8 output needs hidden_dim % 4 == 0 and 8-byte aligned input/weight/residual "
                "rows and 4-byte aligned output rows");
  const int nvec = static_cast<int>(q.hidden / (max_vec / 2));
  Plan p = default_plan(nvec, max_vec, var.res, var.out, q.rows);
  if (p.kind == kTwoPass && q.out_form != kOutSame)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "rows longer than 16384 vectors are supported with a "
                                           "16-bit output only");
  Plan o;
  const bool overridden = override_plan(&o);
  if (overridden && o.knobs_only) {
    p.prefetch = o.prefetch;
    p.early = o.early;
    p.knobs_given = true;
  } else if (overridden) {
    std::string why;
    if (o.vec > max_vec || q.hidden % (o.vec / 2) != 0)
      return fail(HPRN_ERR_INVALID_ARGUMENT, "plan override vector width not allowed here");
    const int onvec = static_cast<int>(q.hidden / (o.vec / 2));
    if (!plan_valid(o, onvec, max_vec, var, &why))
      return fail(HPRN_ERR_INVALID_ARGUMENT, "plan override rejected: " + why);
    p = o;
  }
  default_knobs(&p, var);
  const int epv = p.vec / 2;
  RmsArgs a;
  a.x = static_cast<const uint16_t*>(q.x);
  a.w = static_cast<const uint16_t*>(q.w);
  a.r = static_cast<uint16_t*>(q.r);
  a.out = q.out;
  a.scale = q.scale;
  a.row_scales = q.row_scales;
  a.block_scales = q.block_scales;
  a.rows = q.rows;
  a.x_stride = q.xs;
  a.r_stride = q.rs;
  a.out_stride = q.os;
  a.nvec = static_cast<int>(q.hidden / epv);
  a.slice_vecs = slice_vecs_of(a.nvec, p.cluster, var.out);
  a.rows_per_cta = p.rows_per_cta;
  a.eps = static_cast<float>(q.eps);
  a.inv_hidden = 1.0f / static_cast<float>(q.hidden);
  a.gs_row = q.gs_row;
  a.gs_group = q.gs_group;
  a.group_vecs = q.out_form == kOutFp8Group ? q.group_size / epv : 1;
  a.scale_pow2 = q.scale_pow2 != 0;
  a.lanes_per_row = p.kind == kWarpRows ? p.tpr : 32;
  a.stall_row = g_stall_row.load(std::memory_order_relaxed);
  a.wait_limit_ns = g_stall_wait_ns.load(std::memory_order_relaxed);
  a.prefetch_ctas = 0;  // set per launch
  a.prefetch_ahead_rows = 0;
  a.early_trigger = p.early;
  *plan = p;
  *args = a;
  return HPRN_OK;
}

// Resident CTAs per SM of a TMA-staged kernel at `threads` threads and `smem`
// bytes of ring, cached per (device, kernel, threads, smem); 0 on error.
int tma_ctas_per_sm(const DeviceInfo* dev, KernelFn fn, int threads, int smem) {
  struct Entry {
    int device;
    KernelFn fn;
    int threads, smem, ctas;
  };
  static std::mutex mu;
  static Entry cache[128];
  static int used = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].device == dev->device && cache[i].fn == fn && cache[i].threads == threads &&
        cache[i].smem == smem)
      return cache[i].ctas;
  const int max_dyn = static_cast<int>(dev->smem_per_block_optin) - kTmaStaticSmemReserve;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn) != cudaSuccess)
    return 0;
  int ctas = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, fn, threads, smem) != cudaSuccess) return 0;
  if (used < 128) cache[used++] = Entry{dev->device, fn, threads, smem, ctas};
  return ctas;
}

// One persistent launch of the TMA-staged kernel: as many CTAs as are
// resident at once (or one per row when there are fewer rows).
int launch_tma(const Plan& p, const RmsArgs& a, KernelFn fn, const DeviceInfo* dev,
               cudaStream_t stream, unsigned flags) {
  const int64_t stage_bytes = static_cast<int64_t>(a.r ? 2 : 1) * a.nvec * p.vec;
  const int64_t smem = stage_bytes * p.rows_per_cta;
  if (smem > static_cast<int64_t>(dev->smem_per_block_optin) - kTmaStaticSmemReserve)
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "tma plan " + plan_string(p) + " needs more shared memory than one CTA has");
  const int per_sm = tma_ctas_per_sm(dev, fn, p.tpr, static_cast<int>(smem));
  if (per_sm < 1) {
    cudaGetLastError();
    return fail(HPRN_ERR_INVALID_ARGUMENT, "tma plan " + plan_string(p) + " fits no SM");
  }
  const int64_t resident = static_cast<int64_t>(per_sm) * dev->sm_count;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(static_cast<unsigned>(a.rows < resident ? a.rows : resident), 1, 1);
  cfg.blockDim = dim3(p.tpr, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (flags & HPRN_LAUNCH_PDL) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, fn, a);
  if (e != cudaSuccess)
    return fail(HPRN_ERR_CUDA, std::string("rms_norm launch failed (") + plan_string(p) +
                                   "): " + cudaGetErrorString(e));
  return HPRN_OK;
}

int launch(const Plan& p, RmsArgs a, int dtype, const Variant& var, const DeviceInfo* dev,
           cudaStream_t stream, unsigned flags) {
  KernelFn fn = pick_kernel(dtype, p, var);
  if (!fn) return fail(HPRN_ERR_INVALID_ARGUMENT, "no kernel for plan " + plan_string(p));
  if (p.kind == kTma) return launch_tma(p, a, fn, dev, stream, flags);
  // The instance that triggers once its loads are issued (warp, CTA and
  // cluster kinds; the two-pass kernel has none and triggers after its
  // reduction instead).
  Plan pt = p;
  pt.trig_loads = p.kind != kTwoPass;
  KernelFn fn_tl = pt.trig_loads ? pick_kernel(dtype, pt, var) : fn;
  // Rows handled per CTA-group in grid.x; split very tall problems into launches.
  const int64_t rows_per_unit = p.kind == kWarpRows ? p.rows_per_cta : 1;  // rows per CTA
  const bool clustered = p.kind == kClusterRows || (p.kind == kTwoPass && p.cluster > 1);
  const int64_t ctas_per_unit = clustered ? p.cluster : 1;
  const int64_t max_rows = (kMaxGridX / ctas_per_unit) * rows_per_unit;
  const int threads = p.kind == kWarpRows ? p.rows_per_cta * p.tpr : p.tpr;
  const bool need_wave =
      p.prefetch == kPrefetchFirstWave || p.prefetch == kPrefetchAhead || p.early < 0;
  const int64_t wave = need_wave ? first_wave_ctas(dev, reinterpret_cast<const void*>(fn), threads)
                                 : 0;
  a.prefetch_ctas = p.prefetch == kPrefetchAll ? INT64_MAX : wave;
  // The row the CTA one wave later handles: a wave of CTAs covers wave /
  // ctas_per_unit row units of rows_per_unit rows.
  a.prefetch_ahead_rows =
      p.prefetch == kPrefetchAhead ? wave / ctas_per_unit * rows_per_unit : 0;

  int64_t done = 0;
  while (done < a.rows) {
    RmsArgs c = a;
    const int64_t n = a.rows - done < max_rows ? a.rows - done : max_rows;
    c.x = a.x + done * a.x_stride;
    if (a.r) c.r = a.r + done * a.r_stride;
    const int64_t out_elems = done * a.out_stride;
    c.out = static_cast<char*>(a.out) + (var.out == kOutSame    ? out_elems * 2
                                         : var.out == kOutNvfp4 ? out_elems / 2
                                                                : out_elems);
    if (a.row_scales) c.row_scales = a.row_scales + done * (var.out == kOutFp8Group ? a.gs_row : 1);
    if (a.block_scales) c.block_scales = a.block_scales + done * a.nvec;
    c.rows = n;
    const int64_t units = (n + rows_per_unit - 1) / rows_per_unit;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(static_cast<unsigned>(units * ctas_per_unit), 1, 1);
    // Trigger point by default: once the loads are issued when the grid has
    // more than one wave (the last wave's trigger then lets the next grid's
    // CTAs start and prefetch while this grid's last CTAs finish), after the
    // row reduction when it fits one wave (an earlier trigger there only
    // parks the next grid's CTAs on the SMs: decode batches ran up to 10%
    // slower with it).
    c.early_trigger = p.early >= 0 ? p.early : (units * ctas_per_unit > wave ? 2 : 1);
    KernelFn f = c.early_trigger == 2 ? fn_tl : fn;
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 0;
    if (clustered) {
      attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
      attr[cfg.numAttrs].val.clusterDim.x = p.cluster;
      attr[cfg.numAttrs].val.clusterDim.y = 1;
      attr[cfg.numAttrs].val.clusterDim.z = 1;
      ++cfg.numAttrs;
    }
    if (flags & HPRN_LAUNCH_PDL) {
      attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
      ++cfg.numAttrs;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, f, c);
    if (e != cudaSuccess)
      return fail(HPRN_ERR_CUDA, std::string("rms_norm launch failed (") + plan_string(p) +
                                     "): " + cudaGetErrorString(e));
    done += n;
  }
  return HPRN_OK;
}

int run(const Problem& q, void* stream, unsigned flags) {
  if (flags & ~static_cast<unsigned>(HPRN_LAUNCH_PDL))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "unknown launch flags");
  int st = validate(q);
  if (st != HPRN_OK) return st;
  if (q.rows == 0) return ok();
  const DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != HPRN_OK) return st;
  const Variant var{q.r != nullptr, q.out_form};
  Plan p;
  RmsArgs a;
  if ((st = make_plan(q, var, &p, &a)) != HPRN_OK) return st;
  if ((st = launch(p, a, q.dtype, var, dev, static_cast<cudaStream_t>(stream), flags)) != HPRN_OK)
    return st;
  return ok();
}

}  // namespace hprn

extern "C" {

int hprn_rms_norm(void* input, const void* weight, void* residual, int64_t rows, int64_t hidden,
                  int64_t input_row_stride, int64_t residual_row_stride, double eps, int dtype,
                  void* stream) {
  return hprn_rms_norm_ex(input, weight, residual, rows, hidden, input_row_stride,
                          residual_row_stride, eps, dtype, stream, HPRN_LAUNCH_DEFAULT);
}

int hprn_rms_norm_ex(void* input, const void* weight, void* residual, int64_t rows,
                     int64_t hidden, int64_t input_row_stride, int64_t residual_row_stride,
                     double eps, int dtype, void* stream, unsigned flags) {
  using namespace hprn;
  if (!residual && rows > 0)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "null tensor pointer (residual)");
  Problem q{input, input, weight, residual, rows, hidden, input_row_stride, input_row_stride,
            residual_row_stride, eps, dtype, kOutSame, nullptr, nullptr, nullptr};
  return run(q, stream, flags);
}

int hprn_rms_norm_out(void* out, const void* input, const void* weight, void* residual,
                      int64_t rows, int64_t hidden, int64_t out_row_stride,
                      int64_t input_row_stride, int64_t residual_row_stride, double eps,
                      int dtype, int out_form, const float* scale, float* row_scales,
                      void* stream, unsigned flags) {
  using namespace hprn;
  if (out_form == HPRN_OUT_NVFP4)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "NVFP4 output goes through hprn_rms_norm_nvfp4");
  if (out_form == HPRN_OUT_FP8_E4M3_GROUP)
    return fail(HPRN_ERR_INVALID_ARGUMENT,
                "per-group fp8 output goes through hprn_rms_norm_fp8_group");
  Problem q{out, input, weight, residual, rows, hidden, out_row_stride, input_row_stride,
            residual_row_stride, eps, dtype, out_form, scale, row_scales, nullptr};
  return run(q, stream, flags);
}

int hprn_rms_norm_nvfp4(void* out, uint8_t* block_scales, const void* input, const void* weight,
                        void* residual, int64_t rows, int64_t hidden, int64_t out_row_stride,
                        int64_t input_row_stride, int64_t residual_row_stride, double eps,
                        int dtype, const float* global_scale, void* stream, unsigned flags) {
  using namespace hprn;
  Problem q{out, input, weight, residual, rows, hidden, out_row_stride, input_row_stride,
            residual_row_stride, eps, dtype, kOutNvfp4, global_scale, nullptr, block_scales};
  return run(q, stream, flags);
}

int hprn_rms_norm_fp8_group(void* out, float* scales, int64_t scale_row_stride,
                            int64_t scale_group_stride, const void* input, const void* weight,
                            void* residual, int64_t rows, int64_t hidden, int64_t out_row_stride,
                            int64_t input_row_stride, int64_t residual_row_stride, double eps,
                            int dtype, int group_size, int scale_pow2, void* stream,
                            unsigned flags) {
  using namespace hprn;
  Problem q{out, input, weight, residual, rows, hidden, out_row_stride, input_row_stride,
            residual_row_stride, eps, dtype, kOutFp8Group, nullptr, scales, nullptr,
            scale_row_stride, scale_group_stride, group_size, scale_pow2};
  return run(q, stream, flags);
}

int hprn_rms_norm_plan(int64_t rows, int64_t hidden, int dtype, const void* input,
                       const void* residual, int64_t input_row_stride,
                       int64_t residual_row_stride, char* plan, int plan_len) {
  using namespace hprn;
  if (!plan || plan_len < 1) return fail(HPRN_ERR_INVALID_ARGUMENT, "plan buffer required");
  if (dtype != HPRN_DTYPE_BF16 && dtype != HPRN_DTYPE_FP16)
    return fail(HPRN_ERR_UNSUPPORTED_DTYPE, "dtype must be kFloat16 or kBFloat16");
  if (hidden < 1 || hidden > (static_cast<int64_t>(1) << 30))
    return fail(HPRN_ERR_INVALID_ARGUMENT, "hidden_dim must be in [1, 2^30]");
  // In-place fused form; the weight's alignment is assumed to match the input's.
  void* x = const_cast<void*>(input);
  Problem q{x, input, input, const_cast<void*>(residual), rows < 1 ? 1 : rows, hidden,
            input_row_stride, input_row_stride, residual_row_stride, 1e-6, dtype, kOutSame,
            nullptr, nullptr, nullptr};
  Plan p;
  RmsArgs a;
  const int st = make_plan(q, Variant{true, kOutSame}, &p, &a);
  if (st != HPRN_OK) return st;
  snprintf(plan, plan_len, "%s", plan_string(p).c_str());
  return ok();
}

int hprn_wait_timeouts(unsigned int* count, int reset) {
  using namespace hprn;
  if (!count) return fail(HPRN_ERR_INVALID_ARGUMENT, "count pointer required");
  const DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != HPRN_OK) return st;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v));
  if (e == cudaSuccess && reset && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero));
  }
  if (e != cudaSuccess)
    return fail(HPRN_ERR_CUDA, std::string("reading the wait-timeout count: ") + cudaGetErrorString(e));
  *count = v;
  return ok();
}

int hprn_test_stall_bulk_copy(int64_t row, uint64_t wait_limit_ns) {
  using namespace hprn;
  if (wait_limit_ns > kWaitLimitNs)
    return fail(HPRN_ERR_INVALID_ARGUMENT, "wait_limit_ns must be at most one second");
  g_stall_wait_ns.store(wait_limit_ns ? wait_limit_ns : kWaitLimitNs, std::memory_order_relaxed);
  g_stall_row.store(row < 0 ? -1 : row, std::memory_order_relaxed);
  return ok();
}

int hprn_set_plan_override(const char* plan) {
  using namespace hprn;
  Plan unused;
  override_plan(&unused);  // read the environment first, so this call wins over it
  if (!plan || !*plan) {
    set_override(nullptr);
    return ok();
  }
  Plan p;
  if (!parse_plan(plan, &p)) return fail(HPRN_ERR_INVALID_ARGUMENT, "unparsable plan override");
  set_override(&p);
  return ok();
}

}  // extern "C"
