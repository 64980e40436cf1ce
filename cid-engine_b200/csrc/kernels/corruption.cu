// Training-corruption kernels (fwerkor/cid-engine v1.1.0 semantics):
//  * masked diffusion (csrc/ops.cpp:394-444): one CTA per row (256 or 512
//    threads, eight or four tokens' loads in flight per thread), mask =
//    u < ratio, empty-row fallback on argmin(u); the two metrics come from
//    the exact integer count of masked tokens and a fixed-order double sum
//    of the ratios, so they are bit-identical run to run (the reference CUDA
//    kernel adds them with float atomics): eagerly a second one-block kernel
//    sums per-row counts kept in a caller-provided workspace; inside a CUDA
//    graph the row that finishes last computes them, in one kernel;
//  * thought corruption (csrc/ops.cpp:258-290): one CTA per slot row, alpha
//    computed once per row, every arithmetic step rounded to the storage
//    dtype as ATen does;
//  * display corruption (csrc/ops.cpp:292-391): one CTA of 256 to 1024
//    threads per row, two tokens' loads in flight per thread (four past
//    2048 tokens).
#include <climits>
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kT = 256;

// ---------------------------------------------------------------------------
// masked diffusion
// ---------------------------------------------------------------------------

struct MaskedParams {
  const int64_t* clean;
  const float* ratio_random;
  const float* mask_random;
  int64_t batch, tokens, mask_id;
  float span;  // float32(max - min)
  float lo;    // float32(min)
  int64_t* corrupted;
  uint8_t* masked;
  float* ratio;
  float* metrics;
  int64_t* counts;  // workspace: per-row masked count (two-kernel form)
  // One-kernel form: a zeroed accumulator, (rows done << 40) + masked
  // tokens, that the row finishing last reads back and clears.
  unsigned long long* slot;
};

constexpr int kSlotShift = 40;
constexpr int64_t kSlotMaxRows = (int64_t{1} << (64 - kSlotShift)) - 1;
constexpr int64_t kSlotMaxTokens = int64_t{1} << kSlotShift;

// NaN-first argmin order of ATen min(1).
__device__ __forceinline__ bool min_better(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;
  if (vn) return i < bi;
  return v < bv || (v == bv && i < bi);
}

// ratio = float32(float32(r * span) + lo) (ops.cpp:424-425)
__device__ __forceinline__ float row_ratio(const MaskedParams& p, int64_t row) {
  return __fadd_rn(__fmul_rn(p.ratio_random[row], p.span), p.lo);
}

constexpr int kMetricThreads = 256;  // the ratio sum's order: 256 strided partial sums

// The batch's ratio sum in the metrics kernel's order: thread t of the first
// kMetricThreads adds rows t, t + 256, ... in double, the warps reduce by
// shuffles, warp 0..7 sums are added in order.  `rq` is this thread's
// partial sum; the caller provides s_r[8].  Returns the sum in thread 0.
__device__ __forceinline__ double ratio_sum_tail(double rq, double* s_r) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) rq += __shfl_down_sync(0xffffffffu, rq, d);
  if (threadIdx.x < kMetricThreads && (threadIdx.x & 31) == 0) s_r[threadIdx.x >> 5] = rq;
  __syncthreads();
  double tr = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kMetricThreads / 32; ++w) tr += s_r[w];
  return tr;
}

__device__ __forceinline__ void write_masked_metrics(float* metrics, int64_t masked_total,
                                                     double ratio_sum, int64_t batch,
                                                     int64_t tokens) {
  metrics[0] = static_cast<float>(static_cast<double>(masked_total) /
                                  static_cast<double>(batch * tokens));
  metrics[1] = static_cast<float>(ratio_sum / static_cast<double>(batch));
}

// One CTA of kBT threads per row.  Each thread issues the loads of U tokens
// (kBT apart: every load instruction is coalesced) before it writes any
// output, so a row costs one or two memory round trips, not one per token a
// thread handles.
//
// kOne: the whole op in one kernel.  Each CTA adds (1 << 40) + its row's
// masked count to p.slot with one atomic; the CTA whose add completes the
// batch has every row's count in the value it reads back, so no other data
// crosses CTAs and no fence is needed.  It writes both metrics and clears
// the slot for the next launch.  Batches of up to 256 rows: every CTA loads
// the batch's ratio inputs beside its row and reduces them with its count,
// so the last CTA only adds eight partial sums; larger batches: the last CTA
// sums them after its add.
template <int kBT, int U, bool kOne>
__global__ void __launch_bounds__(kBT) masked_diffusion_kernel(MaskedParams p) {
  static_assert(kBT >= kMetricThreads, "the ratio sum needs 256 threads");
  pdl_wait();
  pdl_trigger();
  constexpr int kW = kBT / 32;
  __shared__ int64_t s_cnt[kW];
  __shared__ float s_min[kW];
  __shared__ int64_t s_idx[kW];
  __shared__ double s_r[kMetricThreads / 32];
  __shared__ unsigned long long s_old;
  const int64_t row = blockIdx.x;
  const int64_t base = row * p.tokens;
  const float r = row_ratio(p, row);
  const bool early_ratios = kOne && p.batch <= kMetricThreads;
  double rq = 0.0;
  if (early_ratios && threadIdx.x < p.batch) rq = static_cast<double>(row_ratio(p, threadIdx.x));
  int64_t cnt = 0;
  float bv = __int_as_float(0x7f800000);  // +inf
  int64_t bi = LLONG_MAX;
  for (int64_t t0 = threadIdx.x; t0 < p.tokens; t0 += int64_t{kBT} * U) {
    float u[U];
    int64_t id[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t t = t0 + int64_t{j} * kBT;
      u[j] = t < p.tokens ? p.mask_random[base + t] : 0.0f;
      id[j] = t < p.tokens ? p.clean[base + t] : 0;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t t = t0 + int64_t{j} * kBT;
      if (t >= p.tokens) break;
      const bool m = u[j] < r;  // ops.cpp:426
      p.masked[base + t] = m;
      p.corrupted[base + t] = m ? p.mask_id : id[j];
      cnt += m;
      if (bi == LLONG_MAX || min_better(u[j], t, bv, bi)) {
        bv = u[j];
        bi = t;
      }
    }
  }
  // block reductions (count; NaN-first argmin)
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    cnt += __shfl_down_sync(0xffffffffu, cnt, d);
    const float ov = __shfl_down_sync(0xffffffffu, bv, d);
    const int64_t oi = __shfl_down_sync(0xffffffffu, bi, d);
    if (oi != LLONG_MAX && (bi == LLONG_MAX || min_better(ov, oi, bv, bi))) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_cnt[warp] = cnt;
    s_min[warp] = bv;
    s_idx[warp] = bi;
  }
  if (early_ratios) {  // uniform over the CTA
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) rq += __shfl_down_sync(0xffffffffu, rq, d);
    if (threadIdx.x < kMetricThreads && (threadIdx.x & 31) == 0) s_r[warp] = rq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t total = 0;
    float mv = s_min[0];
    int64_t mi = s_idx[0];
    for (int w = 0; w < kW; ++w) {
      total += s_cnt[w];
      if (s_idx[w] != LLONG_MAX && (mi == LLONG_MAX || min_better(s_min[w], s_idx[w], mv, mi))) {
        mv = s_min[w];
        mi = s_idx[w];
      }
    }
    if (total == 0) {  // ops.cpp:431-438 empty-row fallback
      p.masked[base + mi] = 1;
      p.corrupted[base + mi] = p.mask_id;
      total = 1;
    }
    p.ratio[row] = r;
    if constexpr (!kOne) {
      p.counts[row] = total;
    } else {
      const unsigned long long add =
          (1ull << kSlotShift) | static_cast<unsigned long long>(total);
      const unsigned long long now = atomicAdd(p.slot, add) + add;
      s_old = now;
      if (early_ratios && static_cast<int64_t>(now >> kSlotShift) == p.batch) {
        double tr = 0.0;
        for (int w = 0; w < kMetricThreads / 32; ++w) tr += s_r[w];
        write_masked_metrics(p.metrics,
                             static_cast<int64_t>(now & ((1ull << kSlotShift) - 1)), tr,
                             p.batch, p.tokens);
        *p.slot = 0;
      }
    }
  }
  if constexpr (kOne) {
    if (early_ratios) return;
    __syncthreads();
    const unsigned long long now = s_old;
    if (static_cast<int64_t>(now >> kSlotShift) != p.batch) return;  // uniform over the CTA
    double rs = 0.0;
    if (threadIdx.x < kMetricThreads)
      for (int64_t b = threadIdx.x; b < p.batch; b += kMetricThreads)
        rs += static_cast<double>(row_ratio(p, b));
    const double tr = ratio_sum_tail(rs, s_r);
    if (threadIdx.x == 0) {
      write_masked_metrics(p.metrics, static_cast<int64_t>(now & ((1ull << kSlotShift) - 1)),
                           tr, p.batch, p.tokens);
      *p.slot = 0;
    }
  }
}

// Rows of up to 4096 tokens: 256 threads with eight tokens' loads in flight
// each; longer rows: 512 threads with four.  (Config-3 rows of 2048 tokens:
// 256 threads 3.1 us a launch, 512 threads 3.8 us, 1024 threads 5.5 us;
// 8 rows of 16384: 512 threads fastest.)
int launch_masked_rows(const MaskedParams& p, cudaStream_t s, bool one_kernel) {
  const dim3 grid(static_cast<unsigned>(p.batch));
  if (p.tokens <= 4096)
    return one_kernel ? launch_pdl(masked_diffusion_kernel<256, 8, true>, grid, dim3(256), 0, s, p)
                      : launch_pdl(masked_diffusion_kernel<256, 8, false>, grid, dim3(256), 0, s, p);
  return one_kernel ? launch_pdl(masked_diffusion_kernel<512, 4, true>, grid, dim3(512), 0, s, p)
                    : launch_pdl(masked_diffusion_kernel<512, 4, false>, grid, dim3(512), 0, s, p);
}

__global__ void __launch_bounds__(kMetricThreads) masked_metrics_kernel(const int64_t* counts,
                                                                        const float* ratio,
                                                                        int64_t batch,
                                                                        int64_t tokens,
                                                                        float* metrics) {
  pdl_wait();
  pdl_trigger();
  constexpr int kMW = kMetricThreads / 32;
  __shared__ int64_t s_c[kMW];
  __shared__ double s_r[kMW];
  int64_t c = 0;
  double rs = 0.0;
  for (int64_t b = threadIdx.x; b < batch; b += kMetricThreads) {
    c += counts[b];
    rs += static_cast<double>(ratio[b]);
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) c += __shfl_down_sync(0xffffffffu, c, d);
  if ((threadIdx.x & 31) == 0) s_c[threadIdx.x >> 5] = c;
  const double tr = ratio_sum_tail(rs, s_r);
  if (threadIdx.x == 0) {
    int64_t tc = 0;
    for (int w = 0; w < kMW; ++w) tc += s_c[w];
    write_masked_metrics(metrics, tc, tr, batch, tokens);
  }
}

// Launches the masked-diffusion row kernel and its metrics: one kernel when
// `slot` (a zeroed accumulator) is given, else the row kernel and the
// one-block metrics kernel over p.counts.
int launch_masked(MaskedParams p, unsigned long long* slot, cudaStream_t s) {
  p.slot = slot;
  int rc = launch_masked_rows(p, s, slot != nullptr);
  if (rc != CID_OK || slot != nullptr) return rc;
  return launch_pdl(masked_metrics_kernel, dim3(1), dim3(kMetricThreads), 0, s,
                    static_cast<const int64_t*>(p.counts), static_cast<const float*>(p.ratio),
                    p.batch, p.tokens, p.metrics);
}

// ---------------------------------------------------------------------------
// thought corruption
// ---------------------------------------------------------------------------

struct ThoughtParams {
  cid_dtype_t sdt;  // semantic dtype
  const void* sem;
  cid_dtype_t tdt;
  const void* ts;
  cid_dtype_t odt;
  const void* occ;
  const void* eps;
  int64_t rows, hidden;
  void* corrupted;
  void* local_noise;
  void* masked_eps;
};

// alpha = cos(t * pi/2)^2 evaluated in the timestep dtype (ops.cpp:277-281),
// returned in double (exact for every storage dtype).
__device__ double thought_alpha(cid_dtype_t tdt, const void* ts, int64_t row) {
  const double half_pi = 1.57079632679489661923;
  if (tdt == CID_DTYPE_F64) {
    const double t = static_cast<const double*>(ts)[row];
    const double c = cos(__dmul_rn(t, half_pi));
    return __dmul_rn(c, c);
  }
  const float t = load_float(tdt, ts, row);
  const float arg = round_to(tdt, __fmul_rn(t, static_cast<float>(half_pi)));
  const float c = round_to(tdt, static_cast<float>(cos(static_cast<double>(arg))));
  return static_cast<double>(round_to(tdt, __fmul_rn(c, c)));
}

__global__ void __launch_bounds__(kT) thought_kernel(ThoughtParams p) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const bool occ = load_truthy(p.odt, p.occ, row);
  const int64_t base = row * p.hidden;
  if (p.sdt == CID_DTYPE_F64) {
    const double* x = static_cast<const double*>(p.sem);
    const double* e = static_cast<const double*>(p.eps);
    double* out = static_cast<double*>(p.corrupted);
    double* me = static_cast<double*>(p.masked_eps);
    const double a = thought_alpha(p.tdt, p.ts, row);  // .to(float64) is exact
    const double sa = __dsqrt_rn(a), sb = __dsqrt_rn(__dsub_rn(1.0, a));
    for (int64_t h = threadIdx.x; h < p.hidden; h += kT) {
      const double ev = e[base + h];
      out[base + h] = occ ? __dadd_rn(__dmul_rn(sa, x[base + h]), __dmul_rn(sb, ev)) : 0.0;
      me[base + h] = occ ? ev : 0.0;
    }
    if (threadIdx.x == 0)
      static_cast<double*>(p.local_noise)[row] = occ ? load_double(p.tdt, p.ts, row) : 0.0;
    return;
  }
  // float32 / float16 / bfloat16 semantic: float arithmetic rounded per op
  const cid_dtype_t S = p.sdt;
  const float a = round_to(S, static_cast<float>(thought_alpha(p.tdt, p.ts, row)));
  const float sa = round_to(S, __fsqrt_rn(a));
  const float sb = round_to(S, __fsqrt_rn(round_to(S, __fsub_rn(1.0f, a))));
  for (int64_t h = threadIdx.x; h < p.hidden; h += kT) {
    const float x = load_float(S, p.sem, base + h);
    const float ev = load_float(S, p.eps, base + h);
    const float v = round_to(S, __fadd_rn(round_to(S, __fmul_rn(sa, x)), round_to(S, __fmul_rn(sb, ev))));
    store_float(S, p.corrupted, base + h, occ ? v : 0.0f);
    store_float(S, p.masked_eps, base + h, occ ? ev : 0.0f);
  }
  if (threadIdx.x == 0) {
    const float t = p.tdt == CID_DTYPE_F64 ? static_cast<float>(static_cast<const double*>(p.ts)[row])
                                           : load_float(p.tdt, p.ts, row);
    store_float(S, p.local_noise, row, occ ? t : 0.0f);
  }
}

// ---------------------------------------------------------------------------
// display corruption
// ---------------------------------------------------------------------------

struct DisplayCorruptParams {
  const int64_t* ids;
  cid_dtype_t tdt;
  const void* ts;
  cid_dtype_t edt;
  const void* elig;
  cid_dtype_t rdt;
  const void* crand;
  cid_dtype_t pdt;
  const void* rrand;
  const int64_t* roff;
  int64_t batch, tokens, mask_id, eos_id, vocab;
  int has_eos;
  int replace;
  float repl_thr;
  int64_t* corrupted;
  int64_t* labels;
  uint8_t* masked;
  uint8_t* replaced;
};

__device__ __forceinline__ int64_t floor_mod(int64_t a, int64_t m) {
  const int64_t r = a % m;
  return (r != 0 && ((r < 0) != (m < 0))) ? r + m : r;
}

// torch.remainder(id + offset, vocab) for vocab >= 3 (ops.cpp:364-365): the
// int64 sum wraps as ATen's does; a sum already in [0, vocab) needs no
// division and one in [0, 2^32) a 32-bit one.
__device__ __forceinline__ int64_t wrap_vocab(int64_t id, int64_t offset, int64_t vocab) {
  const int64_t x = static_cast<int64_t>(static_cast<uint64_t>(id) + static_cast<uint64_t>(offset));
  if (x >= 0 && x < vocab) return x;
  if (x >= 0 && x <= int64_t{UINT32_MAX} && vocab <= int64_t{UINT32_MAX})
    return static_cast<uint32_t>(x) % static_cast<uint32_t>(vocab);
  return floor_mod(x, vocab);
}

// The four outputs of one position (ops.cpp:339-389): corrupted where the
// uniform falls below the timestep on an eligible position, or at the row's
// fallback position; a corrupted position whose replacement uniform is below
// the replacement threshold takes the offset token (skipping the mask id, its
// own id and EOS), every other corrupted position the mask id.
__device__ __forceinline__ void write_display_corrupt(const DisplayCorruptParams& p, int64_t i,
                                                      bool is_fallback, float t, bool el, float u,
                                                      int64_t id, float rr, int64_t off) {
  const bool pos = ((u < t) && el) || is_fallback;
  bool rep = false;
  int64_t value = id;
  if (p.replace) {
    rep = pos && (rr < p.repl_thr);  // ops.cpp:362-363
    int64_t cand = wrap_vocab(id, off, p.vocab);
    for (int it = 0; it < 3; ++it) {  // ops.cpp:366-376; cand stays in [0, vocab)
      const bool forbidden = cand == p.mask_id || cand == id || (p.has_eos && cand == p.eos_id);
      if (forbidden) cand = cand + 1 == p.vocab ? 0 : cand + 1;
    }
    if (rep) value = cand;
  }
  const bool msk = pos && !rep;
  if (msk) value = p.mask_id;
  p.corrupted[i] = value;
  p.labels[i] = pos ? id : -100;  // ops.cpp:386-389
  p.masked[i] = msk;
  p.replaced[i] = rep;
}

// One CTA of kBT threads per row, two passes over the row: the first finds
// whether any eligible position falls below the timestep and the first
// eligible position (the fallback, ops.cpp:326-337); the second writes the
// four outputs.  Each thread issues the loads of U tokens (kBT apart, so
// every load instruction is coalesced) before it uses them.
template <int kBT, int U>
__global__ void __launch_bounds__(kBT) display_corrupt_kernel(DisplayCorruptParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int kW = kBT / 32;
  __shared__ int64_t s_first[kW];
  const int64_t row = blockIdx.x;
  const int64_t base = row * p.tokens;
  const float t = load_float(p.tdt, p.ts, row);  // timesteps.to(float)
  if (p.tokens <= int64_t{kBT} * U) {
    // the row is one batch of loads: every input of the thread's tokens is
    // loaded at once and kept in registers across the reductions (one memory
    // round trip instead of two)
    bool el[U];
    float u[U], rr[U];
    int64_t id[U], off[U];
    int any = 0;
    int64_t first = LLONG_MAX;
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t k = threadIdx.x + int64_t{j} * kBT;
      const bool in = k < p.tokens;
      el[j] = in && load_truthy(p.edt, p.elig, base + k);
      u[j] = in ? load_float(p.rdt, p.crand, base + k) : 1.0f;
      id[j] = in ? p.ids[base + k] : 0;
      rr[j] = in && p.replace ? load_float(p.pdt, p.rrand, base + k) : 1.0f;
      off[j] = in && p.replace ? p.roff[base + k] : 0;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      any |= (u[j] < t) && el[j];  // ops.cpp:326-328
      if (el[j] && first == LLONG_MAX) first = threadIdx.x + int64_t{j} * kBT;
    }
    any = __syncthreads_or(any);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) first = min(first, __shfl_down_sync(0xffffffffu, first, d));
    if ((threadIdx.x & 31) == 0) s_first[threadIdx.x >> 5] = first;
    __syncthreads();
    int64_t fe1 = s_first[0];
#pragma unroll
    for (int w = 1; w < kW; ++w) fe1 = min(fe1, s_first[w]);
    const int64_t fb1 = (!any && t > 0.0f && fe1 != LLONG_MAX) ? fe1 : -1;
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t k = threadIdx.x + int64_t{j} * kBT;
      if (k < p.tokens) write_display_corrupt(p, base + k, k == fb1, t, el[j], u[j], id[j], rr[j], off[j]);
    }
    return;
  }
  int any_corrupt = 0;
  int64_t first_elig = LLONG_MAX;
  for (int64_t k0 = threadIdx.x; k0 < p.tokens; k0 += int64_t{kBT} * U) {
    bool el[U];
    float u[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t k = k0 + int64_t{j} * kBT;
      el[j] = k < p.tokens && load_truthy(p.edt, p.elig, base + k);
      u[j] = k < p.tokens ? load_float(p.rdt, p.crand, base + k) : 1.0f;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      any_corrupt |= (u[j] < t) && el[j];  // ops.cpp:326-328
      if (el[j] && first_elig == LLONG_MAX) first_elig = k0 + int64_t{j} * kBT;
    }
  }
  any_corrupt = __syncthreads_or(any_corrupt);
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) first_elig = min(first_elig, __shfl_down_sync(0xffffffffu, first_elig, d));
  if ((threadIdx.x & 31) == 0) s_first[threadIdx.x >> 5] = first_elig;
  __syncthreads();
  int64_t fe = s_first[0];
#pragma unroll
  for (int w = 1; w < kW; ++w) fe = min(fe, s_first[w]);
  // ops.cpp:330-337 first-eligible fallback
  const int64_t fallback = (!any_corrupt && t > 0.0f && fe != LLONG_MAX) ? fe : -1;
  for (int64_t k0 = threadIdx.x; k0 < p.tokens; k0 += int64_t{kBT} * U) {
    bool el[U];
    float u[U], rr[U];
    int64_t id[U], off[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t k = k0 + int64_t{j} * kBT;
      const bool in = k < p.tokens;
      el[j] = in && load_truthy(p.edt, p.elig, base + k);
      u[j] = in ? load_float(p.rdt, p.crand, base + k) : 1.0f;
      id[j] = in ? p.ids[base + k] : 0;
      rr[j] = in && p.replace ? load_float(p.pdt, p.rrand, base + k) : 1.0f;
      off[j] = in && p.replace ? p.roff[base + k] : 0;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int64_t k = k0 + int64_t{j} * kBT;
      if (k >= p.tokens) break;
      write_display_corrupt(p, base + k, k == fallback, t, el[j], u[j], id[j], rr[j], off[j]);
    }
  }
}

}  // namespace
}  // namespace cid

using namespace cid;

namespace {

// The arguments both masked-diffusion entry points share (csrc/ops.cpp:406,
// :416-420): a non-empty batch x tokens, 0 < min <= max <= 1, aligned and
// non-NULL arrays.
int check_masked(const int64_t* clean_ids, const float* ratio_random, const float* mask_random,
                 int64_t batch, int64_t tokens, double min_mask_ratio, double max_mask_ratio,
                 const int64_t* corrupted, const uint8_t* masked, const float* ratio,
                 const float* metrics) {
  int64_t count = 0;
  if (batch <= 0 || tokens <= 0 || batch > kMaxRows || !count_ok(batch, tokens, &count) ||
      count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  if (!(min_mask_ratio > 0.0 && min_mask_ratio <= max_mask_ratio && max_mask_ratio <= 1.0))
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{clean_ids, 8}, {ratio_random, 4}, {mask_random, 4}, {corrupted, 8},
                  {ratio, 4}, {metrics, 4}}))
    return CID_ERR_MISALIGNED;
  if (any_null({clean_ids, ratio_random, mask_random, corrupted, masked, ratio, metrics}))
    return CID_ERR_INVALID_ARGUMENT;
  return CID_OK;
}

}  // namespace

extern "C" size_t cid_masked_diffusion_workspace_bytes(int64_t batch) {
  return batch > 0 && batch <= kMaxRows ? static_cast<size_t>(batch) * sizeof(int64_t) : 0;
}

// ---------------------------------------------------------------------------
// Masked diffusion captured into a CUDA graph runs as one kernel.  Its
// accumulator must be zero when the kernel starts and the kernel clears it
// when it ends, so a launch takes a slot of its own for as long as the graph
// exists: slots come from a zero-initialised array in the library's device
// image and are never handed out twice.  A graph's replays run one after
// another, so they share its slot safely; two instances of one graph (two
// executable graphs made from it) must not run at the same time.  Eager
// calls, calls captured before any eager call has looked the array up on
// that device (the lookup could invalidate a capture) and calls beyond the
// last slot run the two-kernel form over the caller's workspace, with
// bit-identical results.
// ---------------------------------------------------------------------------

namespace {

constexpr int kMaskedSlots = 4096;
constexpr int kSlotDevices = 64;
static __device__ __align__(256) unsigned long long g_masked_slots[kMaskedSlots];

std::mutex g_slot_mutex;
unsigned long long* g_slot_base[kSlotDevices] = {};
int g_slot_next[kSlotDevices] = {};

// The slot for a launch on `s`, or nullptr for the two-kernel form.
unsigned long long* masked_slot(cudaStream_t s, int64_t batch, int64_t tokens) {
  if (batch > kSlotMaxRows || batch * tokens >= kSlotMaxTokens) return nullptr;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  if (dev < 0 || dev >= kSlotDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_slot_mutex);
  if (st != cudaStreamCaptureStatusActive) {
    if (g_slot_base[dev] == nullptr) {
      void* q = nullptr;
      if (cudaGetSymbolAddress(&q, g_masked_slots) == cudaSuccess)
        g_slot_base[dev] = static_cast<unsigned long long*>(q);
      else
        (void)cudaGetLastError();
    }
    return nullptr;
  }
  if (g_slot_base[dev] == nullptr || g_slot_next[dev] >= kMaskedSlots) return nullptr;
  return g_slot_base[dev] + g_slot_next[dev]++;
}

}  // namespace

extern "C" int cid_masked_diffusion_corrupt(const int64_t* clean_ids, const float* ratio_random,
                                            const float* mask_random, int64_t batch,
                                            int64_t tokens, int64_t mask_token_id,
                                            double min_mask_ratio, double max_mask_ratio,
                                            int64_t* corrupted, uint8_t* masked, float* ratio,
                                            float* metrics, void* workspace, void* stream) {
  int rc = check_masked(clean_ids, ratio_random, mask_random, batch, tokens, min_mask_ratio,
                        max_mask_ratio, corrupted, masked, ratio, metrics);
  if (rc != CID_OK) return rc;
  if (misaligned({{workspace, 16}})) return CID_ERR_MISALIGNED;
  if (workspace == nullptr) return CID_ERR_INVALID_ARGUMENT;
  MaskedParams p;
  p.clean = clean_ids;
  p.ratio_random = ratio_random;
  p.mask_random = mask_random;
  p.batch = batch;
  p.tokens = tokens;
  p.mask_id = mask_token_id;
  p.span = static_cast<float>(max_mask_ratio - min_mask_ratio);
  p.lo = static_cast<float>(min_mask_ratio);
  p.corrupted = corrupted;
  p.masked = masked;
  p.ratio = ratio;
  p.metrics = metrics;
  p.counts = static_cast<int64_t*>(workspace);
  cudaStream_t s = as_stream(stream);
  return launch_masked(p, masked_slot(s, batch, tokens), s);
}

// ---------------------------------------------------------------------------
// Allocation-free masked diffusion.
//
// Some callers cannot hand this library device memory for scratch: a host
// program that reserves all device memory up front for its own pool and
// forbids third-party cudaMalloc, a serving loop that must not pay
// cudaMalloc's latency and implicit synchronisation on its request path, or
// a thin FFI binding with no device allocator to draw a workspace from.
// For them the per-row counts live in a fixed array in the library's own
// device image.  Every GPU that loads the library holds the array until the
// process exits.  Calls on one device share it, so calls that overlap on the
// GPU (e.g. on two streams) race on it.  Each call writes the count of every
// row before the metrics kernel reads it, so nothing needs clearing between
// calls.
// ---------------------------------------------------------------------------

namespace cid {
namespace {

static __device__ __align__(256) int64_t g_no_alloc_counts[CID_NO_ALLOC_MAX_BATCH];

constexpr int kMaxDevices = 64;
std::mutex g_no_alloc_mutex;
int64_t* g_no_alloc_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  Host code only
// holds a host-side stand-in for the symbol, so the address is looked up once
// per device, with that device current.
int no_alloc_scratch(int64_t** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return record_cuda_error(err);
  if (dev < 0 || dev >= kMaxDevices) return CID_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_no_alloc_mutex);
  if (g_no_alloc_addr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_no_alloc_counts);
    if (err != cudaSuccess) return record_cuda_error(err);
    g_no_alloc_addr[dev] = static_cast<int64_t*>(p);
  }
  *out = g_no_alloc_addr[dev];
  return CID_OK;
}

}  // namespace
}  // namespace cid

extern "C" int cid_masked_diffusion_corrupt_no_alloc(
    const int64_t* clean_ids, const float* ratio_random, const float* mask_random,
    int64_t batch, int64_t tokens, int64_t mask_token_id, double min_mask_ratio,
    double max_mask_ratio, int64_t* corrupted, uint8_t* masked, float* ratio, float* metrics,
    void* stream) {
  if (batch > CID_NO_ALLOC_MAX_BATCH) return CID_ERR_SCRATCH_LIMIT;
  int rc = check_masked(clean_ids, ratio_random, mask_random, batch, tokens, min_mask_ratio,
                        max_mask_ratio, corrupted, masked, ratio, metrics);
  if (rc != CID_OK) return rc;
  int64_t* scratch = nullptr;
  rc = no_alloc_scratch(&scratch);
  if (rc != CID_OK) return rc;
  MaskedParams p;
  p.clean = clean_ids;
  p.ratio_random = ratio_random;
  p.mask_random = mask_random;
  p.batch = batch;
  p.tokens = tokens;
  p.mask_id = mask_token_id;
  p.span = static_cast<float>(max_mask_ratio - min_mask_ratio);
  p.lo = static_cast<float>(min_mask_ratio);
  p.corrupted = corrupted;
  p.masked = masked;
  p.ratio = ratio;
  p.metrics = metrics;
  p.counts = scratch;
  return launch_masked(p, nullptr, as_stream(stream));
}

extern "C" int cid_thought_corrupt(cid_dtype_t sem_dtype, const void* semantic,
                                   cid_dtype_t t_dtype, const void* timesteps,
                                   cid_dtype_t occ_dtype, const void* occupancy,
                                   const void* epsilon, int64_t rows, int64_t hidden,
                                   void* corrupted, void* local_noise, void* masked_epsilon,
                                   void* stream) {
  if (!is_float_dtype(sem_dtype) || !is_float_dtype(t_dtype) || !is_known_dtype(occ_dtype))
    return CID_ERR_UNSUPPORTED_DTYPE;
  int64_t count = 0;
  if (!count_ok(rows, hidden, &count) || rows > kMaxRows || count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  const size_t es = static_cast<size_t>(dtype_size(sem_dtype));
  if (misaligned({{semantic, es}, {epsilon, es}, {corrupted, es}, {local_noise, es},
                  {masked_epsilon, es}, {timesteps, static_cast<size_t>(dtype_size(t_dtype))},
                  {occupancy, static_cast<size_t>(dtype_size(occ_dtype))}}))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  // rows x hidden arrays may be NULL when hidden == 0
  if (any_null({timesteps, occupancy, local_noise}) ||
      (hidden > 0 && any_null({semantic, epsilon, corrupted, masked_epsilon})))
    return CID_ERR_INVALID_ARGUMENT;
  ThoughtParams p{sem_dtype, semantic, t_dtype, timesteps, occ_dtype, occupancy, epsilon,
                  rows, hidden, corrupted, local_noise, masked_epsilon};
  return launch_pdl(thought_kernel, dim3(static_cast<unsigned>(rows)), dim3(kT), 0,
                    as_stream(stream), p);
}

extern "C" int cid_display_corrupt(const int64_t* token_ids, cid_dtype_t t_dtype,
                                   const void* timesteps, cid_dtype_t elig_dtype,
                                   const void* eligible, cid_dtype_t rand_dtype,
                                   const void* corruption_random, cid_dtype_t repl_dtype,
                                   const void* replacement_random,
                                   const int64_t* replacement_offsets, int64_t batch,
                                   int64_t tokens, int64_t mask_token_id, int has_eos,
                                   int64_t eos_token_id, int64_t vocab_size,
                                   double replacement_fraction, int64_t* corrupted,
                                   int64_t* labels, uint8_t* masked, uint8_t* replaced,
                                   void* stream) {
  const int replace = replacement_fraction > 0.0;
  if (!is_float_dtype(t_dtype) || !is_known_dtype(elig_dtype) || !is_float_dtype(rand_dtype) ||
      (replace && !is_float_dtype(repl_dtype)))
    return CID_ERR_UNSUPPORTED_DTYPE;
  if (!(replacement_fraction >= 0.0 && replacement_fraction <= 1.0))
    return CID_ERR_INVALID_ARGUMENT;  // ops.cpp:320-322
  if (replace && vocab_size < 3) return CID_ERR_INVALID_ARGUMENT;  // ops.cpp:343-345
  int64_t count = 0;
  if (!count_ok(batch, tokens, &count) || batch > kMaxRows || count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{token_ids, 8}, {timesteps, static_cast<size_t>(dtype_size(t_dtype))},
                  {eligible, static_cast<size_t>(dtype_size(elig_dtype))},
                  {corruption_random, static_cast<size_t>(dtype_size(rand_dtype))},
                  {corrupted, 8}, {labels, 8}}) ||
      (replace && misaligned({{replacement_random, static_cast<size_t>(dtype_size(repl_dtype))},
                              {replacement_offsets, 8}})))
    return CID_ERR_MISALIGNED;
  if (batch == 0 || tokens == 0) return CID_OK;
  // the replacement inputs are read only when replacement_fraction > 0 (ops.cpp:346-348)
  if (any_null({token_ids, timesteps, eligible, corruption_random, corrupted, labels, masked,
                replaced}) ||
      (replace && any_null({replacement_random, replacement_offsets})))
    return CID_ERR_INVALID_ARGUMENT;
  DisplayCorruptParams p{token_ids, t_dtype, timesteps, elig_dtype, eligible, rand_dtype,
                         corruption_random, repl_dtype, replacement_random,
                         replacement_offsets, batch, tokens, mask_token_id, eos_token_id,
                         vocab_size, has_eos, replace,
                         static_cast<float>(replacement_fraction), corrupted, labels, masked,
                         replaced};
  // Two tokens a thread, a row in one batch of loads, up to 2048 tokens; four
  // tokens a thread over 1024 threads beyond.  The per-token work (the
  // replacement's wrap and skips) favours threads over loads in flight: at
  // [64, 1024] 3.6 us against 5.1 with 256 threads x 4 tokens, at [64, 2048]
  // 5.5 against 6.0 with 512 x 4 and 9.7 with 256 x 8 (CUDA-graph replays).
  const unsigned grid = static_cast<unsigned>(batch);
  cudaStream_t s = as_stream(stream);
  if (tokens <= 512)
    return launch_pdl(display_corrupt_kernel<256, 2>, dim3(grid), dim3(256), 0, s, p);
  if (tokens <= 1024)
    return launch_pdl(display_corrupt_kernel<512, 2>, dim3(grid), dim3(512), 0, s, p);
  if (tokens <= 2048)
    return launch_pdl(display_corrupt_kernel<1024, 2>, dim3(grid), dim3(1024), 0, s, p);
  return launch_pdl(display_corrupt_kernel<1024, 4>, dim3(grid), dim3(1024), 0, s, p);
}
