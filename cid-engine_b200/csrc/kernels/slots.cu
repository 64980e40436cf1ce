// Thought-slot state kernels: first-free prefix allocation, the rollout slot
// transition and live occupancy.  One warp per batch row: slot decisions are
// made 32 at a time with warp ballots (first blocking slot = first set bit,
// allocation rank = popcount prefix), so a row of S slots takes ceil(S/32)
// steps instead of the reference kernel's single-thread scan
// (csrc/cuda/prefix_allocation.cu:14-49 of fwerkor/cid-engine v1.1.0).
#include <climits>
#include <cmath>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kWarpsPerBlock = 4;

__device__ __forceinline__ unsigned lanemask_le() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_le;" : "=r"(m));
  return m;
}

// ATen max(-1) index over n values of `dt` starting at element `base`:
// first NaN, else first maximum (compared in double, exact for every dtype).
__device__ __forceinline__ int64_t argmax_first(cid_dtype_t dt, const void* p, int64_t base,
                                                int64_t n) {
  double bv = load_double(dt, p, base);
  int64_t bi = 0;
  for (int64_t k = 1; k < n; ++k) {
    if (bv != bv) break;
    const double v = load_double(dt, p, base + k);
    if (v != v || v > bv) {
      bv = v;
      bi = k;
    }
  }
  return bi;
}

// Shared warp-level prefix allocation over one row, 32 slots per step
// (semantics of csrc/ops.cpp:41-65).  occ(s) -> bool, logit(s) -> float;
// emit(s, selected) is called for every slot s < slots by lane s % 32.
template <typename Occ, typename Logit, typename Emit>
__device__ __forceinline__ void warp_prefix_allocation(int64_t slots, float thr,
                                                       int64_t max_allocations, Occ occ,
                                                       Logit logit, Emit emit) {
  const int lane = threadIdx.x & 31;
  int64_t rank = 0;
  bool blocked = false;
  for (int64_t s0 = 0; s0 < slots; s0 += 32) {
    const int64_t s = s0 + lane;
    const bool in = s < slots;
    const bool occupied = in && occ(s);
    const bool is_free = in && !occupied;
    bool elig = false;
    if (is_free && !blocked) elig = sigmoid_f32(logit(s)) >= thr;  // ops.cpp:59
    // blocked = cumsum(free & !eligible) > 0, the blocking slot included
    const unsigned bl = __ballot_sync(0xffffffffu, is_free && !elig);
    const int first_block = bl ? __ffs(bl) - 1 : 32;
    const bool sel = !blocked && is_free && elig && lane < first_block;
    const unsigned sm = __ballot_sync(0xffffffffu, sel);
    const int64_t r = rank + __popc(sm & lanemask_le());
    if (in) emit(s, sel && r <= max_allocations);  // ops.cpp:63-64
    rank += __popc(sm);
    if (bl) blocked = true;
  }
}

struct PrefixParams {
  cid_dtype_t occ_dtype;
  const void* occ;
  int64_t ors, ocs;
  cid_dtype_t logit_dtype;
  const void* logits;
  int64_t lrs, lcs;
  int64_t batch, slots;
  float thr;
  int64_t max_alloc;
  uint8_t* out;
};

__global__ void prefix_allocation_kernel(PrefixParams p) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.batch) return;
  warp_prefix_allocation(
      p.slots, p.thr, p.max_alloc,
      [&](int64_t s) { return load_truthy(p.occ_dtype, p.occ, row * p.ors + s * p.ocs); },
      [&](int64_t s) { return load_float(p.logit_dtype, p.logits, row * p.lrs + s * p.lcs); },
      [&](int64_t s, bool v) { p.out[row * p.slots + s] = v; });
}

struct RolloutParams {
  cid_dtype_t occ_dtype;
  const void* occ;
  cid_dtype_t dtype;
  const void* alloc;
  const void* life;
  const void* rev;
  const void* in_life;
  int64_t batch, slots, F, Rv;
  float thr;
  int64_t max_alloc, retired;
  uint8_t* next;
  int64_t* life_idx;
  int64_t* rev_idx;
  int64_t* in_idx;
  uint8_t* present;
  uint8_t* live;
  // optional: live occupancy of the next state (csrc/ops.cpp:12-39 applied
  // to next_occupancy, in the lifecycle logits' dtype `live_dtype`)
  cid_dtype_t live_dtype;
  void* live_occ;
};

__device__ __forceinline__ float clamp01f(float x) { return x != x ? x : fminf(fmaxf(x, 0.0f), 1.0f); }
__device__ __forceinline__ double clamp01d(double x) { return x != x ? x : fmin(fmax(x, 0.0), 1.0); }

// csrc/ops.cpp:184-256 fused into one pass per row.
__global__ void rollout_kernel(RolloutParams p) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.batch) return;
  const int64_t base = row * p.slots;
  warp_prefix_allocation(
      p.slots, p.thr, p.max_alloc,
      [&](int64_t s) { return load_truthy(p.occ_dtype, p.occ, base + s); },
      [&](int64_t s) { return load_float(p.dtype, p.alloc, base + s); },
      [&](int64_t s, bool alloc) {
        const int64_t i = base + s;
        const bool occ = load_truthy(p.occ_dtype, p.occ, i);
        const bool nxt = occ || alloc;
        const int64_t li = argmax_first(p.dtype, p.life, i * p.F, p.F);
        const int64_t ri = argmax_first(p.dtype, p.rev, i * p.Rv, p.Rv);
        const int64_t ii = argmax_first(p.dtype, p.in_life, i * p.F, p.F);
        bool present = false;  // abs().sum(-1).ne(0): any non-zero (NaN included)
        for (int64_t k = 0; k < p.F; ++k) present = present || load_truthy(p.dtype, p.in_life, i * p.F + k);
        const bool prev_retired = occ && ii == p.retired;
        const bool newly = nxt && !occ;
        const bool pred_retired = li == p.retired;
        p.next[i] = nxt;
        p.life_idx[i] = li;
        p.rev_idx[i] = ri;
        p.in_idx[i] = ii;
        p.present[i] = present;
        p.live[i] = nxt && !prev_retired && (!pred_retired || newly);
        if (p.live_occ) {  // clamp(next, 0, 1) * (1 - clamp(lifecycle[..., r], 0, 1))
          const int64_t at = i * p.F + p.retired;
          if (p.live_dtype == CID_DTYPE_F64) {
            const double r = clamp01d(load_double(p.dtype, p.life, at));
            static_cast<double*>(p.live_occ)[i] = __dmul_rn(nxt ? 1.0 : 0.0, __dsub_rn(1.0, r));
          } else {
            const float r = clamp01f(load_float(p.dtype, p.life, at));
            const float keep = round_to(p.live_dtype, __fsub_rn(1.0f, r));
            store_float(p.live_dtype, p.live_occ, i, __fmul_rn(nxt ? 1.0f : 0.0f, keep));
          }
        }
      });
}

struct LiveParams {
  cid_dtype_t dtype;
  const void* occ;
  const void* life;
  int64_t rows, F, retired;
  void* out;
};

// csrc/ops.cpp:12-39: clamp(occ, 0, 1) * (1 - clamp(lifecycle[..., r], 0, 1)),
// each op rounded to the storage dtype.
__global__ void live_kernel(LiveParams p) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < p.rows;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (p.dtype == CID_DTYPE_F64) {
      const double o = clamp01d(static_cast<const double*>(p.occ)[i]);
      double v = o;
      if (p.life) {
        const double r = clamp01d(static_cast<const double*>(p.life)[i * p.F + p.retired]);
        v = __dmul_rn(o, __dsub_rn(1.0, r));
      }
      static_cast<double*>(p.out)[i] = v;
    } else {
      const float o = clamp01f(load_float(p.dtype, p.occ, i));
      float v = o;
      if (p.life) {
        const float r = clamp01f(load_float(p.dtype, p.life, i * p.F + p.retired));
        const float keep = round_to(p.dtype, __fsub_rn(1.0f, r));
        v = __fmul_rn(o, keep);
      }
      store_float(p.dtype, p.out, i, v);
    }
  }
}

// A batch x slots strided view: non-negative strides whose largest element
// offset stays within kMaxCount.
bool strided_span_ok(int64_t batch, int64_t slots, int64_t row_stride, int64_t col_stride) {
  int64_t a = 0, b = 0;
  return row_stride >= 0 && col_stride >= 0 && count_ok(batch - 1, row_stride, &a) &&
         count_ok(slots - 1, col_stride, &b) && a <= kMaxCount && b <= kMaxCount - a;
}

}  // namespace
}  // namespace cid

using namespace cid;

extern "C" int cid_prefix_allocation_mask(cid_dtype_t occ_dtype, const void* occupancy,
                                          int64_t occ_row_stride, int64_t occ_col_stride,
                                          cid_dtype_t logit_dtype, const void* logits,
                                          int64_t logit_row_stride, int64_t logit_col_stride,
                                          int64_t batch, int64_t slots, double threshold,
                                          int64_t max_allocations, uint8_t* out, void* stream) {
  if (!is_known_dtype(occ_dtype) || !is_float_dtype(logit_dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (!(threshold >= 0.0 && threshold <= 1.0)) return CID_ERR_INVALID_ARGUMENT;  // ops.cpp:50
  if (max_allocations <= 0) return CID_ERR_INVALID_ARGUMENT;                      // ops.cpp:51
  int64_t count = 0;
  if (!count_ok(batch, slots, &count) || batch > kMaxRows || count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  if (batch > 0 && slots > 0 &&
      (!strided_span_ok(batch, slots, occ_row_stride, occ_col_stride) ||
       !strided_span_ok(batch, slots, logit_row_stride, logit_col_stride)))
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{occupancy, static_cast<size_t>(dtype_size(occ_dtype))},
                  {logits, static_cast<size_t>(dtype_size(logit_dtype))}}))
    return CID_ERR_MISALIGNED;
  if (batch == 0 || slots == 0) return CID_OK;
  if (any_null({occupancy, logits, out})) return CID_ERR_INVALID_ARGUMENT;
  PrefixParams p{occ_dtype, occupancy, occ_row_stride, occ_col_stride, logit_dtype, logits,
                 logit_row_stride, logit_col_stride, batch, slots,
                 static_cast<float>(threshold), max_allocations, out};
  const int64_t blocks = (batch + kWarpsPerBlock - 1) / kWarpsPerBlock;
  return launch_pdl(prefix_allocation_kernel, dim3(static_cast<unsigned>(blocks)),
                    dim3(kWarpsPerBlock * 32), 0, as_stream(stream), p);
}

namespace {

int launch_rollout(const RolloutParams& p, void* stream) {
  const int64_t blocks = (p.batch + kWarpsPerBlock - 1) / kWarpsPerBlock;
  return launch_pdl(rollout_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kWarpsPerBlock * 32),
                    0, as_stream(stream), p);
}

// The arguments of a rollout call (with its live-occupancy output when
// `with_live`): dtypes, scalars (threshold as the caller passed it), extents,
// alignment, and (when there is work) non-NULL arrays.
int check_rollout(const RolloutParams& p, double threshold, bool with_live) {
  if (!is_known_dtype(p.occ_dtype) || !is_float_dtype(p.dtype) ||
      (with_live && !is_float_dtype(p.live_dtype)))
    return CID_ERR_UNSUPPORTED_DTYPE;
  if (p.retired < 0 || p.retired >= p.F) return CID_ERR_INVALID_ARGUMENT;
  if (!(threshold >= 0.0 && threshold <= 1.0)) return CID_ERR_INVALID_ARGUMENT;
  if (p.max_alloc <= 0 || p.Rv <= 0) return CID_ERR_INVALID_ARGUMENT;
  const int64_t widest = p.F > p.Rv ? p.F : p.Rv;
  int64_t count = 0;
  if (!count_ok(p.batch, p.slots, widest, &count) || p.batch > kMaxRows || count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  const size_t es = static_cast<size_t>(dtype_size(p.dtype));
  if (misaligned({{p.occ, static_cast<size_t>(dtype_size(p.occ_dtype))}, {p.alloc, es},
                  {p.life, es}, {p.rev, es}, {p.in_life, es}, {p.life_idx, 8}, {p.rev_idx, 8},
                  {p.in_idx, 8}, {p.live_occ, static_cast<size_t>(dtype_size(p.live_dtype))}}))
    return CID_ERR_MISALIGNED;
  if (p.batch == 0 || p.slots == 0) return CID_OK;
  if (any_null({p.occ, p.alloc, p.life, p.rev, p.in_life, p.next, p.life_idx, p.rev_idx,
                p.in_idx, p.present, p.live}) ||
      (with_live && p.live_occ == nullptr))
    return CID_ERR_INVALID_ARGUMENT;
  return CID_OK;
}

}  // namespace

extern "C" int cid_rollout_slot_transition(
    cid_dtype_t occ_dtype, const void* occupancy, cid_dtype_t dtype,
    const void* allocation_logits, const void* lifecycle_logits, const void* revision_logits,
    const void* input_lifecycle, int64_t batch, int64_t slots, int64_t lifecycles,
    int64_t revisions, double threshold, int64_t max_allocations, int64_t retired_index,
    uint8_t* next_occupancy, int64_t* lifecycle_indices, int64_t* revision_indices,
    int64_t* input_lifecycle_indices, uint8_t* input_lifecycle_present, uint8_t* live_slots,
    void* stream) {
  RolloutParams p{occ_dtype, occupancy, dtype, allocation_logits, lifecycle_logits,
                  revision_logits, input_lifecycle, batch, slots, lifecycles, revisions,
                  static_cast<float>(threshold), max_allocations, retired_index,
                  next_occupancy, lifecycle_indices, revision_indices, input_lifecycle_indices,
                  input_lifecycle_present, live_slots, dtype, nullptr};
  const int rc = check_rollout(p, threshold, false);
  if (rc != CID_OK || batch == 0 || slots == 0) return rc;
  return launch_rollout(p, stream);
}

extern "C" int cid_rollout_slot_transition_live(
    cid_dtype_t occ_dtype, const void* occupancy, cid_dtype_t dtype,
    const void* allocation_logits, const void* lifecycle_logits, const void* revision_logits,
    const void* input_lifecycle, int64_t batch, int64_t slots, int64_t lifecycles,
    int64_t revisions, double threshold, int64_t max_allocations, int64_t retired_index,
    uint8_t* next_occupancy, int64_t* lifecycle_indices, int64_t* revision_indices,
    int64_t* input_lifecycle_indices, uint8_t* input_lifecycle_present, uint8_t* live_slots,
    cid_dtype_t live_dtype, void* live_occupancy, void* stream) {
  RolloutParams p{occ_dtype, occupancy, dtype, allocation_logits, lifecycle_logits,
                  revision_logits, input_lifecycle, batch, slots, lifecycles, revisions,
                  static_cast<float>(threshold), max_allocations, retired_index,
                  next_occupancy, lifecycle_indices, revision_indices, input_lifecycle_indices,
                  input_lifecycle_present, live_slots, live_dtype, live_occupancy};
  const int rc = check_rollout(p, threshold, true);
  if (rc != CID_OK || batch == 0 || slots == 0) return rc;
  return launch_rollout(p, stream);
}

extern "C" int cid_live_slot_occupancy(cid_dtype_t dtype, const void* occupancy,
                                       const void* lifecycle, int64_t rows, int64_t features,
                                       int64_t retired_index, void* out, void* stream) {
  if (!is_float_dtype(dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (lifecycle && (retired_index < 0 || retired_index >= features))
    return CID_ERR_INVALID_ARGUMENT;  // ops.cpp:31-33
  int64_t count = 0;
  if (rows < 0 || rows > kMaxRows ||
      (lifecycle && (!count_ok(rows, features, &count) || count > kMaxCount)))
    return CID_ERR_INVALID_ARGUMENT;
  const size_t es = static_cast<size_t>(dtype_size(dtype));
  if (misaligned({{occupancy, es}, {lifecycle, es}, {out, es}})) return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({occupancy, out})) return CID_ERR_INVALID_ARGUMENT;
  LiveParams p{dtype, occupancy, lifecycle, rows, features, retired_index, out};
  const int threads = 256;
  int64_t blocks = (rows + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  return launch_pdl(live_kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0,
                    as_stream(stream), p);
}
