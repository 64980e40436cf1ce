// Display refinement policy on the device: one CTA per display row.
//
// Semantics are those of the reference CPU policy
// (csrc/refine.cpp:93-429 of fwerkor/cid-engine v1.1.0), which there runs on
// host copies of the statistics (a device->host->device round trip every
// decode step).  Per row:
//   1. first EOS position;
//   2. if an EOS exists and revision_fraction != 0, the structural
//      insert/delete search (refine.cpp:93-218): every changed start proposes
//      at most one insertion and one deletion; the best candidate by
//      (anchor, gain, -|growth|, start) — the earlier of two exactly equal
//      candidates, i.e. the insertion — is spliced in and the row is done;
//   3. otherwise reveal the top ceil(n_masked * reveal) masked positions by
//      confidence, revise the top min(#candidates, ceil(n_visible * revision))
//      visible positions by gain (float32 margin), and expand the EOS;
//   4. mask every position after the first EOS of the result.
// "Top-k by key, descending, stable" is computed as a radix select of the
// k-th largest key (keys mapped to order-preserving integers, 8 bits per pass)
// followed by an index-ordered scan of the keys equal to it, which selects
// exactly the positions std::stable_sort(>) would put first.
#include <climits>
#include <cmath>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kT = 256;
constexpr int kWarps = kT / 32;
constexpr int64_t kSmemLimit = 160 * 1024;

__device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t imax(int64_t a, int64_t b) { return a > b ? a : b; }

struct RefineParams {
  const int64_t* ids;
  const float* conf;
  const int64_t* pred;
  const float* cur;
  int64_t tokens;
  int64_t mask_id;
  int64_t eos_id;
  int has_eos;
  double reveal;
  double revision;
  double margin;
  int64_t* out;
  int use_smem;
};

// Order-preserving map float -> uint32 (larger float, larger key).  -0 and
// +0 share a key (they compare equal); NaN keys sort lowest.
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0u;
  if (f == 0.0f) return 0x80000000u;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct Scratch {
  int64_t i64[kWarps];
  uint32_t u32[kWarps];
  int hist[256];       // radix-select histogram
  uint32_t sel_digit;  // radix-select result of the current pass
  int64_t sel_above;
};

__device__ __forceinline__ int64_t block_sum(int64_t v, Scratch& s) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_down_sync(0xffffffffu, v, d);
  if ((threadIdx.x & 31) == 0) s.i64[threadIdx.x >> 5] = v;
  __syncthreads();
  int64_t r = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) r += s.i64[w];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int64_t block_min(int64_t v, Scratch& s) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = min(v, __shfl_down_sync(0xffffffffu, v, d));
  if ((threadIdx.x & 31) == 0) s.i64[threadIdx.x >> 5] = v;
  __syncthreads();
  int64_t r = s.i64[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) r = min(r, s.i64[w]);
  __syncthreads();
  return r;
}

// Exclusive prefix sum over threads (in thread order) of v.
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, Scratch& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) s.i64[warp] = inc;
  __syncthreads();
  int64_t base = 0;
  for (int w = 0; w < warp; ++w) base += s.i64[w];
  __syncthreads();
  return base + inc - v;
}

// Selects the k positions of [0, L) with elig(i) that come first in a stable
// descending sort by key(i); calls take(i) for each (from any thread).
// The k-th largest order key T is found by a 4-pass radix select (8 bits per
// pass, most significant first, shared-memory histogram); every position with
// a key above T is taken, and of those equal to T the first `need` in index
// order.
template <typename Elig, typename Key, typename Take>
__device__ void select_top_k(int64_t L, int64_t k, Elig elig, Key key, Take take, Scratch& s) {
  if (k <= 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t prefix = 0u;  // decided high bits of T
  int64_t above = 0;     // eligible keys strictly above the prefix range
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = threadIdx.x; i < 256; i += kT) s.hist[i] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < L; i += kT) {
      if (!elig(i)) continue;
      const uint32_t u = order_key(key(i));
      if ((u & hi_mask) == prefix) atomicAdd(&s.hist[(u >> shift) & 255u], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns digits 255-8l .. 248-8l (descending); find the digit where
      // the count from the top first reaches k
      int h[8];
      int sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        h[j] = s.hist[255 - (lane * 8 + j)];
        sum += h[j];
      }
      int incl = sum;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += o;
      }
      int64_t running = above + (incl - sum);
      const bool mine = running < k && running + sum >= k;
      if (mine) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (running + h[j] >= k) {
            s.sel_digit = static_cast<uint32_t>(255 - (lane * 8 + j));
            s.sel_above = running;
            break;
          }
          running += h[j];
        }
      }
    }
    __syncthreads();
    prefix |= s.sel_digit << shift;
    above = s.sel_above;
    __syncthreads();
  }
  const uint32_t T = prefix;
  const int64_t need = k - above;  // ties at T to take, by index
  for (int64_t i = threadIdx.x; i < L; i += kT)
    if (elig(i) && order_key(key(i)) > T) take(i);
  // ties: contiguous ownership so that the scan follows index order
  const int64_t per = (L + kT - 1) / kT;
  const int64_t lo = min(L, per * threadIdx.x), hi = min(L, lo + per);
  int64_t mine = 0;
  for (int64_t i = lo; i < hi; ++i) mine += (elig(i) && order_key(key(i)) == T) ? 1 : 0;
  int64_t rank = block_exclusive_scan(mine, s);
  for (int64_t i = lo; i < hi && rank < need; ++i)
    if (elig(i) && order_key(key(i)) == T) {
      take(i);
      ++rank;
    }
}

struct Candidate {
  int64_t anchor;
  float gain;
  int64_t neg_growth;
  int64_t start;
  int kind;  // 1 = insertion (found first for a start), 0 = deletion
  int64_t del;
  int64_t ins;
  int valid;
};

// Strict order of refine.cpp:30-43 extended by `kind` so that, for one
// start, an equal deletion does not displace the insertion found before it.
__device__ __forceinline__ bool cand_better(const Candidate& a, const Candidate& b) {
  if (!b.valid) return a.valid;
  if (!a.valid) return false;
  if (a.anchor != b.anchor) return a.anchor > b.anchor;
  if (a.gain != b.gain) return a.gain > b.gain;
  if (a.neg_growth != b.neg_growth) return a.neg_growth > b.neg_growth;
  if (a.start != b.start) return a.start > b.start;
  return a.kind > b.kind;
}

__global__ void __launch_bounds__(kT) refine_kernel(RefineParams p) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ Scratch scratch;
  __shared__ Candidate cand_smem[kWarps];
  __shared__ Candidate best_smem;

  const int64_t L = p.tokens;
  const int64_t row = blockIdx.x;
  const int64_t base = row * L;
  const int64_t* g_tok = p.ids + base;
  const int64_t* g_pred = p.pred + base;
  const float* g_conf = p.conf + base;
  const float* g_cur = p.cur + base;
  int64_t* g_out = p.out + base;

  // Stage the row (tok, pred, res, conf, gain) in shared memory when it fits.
  const int64_t* tok;
  const int64_t* pred;
  const float* conf;
  float* gainbuf = nullptr;
  int64_t* res;
  if (p.use_smem) {
    int64_t* s_tok = reinterpret_cast<int64_t*>(dyn);
    int64_t* s_pred = s_tok + L;
    int64_t* s_res = s_pred + L;
    float* s_conf = reinterpret_cast<float*>(s_res + L);
    float* s_gain = s_conf + L;
    for (int64_t i = threadIdx.x; i < L; i += kT) {
      const int64_t t = g_tok[i];
      const float c = g_conf[i];
      s_tok[i] = t;
      s_res[i] = t;
      s_pred[i] = g_pred[i];
      s_conf[i] = c;
      s_gain[i] = __fsub_rn(c, g_cur[i]);  // refine.cpp:277
    }
    tok = s_tok;
    pred = s_pred;
    res = s_res;
    conf = s_conf;
    gainbuf = s_gain;
  } else {
    for (int64_t i = threadIdx.x; i < L; i += kT) g_out[i] = g_tok[i];
    tok = g_tok;
    pred = g_pred;
    res = g_out;
    conf = g_conf;
  }
  __syncthreads();
  auto gain = [&](int64_t i) -> float {
    return gainbuf ? gainbuf[i] : __fsub_rn(g_conf[i], g_cur[i]);
  };

  const int64_t mask = p.mask_id, eos = p.eos_id;
  // 1. first EOS (refine.cpp:280-288)
  int64_t eos_pos = -1;
  if (p.has_eos) {
    int64_t first = LLONG_MAX;
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (tok[i] == eos) { first = i; break; }
    first = block_min(first, scratch);
    eos_pos = first == LLONG_MAX ? -1 : first;
  }

  bool structural_done = false;
  // 2. structural edit (refine.cpp:290-319, 93-218)
  if (eos_pos > 0 && p.revision != 0.0) {
    int64_t budget = static_cast<int64_t>(ceil(static_cast<double>(eos_pos) * p.revision));
    budget = imax(1, imin(32, budget));
    const int64_t alen = eos_pos + 1;  // active = tok[0, eos_pos]
    Candidate best{};
    best.valid = 0;
    for (int64_t s = threadIdx.x; s < eos_pos; s += kT) {
      const float gs = gain(s);
      if (pred[s] == tok[s] || static_cast<double>(gs) < p.margin) continue;
      // insertion: nearest q in (s, s+budget] with pred[q, q+klen) == tok[s, s+klen)
      const int64_t klen = imin(3, alen - s);
      const int64_t qlast = imin(s + budget, L - klen);
      for (int64_t q = s + 1; q <= qlast; ++q) {
        bool eq = true;
        for (int64_t k = 0; k < klen && eq; ++k) eq = pred[q + k] == tok[s + k];
        if (!eq) continue;
        bool ok = true;
        for (int64_t k = s; k < q && ok; ++k) ok = pred[k] != mask && pred[k] != eos;
        if (ok) {
          int64_t anchor = 0;
          while (q + anchor < L && s + anchor < alen && pred[q + anchor] == tok[s + anchor]) ++anchor;
          const int64_t growth = q - s;
          if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 + growth <= L) {
            Candidate c{anchor, gs, -growth, s, 1, 0, growth, 1};
            if (cand_better(c, best)) best = c;
          }
        }
        break;  // only the nearest match is considered
      }
      // deletion: nearest r in (s, min(eos-1, s+budget)] with tok[r, r+dlen) == pred[s, s+dlen)
      const int64_t dlen = imin(3, L - s);
      if (dlen < 2) continue;
      const int64_t rlast = imin(imin(eos_pos - 1, s + budget), alen - dlen);
      for (int64_t r = s + 1; r <= rlast; ++r) {
        bool eq = true;
        for (int64_t k = 0; k < dlen && eq; ++k) eq = tok[r + k] == pred[s + k];
        if (!eq) continue;
        int64_t anchor = 0;
        while (s + anchor < L && r + anchor < alen && pred[s + anchor] == tok[r + anchor]) ++anchor;
        const int64_t del = r - s;
        if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 - del <= L) {
          Candidate c{anchor, gs, -del, s, 0, del, 0, 1};
          if (cand_better(c, best)) best = c;
        }
        break;
      }
    }
    // block arg-best
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int d = 1; d < 32; d <<= 1) {
      Candidate o;
      o.anchor = __shfl_xor_sync(0xffffffffu, best.anchor, d);
      o.gain = __shfl_xor_sync(0xffffffffu, best.gain, d);
      o.neg_growth = __shfl_xor_sync(0xffffffffu, best.neg_growth, d);
      o.start = __shfl_xor_sync(0xffffffffu, best.start, d);
      o.kind = __shfl_xor_sync(0xffffffffu, best.kind, d);
      o.del = __shfl_xor_sync(0xffffffffu, best.del, d);
      o.ins = __shfl_xor_sync(0xffffffffu, best.ins, d);
      o.valid = __shfl_xor_sync(0xffffffffu, best.valid, d);
      if (cand_better(o, best)) best = o;
    }
    if (lane == 0) cand_smem[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      Candidate b = cand_smem[0];
      for (int w = 1; w < kWarps; ++w)
        if (cand_better(cand_smem[w], b)) b = cand_smem[w];
      best_smem = b;
    }
    __syncthreads();
    const Candidate b = best_smem;
    if (b.valid) {
      // splice: tok[0, s) + pred[s, s+ins) + tok[s+del, eos] + mask fill
      for (int64_t i = threadIdx.x; i < L; i += kT) {
        int64_t v;
        if (i < b.start) v = tok[i];
        else if (i < b.start + b.ins) v = pred[i];
        else {
          const int64_t j = i - b.ins + b.del;
          v = j <= eos_pos ? tok[j] : mask;
        }
        res[i] = v;  // each thread writes only its own positions
      }
      structural_done = true;
    }
    __syncthreads();
  }

  if (!structural_done) {
    const int64_t stop = eos_pos >= 0 ? eos_pos : L;  // refine.cpp:321
    // 3a. reveal (refine.cpp:322-342)
    int64_t nm = 0;
    for (int64_t i = threadIdx.x; i < stop; i += kT) nm += tok[i] == mask ? 1 : 0;
    nm = block_sum(nm, scratch);
    if (nm > 0 && p.reveal != 0.0) {
      const int64_t k = static_cast<int64_t>(ceil(static_cast<double>(nm) * p.reveal));
      select_top_k(
          stop, k, [&](int64_t i) { return tok[i] == mask; }, [&](int64_t i) { return conf[i]; },
          [&](int64_t i) { res[i] = pred[i]; }, scratch);
    }
    if (p.revision != 0.0) {
      // 3b. revision (refine.cpp:344-379); the margin is compared in float32
      const float margin_f = static_cast<float>(p.margin);
      const int64_t visible = stop - nm;
      auto is_cand = [&](int64_t i) {
        return tok[i] != mask && pred[i] != tok[i] && gain(i) >= margin_f;
      };
      int64_t nc = 0;
      for (int64_t i = threadIdx.x; i < stop; i += kT) nc += is_cand(i) ? 1 : 0;
      nc = block_sum(nc, scratch);
      if (nc > 0) {
        int64_t k = static_cast<int64_t>(ceil(static_cast<double>(visible) * p.revision));
        k = min(k, nc);
        select_top_k(stop, k, is_cand, gain, [&](int64_t i) { res[i] = pred[i]; }, scratch);
      }
      // 3c. EOS expansion (refine.cpp:381-406), double margin
      if (eos_pos >= 0 && eos_pos + 1 < L && pred[eos_pos] != eos &&
          static_cast<double>(gain(eos_pos)) >= p.margin) {
        const int64_t basec = imax(1, eos_pos + 1);
        const int64_t budget =
            imax(1, static_cast<int64_t>(ceil(static_cast<double>(basec) * p.reveal)));
        int64_t new_eos = imin(L - 1, eos_pos + budget);
        int64_t first = LLONG_MAX;
        for (int64_t t = eos_pos + 1 + threadIdx.x; t <= new_eos; t += kT)
          if (pred[t] == eos) { first = t; break; }
        first = block_min(first, scratch);
        if (first != LLONG_MAX) new_eos = first;
        for (int64_t t = eos_pos + threadIdx.x; t < new_eos; t += kT) res[t] = pred[t];
        if (threadIdx.x == 0) res[new_eos] = eos;
      }
    }
    __syncthreads();
  }

  // 4. mask everything after the first EOS of the result (refine.cpp:410-423)
  int64_t cut = LLONG_MAX;
  if (p.has_eos) {
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (res[i] == eos) { cut = i; break; }
    cut = block_min(cut, scratch);
  }
  if (p.use_smem) {
    for (int64_t i = threadIdx.x; i < L; i += kT) g_out[i] = i > cut ? mask : res[i];
  } else {
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (i > cut) g_out[i] = mask;
  }
}

}  // namespace
}  // namespace cid

using namespace cid;

extern "C" int cid_refine_display(const int64_t* token_ids, const float* confidence,
                                  const int64_t* predicted, const float* current_confidence,
                                  int64_t batch, int64_t tokens, int64_t mask_token_id,
                                  int has_eos, int64_t eos_token_id, double reveal_fraction,
                                  double revision_fraction, double revision_margin,
                                  int64_t* out, void* stream) {
  // refine.cpp:240-244
  if (!(reveal_fraction >= 0.0 && reveal_fraction <= 1.0)) return CID_ERR_INVALID_ARGUMENT;
  if (!(revision_fraction >= 0.0 && revision_fraction <= 1.0)) return CID_ERR_INVALID_ARGUMENT;
  if (!(revision_margin >= 0.0)) return CID_ERR_INVALID_ARGUMENT;
  if (batch < 0 || tokens < 0 || batch > INT_MAX) return CID_ERR_INVALID_ARGUMENT;
  if (batch == 0 || tokens == 0) return CID_OK;
  if (!token_ids || !confidence || !predicted || !current_confidence || !out)
    return CID_ERR_INVALID_ARGUMENT;
  RefineParams p;
  p.ids = token_ids;
  p.conf = confidence;
  p.pred = predicted;
  p.cur = current_confidence;
  p.tokens = tokens;
  p.mask_id = mask_token_id;
  p.eos_id = eos_token_id;
  p.has_eos = has_eos;
  p.reveal = reveal_fraction;
  p.revision = revision_fraction;
  p.margin = revision_margin;
  p.out = out;
  const int64_t smem = tokens * (3 * 8 + 2 * 4);
  p.use_smem = smem <= kSmemLimit;
  const size_t dyn = p.use_smem ? static_cast<size_t>(smem) : 0;
  if (dyn > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(
        refine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  refine_kernel<<<static_cast<unsigned>(batch), kT, dyn, as_stream(stream)>>>(p);
  return launch_result();
}
