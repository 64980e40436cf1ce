// Display refinement policy on the device: one warp per display row for
// rows of up to 128 positions (refine_warp_kernel, no block barriers), one
// CTA per row for longer rows (refine_kernel).
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

// Block size: 256 threads, or 512 for long rows when the batch leaves most
// SMs idle (one CTA per row is then latency-bound; twice the warps hide more
// of it, and 512 threads still leave 128 registers per thread).
constexpr int kMaxWarps = 512 / 32;
constexpr int64_t kSmemLimit = 200 * 1024;

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
  int64_t i64[kMaxWarps];
  int hist[2][2][256];       // radix-select histograms [buffer][class][digit]
  uint32_t sel_digit[2][2];  // radix-select result per [buffer][class]
  int64_t sel_above[2][2];
};

template <int kT>
__device__ __forceinline__ int64_t block_sum(int64_t v, Scratch& s) {
  constexpr int kWarps = kT / 32;
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

template <int kT>
__device__ __forceinline__ int64_t block_min(int64_t v, Scratch& s) {
  constexpr int kWarps = kT / 32;
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
template <int kT>
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

// Two independent stable top-k selections over [0, L) in one radix pass
// sequence.  Position i belongs to class cls(i) (0, 1, or -1 for neither)
// with order key key(i, c) (order_key of its value); class c takes the
// k[c] positions that come first in a stable descending sort of its members
// by key, i.e. std::stable_sort(>) order.  The k[c]-th largest order key
// T[c] is found by a 4-pass radix select (8 bits per pass, most significant
// first, shared-memory histograms, double-buffered so a pass needs two
// barriers); every member with a key
// above T[c] is taken, and of those equal to T[c] the first `need` in index
// order.  take(i, c) is called once per selected position, from any thread.
template <int kT, typename Cls, typename Key, typename Take>
__device__ void select_top_k2(int64_t L, int64_t k0, int64_t k1, Cls cls, Key key, Take take,
                              Scratch& s) {
  if (k0 <= 0 && k1 <= 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // per-class state in scalars (a runtime-indexed array would live on the stack)
  uint32_t prefix0 = 0u, prefix1 = 0u;  // decided high bits of T[c]
  int64_t above0 = 0, above1 = 0;       // members strictly above the prefix range
  auto k_of = [&](int c) { return c == 0 ? k0 : k1; };
  auto prefix_of = [&](int c) { return c == 0 ? prefix0 : prefix1; };
  for (int i = threadIdx.x; i < 2 * 2 * 256; i += kT) (&s.hist[0][0][0])[i] = 0;
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int buf = pass & 1;
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
    // warp-uniform trip count; lanes with the same (class, digit) add once
    // (keys of similar magnitude share their top byte, so per-lane atomics
    // would collide)
    for (int64_t i0 = threadIdx.x - lane; i0 < L; i0 += kT) {
      const int64_t i = i0 + lane;
      int bin = -1;
      if (i < L) {
        const int c = cls(i);
        if (c >= 0 && k_of(c) > 0) {
          const uint32_t u = key(i, c);
          if ((u & hi_mask) == prefix_of(c)) bin = c * 256 + static_cast<int>((u >> shift) & 255u);
        }
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && lane == __ffs(peers) - 1)
        atomicAdd(&s.hist[buf][bin >> 8][bin & 255], __popc(peers));
    }
    // the other buffer was last read before the previous pass's barrier
    for (int i = threadIdx.x; i < 2 * 256; i += kT) (&s.hist[buf ^ 1][0][0])[i] = 0;
    __syncthreads();
    if (warp < 2 && k_of(warp) > 0) {
      // warp c, lane l owns digits 255-8l .. 248-8l (descending) of class c;
      // find the digit where the count from the top first reaches k[c]
      const int c = warp;
      int h[8];
      int sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        h[j] = s.hist[buf][c][255 - (lane * 8 + j)];
        sum += h[j];
      }
      int incl = sum;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += o;
      }
      const int64_t kc = k_of(c);
      int64_t running = (c == 0 ? above0 : above1) + (incl - sum);
      if (running < kc && running + sum >= kc) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (running + h[j] >= kc) {
            s.sel_digit[buf][c] = static_cast<uint32_t>(255 - (lane * 8 + j));
            s.sel_above[buf][c] = running;
            break;
          }
          running += h[j];
        }
      }
    }
    __syncthreads();
    if (k0 > 0) {
      prefix0 |= s.sel_digit[buf][0] << shift;
      above0 = s.sel_above[buf][0];
    }
    if (k1 > 0) {
      prefix1 |= s.sel_digit[buf][1] << shift;
      above1 = s.sel_above[buf][1];
    }
  }
  for (int64_t i = threadIdx.x; i < L; i += kT) {
    const int c = cls(i);
    if (c >= 0 && k_of(c) > 0 && key(i, c) > prefix_of(c)) take(i, c);
  }
  // ties: contiguous ownership so that the scan follows index order; both
  // classes' tie counts (each < 2^31) packed in one scan
  const int64_t need0 = k0 - above0, need1 = k1 - above1;
  const int64_t per = (L + kT - 1) / kT;
  const int64_t lo = min(L, per * threadIdx.x), hi = min(L, lo + per);
  auto tie = [&](int64_t i) -> int {
    const int c = cls(i);
    return (c >= 0 && k_of(c) > 0 && key(i, c) == prefix_of(c)) ? c : -1;
  };
  int64_t mine = 0;
  for (int64_t i = lo; i < hi; ++i) {
    const int c = tie(i);
    if (c >= 0) mine += c == 0 ? 1 : (int64_t{1} << 32);
  }
  const int64_t before = block_exclusive_scan<kT>(mine, s);
  int64_t rank0 = before & 0xffffffffLL, rank1 = before >> 32;
  for (int64_t i = lo; i < hi && (rank0 < need0 || rank1 < need1); ++i) {
    const int c = tie(i);
    if (c == 0 && rank0 < need0) {
      take(i, 0);
      ++rank0;
    } else if (c == 1 && rank1 < need1) {
      take(i, 1);
      ++rank1;
    }
  }
}

// The same address with its provenance hidden from the compiler (generic
// loads): the structural search runs measurably faster through generic
// pointers than through known shared-memory ones.
template <typename P>
__device__ __forceinline__ P* opaque(P* p) {
  uint64_t r;
  asm volatile("mov.b64 %0, %1;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)));
  return reinterpret_cast<P*>(r);
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
// Length of the run i = 0, 1, ... with a[x0 + i] == b[y0 + i], x0 + i < xlim
// and y0 + i < ylim.  Eight positions' loads are issued before any compare
// and the first mismatch is found with one bit scan, so a run of n costs
// n / 8 dependent round trips (anchors on a shifted prediction run to the
// end of the row).
__device__ __forceinline__ int64_t match_run(const int64_t* a, int64_t x0, int64_t xlim,
                                             const int64_t* b, int64_t y0, int64_t ylim) {
  const int64_t n = imin(xlim - x0, ylim - y0);
  if (n <= 0) return 0;
  for (int64_t run = 0;; run += 8) {
    int64_t av[8], bv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool in = run + j < n;
      av[j] = in ? a[x0 + run + j] : 0;
      bv[j] = in ? b[y0 + run + j] : 1;  // past the end: a mismatch
    }
    unsigned miss = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) miss |= static_cast<unsigned>(av[j] != bv[j]) << j;
    if (miss) return run + (__ffs(miss) - 1);
  }
}

__device__ __forceinline__ bool cand_better(const Candidate& a, const Candidate& b) {
  if (!b.valid) return a.valid;
  if (!a.valid) return false;
  if (a.anchor != b.anchor) return a.anchor > b.anchor;
  if (a.gain != b.gain) return a.gain > b.gain;
  if (a.neg_growth != b.neg_growth) return a.neg_growth > b.neg_growth;
  if (a.start != b.start) return a.start > b.start;
  return a.kind > b.kind;
}

template <int kT, bool kStaged>
__global__ void __launch_bounds__(kT) refine_kernel(RefineParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int kWarps = kT / 32;
  constexpr int kChunk = 8;
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ Scratch scratch;
  __shared__ Candidate cand_smem[kMaxWarps];
  __shared__ Candidate best_smem;

  const int64_t L = p.tokens;
  const int64_t row = blockIdx.x;
  const int64_t base = row * L;
  const int64_t* g_tok = p.ids + base;
  const int64_t* g_pred = p.pred + base;
  const float* g_conf = p.conf + base;
  const float* g_cur = p.cur + base;
  int64_t* g_out = p.out + base;

  // Stage the row (tok, pred, res, conf, gain, and each position's class and
  // order key for the selections) in shared memory when it fits.
  const int64_t* tok;
  const int64_t* pred;
  const float* conf;
  float* gainbuf = nullptr;
  int64_t* res;
  uint32_t* okeys = nullptr;
  int8_t* classes = nullptr;
  const float margin_sel = static_cast<float>(p.margin);
  const bool revise_sel = p.revision != 0.0;
  if constexpr (kStaged) {
    int64_t* s_tok = reinterpret_cast<int64_t*>(dyn);
    int64_t* s_pred = s_tok + L;
    int64_t* s_res = s_pred + L;
    float* s_conf = reinterpret_cast<float*>(s_res + L);
    float* s_gain = s_conf + L;
    uint32_t* s_key = reinterpret_cast<uint32_t*>(s_gain + L);
    int8_t* s_cls = reinterpret_cast<int8_t*>(s_key + L);
    // kStage iterations' loads in flight per thread before any store: one
    // HBM latency per kStage * kT positions instead of per kT
    constexpr int kStage = 4;
    for (int64_t i0 = threadIdx.x; i0 < L; i0 += kT * kStage) {
      int64_t t[kStage], pr[kStage];
      float c[kStage], u[kStage];
#pragma unroll
      for (int j = 0; j < kStage; ++j) {
        const int64_t i = i0 + static_cast<int64_t>(j) * kT;
        if (i < L) {
          t[j] = __ldg(g_tok + i);
          pr[j] = __ldg(g_pred + i);
          c[j] = __ldg(g_conf + i);
          u[j] = __ldg(g_cur + i);
        }
      }
#pragma unroll
      for (int j = 0; j < kStage; ++j) {
        const int64_t i = i0 + static_cast<int64_t>(j) * kT;
        if (i < L) {
          s_tok[i] = t[j];
          s_res[i] = t[j];
          s_pred[i] = pr[j];
          s_conf[i] = c[j];
          const float gj = __fsub_rn(c[j], u[j]);  // refine.cpp:277
          s_gain[i] = gj;
          // class and key as the selections of step 3 use them
          const int cj = t[j] == p.mask_id ? 0
                         : (revise_sel && pr[j] != t[j] && gj >= margin_sel) ? 1 : -1;
          s_cls[i] = static_cast<int8_t>(cj);
          s_key[i] = order_key(cj == 0 ? c[j] : gj);
        }
      }
    }
    tok = s_tok;
    pred = s_pred;
    res = s_res;
    conf = s_conf;
    gainbuf = s_gain;
    okeys = s_key;
    classes = s_cls;
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
  const int64_t* const tok_ = tok;
  const int64_t* const pred_ = pred;
  int64_t* const res_ = res;

  const int64_t mask = p.mask_id, eos = p.eos_id;
  // 1. first EOS (refine.cpp:280-288)
  int64_t eos_pos = -1;
  if (p.has_eos) {
    int64_t first = LLONG_MAX;
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (tok[i] == eos) { first = i; break; }
    first = block_min<kT>(first, scratch);
    eos_pos = first == LLONG_MAX ? -1 : first;
  }

  bool structural_done = false;
  // 2. structural edit (refine.cpp:290-319, 93-218).  One start per thread;
  // the offsets 1..budget (<= 32) of a start are scanned in chunks of kChunk
  // with all loads of a chunk issued before any compare (the first-element
  // tests of the insertion and the deletion share the chunk), so a start
  // costs budget/kChunk shared-memory round trips instead of one per offset.
  if (eos_pos > 0 && p.revision != 0.0) {
    const int64_t* tok = opaque(tok_);
    const int64_t* pred = opaque(pred_);
    const float* gb = gainbuf ? opaque(gainbuf) : nullptr;
    auto gain = [&](int64_t i) -> float { return gb ? gb[i] : __fsub_rn(g_conf[i], g_cur[i]); };
    int64_t* res = opaque(res_);
    int64_t budget = static_cast<int64_t>(ceil(static_cast<double>(eos_pos) * p.revision));
    budget = imax(1, imin(32, budget));
    const int64_t alen = eos_pos + 1;  // active = tok[0, eos_pos]
    Candidate best{};
    best.valid = 0;
    for (int64_t s = threadIdx.x; s < eos_pos; s += kT) {
      const float gs = gain(s);
      const int64_t ts = tok[s], ps = pred[s];
      if (ps == ts || static_cast<double>(gs) < p.margin) continue;
      // insertion: nearest q in (s, qlast] with pred[q, q+klen) == tok[s, s+klen);
      // deletion: nearest r in (s, rlast] with tok[r, r+dlen) == pred[s, s+dlen)
      const int64_t klen = imin(3, alen - s);
      const int64_t qlast = imin(s + budget, L - klen);
      const int64_t dlen = imin(3, L - s);
      const int64_t rlast = dlen < 2 ? s : imin(imin(eos_pos - 1, s + budget), alen - dlen);
      int64_t q_hit = -1, r_hit = -1;
      for (int64_t o0 = 1; o0 <= budget && (q_hit < 0 || r_hit < 0); o0 += kChunk) {
        int64_t pv[kChunk], tv[kChunk];
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          const int64_t o = s + o0 + j;
          pv[j] = (q_hit < 0 && o <= qlast) ? pred[o] : ~ts;  // ~x never equals x
          tv[j] = (r_hit < 0 && o <= rlast) ? tok[o] : ~ps;
        }
        unsigned qm = 0, rm = 0;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          qm |= static_cast<unsigned>(pv[j] == ts) << j;
          rm |= static_cast<unsigned>(tv[j] == ps) << j;
        }
        while (qm && q_hit < 0) {  // full k-gram check of the first-element hits
          const int64_t q = s + o0 + (__ffs(qm) - 1);
          bool eq = true;
          for (int64_t k = 1; k < klen && eq; ++k) eq = pred[q + k] == tok[s + k];
          if (eq) q_hit = q;
          qm &= qm - 1;
        }
        while (rm && r_hit < 0) {
          const int64_t r = s + o0 + (__ffs(rm) - 1);
          bool eq = true;
          for (int64_t k = 1; k < dlen && eq; ++k) eq = tok[r + k] == pred[s + k];
          if (eq) r_hit = r;
          rm &= rm - 1;
        }
      }
      if (q_hit >= 0) {
        bool ok = true;  // pred[s, q) must hold neither mask nor EOS
        for (int64_t k = s; k < q_hit && ok; ++k) ok = pred[k] != mask && pred[k] != eos;
        if (ok) {
          const int64_t anchor = match_run(pred, q_hit, L, tok, s, alen);
          const int64_t growth = q_hit - s;
          if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 + growth <= L) {
            const Candidate c{anchor, gs, -growth, s, 1, 0, growth, 1};
            if (cand_better(c, best)) best = c;
          }
        }
      }
      if (r_hit >= 0) {
        const int64_t anchor = match_run(pred, s, L, tok, r_hit, alen);
        const int64_t del = r_hit - s;
        if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 - del <= L) {
          const Candidate c{anchor, gs, -del, s, 0, del, 0, 1};
          if (cand_better(c, best)) best = c;
        }
      }
    }
    // block arg-best: warp shuffles, then warp 0 over the warps' candidates
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
    if (warp == 0) {
      Candidate b{};
      b.valid = 0;
      if (lane < kWarps) b = cand_smem[lane];
      for (int d = 1; d < kWarps; d <<= 1) {
        Candidate o;
        o.anchor = __shfl_xor_sync(0xffffffffu, b.anchor, d);
        o.gain = __shfl_xor_sync(0xffffffffu, b.gain, d);
        o.neg_growth = __shfl_xor_sync(0xffffffffu, b.neg_growth, d);
        o.start = __shfl_xor_sync(0xffffffffu, b.start, d);
        o.kind = __shfl_xor_sync(0xffffffffu, b.kind, d);
        o.del = __shfl_xor_sync(0xffffffffu, b.del, d);
        o.ins = __shfl_xor_sync(0xffffffffu, b.ins, d);
        o.valid = __shfl_xor_sync(0xffffffffu, b.valid, d);
        if (cand_better(o, b)) b = o;
      }
      if (lane == 0) best_smem = b;
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
    // 3a/3b. reveal (refine.cpp:322-342) and revision (refine.cpp:344-379):
    // disjoint member sets (masked / visible positions) and independent
    // counts, so both selections share one radix pass sequence.  The
    // revision margin is compared in float32.
    const float margin_f = static_cast<float>(p.margin);
    const bool revise = p.revision != 0.0;
    auto cls = [&](int64_t i) -> int {
      if constexpr (kStaged) return classes[i];
      const int64_t t = tok[i];
      if (t == mask) return 0;
      return (revise && pred[i] != t && gain(i) >= margin_f) ? 1 : -1;
    };
    int64_t counts = 0;  // masked | candidates << 32 (each < 2^31)
    for (int64_t i = threadIdx.x; i < stop; i += kT) {
      const int c = cls(i);
      counts += c == 0 ? 1 : c == 1 ? (int64_t{1} << 32) : 0;
    }
    counts = block_sum<kT>(counts, scratch);
    const int64_t nm = counts & 0xffffffffLL, nc = counts >> 32;
    int64_t k0 = 0, k1 = 0;
    if (nm > 0 && p.reveal != 0.0)
      k0 = static_cast<int64_t>(ceil(static_cast<double>(nm) * p.reveal));
    if (revise && nc > 0)
      k1 = imin(static_cast<int64_t>(ceil(static_cast<double>(stop - nm) * p.revision)), nc);
    select_top_k2<kT>(
        stop, k0, k1, cls,
        [&](int64_t i, int c) -> uint32_t {
          if constexpr (kStaged) return okeys[i];
          return order_key(c == 0 ? conf[i] : gain(i));
        },
        [&](int64_t i, int) { res[i] = pred[i]; }, scratch);
    // 3c. EOS expansion (refine.cpp:381-406), double margin; writes only
    // positions >= eos_pos, disjoint from the selections above
    if (revise && eos_pos >= 0 && eos_pos + 1 < L && pred[eos_pos] != eos &&
        static_cast<double>(gain(eos_pos)) >= p.margin) {
      const int64_t basec = imax(1, eos_pos + 1);
      const int64_t ebudget =
          imax(1, static_cast<int64_t>(ceil(static_cast<double>(basec) * p.reveal)));
      int64_t new_eos = imin(L - 1, eos_pos + ebudget);
      int64_t first = LLONG_MAX;
      for (int64_t t = eos_pos + 1 + threadIdx.x; t <= new_eos; t += kT)
        if (pred[t] == eos) { first = t; break; }
      first = block_min<kT>(first, scratch);
      if (first != LLONG_MAX) new_eos = first;
      for (int64_t t = eos_pos + threadIdx.x; t < new_eos; t += kT) res[t] = pred[t];
      if (threadIdx.x == 0) res[new_eos] = eos;
    }
    __syncthreads();
  }

  // 4. mask everything after the first EOS of the result (refine.cpp:410-423)
  int64_t cut = LLONG_MAX;
  if (p.has_eos) {
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (res[i] == eos) { cut = i; break; }
    cut = block_min<kT>(cut, scratch);
  }
  if (p.use_smem) {
    for (int64_t i = threadIdx.x; i < L; i += kT) g_out[i] = i > cut ? mask : res[i];
  } else {
    for (int64_t i = threadIdx.x; i < L; i += kT)
      if (i > cut) g_out[i] = mask;
  }
}


// ---------------------------------------------------------------------------
// Warp-per-row refinement for short rows (tokens <= kWarpRowMax): the same
// policy as refine_kernel with no block barrier in it.  A warp stages its row
// in its own slice of shared memory, finds the first EOS with ballots, runs
// the structural search with one start per lane and a shuffle arg-best, and
// selects the reveal / revision top-k by counting, for each member, the
// members of its class ahead of it in stable descending order: a member's
// composite key is (order key << 32) | ~index, so "ahead" is one 64-bit
// compare and the k members with rank < k are exactly those
// std::stable_sort(>) puts first.  Decode steps refine few short rows, where
// the CTA kernel's dozen barriers were most of the step's refinement time.
// ---------------------------------------------------------------------------
constexpr int kWarpPos = 4;                      // positions per lane
constexpr int kWarpRowMax = 32 * kWarpPos;       // 128
constexpr int kWarpRowsPerCta = 4;

struct WarpRow {
  int64_t tok[kWarpRowMax];
  int64_t pred[kWarpRowMax];
  int64_t res[kWarpRowMax];
  uint64_t key[kWarpRowMax];  // composite selection key of a member
  float gain[kWarpRowMax];
  int8_t cls[kWarpRowMax];    // 0 reveal member, 1 revision member, -1 neither
};

// Warp-uniform first index in [lo, hi) where pred == value, -1 if none.
__device__ __forceinline__ int warp_first_pred(const WarpRow& w, int lo, int hi, int64_t value) {
  const int lane = threadIdx.x & 31;
  for (int b = lo; b < hi; b += 32) {
    const int i = b + lane;
    const unsigned bits = __ballot_sync(0xffffffffu, i < hi && w.pred[i] == value);
    if (bits) return b + __ffs(bits) - 1;
  }
  return -1;
}

__device__ __forceinline__ Candidate shfl_cand(const Candidate& c, int d) {
  Candidate o;
  o.anchor = __shfl_xor_sync(0xffffffffu, c.anchor, d);
  o.gain = __shfl_xor_sync(0xffffffffu, c.gain, d);
  o.neg_growth = __shfl_xor_sync(0xffffffffu, c.neg_growth, d);
  o.start = __shfl_xor_sync(0xffffffffu, c.start, d);
  o.kind = __shfl_xor_sync(0xffffffffu, c.kind, d);
  o.del = __shfl_xor_sync(0xffffffffu, c.del, d);
  o.ins = __shfl_xor_sync(0xffffffffu, c.ins, d);
  o.valid = __shfl_xor_sync(0xffffffffu, c.valid, d);
  return o;
}

__global__ void __launch_bounds__(32 * kWarpRowsPerCta) refine_warp_kernel(RefineParams p,
                                                                           int64_t batch) {
  pdl_wait();
  pdl_trigger();
  __shared__ WarpRow rows[kWarpRowsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpRowsPerCta + warp;
  if (row >= batch) return;  // warp-uniform; the kernel has no block barrier
  WarpRow& w = rows[warp];
  const int L = static_cast<int>(p.tokens);
  const int64_t base = row * p.tokens;
  const int64_t mask = p.mask_id, eos = p.eos_id;

  // stage the row: every lane's loads issued before any store
  int64_t t[kWarpPos], pr[kWarpPos];
  float cf[kWarpPos], cu[kWarpPos];
#pragma unroll
  for (int j = 0; j < kWarpPos; ++j) {
    const int i = lane + 32 * j;
    if (i < L) {
      t[j] = __ldg(p.ids + base + i);
      pr[j] = __ldg(p.pred + base + i);
      cf[j] = __ldg(p.conf + base + i);
      cu[j] = __ldg(p.cur + base + i);
    }
  }
#pragma unroll
  for (int j = 0; j < kWarpPos; ++j) {
    const int i = lane + 32 * j;
    if (i < L) {
      w.tok[i] = t[j];
      w.res[i] = t[j];
      w.pred[i] = pr[j];
      w.gain[i] = __fsub_rn(cf[j], cu[j]);  // refine.cpp:277
    }
  }
  __syncwarp();

  // 1. first EOS (refine.cpp:280-288)
  int eos_pos = -1;
  if (p.has_eos) {
#pragma unroll
    for (int j = 0; j < kWarpPos; ++j) {
      const int i = lane + 32 * j;
      const unsigned bits = __ballot_sync(0xffffffffu, i < L && t[j] == eos);
      if (bits) {
        eos_pos = 32 * j + __ffs(bits) - 1;
        break;
      }
    }
  }
  bool structural_done = false;
  // 2. structural edit (refine.cpp:290-319, 93-218): one start per lane, the
  // offsets scanned as in refine_kernel, the best candidate by butterfly
  if (eos_pos > 0 && p.revision != 0.0) {
    constexpr int kChunk = 8;
    int64_t budget = static_cast<int64_t>(ceil(static_cast<double>(eos_pos) * p.revision));
    budget = imax(1, imin(32, budget));
    const int64_t alen = eos_pos + 1;  // active = tok[0, eos_pos]
    const int64_t Ll = L;
    Candidate best{};
    best.valid = 0;
    for (int64_t s = lane; s < eos_pos; s += 32) {
      const float gs = w.gain[s];
      const int64_t ts = w.tok[s], ps = w.pred[s];
      if (ps == ts || static_cast<double>(gs) < p.margin) continue;
      const int64_t klen = imin(3, alen - s);
      const int64_t qlast = imin(s + budget, Ll - klen);
      const int64_t dlen = imin(3, Ll - s);
      const int64_t rlast = dlen < 2 ? s : imin(imin(eos_pos - 1, s + budget), alen - dlen);
      int64_t q_hit = -1, r_hit = -1;
      for (int64_t o0 = 1; o0 <= budget && (q_hit < 0 || r_hit < 0); o0 += kChunk) {
        int64_t pv[kChunk], tv[kChunk];
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          const int64_t o = s + o0 + j;
          pv[j] = (q_hit < 0 && o <= qlast) ? w.pred[o] : ~ts;  // ~x never equals x
          tv[j] = (r_hit < 0 && o <= rlast) ? w.tok[o] : ~ps;
        }
        unsigned qm = 0, rm = 0;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          qm |= static_cast<unsigned>(pv[j] == ts) << j;
          rm |= static_cast<unsigned>(tv[j] == ps) << j;
        }
        while (qm && q_hit < 0) {
          const int64_t q = s + o0 + (__ffs(qm) - 1);
          bool eq = true;
          for (int64_t k = 1; k < klen && eq; ++k) eq = w.pred[q + k] == w.tok[s + k];
          if (eq) q_hit = q;
          qm &= qm - 1;
        }
        while (rm && r_hit < 0) {
          const int64_t r = s + o0 + (__ffs(rm) - 1);
          bool eq = true;
          for (int64_t k = 1; k < dlen && eq; ++k) eq = w.tok[r + k] == w.pred[s + k];
          if (eq) r_hit = r;
          rm &= rm - 1;
        }
      }
      if (q_hit >= 0) {
        bool ok = true;  // pred[s, q) must hold neither mask nor EOS
        for (int64_t k = s; k < q_hit && ok; ++k) ok = w.pred[k] != mask && w.pred[k] != eos;
        if (ok) {
          const int64_t anchor = match_run(w.pred, q_hit, Ll, w.tok, s, alen);
          const int64_t growth = q_hit - s;
          if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 + growth <= Ll) {
            const Candidate c{anchor, gs, -growth, s, 1, 0, growth, 1};
            if (cand_better(c, best)) best = c;
          }
        }
      }
      if (r_hit >= 0) {
        const int64_t anchor = match_run(w.pred, s, Ll, w.tok, r_hit, alen);
        const int64_t del = r_hit - s;
        if (anchor >= 2 && static_cast<double>(gs) >= p.margin && eos_pos + 1 - del <= Ll) {
          const Candidate c{anchor, gs, -del, s, 0, del, 0, 1};
          if (cand_better(c, best)) best = c;
        }
      }
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const Candidate o = shfl_cand(best, d);
      if (cand_better(o, best)) best = o;
    }
    if (best.valid) {
      // splice: tok[0, s) + pred[s, s+ins) + tok[s+del, eos] + mask fill
      for (int64_t i = lane; i < Ll; i += 32) {
        int64_t v;
        if (i < best.start) v = w.tok[i];
        else if (i < best.start + best.ins) v = w.pred[i];
        else {
          const int64_t j = i - best.ins + best.del;
          v = j <= eos_pos ? w.tok[j] : mask;
        }
        w.res[i] = v;
      }
      structural_done = true;
    }
    __syncwarp();
  }

  if (!structural_done) {
    const int stop = eos_pos >= 0 ? eos_pos : L;  // refine.cpp:321
    const float margin_f = static_cast<float>(p.margin);
    const bool revise = p.revision != 0.0;
    // 3a/3b. reveal (refine.cpp:322-342) and revision (refine.cpp:344-379)
    int c_of[kWarpPos];
    unsigned nm = 0, nc = 0;
#pragma unroll
    for (int j = 0; j < kWarpPos; ++j) {
      const int i = lane + 32 * j;
      int c = -1;
      if (i < stop) {
        if (t[j] == mask) c = 0;
        else if (revise && pr[j] != t[j] && w.gain[i] >= margin_f) c = 1;
      }
      c_of[j] = c;
      nm += c == 0;
      nc += c == 1;
    }
    nm = __reduce_add_sync(0xffffffffu, nm);
    nc = __reduce_add_sync(0xffffffffu, nc);
    int64_t k0 = 0, k1 = 0;
    if (nm > 0 && p.reveal != 0.0)
      k0 = static_cast<int64_t>(ceil(static_cast<double>(nm) * p.reveal));
    if (revise && nc > 0)
      k1 = imin(static_cast<int64_t>(ceil(static_cast<double>(stop - static_cast<int>(nm)) *
                                          p.revision)),
                static_cast<int64_t>(nc));
    uint64_t my_key[kWarpPos];
#pragma unroll
    for (int j = 0; j < kWarpPos; ++j) {
      const int i = lane + 32 * j;
      int c = c_of[j];
      if (c >= 0 && (c == 0 ? k0 : k1) <= 0) c = -1;
      c_of[j] = c;
      const uint32_t ok = c < 0 ? 0u : order_key(c == 0 ? cf[j] : w.gain[i]);
      my_key[j] = (static_cast<uint64_t>(ok) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
      if (i < stop) {
        w.key[i] = my_key[j];
        w.cls[i] = static_cast<int8_t>(c);
      }
    }
    __syncwarp();
    if (k0 > 0 || k1 > 0) {
      int rank[kWarpPos] = {};
      for (int jj = 0; jj < stop; ++jj) {
        const uint64_t kj = w.key[jj];  // same address in every lane: a broadcast
        const int cj = w.cls[jj];
#pragma unroll
        for (int j = 0; j < kWarpPos; ++j) rank[j] += (cj == c_of[j] && kj > my_key[j]) ? 1 : 0;
      }
#pragma unroll
      for (int j = 0; j < kWarpPos; ++j) {
        const int i = lane + 32 * j;
        if (c_of[j] >= 0 && rank[j] < (c_of[j] == 0 ? k0 : k1)) w.res[i] = pr[j];
      }
    }
    __syncwarp();
    // 3c. EOS expansion (refine.cpp:381-406), double margin; positions >= eos_pos
    if (revise && eos_pos >= 0 && eos_pos + 1 < L && w.pred[eos_pos] != eos &&
        static_cast<double>(w.gain[eos_pos]) >= p.margin) {
      const int64_t basec = imax(1, eos_pos + 1);
      const int64_t ebudget =
          imax(1, static_cast<int64_t>(ceil(static_cast<double>(basec) * p.reveal)));
      int new_eos = static_cast<int>(imin(L - 1, eos_pos + ebudget));
      const int first = warp_first_pred(w, eos_pos + 1, new_eos + 1, eos);
      if (first >= 0) new_eos = first;
      for (int i = eos_pos + lane; i < new_eos; i += 32) w.res[i] = w.pred[i];
      __syncwarp();
      if (lane == 0) w.res[new_eos] = eos;
    }
    __syncwarp();
  }

  // 4. mask everything after the first EOS of the result (refine.cpp:410-423)
  int cut = L;
  if (p.has_eos) {
    for (int b = 0; b < L; b += 32) {
      const int i = b + lane;
      const unsigned bits = __ballot_sync(0xffffffffu, i < L && w.res[i] == eos);
      if (bits) {
        cut = b + __ffs(bits) - 1;
        break;
      }
    }
  }
  for (int i = lane; i < L; i += 32) p.out[base + i] = i > cut ? mask : w.res[i];
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
  int64_t count = 0;
  if (!count_ok(batch, tokens, &count) || batch > kMaxRows || count > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{token_ids, 8}, {confidence, 4}, {predicted, 8}, {current_confidence, 4},
                  {out, 8}}))
    return CID_ERR_MISALIGNED;
  if (batch == 0 || tokens == 0) return CID_OK;
  if (any_null({token_ids, confidence, predicted, current_confidence, out}))
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
  if (tokens <= kWarpRowMax) {  // one warp per row
    p.use_smem = 1;
    const int64_t grid = (batch + kWarpRowsPerCta - 1) / kWarpRowsPerCta;
    return launch_pdl(refine_warp_kernel, dim3(static_cast<unsigned>(grid)),
                      dim3(32 * kWarpRowsPerCta), 0, as_stream(stream), p, batch);
  }
  constexpr int64_t kRowBytes = 3 * 8 + 2 * 4 + 4 + 1;  // shared bytes per position
  p.use_smem = tokens <= kSmemLimit / kRowBytes;
  const int64_t smem = p.use_smem ? tokens * kRowBytes : 0;
  const size_t dyn = p.use_smem ? static_cast<size_t>(smem) : 0;
  // 512 threads per row when rows are long and too few to fill the SMs
  const bool wide = tokens >= 1024 && batch < 2LL * sm_count();
  if (!p.use_smem) {
    if (wide)
      return launch_pdl(refine_kernel<512, false>, dim3(static_cast<unsigned>(batch)), dim3(512),
                        0, as_stream(stream), p);
    return launch_pdl(refine_kernel<256, false>, dim3(static_cast<unsigned>(batch)), dim3(256), 0,
                      as_stream(stream), p);
  }
  if (dyn > 48 * 1024) {  // per device, so set on every launch (cheap)
    const cudaError_t e = wide ? cudaFuncSetAttribute(refine_kernel<512, true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      static_cast<int>(kSmemLimit))
                               : cudaFuncSetAttribute(refine_kernel<256, true>,
                                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      static_cast<int>(kSmemLimit));
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  if (wide)
    return launch_pdl(refine_kernel<512, true>, dim3(static_cast<unsigned>(batch)), dim3(512), dyn,
                      as_stream(stream), p);
  return launch_pdl(refine_kernel<256, true>, dim3(static_cast<unsigned>(batch)), dim3(256), dyn,
                    as_stream(stream), p);
}
