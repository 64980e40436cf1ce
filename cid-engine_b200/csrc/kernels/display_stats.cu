// Display-token statistics: one streaming pass over each logits row.
//
// For every row of `logits` [rows, vocab] the kernel produces
//   predicted  = argmax (first NaN; otherwise lowest index of the maximum),
//   confidence = 1 / sum_v exp(x_v - max),
//   current    = exp(x_id - max) / sum_v exp(x_v - max)
// which is the reference CPU backend's definition
// (csrc/cpu/display_stats.cpp:14-126 of fwerkor/cid-engine v1.1.0).
//
// Design (HBM-bound: every logit is read once, nothing else is large):
//  * one pass with an online (max, offset, sum, argmax) state per thread;
//    terms are 2^(x*log2e - off) where off = float(max*log2e) is the offset
//    the running sum is kept relative to.  The final confidence is
//    2^(max*log2e - off) / sum with the exponent formed by one fma, so the
//    rounding of `off` cancels exactly between numerator and denominator
//    (this keeps rows like 1e4 + N(0, 0.25) accurate);
//  * 16-byte streaming loads (ld.global.cs), CID_STATS_UNROLL in flight per
//    thread; the chunk maximum is taken on the packed words (max.bf16x2 /
//    max.f16x2) and each value is converted once, for its exp2 term;
//  * rows shorter than the device's appetite are split across a thread-block
//    cluster; partial states are merged through distributed shared memory in
//    cluster-rank order (deterministic);
//  * rows whose maximum is not finite or whose sum is NaN (NaN/inf logits)
//    take a second, rare pass that finds the first NaN / first maximum and
//    writes NaN statistics, as ATen's max(-1) + exp does.
#include <cooperative_groups.h>

#include <climits>
#include <cmath>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace cid {
namespace {

#ifndef CID_STATS_THREADS
#define CID_STATS_THREADS 256
#endif
#ifndef CID_STATS_UNROLL
#define CID_STATS_UNROLL 4
#endif
constexpr int kThreads = CID_STATS_THREADS;  // threads per CTA
constexpr int kUnroll = CID_STATS_UNROLL;    // 16-byte loads in flight per thread
constexpr int kNoIndex = INT_MAX;
constexpr int kMaxCluster = 8;

struct Partial {
  float m;    // running maximum (NaN ignored); -inf when nothing seen
  float off;  // offset of the running sum: float(m * log2e), 0 while m = -inf
  float s;    // sum of 2^(x*log2e - off)
  int idx;    // column of the first maximum, kNoIndex when none
};

__device__ __forceinline__ float offset_of(float m) {
  return m == -INFINITY ? 0.0f : m * kLog2e;
}

// Sum `s` (kept relative to `off`, state maximum `m`) re-expressed relative to
// `new_off`.  A state that has seen only -inf/NaN carries 0 or NaN.
__device__ __forceinline__ float rescale(float s, float m, float off, float new_off) {
  if (m == -INFINITY) return s != s ? s : 0.0f;
  return s * ex2(off - new_off);
}

__device__ __forceinline__ Partial merge(const Partial& a, const Partial& b) {
  const bool take_b = b.m > a.m || (b.m == a.m && b.idx < a.idx);
  Partial w = take_b ? b : a;
  w.s = rescale(a.s, a.m, a.off, w.off) + rescale(b.s, b.m, b.off, w.off);
  return w;
}

__device__ __forceinline__ Partial shfl_down(const Partial& p, int delta) {
  Partial q;
  q.m = __shfl_down_sync(0xffffffffu, p.m, delta);
  q.off = __shfl_down_sync(0xffffffffu, p.off, delta);
  q.s = __shfl_down_sync(0xffffffffu, p.s, delta);
  q.idx = __shfl_down_sync(0xffffffffu, p.idx, delta);
  return q;
}

// Element type traits: a 16-byte vector holds N values, converted to float.
template <typename T> struct VecTraits;
template <> struct VecTraits<float> {
  static constexpr int N = 4;
  __device__ static void to_float(const uint4& v, float* out) {
    out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
  }
  __device__ static float scalar(const void* p, int64_t i) {
    return static_cast<const float*>(p)[i];
  }
  // maximum of the vector's values (NaN ignored)
  __device__ static float vmax(const uint4& v) {
    return fmaxf(fmaxf(__uint_as_float(v.x), __uint_as_float(v.y)),
                 fmaxf(__uint_as_float(v.z), __uint_as_float(v.w)));
  }
  static constexpr uint32_t kNegInfWord = 0xff800000u;
};
template <> struct VecTraits<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void to_float(const uint4& v, float* out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = bf16_bits_lo(w[k]);
      out[2 * k + 1] = bf16_bits_hi(w[k]);
    }
  }
  __device__ static float scalar(const void* p, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
  // maximum on packed bf16x2 (max.bf16x2 ignores NaN), converted once
  __device__ static float vmax(const uint4& v) {
    const __nv_bfloat162 a = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&v.x),
                                     *reinterpret_cast<const __nv_bfloat162*>(&v.y));
    const __nv_bfloat162 b = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&v.z),
                                     *reinterpret_cast<const __nv_bfloat162*>(&v.w));
    const __nv_bfloat162 c = __hmax2(a, b);
    return fmaxf(__low2float(c), __high2float(c));
  }
  static constexpr uint32_t kNegInfWord = 0xff80ff80u;
};
template <> struct VecTraits<__half> {
  static constexpr int N = 8;
  __device__ static void to_float(const uint4& v, float* out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
      float2 f = __half22float2(h);
      out[2 * k] = f.x;
      out[2 * k + 1] = f.y;
    }
  }
  __device__ static float scalar(const void* p, int64_t i) {
    return __half2float(static_cast<const __half*>(p)[i]);
  }
  __device__ static float vmax(const uint4& v) {
    const __half2 a = __hmax2(*reinterpret_cast<const __half2*>(&v.x),
                              *reinterpret_cast<const __half2*>(&v.y));
    const __half2 b = __hmax2(*reinterpret_cast<const __half2*>(&v.z),
                              *reinterpret_cast<const __half2*>(&v.w));
    const __half2 c = __hmax2(a, b);
    return fmaxf(__low2float(c), __high2float(c));
  }
  static constexpr uint32_t kNegInfWord = 0xfc00fc00u;
};
template <> struct VecTraits<double> {
  static constexpr int N = 2;
  __device__ static void to_float(const uint4& v, float* out) {
    out[0] = static_cast<float>(__hiloint2double(static_cast<int>(v.y), static_cast<int>(v.x)));
    out[1] = static_cast<float>(__hiloint2double(static_cast<int>(v.w), static_cast<int>(v.z)));
  }
  __device__ static float scalar(const void* p, int64_t i) {
    return static_cast<float>(static_cast<const double*>(p)[i]);
  }
  __device__ static float vmax(const uint4& v) {
    float f[2];
    to_float(v, f);
    return fmaxf(f[0], f[1]);
  }
};

struct StatsParams {
  const void* logits;
  int64_t row_stride;   // elements between rows
  const int64_t* ids;
  int64_t rows;
  int64_t vocab;        // columns held by this launch
  float* confidence;
  int64_t* predicted;
  float* current;
  uint32_t* status;
  // repetition variant
  int64_t tokens;
  int64_t mask_id;
  int64_t eos_id;
  int has_eos;
  double log_multiplier;
  // vocabulary-shard variant
  cid_shard_record_t* records;
  int64_t vocab_offset;
  int64_t total_vocab;
};

enum class Mode { kFinal, kRecord };

// Adjacent-run repetition patch of one row: up to two columns whose logit is
// raised by count*log(multiplier) (csrc/ops.cpp:505-551).
struct Patch {
  int64_t col[2];
  float delta[2];
  int n;
};

__device__ __forceinline__ float patched(const Patch& pt, int64_t col, float x) {
#pragma unroll
  for (int k = 0; k < 2; ++k)
    if (k < pt.n && col == pt.col[k]) x = __fadd_rn(x, pt.delta[k]);
  return x;
}

// Length of the run of `tok` starting at position q and moving by `dir`
// within [0, tokens) of the sequence at `seq` (one warp, ballot scan).
__device__ int64_t run_length(const int64_t* seq, int64_t tokens, int64_t q, int dir,
                              int64_t tok) {
  const int lane = threadIdx.x & 31;
  int64_t n = 0;
  for (;;) {
    const int64_t at = q + dir * static_cast<int64_t>(lane);
    const bool stop = at < 0 || at >= tokens || seq[at] != tok;
    const unsigned b = __ballot_sync(0xffffffffu, stop);
    if (b) return n + (__ffs(b) - 1);
    n += 32;
    q += dir * 32;
  }
}

// Computes the repetition patch for row `row` (warp 0 of the CTA).
__device__ void repetition_patch(const StatsParams& p, int64_t row, Patch* out) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = row % p.tokens;
  const int64_t* seq = p.ids + (row - pos);
  Patch pt;
  pt.n = 0;
  int64_t cnt[2] = {0, 0};
  for (int side = 0; side < 2; ++side) {
    const int dir = side == 0 ? -1 : 1;
    const int64_t q = pos + dir;
    if (q < 0 || q >= p.tokens) continue;
    const int64_t tok = seq[q];
    const int64_t n = 1 + run_length(seq, p.tokens, q + dir, dir, tok);
    if (tok == p.mask_id || (p.has_eos && tok == p.eos_id)) continue;
    if (pt.n == 1 && pt.col[0] == tok) {
      cnt[0] += n;
    } else {
      pt.col[pt.n] = tok;
      cnt[pt.n] = n;
      ++pt.n;
    }
  }
  for (int k = 0; k < pt.n; ++k) {
    if (pt.col[k] < 0 || pt.col[k] >= p.vocab) {
      if (lane == 0 && p.status) atomicOr(p.status, CID_STATUS_REPETITION_ID_OUT_OF_RANGE);
      pt.col[k] = -1;  // matches no column
    }
    // float32(count * log(multiplier)) as the double scalar is rounded
    pt.delta[k] = static_cast<float>(static_cast<double>(cnt[k]) * p.log_multiplier);
  }
  if (lane == 0) *out = pt;
}

template <typename T, bool kRep>
__device__ __forceinline__ void consume_scalar(Partial& st, float& acc, float x, int64_t col,
                                               const Patch& pt) {
  if (kRep) x = patched(pt, col, x);
  if (x > st.m) {
    const float noff = offset_of(x);
    st.s = rescale(st.s + acc, st.m, st.off, noff);
    acc = 0.0f;
    st.m = x;
    st.off = noff;
    st.idx = static_cast<int>(col);
  }
  acc += ex2(fmaf(x, kLog2e, -st.off));
}

// Streams columns [c_beg, c_end) of one row into `st` (this thread's share).
// Vector part: 16-byte vectors [v_beg, v_end) of the aligned region that
// starts at column `head`; scalar part: the unaligned head and tail columns
// owned by this CTA.
template <typename T, bool kRep>
__device__ void stream_row(const T* row, int64_t head, int64_t v_beg, int64_t v_end,
                           int64_t s_head_end, int64_t s_tail_beg, int64_t s_tail_end,
                           const Patch& pt, Partial& st) {
  using VT = VecTraits<T>;
  constexpr int N = VT::N;
  const int tid = threadIdx.x;
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  // head columns [0, s_head_end): lowest columns first
  for (int64_t c = tid; c < s_head_end; c += kThreads)
    consume_scalar<T, kRep>(st, acc0, VT::scalar(row, c), c, pt);

  const uint4* vrow = reinterpret_cast<const uint4*>(row + head);
  for (int64_t v = v_beg + tid; v < v_end; v += kThreads * kUnroll) {
    uint4 d[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int64_t vi = v + static_cast<int64_t>(k) * kThreads;
      if (vi < v_end) {
        d[k] = __ldcs(vrow + vi);
      } else if constexpr (sizeof(T) == 8) {
        const uint32_t hi = 0xfff00000u;  // -inf as double: 0xfff0000000000000
        d[k] = make_uint4(0u, hi, 0u, hi);
      } else {
        d[k] = make_uint4(VT::kNegInfWord, VT::kNegInfWord, VT::kNegInfWord, VT::kNegInfWord);
      }
    }
    if (kRep) {
      // repetition variant: patched values take part in the maximum
      float x[kUnroll][N];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        VT::to_float(d[k], x[k]);
        const int64_t c0 = head + (v + static_cast<int64_t>(k) * kThreads) * N;
#pragma unroll
        for (int j = 0; j < N; ++j) x[k][j] = patched(pt, c0 + j, x[k][j]);
      }
      float cm = x[0][0];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k)
#pragma unroll
        for (int j = 0; j < N; ++j) cm = fmaxf(cm, x[k][j]);
      if (cm > st.m) {
        int64_t col = 0;
        bool found = false;
#pragma unroll
        for (int k = 0; k < kUnroll; ++k)
#pragma unroll
          for (int j = 0; j < N; ++j)
            if (!found && x[k][j] == cm) {
              found = true;
              col = head + (v + static_cast<int64_t>(k) * kThreads) * N + j;
            }
        const float noff = offset_of(cm);
        st.s = rescale(st.s + ((acc0 + acc1) + (acc2 + acc3)), st.m, st.off, noff);
        acc0 = acc1 = acc2 = acc3 = 0.f;
        st.m = cm;
        st.off = noff;
        st.idx = static_cast<int>(col);
      }
      const float noff = -st.off;
#pragma unroll
      for (int k = 0; k < kUnroll; ++k)
#pragma unroll
        for (int j = 0; j < N; j += 2) {
          const float e0 = ex2(fmaf(x[k][j], kLog2e, noff));
          const float e1 = ex2(fmaf(x[k][j + 1], kLog2e, noff));
          if ((k & 1) == 0) { acc0 += e0; acc1 += e1; } else { acc2 += e0; acc3 += e1; }
        }
      continue;
    }
    // chunk maximum on the packed words, then one conversion per term
    float cm = VT::vmax(d[0]);
#pragma unroll
    for (int k = 1; k < kUnroll; ++k) cm = fmaxf(cm, VT::vmax(d[k]));
    if (cm > st.m) {
      // new running maximum (rare): its first column, in ascending order
      int64_t col = 0;
      bool found = false;
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        float x[N];
        VT::to_float(d[k], x);
#pragma unroll
        for (int j = 0; j < N; ++j)
          if (!found && x[j] == cm) {
            found = true;
            col = head + (v + static_cast<int64_t>(k) * kThreads) * N + j;
          }
      }
      const float noff = offset_of(cm);
      st.s = rescale(st.s + ((acc0 + acc1) + (acc2 + acc3)), st.m, st.off, noff);
      acc0 = acc1 = acc2 = acc3 = 0.f;
      st.m = cm;
      st.off = noff;
      st.idx = static_cast<int>(col);
    }
    const float noff = -st.off;
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      float x[N];
      VT::to_float(d[k], x);
#pragma unroll
      for (int j = 0; j < N; j += 2) {
        const float e0 = ex2(fmaf(x[j], kLog2e, noff));
        const float e1 = ex2(fmaf(x[j + 1], kLog2e, noff));
        if ((k & 1) == 0) { acc0 += e0; acc1 += e1; } else { acc2 += e0; acc3 += e1; }
      }
    }
  }
  // fold the vector accumulators (all relative to st.off) before the tail can
  // move the offset
  st.s = st.s + ((acc0 + acc1) + (acc2 + acc3));
  float acc = 0.f;
  // tail columns [s_tail_beg, s_tail_end): highest columns last
  for (int64_t c = s_tail_beg + tid; c < s_tail_end; c += kThreads)
    consume_scalar<T, kRep>(st, acc, VT::scalar(row, c), c, pt);
  st.s = st.s + acc;
}

// Block-wide merge of per-thread partials in a fixed order.
__device__ Partial block_merge(Partial st, Partial* smem_warps) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) st = merge(st, shfl_down(st, d));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem_warps[warp] = st;
  __syncthreads();
  Partial out = smem_warps[0];
  if (threadIdx.x == 0)
    for (int w = 1; w < kThreads / 32; ++w) out = merge(out, smem_warps[w]);
  return out;  // valid in thread 0
}

__device__ __forceinline__ unsigned block_min_u32(unsigned v, unsigned* smem) {
  v = __reduce_min_sync(0xffffffffu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  unsigned r = smem[0];
  for (int w = 1; w < kThreads / 32; ++w) r = min(r, smem[w]);
  __syncthreads();
  return r;
}

template <typename T, bool kRep, Mode kMode>
__global__ void __launch_bounds__(kThreads) display_stats_kernel(StatsParams p) {
  using VT = VecTraits<T>;
  constexpr int N = VT::N;
  __shared__ Partial warp_parts[kThreads / 32];
  __shared__ Partial cta_part;
  __shared__ Patch patch;
  __shared__ unsigned red[kThreads / 32];
  __shared__ int special;

  cg::cluster_group cluster = cg::this_cluster();
  const int nrank = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t row = static_cast<int64_t>(blockIdx.x) / nrank;
  const T* rowp = static_cast<const T*>(p.logits) + row * p.row_stride;
  const int64_t V = p.vocab;

  if (kRep) {
    if (threadIdx.x < 32) repetition_patch(p, row, &patch);
  } else if (threadIdx.x == 0) {
    patch.n = 0;
  }
  __syncthreads();
  const Patch pt = patch;

  // split the row: unaligned head, 16-byte vectors, tail
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp);
  int64_t head = static_cast<int64_t>(((16 - (addr & 15)) & 15) / sizeof(T));
  if (head > V) head = V;
  const int64_t nvec = (V - head) / N;
  const int64_t tail_beg = head + nvec * N;
  const int64_t v_beg = nvec * rank / nrank;
  const int64_t v_end = nvec * (rank + 1) / nrank;
  const int64_t h_end = rank == 0 ? head : 0;
  const int64_t t_beg = rank == nrank - 1 ? tail_beg : V;

  Partial st{-INFINITY, 0.0f, 0.0f, kNoIndex};
  stream_row<T, kRep>(rowp, head, v_beg, v_end, h_end, t_beg, V, pt, st);
  Partial merged = block_merge(st, warp_parts);
  if (threadIdx.x == 0) cta_part = merged;

  if (nrank > 1) {
    cluster.sync();  // every CTA's partial is visible cluster-wide
    if (rank == 0 && threadIdx.x == 0) {
      for (int r = 1; r < nrank; ++r) merged = merge(merged, *cluster.map_shared_rank(&cta_part, r));
      cta_part = merged;
    }
    cluster.sync();  // remote partials have been read; other CTAs may exit
    if (rank != 0) return;
  }
  if (threadIdx.x == 0) {
    const Partial m = cta_part;
    special = !isfinite(m.m) || (m.s != m.s);
  }
  __syncthreads();
  const Partial fin = cta_part;

  if (special) {
    // Rare path: first NaN column, else first column equal to the maximum.
    unsigned first_nan = UINT_MAX, first_max = UINT_MAX;
    for (int64_t c = threadIdx.x; c < V; c += kThreads) {
      float x = VT::scalar(rowp, c);
      if (kRep) x = patched(pt, c, x);
      if (x != x && first_nan == UINT_MAX) first_nan = static_cast<unsigned>(c);
      if (x == fin.m && first_max == UINT_MAX) first_max = static_cast<unsigned>(c);
    }
    first_nan = block_min_u32(first_nan, red);
    first_max = block_min_u32(first_max, red);
    if (threadIdx.x == 0) {
      const float qnan = __int_as_float(0x7fffffff);
      if (kMode == Mode::kFinal) {
        p.predicted[row] = first_nan != UINT_MAX ? first_nan : (first_max != UINT_MAX ? first_max : 0);
        p.confidence[row] = qnan;
        p.current[row] = qnan;
      } else {
        cid_shard_record_t rec;
        rec.max_logit = fin.m;
        rec.sum_exp = fin.m == -INFINITY ? 0.0f : qnan;
        const int64_t local = first_nan != UINT_MAX ? first_nan : (first_max != UINT_MAX ? first_max : 0);
        rec.index = static_cast<int32_t>(p.vocab_offset + local) |
                    (first_nan != UINT_MAX ? static_cast<int32_t>(0x80000000u) : 0);
        const int64_t id = p.ids[row] - p.vocab_offset;
        rec.current = (id >= 0 && id < V) ? VT::scalar(rowp, id) : 0.0f;
        p.records[row] = rec;
      }
    }
    return;
  }
  if (threadIdx.x != 0) return;
  const float top = ex2(fmaf(fin.m, kLog2e, -fin.off));  // 2^(max*log2e - off)
  if (kMode == Mode::kFinal) {
    const int64_t id = p.ids[row];
    float cur;
    if (id >= 0 && id < V) {
      float x = VT::scalar(rowp, id);
      if (kRep) x = patched(pt, id, x);
      cur = __fdiv_rn(ex2(fmaf(x, kLog2e, -fin.off)), fin.s);
    } else {
      cur = __int_as_float(0x7fffffff);
      if (p.status) atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
    }
    p.confidence[row] = __fdiv_rn(top, fin.s);
    p.predicted[row] = fin.idx;
    p.current[row] = cur;
  } else {
    cid_shard_record_t rec;
    rec.max_logit = fin.m;
    rec.sum_exp = __fdiv_rn(fin.s, top);  // sum of exp(x - max) over the shard
    rec.index = static_cast<int32_t>(p.vocab_offset + fin.idx);
    const int64_t id = p.ids[row] - p.vocab_offset;
    rec.current = (id >= 0 && id < V) ? VT::scalar(rowp, id) : 0.0f;
    p.records[row] = rec;
  }
}

// ---------------------------------------------------------------------------
// Record combine (vocabulary-parallel statistics)
// ---------------------------------------------------------------------------

constexpr int kMaxWorld = 64;
struct CombineParams {
  const cid_shard_record_t* records;
  int world;
  int64_t offsets[kMaxWorld + 1];
  const int64_t* ids;
  int64_t rows;
  float* confidence;
  int64_t* predicted;
  float* current;
  uint32_t* status;
};

__global__ void combine_records_kernel(CombineParams p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= p.rows) return;
  const float qnan = __int_as_float(0x7fffffff);
  // NaN anywhere: the lowest rank's first NaN (ranks hold ascending columns)
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.rows + row];
    if (rec.index < 0) {
      p.predicted[row] = rec.index & 0x7fffffff;
      p.confidence[row] = qnan;
      p.current[row] = qnan;
      return;
    }
  }
  float M = -INFINITY;
  int32_t idx = p.records[row].index;
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.rows + row];
    if (rec.max_logit > M) {
      M = rec.max_logit;
      idx = rec.index;
    }
  }
  p.predicted[row] = idx;
  if (!isfinite(M)) {
    p.confidence[row] = qnan;
    p.current[row] = qnan;
    return;
  }
  float S = 0.0f;
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.rows + row];
    if (rec.max_logit == -INFINITY) continue;
    S += rec.sum_exp * ex2((rec.max_logit - M) * kLog2e);
  }
  const int64_t id = p.ids[row];
  int owner = -1;
  for (int r = 0; r < p.world; ++r)
    if (id >= p.offsets[r] && id < p.offsets[r + 1]) owner = r;
  float cur = qnan;
  if (owner >= 0) {
    const float x = p.records[static_cast<int64_t>(owner) * p.rows + row].current;
    cur = __fdiv_rn(ex2((x - M) * kLog2e), S);
  } else if (p.status) {
    atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
  }
  p.confidence[row] = __fdiv_rn(1.0f, S);
  p.current[row] = cur;
}

// ---------------------------------------------------------------------------
// Launch helpers
// ---------------------------------------------------------------------------

// Cluster size: split rows until the grid has at least ~4 resident waves of
// CTAs, keeping at least 64 vectors (1-2 KB) per CTA.
int cluster_size(int64_t rows, int64_t vocab, int esize) {
  const int64_t want = static_cast<int64_t>(sm_count()) * 8 * 4;
  const int64_t vecs = vocab * esize / 16;
  int P = 1;
  while (P < kMaxCluster && rows * P < want && vecs / (2 * P) >= 64) P *= 2;
  return P;
}

template <typename T, bool kRep, Mode kMode>
int launch_stats(const StatsParams& prm, cudaStream_t stream) {
  const int P = cluster_size(prm.rows, prm.vocab, sizeof(T));
  const int64_t blocks = prm.rows * P;
  if (blocks > INT_MAX) return CID_ERR_INVALID_ARGUMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, display_stats_kernel<T, kRep, kMode>, prm);
  return record_cuda_error(err);
}

template <bool kRep, Mode kMode>
int dispatch_stats(cid_dtype_t dtype, const StatsParams& prm, cudaStream_t stream) {
  switch (dtype) {
    case CID_DTYPE_F32: return launch_stats<float, kRep, kMode>(prm, stream);
    case CID_DTYPE_BF16: return launch_stats<__nv_bfloat16, kRep, kMode>(prm, stream);
    case CID_DTYPE_F16: return launch_stats<__half, kRep, kMode>(prm, stream);
    case CID_DTYPE_F64: return launch_stats<double, kRep, kMode>(prm, stream);
    default: return CID_ERR_UNSUPPORTED_DTYPE;
  }
}

int check_logits(cid_dtype_t dtype, const void* logits, int64_t row_stride, int64_t rows,
                 int64_t vocab) {
  if (!is_float_dtype(dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (rows < 0 || vocab <= 0 || vocab > INT_MAX - 16) return CID_ERR_INVALID_ARGUMENT;
  if (rows > 0 && (logits == nullptr || row_stride < vocab)) return CID_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(logits) % dtype_size(dtype) != 0) return CID_ERR_MISALIGNED;
  return CID_OK;
}

}  // namespace
}  // namespace cid

using namespace cid;

extern "C" int cid_display_token_statistics(cid_dtype_t dtype, const void* logits,
                                            int64_t row_stride, const int64_t* token_ids,
                                            int64_t rows, int64_t vocab, float* confidence,
                                            int64_t* predicted, float* current_confidence,
                                            uint32_t* status, void* stream) {
  int rc = check_logits(dtype, logits, row_stride, rows, vocab);
  if (rc != CID_OK) return rc;
  if (rows == 0) return CID_OK;
  if (!token_ids || !confidence || !predicted || !current_confidence) return CID_ERR_INVALID_ARGUMENT;
  StatsParams prm = {};
  prm.logits = logits;
  prm.row_stride = row_stride;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.vocab = vocab;
  prm.confidence = confidence;
  prm.predicted = predicted;
  prm.current = current_confidence;
  prm.status = status;
  prm.tokens = 1;
  return dispatch_stats<false, Mode::kFinal>(dtype, prm, as_stream(stream));
}

extern "C" int cid_display_token_statistics_with_repetition(
    cid_dtype_t dtype, const void* logits, int64_t row_stride, const int64_t* token_ids,
    int64_t batch, int64_t tokens, int64_t vocab, int64_t mask_token_id, int has_eos,
    int64_t eos_token_id, double multiplier, float* confidence, int64_t* predicted,
    float* current_confidence, uint32_t* status, void* stream) {
  if (!(multiplier > 0.0 && multiplier <= 1.0)) return CID_ERR_INVALID_ARGUMENT;
  if (batch < 0 || tokens < 0) return CID_ERR_INVALID_ARGUMENT;
  const int64_t rows = batch * tokens;
  if (multiplier == 1.0 || tokens <= 1)  // csrc/ops.cpp:494-496
    return cid_display_token_statistics(dtype, logits, row_stride, token_ids, rows, vocab,
                                        confidence, predicted, current_confidence, status,
                                        stream);
  int rc = check_logits(dtype, logits, row_stride, rows, vocab);
  if (rc != CID_OK) return rc;
  if (rows == 0) return CID_OK;
  if (!token_ids || !confidence || !predicted || !current_confidence) return CID_ERR_INVALID_ARGUMENT;
  StatsParams prm = {};
  prm.logits = logits;
  prm.row_stride = row_stride;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.vocab = vocab;
  prm.confidence = confidence;
  prm.predicted = predicted;
  prm.current = current_confidence;
  prm.status = status;
  prm.tokens = tokens;
  prm.mask_id = mask_token_id;
  prm.eos_id = eos_token_id;
  prm.has_eos = has_eos;
  prm.log_multiplier = std::log(multiplier);
  return dispatch_stats<true, Mode::kFinal>(dtype, prm, as_stream(stream));
}

extern "C" int cid_display_shard_records(cid_dtype_t dtype, const void* logits,
                                         int64_t row_stride, const int64_t* token_ids,
                                         int64_t rows, int64_t shard_vocab,
                                         int64_t vocab_offset, int64_t total_vocab,
                                         cid_shard_record_t* records, uint32_t* status,
                                         void* stream) {
  int rc = check_logits(dtype, logits, row_stride, rows, shard_vocab);
  if (rc != CID_OK) return rc;
  if (vocab_offset < 0 || vocab_offset + shard_vocab > total_vocab || total_vocab > INT_MAX)
    return CID_ERR_INVALID_ARGUMENT;
  if (rows == 0) return CID_OK;
  if (!token_ids || !records) return CID_ERR_INVALID_ARGUMENT;
  StatsParams prm = {};
  prm.logits = logits;
  prm.row_stride = row_stride;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.vocab = shard_vocab;
  prm.status = status;
  prm.tokens = 1;
  prm.records = records;
  prm.vocab_offset = vocab_offset;
  prm.total_vocab = total_vocab;
  return dispatch_stats<false, Mode::kRecord>(dtype, prm, as_stream(stream));
}

extern "C" int cid_display_combine_records(const cid_shard_record_t* records, int world,
                                           const int64_t* shard_offsets_host,
                                           const int64_t* token_ids, int64_t rows,
                                           float* confidence, int64_t* predicted,
                                           float* current_confidence, uint32_t* status,
                                           void* stream) {
  if (world < 1 || world > kMaxWorld || rows < 0 || !shard_offsets_host)
    return CID_ERR_INVALID_ARGUMENT;
  if (rows == 0) return CID_OK;
  if (!records || !token_ids || !confidence || !predicted || !current_confidence)
    return CID_ERR_INVALID_ARGUMENT;
  CombineParams prm = {};
  prm.records = records;
  prm.world = world;
  for (int r = 0; r <= world; ++r) {
    prm.offsets[r] = shard_offsets_host[r];
    if (r > 0 && prm.offsets[r] < prm.offsets[r - 1]) return CID_ERR_INVALID_ARGUMENT;
  }
  prm.ids = token_ids;
  prm.rows = rows;
  prm.confidence = confidence;
  prm.predicted = predicted;
  prm.current = current_confidence;
  prm.status = status;
  const int threads = 256;
  const int64_t blocks = (rows + threads - 1) / threads;
  combine_records_kernel<<<static_cast<unsigned>(blocks), threads, 0, as_stream(stream)>>>(prm);
  return launch_result();
}
