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
//  * one pass; each thread keeps (running max m, offset off, sums s) with
//    terms 2^(x*log2e - off).  The offset is re-set only when the running
//    maximum passes the maximum it was set from by more than kGap (terms stay
//    below e^kGap), so the rescale branch is rare; the final confidence is
//    2^(max*log2e - off) / sum with the exponent formed by one fma, so the
//    rounding of `off` cancels exactly between numerator and denominator
//    (this keeps rows like 1e4 + N(0, 0.25) accurate);
//  * the argmax is tracked lazily: a thread records only WHICH chunk last
//    raised its maximum (two predicated selects, no branch); once the row
//    maximum is known, the threads holding it re-read that one chunk to find
//    their first column and the smallest wins;
//  * 32-byte streaming loads (sm_100 ld.global.nc.v8.b32; rows are peeled to
//    32-byte alignment), 4 in flight per thread; the chunk maximum is
//    taken on the packed words (max.bf16x2 / max.f16x2); the exp2 arguments
//    and the sums use packed fma.rn.f32x2 / add.rn.f32x2 (sm_100);
//  * rows shorter than the device's appetite are split across a thread-block
//    cluster; partial states are merged through distributed shared memory in
//    cluster-rank order (deterministic);
//  * rows whose maximum is not finite or whose sum is NaN (NaN/inf logits)
//    take a second, rare pass that finds the first NaN / first maximum and
//    writes NaN statistics, as ATen's max(-1) + exp does.
#include <cooperative_groups.h>

#include <climits>
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace cid {
namespace {

// Threads per CTA of the CTA (cluster) kernel: 256 by default; 128 and 512
// where the launch's shape favours them (launch_stats).
constexpr int kThreads = 256;
constexpr int kMaxCluster = 16;  // above 8: non-portable, opted into per kernel
constexpr float kGap = 5.0f;  // natural-log units; terms stay <= e^5
constexpr int64_t kNone = LLONG_MAX;
constexpr int kMaxPeers = 8;  // ranks of a peer record exchange

// packed float32 pair ops (sm_100)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %4};\n"
      " mov.b64 rc, {%5, %5};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  asm("{\n .reg .b64 ra, rb;\n mov.b64 ra, {%0, %1};\n mov.b64 rb, {%2, %3};\n"
      " add.rn.f32x2 ra, ra, rb;\n mov.b64 {%0, %1}, ra;\n}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}

// Per-thread streaming state.
struct Acc {
  float m;       // running maximum (NaN ignored), -inf when nothing seen
  float om;      // maximum the offset was set from; -inf = offset unset
  float off;     // float(om * log2e), 0 while unset
  float s0, s1;  // sums of 2^(x*log2e - off)
  int64_t where; // chunk that last raised m: its first vector index (>= 0),
                 // or -(column+1) for a scalar head/tail column
};

// Sum relative to `off` (state with offset maximum `om`) re-expressed
// relative to `new_off`; a state without offset carries only 0 or NaN.
__device__ __forceinline__ float rescale(float s, float om, float off, float new_off) {
  if (om == -INFINITY) return s != s ? s : 0.0f;
  return s * ex2(off - new_off);
}

// Re-sets the offset when the running maximum has outgrown it (rare).
__device__ __forceinline__ void maybe_reoffset(Acc& a) {
  if (a.m > a.om + kGap) {
    const float noff = a.m * kLog2e;
    a.s0 = rescale(a.s0, a.om, a.off, noff);
    a.s1 = rescale(a.s1, a.om, a.off, noff);
    a.om = a.m;
    a.off = noff;
  }
}

// Reduced state of a group of threads: (m, om, off, s); the argmax column is
// resolved separately.
struct Partial {
  float m, om, off, s;
};

__device__ __forceinline__ Partial merge(const Partial& a, const Partial& b) {
  Partial w;
  w.m = fmaxf(a.m, b.m);
  if (a.om == -INFINITY && b.om == -INFINITY) {
    w.om = -INFINITY;
    w.off = 0.0f;
    w.s = a.s + b.s;  // 0 or NaN
    return w;
  }
  if (a.om == -INFINITY || (b.om != -INFINITY && b.off > a.off)) {
    w.om = b.om;
    w.off = b.off;
  } else {
    w.om = a.om;
    w.off = a.off;
  }
  w.s = rescale(a.s, a.om, a.off, w.off) + rescale(b.s, b.om, b.off, w.off);
  return w;
}

__device__ __forceinline__ Partial shfl_xor(const Partial& p, int mask) {
  Partial q;
  q.m = __shfl_xor_sync(0xffffffffu, p.m, mask);
  q.om = __shfl_xor_sync(0xffffffffu, p.om, mask);
  q.off = __shfl_xor_sync(0xffffffffu, p.off, mask);
  q.s = __shfl_xor_sync(0xffffffffu, p.s, mask);
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
  int records_v4;  // records (and peer_records) 16-byte aligned: one vector store each
  // peer exchange: this rank's slot in the other ranks' inboxes, where each
  // record is stored too, over NVLink, while the kernel streams its logits
  int peers;
  cid_shard_record_t* peer_records[kMaxPeers - 1];
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

// Computes the repetition patch for row `row` (one whole warp).  Lanes 0-15
// read the 16 positions left of the row's position, lanes 16-31 the 16 to
// its right, in one round of loads; a run that fills its 16 lanes is
// finished by the ballot scan.
__device__ void repetition_patch(const StatsParams& p, int64_t row, Patch* out) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = row % p.tokens;
  const int64_t* seq = p.ids + (row - pos);
  const int my_dir = lane < 16 ? -1 : 1;
  const int64_t at = pos + my_dir * (1 + (lane & 15));
  const bool in = at >= 0 && at < p.tokens;
  const int64_t v = in ? seq[at] : 0;
  const unsigned full = 0xffffffffu;
  Patch pt;
  pt.n = 0;
  int64_t cnt[2] = {0, 0};
  for (int side = 0; side < 2; ++side) {  // left, then right (csrc/ops.cpp:505-533)
    const int dir = side == 0 ? -1 : 1;
    const int64_t q = pos + dir;
    if (q < 0 || q >= p.tokens) continue;
    const int64_t tok = __shfl_sync(full, v, side * 16);  // seq[q]
    const unsigned stop = (__ballot_sync(full, !in || v != tok) >> (side * 16)) & 0xffffu;
    const int64_t n = stop ? __ffs(stop) - 1 : 16 + run_length(seq, p.tokens, q + 16 * dir, dir, tok);
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

template <bool kRep>
__device__ __forceinline__ void consume_scalar(Acc& a, float x, int64_t col, const Patch& pt) {
  if (kRep) x = patched(pt, col, x);
  const bool up = x > a.m;
  a.m = up ? x : a.m;
  a.where = up ? -(col + 1) : a.where;
  maybe_reoffset(a);
  a.s0 += ex2(fmaf(x, kLog2e, -a.off));
}

// A 32-byte vector: two 16-byte halves, read with one sm_100 256-bit load on
// the non-coherent path without L1 allocation (every logit is read once).
struct Vec32 {
  uint4 lo, hi;
};
constexpr int kVecBytes = 32;

__device__ __forceinline__ Vec32 load_vec32(const Vec32* p) {
  Vec32 v;
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.lo.x), "=r"(v.lo.y), "=r"(v.lo.z), "=r"(v.lo.w), "=r"(v.hi.x),
                 "=r"(v.hi.y), "=r"(v.hi.z), "=r"(v.hi.w)
               : "l"(p));
  return v;
}

// -inf in every element (fills the lanes past the end of a thread's range).
template <typename T>
__device__ __forceinline__ Vec32 neg_inf_vec32() {
  if constexpr (sizeof(T) == 8) {
    const uint4 h = make_uint4(0u, 0xfff00000u, 0u, 0xfff00000u);
    return Vec32{h, h};
  } else {
    const uint32_t w = VecTraits<T>::kNegInfWord;
    return Vec32{make_uint4(w, w, w, w), make_uint4(w, w, w, w)};
  }
}

template <typename T>
__device__ __forceinline__ float vmax32(const Vec32& v) {
  return fmaxf(VecTraits<T>::vmax(v.lo), VecTraits<T>::vmax(v.hi));
}

template <typename T>
__device__ __forceinline__ void to_float32(const Vec32& v, float* x) {
  VecTraits<T>::to_float(v.lo, x);
  VecTraits<T>::to_float(v.hi, x + VecTraits<T>::N);
}

// d[k] for a run-time k, by selects over the constant-index registers (a
// run-time index into d would place the array in local memory).
template <int U>
__device__ __forceinline__ Vec32 pick(const Vec32 (&d)[U], int k) {
  Vec32 r = d[0];
#pragma unroll
  for (int i = 1; i < U; ++i)
    if (k == i) r = d[i];
  return r;
}

// Streams this thread's share of one row: the unaligned head columns
// [0, s_head_end), 32-byte vectors [v_beg, v_end) of the aligned region that
// starts at column `head` (thread t takes v_beg + t, + stride, ...; U loads
// in flight), and the tail columns [s_tail_beg, s_tail_end) — in ascending
// column order, so a strict `>` keeps each thread's first occurrence of its
// maximum.
template <typename T, bool kRep, int kStride, int U>
__device__ void stream_row(const T* row, int64_t head, int64_t v_beg, int64_t v_end,
                           int64_t s_head_end, int64_t s_tail_beg, int64_t s_tail_end,
                           const Patch& pt, Acc& a, int tid) {
  using VT = VecTraits<T>;
  constexpr int N = 2 * VT::N;  // values per 32-byte vector
  for (int64_t c = tid; c < s_head_end; c += kStride) consume_scalar<kRep>(a, VT::scalar(row, c), c, pt);

  const Vec32* vrow = reinterpret_cast<const Vec32*>(row + head);
  // repetition variant: the vectors (relative to `head`) holding the patched
  // columns, -1 where none; only a chunk holding one takes the element-wise
  // path below
  int64_t pvec[2] = {-1, -1};
  if (kRep) {
#pragma unroll
    for (int q = 0; q < 2; ++q)
      if (q < pt.n && pt.col[q] >= head) pvec[q] = (pt.col[q] - head) / N;
  }
  for (int64_t v = v_beg + tid; v < v_end; v += kStride * U) {
    Vec32 d[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t vi = v + static_cast<int64_t>(k) * kStride;
      d[k] = vi < v_end ? load_vec32(vrow + vi) : neg_inf_vec32<T>();
    }
    bool hit = false;
    if (kRep) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int64_t dv = pvec[q] - v;
        hit |= dv >= 0 && dv < int64_t{kStride} * U && dv % kStride == 0;
      }
    }
    if (hit) {
      // patched values take part in the maximum; two sweeps over the loaded
      // vectors (maximum, then sums), one vector at a time, so this rare
      // path adds few registers to the kernel
      float cm = -INFINITY;
#pragma unroll 1
      for (int k = 0; k < U; ++k) {
        float x[N];
        to_float32<T>(pick(d, k), x);
        const int64_t c0 = head + (v + static_cast<int64_t>(k) * kStride) * N;
#pragma unroll
        for (int j = 0; j < N; ++j) cm = fmaxf(cm, patched(pt, c0 + j, x[j]));
      }
      const bool up = cm > a.m;
      a.m = up ? cm : a.m;
      a.where = up ? v : a.where;
      maybe_reoffset(a);
      const float noff = -a.off;
#pragma unroll 1
      for (int k = 0; k < U; ++k) {
        float x[N];
        to_float32<T>(pick(d, k), x);
        const int64_t c0 = head + (v + static_cast<int64_t>(k) * kStride) * N;
#pragma unroll
        for (int j = 0; j < N; j += 2) {
          float t0, t1;
          fma2(t0, t1, patched(pt, c0 + j, x[j]), patched(pt, c0 + j + 1, x[j + 1]), kLog2e,
               noff);
          add2(a.s0, a.s1, ex2(t0), ex2(t1));
        }
      }
      continue;
    }
    float cm = vmax32<T>(d[0]);
#pragma unroll
    for (int k = 1; k < U; ++k) cm = fmaxf(cm, vmax32<T>(d[k]));
    const bool up = cm > a.m;  // lazy argmax: remember the chunk only
    a.m = up ? cm : a.m;
    a.where = up ? v : a.where;
    maybe_reoffset(a);
    const float noff = -a.off;
#pragma unroll
    for (int k = 0; k < U; ++k) {
      float x[N];
      to_float32<T>(d[k], x);
#pragma unroll
      for (int j = 0; j < N; j += 2) {
        float t0, t1;
        fma2(t0, t1, x[j], x[j + 1], kLog2e, noff);
        add2(a.s0, a.s1, ex2(t0), ex2(t1));
      }
    }
  }
  for (int64_t c = s_tail_beg + tid; c < s_tail_end; c += kStride)
    consume_scalar<kRep>(a, VT::scalar(row, c), c, pt);
}

// First column holding `target` among this thread's elements, from the chunk
// recorded in `where` (re-read from memory); kNone when the thread's maximum
// is not `target`.
template <typename T, bool kRep, int kStride, int U>
__device__ int64_t first_column(const Acc& a, float target, const T* row, int64_t head,
                                int64_t v_end, const Patch& pt) {
  constexpr int N = 2 * VecTraits<T>::N;
  if (!(a.m == target)) return kNone;
  if (a.where < 0) return -a.where - 1;
  const Vec32* vrow = reinterpret_cast<const Vec32*>(row + head);
  // all U vectors of the chunk requested before any is scanned: one L2
  // round trip instead of up to U dependent ones
  Vec32 v[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t vi = a.where + static_cast<int64_t>(k) * kStride;
    if (vi < v_end) v[k] = vrow[vi];
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t vi = a.where + static_cast<int64_t>(k) * kStride;
    if (vi >= v_end) break;
    float x[N];
    to_float32<T>(v[k], x);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const int64_t col = head + vi * N + j;
      const float y = kRep ? patched(pt, col, x[j]) : x[j];
      if (y == target) return col;
    }
  }
  return kNone;
}

// Partial of no values: merging it changes nothing.
__device__ __forceinline__ Partial empty_partial() { return Partial{-INFINITY, -INFINITY, 0.0f, 0.0f}; }

// Merge of the `n` (<= 32) partials in lanes 0..n-1 of a warp by a fixed
// butterfly (deterministic; the result is read from lane 0).
__device__ __forceinline__ Partial warp_merge_n(Partial q, int n) {
  for (int d = 1; d < n; d <<= 1) q = merge(q, shfl_xor(q, d));
  return q;
}

// Block-wide merge of per-thread partials in a fixed order: butterflies
// within each warp, then the warps' partials by a butterfly in warp 0
// (result valid in every thread).
template <int kBT>
__device__ Partial block_merge(Partial st, Partial* smem_warps, Partial* smem_out) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) st = merge(st, shfl_xor(st, d));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem_warps[warp] = st;
  __syncthreads();
  if (warp == 0) {
    Partial q = lane < kBT / 32 ? smem_warps[lane] : empty_partial();
    q = warp_merge_n(q, kBT / 32);
    if (lane == 0) *smem_out = q;
  }
  __syncthreads();
  return *smem_out;
}

// Minimum of v over the block, valid in thread 0 (the barrier on entry
// makes `smem` reusable by consecutive calls).
template <int kBT>
__device__ __forceinline__ int64_t block_min_i64(int64_t v, int64_t* smem) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kBT / 32 ? smem[lane] : kNone;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, d));
  }
  return v;
}

// Split cluster barrier: arrive (relaxed) early, wait later.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// The row's token id relative to this launch's columns, and the logit there
// (0 outside them); loaded by the row's writer when the row starts, so that
// both dependent loads complete under the streaming instead of after it.
template <typename T, Mode kMode>
__device__ __forceinline__ void load_current(const StatsParams& p, int64_t row, const T* rowp,
                                             int64_t V, int64_t& id, float& x) {
  id = __ldg(p.ids + row) - (kMode == Mode::kRecord ? p.vocab_offset : 0);
  x = (id >= 0 && id < V) ? VecTraits<T>::scalar(rowp, id) : 0.0f;
}

// The record of one row, into this launch's records and, in a peer exchange,
// into this rank's slot of every other rank's inbox (remote stores that
// overlap the streaming of later rows; the publish kernel that follows the
// launch orders them before the epoch flag).
__device__ __forceinline__ void store_record(const StatsParams& p, int64_t row,
                                             const cid_shard_record_t& rec) {
  if (p.records_v4) {
    const uint4 v = make_uint4(__float_as_uint(rec.max_logit), __float_as_uint(rec.sum_exp),
                               static_cast<uint32_t>(rec.index), __float_as_uint(rec.current));
    *reinterpret_cast<uint4*>(p.records + row) = v;
    for (int q = 0; q < p.peers; ++q) *reinterpret_cast<uint4*>(p.peer_records[q] + row) = v;
  } else {
    p.records[row] = rec;
  }
}

// Outputs of one row whose maximum is not finite or whose sum is NaN:
// predicted = first NaN, else first maximum; statistics NaN.
template <typename T, Mode kMode>
__device__ void write_special(const StatsParams& p, int64_t row, float cur_x, float m,
                              int64_t first_nan, int64_t first_max) {
  const float qnan = __int_as_float(0x7fffffff);
  const int64_t local = first_nan != kNone ? first_nan : (first_max != kNone ? first_max : 0);
  if (kMode == Mode::kFinal) {
    p.predicted[row] = local;
    p.confidence[row] = qnan;
    p.current[row] = qnan;
  } else {
    cid_shard_record_t rec;
    rec.max_logit = m;
    rec.sum_exp = m == -INFINITY ? 0.0f : qnan;
    rec.index = static_cast<int32_t>(p.vocab_offset + local) |
                (first_nan != kNone ? static_cast<int32_t>(0x80000000u) : 0);
    rec.current = cur_x;
    store_record(p, row, rec);
  }
}

// Outputs of one ordinary row from its merged partial and argmax column.
template <typename T, bool kRep, Mode kMode>
__device__ void write_normal(const StatsParams& p, int64_t row, int64_t V, int64_t id,
                             float cur_x, const Patch& pt, const Partial& fin, int64_t col) {
  const float top = ex2(fmaf(fin.m, kLog2e, -fin.off));  // 2^(max*log2e - off)
  if (kMode == Mode::kFinal) {
    float cur;
    if (id >= 0 && id < V) {
      float x = cur_x;
      if (kRep) x = patched(pt, id, x);
      cur = __fdiv_rn(ex2(fmaf(x, kLog2e, -fin.off)), fin.s);
    } else {
      cur = __int_as_float(0x7fffffff);
      if (p.status) atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
    }
    p.confidence[row] = __fdiv_rn(top, fin.s);
    p.predicted[row] = col;
    p.current[row] = cur;
  } else {
    cid_shard_record_t rec;
    rec.max_logit = fin.m;
    rec.sum_exp = __fdiv_rn(fin.s, top);  // sum of exp(x - max) over the shard
    rec.index = static_cast<int32_t>(p.vocab_offset + col);
    rec.current = cur_x;
    store_record(p, row, rec);
  }
}

// Resident CTAs per SM asked of the register allocator: 0 (no request) for
// the plain statistics, whose natural allocation already fits 1024 threads;
// the repetition variant is held to 1024 threads (62 registers at 256
// threads, no spills; measured 13 % faster than its natural 74 on fp32
// [1024, 32000]).  An explicit 1 would lift the default cap and raise the
// plain kernels to 92-124 registers.
template <typename T, bool kRep, Mode kMode, int U, int kBT>
__global__ void __launch_bounds__(kBT, kRep ? 1024 / kBT : 0) display_stats_kernel(StatsParams p) {
  pdl_wait();
  using VT = VecTraits<T>;
  constexpr int N = 2 * VT::N;
  __shared__ Partial warp_parts[kBT / 32];
  __shared__ Partial cta_part;               // this CTA's merged partial
  __shared__ Partial parts[kMaxCluster];     // rank 0: every CTA's partial
  __shared__ float2 heads[kMaxCluster];      // every CTA: (max, sum) of every CTA
  __shared__ int64_t cols[kMaxCluster];      // rank 0: every CTA's first column
  __shared__ int64_t red[kBT / 32];
  __shared__ Patch patch;

  cg::cluster_group cluster = cg::this_cluster();
  const int nrank = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int64_t row = static_cast<int64_t>(blockIdx.x) / nrank;
  const T* rowp = static_cast<const T*>(p.logits) + row * p.row_stride;
  const int64_t V = p.vocab;
  // every CTA of the cluster must have started before its shared memory is
  // written remotely: arrive now, wait once the streaming is done
  if (nrank > 1) cluster_arrive_relaxed();

  if (kRep) {
    if (threadIdx.x < 32) repetition_patch(p, row, &patch);
  } else if (threadIdx.x == 0) {
    patch.n = 0;
  }
  __syncthreads();
  const Patch pt = patch;

  // split the row: unaligned head, 32-byte vectors, tail
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp);
  int64_t head = static_cast<int64_t>(((kVecBytes - (addr & (kVecBytes - 1))) & (kVecBytes - 1)) / sizeof(T));
  if (head > V) head = V;
  const int64_t nvec = (V - head) / N;
  const int64_t tail_beg = head + nvec * N;
  const int64_t v_beg = nvec * rank / nrank;
  const int64_t v_end = nvec * (rank + 1) / nrank;
  const int64_t h_end = rank == 0 ? head : 0;
  const int64_t t_beg = rank == nrank - 1 ? tail_beg : V;

  Acc a{-INFINITY, -INFINITY, 0.0f, 0.0f, 0.0f, kNone};
  // the row's writer fetches its token id now and the logit there once the
  // streaming is done (an L2 hit by then), so that warp 0 does not wait on
  // the dependent pair before streaming and the second load overlaps the
  // merges below
  const bool writer = threadIdx.x == 0 && rank == 0;
  int64_t cur_id = 0;
  float cur_x = 0.0f;
  if (writer) cur_id = __ldg(p.ids + row) - (kMode == Mode::kRecord ? p.vocab_offset : 0);
  stream_row<T, kRep, kBT, U>(rowp, head, v_beg, v_end, h_end, t_beg, V, pt, a, threadIdx.x);
  if (writer && cur_id >= 0 && cur_id < V) cur_x = VT::scalar(rowp, cur_id);
  Partial mine{a.m, a.om, a.off, a.s0 + a.s1};
  const Partial cta = block_merge<kBT>(mine, warp_parts, &cta_part);

  // The row's maximum (every CTA: its column search needs it) and, in rank
  // 0, the row's merged partial.  Lane k of warp 0 stores this CTA's
  // (max, sum) into CTA k and its partial into rank 0, all in parallel; one
  // barrier later every CTA reads them from its own shared memory.
  Partial fin = cta;
  float target = cta.m;
  bool special = !isfinite(cta.m) || (cta.s != cta.s);
  if (nrank > 1) {
    cluster_wait();
    if (threadIdx.x < nrank) {
      *cluster.map_shared_rank(&heads[rank], static_cast<int>(threadIdx.x)) =
          make_float2(cta.m, cta.s);
      if (threadIdx.x == 0) *cluster.map_shared_rank(&parts[rank], 0) = cta;
    }
    cluster.sync();
    float M = -INFINITY;
    bool nan_sum = false;
    for (int k = 0; k < nrank; ++k) {
      M = fmaxf(M, heads[k].x);
      nan_sum |= heads[k].y != heads[k].y;
    }
    target = M;
    special = !isfinite(M) || nan_sum;
    if (rank == 0 && threadIdx.x < 32) {
      Partial q = static_cast<int>(threadIdx.x) < nrank ? parts[threadIdx.x] : empty_partial();
      fin = warp_merge_n(q, nrank);  // lane 0 (thread 0) holds the row's partial
    }
  }

  // first column of the maximum: threads that hold it re-read their chunk
  int64_t col = kNone;
  if (!special) col = first_column<T, kRep, kBT, U>(a, target, rowp, head, v_end, pt);
  col = block_min_i64<kBT>(col, red);  // valid in thread 0
  if (nrank > 1) {
    if (threadIdx.x == 0) *cluster.map_shared_rank(&cols[rank], 0) = col;
    cluster.sync();  // every CTA's column has landed in rank 0
    if (rank != 0) return;
    if (threadIdx.x < 32) {
      int64_t c = static_cast<int>(threadIdx.x) < nrank ? cols[threadIdx.x] : kNone;
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) c = min(c, __shfl_xor_sync(0xffffffffu, c, d));
      col = c;
    }
  }

  // The next kernel may be scheduled from here on.  Measured on B200 with
  // CUDA graphs: this late point keeps back-to-back statistics launches as
  // fast as without programmatic launch (an early trigger placed the next
  // launch's CTAs unevenly: +15 % at 64 rows) and still hides most of the
  // refinement kernel's launch after the statistics (64 rows: 17.3 against
  // 17.7 us for the pair).
  pdl_trigger();
  if (special) {
    // Rare path: first NaN column, else first column equal to the maximum.
    int64_t first_nan = kNone, first_max = kNone;
    for (int64_t c = threadIdx.x; c < V; c += kBT) {
      float x = VT::scalar(rowp, c);
      if (kRep) x = patched(pt, c, x);
      if (x != x && first_nan == kNone) first_nan = c;
      if (x == target && first_max == kNone) first_max = c;
    }
    first_nan = block_min_i64<kBT>(first_nan, red);
    first_max = block_min_i64<kBT>(first_max, red);
    if (threadIdx.x == 0) write_special<T, kMode>(p, row, cur_x, target, first_nan, first_max);
    return;
  }
  if (threadIdx.x == 0) write_normal<T, kRep, kMode>(p, row, V, cur_id, cur_x, pt, fin, col);
}

// One warp per row (no block barriers): for many rows of moderate length,
// where a CTA per row would spend too much of its short life in block
// reductions.
constexpr int kRowWarps = 4;

__device__ __forceinline__ int64_t warp_min_i64(int64_t v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// Plain statistics: no residency request (as above); the repetition
// variant is held to seven 4-warp blocks per SM (72 registers; measured 6 %
// faster than its natural 80 on bf16 [32768, 128256]).
template <typename T, bool kRep, Mode kMode, int U>
__global__ void __launch_bounds__(kRowWarps * 32, kRep ? 7 : 0) display_stats_rows_kernel(StatsParams p) {
  pdl_wait();
  using VT = VecTraits<T>;
  constexpr int N = 2 * VT::N;
  __shared__ Patch patches[kRowWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowWarps + warp;
  if (row >= p.rows) return;  // uniform per warp
  Patch pt;
  pt.n = 0;
  if (kRep) {
    repetition_patch(p, row, &patches[warp]);
    __syncwarp();
    pt = patches[warp];
  }
  const T* rowp = static_cast<const T*>(p.logits) + row * p.row_stride;
  const int64_t V = p.vocab;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(rowp);
  int64_t head = static_cast<int64_t>(((kVecBytes - (addr & (kVecBytes - 1))) & (kVecBytes - 1)) / sizeof(T));
  if (head > V) head = V;
  const int64_t nvec = (V - head) / N;
  const int64_t tail_beg = head + nvec * N;

  Acc a{-INFINITY, -INFINITY, 0.0f, 0.0f, 0.0f, kNone};
  int64_t cur_id = 0;
  float cur_x = 0.0f;
  if (lane == 0) load_current<T, kMode>(p, row, rowp, V, cur_id, cur_x);
  stream_row<T, kRep, 32, U>(rowp, head, 0, nvec, head, tail_beg, V, pt, a, lane);
  pdl_trigger();
  Partial fin{a.m, a.om, a.off, a.s0 + a.s1};
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) fin = merge(fin, shfl_xor(fin, d));
  const bool special = !isfinite(fin.m) || (fin.s != fin.s);
  if (special) {
    int64_t first_nan = kNone, first_max = kNone;
    for (int64_t c = lane; c < V; c += 32) {
      float x = VT::scalar(rowp, c);
      if (kRep) x = patched(pt, c, x);
      if (x != x && first_nan == kNone) first_nan = c;
      if (x == fin.m && first_max == kNone) first_max = c;
    }
    first_nan = warp_min_i64(first_nan);
    first_max = warp_min_i64(first_max);
    if (lane == 0) write_special<T, kMode>(p, row, cur_x, fin.m, first_nan, first_max);
    return;
  }
  const int64_t col = warp_min_i64(first_column<T, kRep, 32, U>(a, fin.m, rowp, head, nvec, pt));
  // the plain statistics re-read the token id here rather than keep it live
  // through the streaming loop (two registers that cost the loop ~5 %)
  if (lane == 0) {
    const int64_t id = (kMode == Mode::kFinal && !kRep) ? __ldg(p.ids + row) : cur_id;
    write_normal<T, kRep, kMode>(p, row, V, id, cur_x, pt, fin, col);
  }
}

// ---------------------------------------------------------------------------
// Record combine (vocabulary-parallel statistics)
// ---------------------------------------------------------------------------

constexpr int kMaxWorld = 256;
// Record merges over more ranks than this take a warp per row.
constexpr int kWarpMergeWorld = 32;
struct CombineParams {
  const cid_shard_record_t* records;
  int64_t stride;  // records between ranks (rows, or an inbox's capacity)
  int world;
  int64_t offsets[kMaxWorld + 1];
  const int64_t* ids;
  int64_t rows;
  float* confidence;
  int64_t* predicted;
  float* current;
  uint32_t* status;
};

// The statistics of one row from its ranks' records.
__device__ __forceinline__ void combine_row(const CombineParams& p, int64_t row) {
  const float qnan = __int_as_float(0x7fffffff);
  // NaN anywhere: the lowest rank's first NaN (ranks hold ascending columns)
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
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
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
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
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
    if (rec.max_logit == -INFINITY) continue;
    S += rec.sum_exp * ex2((rec.max_logit - M) * kLog2e);
  }
  const int64_t id = p.ids[row];
  int owner = -1;
  for (int r = 0; r < p.world; ++r)
    if (id >= p.offsets[r] && id < p.offsets[r + 1]) owner = r;
  float cur = qnan;
  if (owner >= 0) {
    const float x = p.records[static_cast<int64_t>(owner) * p.stride + row].current;
    cur = __fdiv_rn(ex2((x - M) * kLog2e), S);
  } else if (p.status) {
    atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
  }
  p.confidence[row] = __fdiv_rn(1.0f, S);
  p.current[row] = cur;
}

__global__ void combine_records_kernel(CombineParams p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= p.rows) return;
  combine_row(p, row);
}

// Combine from this rank's inbox once every rank has published `epoch` in
// its flag word there (one warp waits, acquire at system scope, bounded by
// wait_ns; a wait that runs out sets CID_STATUS_PEER_TIMEOUT and the merge
// writes NaN statistics with predicted 0).
//
// A rank can run at most one epoch ahead of another while every combine
// waits for all flags (its records of epoch e+2 are ordered after a combine of
// e+1 that needs this rank's e+1 records, which follow this rank's combine of
// e), so a flag of epoch or epoch+1 means the parity slot of `epoch` holds
// that epoch's records.  A flag two or more epochs ahead means that peer gave
// up waiting on this rank earlier and may already have overwritten the slot:
// the wait sets CID_STATUS_PEER_OUT_OF_STEP and the merge writes NaN.  The
// flags are read once more after the rows are combined, so a peer that overtook
// the slot while it was being read is caught too (the step's statistics are
// then invalid and the bit says so).  Once either peer bit is set in the
// status word the exchange is poisoned: later combines write NaN without
// waiting until the host clears the word and rebuilds the exchange.
__device__ __forceinline__ int32_t peer_lead(const uint32_t* flag, uint32_t epoch) {
  uint32_t f;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
  return static_cast<int32_t>(f - epoch);
}

// The statistics of one row from its ranks' records in an inbox (16-byte
// aligned slots, world <= kMaxPeers): each record read once, as one vector,
// into registers; the arithmetic and order are combine_row's.
__device__ __forceinline__ void combine_row_inbox(const CombineParams& p, int64_t row) {
  const float qnan = __int_as_float(0x7fffffff);
  float mx[kMaxPeers], se[kMaxPeers], cu[kMaxPeers];
  int32_t ix[kMaxPeers];
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r < p.world) {
      const uint4 v =
          *reinterpret_cast<const uint4*>(p.records + static_cast<int64_t>(r) * p.stride + row);
      mx[r] = __uint_as_float(v.x);
      se[r] = __uint_as_float(v.y);
      ix[r] = static_cast<int32_t>(v.z);
      cu[r] = __uint_as_float(v.w);
    } else {
      mx[r] = -INFINITY;
      se[r] = 0.0f;
      ix[r] = 0;
      cu[r] = 0.0f;
    }
  }
  // NaN anywhere: the lowest rank's first NaN (ranks hold ascending columns)
  int nan_rank = -1;
#pragma unroll
  for (int r = kMaxPeers - 1; r >= 0; --r)
    if (r < p.world && ix[r] < 0) nan_rank = r;
  if (nan_rank >= 0) {
    int32_t idx = 0;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r == nan_rank) idx = ix[r];
    p.predicted[row] = idx & 0x7fffffff;
    p.confidence[row] = qnan;
    p.current[row] = qnan;
    return;
  }
  float M = -INFINITY;
  int32_t idx = ix[0];
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r < p.world && mx[r] > M) {
      M = mx[r];
      idx = ix[r];
    }
  }
  p.predicted[row] = idx;
  if (!isfinite(M)) {
    p.confidence[row] = qnan;
    p.current[row] = qnan;
    return;
  }
  float S = 0.0f;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) {
    if (r >= p.world || mx[r] == -INFINITY) continue;
    S += se[r] * ex2((mx[r] - M) * kLog2e);
  }
  const int64_t id = p.ids[row];
  int owner = -1;
  for (int r = 0; r < p.world; ++r)
    if (id >= p.offsets[r] && id < p.offsets[r + 1]) owner = r;
  float cur = qnan;
  if (owner >= 0) {
    float x = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r == owner) x = cu[r];
    cur = __fdiv_rn(ex2((x - M) * kLog2e), S);
  } else if (p.status) {
    atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
  }
  p.confidence[row] = __fdiv_rn(1.0f, S);
  p.current[row] = cur;
}

// Lanes 0..world-1 of warp 0 wait for their rank's flag in parallel; the
// CTA's verdict (0 go, else the status bit) is returned to every lane of the
// warp.
__device__ __forceinline__ uint32_t wait_flags(const uint32_t* flags, int world, uint32_t epoch,
                                               unsigned long long wait_ns) {
  const int lane = threadIdx.x & 31;
  uint32_t bit = 0;
  if (lane < world) {
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      const int32_t lead = peer_lead(flags + lane, epoch);
      if (lead == 0 || lead == 1) break;
      if (lead > 1) {
        bit = CID_STATUS_PEER_OUT_OF_STEP;
        break;
      }
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > wait_ns) {
        bit = CID_STATUS_PEER_TIMEOUT;
        break;
      }
      __nanosleep(256);
    }
  }
  // out of step outranks a timeout (a peer that moved on explains the wait)
  const unsigned oos = __ballot_sync(0xffffffffu, bit == CID_STATUS_PEER_OUT_OF_STEP);
  const unsigned tmo = __ballot_sync(0xffffffffu, bit == CID_STATUS_PEER_TIMEOUT);
  return oos ? CID_STATUS_PEER_OUT_OF_STEP : (tmo ? CID_STATUS_PEER_TIMEOUT : 0u);
}

// The wait and the merge are two launches: one warp waits for the flags
// (acquire at system scope, in wait_flags) and leaves its verdict in the
// inbox's own verdict word; the merge kernel, launched as its programmatic
// dependent, starts after the wait kernel has completed, so its plain loads
// see every record the flags published, and none of its CTAs issues a
// system-scope acquire (one per CTA cost tens of microseconds per step on
// peer-mapped inboxes).
__global__ void wait_inbox_kernel(const uint32_t* flags, uint32_t* verdict, int world,
                                  uint32_t epoch, unsigned long long wait_ns, uint32_t* status) {
  constexpr uint32_t kPoisoned = CID_STATUS_PEER_TIMEOUT | CID_STATUS_PEER_OUT_OF_STEP;
  pdl_wait();
  pdl_trigger();
  const bool poisoned = status && (*reinterpret_cast<volatile uint32_t*>(status) & kPoisoned);
  const uint32_t bit = poisoned ? 0u : wait_flags(flags, world, epoch, wait_ns);
  if (threadIdx.x == 0) {
    if (bit && status) atomicOr(status, bit);
    *verdict = (!poisoned && bit == 0) ? epoch : ~epoch;
  }
}

__device__ __forceinline__ int32_t peer_lead_relaxed(const uint32_t* flag, uint32_t epoch) {
  uint32_t f;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
  return static_cast<int32_t>(f - epoch);
}

__global__ void combine_inbox_kernel(CombineParams p, const uint32_t* flags,
                                     const uint32_t* verdict, uint32_t epoch) {
  pdl_wait();  // the wait kernel has completed
  pdl_trigger();
  const bool ready = *verdict == epoch;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (!ready) {
    if (row < p.rows) {
      p.predicted[row] = 0;
      p.confidence[row] = __int_as_float(0x7fffffff);
      p.current[row] = __int_as_float(0x7fffffff);
    }
    return;
  }
  if (row < p.rows) combine_row_inbox(p, row);
  __syncthreads();
  if (threadIdx.x < 32) {  // a peer that overtook the slot while it was read
    const bool ahead = threadIdx.x < p.world && peer_lead_relaxed(flags + threadIdx.x, epoch) > 1;
    if (__ballot_sync(0xffffffffu, ahead) && threadIdx.x == 0 && p.status)
      atomicOr(p.status, CID_STATUS_PEER_OUT_OF_STEP);
  }
}

// A row's merge over many ranks (the vocabulary groups of the fused LM head)
// by one warp: lane l holds ranks l, l + 32, ... in ascending order; the
// first NaN rank and the maximum (lowest rank on ties) are warp minima, the
// sum is each lane's ascending partial sum, then a fixed butterfly over the
// lanes.  Every lane returns the merged record of the row; `owner` is the
// rank holding the row's token id (-1 when none does).
struct WarpMerged {
  cid_shard_record_t rec;  // max, sum of exp(x - max), index (NaN flag), current
  int nan_rank;            // first rank with a NaN, kMaxWorld when none
  bool owned;
};

__device__ __forceinline__ WarpMerged warp_merge_row(const CombineParams& p, int64_t row,
                                                     int64_t id) {
  const int lane = threadIdx.x & 31;
  int nan_rank = kMaxWorld;
  float mx = -INFINITY;
  int mr = kMaxWorld;  // rank of the lane's first maximum
  int owner = -1;
  for (int r = lane; r < p.world; r += 32) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
    if (rec.index < 0 && nan_rank == kMaxWorld) nan_rank = r;
    if (mr == kMaxWorld || rec.max_logit > mx) {  // the lane's first maximum
      mx = rec.max_logit;
      mr = r;
    }
    if (id >= p.offsets[r] && id < p.offsets[r + 1]) owner = r;
  }
  // maximum with the lowest rank on ties (NaN maxima never occur without a
  // NaN flag, which takes the other path)
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, d);
    const int orr = __shfl_xor_sync(0xffffffffu, mr, d);
    if (om > mx || (om == mx && orr < mr)) {
      mx = om;
      mr = orr;
    }
    nan_rank = min(nan_rank, __shfl_xor_sync(0xffffffffu, nan_rank, d));
    owner = max(owner, __shfl_xor_sync(0xffffffffu, owner, d));
  }
  WarpMerged out;
  out.nan_rank = nan_rank;
  out.owned = owner >= 0;
  const int src = nan_rank < kMaxWorld ? nan_rank : (mr < kMaxWorld ? mr : 0);
  const cid_shard_record_t pick = p.records[static_cast<int64_t>(src) * p.stride + row];
  out.rec.index = pick.index;
  out.rec.max_logit = nan_rank < kMaxWorld ? pick.max_logit : mx;
  out.rec.current =
      owner >= 0 ? p.records[static_cast<int64_t>(owner) * p.stride + row].current : 0.0f;
  float S = 0.0f;
  if (nan_rank == kMaxWorld && isfinite(mx)) {
    for (int r = lane; r < p.world; r += 32) {
      const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
      if (rec.max_logit == -INFINITY) continue;
      S += rec.sum_exp * ex2((rec.max_logit - mx) * kLog2e);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) S += __shfl_xor_sync(0xffffffffu, S, d);
  }
  out.rec.sum_exp = S;
  return out;
}

// combine_records_kernel with a warp per row (world > kWarpMergeWorld).
__global__ void combine_records_warp_kernel(CombineParams p) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= p.rows) return;  // warp-uniform
  const int64_t id = p.ids[row];
  const WarpMerged w = warp_merge_row(p, row, id);
  if ((threadIdx.x & 31) != 0) return;
  const float qnan = __int_as_float(0x7fffffff);
  if (w.nan_rank < kMaxWorld) {
    p.predicted[row] = w.rec.index & 0x7fffffff;
    p.confidence[row] = qnan;
    p.current[row] = qnan;
    return;
  }
  const float M = w.rec.max_logit;
  p.predicted[row] = w.rec.index;
  if (!isfinite(M)) {
    p.confidence[row] = qnan;
    p.current[row] = qnan;
    return;
  }
  const float S = w.rec.sum_exp;
  float cur = qnan;
  if (w.owned) {
    cur = __fdiv_rn(ex2((w.rec.current - M) * kLog2e), S);
  } else if (p.status) {
    atomicOr(p.status, CID_STATUS_TOKEN_ID_OUT_OF_RANGE);
  }
  p.confidence[row] = __fdiv_rn(1.0f, S);
  p.current[row] = cur;
}

// merge_records_kernel with a warp per row (world > kWarpMergeWorld).
__global__ void merge_records_warp_kernel(CombineParams p, cid_shard_record_t* out) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= p.rows) return;  // warp-uniform
  const WarpMerged w = warp_merge_row(p, row, p.ids[row]);
  if ((threadIdx.x & 31) != 0) return;
  cid_shard_record_t m = w.rec;
  if (w.nan_rank < kMaxWorld) {
    m.sum_exp = __int_as_float(0x7fffffff);
  } else if (!isfinite(m.max_logit)) {
    m.sum_exp = m.max_logit == -INFINITY ? 0.0f : __int_as_float(0x7fffffff);
  }
  out[row] = m;
}

// Merges the records of W ascending column ranges of each row into the one
// record of their union (the record of the concatenated shard): lowest range
// wins max ties, a NaN flag wins over everything (first range holding one),
// sums re-expressed relative to the merged maximum, the current logit taken
// from the range that holds the row's token id (0 when none does).
__global__ void merge_records_kernel(CombineParams p, cid_shard_record_t* out) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= p.rows) return;
  const int64_t id = p.ids[row];
  float cur = 0.0f;
  for (int r = 0; r < p.world; ++r)
    if (id >= p.offsets[r] && id < p.offsets[r + 1])
      cur = p.records[static_cast<int64_t>(r) * p.stride + row].current;
  cid_shard_record_t m;
  m.current = cur;
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
    if (rec.index < 0) {
      m.max_logit = rec.max_logit;
      m.sum_exp = __int_as_float(0x7fffffff);
      m.index = rec.index;
      out[row] = m;
      return;
    }
  }
  float M = -INFINITY;
  int32_t idx = p.records[row].index;
  for (int r = 0; r < p.world; ++r) {
    const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
    if (rec.max_logit > M) {
      M = rec.max_logit;
      idx = rec.index;
    }
  }
  m.max_logit = M;
  m.index = idx;
  if (!isfinite(M)) {
    m.sum_exp = M == -INFINITY ? 0.0f : __int_as_float(0x7fffffff);
  } else {
    float S = 0.0f;
    for (int r = 0; r < p.world; ++r) {
      const cid_shard_record_t rec = p.records[static_cast<int64_t>(r) * p.stride + row];
      if (rec.max_logit == -INFINITY) continue;
      S += rec.sum_exp * ex2((rec.max_logit - M) * kLog2e);
    }
    m.sum_exp = S;
  }
  out[row] = m;
}

// ---------------------------------------------------------------------------
// Launch helpers
// ---------------------------------------------------------------------------

// 32-byte loads in flight per thread, both kernels (measured: 8 raises the
// CTA kernel to 98 registers and 2 resident CTAs per SM, which is slower).
constexpr int kUnroll = 4;

// Largest cluster this kernel instance can be launched with: 16 where the
// device schedules 16-CTA clusters of it (a non-portable size, opted into
// once per instance), else the portable 8.
template <typename T, bool kRep, Mode kMode, int kBT>
int max_cluster() {
  static const int n = [] {  // thread-safe one-time init
    auto* fn = display_stats_kernel<T, kRep, kMode, kUnroll, kBT>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
        cudaSuccess) {
      cudaGetLastError();
      return 8;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kMaxCluster);
    cfg.blockDim = dim3(kBT);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kMaxCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      return 8;
    }
    return kMaxCluster;
  }();
  return n;
}

// Cluster size: split rows over P CTAs (power of two) while the grid stays
// within two CTAs per SM and each CTA keeps at least half a round of 32-byte
// loads (kBT * kUnroll / 2 vectors).  Measured on B200 over [1, rows,
// 155136] bf16 with 256 threads (CUDA-graph replays): rows x P near 2 x SMs
// is the fastest split (32 rows: P = 8, 9.5 us; 64: 4, 11.2 us; 128: 2,
// 14.6 us; 256: 1, 21 us); larger clusters spend more in their merges than
// the extra SMs save, smaller ones leave SMs idle.  A 16-CTA cluster only
// while the grid keeps to one CTA per SM: at 16 rows of 155136 bf16, P = 8
// with 128-thread CTAs took 6.5 us against 7.3 for P = 16 (256 threads) and
// 7.0 for P = 16 (128 threads); at 8 rows P = 16 stays fastest (5.8 us).
template <typename T, bool kRep, Mode kMode, int kBT>
int cluster_size(int64_t rows, int64_t vocab) {
  const int64_t target = 2LL * sm_count();
  const int64_t vecs = vocab * static_cast<int64_t>(sizeof(T)) / kVecBytes;
  const int64_t min_vecs = static_cast<int64_t>(kBT) * kUnroll / 2;
  const int pmax = max_cluster<T, kRep, kMode, kBT>();
  int P = 1;
  while (P < pmax && rows * P * 2 <= target && vecs / (2 * P) >= min_vecs) P *= 2;
  if (P > 8 && rows * P > sm_count()) P = 8;
  return P;
}

// CTAs of the 256-thread kernel resident on the device at once.
template <typename T, bool kRep, Mode kMode>
int64_t cta_slots() {
  static const int64_t n = [] {  // thread-safe one-time init
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &b, display_stats_kernel<T, kRep, kMode, kUnroll, kThreads>, kThreads, 0) !=
            cudaSuccess ||
        b <= 0) {
      cudaGetLastError();
      b = 4;
    }
    return static_cast<int64_t>(b) * sm_count();
  }();
  return n;
}

#ifndef CID_STATS_ROW_MODE
#define CID_STATS_ROW_MODE 0  // 0: automatic, 1: CTA (cluster) per row, 2: warp per row
#endif

// Warp per row when the rows alone fill at least two waves of resident warps
// (measured on 32768 rows x 128256: 11% faster than a CTA per row); a CTA (or
// a cluster of CTAs) per row for fewer rows.
template <typename T, bool kRep, Mode kMode>
bool use_row_warps(int64_t rows) {
  if (CID_STATS_ROW_MODE != 0) return CID_STATS_ROW_MODE == 2;
  static const int warps_per_sm = [] {  // thread-safe one-time init
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n, display_stats_rows_kernel<T, kRep, kMode, kUnroll>, kRowWarps * 32, 0) !=
            cudaSuccess ||
        n <= 0)
      n = 8;
    return n * kRowWarps;
  }();
  return rows >= 2LL * sm_count() * warps_per_sm;
}

template <typename T, bool kRep, Mode kMode, int U, int kBT>
int launch_cta_kernel(const StatsParams& prm, int P, cudaStream_t stream) {
  const int64_t blocks = prm.rows * P;
  if (blocks > INT_MAX) return CID_ERR_INVALID_ARGUMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kBT);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return record_cuda_error(
      cudaLaunchKernelEx(&cfg, display_stats_kernel<T, kRep, kMode, U, kBT>, prm));
}

// The CTA kernel's block size from the bytes one CTA streams (with the
// 256-thread cluster split) and the CTA count.  Measured on B200 (CUDA-graph
// replays, 128 / 256 / 512 threads, us): bf16 [1, 155136] (19 KB a CTA)
// 5.1 / 5.2 / 6.1; [8, 155136] (19 KB) 6.0 / 5.8 / 6.4; [32, 155136]
// (39 KB) 6.7 / 7.9 / 8.2; [64, 155136] (78 KB) 8.8 / 9.2 / 10.3; [128,
// 155136] (155 KB) 17.0 / 14.2 / 15.3; [256, 155136] (310 KB) 26.2 / 21.1 /
// 19.4; fp32 [128, 155136] (310 KB) 30.5 / 19.3 / 17.9; fp32 [8, 32000]
// (32 KB) 4.8 / 5.1 / 5.7; fp32 [512, 32000] (128 KB, one wave) 17.4 / 14.7 /
// 17.7; fp32 [1024, 32000] (two waves at 256 threads) 25.0 / 26.5 / 33.4;
// bf16 [4096, 32000] 48.6 / 57.0 / 85.4; whole rows at up to two CTAs per
// SM: fp32 [256, 32000] (128 KB) 14.7 / 10.3 / 9.7, bf16 [256, 128256]
// (250 KB) 22.9 / 18.2 / 17.1, fp16 [256, 50257] (100 KB) 14.4 / 10.6 /
// 10.5; bf16 [1024, 128256] 45.6 / 47.6 / 51.0.  Fewer threads win where a
// CTA's merges and barriers weigh against a short chunk, or where smaller
// CTAs fit the whole grid in one wave; more threads where a long chunk needs
// more loads in flight and the grid is small.
template <typename T, bool kRep, Mode kMode>
int launch_stats(const StatsParams& prm, cudaStream_t stream) {
  if (use_row_warps<T, kRep, kMode>(prm.rows)) {
    const int64_t blocks = (prm.rows + kRowWarps - 1) / kRowWarps;
    if (blocks > INT_MAX) return CID_ERR_INVALID_ARGUMENT;
    return launch_pdl(display_stats_rows_kernel<T, kRep, kMode, kUnroll>,
                      dim3(static_cast<unsigned>(blocks)), dim3(kRowWarps * 32), 0, stream, prm);
  }
  const int P = cluster_size<T, kRep, kMode, kThreads>(prm.rows, prm.vocab);
  const int64_t chunk = prm.vocab * static_cast<int64_t>(sizeof(T)) / P;
  const bool few = prm.rows * P <= 2LL * sm_count();  // at most two CTAs per SM
  if (few && (chunk >= (int64_t{256} << 10) || (P == 1 && chunk >= (int64_t{96} << 10))))
    return launch_cta_kernel<T, kRep, kMode, kUnroll, 512>(
        prm, cluster_size<T, kRep, kMode, 512>(prm.rows, prm.vocab), stream);
  if (prm.rows * P > cta_slots<T, kRep, kMode>() ||
      (chunk > (int64_t{24} << 10) && chunk <= (int64_t{96} << 10)))
    return launch_cta_kernel<T, kRep, kMode, kUnroll, 128>(
        prm, cluster_size<T, kRep, kMode, 128>(prm.rows, prm.vocab), stream);
  return launch_cta_kernel<T, kRep, kMode, kUnroll, kThreads>(prm, P, stream);
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

// The dtype, extents and alignment of a logits argument: rows x vocab with
// row r at logits + r*row_stride (row_stride >= vocab), the whole span
// (rows-1)*row_stride + vocab within kMaxCount elements.
int check_logits(cid_dtype_t dtype, const void* logits, int64_t row_stride, int64_t rows,
                 int64_t vocab) {
  if (!is_float_dtype(dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (rows < 0 || rows > kMaxRows || vocab <= 0 || vocab > INT_MAX - 16)
    return CID_ERR_INVALID_ARGUMENT;
  int64_t span = 0;
  if (rows > 0 && (row_stride < vocab || !count_ok(rows - 1, row_stride, &span) ||
                   span > kMaxCount - vocab))
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{logits, static_cast<size_t>(dtype_size(dtype))}})) return CID_ERR_MISALIGNED;
  return CID_OK;
}

// Host shard offsets of a record merge: world + 1 ascending column offsets
// within [0, INT_MAX] (the records hold 32-bit global columns).
int check_offsets(const int64_t* offsets, int world, int max_world, int64_t (&out)[kMaxWorld + 1]) {
  if (world < 1 || world > max_world || offsets == nullptr) return CID_ERR_INVALID_ARGUMENT;
  for (int r = 0; r <= world; ++r) {
    out[r] = offsets[r];
    if (r > 0 && out[r] < out[r - 1]) return CID_ERR_INVALID_ARGUMENT;
  }
  if (out[0] < 0 || out[world] > INT_MAX) return CID_ERR_INVALID_ARGUMENT;
  return CID_OK;
}

// The vocabulary range of a shard: [vocab_offset, vocab_offset + shard_vocab)
// inside [0, total_vocab), total_vocab <= INT_MAX.
bool shard_range_ok(int64_t shard_vocab, int64_t vocab_offset, int64_t total_vocab) {
  return shard_vocab > 0 && vocab_offset >= 0 && total_vocab <= INT_MAX &&
         total_vocab >= shard_vocab && vocab_offset <= total_vocab - shard_vocab;
}

// The statistics outputs of one call.
bool stats_outputs_misaligned(const int64_t* ids, const float* confidence,
                              const int64_t* predicted, const float* current,
                              const uint32_t* status) {
  return misaligned({{ids, 8}, {confidence, 4}, {predicted, 8}, {current, 4}, {status, 4}});
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
  if (stats_outputs_misaligned(token_ids, confidence, predicted, current_confidence, status))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({logits, token_ids, confidence, predicted, current_confidence}))
    return CID_ERR_INVALID_ARGUMENT;
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
  if (!is_float_dtype(dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (!(multiplier > 0.0 && multiplier <= 1.0)) return CID_ERR_INVALID_ARGUMENT;
  int64_t rows = 0;
  if (!count_ok(batch, tokens, &rows) || rows > kMaxRows) return CID_ERR_INVALID_ARGUMENT;
  if (multiplier == 1.0 || tokens <= 1)  // csrc/ops.cpp:494-496
    return cid_display_token_statistics(dtype, logits, row_stride, token_ids, rows, vocab,
                                        confidence, predicted, current_confidence, status,
                                        stream);
  int rc = check_logits(dtype, logits, row_stride, rows, vocab);
  if (rc != CID_OK) return rc;
  if (stats_outputs_misaligned(token_ids, confidence, predicted, current_confidence, status))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({logits, token_ids, confidence, predicted, current_confidence}))
    return CID_ERR_INVALID_ARGUMENT;
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
  if (!shard_range_ok(shard_vocab, vocab_offset, total_vocab)) return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{token_ids, 8}, {records, 4}, {status, 4}})) return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({logits, token_ids, records})) return CID_ERR_INVALID_ARGUMENT;
  StatsParams prm = {};
  prm.records_v4 = reinterpret_cast<uintptr_t>(records) % 16 == 0;
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

extern "C" int cid_display_merge_records(const cid_shard_record_t* records, int world,
                                         const int64_t* shard_offsets_host,
                                         const int64_t* token_ids, int64_t rows,
                                         cid_shard_record_t* merged, void* stream) {
  CombineParams prm = {};
  int rc = check_offsets(shard_offsets_host, world, kMaxWorld, prm.offsets);
  if (rc != CID_OK) return rc;
  if (rows < 0 || rows > kMaxRows) return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{records, 4}, {token_ids, 8}, {merged, 4}})) return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({records, token_ids, merged})) return CID_ERR_INVALID_ARGUMENT;
  prm.records = records;
  prm.world = world;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.stride = rows;
  const int threads = 256;
  const int64_t blocks = (rows + threads - 1) / threads;
  if (world > kWarpMergeWorld) {  // a warp per row
    const int64_t wblocks = (rows * 32 + threads - 1) / threads;
    merge_records_warp_kernel<<<static_cast<unsigned>(wblocks), threads, 0,
                                as_stream(stream)>>>(prm, merged);
    return launch_result();
  }
  merge_records_kernel<<<static_cast<unsigned>(blocks), threads, 0, as_stream(stream)>>>(prm,
                                                                                         merged);
  return launch_result();
}

extern "C" int cid_display_combine_records(const cid_shard_record_t* records, int world,
                                           const int64_t* shard_offsets_host,
                                           const int64_t* token_ids, int64_t rows,
                                           float* confidence, int64_t* predicted,
                                           float* current_confidence, uint32_t* status,
                                           void* stream) {
  CombineParams prm = {};
  int rc = check_offsets(shard_offsets_host, world, kMaxWorld, prm.offsets);
  if (rc != CID_OK) return rc;
  if (rows < 0 || rows > kMaxRows) return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{records, 4}}) ||
      stats_outputs_misaligned(token_ids, confidence, predicted, current_confidence, status))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({records, token_ids, confidence, predicted, current_confidence}))
    return CID_ERR_INVALID_ARGUMENT;
  prm.records = records;
  prm.world = world;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.stride = rows;
  prm.confidence = confidence;
  prm.predicted = predicted;
  prm.current = current_confidence;
  prm.status = status;
  const int threads = 256;
  if (world > kWarpMergeWorld) {  // a warp per row
    const int64_t blocks = (rows * 32 + threads - 1) / threads;
    combine_records_warp_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                                  as_stream(stream)>>>(prm);
    return launch_result();
  }
  const int64_t blocks = (rows + threads - 1) / threads;
  combine_records_kernel<<<static_cast<unsigned>(blocks), threads, 0, as_stream(stream)>>>(prm);
  return launch_result();
}

// ---------------------------------------------------------------------------
// Peer record exchange: the vocabulary-parallel records stored by the
// statistics kernel straight into every rank's inbox, instead of a
// collective after it.
//
// Inbox layout (one cudaMalloc per rank, mapped into the other ranks with
// CUDA IPC): records [2 parities][world][rows_capacity] (16 B each), then a
// 256-byte tail whose first words are the flags [world] (uint32, rank q's
// last published epoch).
// ---------------------------------------------------------------------------

namespace cid {
namespace {

struct PeerSlots {
  cid_shard_record_t* dst[kMaxPeers];  // this rank's slot in the other ranks' inboxes
  uint32_t* flags[kMaxPeers];          // this rank's flag word in every inbox
};

// Copies this rank's records (its slot in its own inbox) into its slot in
// every other rank's inbox: coalesced 16-byte stores over NVLink.
__global__ void push_records_kernel(const cid_shard_record_t* src, PeerSlots slots, int others,
                                    int64_t rows) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const cid_shard_record_t rec = src[row];
  for (int q = 0; q < others; ++q) slots.dst[q][row] = rec;
}

// Launched on the stream after the kernel that stored this rank's records
// into every inbox (the record kernel, or push_records_kernel for records
// made elsewhere), as a programmatic dependent that waits for its completion:
// a system-scope fence, then the epoch released into this rank's flag word of
// every inbox.  A rank that acquires the flag (wait_inbox_kernel) sees every
// record of the epoch.
__global__ void publish_epoch_kernel(PeerSlots slots, int world, uint32_t epoch) {
  pdl_wait();  // the record kernel has completed and its stores are performed
  pdl_trigger();
  __threadfence_system();
  const int q = threadIdx.x;
  if (q < world)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slots.flags[q]), "r"(epoch)
                 : "memory");
}

constexpr size_t kInboxTail = 256;
// Word of an inbox's tail (after the ranks' flag words) where this rank's
// wait kernel leaves the epoch whose flags it saw complete; no peer writes it.
constexpr int kVerdictWord = 32;
static_assert(kMaxPeers <= kVerdictWord && (kVerdictWord + 1) * 4 <= kInboxTail, "inbox tail");

size_t inbox_record_bytes(int world, int64_t capacity) {
  return 2 * static_cast<size_t>(world) * static_cast<size_t>(capacity) *
         sizeof(cid_shard_record_t);
}
cid_shard_record_t* inbox_records(void* inbox, int world, int64_t capacity, uint32_t parity,
                                  int src) {
  return static_cast<cid_shard_record_t*>(inbox) +
         (static_cast<int64_t>(parity) * world + src) * capacity;
}
uint32_t* inbox_flags(void* inbox, int world, int64_t capacity) {
  return reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(inbox) +
                                     inbox_record_bytes(world, capacity));
}

// The rank arguments of a peer exchange call: 1 <= world <= kMaxPeers,
// 0 <= rank < world, 1 <= rows <= rows_capacity <= kMaxRows, and `world`
// non-NULL inbox pointers, 16-byte aligned (records are stored as one
// 16-byte vector each; cudaMalloc and IPC mappings are 256-byte aligned).
int check_peers(int64_t rows, int rank, int world, void* const* inboxes, int64_t rows_capacity) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || inboxes == nullptr)
    return CID_ERR_INVALID_ARGUMENT;
  // every rank publishes each epoch, so rows == 0 is not a call
  if (rows < 1 || rows > rows_capacity || rows_capacity > kMaxRows) return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{inboxes, alignof(void*)}})) return CID_ERR_MISALIGNED;
  for (int q = 0; q < world; ++q) {
    if (inboxes[q] == nullptr) return CID_ERR_INVALID_ARGUMENT;
    if (misaligned({{inboxes[q], 16}})) return CID_ERR_MISALIGNED;
  }
  return CID_OK;
}

}  // namespace
}  // namespace cid

extern "C" size_t cid_peer_inbox_bytes(int world, int64_t rows_capacity) {
  if (world < 1 || world > kMaxPeers || rows_capacity < 0 || rows_capacity > kMaxRows) return 0;
  return inbox_record_bytes(world, rows_capacity) + kInboxTail;
}

extern "C" int cid_peer_inbox_alloc(size_t bytes, void** inbox) {
  if (!inbox || bytes == 0) return CID_ERR_INVALID_ARGUMENT;
  *inbox = nullptr;
  cudaError_t e = cudaMalloc(inbox, bytes);
  if (e != cudaSuccess) return record_cuda_error(e);
  e = cudaMemset(*inbox, 0, bytes);  // flags 0: no epoch published yet
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(*inbox);
    *inbox = nullptr;
    return record_cuda_error(e);
  }
  return CID_OK;
}

extern "C" int cid_peer_inbox_free(void* inbox) {
  if (!inbox) return CID_OK;
  return record_cuda_error(cudaFree(inbox));
}

extern "C" int cid_peer_inbox_export(void* inbox, unsigned char handle[64]) {
  if (!inbox || !handle) return CID_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, inbox);
  if (e != cudaSuccess) return record_cuda_error(e);
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, sizeof(h));
  return CID_OK;
}

extern "C" int cid_peer_inbox_import(const unsigned char handle[64], void** peer_inbox) {
  if (!handle || !peer_inbox) return CID_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *peer_inbox = nullptr;
  return record_cuda_error(
      cudaIpcOpenMemHandle(peer_inbox, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int cid_peer_inbox_release(void* peer_inbox) {
  if (!peer_inbox) return CID_OK;
  return record_cuda_error(cudaIpcCloseMemHandle(peer_inbox));
}

extern "C" int cid_display_shard_records_to_peers(
    cid_dtype_t dtype, const void* logits, int64_t row_stride, const int64_t* token_ids,
    int64_t rows, int64_t shard_vocab, int64_t vocab_offset, int64_t total_vocab, int rank,
    int world, void* const* inboxes, int64_t rows_capacity, uint32_t epoch, uint32_t* status,
    void* stream) {
  int rc = check_logits(dtype, logits, row_stride, rows, shard_vocab);
  if (rc != CID_OK) return rc;
  if (!shard_range_ok(shard_vocab, vocab_offset, total_vocab)) return CID_ERR_INVALID_ARGUMENT;
  rc = check_peers(rows, rank, world, inboxes, rows_capacity);
  if (rc != CID_OK) return rc;
  if (misaligned({{token_ids, 8}, {status, 4}})) return CID_ERR_MISALIGNED;
  if (any_null({logits, token_ids})) return CID_ERR_INVALID_ARGUMENT;
  StatsParams prm = {};
  prm.logits = logits;
  prm.row_stride = row_stride;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.vocab = shard_vocab;
  prm.status = status;
  prm.tokens = 1;
  prm.vocab_offset = vocab_offset;
  prm.total_vocab = total_vocab;
  // the statistics kernel stores each record into this rank's slot of every
  // inbox, its own and (over NVLink) the other ranks', as it finishes the row
  prm.records = inbox_records(inboxes[rank], world, rows_capacity, epoch & 1u, rank);
  prm.records_v4 = 1;  // inbox slots are 16-byte aligned (check_peers)
  PeerSlots slots = {};
  for (int q = 0; q < world; ++q) {
    slots.flags[q] = inbox_flags(inboxes[q], world, rows_capacity) + rank;
    if (q != rank)
      prm.peer_records[prm.peers++] =
          inbox_records(inboxes[q], world, rows_capacity, epoch & 1u, rank);
  }
  rc = dispatch_stats<false, Mode::kRecord>(dtype, prm, as_stream(stream));
  if (rc != CID_OK) return rc;
  // a plain launch: it starts once every record store above has completed
  return launch_pdl(publish_epoch_kernel, dim3(1), dim3(32), 0, as_stream(stream), slots, world,
                    epoch);
}

extern "C" int cid_display_combine_inbox(void* inbox, int world,
                                         const int64_t* shard_offsets_host,
                                         const int64_t* token_ids, int64_t rows,
                                         int64_t rows_capacity, uint32_t epoch,
                                         double wait_seconds, float* confidence,
                                         int64_t* predicted, float* current_confidence,
                                         uint32_t* status, void* stream) {
  CombineParams prm = {};
  int rc = check_offsets(shard_offsets_host, world, kMaxPeers, prm.offsets);
  if (rc != CID_OK) return rc;
  if (rows < 1 || rows > rows_capacity || rows_capacity > kMaxRows ||
      !(wait_seconds > 0.0 && wait_seconds <= 60.0))
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{inbox, 16}}) ||
      stats_outputs_misaligned(token_ids, confidence, predicted, current_confidence, status))
    return CID_ERR_MISALIGNED;
  if (any_null({inbox, token_ids, confidence, predicted, current_confidence}))
    return CID_ERR_INVALID_ARGUMENT;
  prm.records = inbox_records(inbox, world, rows_capacity, epoch & 1u, 0);
  prm.stride = rows_capacity;
  prm.world = world;
  prm.ids = token_ids;
  prm.rows = rows;
  prm.confidence = confidence;
  prm.predicted = predicted;
  prm.current = current_confidence;
  prm.status = status;
  const int threads = 256;
  const int64_t blocks = (rows + threads - 1) / threads;
  uint32_t* flags = inbox_flags(inbox, world, rows_capacity);
  uint32_t* verdict = flags + kVerdictWord;
  rc = launch_pdl(wait_inbox_kernel, dim3(1), dim3(32), 0, as_stream(stream),
                  static_cast<const uint32_t*>(flags), verdict, world, epoch,
                  static_cast<unsigned long long>(wait_seconds * 1e9), status);
  if (rc != CID_OK) return rc;
  return launch_pdl(combine_inbox_kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0,
                    as_stream(stream), prm, static_cast<const uint32_t*>(flags),
                    static_cast<const uint32_t*>(verdict), epoch);
}

extern "C" int cid_peer_push_records(const cid_shard_record_t* records, int64_t rows, int rank,
                                     int world, void* const* inboxes, int64_t rows_capacity,
                                     uint32_t epoch, void* stream) {
  int rc = check_peers(rows, rank, world, inboxes, rows_capacity);
  if (rc != CID_OK) return rc;
  if (misaligned({{records, 4}})) return CID_ERR_MISALIGNED;
  if (any_null({records})) return CID_ERR_INVALID_ARGUMENT;
  PeerSlots slots = {};
  for (int q = 0; q < world; ++q) {
    slots.dst[q] = inbox_records(inboxes[q], world, rows_capacity, epoch & 1u, rank);
    slots.flags[q] = inbox_flags(inboxes[q], world, rows_capacity) + rank;
  }
  const int threads = 256;
  const int64_t blocks = (rows + threads - 1) / threads;
  push_records_kernel<<<static_cast<unsigned>(blocks), threads, 0, as_stream(stream)>>>(
      records, slots, world, rows);
  rc = launch_result();
  if (rc != CID_OK) return rc;
  return launch_pdl(publish_epoch_kernel, dim3(1), dim3(32), 0, as_stream(stream), slots, world,
                    epoch);
}
