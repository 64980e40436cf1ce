/*
 * CPU oracle for the cid-engine display-refinement path — TEST INFRASTRUCTURE
 * ONLY (see cid_oracle.h).  Each function restates one reference CPU
 * operator; citations are path:line inside fwerkor/cid-engine v1.1.0.
 *
 * Rounding model.  ATen evaluates float16/bfloat16 elementwise ops in float
 * and rounds the result to the storage type; float32 ops round once.  Basic
 * operations (+ - * / sqrt) are evaluated here in double and rounded to the
 * storage type, which gives the same float32 result (double carries more than
 * 2p+2 bits, so the double rounding is innocuous for these operations).
 * Transcendentals (exp, cos) are evaluated in double and rounded to float:
 * this is the correctly rounded value except in vanishingly rare cases, while
 * ATen's vectorised versions carry up to 1 ulp of error; the tests allow for
 * this with a tolerance wherever a transcendental reaches a float output.
 */
#include "cid_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* scalar type helpers                                                       */
/* ------------------------------------------------------------------------ */

static float bf16_to_float(uint16_t bits) {
  uint32_t u = (uint32_t)bits << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t float_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float f16_to_float(uint16_t bits) {
  _Float16 h;
  memcpy(&h, &bits, 2);
  return (float)h;
}

static uint16_t float_to_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t bits;
  memcpy(&bits, &h, 2);
  return bits;
}

/* Value of element i of a floating (or integer/bool) array as double. */
static double load(int dtype, const void* p, int64_t i) {
  switch (dtype) {
    case CID_DT_F32: return ((const float*)p)[i];
    case CID_DT_F64: return ((const double*)p)[i];
    case CID_DT_F16: return f16_to_float(((const uint16_t*)p)[i]);
    case CID_DT_BF16: return bf16_to_float(((const uint16_t*)p)[i]);
    case CID_DT_BOOL: return ((const uint8_t*)p)[i] ? 1.0 : 0.0;
    case CID_DT_U8: return ((const uint8_t*)p)[i];
    case CID_DT_I8: return ((const int8_t*)p)[i];
    case CID_DT_I16: return ((const int16_t*)p)[i];
    case CID_DT_I32: return ((const int32_t*)p)[i];
    case CID_DT_I64: return (double)((const int64_t*)p)[i];
    default: return NAN;
  }
}

/* x rounded to the storage type `dtype` (returned as double). */
static double rnd(int dtype, double x) {
  switch (dtype) {
    case CID_DT_F64: return x;
    case CID_DT_F32: return (float)x;
    case CID_DT_F16: return f16_to_float(float_to_f16((float)x));
    case CID_DT_BF16: return bf16_to_float(float_to_bf16((float)x));
    default: return x;
  }
}

static void store(int dtype, void* p, int64_t i, double x) {
  switch (dtype) {
    case CID_DT_F64: ((double*)p)[i] = x; break;
    case CID_DT_F32: ((float*)p)[i] = (float)x; break;
    case CID_DT_F16: ((uint16_t*)p)[i] = float_to_f16((float)x); break;
    case CID_DT_BF16: ((uint16_t*)p)[i] = float_to_bf16((float)x); break;
    default: break;
  }
}

/* Truthiness of `tensor.to(torch.bool)`: any non-zero value (NaN included). */
static int truthy(int dtype, const void* p, int64_t i) {
  double v = load(dtype, p, i);
  return v != 0.0 || isnan(v);
}

/* float32 sigmoid as ATen evaluates it: 1 / (1 + exp(-x)), each step rounded
 * to float32 (aten/src/ATen/native/cpu/UnaryOpsKernel.cpp sigmoid kernel). */
static float sigmoid_f32(float x) {
  float e = (float)exp(-(double)x);
  float d = 1.0f + e;
  return 1.0f / d;
}

/* ATen max(-1)/argmax semantics: NaN wins (first NaN), otherwise the largest
 * value, first index on ties.  Values are given as float32. */
static int64_t first_argmax_f(const float* v, int64_t n, float* value) {
  int64_t best = 0;
  float bv = v[0];
  for (int64_t i = 1; i < n; ++i) {
    if (isnan(bv)) break;
    if (isnan(v[i]) || v[i] > bv) {
      bv = v[i];
      best = i;
    }
  }
  if (value) *value = bv;
  return best;
}

/* Same, reading element k of a strided small vector of any float dtype. */
static int64_t first_argmax_dt(int dtype, const void* p, int64_t base,
                               int64_t n) {
  int64_t best = 0;
  double bv = load(dtype, p, base);
  for (int64_t i = 1; i < n; ++i) {
    if (isnan(bv)) break;
    double x = load(dtype, p, base + i);
    if (isnan(x) || x > bv) {
      bv = x;
      best = i;
    }
  }
  return best;
}

/* ------------------------------------------------------------------------ */
/* display_token_statistics — csrc/cpu/display_stats.cpp:14-126 (f32/f16/   */
/* bf16), csrc/ops.cpp:446-474 (other dtypes: logits.to(float) first).      */
/* ------------------------------------------------------------------------ */

static void stats_row(const float* x, int64_t vocab, int64_t id, float* conf,
                      int64_t* pred, float* cur) {
  float m;
  *pred = first_argmax_f(x, vocab, &m); /* display_stats.cpp:86-88 */
  double s = 0.0;
  for (int64_t v = 0; v < vocab; ++v) s += exp((double)x[v] - (double)m);
  /* display_stats.cpp:44-47: conf = 1/sum, cur = exp(x_id - max)/sum.  A
   * non-finite max (NaN, +inf, or an all -inf row) makes the sum NaN. */
  if (!isfinite(m)) s = NAN;
  *conf = (float)(1.0 / s);
  *cur = (float)(exp((double)x[id] - (double)m) / s);
}

/* Reference-order statistics.  The reference's CPU kernel sums
 * exp(x - max) in float32 through at::vec::map_reduce_all
 * (csrc/cpu/display_stats.cpp:37-42).  That translation unit is built
 * without ATen's CPU_CAPABILITY dispatch macros, so Vectorized<float> is
 * ATen's generic 32-byte vector: 8 float lanes, exp() applied lane by lane
 * with std::exp (libm expf), lanes summed element-wise, and the final
 * horizontal sum taken serially, lane 0 + lane 1 + ... + lane 7
 * (ATen/cpu/vec/functional_base.h map_reduce_all / vec_reduce_all).  For
 * f16/bf16 logits the reduced-float overload
 * (ATen/cpu/vec/functional_bfloat16.h) loads 16 values, converts them to two
 * float vectors with one accumulator each, and adds the second accumulator
 * into the first before the serial horizontal sum.  Tails shorter than a
 * vector update only their own lanes; rows shorter than a vector sum their
 * lanes serially.  Evaluated in this order with the same expf, the float32
 * result reproduces the reference's own rounding, which the double-precision
 * stats_row above does not (it returns the exactly rounded value). */
enum { REF_LANES = 8 };

static float ref_serial_lanes(const float* lanes, int64_t n) {
  float r = lanes[0];
  for (int64_t j = 1; j < n; ++j) r += lanes[j];
  return r;
}

static float ref_sum_f32(const float* x, int64_t n, float m) {
  float acc[REF_LANES];
  if (n < REF_LANES) {
    for (int64_t j = 0; j < n; ++j) acc[j] = expf(x[j] - m);
    return ref_serial_lanes(acc, n);
  }
  for (int j = 0; j < REF_LANES; ++j) acc[j] = expf(x[j] - m);
  int64_t d = REF_LANES;
  const int64_t body = n - n % REF_LANES;
  for (; d < body; d += REF_LANES)
    for (int j = 0; j < REF_LANES; ++j) acc[j] += expf(x[d + j] - m);
  for (int64_t j = 0; j < n - d; ++j) acc[j] += expf(x[d + j] - m);
  return ref_serial_lanes(acc, REF_LANES);
}

static float ref_sum_reduced(const float* x, int64_t n, float m) {
  enum { W = REF_LANES, B = 2 * REF_LANES };
  float a0[W], a1[W];
  if (n < B) {
    if (n > W) {
      for (int j = 0; j < W; ++j) a0[j] = expf(x[j] - m);
      for (int64_t j = 0; j < n - W; ++j) a0[j] += expf(x[W + j] - m);
      return ref_serial_lanes(a0, W);
    }
    for (int64_t j = 0; j < n; ++j) a0[j] = expf(x[j] - m);
    return ref_serial_lanes(a0, n);
  }
  for (int j = 0; j < W; ++j) {
    a0[j] = expf(x[j] - m);
    a1[j] = expf(x[W + j] - m);
  }
  int64_t d = B;
  const int64_t body = n - n % B;
  for (; d < body; d += B)
    for (int j = 0; j < W; ++j) {
      a0[j] += expf(x[d + j] - m);
      a1[j] += expf(x[d + W + j] - m);
    }
  const int64_t r = n - d;
  if (r > W) {
    for (int j = 0; j < W; ++j) a0[j] += expf(x[d + j] - m);
    for (int64_t j = 0; j < r - W; ++j) a1[j] += expf(x[d + W + j] - m);
  } else {
    for (int64_t j = 0; j < r; ++j) a0[j] += expf(x[d + j] - m);
  }
  for (int j = 0; j < W; ++j) a0[j] += a1[j];
  return ref_serial_lanes(a0, W);
}

static void stats_row_reference_order(int dtype, const float* x, int64_t vocab,
                                      int64_t id, float* conf, int64_t* pred,
                                      float* cur) {
  float m;
  *pred = first_argmax_f(x, vocab, &m); /* display_stats.cpp:86-88 */
  const float s = dtype == CID_DT_F32 ? ref_sum_f32(x, vocab, m)
                                      : ref_sum_reduced(x, vocab, m);
  *conf = 1.0f / s;                    /* display_stats.cpp:46 */
  *cur = expf(x[id] - m) / s;          /* display_stats.cpp:44-47 */
}

static void row_to_float(int dtype, const void* logits, int64_t row,
                         int64_t vocab, float* dst) {
  for (int64_t v = 0; v < vocab; ++v)
    dst[v] = (float)load(dtype, logits, row * vocab + v);
}

static int stats_rows(int dtype, const void* logits, const int64_t* ids,
                      int64_t rows, int64_t vocab, float* confidence,
                      int64_t* predicted, float* current, int reference_order) {
  if (vocab <= 0) return -1; /* ops.cpp:456 */
  int bad = 0;
#pragma omp parallel
  {
    float* buf = (float*)malloc(sizeof(float) * (size_t)vocab);
#pragma omp for schedule(static) reduction(| : bad)
    for (int64_t r = 0; r < rows; ++r) {
      int64_t id = ids[r];
      if (id < 0 || id >= vocab) { /* display_stats.cpp:32-34 IndexError */
        bad |= 1;
        continue;
      }
      row_to_float(dtype, logits, r, vocab, buf);
      if (reference_order)
        stats_row_reference_order(dtype, buf, vocab, id, &confidence[r],
                                  &predicted[r], &current[r]);
      else
        stats_row(buf, vocab, id, &confidence[r], &predicted[r], &current[r]);
    }
    free(buf);
  }
  return bad ? -2 : 0;
}

int cid_oracle_display_stats(int dtype, const void* logits, const int64_t* ids,
                             int64_t rows, int64_t vocab, float* confidence,
                             int64_t* predicted, float* current) {
  return stats_rows(dtype, logits, ids, rows, vocab, confidence, predicted,
                    current, 0);
}

/* f32/f16/bf16 logits take the reference's CPU kernel
 * (csrc/cpu/display_stats.cpp:14-50) in its own float32 summation order;
 * other dtypes go through the reference's composite (csrc/ops.cpp:446-474,
 * ATen logsumexp), whose order depends on the host's SIMD dispatch, so
 * there this returns the exactly rounded value like
 * cid_oracle_display_stats. */
int cid_oracle_display_stats_reference_order(int dtype, const void* logits,
                                             const int64_t* ids, int64_t rows,
                                             int64_t vocab, float* confidence,
                                             int64_t* predicted,
                                             float* current) {
  const int ref = dtype == CID_DT_F32 || dtype == CID_DT_F16 || dtype == CID_DT_BF16;
  return stats_rows(dtype, logits, ids, rows, vocab, confidence, predicted,
                    current, ref);
}

/* display_token_statistics_with_repetition — csrc/ops.cpp:477-552.  The
 * adjacent run on each side (ops.cpp:523-542), skipping mask/EOS ids
 * (ops.cpp:510-513), adds count*log(multiplier) to that id's logit; both
 * sides accumulate into one count when they carry the same id
 * (ops.cpp:514-519).  The adjusted logit is float32(x + float32(c*log m)):
 * a float tensor plus a double scalar (ops.cpp:544-547). */
int cid_oracle_display_stats_repetition(
    int dtype, const void* logits, const int64_t* ids, int64_t batch,
    int64_t tokens, int64_t vocab, int64_t mask_id, int has_eos, int64_t eos_id,
    double multiplier, float* confidence, int64_t* predicted, float* current) {
  if (!(multiplier > 0.0 && multiplier <= 1.0)) return -1; /* ops.cpp:484 */
  if (multiplier == 1.0 || tokens <= 1) /* ops.cpp:494-496 */
    return cid_oracle_display_stats(dtype, logits, ids, batch * tokens, vocab,
                                    confidence, predicted, current);
  if (vocab <= 0) return -1;
  const double log_m = log(multiplier);
  int bad = 0;
#pragma omp parallel
  {
    float* buf = (float*)malloc(sizeof(float) * (size_t)vocab);
#pragma omp for schedule(static) reduction(| : bad)
    for (int64_t r = 0; r < batch * tokens; ++r) {
      const int64_t b = r / tokens, p = r % tokens;
      const int64_t* row_ids = ids + b * tokens;
      int64_t run_id[2];
      int64_t run_n[2];
      int nruns = 0;
      for (int side = 0; side < 2; ++side) {
        int64_t q = side == 0 ? p - 1 : p + 1;
        if (q < 0 || q >= tokens) continue;
        int64_t tok = row_ids[q];
        int64_t n = 1;
        if (side == 0)
          for (int64_t c = p - 2; c >= 0 && row_ids[c] == tok; --c) ++n;
        else
          for (int64_t c = p + 2; c < tokens && row_ids[c] == tok; ++c) ++n;
        if (tok == mask_id || (has_eos && tok == eos_id)) continue;
        if (nruns == 1 && run_id[0] == tok) {
          run_n[0] += n;
        } else {
          run_id[nruns] = tok;
          run_n[nruns] = n;
          ++nruns;
        }
      }
      row_to_float(dtype, logits, r, vocab, buf);
      int oob = 0;
      for (int k = 0; k < nruns; ++k) {
        if (run_id[k] < 0 || run_id[k] >= vocab) {
          oob = 1;
          continue;
        }
        float delta = (float)((double)run_n[k] * log_m);
        buf[run_id[k]] = (float)((double)buf[run_id[k]] + (double)delta);
      }
      int64_t id = ids[r];
      if (oob || id < 0 || id >= vocab) {
        bad |= 1;
        continue;
      }
      stats_row(buf, vocab, id, &confidence[r], &predicted[r], &current[r]);
    }
    free(buf);
  }
  return bad ? -2 : 0;
}

/* ------------------------------------------------------------------------ */
/* refine_display_from_statistics — csrc/refine.cpp:93-429                   */
/* ------------------------------------------------------------------------ */

typedef struct {
  int64_t anchor;
  float gain;
  int64_t neg_abs_growth;
  int64_t start;
  int64_t delete_count;
  int64_t insert_from; /* inserted tokens are predicted[start, insert_to) */
  int64_t insert_to;
  int valid;
} edit_t;

/* refine.cpp:30-43: strict lexicographic (anchor, gain, -|growth|, start). */
static int edit_better(const edit_t* a, const edit_t* b) {
  if (a->anchor != b->anchor) return a->anchor > b->anchor;
  if (a->gain != b->gain) return a->gain > b->gain;
  if (a->neg_abs_growth != b->neg_abs_growth)
    return a->neg_abs_growth > b->neg_abs_growth;
  return a->start > b->start;
}

/* refine.cpp:45-57 */
static int64_t common_prefix(const int64_t* a, int64_t a_len, int64_t a0,
                             const int64_t* b, int64_t b_len, int64_t b0) {
  int64_t n = 0;
  while (a0 + n < a_len && b0 + n < b_len && a[a0 + n] == b[b0 + n]) ++n;
  return n;
}

/* refine.cpp:59-91: first position q in (start, maximum] with
 * seq[q, q+klen) == key; -1 when none. */
static int64_t next_match(const int64_t* seq, int64_t seq_len,
                          const int64_t* key, int64_t klen, int64_t start,
                          int64_t maximum) {
  int64_t last = maximum < seq_len - klen ? maximum : seq_len - klen;
  for (int64_t q = start + 1; q <= last; ++q) {
    int ok = 1;
    for (int64_t k = 0; k < klen && ok; ++k) ok = seq[q + k] == key[k];
    if (ok) return q;
  }
  return -1;
}

/* refine.cpp:93-218 */
static edit_t structural_edit(const int64_t* tok, const int64_t* pred,
                              const float* gain, int64_t L, int64_t eos_pos,
                              double revision_fraction, double margin,
                              int64_t mask_id, int64_t eos_id) {
  edit_t best;
  memset(&best, 0, sizeof(best));
  if (eos_pos <= 0) return best;
  const int64_t active_len = eos_pos + 1; /* active = tok[0, eos_pos] */
  int64_t budget = (int64_t)ceil((double)eos_pos * revision_fraction);
  if (budget < 1) budget = 1;
  if (budget > 32) budget = 32;
  for (int64_t s = 0; s < eos_pos; ++s) {
    if (pred[s] == tok[s] || (double)gain[s] < margin) continue;
    /* insertion: refine.cpp:123-165 */
    int64_t klen = active_len - s < 3 ? active_len - s : 3;
    int64_t q = next_match(pred, L, tok + s, klen, s, s + budget);
    if (q >= 0) {
      int valid = 1;
      for (int64_t k = s; k < q; ++k)
        if (pred[k] == mask_id || pred[k] == eos_id) valid = 0;
      if (valid) {
        int64_t anchor = common_prefix(pred, L, q, tok, active_len, s);
        int64_t growth = q - s;
        if (anchor >= 2 && (double)gain[s] >= margin &&
            eos_pos + 1 + growth <= L) {
          edit_t c = {anchor, gain[s], -growth, s, 0, s, q, 1};
          if (!best.valid || edit_better(&c, &best)) best = c;
        }
      }
    }
    /* deletion: refine.cpp:167-201 */
    int64_t dlen = L - s < 3 ? L - s : 3;
    if (dlen < 2) continue;
    int64_t lim = eos_pos - 1 < s + budget ? eos_pos - 1 : s + budget;
    int64_t r = next_match(tok, active_len, pred + s, dlen, s, lim);
    if (r >= 0) {
      int64_t del = r - s;
      int64_t anchor = common_prefix(pred, L, s, tok, active_len, r);
      if (anchor >= 2 && (double)gain[s] >= margin &&
          eos_pos + 1 - del <= L) {
        edit_t c = {anchor, gain[s], -del, s, del, s, s, 1};
        if (!best.valid || edit_better(&c, &best)) best = c;
      }
    }
  }
  return best;
}

/* Positions (taken from `pos`, n of them) ordered by key descending with the
 * original order kept among equal keys — std::stable_sort with `>`
 * (refine.cpp:332-337, 369-374). */
static void stable_desc(int64_t* pos, int64_t n, const float* key,
                        int64_t* tmp) {
  /* bottom-up merge sort, stable */
  for (int64_t width = 1; width < n; width *= 2) {
    for (int64_t lo = 0; lo < n; lo += 2 * width) {
      int64_t mid = lo + width < n ? lo + width : n;
      int64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      int64_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) {
        if (key[pos[j]] > key[pos[i]])
          tmp[k++] = pos[j++];
        else
          tmp[k++] = pos[i++];
      }
      while (i < mid) tmp[k++] = pos[i++];
      while (j < hi) tmp[k++] = pos[j++];
    }
    memcpy(pos, tmp, sizeof(int64_t) * (size_t)n);
  }
}

int cid_oracle_refine(const int64_t* ids, const float* confidence,
                      const int64_t* predicted, const float* current,
                      int64_t batch, int64_t tokens, int64_t mask_id,
                      int has_eos, int64_t eos_id, double reveal_fraction,
                      double revision_fraction, double revision_margin,
                      int64_t* out) {
  /* refine.cpp:240-244 */
  if (!(reveal_fraction >= 0.0 && reveal_fraction <= 1.0)) return -1;
  if (!(revision_fraction >= 0.0 && revision_fraction <= 1.0)) return -1;
  if (!(revision_margin >= 0.0)) return -1;
  const int64_t L = tokens;
  const float margin_f32 = (float)revision_margin; /* refine.cpp:357 */
#pragma omp parallel
  {
    float* gain = (float*)malloc(sizeof(float) * (size_t)(L + 1));
    int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)(L + 1));
    int64_t* tmp = (int64_t*)malloc(sizeof(int64_t) * (size_t)(L + 1));
#pragma omp for schedule(dynamic, 4)
    for (int64_t b = 0; b < batch; ++b) {
      const int64_t* tok = ids + b * L;
      const int64_t* pred = predicted + b * L;
      const float* conf = confidence + b * L;
      const float* cur = current + b * L;
      int64_t* res = out + b * L;
      memcpy(res, tok, sizeof(int64_t) * (size_t)L);
      for (int64_t i = 0; i < L; ++i) gain[i] = conf[i] - cur[i]; /* :277 */

      int64_t eos_pos = -1; /* refine.cpp:280-288 */
      if (has_eos)
        for (int64_t i = 0; i < L; ++i)
          if (tok[i] == eos_id) {
            eos_pos = i;
            break;
          }

      if (eos_pos >= 0 && revision_fraction != 0.0) { /* refine.cpp:290-319 */
        edit_t e = structural_edit(tok, pred, gain, L, eos_pos,
                                   revision_fraction, revision_margin, mask_id,
                                   eos_id);
        if (e.valid) {
          int64_t w = 0;
          for (int64_t i = 0; i < e.start; ++i) res[w++] = tok[i];
          for (int64_t i = e.insert_from; i < e.insert_to; ++i)
            res[w++] = pred[i];
          for (int64_t i = e.start + e.delete_count; i <= eos_pos; ++i)
            res[w++] = tok[i];
          while (w < L) res[w++] = mask_id;
          continue;
        }
      }

      const int64_t stop = eos_pos >= 0 ? eos_pos : L; /* refine.cpp:321 */
      /* reveal: refine.cpp:322-342 */
      int64_t n = 0;
      for (int64_t i = 0; i < stop; ++i)
        if (tok[i] == mask_id) pos[n++] = i;
      if (n > 0 && reveal_fraction != 0.0) {
        int64_t count = (int64_t)ceil((double)n * reveal_fraction);
        stable_desc(pos, n, conf, tmp);
        for (int64_t k = 0; k < count; ++k) res[pos[k]] = pred[pos[k]];
      }
      if (revision_fraction == 0.0) continue; /* refine.cpp:344 */
      /* revision: refine.cpp:345-379 */
      int64_t visible = 0;
      n = 0;
      for (int64_t i = 0; i < stop; ++i) {
        if (tok[i] == mask_id) continue;
        ++visible;
        if (pred[i] != tok[i] && gain[i] >= margin_f32) pos[n++] = i;
      }
      if (n > 0) {
        int64_t count = (int64_t)ceil((double)visible * revision_fraction);
        if (count > n) count = n;
        stable_desc(pos, n, gain, tmp);
        for (int64_t k = 0; k < count; ++k) res[pos[k]] = pred[pos[k]];
      }
      /* EOS expansion: refine.cpp:381-406 */
      if (eos_pos >= 0 && eos_pos + 1 < L) {
        if (pred[eos_pos] != eos_id &&
            (double)gain[eos_pos] >= revision_margin) {
          int64_t base = eos_pos + 1 > 1 ? eos_pos + 1 : 1;
          int64_t budget = (int64_t)ceil((double)base * reveal_fraction);
          if (budget < 1) budget = 1;
          int64_t new_eos = eos_pos + budget < L - 1 ? eos_pos + budget : L - 1;
          for (int64_t t = eos_pos + 1; t <= new_eos; ++t)
            if (pred[t] == eos_id) {
              new_eos = t;
              break;
            }
          for (int64_t t = eos_pos; t < new_eos; ++t) res[t] = pred[t];
          res[new_eos] = eos_id;
        }
      }
    }
    free(gain);
    free(pos);
    free(tmp);
  }
  if (has_eos) /* refine.cpp:410-423 */
    for (int64_t b = 0; b < batch; ++b) {
      int64_t* res = out + b * L;
      for (int64_t i = 0; i < L; ++i)
        if (res[i] == eos_id) {
          for (int64_t j = i + 1; j < L; ++j) res[j] = mask_id;
          break;
        }
    }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* prefix_allocation_mask — csrc/ops.cpp:41-65                               */
/* ------------------------------------------------------------------------ */

static void prefix_row(int occ_dtype, const void* occ, int logit_dtype,
                       const void* logits, int64_t base, int64_t slots,
                       float thr, int64_t max_allocations, uint8_t* out) {
  int blocked = 0;
  int64_t rank = 0;
  for (int64_t s = 0; s < slots; ++s) {
    int occupied = truthy(occ_dtype, occ, base + s);       /* :58 */
    float x = (float)load(logit_dtype, logits, base + s);  /* :59 to(kFloat) */
    int eligible = sigmoid_f32(x) >= thr;                  /* :59 ge */
    int is_free = !occupied;
    if (is_free && !eligible) blocked = 1;                 /* :61 cumsum>0 */
    int sel = is_free && eligible && !blocked;             /* :62 */
    if (sel) ++rank;                                       /* :63 */
    out[base + s] = (uint8_t)(sel && rank <= max_allocations); /* :64 */
  }
}

int cid_oracle_prefix_allocation(int occ_dtype, const void* occupancy,
                                 int logit_dtype, const void* logits,
                                 int64_t batch, int64_t slots, double threshold,
                                 int64_t max_allocations, uint8_t* out) {
  if (!(threshold >= 0.0 && threshold <= 1.0)) return -1; /* ops.cpp:50 */
  if (max_allocations <= 0) return -1;                    /* ops.cpp:51 */
  /* `sigmoid >= threshold`: a float32 tensor against a double scalar is
   * evaluated in float32, so the threshold is rounded to float32. */
  const float thr = (float)threshold;
  for (int64_t b = 0; b < batch; ++b)
    prefix_row(occ_dtype, occupancy, logit_dtype, logits, b * slots, slots, thr,
               max_allocations, out);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* rollout_slot_transition — csrc/ops.cpp:184-256                            */
/* ------------------------------------------------------------------------ */

int cid_oracle_rollout(int occ_dtype, const void* occupancy, int dtype,
                       const void* allocation_logits,
                       const void* lifecycle_logits,
                       const void* revision_logits,
                       const void* input_lifecycle, int64_t batch,
                       int64_t slots, int64_t lifecycles, int64_t revisions,
                       double threshold, int64_t max_allocations,
                       int64_t retired_index, uint8_t* next_occupancy,
                       int64_t* lifecycle_index, int64_t* revision_index,
                       int64_t* input_index, uint8_t* input_present,
                       uint8_t* live) {
  if (retired_index < 0 || retired_index >= lifecycles) return -1; /* :222 */
  if (!(threshold >= 0.0 && threshold <= 1.0)) return -1;          /* :225 */
  if (max_allocations <= 0) return -1;                             /* :226 */
  if (lifecycles <= 0 || revisions <= 0) return -1; /* max(-1) of empty dim */
  const int64_t n = batch * slots;
  uint8_t* occ = (uint8_t*)malloc((size_t)(n > 0 ? n : 1));
  uint8_t* alloc = (uint8_t*)malloc((size_t)(n > 0 ? n : 1));
  for (int64_t i = 0; i < n; ++i) occ[i] = (uint8_t)truthy(occ_dtype, occupancy, i);
  /* :228-233 prefix allocation over the boolean occupancy */
  cid_oracle_prefix_allocation(CID_DT_BOOL, occ, dtype, allocation_logits,
                               batch, slots, threshold, max_allocations, alloc);
  for (int64_t i = 0; i < n; ++i) {
    int o = occ[i];
    int nxt = o || alloc[i];                                         /* :234 */
    int64_t li = first_argmax_dt(dtype, lifecycle_logits, i * lifecycles,
                                 lifecycles);                        /* :235 */
    int64_t ri = first_argmax_dt(dtype, revision_logits, i * revisions,
                                 revisions);                         /* :236 */
    int64_t ii = first_argmax_dt(dtype, input_lifecycle, i * lifecycles,
                                 lifecycles);                        /* :237 */
    int present = 0;                                             /* :238-239 */
    for (int64_t k = 0; k < lifecycles; ++k) {
      double v = load(dtype, input_lifecycle, i * lifecycles + k);
      if (v != 0.0 || isnan(v)) present = 1;
    }
    int prev_retired = o && ii == retired_index;                     /* :240 */
    int newly = nxt && !o;                                           /* :242 */
    int pred_retired = li == retired_index;                          /* :244 */
    next_occupancy[i] = (uint8_t)nxt;
    lifecycle_index[i] = li;
    revision_index[i] = ri;
    input_index[i] = ii;
    input_present[i] = (uint8_t)present;
    live[i] = (uint8_t)(nxt && !prev_retired && (!pred_retired || newly));
  }
  free(occ);
  free(alloc);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* live_slot_occupancy — csrc/ops.cpp:12-39                                  */
/* ------------------------------------------------------------------------ */

static double clamp01(double x) {
  if (isnan(x)) return x; /* at::clamp propagates NaN */
  return x < 0.0 ? 0.0 : (x > 1.0 ? 1.0 : x);
}

int cid_oracle_live_occupancy(int dtype, const void* occupancy,
                              const void* lifecycle, int64_t rows,
                              int64_t features, int64_t retired_index,
                              void* out) {
  if (lifecycle && (retired_index < 0 || retired_index >= features))
    return -1; /* :31-33 */
  for (int64_t r = 0; r < rows; ++r) {
    double occ = clamp01(load(dtype, occupancy, r)); /* :20 */
    if (!lifecycle) {
      store(dtype, out, r, occ);
      continue;
    }
    double ret = clamp01(load(dtype, lifecycle, r * features + retired_index));
    double keep = rnd(dtype, 1.0 - ret);       /* :38 (1.0 - retired) */
    store(dtype, out, r, rnd(dtype, occ * keep)); /* :38 occupancy * ... */
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* materialize_cell_snapshot — csrc/ops.cpp:556-615                          */
/* ------------------------------------------------------------------------ */

int cid_oracle_snapshot(int sem_dtype, const void* semantic, int64_t hidden,
                        int role_dtype, const void* roles, int64_t nroles,
                        int unc_dtype, const void* uncertainty, int noise_dtype,
                        const void* noise, int life_dtype, const void* lifecycle,
                        int64_t lifecycles, const uint8_t* selected,
                        const int64_t* indices, int64_t nindices, int64_t rows,
                        float* out) {
  for (int64_t k = 0; k < nindices; ++k) /* :596-601 */
    if (indices[k] < 0 || indices[k] >= hidden) return -3;
  if (lifecycles <= 0) return -1;
  const int64_t width = 4 + nroles + nindices;
  for (int64_t r = 0; r < rows; ++r) {
    float* o = out + r * width;
    o[0] = selected[r] ? 1.0f : 0.0f; /* :603 */
    /* :604-606 argmax of lifecycle.to(float) */
    float* tmp = (float*)malloc(sizeof(float) * (size_t)lifecycles);
    for (int64_t k = 0; k < lifecycles; ++k)
      tmp[k] = (float)load(life_dtype, lifecycle, r * lifecycles + k);
    o[1] = (float)first_argmax_f(tmp, lifecycles, NULL);
    free(tmp);
    o[2] = (float)load(unc_dtype, uncertainty, r);  /* :607 */
    o[3] = (float)load(noise_dtype, noise, r);      /* :608 */
    for (int64_t k = 0; k < nroles; ++k)            /* :609 sigmoid(float) */
      o[4 + k] = sigmoid_f32((float)load(role_dtype, roles, r * nroles + k));
    for (int64_t k = 0; k < nindices; ++k)          /* :610-611 */
      o[4 + nroles + k] =
          (float)load(sem_dtype, semantic, r * hidden + indices[k]);
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* masked_diffusion_corrupt_from_random — csrc/ops.cpp:394-444               */
/* ------------------------------------------------------------------------ */

int cid_oracle_masked_diffusion(const int64_t* clean, int ratio_dtype,
                                const void* ratio_random, int mask_dtype,
                                const void* mask_random, int64_t batch,
                                int64_t tokens, int64_t mask_id,
                                double min_ratio, double max_ratio,
                                int64_t* corrupted, uint8_t* masked,
                                float* ratio, float* metrics) {
  if (batch <= 0 || tokens <= 0) return -1; /* :406 */
  if (!(min_ratio > 0.0 && min_ratio <= max_ratio && max_ratio <= 1.0))
    return -1; /* :416-420 */
  /* :424-425: (max-min) is a double scalar times a float32 tensor, then a
   * double scalar plus that float32 tensor: two float32 roundings with the
   * scalars rounded to float32. */
  const float span = (float)(max_ratio - min_ratio);
  const float lo = (float)min_ratio;
  int64_t total_masked = 0;
  double ratio_sum = 0.0;
  for (int64_t b = 0; b < batch; ++b) {
    float rr = (float)load(ratio_dtype, ratio_random, b);
    float scaled = (float)((double)rr * (double)span);
    float mr = (float)((double)scaled + (double)lo);
    ratio[b] = mr;
    ratio_sum += mr;
    int64_t count = 0;
    int64_t argmin = 0;
    float umin = (float)load(mask_dtype, mask_random, b * tokens);
    for (int64_t t = 0; t < tokens; ++t) {
      float u = (float)load(mask_dtype, mask_random, b * tokens + t);
      int m = u < mr; /* :426 */
      masked[b * tokens + t] = (uint8_t)m;
      count += m;
      /* :432 min(1): first NaN, else first minimum */
      if (t > 0 && !isnan(umin) && (isnan(u) || u < umin)) {
        umin = u;
        argmin = t;
      }
    }
    if (count == 0) { /* :431-438 empty-row fallback */
      masked[b * tokens + argmin] = 1;
      count = 1;
    }
    total_masked += count;
    for (int64_t t = 0; t < tokens; ++t) /* :440 */
      corrupted[b * tokens + t] =
          masked[b * tokens + t] ? mask_id : clean[b * tokens + t];
  }
  /* :441-442 means, evaluated exactly and rounded once */
  metrics[0] = (float)((double)total_masked / (double)(batch * tokens));
  metrics[1] = (float)(ratio_sum / (double)batch);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* thought_corrupt_from_epsilon — csrc/ops.cpp:258-290                       */
/* ------------------------------------------------------------------------ */

int cid_oracle_thought(int sem_dtype, const void* semantic, int t_dtype,
                       const void* timesteps, int occ_dtype,
                       const void* occupancy, const void* epsilon,
                       int64_t rows, int64_t hidden, void* corrupted,
                       void* local_noise, void* masked_epsilon) {
  const double half_pi = 1.57079632679489661923;
  for (int64_t r = 0; r < rows; ++r) {
    const int occ = truthy(occ_dtype, occupancy, r); /* :283 */
    const double t = load(t_dtype, timesteps, r);
    /* :278-281 alpha = cos(t*pi/2)^2 in the timestep dtype, then cast to
     * the semantic dtype. */
    double arg = rnd(t_dtype, t * rnd(t_dtype == CID_DT_F64 ? CID_DT_F64
                                                            : CID_DT_F32,
                                      half_pi));
    double c = rnd(t_dtype, cos(arg));
    double alpha = rnd(sem_dtype, rnd(t_dtype, c * c));
    double sa = rnd(sem_dtype, sqrt(alpha));                 /* :282 */
    double one_minus = rnd(sem_dtype, 1.0 - alpha);
    double sb = rnd(sem_dtype, sqrt(one_minus));
    for (int64_t h = 0; h < hidden; ++h) {
      const int64_t i = r * hidden + h;
      double x = load(sem_dtype, semantic, i);
      double e = load(sem_dtype, epsilon, i);
      double v = rnd(sem_dtype, rnd(sem_dtype, sa * x) + rnd(sem_dtype, sb * e));
      store(sem_dtype, corrupted, i, occ ? v : 0.0);        /* :285 */
      store(sem_dtype, masked_epsilon, i, occ ? e : 0.0);   /* :286 */
    }
    store(sem_dtype, local_noise, r, occ ? rnd(sem_dtype, t) : 0.0); /* :287 */
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* display_corrupt_from_random — csrc/ops.cpp:292-391                        */
/* ------------------------------------------------------------------------ */

static int64_t floor_mod(int64_t a, int64_t m) {
  int64_t r = a % m;
  return (r != 0 && ((r < 0) != (m < 0))) ? r + m : r;
}

int cid_oracle_display_corrupt(const int64_t* ids, int t_dtype,
                               const void* timesteps, int elig_dtype,
                               const void* eligible, int rand_dtype,
                               const void* corruption_random, int repl_dtype,
                               const void* replacement_random,
                               const int64_t* replacement_offsets,
                               int64_t batch, int64_t tokens, int64_t mask_id,
                               int has_eos, int64_t eos_id, int64_t vocab,
                               double replacement_fraction, int64_t* corrupted,
                               int64_t* labels, uint8_t* masked,
                               uint8_t* replaced) {
  if (!(replacement_fraction >= 0.0 && replacement_fraction <= 1.0))
    return -1; /* :320-322 */
  const int replace = replacement_fraction > 0.0;
  /* :343-360; an empty replacement tensor has a null data pointer, so the
     presence check on empty inputs is left to the caller */
  if (replace && (vocab < 3 || (batch * tokens > 0 &&
                                (!replacement_random || !replacement_offsets))))
    return -1;
  const float repl_thr = (float)replacement_fraction;
  for (int64_t b = 0; b < batch; ++b) {
    const float t = (float)load(t_dtype, timesteps, b); /* :325 */
    int any_corrupt = 0, any_elig = 0;
    int64_t first_elig = 0;
    for (int64_t k = 0; k < tokens; ++k) {
      const int64_t i = b * tokens + k;
      int el = truthy(elig_dtype, eligible, i);
      float u = (float)load(rand_dtype, corruption_random, i);
      int c = (u < t) && el; /* :326-328 */
      masked[i] = (uint8_t)c; /* holds corrupted_positions for now */
      any_corrupt |= c;
      if (el && !any_elig) first_elig = k; /* :333-334 argmax of long mask */
      any_elig |= el;
    }
    /* :330-337 fallback on the first eligible position */
    if (!any_corrupt && t > 0.0f && any_elig) masked[b * tokens + first_elig] = 1;
    for (int64_t k = 0; k < tokens; ++k) {
      const int64_t i = b * tokens + k;
      const int pos = masked[i];
      const int64_t id = ids[i];
      int rep = 0;
      int64_t value = id;
      if (replace) {
        rep = pos && ((float)load(repl_dtype, replacement_random, i) < repl_thr);
        /* :364, the int64 sum wrapping as ATen's add does */
        int64_t cand = floor_mod((int64_t)((uint64_t)id + (uint64_t)replacement_offsets[i]), vocab);
        for (int it = 0; it < 3; ++it) {                            /* :366 */
          int forbidden = cand == mask_id || cand == id ||
                          (has_eos && cand == eos_id);
          if (forbidden) cand = floor_mod(cand + 1, vocab);
        }
        if (rep) value = cand;
      }
      const int msk = pos && !rep; /* :377 / :382 */
      if (msk) value = mask_id;
      corrupted[i] = value;
      labels[i] = pos ? id : -100; /* :386-389 */
      masked[i] = (uint8_t)msk;
      replaced[i] = (uint8_t)rep;
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Vocabulary-sharded statistics: the decomposition of                       */
/* display_token_statistics (csrc/cpu/display_stats.cpp:14-126) over         */
/* contiguous column ranges.  Record layout as cid_shard_record_t.           */
/* ------------------------------------------------------------------------ */

typedef struct {
  float max_logit;
  float sum_exp;
  int32_t index;
  float current;
} oracle_record_t;

int cid_oracle_shard_records(int dtype, const void* logits, const int64_t* ids,
                             int64_t rows, int64_t shard_vocab,
                             int64_t vocab_offset, void* records_out) {
  oracle_record_t* out = (oracle_record_t*)records_out;
  if (shard_vocab <= 0) return -1;
#pragma omp parallel
  {
    float* buf = (float*)malloc(sizeof(float) * (size_t)shard_vocab);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      row_to_float(dtype, logits, r, shard_vocab, buf);
      int64_t first_nan = -1, first_max = 0;
      float m = -INFINITY;
      int seen = 0;
      for (int64_t v = 0; v < shard_vocab; ++v) {
        float x = buf[v];
        if (isnan(x)) {
          if (first_nan < 0) first_nan = v;
          continue;
        }
        if (!seen || x > m) {
          m = x;
          first_max = v;
          seen = 1;
        }
      }
      oracle_record_t rec;
      rec.max_logit = m;
      double s = 0.0;
      if (isfinite(m))
        for (int64_t v = 0; v < shard_vocab; ++v) s += exp((double)buf[v] - (double)m);
      rec.sum_exp = first_nan >= 0 ? NAN : (m == -INFINITY ? 0.0f : (isfinite(m) ? (float)s : NAN));
      rec.index = (int32_t)(vocab_offset + (first_nan >= 0 ? first_nan : first_max));
      if (first_nan >= 0) rec.index |= (int32_t)0x80000000u;
      int64_t local = ids[r] - vocab_offset;
      rec.current = (local >= 0 && local < shard_vocab) ? buf[local] : 0.0f;
      out[r] = rec;
    }
    free(buf);
  }
  return 0;
}

int cid_oracle_combine_records(const void* records_in, int world,
                               const int64_t* offsets, const int64_t* ids,
                               int64_t rows, float* confidence,
                               int64_t* predicted, float* current) {
  const oracle_record_t* rec = (const oracle_record_t*)records_in;
  for (int64_t r = 0; r < rows; ++r) {
    int done = 0;
    for (int k = 0; k < world && !done; ++k) {
      oracle_record_t x = rec[(int64_t)k * rows + r];
      if (x.index < 0) { /* lowest rank holding a NaN: its first NaN */
        predicted[r] = x.index & 0x7fffffff;
        confidence[r] = NAN;
        current[r] = NAN;
        done = 1;
      }
    }
    if (done) continue;
    float M = -INFINITY;
    int32_t idx = rec[r].index;
    for (int k = 0; k < world; ++k) {
      oracle_record_t x = rec[(int64_t)k * rows + r];
      if (x.max_logit > M) {
        M = x.max_logit;
        idx = x.index;
      }
    }
    predicted[r] = idx;
    if (!isfinite(M)) {
      confidence[r] = NAN;
      current[r] = NAN;
      continue;
    }
    double S = 0.0;
    for (int k = 0; k < world; ++k) {
      oracle_record_t x = rec[(int64_t)k * rows + r];
      if (x.max_logit == -INFINITY) continue;
      S += (double)x.sum_exp * exp((double)x.max_logit - (double)M);
    }
    int owner = -1;
    for (int k = 0; k < world; ++k)
      if (ids[r] >= offsets[k] && ids[r] < offsets[k + 1]) owner = k;
    confidence[r] = (float)(1.0 / S);
    current[r] = owner < 0 ? NAN
                           : (float)(exp((double)rec[(int64_t)owner * rows + r].current - (double)M) / S);
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* batched_linear_assignment — csrc/ops.cpp:68-175 (Hungarian method with    */
/* potentials, double precision, first column on ties).                      */
/* ------------------------------------------------------------------------ */

int cid_oracle_linear_assignment(int dtype, const void* costs,
                                 const int64_t* row_counts, int64_t batch,
                                 int64_t rows, int64_t columns, int64_t* out) {
  if (rows > columns || columns > 16) return -1; /* :73-78 */
  for (int64_t b = 0; b < batch; ++b) {
    const int64_t active = row_counts[b];
    if (active < 0 || active > rows) return -1; /* :104-106 */
    for (int64_t r = 0; r < rows; ++r) out[b * rows + r] = -1;
    if (active == 0) continue;
    double u[17] = {0}, v[17] = {0};
    int64_t p[17] = {0}, way[17] = {0};
    const int64_t base = b * rows * columns;
    for (int64_t row = 1; row <= active; ++row) {
      p[0] = row;
      int64_t j0 = 0;
      double minv[17];
      int used[17] = {0};
      for (int64_t j = 0; j <= columns; ++j) minv[j] = INFINITY;
      int steps = 0;
      do {
        used[j0] = 1;
        const int64_t i0 = p[j0];
        double delta = INFINITY;
        int64_t j1 = 0;
        for (int64_t j = 1; j <= columns; ++j) {
          if (used[j]) continue;
          const double c = (double)(float)load(dtype, costs, base + (i0 - 1) * columns + (j - 1));
          const double cur = c - u[i0] - v[j];
          if (cur < minv[j]) {
            minv[j] = cur;
            way[j] = j0;
          }
          if (minv[j] < delta) {
            delta = minv[j];
            j1 = j;
          }
        }
        for (int64_t j = 0; j <= columns; ++j) {
          if (used[j]) {
            u[p[j]] += delta;
            v[j] -= delta;
          } else {
            minv[j] -= delta;
          }
        }
        j0 = j1;
        if (++steps > columns + 2) return -3; /* search cannot complete */
      } while (p[j0] != 0);
      do {
        const int64_t j1 = way[j0];
        p[j0] = p[j1];
        j0 = j1;
      } while (j0 != 0);
    }
    for (int64_t j = 1; j <= columns; ++j)
      if (p[j] > 0 && p[j] <= active) out[b * rows + (p[j] - 1)] = j - 1;
  }
  return 0;
}
