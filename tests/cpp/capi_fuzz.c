/*
 * Byte-driven fuzz target for the host-side argument validation of the C ABI
 * (include/cid_engine_b200.h).  It plays the part of the reference's
 * libFuzzer target over its C++ operators (tests/fuzz/fuzz_engine.cpp:279-307
 * of fwerkor/cid-engine v1.1.0, built with AddressSanitizer and
 * UndefinedBehaviorSanitizer by CMakeLists.txt:31-52).  The reference target
 * runs its CPU operators; this library computes on the GPU, so what is
 * fuzzed here is everything an entry point does on the host before its first
 * CUDA call.
 *
 * Each input picks one entry point and draws its arguments from pools of
 * boundary values: sizes (negative, zero, small, 2^31 - 1 and its
 * neighbours, 2^32, 2^58, 2^62, INT64_MAX, INT64_MIN), reals (NaN,
 * infinities, -0, the ends of [0, 1] and values just outside), pointers
 * (NULL, aligned, misaligned by 1, 2, 4 or 8 bytes), every dtype code and
 * unknown ones, world sizes and ranks in and out of range, shard offsets in
 * and out of order.  The result must follow the contract the header states:
 *
 *   - arguments outside it return a validation code (CID_ERR_INVALID_ARGUMENT,
 *     _UNSUPPORTED_DTYPE, _MISALIGNED or _SCRATCH_LIMIT), never CID_OK and
 *     never a CUDA error, which would mean the call went on to the device;
 *   - arguments inside it with no work return CID_OK; with work, the error
 *     of the first CUDA call (the driver below runs with no GPU visible);
 *   - host arrays (shard offsets, inbox lists, IPC handles) are read only
 *     within their documented extents and no host arithmetic overflows:
 *     the sanitizers stop the run otherwise (the harness allocates each host
 *     array at exactly its documented size).
 *
 * Device pointers are addresses in a host arena that the library never
 * dereferences.  The standalone driver (main, left out when built with
 * -DCID_LIBFUZZER for libFuzzer) feeds seeded random inputs and refuses to
 * run when a GPU is visible, so that no call with host addresses can ever
 * reach a device.  Usage: capi_fuzz [iterations] [seed].
 */
#include <limits.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cid_engine_b200.h"

int cudaGetDeviceCount(int* count); /* CUDA runtime, linked statically */

#define MAX_ROWS ((int64_t)INT32_MAX)
#define MAX_COUNT ((int64_t)1 << 58)
#define MAX_LM_ROWS ((int64_t)INT32_MAX - 128)
#define NELEM(a) (sizeof(a) / sizeof((a)[0]))

/* ------------------------------------------------------------------------ */
/* Input decoding                                                            */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint8_t* data;
  size_t size, off;
} input_t;

static const input_t* g_current;
static const char* g_entry;

static uint8_t take(input_t* in) { return in->off < in->size ? in->data[in->off++] : 0; }

static const int64_t kSmall[] = {0, 1, 2, 3, 4, 5, 7, 8, 9, 16, 17, 33, 64, 100, 256, 1000};
static const int64_t kEdge[] = {
    -1, -2, -4096, INT64_MIN, INT64_MIN + 1, (int64_t)INT32_MAX - 128, (int64_t)INT32_MAX - 127,
    (int64_t)INT32_MAX - 64, (int64_t)INT32_MAX - 16, (int64_t)INT32_MAX - 15, INT32_MAX,
    (int64_t)INT32_MAX + 1, (int64_t)UINT32_MAX, (int64_t)1 << 32, 65536, 65537,
    (int64_t)1 << 40, ((int64_t)1 << 58) - 1, (int64_t)1 << 58, ((int64_t)1 << 58) + 1,
    (int64_t)1 << 62, INT64_MAX - 1, INT64_MAX};

/* Mostly small sizes, a quarter of the time a boundary value. */
static int64_t size_of(input_t* in) {
  const uint8_t b = take(in);
  if (b < 192) return kSmall[b % NELEM(kSmall)];
  return kEdge[b % NELEM(kEdge)];
}

static double real_of(input_t* in) {
  static const double v[] = {0.0,   1e-7,     0.25,      0.5,   1.0,   0.999999, 1.0000000000000002,
                             1.5,   -0.0,     -1e-9,     NAN,   INFINITY, -INFINITY, 60.0,
                             60.000001, 1e300, 5e-324,   2.0};
  return v[take(in) % NELEM(v)];
}

/* Mostly valid dtype codes, sometimes unknown ones. */
static int dtype_of(input_t* in) {
  static const int bad[] = {-1, 10, 11, 255, INT_MAX, INT_MIN};
  const uint8_t b = take(in);
  if (b < 224) return b % 10;
  return bad[b % NELEM(bad)];
}

static int world_of(input_t* in, int max_world) {
  const int v[] = {1, 2, 3, 4, 8, max_world, max_world + 1, 0, -1, INT_MAX, INT_MIN, 5, 7};
  return v[take(in) % NELEM(v)];
}

static unsigned char g_arena[64 * 32] __attribute__((aligned(256)));

/* A device-pointer stand-in: NULL, 64-byte aligned, or misaligned. */
static void* ptr_of(input_t* in, int slot) {
  unsigned char* base = g_arena + 64 * (slot % 32);
  switch (take(in) % 16) {
    case 0: return NULL;
    case 1: return base + 1;
    case 2: return base + 2;
    case 3: return base + 4;
    case 4: return base + 8;
    default: return base;
  }
}

/* ------------------------------------------------------------------------ */
/* The contract                                                              */
/* ------------------------------------------------------------------------ */

static int is_float(int dt) { return dt >= 0 && dt <= 3; }
static int is_known(int dt) { return dt >= 0 && dt <= 9; }

static size_t esize(int dt) {
  switch (dt) {
    case 1: case 5: return 8;
    case 0: case 6: return 4;
    case 2: case 3: case 9: return 2;
    default: return 1;
  }
}

static int mis(const void* p, size_t align) {
  return p != NULL && ((uintptr_t)p % align) != 0;
}

/* a * b as an element count within MAX_COUNT. */
static int fits(int64_t a, int64_t b) {
  int64_t r;
  if (a < 0 || b < 0 || __builtin_mul_overflow(a, b, &r)) return 0;
  return r <= MAX_COUNT;
}

static int fits3(int64_t a, int64_t b, int64_t c) {
  int64_t ab;
  if (a < 0 || b < 0 || __builtin_mul_overflow(a, b, &ab)) return 0;
  return fits(ab, c);
}

static void fail(const char* why, int rc, int bad, int empty) {
  fprintf(stderr, "capi_fuzz: %s: %s (rc %d, outside contract %d, no work %d)\n  input:",
          g_entry, why, rc, bad, empty);
  for (size_t i = 0; g_current && i < g_current->size; ++i)
    fprintf(stderr, " %02x", g_current->data[i]);
  fprintf(stderr, "\n");
  abort();
}

static void expect(int rc, int bad, int empty) {
  const int validation = rc == CID_ERR_INVALID_ARGUMENT || rc == CID_ERR_UNSUPPORTED_DTYPE ||
                         rc == CID_ERR_MISALIGNED || rc == CID_ERR_SCRATCH_LIMIT;
  if (rc < CID_OK || rc > CID_ERR_SCRATCH_LIMIT) fail("result outside cid_result_t", rc, bad, empty);
  if (bad) {
    if (!validation) fail("arguments outside the contract were not rejected", rc, bad, empty);
  } else if (empty) {
    if (rc != CID_OK) fail("a call with no work did not return CID_OK", rc, bad, empty);
  } else if (rc != CID_ERR_CUDA && rc != CID_ERR_LAUNCH) {
    fail("valid arguments did not reach the CUDA runtime", rc, bad, empty);
  }
}

/* A logits argument: rows x vocab, row_stride >= vocab, span within MAX_COUNT. */
static int logits_bad(int dt, const void* logits, int64_t row_stride, int64_t rows,
                      int64_t vocab) {
  if (!is_float(dt)) return 1;
  if (rows < 0 || rows > MAX_ROWS || vocab <= 0 || vocab > INT_MAX - 16) return 1;
  if (rows > 0) {
    int64_t span;
    if (row_stride < vocab || rows - 1 < 0 || row_stride < 0 ||
        __builtin_mul_overflow(rows - 1, row_stride, &span) || span > MAX_COUNT - vocab)
      return 1;
  }
  return mis(logits, esize(dt));
}

static int range_bad(int64_t shard_vocab, int64_t offset, int64_t total) {
  return !(shard_vocab > 0 && offset >= 0 && total <= INT_MAX && total >= shard_vocab &&
           offset <= total - shard_vocab);
}

static int outputs_mis(const void* ids, const void* conf, const void* pred, const void* cur,
                       const void* status) {
  return mis(ids, 8) || mis(conf, 4) || mis(pred, 8) || mis(cur, 4) || mis(status, 4);
}

/* A row stride: mostly the vocabulary itself or a little more. */
static int64_t stride_of(input_t* in, int64_t vocab) {
  const uint8_t b = take(in);
  if (b < 200 && vocab >= 0 && vocab < INT64_MAX - 8) return vocab + b % 3;
  return size_of(in);
}

/* World + 1 ascending offsets (allocated at exactly that size when the world
 * is in range, one element otherwise), sometimes NULL or out of order. */
static int64_t* offsets_of(input_t* in, int world, int max_world, int* bad) {
  if (take(in) % 10 == 0) {
    *bad = 1;
    return NULL;
  }
  const int in_range = world >= 1 && world <= max_world;
  const int n = in_range ? world + 1 : 1;
  int64_t* o = malloc(sizeof(int64_t) * (size_t)n);
  int64_t x = take(in) % 4 == 0 ? 0 : (int64_t)(take(in) % 100);
  for (int r = 0; r < n; ++r) {
    o[r] = x;
    x += take(in) % 300;
  }
  switch (take(in) % 12) {
    case 0: o[0] = -1 - (int64_t)(take(in) % 3); break;
    case 1: o[n - 1] = (int64_t)INT_MAX + 1; break;
    case 2: o[n - 1] = INT_MAX; break;
    case 3:
      if (n > 2) o[1] = o[2] + 1;
      break;
    default: break;
  }
  if (!in_range) {
    *bad = 1;
  } else {
    int b = o[0] < 0 || o[world] > INT_MAX;
    for (int r = 1; r <= world; ++r) b |= o[r] < o[r - 1];
    *bad = b;
  }
  return o;
}

/* An inbox list of `world` pointers (exact size when in range; each must be
 * non-NULL and 16-byte aligned), or NULL. */
static void** inboxes_of(input_t* in, int world, int* bad) {
  if (take(in) % 10 == 0) {
    *bad = 1;
    return NULL;
  }
  const int in_range = world >= 1 && world <= 8;
  const int n = in_range ? world : 1;
  void** list = malloc(sizeof(void*) * (size_t)n);
  int b = 0;
  for (int q = 0; q < n; ++q) {
    list[q] = take(in) % 6 == 0 ? ptr_of(in, 20 + q) : g_arena + 64 * (20 + q);
    b |= list[q] == NULL || mis(list[q], 16);
  }
  *bad = b;
  return list;
}

/* ------------------------------------------------------------------------ */
/* Entry points                                                              */
/* ------------------------------------------------------------------------ */

static void fuzz_stats(input_t* in) {
  const int dt = dtype_of(in);
  const void* logits = ptr_of(in, 0);
  const int64_t rows = size_of(in), vocab = size_of(in), stride = stride_of(in, vocab);
  int64_t* ids = ptr_of(in, 1);
  float* conf = ptr_of(in, 2);
  int64_t* pred = ptr_of(in, 3);
  float* cur = ptr_of(in, 4);
  uint32_t* st = ptr_of(in, 5);
  int bad = logits_bad(dt, logits, stride, rows, vocab) || outputs_mis(ids, conf, pred, cur, st);
  const int empty = rows == 0;
  if (!bad && !empty) bad = !logits || !ids || !conf || !pred || !cur;
  expect(cid_display_token_statistics((cid_dtype_t)dt, logits, stride, ids, rows, vocab, conf,
                                      pred, cur, st, NULL),
         bad, empty);
}

static void fuzz_repetition(input_t* in) {
  const int dt = dtype_of(in);
  const void* logits = ptr_of(in, 0);
  const int64_t batch = size_of(in), tokens = size_of(in), vocab = size_of(in);
  const int64_t stride = stride_of(in, vocab);
  const int64_t mask = size_of(in), eos = size_of(in);
  const int has_eos = take(in) & 1;
  const double mult = real_of(in);
  int64_t* ids = ptr_of(in, 1);
  float* conf = ptr_of(in, 2);
  int64_t* pred = ptr_of(in, 3);
  float* cur = ptr_of(in, 4);
  uint32_t* st = ptr_of(in, 5);
  int64_t rows = 0;
  int bad = !is_float(dt) || !(mult > 0.0 && mult <= 1.0) || batch < 0 || tokens < 0 ||
            __builtin_mul_overflow(batch, tokens, &rows) || rows > MAX_ROWS;
  int empty = 0;
  if (!bad) {
    bad = logits_bad(dt, logits, stride, rows, vocab) || outputs_mis(ids, conf, pred, cur, st);
    empty = rows == 0;
    if (!bad && !empty) bad = !logits || !ids || !conf || !pred || !cur;
  }
  expect(cid_display_token_statistics_with_repetition((cid_dtype_t)dt, logits, stride, ids, batch,
                                                      tokens, vocab, mask, has_eos, eos, mult,
                                                      conf, pred, cur, st, NULL),
         bad, empty);
}

static void shard_range_of(input_t* in, int64_t shard_vocab, int64_t* offset, int64_t* total) {
  if (take(in) < 160 && shard_vocab >= 0 && shard_vocab < INT_MAX) {
    *offset = kSmall[take(in) % NELEM(kSmall)];
    *total = *offset + shard_vocab + (take(in) % 3);
  } else {
    *offset = size_of(in);
    *total = size_of(in);
  }
}

static void fuzz_shard_records(input_t* in) {
  const int dt = dtype_of(in);
  const void* logits = ptr_of(in, 0);
  const int64_t rows = size_of(in), sv = size_of(in), stride = stride_of(in, sv);
  int64_t off, total;
  shard_range_of(in, sv, &off, &total);
  int64_t* ids = ptr_of(in, 1);
  cid_shard_record_t* rec = ptr_of(in, 2);
  uint32_t* st = ptr_of(in, 5);
  int bad = logits_bad(dt, logits, stride, rows, sv) || range_bad(sv, off, total) ||
            mis(ids, 8) || mis(rec, 4) || mis(st, 4);
  const int empty = rows == 0;
  if (!bad && !empty) bad = !logits || !ids || !rec;
  expect(cid_display_shard_records((cid_dtype_t)dt, logits, stride, ids, rows, sv, off, total,
                                   rec, st, NULL),
         bad, empty);
}

static void fuzz_merge_combine(input_t* in, int combine) {
  const int world = world_of(in, 256);
  int offsets_bad = 0;
  int64_t* offs = offsets_of(in, world, 256, &offsets_bad);
  const cid_shard_record_t* rec = ptr_of(in, 0);
  int64_t* ids = ptr_of(in, 1);
  const int64_t rows = size_of(in);
  cid_shard_record_t* merged = ptr_of(in, 2);
  float* conf = ptr_of(in, 3);
  int64_t* pred = ptr_of(in, 4);
  float* cur = ptr_of(in, 5);
  uint32_t* st = ptr_of(in, 6);
  int bad = offsets_bad || rows < 0 || rows > MAX_ROWS || mis(rec, 4) || mis(ids, 8);
  bad |= combine ? outputs_mis(ids, conf, pred, cur, st) : mis(merged, 4);
  const int empty = rows == 0;
  if (!bad && !empty)
    bad = !rec || !ids || (combine ? (!conf || !pred || !cur) : !merged);
  const int rc = combine ? cid_display_combine_records(rec, world, offs, ids, rows, conf, pred,
                                                       cur, st, NULL)
                         : cid_display_merge_records(rec, world, offs, ids, rows, merged, NULL);
  expect(rc, bad, empty);
  free(offs);
}

static void fuzz_refine(input_t* in) {
  int64_t* ids = ptr_of(in, 0);
  float* conf = ptr_of(in, 1);
  int64_t* pred = ptr_of(in, 2);
  float* cur = ptr_of(in, 3);
  int64_t* out = ptr_of(in, 4);
  const int64_t batch = size_of(in), tokens = size_of(in), mask = size_of(in), eos = size_of(in);
  const int has_eos = take(in) & 1;
  const double reveal = real_of(in), revision = real_of(in), margin = real_of(in);
  int bad = !(reveal >= 0.0 && reveal <= 1.0) || !(revision >= 0.0 && revision <= 1.0) ||
            !(margin >= 0.0) || !fits(batch, tokens) || batch > MAX_ROWS || mis(ids, 8) ||
            mis(conf, 4) || mis(pred, 8) || mis(cur, 4) || mis(out, 8);
  const int empty = batch == 0 || tokens == 0;
  if (!bad && !empty) bad = !ids || !conf || !pred || !cur || !out;
  expect(cid_refine_display(ids, conf, pred, cur, batch, tokens, mask, has_eos, eos, reveal,
                            revision, margin, out, NULL),
         bad, empty);
}

static int span_bad(int64_t batch, int64_t slots, int64_t rs, int64_t cs) {
  int64_t a, b;
  if (rs < 0 || cs < 0) return 1;
  if (__builtin_mul_overflow(batch - 1, rs, &a) || __builtin_mul_overflow(slots - 1, cs, &b))
    return 1;
  return a > MAX_COUNT || b > MAX_COUNT - a;
}

static void fuzz_prefix(input_t* in) {
  const int odt = dtype_of(in), ldt = dtype_of(in);
  const void* occ = ptr_of(in, 0);
  const void* logits = ptr_of(in, 1);
  uint8_t* out = ptr_of(in, 2);
  const int64_t batch = size_of(in), slots = size_of(in);
  const int64_t ors = take(in) < 128 ? slots : size_of(in), ocs = take(in) < 128 ? 1 : size_of(in);
  const int64_t lrs = take(in) < 128 ? slots : size_of(in), lcs = take(in) < 128 ? 1 : size_of(in);
  const double thr = real_of(in);
  const int64_t max_alloc = size_of(in);
  int bad = !is_known(odt) || !is_float(ldt) || !(thr >= 0.0 && thr <= 1.0) || max_alloc <= 0 ||
            !fits(batch, slots) || batch > MAX_ROWS;
  if (!bad && batch > 0 && slots > 0)
    bad = span_bad(batch, slots, ors, ocs) || span_bad(batch, slots, lrs, lcs);
  bad |= mis(occ, esize(odt)) || mis(logits, esize(ldt));
  const int empty = batch == 0 || slots == 0;
  if (!bad && !empty) bad = !occ || !logits || !out;
  expect(cid_prefix_allocation_mask((cid_dtype_t)odt, occ, ors, ocs, (cid_dtype_t)ldt, logits, lrs,
                                    lcs, batch, slots, thr, max_alloc, out, NULL),
         bad, empty);
}

static void fuzz_rollout(input_t* in, int live) {
  const int odt = dtype_of(in), dt = dtype_of(in), live_dt = dtype_of(in);
  const void* occ = ptr_of(in, 0);
  const void* alloc = ptr_of(in, 1);
  const void* life = ptr_of(in, 2);
  const void* rev = ptr_of(in, 3);
  const void* in_life = ptr_of(in, 4);
  uint8_t* next = ptr_of(in, 5);
  int64_t* life_idx = ptr_of(in, 6);
  int64_t* rev_idx = ptr_of(in, 7);
  int64_t* in_idx = ptr_of(in, 8);
  uint8_t* present = ptr_of(in, 9);
  uint8_t* live_slots = ptr_of(in, 10);
  void* live_occ = ptr_of(in, 11);
  const int64_t batch = size_of(in), slots = size_of(in), F = size_of(in), R = size_of(in);
  const int64_t retired = take(in) < 160 ? (int64_t)(take(in) % 4) : size_of(in);
  const double thr = real_of(in);
  const int64_t max_alloc = size_of(in);
  const size_t es = esize(dt);
  int bad = !is_known(odt) || !is_float(dt) || (live && !is_float(live_dt)) || retired < 0 ||
            retired >= F || !(thr >= 0.0 && thr <= 1.0) || max_alloc <= 0 || R <= 0 ||
            !fits3(batch, slots, F > R ? F : R) || batch > MAX_ROWS;
  bad |= mis(occ, esize(odt)) || mis(alloc, es) || mis(life, es) || mis(rev, es) ||
         mis(in_life, es) || mis(life_idx, 8) || mis(rev_idx, 8) || mis(in_idx, 8) ||
         (live && mis(live_occ, esize(live_dt)));
  const int empty = batch == 0 || slots == 0;
  if (!bad && !empty)
    bad = !occ || !alloc || !life || !rev || !in_life || !next || !life_idx || !rev_idx ||
          !in_idx || !present || !live_slots || (live && !live_occ);
  const int rc =
      live ? cid_rollout_slot_transition_live(
                 (cid_dtype_t)odt, occ, (cid_dtype_t)dt, alloc, life, rev, in_life, batch, slots,
                 F, R, thr, max_alloc, retired, next, life_idx, rev_idx, in_idx, present,
                 live_slots, (cid_dtype_t)live_dt, live_occ, NULL)
           : cid_rollout_slot_transition((cid_dtype_t)odt, occ, (cid_dtype_t)dt, alloc, life, rev,
                                         in_life, batch, slots, F, R, thr, max_alloc, retired,
                                         next, life_idx, rev_idx, in_idx, present, live_slots,
                                         NULL);
  expect(rc, bad, empty);
}

static void fuzz_live(input_t* in) {
  const int dt = dtype_of(in);
  const void* occ = ptr_of(in, 0);
  const void* life = ptr_of(in, 1);
  void* out = ptr_of(in, 2);
  const int64_t rows = size_of(in), features = size_of(in);
  const int64_t retired = take(in) < 160 ? (int64_t)(take(in) % 4) : size_of(in);
  const size_t es = esize(dt);
  int bad = !is_float(dt) || (life && (retired < 0 || retired >= features)) || rows < 0 ||
            rows > MAX_ROWS || (life && !fits(rows, features)) || mis(occ, es) ||
            mis(life, es) || mis(out, es);
  const int empty = rows == 0;
  if (!bad && !empty) bad = !occ || !out;
  expect(cid_live_slot_occupancy((cid_dtype_t)dt, occ, life, rows, features, retired, out, NULL),
         bad, empty);
}

static void fuzz_snapshot(input_t* in) {
  int dts[5];
  for (int k = 0; k < 5; ++k) dts[k] = dtype_of(in);
  const void* sem = ptr_of(in, 0);
  const void* roles = ptr_of(in, 1);
  const void* unc = ptr_of(in, 2);
  const void* noise = ptr_of(in, 3);
  const void* life = ptr_of(in, 4);
  const uint8_t* sel = ptr_of(in, 5);
  const int64_t* idx = ptr_of(in, 6);
  float* out = ptr_of(in, 7);
  uint32_t* st = ptr_of(in, 8);
  const int64_t rows = size_of(in), hidden = size_of(in), nroles = size_of(in);
  const int64_t L = size_of(in), nidx = size_of(in);
  int bad = 0;
  for (int k = 0; k < 5; ++k) bad |= !is_float(dts[k]);
  bad |= rows < 0 || rows > MAX_ROWS || L <= 0 || nroles < 0 || nroles > MAX_COUNT ||
         nidx < 0 || nidx > MAX_COUNT;
  if (!bad)
    bad = !fits(rows, hidden) || !fits(rows, nroles) || !fits(rows, L) ||
          !fits(rows, 4 + nroles + nidx);
  bad |= mis(sem, esize(dts[0])) || mis(roles, esize(dts[1])) || mis(unc, esize(dts[2])) ||
         mis(noise, esize(dts[3])) || mis(life, esize(dts[4])) || mis(idx, 8) || mis(out, 4) ||
         mis(st, 4);
  const int empty = rows == 0;
  if (!bad && !empty)
    bad = !out || !sel || !unc || !noise || !life || (nroles > 0 && !roles) ||
          (nidx > 0 && !idx) || (nidx > 0 && hidden > 0 && !sem);
  expect(cid_materialize_cell_snapshot((cid_dtype_t)dts[0], sem, hidden, (cid_dtype_t)dts[1],
                                       roles, nroles, (cid_dtype_t)dts[2], unc,
                                       (cid_dtype_t)dts[3], noise, (cid_dtype_t)dts[4], life, L,
                                       sel, idx, nidx, rows, out, st, NULL),
         bad, empty);
}

static void fuzz_assignment(input_t* in) {
  const int dt = dtype_of(in);
  const void* costs = ptr_of(in, 0);
  const int64_t* counts = ptr_of(in, 1);
  int64_t* out = ptr_of(in, 2);
  uint32_t* st = ptr_of(in, 3);
  const int64_t batch = size_of(in), rows = size_of(in), cols = size_of(in);
  int bad = !is_float(dt) || batch < 0 || batch > MAX_ROWS || rows < 0 || cols < 0 ||
            rows > cols || cols > 16 || mis(costs, esize(dt)) || mis(counts, 8) || mis(out, 8) ||
            mis(st, 4);
  const int empty = batch == 0 || rows == 0;
  if (!bad && !empty) bad = !costs || !counts || !out;
  expect(cid_batched_linear_assignment((cid_dtype_t)dt, costs, counts, batch, rows, cols, out, st,
                                       NULL),
         bad, empty);
}

static void fuzz_masked(input_t* in, int no_alloc) {
  const int64_t* clean = ptr_of(in, 0);
  const float* rr = ptr_of(in, 1);
  const float* mr = ptr_of(in, 2);
  int64_t* corrupted = ptr_of(in, 3);
  uint8_t* masked = ptr_of(in, 4);
  float* ratio = ptr_of(in, 5);
  float* metrics = ptr_of(in, 6);
  void* ws = ptr_of(in, 7);
  const int64_t batch = size_of(in), tokens = size_of(in), mask = size_of(in);
  const double lo = real_of(in), hi = real_of(in);
  int bad = batch <= 0 || tokens <= 0 || batch > MAX_ROWS || !fits(batch, tokens) ||
            !(lo > 0.0 && lo <= hi && hi <= 1.0) || mis(clean, 8) || mis(rr, 4) || mis(mr, 4) ||
            mis(corrupted, 8) || mis(ratio, 4) || mis(metrics, 4) ||
            !clean || !rr || !mr || !corrupted || !masked || !ratio || !metrics;
  if (no_alloc) {
    bad |= batch > CID_NO_ALLOC_MAX_BATCH;
    expect(cid_masked_diffusion_corrupt_no_alloc(clean, rr, mr, batch, tokens, mask, lo, hi,
                                                 corrupted, masked, ratio, metrics, NULL),
           bad, 0);
  } else {
    bad |= mis(ws, 16) || !ws;
    expect(cid_masked_diffusion_corrupt(clean, rr, mr, batch, tokens, mask, lo, hi, corrupted,
                                        masked, ratio, metrics, ws, NULL),
           bad, 0);
  }
  const size_t want = batch > 0 && batch <= MAX_ROWS ? (size_t)batch * 8 : 0;
  if (cid_masked_diffusion_workspace_bytes(batch) != want)
    fail("cid_masked_diffusion_workspace_bytes", 0, 0, 0);
}

static void fuzz_thought(input_t* in) {
  const int sdt = dtype_of(in), tdt = dtype_of(in), odt = dtype_of(in);
  const void* sem = ptr_of(in, 0);
  const void* ts = ptr_of(in, 1);
  const void* occ = ptr_of(in, 2);
  const void* eps = ptr_of(in, 3);
  void* corrupted = ptr_of(in, 4);
  void* noise = ptr_of(in, 5);
  void* masked = ptr_of(in, 6);
  const int64_t rows = size_of(in), hidden = size_of(in);
  const size_t es = esize(sdt);
  int bad = !is_float(sdt) || !is_float(tdt) || !is_known(odt) || !fits(rows, hidden) ||
            rows > MAX_ROWS || mis(sem, es) || mis(eps, es) || mis(corrupted, es) ||
            mis(noise, es) || mis(masked, es) || mis(ts, esize(tdt)) || mis(occ, esize(odt));
  const int empty = rows == 0;
  if (!bad && !empty)
    bad = !ts || !occ || !noise || (hidden > 0 && (!sem || !eps || !corrupted || !masked));
  expect(cid_thought_corrupt((cid_dtype_t)sdt, sem, (cid_dtype_t)tdt, ts, (cid_dtype_t)odt, occ,
                             eps, rows, hidden, corrupted, noise, masked, NULL),
         bad, empty);
}

static void fuzz_display_corrupt(input_t* in) {
  const int tdt = dtype_of(in), edt = dtype_of(in), rdt = dtype_of(in), pdt = dtype_of(in);
  const int64_t* ids = ptr_of(in, 0);
  const void* ts = ptr_of(in, 1);
  const void* el = ptr_of(in, 2);
  const void* cr = ptr_of(in, 3);
  const void* rr = ptr_of(in, 4);
  const int64_t* ro = ptr_of(in, 5);
  int64_t* corrupted = ptr_of(in, 6);
  int64_t* labels = ptr_of(in, 7);
  uint8_t* masked = ptr_of(in, 8);
  uint8_t* replaced = ptr_of(in, 9);
  const int64_t batch = size_of(in), tokens = size_of(in), mask = size_of(in), eos = size_of(in);
  const int64_t vocab = size_of(in);
  const int has_eos = take(in) & 1;
  const double frac = real_of(in);
  const int replace = frac > 0.0;
  int bad = !is_float(tdt) || !is_known(edt) || !is_float(rdt) || (replace && !is_float(pdt)) ||
            !(frac >= 0.0 && frac <= 1.0) || (replace && vocab < 3) || !fits(batch, tokens) ||
            batch > MAX_ROWS;
  bad |= mis(ids, 8) || mis(ts, esize(tdt)) || mis(el, esize(edt)) || mis(cr, esize(rdt)) ||
         mis(corrupted, 8) || mis(labels, 8) ||
         (replace && (mis(rr, esize(pdt)) || mis(ro, 8)));
  const int empty = batch == 0 || tokens == 0;
  if (!bad && !empty)
    bad = !ids || !ts || !el || !cr || !corrupted || !labels || !masked || !replaced ||
          (replace && (!rr || !ro));
  expect(cid_display_corrupt(ids, (cid_dtype_t)tdt, ts, (cid_dtype_t)edt, el, (cid_dtype_t)rdt, cr,
                             (cid_dtype_t)pdt, rr, ro, batch, tokens, mask, has_eos, eos, vocab,
                             frac, corrupted, labels, masked, replaced, NULL),
         bad, empty);
}

static int lm_shape_bad(int64_t rows, int64_t hd, int64_t vocab) {
  return rows < 0 || rows > MAX_LM_ROWS || hd <= 0 || hd % 8 != 0 || hd > INT32_MAX - 64 ||
         vocab <= 0 || vocab > INT32_MAX || !fits(rows, hd) || !fits(vocab, hd);
}

static size_t lm_workspace_of(input_t* in, int64_t rows, int64_t vocab, size_t* need) {
  *need = cid_lm_head_workspace_bytes(rows, vocab);
  const int ok = rows > 0 && rows <= MAX_LM_ROWS && vocab > 0 && vocab <= INT32_MAX;
  if ((*need == 0) == ok) fail("cid_lm_head_workspace_bytes is 0 exactly for invalid shapes", 0, 0, 0);
  if (ok && *need % ((size_t)rows * sizeof(cid_shard_record_t)) != 0)
    fail("cid_lm_head_workspace_bytes is not a whole number of record rows", 0, 0, 0);
  switch (take(in) % 5) {
    case 0: return 0;
    case 1: return *need > 0 ? *need - 1 : 0;
    case 2: return SIZE_MAX;
    default: return *need;
  }
}

static void fuzz_lm_head(input_t* in, int shard) {
  const void* hidden = ptr_of(in, 0);
  const void* weight = ptr_of(in, 1);
  const int64_t* ids = ptr_of(in, 2);
  float* conf = ptr_of(in, 3);
  int64_t* pred = ptr_of(in, 4);
  float* cur = ptr_of(in, 5);
  void* ws = ptr_of(in, 6);
  uint32_t* st = ptr_of(in, 7);
  cid_shard_record_t* rec = ptr_of(in, 8);
  const int64_t rows = size_of(in), hd = size_of(in), vocab = size_of(in);
  int64_t off = 0, total = 0;
  if (shard) shard_range_of(in, vocab, &off, &total);
  size_t need;
  const size_t ws_bytes = lm_workspace_of(in, rows, vocab, &need);
  int bad = lm_shape_bad(rows, hd, vocab) || mis(hidden, 16) || mis(weight, 16) || mis(ids, 8) ||
            mis(ws, 16) || mis(st, 4);
  bad |= shard ? (range_bad(vocab, off, total) || mis(rec, 4))
               : (mis(conf, 4) || mis(pred, 8) || mis(cur, 4));
  const int empty = rows == 0;
  if (!bad && !empty) {
    bad = !hidden || !weight || !ids || !ws || (shard ? !rec : (!conf || !pred || !cur));
    bad |= ws_bytes < need;
  }
  const int rc = shard ? cid_lm_head_shard_records(hidden, rows, hd, weight, vocab, off, total, ids,
                                                   1, rec, ws, ws_bytes, st, NULL)
                       : cid_lm_head_display_statistics(hidden, rows, hd, weight, vocab, ids, 1,
                                                        conf, pred, cur, ws, ws_bytes, st, NULL);
  expect(rc, bad, empty);
}

static void fuzz_inbox_handles(input_t* in) {
  const int world = world_of(in, 8);
  const int64_t cap = size_of(in);
  const size_t bytes = cid_peer_inbox_bytes(world, cap);
  const int ok = world >= 1 && world <= 8 && cap >= 0 && cap <= MAX_ROWS;
  const size_t want = ok ? 2 * (size_t)world * (size_t)cap * 16 + 256 : 0;
  if (bytes != want) fail("cid_peer_inbox_bytes", 0, 0, 0);

  void* slot = NULL;
  const size_t alloc_bytes = take(in) % 3 == 0 ? 0 : (size_t)(take(in) + 1) * 256;
  void** where = take(in) % 4 == 0 ? NULL : &slot;
  expect(cid_peer_inbox_alloc(alloc_bytes, where), !where || alloc_bytes == 0, 0);

  unsigned char* handle = take(in) % 4 == 0 ? NULL : malloc(64);
  if (handle) memset(handle, take(in), 64);
  void* inbox = ptr_of(in, 0);
  switch (take(in) % 4) {
    case 0:
      expect(cid_peer_inbox_export(inbox, handle), !inbox || !handle, 0);
      break;
    case 1: {
      void* mapped = NULL;
      void** out = take(in) % 4 == 0 ? NULL : &mapped;
      expect(cid_peer_inbox_import(handle, out), !handle || !out, 0);
      break;
    }
    case 2: expect(cid_peer_inbox_free(inbox), 0, inbox == NULL); break;
    default: expect(cid_peer_inbox_release(inbox), 0, inbox == NULL); break;
  }
  free(handle);
}

static int peers_bad(int64_t rows, int rank, int world, int list_bad, int64_t cap) {
  return world < 1 || world > 8 || rank < 0 || rank >= world || list_bad || rows < 1 ||
         rows > cap || cap > MAX_ROWS;
}

static void fuzz_to_peers(input_t* in) {
  const int dt = dtype_of(in);
  const void* logits = ptr_of(in, 0);
  const int64_t rows = size_of(in), sv = size_of(in), stride = stride_of(in, sv);
  int64_t off, total;
  shard_range_of(in, sv, &off, &total);
  const int world = world_of(in, 8);
  const int rank = take(in) < 200 ? (int)(take(in) % 9) : world_of(in, 8);
  int list_bad = 0;
  void** inboxes = inboxes_of(in, world, &list_bad);
  const int64_t cap = take(in) < 128 && rows < INT64_MAX - 4 ? rows + take(in) % 3 : size_of(in);
  const uint32_t epoch = take(in);
  int64_t* ids = ptr_of(in, 1);
  uint32_t* st = ptr_of(in, 2);
  int bad = logits_bad(dt, logits, stride, rows, sv) || range_bad(sv, off, total) ||
            peers_bad(rows, rank, world, list_bad, cap) || mis(ids, 8) || mis(st, 4) ||
            !logits || !ids;
  expect(cid_display_shard_records_to_peers((cid_dtype_t)dt, logits, stride, ids, rows, sv, off,
                                            total, rank, world, (void* const*)inboxes, cap, epoch,
                                            st, NULL),
         bad, 0);
  free(inboxes);
}

static void fuzz_push(input_t* in) {
  const cid_shard_record_t* rec = ptr_of(in, 0);
  const int64_t rows = size_of(in);
  const int world = world_of(in, 8);
  const int rank = take(in) < 200 ? (int)(take(in) % 9) : world_of(in, 8);
  int list_bad = 0;
  void** inboxes = inboxes_of(in, world, &list_bad);
  const int64_t cap = take(in) < 128 && rows < INT64_MAX - 4 ? rows + take(in) % 3 : size_of(in);
  const int bad = peers_bad(rows, rank, world, list_bad, cap) || mis(rec, 4) || !rec;
  expect(cid_peer_push_records(rec, rows, rank, world, (void* const*)inboxes, cap, take(in), NULL),
         bad, 0);
  free(inboxes);
}

static void fuzz_combine_inbox(input_t* in) {
  void* inbox = ptr_of(in, 0);
  const int world = world_of(in, 8);
  int offsets_bad = 0;
  int64_t* offs = offsets_of(in, world, 8, &offsets_bad);
  const int64_t* ids = ptr_of(in, 1);
  const int64_t rows = size_of(in);
  const int64_t cap = take(in) < 128 && rows < INT64_MAX - 4 ? rows + take(in) % 3 : size_of(in);
  const double wait = real_of(in);
  float* conf = ptr_of(in, 2);
  int64_t* pred = ptr_of(in, 3);
  float* cur = ptr_of(in, 4);
  uint32_t* st = ptr_of(in, 5);
  const int bad = offsets_bad || rows < 1 || rows > cap || cap > MAX_ROWS ||
                  !(wait > 0.0 && wait <= 60.0) || mis(inbox, 16) ||
                  outputs_mis(ids, conf, pred, cur, st) || !inbox || !ids || !conf || !pred ||
                  !cur;
  expect(cid_display_combine_inbox(inbox, world, offs, ids, rows, cap, take(in), wait, conf, pred,
                                   cur, st, NULL),
         bad, 0);
  free(offs);
}

int LLVMFuzzerTestOneInput(const uint8_t* data, size_t size) {
  input_t in = {data, size, 0};
  g_current = &in;
  switch (take(&in) % 22) {
    case 0: g_entry = "cid_display_token_statistics"; fuzz_stats(&in); break;
    case 1: g_entry = "cid_display_token_statistics_with_repetition"; fuzz_repetition(&in); break;
    case 2: g_entry = "cid_display_shard_records"; fuzz_shard_records(&in); break;
    case 3: g_entry = "cid_display_merge_records"; fuzz_merge_combine(&in, 0); break;
    case 4: g_entry = "cid_display_combine_records"; fuzz_merge_combine(&in, 1); break;
    case 5: g_entry = "cid_refine_display"; fuzz_refine(&in); break;
    case 6: g_entry = "cid_prefix_allocation_mask"; fuzz_prefix(&in); break;
    case 7: g_entry = "cid_rollout_slot_transition"; fuzz_rollout(&in, 0); break;
    case 8: g_entry = "cid_rollout_slot_transition_live"; fuzz_rollout(&in, 1); break;
    case 9: g_entry = "cid_live_slot_occupancy"; fuzz_live(&in); break;
    case 10: g_entry = "cid_materialize_cell_snapshot"; fuzz_snapshot(&in); break;
    case 11: g_entry = "cid_batched_linear_assignment"; fuzz_assignment(&in); break;
    case 12: g_entry = "cid_masked_diffusion_corrupt"; fuzz_masked(&in, 0); break;
    case 13: g_entry = "cid_masked_diffusion_corrupt_no_alloc"; fuzz_masked(&in, 1); break;
    case 14: g_entry = "cid_thought_corrupt"; fuzz_thought(&in); break;
    case 15: g_entry = "cid_display_corrupt"; fuzz_display_corrupt(&in); break;
    case 16: g_entry = "cid_lm_head_display_statistics"; fuzz_lm_head(&in, 0); break;
    case 17: g_entry = "cid_lm_head_shard_records"; fuzz_lm_head(&in, 1); break;
    case 18: g_entry = "cid_peer_inbox_*"; fuzz_inbox_handles(&in); break;
    case 19: g_entry = "cid_display_shard_records_to_peers"; fuzz_to_peers(&in); break;
    case 20: g_entry = "cid_peer_push_records"; fuzz_push(&in); break;
    default: g_entry = "cid_display_combine_inbox"; fuzz_combine_inbox(&in); break;
  }
  g_current = NULL;
  return 0;
}

#ifndef CID_LIBFUZZER
static uint64_t next_random(uint64_t* s) {
  /* xorshift64* */
  *s ^= *s >> 12;
  *s ^= *s << 25;
  *s ^= *s >> 27;
  return *s * 0x2545F4914F6CDD1DULL;
}

int main(int argc, char** argv) {
  const long iterations = argc > 1 ? atol(argv[1]) : 200000;
  uint64_t state = argc > 2 ? strtoull(argv[2], NULL, 10) : 1;
  if (state == 0) state = 1;
  int devices = 0;
  if (cudaGetDeviceCount(&devices) == 0 && devices > 0) {
    fprintf(stderr, "capi_fuzz: a GPU is visible; run with CUDA_VISIBLE_DEVICES= (the harness "
                    "passes host addresses as device pointers)\n");
    return 77;
  }
  uint8_t buf[160];
  for (long it = 0; it < iterations; ++it) {
    const size_t n = 1 + next_random(&state) % sizeof(buf);
    for (size_t i = 0; i < n; ++i) buf[i] = (uint8_t)(next_random(&state) >> 56);
    LLVMFuzzerTestOneInput(buf, n);
  }
  printf("capi_fuzz: %ld inputs, every result within the contract\n", iterations);
  return 0;
}
#endif
