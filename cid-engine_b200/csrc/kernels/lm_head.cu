// LM head fused with the display statistics: the statistics of
// logits = hidden @ weight^T (bf16 operands, f32 accumulation, optionally
// rounded to bf16 as a bf16 LM head would store them) without writing the
// [rows, vocab] logits to memory.
//
// The reference has no LM head (its statistics operator takes materialised
// logits); this is the producer side of the display path on B200.  Two
// kernels share the work-unit, record and bounded-wait scheme below:
//
// * wide tiles (bf16-rounded logits, launches of at least kWideMinRows
//   rows): one persistent CTA per SM computes 256 rows x 256 columns, two
//   M=128 MMAs per K step sharing the weight slice (a third less operand
//   traffic from L2 into shared memory per FLOP than 128 x 256); the tile
//   fills all of TMEM, so eight epilogue warps drain it into registers as
//   bf16 pairs (128 registers a thread, after a setmaxnreg split that moves
//   registers from the TMA/MMA warpgroup to the two epilogue warpgroups),
//   release it at once and fold the 256 columns while the next tile
//   accumulates;
// * 128-row tiles (every other launch), described next.
//
// * one persistent CTA per SM, warp-specialised: warp 0 issues TMA loads of
//   128 x 64 hidden tiles and 256 x 64 weight tiles (128-byte swizzle) into a
//   4-stage shared-memory ring; warp 1 issues tcgen05.mma (M=128, N=256,
//   K=16, kind::f16 with bf16 A and B) into one of two 256-column TMEM
//   accumulators; warps 2-5 read the finished accumulator with tcgen05.ld
//   (thread = row, TMEM lane = row) and fold its 256 columns into the row's
//   online (max, sum of exp, first argmax, current-token logit) state while
//   the other accumulator fills;
// * a work unit is (block of 128 rows, group of G consecutive 256-column
//   vocabulary tiles); each unit ends in one 16-byte shard record per row
//   (the same record as the vocabulary-parallel statistics), and the record
//   combine kernel merges the groups of a row into its statistics;
// * units are ordered in groups of 32 row blocks, so the CTAs running at a
//   time share their hidden blocks and weight tiles in L2;
// * every mbarrier wait is bounded (2 s of %globaltimer); a wait that runs
//   out sets CID_STATUS_LM_HEAD_TIMEOUT and a shared abort flag, every role
//   leaves its loop, in-flight TMA copies and MMAs are waited for (bounded)
//   and the TMEM is freed before the CTA exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <climits>
#include <cmath>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kBM = 128;  // rows per tile (UMMA M)
constexpr int kBN = 256;  // vocabulary columns per tile (UMMA N)
constexpr int kBK = 64;   // hidden elements per stage: one 128-byte swizzle row
constexpr int kUmmaK = 16;
constexpr int kStages = 4;
constexpr int kAccBufs = 2;
constexpr uint32_t kTmemCols = kAccBufs * kBN;  // 512: all of TMEM
// Row blocks per raster group.  The CTAs running at once cover about
// 148 / kRowGroup vocabulary groups and kRowGroup hidden blocks (1 MB each);
// with 8-tile units (16 MB of weight a group) 32 kept that set under the
// 126 MB L2 (16 did not: ~150 MB), measured 1-2 % faster at 32768 x 128256
// x 4096; 64 and 128 were slower.
constexpr int kRowGroup = 32;
constexpr int kMaxGroups = 256;                 // record combine limit
// Wide tiles: 256 rows, 3 stages of 64 KiB (32 KiB hidden + 32 KiB weight).
// Raster groups of 16 row blocks (4096 rows, the hidden set of kRowGroup
// 128-row blocks): measured at 32768 x 128256 x 4096 with 8-tile units, DRAM
// reads 18.7 GB with 16, 24.8 GB with 8, 34.6 GB with 4.
constexpr int kWRows = 256;
constexpr int kWStages = 3;
constexpr int kWRowGroup = 16;
constexpr uint32_t kWStageA = kWRows * kBK * 2;  // 32 KiB
constexpr uint32_t kWStageB = kBN * kBK * 2;     // 32 KiB
constexpr uint32_t kWStageBytes = kWStageA + kWStageB;
constexpr size_t kWSmemBytes = kWStages * size_t{kWStageBytes} + 1024 + 256;
// Warpgroup 0: warp 0 TMA, warp 1 MMA, warps 2-3 idle; warpgroups 1-2: the
// epilogue.  The register file is split per SM sub-partition (16384 each),
// and warp w runs on sub-partition w % 4: at launch 3 warps x 168 registers
// fit one; after the split each holds one control warp at 56 and two
// epilogue warps at 224 (32 x (56 + 2 x 224) = 16128).
constexpr int kWThreads = 384;
constexpr int kWLaunchRegs = 168;
constexpr int kWCtrlRegs = 56;
constexpr int kWEpiRegs = 224;
static_assert(128 * kWCtrlRegs + 256 * kWEpiRegs <= kWThreads * kWLaunchRegs,
              "setmaxnreg.inc draws only on the registers the CTA was launched with");
constexpr int kThreads = 192;                   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kStageA = kBM * kBK * 2;     // 16 KiB
constexpr uint32_t kStageB = kBN * kBK * 2;     // 32 KiB
constexpr uint32_t kStageBytes = kStageA + kStageB;
constexpr size_t kSmemBytes = kStages * size_t{kStageBytes} + 1024 /* align */ + 256 /* barriers */;
constexpr unsigned long long kWaitNs = 2000000000ull;  // bounded waits: 2 s
constexpr unsigned long long kDrainNs = 200000000ull;  // drain after an abort: 0.2 s
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kGap = 5.0f;  // offset re-set threshold (natural units), as the stats kernels

// Instruction descriptor of tcgen05.mma kind::f16: D f32 (bits 4-5 = 1),
// A and B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bit 17,
// M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kBN >> 3) << 17) |
                            (uint32_t(kBM >> 4) << 24);

struct LmParams {
  int64_t rows;         // hidden rows
  int64_t vocab;        // weight rows (columns of the logits)
  int64_t vocab_offset; // global column of weight row 0
  int64_t ktiles;       // ceil(hidden / kBK)
  int64_t tiles;        // ceil(vocab / kBN)
  int64_t group_tiles;  // vocabulary tiles per work unit
  int64_t groups;       // ceil(tiles / group_tiles)
  int64_t row_blocks;   // ceil(rows / rows per tile)
  int64_t units;        // row_blocks * groups
  int64_t row_group;    // row blocks per raster group
  const int64_t* ids;
  cid_shard_record_t* records;  // [groups][rows]
  uint32_t* status;
  int round_bf16;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase of `bar` with the given parity; false when `abort` is
// raised or `limit_ns` passes first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          unsigned long long limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (global_ns() - t0 > limit_ns) return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout TMA writes: rows of 128 bytes, 8-row atoms 1024 bytes apart
// (stride byte offset), version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3fffu) | (uint64_t{1} << 16) |
         (uint64_t{1024 >> 4} << 32) | (uint64_t{1} << 46) | (uint64_t{2} << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once all tcgen05.mma issued so far by this thread are done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// Issues the load of 32 consecutive f32 columns of this thread's TMEM lane
// without waiting; the registers are valid after tmem_wait32 on them.
__device__ __forceinline__ void tmem_issue32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Waits for this thread's outstanding TMEM loads; the registers are in-out
// operands so that no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Packed f32 pair arithmetic (sm_100): {a0,a1} * {b,b} + {c,c} and {s0,s1} += {a0,a1}.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %4};\n"
      " mov.b64 rc, {%5, %5};\n fma.rn.f32x2 ra, ra, rb, rc;\n mov.b64 {%0, %1}, ra;\n}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  asm("{\n .reg .b64 ra, rb;\n mov.b64 ra, {%0, %1};\n mov.b64 rb, {%2, %3};\n"
      " add.rn.f32x2 ra, ra, rb;\n mov.b64 {%0, %1}, ra;\n}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}

// ---------------------------------------------------------------------------
// Work units
// ---------------------------------------------------------------------------

__device__ __forceinline__ void unit_coords(const LmParams& p, int64_t u, int64_t& rb,
                                            int64_t& vg) {
  const int64_t per_group = p.row_group * p.groups;
  const int64_t gi = u / per_group;
  const int64_t first = gi * p.row_group;
  const int64_t rows_in = p.row_blocks - first < p.row_group ? p.row_blocks - first : p.row_group;
  const int64_t local = u - gi * per_group;
  rb = first + local % rows_in;
  vg = local / rows_in;
}

__device__ __forceinline__ void raise_abort(volatile int* abort, uint32_t* status) {
  *abort = 1;
  if (status) atomicOr(status, CID_STATUS_LM_HEAD_TIMEOUT);
}

// Per-row online state over the columns of one work unit.
struct RowState {
  float m, om, off, s;
  int64_t where;      // weight column of the first maximum, -1 before any
  int64_t first_nan;  // weight column of the first NaN, -1 if none
  float cur;          // logit at the row's token id (when in the unit)
};

// Folds 32 consecutive logits (weight columns c0..c0+31, already rounded as
// the launch asks) into the state: exponent arguments and sums in packed f32
// pairs.
__device__ __forceinline__ void fold32v(RowState& st, float (&x)[32], int64_t c0, int64_t vocab,
                                        int64_t local_id) {
  if (c0 + 32 > vocab) {  // padding columns of the last tile
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c0 + j >= vocab) x[j] = -INFINITY;
  }
  const int64_t rel = local_id - c0;
  if (rel >= 0 && rel < 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j == rel) st.cur = x[j];
  }
  float cm = x[0];
#pragma unroll
  for (int j = 1; j < 32; ++j) cm = fmaxf(cm, x[j]);  // NaN ignored
  if (cm > st.m) {
    int jj = 0;
#pragma unroll
    for (int j = 31; j >= 0; --j)
      if (x[j] == cm) jj = j;
    st.m = cm;
    st.where = c0 + jj;
    if (st.m > st.om + kGap) {
      const float noff = st.m * kLog2e;
      st.s = st.om == -INFINITY ? (st.s != st.s ? st.s : 0.0f) : st.s * exp2f(st.off - noff);
      st.om = st.m;
      st.off = noff;
    }
  }
  float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
  const float moff = -st.off;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float e0, e1, e2, e3;
    fma2(e0, e1, x[j], x[j + 1], kLog2e, moff);
    fma2(e2, e3, x[j + 2], x[j + 3], kLog2e, moff);
    add2(a0, a1, ex2(e0), ex2(e1));
    add2(b0, b1, ex2(e2), ex2(e3));
  }
  const float cs = (a0 + a1) + (b0 + b1);
  if (cs != cs && st.first_nan < 0) {  // a NaN column (or inf - inf) in the chunk
    int jn = -1;
#pragma unroll
    for (int j = 31; j >= 0; --j)
      if (x[j] != x[j]) jn = j;
    if (jn >= 0) st.first_nan = c0 + jn;
  }
  st.s += cs;
}

// Folds 32 consecutive columns (raw f32 bits from TMEM), rounded to bf16 in
// pairs (one cvt per two) when the launch asks for it.
__device__ __forceinline__ void fold32(RowState& st, const uint32_t (&r)[32], int64_t c0,
                                       int64_t vocab, int64_t local_id, int round_bf16) {
  float x[32];
  if (round_bf16) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      uint32_t pk;  // upper half: column j + 1, lower half: column j
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
          : "=r"(pk)
          : "f"(__uint_as_float(r[j + 1])), "f"(__uint_as_float(r[j])));
      x[j] = __uint_as_float(pk << 16);
      x[j + 1] = __uint_as_float(pk & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]);
  }
  fold32v(st, x, c0, vocab, local_id);
}

// The shard record of one row over one work unit's columns [c_lo, ...):
// (max, sum of exp(x - max), global first argmax with the NaN flag, logit at
// the row's token id).
__device__ __forceinline__ void store_unit_record(const LmParams& p, const RowState& st,
                                                  int64_t vg, int64_t row, int64_t c_lo,
                                                  int64_t local_id) {
  cid_shard_record_t rec;
  rec.max_logit = st.m;
  const bool special = !(st.m > -INFINITY && st.m < INFINITY) || st.s != st.s;
  if (special) {
    const int64_t local = st.first_nan >= 0 ? st.first_nan : (st.where >= 0 ? st.where : c_lo);
    rec.sum_exp = st.m == -INFINITY ? 0.0f : __int_as_float(0x7fffffff);
    rec.index = static_cast<int32_t>(p.vocab_offset + local) |
                (st.first_nan >= 0 ? static_cast<int32_t>(0x80000000u) : 0);
  } else {
    const float top = ex2(fmaf(st.m, kLog2e, -st.off));
    rec.sum_exp = __fdiv_rn(st.s, top);
    rec.index = static_cast<int32_t>(p.vocab_offset + st.where);
  }
  rec.current = local_id >= 0 ? st.cur : 0.0f;
  p.records[vg * p.rows + row] = rec;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads, 1)
    lm_head_stats_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, LmParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-byte aligned
  unsigned char* stage_a = smem;
  unsigned char* stage_b = smem + kStages * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + kAccBufs);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issue_par = 0;  // per-stage bits: ever issued, parity of last issue
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        int64_t rb, vg;
        unit_coords(p, u, rb, vg);
        const int64_t t0 = vg * p.group_tiles;
        const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
        for (int64_t t = t0; ok && t < t1; ++t) {
          for (int64_t kt = 0; kt < p.ktiles; ++kt) {
            if (!mbar_wait(&empty[s], ph ^ 1u, abort, kWaitNs)) {
              if (!*abort) raise_abort(abort, p.status);
              ok = false;
              break;
            }
            mbar_expect_tx(&full[s], kStageBytes);
            tma_load_2d(stage_a + s * kStageA, &map_a, static_cast<int32_t>(kt * kBK),
                        static_cast<int32_t>(rb * kBM), &full[s]);
            tma_load_2d(stage_b + s * kStageB, &map_b, static_cast<int32_t>(kt * kBK),
                        static_cast<int32_t>(t * kBN), &full[s]);
            issued |= 1u << s;
            issue_par = (issue_par & ~(1u << s)) | (ph << s);
            if (++s == kStages) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      // copies in flight land before the CTA exits (immediate unless aborted)
      for (int i = 0; i < kStages; ++i)
        if (issued & (1u << i)) mbar_wait(&full[i], (issue_par >> i) & 1u, nullptr, kDrainNs);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int s = 0, buf = 0;
      uint32_t ph = 0, aph = 0;
      uint64_t* last_bar = nullptr;  // barrier of the last commit and its phase parity
      uint32_t last_par = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        int64_t rb, vg;
        unit_coords(p, u, rb, vg);
        const int64_t t0 = vg * p.group_tiles;
        const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
        for (int64_t t = t0; ok && t < t1; ++t) {
          if (!mbar_wait(&acc_empty[buf], aph ^ 1u, abort, kWaitNs)) {
            if (!*abort) raise_abort(abort, p.status);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kBN);
          for (int64_t kt = 0; kt < p.ktiles; ++kt) {
            if (!mbar_wait(&full[s], ph, abort, kWaitNs)) {
              if (!*abort) raise_abort(abort, p.status);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(stage_a + s * kStageA);
            const uint32_t b0 = smem_u32(stage_b + s * kStageB);
#pragma unroll
            for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
              // K advance inside the 128-byte swizzle atom: +32 bytes per 16 elements
              umma_bf16(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32),
                        (kt | kk) != 0 ? 1u : 0u);
            }
            umma_commit(&empty[s]);  // frees the stage once these MMAs are done
            last_bar = &empty[s];
            last_par = ph;
            if (++s == kStages) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&acc_full[buf]);  // the accumulator is complete
          last_bar = &acc_full[buf];
          last_par = aph;
          if (++buf == kAccBufs) {
            buf = 0;
            aph ^= 1u;
          }
        }
      }
      // MMAs in flight finish before the TMEM is freed (immediate unless aborted)
      if (last_bar != nullptr) mbar_wait(last_bar, last_par, nullptr, kDrainNs);
    }
  } else {
    // ---------------- epilogue: thread = row, TMEM lane = row ----------------
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 for this warp
    const int row_in_block = quarter * 32 + lane;
    int buf = 0;
    uint32_t aph = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      int64_t rb, vg;
      unit_coords(p, u, rb, vg);
      const int64_t t0 = vg * p.group_tiles;
      const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
      const int64_t row = rb * kBM + row_in_block;
      const bool valid = row < p.rows;
      const int64_t c_lo = t0 * kBN;                                        // weight columns
      const int64_t c_hi = t1 * kBN < p.vocab ? t1 * kBN : p.vocab;          // of this unit
      const int64_t id = valid ? p.ids[row] - p.vocab_offset : -1;
      const int64_t local_id = (id >= c_lo && id < c_hi) ? id : INT64_MIN / 2;
      RowState st{-INFINITY, -INFINITY, 0.0f, 0.0f, -1, -1, 0.0f};
      for (int64_t t = t0; t < t1; ++t) {
        bool got = mbar_wait(&acc_full[buf], aph, abort, kWaitNs);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          if (lane == 0 && !*abort) raise_abort(abort, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * kBN);
        // each chunk's TMEM load is in flight while the previous chunk folds
        uint32_t ra[32], rb[32];
        tmem_issue32(taddr, ra);
        tmem_wait32(ra);
#pragma unroll
        for (int c = 0; c < kBN / 32; c += 2) {
          tmem_issue32(taddr + static_cast<uint32_t>((c + 1) * 32), rb);
          fold32(st, ra, t * kBN + c * 32, p.vocab, local_id, p.round_bf16);
          tmem_wait32(rb);
          if (c + 2 < kBN / 32) tmem_issue32(taddr + static_cast<uint32_t>((c + 2) * 32), ra);
          fold32(st, rb, t * kBN + (c + 1) * 32, p.vocab, local_id, p.round_bf16);
          if (c + 2 < kBN / 32) tmem_wait32(ra);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        if (++buf == kAccBufs) {
          buf = 0;
          aph ^= 1u;
        }
      }
      if (!ok) break;
      if (valid) store_unit_record(p, st, vg, row, c_lo, local_id);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// The wide-tile kernel: 256 rows x 256 columns per CTA
// ---------------------------------------------------------------------------
//
// Per K step the MMA warp issues two M=128 MMAs that share the weight slice:
// rows 0-127 of the tile into TMEM columns 0-255, rows 128-255 into columns
// 256-511.  The tile holds all of TMEM, so the epilogue cannot work on one
// accumulator while the other fills; instead each of the eight epilogue
// warps (two per TMEM lane quarter, one per half of the tile) reads its row's
// 256 columns with tcgen05.ld, rounds them to bf16 pairs into 128 registers,
// and releases the accumulator; the fold of those registers then overlaps
// the next tile's MMAs.  The registers come from a setmaxnreg split: the
// control warpgroup (warp 0 TMA, warp 1 MMA, warps 2-3 idle) gives up
// registers, the two epilogue warpgroups take them.  Bitwise the same
// records as the 128-row kernel: every logit is accumulated over K in the
// same order and rounded the same way.
__global__ void __launch_bounds__(kWThreads, 1)
    lm_head_wide_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_b, LmParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-byte aligned
  unsigned char* stage_a = smem;
  unsigned char* stage_b = smem + kWStages * kWStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWStages * kWStageBytes);
  uint64_t* empty = full + kWStages;
  uint64_t* acc_full = empty + kWStages;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);  // one arrival per epilogue warp
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kWCtrlRegs));
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issue_par = 0;  // per-stage bits: ever issued, parity of last issue
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        int64_t rb, vg;
        unit_coords(p, u, rb, vg);
        const int64_t t0 = vg * p.group_tiles;
        const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
        for (int64_t t = t0; ok && t < t1; ++t) {
          for (int64_t kt = 0; kt < p.ktiles; ++kt) {
            if (!mbar_wait(&empty[s], ph ^ 1u, abort, kWaitNs)) {
              if (!*abort) raise_abort(abort, p.status);
              ok = false;
              break;
            }
            mbar_expect_tx(&full[s], kWStageBytes);
            tma_load_2d(stage_a + s * kWStageA, &map_a, static_cast<int32_t>(kt * kBK),
                        static_cast<int32_t>(rb * kWRows), &full[s]);
            tma_load_2d(stage_b + s * kWStageB, &map_b, static_cast<int32_t>(kt * kBK),
                        static_cast<int32_t>(t * kBN), &full[s]);
            issued |= 1u << s;
            issue_par = (issue_par & ~(1u << s)) | (ph << s);
            if (++s == kWStages) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      // copies in flight land before the CTA exits (immediate unless aborted)
      for (int i = 0; i < kWStages; ++i)
        if (issued & (1u << i)) mbar_wait(&full[i], (issue_par >> i) & 1u, nullptr, kDrainNs);
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      int s = 0;
      uint32_t ph = 0, aph = 0;
      uint64_t* last_bar = nullptr;  // barrier of the last commit and its phase parity
      uint32_t last_par = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        int64_t rb, vg;
        unit_coords(p, u, rb, vg);
        const int64_t t0 = vg * p.group_tiles;
        const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
        for (int64_t t = t0; ok && t < t1; ++t) {
          if (!mbar_wait(acc_empty, aph ^ 1u, abort, kWaitNs)) {
            if (!*abort) raise_abort(abort, p.status);
            ok = false;
            break;
          }
          tc_fence_after();
          for (int64_t kt = 0; kt < p.ktiles; ++kt) {
            if (!mbar_wait(&full[s], ph, abort, kWaitNs)) {
              if (!*abort) raise_abort(abort, p.status);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(stage_a + s * kWStageA);
            const uint32_t b0 = smem_u32(stage_b + s * kWStageB);
#pragma unroll
            for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
              // K advance inside the 128-byte swizzle atom: +32 bytes per 16
              // elements; rows 128-255 of the hidden slice start 128 rows
              // (16 KiB, sixteen 1024-byte atoms) further
              const uint32_t acc = (kt | kk) != 0 ? 1u : 0u;
              const uint64_t bd = sw128_desc(b0 + kk * 32);
              umma_bf16(tmem_base, sw128_desc(a0 + kk * 32), bd, acc);
              umma_bf16(tmem_base + kBN, sw128_desc(a0 + kBM * 128 + kk * 32), bd, acc);
            }
            umma_commit(&empty[s]);  // frees the stage once these MMAs are done
            last_bar = &empty[s];
            last_par = ph;
            if (++s == kWStages) {
              s = 0;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(acc_full);  // the tile is complete
          last_bar = acc_full;
          last_par = aph;
          aph ^= 1u;
        }
      }
      // MMAs in flight finish before the TMEM is freed (immediate unless aborted)
      if (last_bar != nullptr) mbar_wait(last_bar, last_par, nullptr, kDrainNs);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kWEpiRegs));
    // ---------------- epilogue: thread = row ----------------
    const int half = (warp - 4) >> 2;  // tile rows 0-127 (TMEM columns 0-255) or 128-255
    const int quarter = warp & 3;      // TMEM lanes 32*quarter .. +31
    const int row_in_block = half * kBM + quarter * 32 + lane;
    uint32_t aph = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      int64_t rb, vg;
      unit_coords(p, u, rb, vg);
      const int64_t t0 = vg * p.group_tiles;
      const int64_t t1 = t0 + p.group_tiles < p.tiles ? t0 + p.group_tiles : p.tiles;
      const int64_t row = rb * kWRows + row_in_block;
      const bool valid = row < p.rows;
      const int64_t c_lo = t0 * kBN;                                // weight columns
      const int64_t c_hi = t1 * kBN < p.vocab ? t1 * kBN : p.vocab;  // of this unit
      const int64_t id = valid ? p.ids[row] - p.vocab_offset : -1;
      const int64_t local_id = (id >= c_lo && id < c_hi) ? id : INT64_MIN / 2;
      RowState st{-INFINITY, -INFINITY, 0.0f, 0.0f, -1, -1, 0.0f};
      for (int64_t t = t0; t < t1; ++t) {
        bool got = mbar_wait(acc_full, aph, abort, kWaitNs);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          if (lane == 0 && !*abort) raise_abort(abort, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(half * kBN);
        uint32_t pk[kBN / 2];  // bf16 pairs: columns 2j (low half) and 2j + 1
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t r[32];
          tmem_issue32(taddr + static_cast<uint32_t>(c * 32), r);
          tmem_wait32(r);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
                : "=r"(pk[c * 16 + j])
                : "f"(__uint_as_float(r[2 * j + 1])), "f"(__uint_as_float(r[2 * j])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);  // the next tile may accumulate
        aph ^= 1u;
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          float x[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            x[2 * j] = __uint_as_float(pk[c * 16 + j] << 16);
            x[2 * j + 1] = __uint_as_float(pk[c * 16 + j] & 0xffff0000u);
          }
          fold32v(st, x, t * kBN + c * 32, p.vocab, local_id);
        }
      }
      if (!ok) break;
      if (valid) store_unit_record(p, st, vg, row, c_lo, local_id);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}


PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {  // thread-safe one-time init
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// 2-D bf16 tensor map over a row-major [outer, inner] matrix, box
// [box_outer, 64] with the 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_outer) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return record_cuda_error(cudaErrorNotSupported);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? CID_OK
             : CID_ERR_INVALID_ARGUMENT;
}

struct Plan {
  int64_t tiles, group_tiles, groups, row_blocks, units;
};

// Work units of a launch whose tiles are tile_rows high (the vocabulary
// grouping, and so the workspace, does not depend on it).
// Two vocabulary tiles per work unit (more when the vocabulary has more than
// 2 * kMaxGroups tiles): many units balance the persistent CTAs' waves and let
// every SM stream weight in launches of few row blocks.  Measured against 8
// tiles at 128256 x 4096: 64 rows 177 vs 242 us, 1024 rows 727-759 vs
// 813-878 us, 8192 rows 5.98 vs 6.03-6.12 ms, 32768 rows 23.9-24.2 vs
// 24.6-24.7 ms.  It depends on the vocabulary only, so the workspace size
// does too.
Plan plan(int64_t rows, int64_t vocab, int64_t tile_rows = kBM) {
  Plan pl;
  pl.tiles = (vocab + kBN - 1) / kBN;
  pl.group_tiles = 2;
  const int64_t least = (pl.tiles + kMaxGroups - 1) / kMaxGroups;
  if (pl.group_tiles < least) pl.group_tiles = least;
  pl.groups = (pl.tiles + pl.group_tiles - 1) / pl.group_tiles;
  pl.row_blocks = (rows + tile_rows - 1) / tile_rows;
  pl.units = pl.row_blocks * pl.groups;
  return pl;
}

// Smallest launch served by the wide-tile kernel.  Measured at 128256 x 4096
// against the 128-row kernel: 1024 rows 0.77 vs 0.90 ms, 2048 rows level,
// 4096 rows 2.95 vs 3.29 ms, 8192 rows 6.03 vs 6.61 ms.  Fewer rows are a
// handful of row blocks, where 256-row tiles leave SMs idle.
constexpr int64_t kWideMinRows = 1024;

// The wide kernel's setmaxnreg split is sized for kWLaunchRegs registers a
// thread at launch; a build whose register allocation differs uses the
// 128-row kernel instead (a split above the launch's registers would never
// complete).
bool wide_kernel_ready() {
  static const bool ok = [] {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, lm_head_wide_kernel) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return fa.numRegs == kWLaunchRegs;
  }();
  return ok;
}

}  // namespace
}  // namespace cid

using namespace cid;

namespace {

// Row limit of the fused LM head (the last row tile's index stays in int32).
constexpr int64_t kMaxLmRows = INT32_MAX - kBM;

// The operands every LM-head call shares: rows x hidden_dim and
// vocab x hidden_dim bf16, hidden_dim a positive multiple of 8 (16-byte TMA
// rows) up to INT32_MAX - kBK, 16-byte-aligned operands and workspace.
int check_lm_head(const void* hidden, int64_t rows, int64_t hidden_dim, const void* weight,
                  int64_t vocab, const int64_t* token_ids, const void* workspace,
                  const uint32_t* status) {
  int64_t n = 0;
  if (rows < 0 || rows > kMaxLmRows || hidden_dim <= 0 || hidden_dim % 8 != 0 ||
      hidden_dim > INT32_MAX - kBK || vocab <= 0 || vocab > INT32_MAX ||
      !count_ok(rows, hidden_dim, &n) || n > kMaxCount || !count_ok(vocab, hidden_dim, &n) ||
      n > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{hidden, 16}, {weight, 16}, {token_ids, 8}, {workspace, 16}, {status, 4}}))
    return CID_ERR_MISALIGNED;
  return CID_OK;
}

}  // namespace

extern "C" size_t cid_lm_head_workspace_bytes(int64_t rows, int64_t vocab) {
  if (rows <= 0 || rows > kMaxLmRows || vocab <= 0 || vocab > INT32_MAX) return 0;
  const Plan pl = plan(rows, vocab);
  return static_cast<size_t>(pl.groups) * static_cast<size_t>(rows) * sizeof(cid_shard_record_t);
}

namespace {

// Validates, launches the fused kernel (records of every row and vocabulary
// group into `workspace`) and fills the groups' global column offsets.
int launch_lm_head(const void* hidden, int64_t rows, int64_t hidden_dim, const void* weight,
                   int64_t vocab, int64_t vocab_offset, const int64_t* token_ids, int round_bf16,
                   void* workspace, size_t workspace_bytes, uint32_t* status, void* stream,
                   int64_t (&offsets)[kMaxGroups + 1], int& groups) {
  // TMA: row strides and base addresses 16-byte aligned
  if (workspace_bytes < cid_lm_head_workspace_bytes(rows, vocab)) return CID_ERR_SCRATCH_LIMIT;
  const bool wide = round_bf16 && rows >= kWideMinRows && rows <= INT32_MAX - kWRows &&
                    wide_kernel_ready();
  const int64_t tile_rows = wide ? kWRows : kBM;
  const Plan pl = plan(rows, vocab, tile_rows);
  CUtensorMap map_a, map_b;
  int rc = make_map(&map_a, hidden, hidden_dim, rows, static_cast<int>(tile_rows));
  if (rc == CID_OK) rc = make_map(&map_b, weight, hidden_dim, vocab, kBN);
  if (rc != CID_OK) return rc;
  LmParams p = {};
  p.rows = rows;
  p.vocab = vocab;
  p.vocab_offset = vocab_offset;
  p.ktiles = (hidden_dim + kBK - 1) / kBK;
  p.tiles = pl.tiles;
  p.group_tiles = pl.group_tiles;
  p.groups = pl.groups;
  p.row_blocks = pl.row_blocks;
  p.units = pl.units;
  p.row_group = wide ? kWRowGroup : kRowGroup;
  p.ids = token_ids;
  p.records = static_cast<cid_shard_record_t*>(workspace);
  p.status = status;
  p.round_bf16 = round_bf16 ? 1 : 0;
  const int64_t grid = pl.units < sm_count() ? pl.units : sm_count();
  if (wide) {
    cudaError_t e = cudaFuncSetAttribute(lm_head_wide_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kWSmemBytes));
    if (e != cudaSuccess) return record_cuda_error(e);
    lm_head_wide_kernel<<<static_cast<unsigned>(grid), kWThreads, kWSmemBytes,
                          as_stream(stream)>>>(map_a, map_b, p);
  } else {
    cudaError_t e = cudaFuncSetAttribute(lm_head_stats_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return record_cuda_error(e);
    lm_head_stats_kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes,
                           as_stream(stream)>>>(map_a, map_b, p);
  }
  rc = launch_result();
  if (rc != CID_OK) return rc;
  groups = static_cast<int>(pl.groups);
  for (int64_t g = 0; g < pl.groups; ++g) offsets[g] = vocab_offset + g * pl.group_tiles * kBN;
  offsets[pl.groups] = vocab_offset + vocab;
  return CID_OK;
}

}  // namespace

extern "C" int cid_lm_head_display_statistics(const void* hidden, int64_t rows, int64_t hidden_dim,
                                              const void* weight, int64_t vocab,
                                              const int64_t* token_ids, int round_bf16,
                                              float* confidence, int64_t* predicted,
                                              float* current_confidence, void* workspace,
                                              size_t workspace_bytes, uint32_t* status,
                                              void* stream) {
  int rc = check_lm_head(hidden, rows, hidden_dim, weight, vocab, token_ids, workspace, status);
  if (rc != CID_OK) return rc;
  if (misaligned({{confidence, 4}, {predicted, 8}, {current_confidence, 4}}))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({hidden, weight, token_ids, workspace, confidence, predicted, current_confidence}))
    return CID_ERR_INVALID_ARGUMENT;
  int64_t offsets[kMaxGroups + 1];
  int groups = 0;
  rc = launch_lm_head(hidden, rows, hidden_dim, weight, vocab, 0, token_ids, round_bf16,
                      workspace, workspace_bytes, status, stream, offsets, groups);
  if (rc != CID_OK) return rc;
  // merge the groups of every row (ascending column ranges) into its statistics
  return cid_display_combine_records(static_cast<const cid_shard_record_t*>(workspace), groups,
                                     offsets, token_ids, rows, confidence, predicted,
                                     current_confidence, status, stream);
}

extern "C" int cid_lm_head_shard_records(const void* hidden, int64_t rows, int64_t hidden_dim,
                                         const void* weight_shard, int64_t vocab_shard,
                                         int64_t vocab_offset, int64_t total_vocab,
                                         const int64_t* token_ids, int round_bf16,
                                         cid_shard_record_t* records, void* workspace,
                                         size_t workspace_bytes, uint32_t* status, void* stream) {
  int rc = check_lm_head(hidden, rows, hidden_dim, weight_shard, vocab_shard, token_ids,
                         workspace, status);
  if (rc != CID_OK) return rc;
  if (vocab_offset < 0 || total_vocab > INT32_MAX || total_vocab < vocab_shard ||
      vocab_offset > total_vocab - vocab_shard)
    return CID_ERR_INVALID_ARGUMENT;
  if (misaligned({{records, 4}})) return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  if (any_null({hidden, weight_shard, token_ids, workspace, records}))
    return CID_ERR_INVALID_ARGUMENT;
  int64_t offsets[kMaxGroups + 1];
  int groups = 0;
  rc = launch_lm_head(hidden, rows, hidden_dim, weight_shard, vocab_shard, vocab_offset,
                      token_ids, round_bf16, workspace, workspace_bytes, status, stream, offsets,
                      groups);
  if (rc != CID_OK) return rc;
  // one record per row over the whole shard
  return cid_display_merge_records(static_cast<const cid_shard_record_t*>(workspace), groups,
                                   offsets, token_ids, rows, records, stream);
}
