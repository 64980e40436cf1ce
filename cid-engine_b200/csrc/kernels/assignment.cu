// Batched linear assignment (Hungarian method with potentials) for at most 16
// columns: one warp per batch element, lane j owning column j (lane 0 is the
// method's virtual column 0) with the column's potential, its matched row and
// that row's potential, all in registers.  Semantics of the reference
// (csrc/ops.cpp:68-175 of fwerkor/cid-engine v1.1.0): costs are read as
// float32 and every reduced cost, potential and slack is computed in double
// with the same operations in the same order, so the assignment is
// bit-identical; among equal slacks the lowest column is taken, as the
// reference's sequential scan does.
//
// The column search of one row ends after at most columns + 1 steps on finite
// costs; the loop is bounded by that count, and a batch element whose search
// does not end (non-finite costs) or whose row count lies outside [0, rows]
// keeps -1 everywhere and sets CID_STATUS_ASSIGNMENT_INVALID.
#include <cmath>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kMaxColumns = 16;
constexpr int kWarpsPerBlock = 4;

struct AssignParams {
  cid_dtype_t dtype;
  const void* costs;
  const int64_t* row_counts;
  int64_t batch, rows, columns;
  int64_t* out;
  uint32_t* status;
};

// Unsigned key whose order is the order of doubles (no NaN): -0 and +0 give
// the same key, as they compare equal.
__device__ __forceinline__ unsigned long long order_key(double x) {
  long long b = __double_as_longlong(x);
  if (b == static_cast<long long>(0x8000000000000000ull)) b = 0;  // -0 -> +0
  return b >= 0 ? static_cast<unsigned long long>(b) ^ 0x8000000000000000ull
                : ~static_cast<unsigned long long>(b);
}

__global__ void assignment_kernel(AssignParams p) {
  // the batch element's active rows of costs, as float32 (one coalesced
  // read; the column search then reads shared memory, not one dependent
  // global load per step)
  __shared__ float c_all[kWarpsPerBlock][kMaxColumns * kMaxColumns];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + warp;
  if (b >= p.batch) return;  // uniform per warp
  const int m = static_cast<int>(p.columns);
  const int64_t rows = p.rows;
  for (int64_t r = lane; r < rows; r += 32) p.out[b * rows + r] = -1;
  __syncwarp();  // the -1 fill is ordered before other lanes' final writes
  const int64_t active = p.row_counts[b];
  if (active < 0 || active > rows) {
    if (lane == 0 && p.status) atomicOr(p.status, CID_STATUS_ASSIGNMENT_INVALID);
    return;
  }
  float* cost = c_all[warp];
  const int64_t base = b * rows * m;
  for (int64_t e = lane; e < active * m; e += 32)
    cost[e] = load_float(p.dtype, p.costs, base + e);
  __syncwarp();
  const bool col = lane >= 1 && lane <= m;  // a real column
  double v = 0.0;                           // potential of column `lane`
  int pj = 0;                               // row matched to column `lane` (0 = none)
  double uj = 0.0;                          // potential of row `pj` (moves with the row)
  int way = 0;
  bool ok = true;
  for (int row = 1; row <= active && ok; ++row) {
    if (lane == 0) {
      pj = row;
      uj = 0.0;  // a row's potential is 0 until its own search starts
    }
    int j0 = 0;
    double minv = INFINITY;
    bool used = false;
    int steps = 0;
    for (;;) {
      if (lane == j0) used = true;
      const int i0 = __shfl_sync(0xffffffffu, pj, j0);
      const double ui0 = __shfl_sync(0xffffffffu, uj, j0);  // u[i0]
      // reduced costs of the unused columns, in double: (c - u[i0]) - v[j]
      if (col && !used) {
        const double c = static_cast<double>(cost[(i0 - 1) * m + (lane - 1)]);
        const double cur = __dsub_rn(__dsub_rn(c, ui0), v);
        if (cur < minv) {
          minv = cur;
          way = j0;
        }
      }
      // delta = smallest slack among unused columns, lowest column on ties;
      // only values below +inf can be chosen (the reference's strict `<`):
      // three warp min-reductions over the slack's order key (high word, low
      // word, then the lane among equal keys), the winner's slack by shuffle
      const bool cand = col && !used && minv < INFINITY;
      const unsigned long long key = cand ? order_key(minv) : ~0ull;
      const unsigned khi = static_cast<unsigned>(key >> 32), klo = static_cast<unsigned>(key);
      const unsigned hi = __reduce_min_sync(0xffffffffu, khi);
      const unsigned lo = __reduce_min_sync(0xffffffffu, khi == hi ? klo : 0xffffffffu);
      const unsigned wl =
          __reduce_min_sync(0xffffffffu, cand && khi == hi && klo == lo ? unsigned(lane) : 32u);
      const double win = __shfl_sync(0xffffffffu, minv, wl & 31u);
      const double delta = wl < 32u ? win : INFINITY;
      const int j1 = wl < 32u ? static_cast<int>(wl) : 0;
      // potentials: u[p[j]] += delta, v[j] -= delta for used columns (each
      // used column holds a distinct row); slack -= delta for the others
      if (lane <= m) {
        if (used) {
          uj = __dadd_rn(uj, delta);
          v = __dsub_rn(v, delta);
        } else {
          minv = __dsub_rn(minv, delta);
        }
      }
      j0 = j1;
      const int pj0 = __shfl_sync(0xffffffffu, pj, j0);
      if (pj0 == 0) break;
      if (++steps > m + 1 || j1 == 0) {  // no free column reachable: give up
        ok = false;
        break;
      }
    }
    if (!ok) break;
    // augment along `way` back to the virtual column
    for (int k = 0; k <= m + 1; ++k) {
      const int j1 = __shfl_sync(0xffffffffu, way, j0);
      const int pnew = __shfl_sync(0xffffffffu, pj, j1);
      const double unew = __shfl_sync(0xffffffffu, uj, j1);
      if (lane == j0) {
        pj = pnew;
        uj = unew;
      }
      j0 = j1;
      if (j0 == 0) break;
    }
  }
  if (!ok) {
    if (lane == 0 && p.status) atomicOr(p.status, CID_STATUS_ASSIGNMENT_INVALID);
    return;
  }
  if (col && pj > 0 && pj <= active) p.out[b * rows + (pj - 1)] = lane - 1;
}

}  // namespace
}  // namespace cid

using namespace cid;

extern "C" int cid_batched_linear_assignment(cid_dtype_t cost_dtype, const void* costs,
                                             const int64_t* row_counts, int64_t batch,
                                             int64_t rows, int64_t columns, int64_t* out,
                                             uint32_t* status, void* stream) {
  if (!is_float_dtype(cost_dtype)) return CID_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || batch > kMaxRows || rows < 0 || columns < 0 || rows > columns ||
      columns > kMaxColumns)
    return CID_ERR_INVALID_ARGUMENT;  // csrc/ops.cpp:71-86
  if (misaligned({{costs, static_cast<size_t>(dtype_size(cost_dtype))}, {row_counts, 8},
                  {out, 8}, {status, 4}}))
    return CID_ERR_MISALIGNED;
  if (batch == 0 || rows == 0) return CID_OK;
  if (any_null({costs, row_counts, out})) return CID_ERR_INVALID_ARGUMENT;
  AssignParams p{cost_dtype, costs, row_counts, batch, rows, columns, out, status};
  const int64_t blocks = (batch + kWarpsPerBlock - 1) / kWarpsPerBlock;
  assignment_kernel<<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, as_stream(stream)>>>(p);
  return launch_result();
}
