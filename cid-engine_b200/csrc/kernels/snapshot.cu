// Compact materialisation snapshot: one warp per (batch, slot) row packs
//   [selected, argmax(lifecycle), uncertainty, noise_delta,
//    sigmoid(roles[0..R)), semantic[indices[0..K)]]
// into a float32 row of width 4 + R + K (csrc/ops.cpp:556-615 of
// fwerkor/cid-engine v1.1.0).  Lanes cover consecutive output columns, so
// the row is written with coalesced stores.  Indices outside the semantic
// width are not read: the column is written as NaN and a status bit is set
// (the reference CPU path raises after a host sync instead).
#include <cmath>

#include "common.cuh"

namespace cid {
namespace {

constexpr int kWarpsPerBlock = 8;

struct SnapshotParams {
  cid_dtype_t sem_dt;
  const void* sem;
  int64_t hidden;
  cid_dtype_t role_dt;
  const void* roles;
  int64_t nroles;
  cid_dtype_t unc_dt;
  const void* unc;
  cid_dtype_t noise_dt;
  const void* noise;
  cid_dtype_t life_dt;
  const void* life;
  int64_t F;
  const uint8_t* selected;
  const int64_t* idx;
  int64_t K;
  int64_t rows;
  float* out;
  uint32_t* status;
};

__global__ void snapshot_kernel(SnapshotParams p) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t W = 4 + p.nroles + p.K;
  float* o = p.out + row * W;
  for (int64_t c = lane; c < W; c += 32) {
    float v;
    if (c == 0) {
      v = p.selected[row] ? 1.0f : 0.0f;
    } else if (c == 1) {
      // argmax of lifecycle.to(float) (ops.cpp:604-606): first NaN, else first max
      float bv = load_float(p.life_dt, p.life, row * p.F);
      int64_t bi = 0;
      for (int64_t k = 1; k < p.F; ++k) {
        if (bv != bv) break;
        const float x = load_float(p.life_dt, p.life, row * p.F + k);
        if (x != x || x > bv) {
          bv = x;
          bi = k;
        }
      }
      v = static_cast<float>(bi);
    } else if (c == 2) {
      v = load_float(p.unc_dt, p.unc, row);
    } else if (c == 3) {
      v = load_float(p.noise_dt, p.noise, row);
    } else if (c < 4 + p.nroles) {
      v = sigmoid_f32(load_float(p.role_dt, p.roles, row * p.nroles + (c - 4)));
    } else {
      const int64_t j = p.idx[c - 4 - p.nroles];
      if (j >= 0 && j < p.hidden) {
        v = load_float(p.sem_dt, p.sem, row * p.hidden + j);
      } else {
        v = __int_as_float(0x7fffffff);
        if (p.status) atomicOr(p.status, CID_STATUS_SEMANTIC_INDEX_OUT_OF_RANGE);
      }
    }
    o[c] = v;
  }
}

}  // namespace
}  // namespace cid

using namespace cid;

extern "C" int cid_materialize_cell_snapshot(
    cid_dtype_t sem_dtype, const void* semantic, int64_t hidden, cid_dtype_t role_dtype,
    const void* roles, int64_t nroles, cid_dtype_t unc_dtype, const void* uncertainty,
    cid_dtype_t noise_dtype, const void* noise_delta, cid_dtype_t life_dtype,
    const void* lifecycle, int64_t lifecycles, const uint8_t* selected, const int64_t* indices,
    int64_t nindices, int64_t rows, float* out, uint32_t* status, void* stream) {
  if (!is_float_dtype(sem_dtype) || !is_float_dtype(role_dtype) || !is_float_dtype(unc_dtype) ||
      !is_float_dtype(noise_dtype) || !is_float_dtype(life_dtype))
    return CID_ERR_UNSUPPORTED_DTYPE;
  // rows x hidden, roles and lifecycles inputs; rows x (4 + roles + indices) output
  int64_t n = 0;
  if (rows < 0 || rows > kMaxRows || lifecycles <= 0 || nroles < 0 || nroles > kMaxCount ||
      nindices < 0 || nindices > kMaxCount || !count_ok(rows, hidden, &n) || n > kMaxCount ||
      !count_ok(rows, nroles, &n) || n > kMaxCount || !count_ok(rows, lifecycles, &n) ||
      n > kMaxCount || !count_ok(rows, 4 + nroles + nindices, &n) || n > kMaxCount)
    return CID_ERR_INVALID_ARGUMENT;
  auto es = [](cid_dtype_t dt) { return static_cast<size_t>(dtype_size(dt)); };
  if (misaligned({{semantic, es(sem_dtype)}, {roles, es(role_dtype)},
                  {uncertainty, es(unc_dtype)}, {noise_delta, es(noise_dtype)},
                  {lifecycle, es(life_dtype)}, {indices, 8}, {out, 4}, {status, 4}}))
    return CID_ERR_MISALIGNED;
  if (rows == 0) return CID_OK;
  // the semantic values are read only at the indices, and only when the
  // width is non-zero (every index is out of range otherwise)
  if (any_null({out, selected, uncertainty, noise_delta, lifecycle}) ||
      (nroles > 0 && roles == nullptr) || (nindices > 0 && indices == nullptr) ||
      (nindices > 0 && hidden > 0 && semantic == nullptr))
    return CID_ERR_INVALID_ARGUMENT;
  SnapshotParams p{sem_dtype, semantic, hidden, role_dtype, roles, nroles, unc_dtype,
                   uncertainty, noise_dtype, noise_delta, life_dtype, lifecycle, lifecycles,
                   selected, indices, nindices, rows, out, status};
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  return launch_pdl(snapshot_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kWarpsPerBlock * 32),
                    0, as_stream(stream), p);
}
