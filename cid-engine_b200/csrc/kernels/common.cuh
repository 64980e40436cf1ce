// Shared device/host helpers for the sm_100a kernels behind the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <initializer_list>

#include "cid_engine_b200.h"

namespace cid {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Host-side helpers
// ---------------------------------------------------------------------------

// Records the CUDA error (for cid_last_cuda_error) and maps it to a result.
int record_cuda_error(cudaError_t err);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool is_float_dtype(cid_dtype_t dt) {
  return dt == CID_DTYPE_F32 || dt == CID_DTYPE_F64 || dt == CID_DTYPE_F16 ||
         dt == CID_DTYPE_BF16;
}

inline bool is_known_dtype(int dt) { return dt >= 0 && dt <= CID_DTYPE_I16; }

inline int dtype_size(cid_dtype_t dt) {
  switch (dt) {
    case CID_DTYPE_F64:
    case CID_DTYPE_I64: return 8;
    case CID_DTYPE_F32:
    case CID_DTYPE_I32: return 4;
    case CID_DTYPE_F16:
    case CID_DTYPE_BF16:
    case CID_DTYPE_I16: return 2;
    default: return 1;
  }
}

// Argument checks shared by the entry points.  Each entry point checks, in
// this order and before any CUDA call: its dtype codes
// (CID_ERR_UNSUPPORTED_DTYPE); its scalar arguments and extents
// (CID_ERR_INVALID_ARGUMENT: negative extents, element counts that overflow
// int64, row counts above kMaxRows); the alignment of every non-NULL pointer
// to its element size (CID_ERR_MISALIGNED); then it returns CID_OK when there
// is no work, and otherwise requires every array of non-zero extent to be
// non-NULL (CID_ERR_INVALID_ARGUMENT).

// Largest row (or batch) count of any entry point: grid dimensions and the
// kernels' 32-bit row indexes stay in range.
constexpr int64_t kMaxRows = INT32_MAX;
// Largest element count of any array argument (2^58): byte offsets of
// elements up to 16 bytes wide stay within int64.
constexpr int64_t kMaxCount = int64_t{1} << 58;

// a * b as an element count: false when either is negative or the product
// does not fit in int64 (callers compare the product with kMaxCount).
inline bool count_ok(int64_t a, int64_t b, int64_t* product = nullptr) {
  int64_t r = 0;
  if (a < 0 || b < 0 || __builtin_mul_overflow(a, b, &r)) return false;
  if (product) *product = r;
  return true;
}

// a * b * c likewise.
inline bool count_ok(int64_t a, int64_t b, int64_t c, int64_t* product = nullptr) {
  int64_t ab = 0;
  return count_ok(a, b, &ab) && count_ok(ab, c, product);
}

struct Aligned {
  const void* ptr;
  size_t bytes;
};

// True when a non-NULL pointer of the list is not a multiple of its bytes.
inline bool misaligned(std::initializer_list<Aligned> ptrs) {
  for (const Aligned& a : ptrs)
    if (a.ptr != nullptr && reinterpret_cast<uintptr_t>(a.ptr) % a.bytes != 0) return true;
  return false;
}

inline bool any_null(std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (p == nullptr) return true;
  return false;
}

// Checks the launch that was just enqueued.
inline int launch_result() { return record_cuda_error(cudaGetLastError()); }

inline int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Programmatic dependent launch (sm_90 and later).  A kernel launched with
// launch_pdl may be scheduled while the kernel before it in the stream is
// still running, so its launch latency hides under that kernel's tail.  Such
// a kernel calls pdl_wait() before its first global memory access, read or
// write (the wait returns once the previous kernel has completed and its
// writes are visible), and pdl_trigger() once its own dependents may be
// scheduled.  In a kernel launched without the attribute both are no-ops.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record_cuda_error(cudaLaunchKernelEx(&cfg, kernel, args...));
}

// ---------------------------------------------------------------------------
// Device-side helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// 2^x with the SFU (ex2.approx.ftz.f32: a few ulp of relative error).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float bf16_bits_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_bits_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Value of element i of an array of runtime dtype `dt`, as float.  Used by
// the small slot/snapshot kernels, whose inputs come in any dtype.
__device__ __forceinline__ float load_float(cid_dtype_t dt, const void* p, int64_t i) {
  switch (dt) {
    case CID_DTYPE_F32: return static_cast<const float*>(p)[i];
    case CID_DTYPE_F64: return static_cast<float>(static_cast<const double*>(p)[i]);
    case CID_DTYPE_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case CID_DTYPE_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case CID_DTYPE_BOOL:
    case CID_DTYPE_U8: return static_cast<float>(static_cast<const uint8_t*>(p)[i]);
    case CID_DTYPE_I8: return static_cast<float>(static_cast<const int8_t*>(p)[i]);
    case CID_DTYPE_I16: return static_cast<float>(static_cast<const int16_t*>(p)[i]);
    case CID_DTYPE_I32: return static_cast<float>(static_cast<const int32_t*>(p)[i]);
    case CID_DTYPE_I64: return static_cast<float>(static_cast<const int64_t*>(p)[i]);
  }
  return __int_as_float(0x7fc00000);
}

__device__ __forceinline__ double load_double(cid_dtype_t dt, const void* p, int64_t i) {
  if (dt == CID_DTYPE_F64) return static_cast<const double*>(p)[i];
  if (dt == CID_DTYPE_I64) return static_cast<double>(static_cast<const int64_t*>(p)[i]);
  return static_cast<double>(load_float(dt, p, i));
}

// `tensor.to(torch.bool)`: non-zero (NaN included) is true.
__device__ __forceinline__ bool load_truthy(cid_dtype_t dt, const void* p, int64_t i) {
  switch (dt) {
    case CID_DTYPE_BOOL:
    case CID_DTYPE_U8:
    case CID_DTYPE_I8: return static_cast<const uint8_t*>(p)[i] != 0;
    case CID_DTYPE_I16: return static_cast<const int16_t*>(p)[i] != 0;
    case CID_DTYPE_F16:
    case CID_DTYPE_BF16: return (static_cast<const uint16_t*>(p)[i] & 0x7fffu) != 0;
    case CID_DTYPE_I32: return static_cast<const int32_t*>(p)[i] != 0;
    case CID_DTYPE_F32: return (static_cast<const uint32_t*>(p)[i] & 0x7fffffffu) != 0;
    case CID_DTYPE_I64: return static_cast<const int64_t*>(p)[i] != 0;
    case CID_DTYPE_F64:
      return (static_cast<const uint64_t*>(p)[i] & 0x7fffffffffffffffull) != 0;
  }
  return false;
}

// Round a float result to the storage type of `dt` and back (ATen evaluates
// half/bfloat16 elementwise ops in float and rounds the result).
__device__ __forceinline__ float round_to(cid_dtype_t dt, float x) {
  if (dt == CID_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dt == CID_DTYPE_F16) return __half2float(__float2half_rn(x));
  return x;
}

__device__ __forceinline__ void store_float(cid_dtype_t dt, void* p, int64_t i, float x) {
  switch (dt) {
    case CID_DTYPE_F32: static_cast<float*>(p)[i] = x; break;
    case CID_DTYPE_F16: static_cast<__half*>(p)[i] = __float2half_rn(x); break;
    case CID_DTYPE_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x); break;
    case CID_DTYPE_F64: static_cast<double*>(p)[i] = static_cast<double>(x); break;
    default: break;
  }
}

// float32 sigmoid as 1 / (1 + exp(-x)) with each step rounded to float32 and
// exp evaluated in double (correctly rounded to float32 but for vanishingly
// rare double-rounding cases).  ATen's scalar sigmoid loop agrees with this;
// its vectorised loop can differ by up to two ulps.
__device__ __forceinline__ float sigmoid_f32(float x) {
  const float e = static_cast<float>(exp(-static_cast<double>(x)));
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

// ATen max/argmax order: NaN first (lowest index), then larger value, then
// lower index.  Returns true when (v, i) should replace (bv, bi).
__device__ __forceinline__ bool argmax_better(float v, int64_t i, float bv, int64_t bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;
  if (vn) return i < bi;
  return v > bv || (v == bv && i < bi);
}

}  // namespace cid
