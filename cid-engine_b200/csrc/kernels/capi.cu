// ABI version, result strings and the per-thread record of the last CUDA
// error seen inside the library.
#include <cstdio>

#include "common.cuh"

namespace cid {
namespace {
thread_local char g_last_error[256] = "";
}  // namespace

int record_cuda_error(cudaError_t err) {
  if (err == cudaSuccess) return CID_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(err),
                cudaGetErrorString(err));
  return err == cudaErrorInvalidConfiguration || err == cudaErrorLaunchOutOfResources
             ? CID_ERR_LAUNCH
             : CID_ERR_CUDA;
}

}  // namespace cid

extern "C" int cid_abi_version(void) { return CID_ENGINE_B200_ABI_VERSION; }

extern "C" const char* cid_result_string(int result) {
  switch (result) {
    case CID_OK: return "ok";
    case CID_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CID_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case CID_ERR_LAUNCH: return "kernel launch failed (configuration or resources)";
    case CID_ERR_MISALIGNED: return "misaligned pointer";
    case CID_ERR_CUDA: return "CUDA runtime error";
    case CID_ERR_SCRATCH_LIMIT:
      return "batch exceeds the allocation-free entry point's fixed scratch (CID_NO_ALLOC_MAX_BATCH rows)";
    default: return "unknown result";
  }
}

extern "C" const char* cid_last_cuda_error(void) { return cid::g_last_error; }
