// Status strings, error detail and build tag of the C ABI.
#include <stdio.h>

#include "common.cuh"

namespace nf4b {

static thread_local char g_last_error[256] = "";

void record_cuda_error(const char* where, cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorName(e),
           cudaGetErrorString(e));
}

void record_driver_error(const char* where, int cu_result) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: CUresult %d", where, cu_result);
}

void record_message(const char* msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

}  // namespace nf4b

extern "C" const char* nf4b_status_string(int status) {
  switch (status) {
    case NF4B_OK: return "ok";
    case NF4B_ERR_INVALID_ARG: return "invalid argument (null pointer or inconsistent size)";
    case NF4B_ERR_UNSUPPORTED: return "unsupported input (outside the kernel envelope); nothing launched";
    case NF4B_ERR_ALIGNMENT: return "misaligned pointer or row stride";
    case NF4B_ERR_CUDA: return "CUDA runtime or launch error";
    case NF4B_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    default: return "unknown status";
  }
}

extern "C" const char* nf4b_last_error(void) { return nf4b::g_last_error; }

extern "C" const char* nf4b_version(void) { return "stew_nf4 sm_100a 0.1"; }
