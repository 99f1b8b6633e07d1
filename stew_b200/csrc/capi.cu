// Status strings and build tag of the C ABI.
#include "common.cuh"

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

extern "C" const char* nf4b_version(void) { return "stew_nf4 sm_100a 0.1"; }
