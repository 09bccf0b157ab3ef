// abi.cu — status strings and version of the C ABI (include/cek.h).
#include "common.cuh"

extern "C" const char* cek_status_string(int status) {
  switch (status) {
    case CEK_OK: return "ok";
    case CEK_ERR_INVALID_ARG: return "invalid argument";
    case CEK_ERR_UNSUPPORTED: return "unsupported argument combination";
    case CEK_ERR_ALIGNMENT: return "pointer or pitch not 16-byte aligned";
    case CEK_ERR_LAUNCH: return "CUDA launch failed";
    case CEK_ERR_TIMEOUT: return "bounded device wait timed out";
    case CEK_ERR_SCRATCH_LIMIT: return "size exceeds the fixed scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

extern "C" const char* cek_version(void) { return "cek_b200 0.1 sm_100a"; }
