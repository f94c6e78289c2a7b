// Status strings and version of the mamba4_b200 C ABI.
#include "common.cuh"

extern "C" const char* m4_status_string(int status) {
  switch (status) {
    case M4_OK: return "ok";
    case M4_ERR_DIMS: return "invalid dimensions";
    case M4_ERR_UNSUPPORTED: return "unsupported dimensions for this build";
    case M4_ERR_NULL: return "required pointer is NULL";
    case M4_ERR_ALIGN: return "pointer not 16-byte aligned";
    case M4_ERR_LAUNCH: return "CUDA launch failed";
    case M4_ERR_WORKSPACE: return "residual or workspace buffer too small";
    case M4_ERR_TIMEOUT: return "a bounded wait for the tensor cores gave up";
    default: return "unknown status";
  }
}

extern "C" const char* m4_version(void) { return "mamba4_b200 0.1 sm_100a"; }
