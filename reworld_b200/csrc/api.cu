// Library-wide C-ABI entry points (error strings, ABI version).
#include "../../include/reworld_b200.h"

extern "C" const char* rw_error_string(int code) {
  switch (code) {
    case RW_OK: return "ok";
    case RW_ERR_INVALID_ARG: return "invalid argument (null pointer, size, alignment or stride)";
    case RW_ERR_UNSUPPORTED: return "unsupported configuration (head_dim must be 128)";
    case RW_ERR_CUDA: return "CUDA runtime error (launch failed)";
    case RW_ERR_DRIVER: return "TMA descriptor encoding failed";
    case RW_ERR_CAPACITY: return "request exceeds a fixed capacity";
    default: return "unknown error";
  }
}

extern "C" int rw_abi_version(void) { return 4; }
