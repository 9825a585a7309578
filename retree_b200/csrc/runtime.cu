// Library-level entry points: ABI version, error reporting.
#include "common.cuh"
#include "host_util.h"

#include <cstdlib>
#include <cstring>

namespace rt {
thread_local int g_last_cuda_error = 0;

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("RETREE_B200_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}
}

extern "C" int rt_abi_version(void) { return 2; }

extern "C" int rt_last_cuda_error(void) { return rt::g_last_cuda_error; }

extern "C" const char* rt_status_string(int code) {
  switch (code) {
    case RT_OK: return "ok";
    case RT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RT_ERR_UNSUPPORTED: return "unsupported shape or layout";
    case RT_ERR_WORKSPACE: return "workspace missing or too small";
    case RT_ERR_CUDA: return "CUDA launch or driver error";
    case RT_DEV_WAIT_TIMEOUT: return "device: a bounded wait ran out";
    case RT_DEV_BAD_INDEX: return "device: index out of range";
    case RT_DEV_OVERFLOW: return "device: capacity exceeded";
    default: return "unknown status";
  }
}
