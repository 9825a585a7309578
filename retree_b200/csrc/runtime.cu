// Library-level entry points: ABI version, error reporting.
#include "common.cuh"
#include "host_util.h"

#include <atomic>
#include <cstdlib>
#include <cstring>

namespace rt {
thread_local int g_last_cuda_error = 0;

namespace {
std::atomic<int> g_pdl{-1};  // -1: not decided yet (environment), 0 off, 1 on
}

bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = std::getenv("RETREE_B200_PDL");
    v = (e == nullptr || std::strcmp(e, "0") != 0) ? 1 : 0;
    int expected = -1;
    g_pdl.compare_exchange_strong(expected, v);
    v = g_pdl.load(std::memory_order_relaxed);
  }
  return v != 0;
}
}  // namespace rt

extern "C" void rt_set_pdl(int enabled) { rt::g_pdl.store(enabled ? 1 : 0); }

extern "C" int rt_pdl_enabled(void) { return rt::pdl_enabled() ? 1 : 0; }

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
