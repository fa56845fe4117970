// Status strings and the per-thread error detail behind oq_last_error().
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
std::atomic<int> g_wait_polls{oq::kDefaultWaitPolls};
}

namespace oq {

int fail(int status, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return status;
}

int ok() {
  g_last_error[0] = '\0';
  return OQ_OK;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return fail(OQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return ok();
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

int wait_polls() { return g_wait_polls.load(std::memory_order_relaxed); }

}  // namespace oq

extern "C" int oq_debug_set_wait_polls(int polls) {
  return g_wait_polls.exchange(polls < 0 ? oq::kDefaultWaitPolls : polls);
}

extern "C" const char* oq_status_string(int status) {
  switch (status) {
    case OQ_OK: return "ok";
    case OQ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case OQ_ERR_UNSUPPORTED: return "unsupported shape, dtype or configuration";
    case OQ_ERR_MISALIGNED: return "misaligned pointer or stride";
    case OQ_ERR_WORKSPACE: return "workspace missing or too small";
    case OQ_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

extern "C" const char* oq_last_error(void) { return g_last_error; }

extern "C" int oq_abi_version(void) { return 3; }
