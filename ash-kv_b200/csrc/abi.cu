// Library-level entry points: version, status text, last CUDA error.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace ashkv {

static thread_local char g_last_error[256] = "";

void set_error(const char* what, cudaError_t err) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", what, cudaGetErrorString(err), int(err));
}

void set_message(const char* text) { std::snprintf(g_last_error, sizeof(g_last_error), "%s", text); }

ashkv_status_t check_launch(const char* what) {
  const cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) return ASHKV_OK;
  set_error(what, err);
  return ASHKV_LAUNCH_ERROR;
}

void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = ptr;
    else
      cudaGetLastError();
  });
  return fn;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

}  // namespace ashkv

extern "C" int32_t ashkv_version(void) { return 100; }

extern "C" const char* ashkv_status_string(ashkv_status_t status) {
  switch (status) {
    case ASHKV_OK: return "ok";
    case ASHKV_BAD_ARGUMENT: return "bad argument";
    case ASHKV_OUTLIER_OVERFLOW: return "outlier capacity overflow";
    case ASHKV_LAUNCH_ERROR: return "CUDA launch error";
    case ASHKV_TIMEOUT: return "timeout";
    default: return "unknown status";
  }
}

extern "C" const char* ashkv_last_error(void) { return ashkv::g_last_error; }

extern "C" int32_t ashkv_device_sm_count(void) { return ashkv::sm_count(); }
