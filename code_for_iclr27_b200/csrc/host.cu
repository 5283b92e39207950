// Host-side parts of liblrk: error plumbing, device queries, dtype sizes and
// host-memory registration for the recall transport's DMA slots.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace lrk {

namespace {
thread_local char g_error[512] = "";
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

void set_error(const char *format, ...) {
  va_list args;
  va_start(args, format);
  vsnprintf(g_error, sizeof(g_error), format, args);
  va_end(args);
}

void clear_error() { g_error[0] = '\0'; }

int sm_count() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return 148;
  if (g_sm_count[device] == 0) {
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || count <= 0)
      count = 148;
    g_sm_count[device] = count;
  }
  return g_sm_count[device];
}

}  // namespace lrk

extern "C" const char *lrk_last_error(void) { return lrk::g_error; }

extern "C" int lrk_version(void) { return 100; }

extern "C" int lrk_dtype_size(int dtype) {
  switch (dtype) {
    case LRK_F32: return 4;
    case LRK_F64: return 8;
    case LRK_F16: return 2;
    case LRK_BF16: return 2;
    default: return 0;
  }
}

extern "C" int lrk_register_host(void *address, size_t bytes) {
  lrk::clear_error();
  cudaError_t status = cudaHostRegister(address, bytes, cudaHostRegisterDefault);
  if (status != cudaSuccess) {
    cudaGetLastError();
    lrk::set_error("cudaHostRegister failed: %s", cudaGetErrorString(status));
    return LRK_ERR_CUDA;
  }
  return LRK_OK;
}

extern "C" int lrk_unregister_host(void *address) {
  lrk::clear_error();
  cudaError_t status = cudaHostUnregister(address);
  if (status != cudaSuccess) {
    cudaGetLastError();
    lrk::set_error("cudaHostUnregister failed: %s", cudaGetErrorString(status));
    return LRK_ERR_CUDA;
  }
  return LRK_OK;
}

extern "C" int lrk_host_device_pointer(void *host, void **device) {
  lrk::clear_error();
  if (host == nullptr || device == nullptr) return lrk::fail(LRK_ERR_INVALID, "null pointer");
  cudaError_t status = cudaHostGetDevicePointer(device, host, 0);
  if (status != cudaSuccess) {
    cudaGetLastError();
    *device = nullptr;
    lrk::set_error("cudaHostGetDevicePointer: %s (register the memory with lrk_register_host first)",
                   cudaGetErrorString(status));
    return LRK_ERR_INVALID;
  }
  return LRK_OK;
}
