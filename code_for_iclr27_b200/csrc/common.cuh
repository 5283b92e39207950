// Shared helpers of liblrk: status/error plumbing, launch sizing, vector types.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "lrk.h"

namespace lrk {

// Thread-local message behind lrk_last_error().
void set_error(const char *format, ...);
void clear_error();

inline int fail(int code, const char *message) {
  set_error("%s", message);
  return code;
}

// Check the launch just issued (asynchronous faults surface at the next sync).
inline int launch_status(const char *what) {
  cudaError_t error = cudaGetLastError();
  if (error != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(error));
    return LRK_ERR_CUDA;
  }
  return LRK_OK;
}

#define LRK_REQUIRE(condition, message) \
  do {                                  \
    if (!(condition)) return ::lrk::fail(LRK_ERR_INVALID, message); \
  } while (0)

// Number of SMs of the current device, cached per device.
int sm_count();

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__host__ __device__ __forceinline__ int64_t lmin(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t lmax(int64_t a, int64_t b) { return a > b ? a : b; }

inline bool aligned(const void *pointer, int64_t bytes) {
  return (reinterpret_cast<uintptr_t>(pointer) % static_cast<uintptr_t>(bytes)) == 0;
}

// Fixed-width bit containers for row copies.
template <int Bytes> struct Bits;
template <> struct Bits<16> { using type = uint4; };
template <> struct Bits<8> { using type = uint2; };
template <> struct Bits<4> { using type = uint32_t; };
template <> struct Bits<2> { using type = uint16_t; };

}  // namespace lrk
