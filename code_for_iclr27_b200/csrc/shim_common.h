// Helpers shared by the torch extension modules that front liblrk.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "lrk.h"

namespace lrk_shim {

inline void check_status(int status) { TORCH_CHECK(status == LRK_OK, "liblrk: ", lrk_last_error()); }

inline lrk_stream_t current_stream() {
  return reinterpret_cast<lrk_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

// Element types the reference dispatches with AT_DISPATCH_FLOATING_TYPES_AND2(Half, BFloat16).
inline int dtype_code(at::ScalarType type) {
  switch (type) {
    case at::kFloat: return LRK_F32;
    case at::kDouble: return LRK_F64;
    case at::kHalf: return LRK_F16;
    case at::kBFloat16: return LRK_BF16;
    default: TORCH_CHECK(false, "Unsupported dtype ", type); return -1;
  }
}

}  // namespace lrk_shim
