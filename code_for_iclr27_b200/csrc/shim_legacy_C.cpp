// lazy_recall._legacy_C, backed by liblrk.  Same three operators, signatures
// and checks as the reference module (csrc/cache_legacy.cu:145-308).
#include <vector>

#include "shim_common.h"

using lrk_shim::check_status;
using lrk_shim::current_stream;
using lrk_shim::dtype_code;

namespace {

void check_flat_matrix(const torch::Tensor &tensor, const char *name) {
  TORCH_CHECK(tensor.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(tensor.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(tensor.dim() == 2, name, " must be rank two");
}

// csrc/cache_legacy.cu:145-197
torch::Tensor append_flattened_cache(const torch::Tensor &cache, const torch::Tensor &states,
                                     const torch::Tensor &head_lens, const torch::Tensor &cu_head_lens) {
  check_flat_matrix(cache, "cache");
  TORCH_CHECK(states.is_cuda() && states.is_contiguous(), "states must be contiguous CUDA");
  TORCH_CHECK(states.dim() == 4, "states must have shape [B,H,N,D]");
  TORCH_CHECK(cache.scalar_type() == states.scalar_type(), "cache and states must share dtype");
  TORCH_CHECK(head_lens.scalar_type() == torch::kInt32, "head_lens must be int32");
  TORCH_CHECK(cu_head_lens.scalar_type() == torch::kInt32, "cu_head_lens must be int32");
  TORCH_CHECK(head_lens.is_cuda() && cu_head_lens.is_cuda(), "length metadata must be CUDA");
  TORCH_CHECK(head_lens.is_contiguous() && cu_head_lens.is_contiguous(), "length metadata must be contiguous");
  TORCH_CHECK(cache.device() == states.device() && cache.device() == head_lens.device() &&
                  cache.device() == cu_head_lens.device(),
              "append inputs must share one CUDA device");
  TORCH_CHECK(cache.size(1) == states.size(3), "head_dim mismatch");
  c10::cuda::CUDAGuard guard(cache.device());
  const int64_t total_heads = states.size(0) * states.size(1);
  const int64_t new_length = states.size(2);
  const int64_t head_dim = cache.size(1);
  TORCH_CHECK(head_lens.numel() == total_heads, "head count mismatch");
  TORCH_CHECK(cu_head_lens.numel() == total_heads + 1, "cumulative length count mismatch");
  const int64_t out_rows = cache.size(0) + total_heads * new_length;
  auto output = torch::empty({out_rows, head_dim}, cache.options());
  check_status(lrk_append_flattened(cache.data_ptr(), cache.size(0), states.data_ptr(), total_heads, new_length,
                                    head_dim, dtype_code(cache.scalar_type()), head_lens.data_ptr<int32_t>(),
                                    cu_head_lens.data_ptr<int32_t>(), output.data_ptr(), out_rows, current_stream()));
  return output;
}

// csrc/cache_legacy.cu:199-242
std::vector<torch::Tensor> compact_flattened_kv(const torch::Tensor &keys, const torch::Tensor &values,
                                                const torch::Tensor &keep_indices) {
  check_flat_matrix(keys, "keys");
  check_flat_matrix(values, "values");
  TORCH_CHECK(keys.sizes() == values.sizes(), "K/V shape mismatch");
  TORCH_CHECK(keys.scalar_type() == values.scalar_type(), "K/V dtype mismatch");
  TORCH_CHECK(keep_indices.is_cuda() && keep_indices.is_contiguous(), "keep_indices must be contiguous CUDA");
  TORCH_CHECK(keep_indices.scalar_type() == torch::kInt64, "keep_indices must be int64");
  TORCH_CHECK(keep_indices.dim() == 1, "keep_indices must be rank one");
  TORCH_CHECK(keys.device() == values.device() && keys.device() == keep_indices.device(),
              "compaction inputs must share one CUDA device");
  c10::cuda::CUDAGuard guard(keys.device());
  const int64_t rows = keep_indices.numel();
  const int64_t head_dim = keys.size(1);
  auto output_keys = torch::empty({rows, head_dim}, keys.options());
  auto output_values = torch::empty({rows, head_dim}, values.options());
  if (rows == 0) return {output_keys, output_values};
  check_status(lrk_compact_flattened(keys.data_ptr(), values.data_ptr(), keys.size(0), head_dim,
                                     dtype_code(keys.scalar_type()), keep_indices.data_ptr<int64_t>(), rows,
                                     output_keys.data_ptr(), output_values.data_ptr(), current_stream()));
  return {output_keys, output_values};
}

// csrc/cache_legacy.cu:244-302
torch::Tensor decision_risk_scores(const torch::Tensor &probabilities, const torch::Tensor &values,
                                   const torch::Tensor &head_outputs, const torch::Tensor &gradients,
                                   double base_margin, double denominator_epsilon) {
  check_flat_matrix(probabilities, "probabilities");
  check_flat_matrix(values, "values");
  check_flat_matrix(head_outputs, "head_outputs");
  check_flat_matrix(gradients, "gradients");
  TORCH_CHECK(probabilities.scalar_type() == torch::kFloat32, "probabilities must be float32");
  TORCH_CHECK(head_outputs.scalar_type() == torch::kFloat32, "head_outputs must be float32");
  TORCH_CHECK(gradients.scalar_type() == torch::kFloat32, "gradients must be float32");
  TORCH_CHECK(probabilities.size(0) == head_outputs.size(0), "mapped-query-head mismatch");
  TORCH_CHECK(head_outputs.sizes() == gradients.sizes(), "head output/gradient mismatch");
  TORCH_CHECK(probabilities.size(1) == values.size(0), "candidate count mismatch");
  TORCH_CHECK(values.size(1) == head_outputs.size(1), "head_dim mismatch");
  TORCH_CHECK(probabilities.device() == values.device() && probabilities.device() == head_outputs.device() &&
                  probabilities.device() == gradients.device(),
              "score inputs must share one CUDA device");
  TORCH_CHECK(denominator_epsilon > 0.0 && denominator_epsilon < 1.0, "denominator_epsilon must be in (0,1)");
  c10::cuda::CUDAGuard guard(values.device());
  const int64_t groups = probabilities.size(0);
  const int64_t candidates = probabilities.size(1);
  const int64_t head_dim = values.size(1);
  auto scores = torch::empty({candidates}, probabilities.options());
  if (candidates == 0) return scores;
  check_status(lrk_decision_risk(probabilities.data_ptr<float>(), values.data_ptr(),
                                 dtype_code(values.scalar_type()), head_outputs.data_ptr<float>(),
                                 gradients.data_ptr<float>(), groups, candidates, head_dim, base_margin,
                                 static_cast<float>(denominator_epsilon), scores.data_ptr<float>(),
                                 current_stream()));
  return scores;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("append_flattened_cache", &append_flattened_cache);
  module.def("compact_flattened_kv", &compact_flattened_kv);
  module.def("decision_risk_scores", &decision_risk_scores);
}
