// lazy_recall._C, backed by liblrk.
//
// The eight operators keep the reference's positional signatures
// (csrc/bindings.cpp:20-29), its argument checks and messages (TORCH_CHECK ->
// RuntimeError), its output allocation (torch::empty on the input's device,
// through the caching allocator) and its stream (the current CUDA stream).
// Added operators: refine and topk_smallest (selection); temporal_scores,
// scores_from_keys, project_values, logits and logits_heads (scoring); compact_layers and
// merge_layers (eviction and recall over several layers in one call);
// select_histogram and select_pick (layer-group selection across GPUs);
// arena_append and arena_compact (the gapped per-head KV arena).
#include <vector>

#include "shim_common.h"

using lrk_shim::check_status;
using lrk_shim::current_stream;
using lrk_shim::dtype_code;

namespace {

void check_cuda(const torch::Tensor &tensor, const torch::Tensor &reference) {
  TORCH_CHECK(tensor.is_cuda() && tensor.is_contiguous(), "Expected contiguous CUDA tensor");
  TORCH_CHECK(tensor.device() == reference.device(), "CUDA devices differ");
}

void check_recall_tensor(const torch::Tensor &tensor, const torch::Tensor &reference) {
  TORCH_CHECK(tensor.is_cuda() && tensor.is_contiguous(), "Expected contiguous CUDA tensor");
  TORCH_CHECK(tensor.device() == reference.device(), "Recall devices differ");
}

void check_cache(const torch::Tensor &keys, const torch::Tensor &values, const torch::Tensor &positions) {
  for (const auto &tensor : {keys, values, positions}) check_cuda(tensor, keys);
  TORCH_CHECK(keys.dim() == 2 && keys.size(1) > 0 && keys.sizes() == values.sizes() &&
                  keys.scalar_type() == values.scalar_type(),
              "Invalid KV layout");
  TORCH_CHECK(positions.scalar_type() == at::kFloat && positions.numel() == keys.size(0), "Invalid positions");
}

// csrc/scoring.cu:205-233
std::vector<torch::Tensor> temporal_probabilities(torch::Tensor logits, torch::Tensor projected_values,
                                                  torch::Tensor query_positions, torch::Tensor key_positions,
                                                  double scale) {
  check_cuda(logits, logits);
  check_cuda(projected_values, logits);
  check_cuda(query_positions, logits);
  check_cuda(key_positions, logits);
  TORCH_CHECK(logits.dim() == 3, "logits must be [window, groups, positions]");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kHalf ||
                  logits.scalar_type() == at::kBFloat16,
              "Only FP32/FP16/BF16 scores are supported");
  const int64_t window = logits.size(0), groups = logits.size(1), length = logits.size(2);
  TORCH_CHECK(window > 0 && groups > 0 && length > 0, "Empty attention dimensions");
  TORCH_CHECK(projected_values.scalar_type() == at::kFloat && projected_values.dim() == 2 &&
                  projected_values.size(0) == groups && projected_values.size(1) == length,
              "Invalid projected values");
  TORCH_CHECK(query_positions.scalar_type() == at::kLong && query_positions.numel() == window,
              "Invalid query positions");
  TORCH_CHECK(key_positions.scalar_type() == at::kFloat && key_positions.numel() == length, "Invalid key positions");
  c10::cuda::CUDAGuard guard(logits.device());
  auto probabilities = torch::empty(logits.sizes(), logits.options().dtype(at::kFloat));
  auto output = torch::empty({window, groups}, probabilities.options());
  check_status(lrk_temporal_probabilities(logits.data_ptr(), dtype_code(logits.scalar_type()),
                                          projected_values.data_ptr<float>(), query_positions.data_ptr<int64_t>(),
                                          key_positions.data_ptr<float>(), probabilities.data_ptr<float>(),
                                          output.data_ptr<float>(), window, groups, length,
                                          static_cast<float>(scale), current_stream()));
  return {probabilities, output};
}

// csrc/scoring.cu:235-255
torch::Tensor temporal_risk(torch::Tensor probabilities, torch::Tensor output_projection,
                            torch::Tensor projected_values, torch::Tensor margin, int64_t first, int64_t last,
                            double epsilon) {
  for (const auto &tensor : {probabilities, output_projection, projected_values, margin}) {
    check_cuda(tensor, probabilities);
    TORCH_CHECK(tensor.scalar_type() == at::kFloat, "Risk inputs must be float32");
  }
  TORCH_CHECK(probabilities.dim() == 3, "Invalid probability dimensions");
  const int64_t window = probabilities.size(0), groups = probabilities.size(1), length = probabilities.size(2);
  TORCH_CHECK(window > 0 && groups > 0 && first >= 0 && last > first && last <= length && epsilon > 0,
              "Invalid risk interval");
  TORCH_CHECK(margin.numel() == 1 && output_projection.numel() == window * groups &&
                  projected_values.numel() == groups * length,
              "Risk shapes differ");
  c10::cuda::CUDAGuard guard(probabilities.device());
  auto result = torch::empty({last - first}, probabilities.options());
  check_status(lrk_temporal_risk(probabilities.data_ptr<float>(), output_projection.data_ptr<float>(),
                                 projected_values.data_ptr<float>(), margin.data_ptr<float>(),
                                 result.data_ptr<float>(), window, groups, length, first, last,
                                 static_cast<float>(epsilon), current_stream()));
  return result;
}

// csrc/scoring.cu:264-292
std::vector<torch::Tensor> append(torch::Tensor keys, torch::Tensor values, torch::Tensor positions,
                                  torch::Tensor new_keys, torch::Tensor new_values, torch::Tensor cumulative,
                                  int64_t logical_start, int64_t maximum_length) {
  check_cache(keys, values, positions);
  for (const auto &tensor : {new_keys, new_values, cumulative}) check_cuda(tensor, keys);
  TORCH_CHECK(new_keys.dim() == 4 && new_keys.size(0) == 1 && new_keys.sizes() == new_values.sizes() &&
                  new_keys.scalar_type() == keys.scalar_type() && new_values.scalar_type() == keys.scalar_type(),
              "Invalid appended KV");
  const int64_t heads = new_keys.size(1), added = new_keys.size(2), dimension = keys.size(1);
  TORCH_CHECK(heads > 0 && added > 0 && new_keys.size(3) == dimension && maximum_length >= 0,
              "Invalid appended shape");
  TORCH_CHECK(cumulative.scalar_type() == at::kInt && cumulative.numel() == heads + 1, "Invalid cumulative lengths");
  c10::cuda::CUDAGuard guard(keys.device());
  const int64_t rows = keys.size(0) + heads * added;
  auto output_keys = torch::empty({rows, dimension}, keys.options());
  auto output_values = torch::empty_like(output_keys);
  auto output_positions = torch::empty({rows, 1}, positions.options());
  auto output_cumulative = torch::empty_like(cumulative);
  auto output_lengths = torch::empty({heads}, cumulative.options());
  check_status(lrk_append(keys.data_ptr(), values.data_ptr(), positions.data_ptr<float>(), keys.size(0),
                          new_keys.data_ptr(), new_values.data_ptr(), cumulative.data_ptr<int32_t>(), heads, added,
                          dimension, dtype_code(keys.scalar_type()), logical_start, output_keys.data_ptr(),
                          output_values.data_ptr(), output_positions.data_ptr<float>(),
                          output_cumulative.data_ptr<int32_t>(), output_lengths.data_ptr<int32_t>(),
                          current_stream()));
  return {output_keys, output_values, output_positions, output_cumulative, output_lengths};
}

// csrc/scoring.cu:294-314
std::vector<torch::Tensor> compact(torch::Tensor keys, torch::Tensor values, torch::Tensor positions,
                                   torch::Tensor removed) {
  check_cache(keys, values, positions);
  check_cuda(removed, keys);
  TORCH_CHECK(removed.scalar_type() == at::kLong && removed.dim() == 1 && removed.numel() <= keys.size(0),
              "Invalid removals");
  c10::cuda::CUDAGuard guard(keys.device());
  const int64_t rows = keys.size(0) - removed.numel(), dimension = keys.size(1);
  auto output_keys = torch::empty({rows, dimension}, keys.options());
  auto output_values = torch::empty_like(output_keys);
  auto output_positions = torch::empty({rows, 1}, positions.options());
  if (rows > 0) {
    check_status(lrk_compact(keys.data_ptr(), values.data_ptr(), positions.data_ptr<float>(), keys.size(0),
                             dimension, dtype_code(keys.scalar_type()), removed.data_ptr<int64_t>(), removed.numel(),
                             output_keys.data_ptr(), output_values.data_ptr(), output_positions.data_ptr<float>(),
                             current_stream()));
  }
  return {output_keys, output_values, output_positions};
}

// compact() over several layers in one call: layer i drops the sorted rows
// removed[offsets[i] : offsets[i + 1]].  The per-layer checks, allocations
// and launches run here instead of once per layer from Python.
std::vector<std::vector<torch::Tensor>> compact_layers(std::vector<torch::Tensor> keys,
                                                       std::vector<torch::Tensor> values,
                                                       std::vector<torch::Tensor> positions, torch::Tensor removed,
                                                       std::vector<int64_t> offsets) {
  const size_t n = keys.size();
  TORCH_CHECK(values.size() == n && positions.size() == n && offsets.size() == n + 1,
              "compact_layers: one keys/values/positions tensor per layer and layers + 1 offsets");
  TORCH_CHECK(removed.scalar_type() == at::kLong && removed.dim() == 1 && removed.is_contiguous(), "Invalid removals");
  TORCH_CHECK(offsets[0] == 0 && offsets[n] == removed.numel(), "compact_layers: offsets must span the removals");
  std::vector<std::vector<torch::Tensor>> out(3);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(offsets[i + 1] >= offsets[i], "compact_layers: offsets must not decrease");
    auto layer = compact(keys[i], values[i], positions[i], removed.narrow(0, offsets[i], offsets[i + 1] - offsets[i]));
    for (int k = 0; k < 3; ++k) out[k].push_back(layer[k]);
  }
  return out;
}

// csrc/scoring.cu:316-329
torch::Tensor pool(torch::Tensor scores, torch::Tensor bounds, int64_t maximum_count, int64_t width) {
  check_cuda(scores, scores);
  check_cuda(bounds, scores);
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.dim() == 1 && bounds.scalar_type() == at::kLong &&
                  bounds.dim() == 1 && bounds.numel() >= 2,
              "Invalid pool layout");
  TORCH_CHECK(width > 0 && width % 2 == 1 && maximum_count > 0, "Invalid pool configuration");
  c10::cuda::CUDAGuard guard(scores.device());
  auto output = torch::empty_like(scores);
  check_status(lrk_pool(scores.data_ptr<float>(), scores.numel(), bounds.data_ptr<int64_t>(), bounds.numel() - 1,
                        maximum_count, width, output.data_ptr<float>(), current_stream()));
  return output;
}

// csrc/recall.cu:54-84
std::vector<torch::Tensor> merge(torch::Tensor keys, torch::Tensor values, torch::Tensor positions,
                                 torch::Tensor recalled, torch::Tensor recalled_positions, torch::Tensor mapping) {
  for (const auto &tensor : {keys, values, positions, recalled, recalled_positions, mapping})
    check_recall_tensor(tensor, keys);
  TORCH_CHECK(keys.dim() == 2 && keys.size(1) > 0 && keys.sizes() == values.sizes(), "Invalid K/V shape");
  TORCH_CHECK(recalled.dim() == 3 && recalled.size(1) == 2 && recalled.size(2) == keys.size(1),
              "Invalid recalled shape");
  TORCH_CHECK(keys.scalar_type() == values.scalar_type() && keys.scalar_type() == recalled.scalar_type(),
              "K/V dtypes differ");
  TORCH_CHECK(positions.scalar_type() == at::kFloat && recalled_positions.scalar_type() == at::kFloat &&
                  positions.numel() == keys.size(0) && recalled_positions.numel() == recalled.size(0),
              "Invalid positions");
  TORCH_CHECK(mapping.dim() == 1 && mapping.scalar_type() == at::kLong, "Mapping must be int64");
  c10::cuda::CUDAGuard guard(keys.device());
  const auto rows = mapping.numel();
  const auto dimension = keys.size(1);
  auto output_keys = torch::empty({rows, dimension}, keys.options());
  auto output_values = torch::empty_like(output_keys);
  auto output_positions = torch::empty({rows, 1}, positions.options());
  if (rows) {
    check_status(lrk_merge(keys.data_ptr(), values.data_ptr(), positions.data_ptr<float>(), keys.size(0),
                           recalled.data_ptr(), recalled_positions.data_ptr<float>(), recalled.size(0),
                           mapping.data_ptr<int64_t>(), rows, dimension, dtype_code(keys.scalar_type()),
                           output_keys.data_ptr(), output_values.data_ptr(), output_positions.data_ptr<float>(),
                           current_stream()));
  }
  return {output_keys, output_values, output_positions};
}

// merge() of several layers in one launch (lrk_merge_layers): the same
// checks per layer; the outputs are views into one allocation per tensor kind.
std::vector<std::vector<torch::Tensor>> merge_layers(std::vector<torch::Tensor> keys, std::vector<torch::Tensor> values,
                                                     std::vector<torch::Tensor> positions,
                                                     std::vector<torch::Tensor> recalled,
                                                     std::vector<torch::Tensor> recalled_positions,
                                                     std::vector<torch::Tensor> mappings) {
  const size_t n = keys.size();
  TORCH_CHECK(n > 0 && values.size() == n && positions.size() == n && recalled.size() == n &&
                  recalled_positions.size() == n && mappings.size() == n,
              "merge_layers: one tensor of each kind per layer");
  const auto dimension = keys[0].size(1);
  std::vector<lrk_merge_layer> table(n);
  int64_t total = 0;
  for (size_t i = 0; i < n; ++i) {
    for (const auto &tensor : {keys[i], values[i], positions[i], recalled[i], recalled_positions[i], mappings[i]})
      check_recall_tensor(tensor, keys[0]);
    TORCH_CHECK(keys[i].dim() == 2 && keys[i].size(1) == dimension && keys[i].sizes() == values[i].sizes(),
                "Invalid K/V shape");
    TORCH_CHECK(recalled[i].dim() == 3 && recalled[i].size(1) == 2 && recalled[i].size(2) == dimension,
                "Invalid recalled shape");
    TORCH_CHECK(keys[i].scalar_type() == keys[0].scalar_type() && values[i].scalar_type() == keys[0].scalar_type() &&
                    recalled[i].scalar_type() == keys[0].scalar_type(),
                "K/V dtypes differ");
    TORCH_CHECK(positions[i].scalar_type() == at::kFloat && recalled_positions[i].scalar_type() == at::kFloat &&
                    positions[i].numel() == keys[i].size(0) && recalled_positions[i].numel() == recalled[i].size(0),
                "Invalid positions");
    TORCH_CHECK(mappings[i].dim() == 1 && mappings[i].scalar_type() == at::kLong, "Mapping must be int64");
    table[i] = {keys[i].data_ptr(), values[i].data_ptr(), positions[i].data_ptr<float>(), keys[i].size(0),
                recalled[i].data_ptr(), recalled_positions[i].data_ptr<float>(), recalled[i].size(0),
                mappings[i].data_ptr<int64_t>(), mappings[i].numel()};
    total += mappings[i].numel();
  }
  c10::cuda::CUDAGuard guard(keys[0].device());
  auto all_keys = torch::empty({total, dimension}, keys[0].options());
  auto all_values = torch::empty_like(all_keys);
  auto all_positions = torch::empty({total, 1}, positions[0].options());
  if (total) {
    check_status(lrk_merge_layers(table.data(), static_cast<int64_t>(n), dimension, dtype_code(keys[0].scalar_type()),
                                  all_keys.data_ptr(), all_values.data_ptr(), all_positions.data_ptr<float>(),
                                  current_stream()));
  }
  std::vector<std::vector<torch::Tensor>> out(3);
  int64_t first = 0;
  for (size_t i = 0; i < n; ++i) {
    const int64_t rows = mappings[i].numel();
    out[0].push_back(all_keys.narrow(0, first, rows));
    out[1].push_back(all_values.narrow(0, first, rows));
    out[2].push_back(all_positions.narrow(0, first, rows));
    first += rows;
  }
  return out;
}

// csrc/recall.cu:86-111
void pack(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor indices,
          torch::Tensor heads, int64_t layer, torch::Tensor payload, torch::Tensor metadata) {
  for (const auto &tensor : {keys, values, positions, indices, heads, payload, metadata})
    check_recall_tensor(tensor, keys);
  TORCH_CHECK(keys.dim() == 2 && keys.size(1) > 0 && keys.sizes() == values.sizes(), "Invalid K/V shape");
  TORCH_CHECK(keys.scalar_type() == values.scalar_type() && keys.scalar_type() == payload.scalar_type(),
              "Dtype mismatch");
  TORCH_CHECK(indices.dim() == 1 && indices.scalar_type() == at::kLong && heads.sizes() == indices.sizes() &&
                  heads.scalar_type() == at::kLong,
              "Invalid gather indices");
  const auto rows = indices.numel();
  const auto dimension = keys.size(1);
  TORCH_CHECK(payload.dim() == 3 && payload.size(0) == rows && payload.size(1) == 2 && payload.size(2) == dimension,
              "Invalid payload buffer");
  TORCH_CHECK(positions.numel() == keys.size(0) && positions.scalar_type() == at::kFloat, "Invalid positions");
  TORCH_CHECK(metadata.dim() == 2 && metadata.size(0) == rows && metadata.size(1) == 3 &&
                  metadata.scalar_type() == at::kLong,
              "Invalid identity buffer");
  c10::cuda::CUDAGuard guard(keys.device());
  if (!rows) return;
  check_status(lrk_pack(keys.data_ptr(), values.data_ptr(), positions.data_ptr<float>(), keys.size(0), dimension,
                        dtype_code(keys.scalar_type()), indices.data_ptr<int64_t>(), heads.data_ptr<int64_t>(), rows,
                        layer, payload.data_ptr(), metadata.data_ptr<int64_t>(), current_stream()));
}

// csrc/batch_append.cu:36-94.  The descriptor table stays on the host and
// reaches the kernel as a launch parameter: no pageable copy, no sync.
std::vector<torch::Tensor> batch_append(std::vector<torch::Tensor> keys, std::vector<torch::Tensor> values,
                                        std::vector<torch::Tensor> positions, torch::Tensor new_keys,
                                        torch::Tensor new_values, std::vector<std::vector<int64_t>> lengths,
                                        std::vector<int64_t> logical_positions) {
  TORCH_CHECK(new_keys.is_cuda() && new_keys.is_contiguous() && new_values.is_contiguous(),
              "Contiguous CUDA states required");
  TORCH_CHECK(new_keys.dim() == 4 && new_keys.size(2) == 1 && new_keys.size(3) > 0,
              "Only batched one-token append is supported");
  TORCH_CHECK(new_keys.sizes() == new_values.sizes() && new_keys.scalar_type() == new_values.scalar_type() &&
                  new_keys.device() == new_values.device(),
              "New K/V mismatch");
  const int64_t requests = new_keys.size(0), heads = new_keys.size(1), dimension = new_keys.size(3);
  TORCH_CHECK(requests > 0 && heads > 0 && static_cast<int64_t>(keys.size()) == requests &&
                  static_cast<int64_t>(values.size()) == requests &&
                  static_cast<int64_t>(positions.size()) == requests &&
                  static_cast<int64_t>(lengths.size()) == requests &&
                  static_cast<int64_t>(logical_positions.size()) == requests,
              "Request metadata mismatch");
  c10::cuda::CUDAGuard guard(new_keys.device());
  std::vector<lrk_segment> segments(static_cast<size_t>(requests * heads));
  int64_t destination = 0;
  for (int64_t request = 0; request < requests; ++request) {
    TORCH_CHECK(keys[request].is_cuda() && keys[request].is_contiguous() && values[request].is_contiguous() &&
                    positions[request].is_contiguous(),
                "Contiguous CUDA cache required");
    TORCH_CHECK(keys[request].device() == new_keys.device() && values[request].device() == new_keys.device() &&
                    positions[request].device() == new_keys.device(),
                "Cache devices differ");
    TORCH_CHECK(keys[request].dim() == 2 && keys[request].size(1) == dimension &&
                    keys[request].sizes() == values[request].sizes() &&
                    keys[request].scalar_type() == new_keys.scalar_type() &&
                    values[request].scalar_type() == new_keys.scalar_type(),
                "Cache K/V mismatch");
    TORCH_CHECK(positions[request].scalar_type() == at::kFloat &&
                    positions[request].numel() == keys[request].size(0) &&
                    static_cast<int64_t>(lengths[request].size()) == heads && logical_positions[request] >= 0 &&
                    logical_positions[request] < (1 << 24),
                "Invalid positions or head metadata");
    int64_t source = 0;
    for (int64_t head = 0; head < heads; ++head) {
      const int64_t length = lengths[request][head];
      TORCH_CHECK(length >= 0 && source + length <= keys[request].size(0), "Invalid head length");
      lrk_segment &segment = segments[static_cast<size_t>(request * heads + head)];
      segment.keys = keys[request].data_ptr();
      segment.values = values[request].data_ptr();
      segment.positions = positions[request].data_ptr<float>();
      segment.source_row = source;
      segment.length = length;
      segment.destination_row = destination;
      segment.logical_position = logical_positions[request];
      source += length;
      destination += length + 1;
    }
    TORCH_CHECK(source == keys[request].size(0), "Head lengths do not cover cache rows");
  }
  auto output_keys = torch::empty({destination, dimension}, new_keys.options());
  auto output_values = torch::empty_like(output_keys);
  auto output_positions = torch::empty({destination, 1}, new_keys.options().dtype(torch::kFloat));
  check_status(lrk_batch_append(segments.data(), static_cast<int64_t>(segments.size()), new_keys.data_ptr(),
                                new_values.data_ptr(), dimension, dtype_code(new_keys.scalar_type()),
                                output_keys.data_ptr(), output_values.data_ptr(), output_positions.data_ptr<float>(),
                                destination, current_stream()));
  return {output_keys, output_values, output_positions};
}

// Selection (selection.py:52-88): raw/pooled [n] f32; ends, position_starts
// [segments] i64 on the same device.  Returns (values f32 [count], segment ids
// i64 [count], positions i64 [count], stats i64 [2]) on the device.
std::vector<torch::Tensor> refine(torch::Tensor raw, torch::Tensor pooled, torch::Tensor ends,
                                  torch::Tensor position_starts, int64_t count) {
  for (const auto &tensor : {raw, pooled, ends, position_starts}) check_cuda(tensor, raw);
  TORCH_CHECK(raw.scalar_type() == at::kFloat && pooled.scalar_type() == at::kFloat && raw.dim() == 1 &&
                  pooled.sizes() == raw.sizes(),
              "Refine scores must be matching 1-D float32 tensors");
  TORCH_CHECK(ends.scalar_type() == at::kLong && position_starts.scalar_type() == at::kLong && ends.dim() == 1 &&
                  ends.numel() >= 1 && position_starts.sizes() == ends.sizes(),
              "Invalid segment bounds");
  TORCH_CHECK(count >= 0 && count <= raw.numel(), "Invalid selection count");
  c10::cuda::CUDAGuard guard(raw.device());
  const int64_t n = raw.numel(), segments = ends.numel();
  auto values = torch::empty({count}, raw.options());
  auto segment_ids = torch::empty({count}, ends.options());
  auto positions = torch::empty({count}, ends.options());
  auto stats = torch::empty({2}, ends.options());
  const size_t bytes = lrk_refine_workspace_bytes(n, segments);
  auto workspace = torch::empty({static_cast<int64_t>(bytes)}, raw.options().dtype(at::kByte));
  check_status(lrk_refine(raw.data_ptr<float>(), pooled.data_ptr<float>(), n, ends.data_ptr<int64_t>(),
                          position_starts.data_ptr<int64_t>(), segments, count, workspace.data_ptr(), bytes,
                          values.data_ptr<float>(), segment_ids.data_ptr<int64_t>(), positions.data_ptr<int64_t>(),
                          stats.data_ptr<int64_t>(), current_stream()));
  return {values, segment_ids, positions, stats};
}

// torch.topk(x, k, largest=False, sorted=True) for a 1-D float32 CUDA tensor.
std::vector<torch::Tensor> topk_smallest(torch::Tensor x, int64_t k) {
  check_cuda(x, x);
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.dim() == 1, "topk_smallest expects a 1-D float32 tensor");
  TORCH_CHECK(k >= 0 && k <= x.numel(), "selected index k out of range");
  c10::cuda::CUDAGuard guard(x.device());
  auto values = torch::empty({k}, x.options());
  auto indices = torch::empty({k}, x.options().dtype(at::kLong));
  const size_t bytes = lrk_topk_workspace_bytes(x.numel());
  auto workspace = torch::empty({static_cast<int64_t>(bytes)}, x.options().dtype(at::kByte));
  check_status(lrk_topk_smallest(x.data_ptr<float>(), x.numel(), k, workspace.data_ptr(), bytes,
                                 values.data_ptr<float>(), indices.data_ptr<int64_t>(), current_stream()));
  return {values, indices};
}

// Fused scoring of many (layer, head) segments from bf16/fp16/fp32 logits
// (lrk_temporal_scores).  projected_values[i] may be a strided view (row
// stride >= length, unit column stride).  Returns the concatenated scores of
// all segments, in order -- the layout compute_score_table builds with
// torch.cat (scoring.py:291).
torch::Tensor temporal_scores(std::vector<torch::Tensor> logits, std::vector<torch::Tensor> projected_values,
                              std::vector<torch::Tensor> key_positions, std::vector<int64_t> first,
                              std::vector<int64_t> last, torch::Tensor query_positions, torch::Tensor margin,
                              double scale, double epsilon, std::vector<int64_t> query_chunks, bool probability_stash) {
  const size_t count = logits.size();
  TORCH_CHECK(count > 0 && projected_values.size() == count && key_positions.size() == count &&
                  first.size() == count && last.size() == count &&
                  (query_chunks.empty() || query_chunks.size() == count),
              "Segment lists differ in length");
  check_cuda(query_positions, logits[0]);
  check_cuda(margin, logits[0]);
  TORCH_CHECK(query_positions.scalar_type() == at::kLong && margin.scalar_type() == at::kFloat &&
                  margin.numel() == 1,
              "Invalid query positions or margin");
  const auto dtype = logits[0].scalar_type();
  TORCH_CHECK(dtype == at::kFloat || dtype == at::kHalf || dtype == at::kBFloat16,
              "Only FP32/FP16/BF16 scores are supported");
  const int64_t window = logits[0].size(0), groups = logits[0].size(1);
  TORCH_CHECK(query_positions.numel() == window, "Invalid query positions");
  c10::cuda::CUDAGuard guard(logits[0].device());
  int64_t total = 0;
  for (size_t i = 0; i < count; ++i) total += last[i] - first[i];
  auto scores = torch::empty({total}, margin.options());
  std::vector<lrk_score_segment> segments(count);
  int64_t offset = 0;
  for (size_t i = 0; i < count; ++i) {
    const auto &lg = logits[i];
    TORCH_CHECK(lg.is_cuda() && lg.device() == logits[0].device(), "Expected CUDA logits on one device");
    TORCH_CHECK(lg.dim() == 3 && lg.size(0) == window && lg.size(1) == groups && lg.scalar_type() == dtype,
                "logits must be [window, groups, positions] of one dtype");
    const int64_t length = lg.size(2);
    // Rows may be padded: [window, groups, length] with a row stride >= length.
    TORCH_CHECK(lg.stride(2) == 1 && lg.stride(1) >= length && lg.stride(0) == groups * lg.stride(1),
                "logits rows must be unit-stride with a common row stride");
    const auto &pv = projected_values[i];
    TORCH_CHECK(pv.is_cuda() && pv.device() == logits[0].device() && pv.scalar_type() == at::kFloat &&
                    pv.dim() == 2 && pv.size(0) == groups && pv.size(1) == length && pv.stride(1) == 1,
                "Invalid projected values");
    check_cuda(key_positions[i], logits[0]);
    TORCH_CHECK(key_positions[i].scalar_type() == at::kFloat && key_positions[i].numel() == length,
                "Invalid key positions");
    lrk_score_segment &s = segments[i];
    s.logits = logits[i].data_ptr();
    s.projected_values = pv.data_ptr<float>();
    s.projected_stride = groups > 1 ? pv.stride(0) : length;
    s.key_positions = key_positions[i].data_ptr<float>();
    s.length = length;
    s.first = first[i];
    s.last = last[i];
    s.scores = scores.data_ptr<float>() + offset;
    s.logits_stride = lg.stride(1);
    s.query_chunk = query_chunks.empty() ? 0 : query_chunks[i];
    offset += last[i] - first[i];
  }
  // With the probability stash the statistics pass stores each candidate's
  // probability and the risk reads it (bit-identical to recomputing it).
  const size_t bytes = lrk_temporal_scores_workspace_bytes(static_cast<int64_t>(count), window, groups) +
                       (probability_stash ? lrk_temporal_scores_stash_bytes(segments.data(), static_cast<int64_t>(count),
                                                                      window, groups)
                                    : 0);
  auto workspace = torch::empty({static_cast<int64_t>(bytes)}, margin.options().dtype(at::kByte));
  check_status(lrk_temporal_scores(segments.data(), static_cast<int64_t>(count), dtype_code(dtype),
                                   query_positions.data_ptr<int64_t>(), window, groups, static_cast<float>(scale),
                                   margin.data_ptr<float>(), static_cast<float>(epsilon), workspace.data_ptr(), bytes,
                                   current_stream()));
  return scores;
}

// Per-layer projected values [groups, rows] (lrk_project_values): each row of
// the packed layer against its own head's margin gradients.
torch::Tensor project_values(torch::Tensor values, torch::Tensor gradients, torch::Tensor cumulative, int64_t groups) {
  check_cuda(values, values);
  check_cuda(gradients, values);
  check_cuda(cumulative, values);
  TORCH_CHECK(values.dim() == 2 && gradients.dim() == 2 && gradients.size(1) == values.size(1) &&
                  gradients.scalar_type() == at::kFloat && cumulative.scalar_type() == at::kInt && groups > 0 &&
                  gradients.size(0) == (cumulative.numel() - 1) * groups && values.is_contiguous() &&
                  gradients.is_contiguous() && cumulative.is_contiguous(),
              "Invalid projection inputs");
  c10::cuda::CUDAGuard guard(values.device());
  auto out = torch::empty({groups, values.size(0)}, gradients.options());
  check_status(lrk_project_values(values.data_ptr(), dtype_code(values.scalar_type()), values.size(0), values.size(1),
                                  gradients.data_ptr<float>(), cumulative.data_ptr<int32_t>(), cumulative.numel() - 1,
                                  groups, out.data_ptr<float>(), current_stream()));
  return out;
}

// Logits [rows, out_stride] bf16 (the first `count` columns are the keys')
// in torch.matmul's accumulation order for k_step-term steps (lrk_logits).
torch::Tensor logits(torch::Tensor queries, torch::Tensor keys, int64_t k_step, int64_t out_stride) {
  check_cuda(queries, queries);
  check_cuda(keys, queries);
  TORCH_CHECK(queries.dim() == 2 && keys.dim() == 2 && queries.size(1) == keys.size(1) &&
                  queries.scalar_type() == at::kBFloat16 && keys.scalar_type() == at::kBFloat16 &&
                  queries.is_contiguous() && keys.is_contiguous(),
              "logits takes contiguous bf16 [rows, D] queries and [count, D] keys");
  c10::cuda::CUDAGuard guard(queries.device());
  auto out = torch::empty({queries.size(0), out_stride}, queries.options());
  check_status(lrk_logits(queries.data_ptr(), queries.size(0), keys.data_ptr(), keys.size(0), keys.size(1), k_step,
                          out.data_ptr(), out_stride, current_stream()));
  return out;
}

// Logits of several heads of one layer in one launch (lrk_logits_heads):
// entry i multiplies queries[heads[i]] ([H, rows, D] bf16) by the key rows
// starts[i] .. ends[i] of keys ([N, D] bf16) in k_steps[i]-term steps.  One
// allocation holds every entry's [rows, stride_i] output; the views are
// returned in entry order.  stride_i is the key count rounded up to 128
// elements: rows on 256-byte boundaries make every 128-byte TMA row segment
// one whole L2 line (measured on B200: 138 instead of 143-146 us per
// configs[1] layer with a stride rounded to 8).
std::vector<torch::Tensor> logits_heads(torch::Tensor queries, torch::Tensor keys, std::vector<int64_t> heads,
                                        std::vector<int64_t> starts, std::vector<int64_t> ends,
                                        std::vector<int64_t> k_steps, int64_t groups) {
  check_cuda(queries, queries);
  check_cuda(keys, queries);
  TORCH_CHECK(queries.dim() == 3 && keys.dim() == 2 && queries.size(2) == keys.size(1) &&
                  queries.scalar_type() == at::kBFloat16 && keys.scalar_type() == at::kBFloat16 &&
                  queries.is_contiguous() && keys.is_contiguous(),
              "logits_heads takes contiguous bf16 [H, rows, D] queries and [N, D] keys");
  const size_t n = heads.size();
  TORCH_CHECK(starts.size() == n && ends.size() == n && k_steps.size() == n,
              "heads, starts, ends and k_steps must have one entry per head");
  const int64_t rows = queries.size(1), dim = queries.size(2);
  TORCH_CHECK(groups >= 0 && (groups == 0 || rows % groups == 0), "groups must divide the query rows");
  std::vector<int64_t> offsets(n + 1, 0);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(heads[i] >= 0 && heads[i] < queries.size(0), "head index out of range");
    TORCH_CHECK(0 <= starts[i] && starts[i] <= ends[i] && ends[i] <= keys.size(0), "key range out of bounds");
    offsets[i + 1] = offsets[i] + rows * ((ends[i] - starts[i] + 127) / 128 * 128);
  }
  c10::cuda::CUDAGuard guard(queries.device());
  auto flat = torch::empty({offsets[n]}, queries.options());
  std::vector<lrk_logits_head> table(n);
  std::vector<torch::Tensor> out;
  out.reserve(n);
  const auto element = keys.element_size();
  for (size_t i = 0; i < n; ++i) {
    const int64_t count = ends[i] - starts[i], stride = (count + 127) / 128 * 128;
    lrk_logits_head &h = table[i];
    h.queries = static_cast<const char *>(queries.data_ptr()) + heads[i] * rows * dim * element;
    h.keys = static_cast<const char *>(keys.data_ptr()) + starts[i] * dim * element;
    h.count = count;
    h.k_step = k_steps[i];
    h.out = static_cast<char *>(flat.data_ptr()) + offsets[i] * element;
    h.out_stride = stride;
    auto head_logits = flat.narrow(0, offsets[i], rows * stride).view({rows, stride});
    // groups > 0: the head's [window, groups, count] view (rows = window * groups).
    out.push_back(groups > 0 ? head_logits.view({rows / groups, groups, stride}).narrow(2, 0, count) : head_logits);
  }
  check_status(lrk_logits_heads(table.data(), static_cast<int64_t>(n), rows, dim, current_stream()));
  return out;
}

// Temporal-risk scores of many heads straight from queries and keys
// (lrk_scores_from_keys).  Per layer l: keys[l] bf16 [rows, D], queries[l]
// bf16 [window, heads * groups, D] (query heads of KV head h at h * groups ..),
// projected[l] f32 [groups, rows] (project_values: each row against its own
// head's gradients), positions[l] f32 [rows].
// segments: (layer, head, key_row, length, first, last, query_chunk) per
// head.  Returns the segments' scores concatenated in segment order.
torch::Tensor scores_from_keys(std::vector<torch::Tensor> keys, std::vector<torch::Tensor> queries,
                               std::vector<torch::Tensor> projected, std::vector<torch::Tensor> positions,
                               std::vector<std::vector<int64_t>> segments, int64_t groups,
                               torch::Tensor query_positions, torch::Tensor margin, double scale, double epsilon) {
  const size_t layers = keys.size();
  TORCH_CHECK(layers > 0 && queries.size() == layers && projected.size() == layers && positions.size() == layers,
              "scores_from_keys: one keys, queries, projected and positions tensor per layer");
  TORCH_CHECK(!segments.empty() && groups > 0, "scores_from_keys: no segments");
  const torch::Tensor &reference = keys[0];
  check_cuda(query_positions, reference);
  check_cuda(margin, reference);
  TORCH_CHECK(query_positions.scalar_type() == at::kLong && margin.scalar_type() == at::kFloat && margin.numel() == 1,
              "scores_from_keys: int64 query positions and one float32 margin");
  const int64_t dim = reference.size(1), window = queries[0].size(0);
  TORCH_CHECK(query_positions.numel() == window, "scores_from_keys: one position per query");
  std::vector<lrk_key_layer> layer_table(layers);
  for (size_t l = 0; l < layers; ++l) {
    for (const auto &t : {keys[l], queries[l], projected[l], positions[l]}) check_cuda(t, reference);
    TORCH_CHECK(keys[l].dim() == 2 && keys[l].size(1) == dim && keys[l].scalar_type() == at::kBFloat16,
                "scores_from_keys: bf16 [rows, D] keys");
    TORCH_CHECK(queries[l].dim() == 3 && queries[l].size(0) == window && queries[l].size(1) % groups == 0 &&
                    queries[l].size(2) == dim && queries[l].scalar_type() == at::kBFloat16,
                "scores_from_keys: bf16 [window, heads * groups, D] queries");
    TORCH_CHECK(projected[l].dim() == 2 && projected[l].size(0) == groups &&
                    projected[l].size(1) == keys[l].size(0) && projected[l].scalar_type() == at::kFloat,
                "scores_from_keys: float32 [groups, rows] projected values");
    TORCH_CHECK(positions[l].numel() == keys[l].size(0) && positions[l].scalar_type() == at::kFloat,
                "scores_from_keys: float32 positions per key row");
    layer_table[l] = {keys[l].data_ptr(), keys[l].size(0)};
  }
  const int64_t count = static_cast<int64_t>(segments.size());
  std::vector<lrk_key_segment> table(count);
  std::vector<int64_t> offsets(count);
  int64_t total = 0;
  for (int64_t i = 0; i < count; ++i) {
    const auto &s = segments[i];
    TORCH_CHECK(s.size() == 7, "scores_from_keys: segments are (layer, head, key_row, length, first, last, chunk)");
    const int64_t l = s[0], head = s[1];
    TORCH_CHECK(l >= 0 && l < static_cast<int64_t>(layers), "scores_from_keys: layer out of range");
    TORCH_CHECK(head >= 0 && (head + 1) * groups <= queries[l].size(1), "scores_from_keys: head out of range");
    TORCH_CHECK(s[3] > 0 && s[2] >= 0 && s[2] + s[3] <= keys[l].size(0), "scores_from_keys: keys outside the layer");
    TORCH_CHECK(s[4] >= 0 && s[5] > s[4] && s[5] <= s[3], "Invalid risk interval");
    lrk_key_segment &t = table[i];
    t.layer = l;
    t.queries = static_cast<const at::BFloat16 *>(queries[l].data_ptr()) + head * groups * dim;
    t.query_stride = queries[l].size(1) * dim;
    t.projected_values = projected[l].data_ptr<float>() + s[2];
    t.projected_stride = projected[l].size(1);
    t.key_positions = positions[l].data_ptr<float>() + s[2];
    t.key_row = s[2];
    t.length = s[3];
    t.first = s[4];
    t.last = s[5];
    t.query_chunk = s[6];
    offsets[i] = total;
    total += s[5] - s[4];
  }
  c10::cuda::CUDAGuard guard(reference.device());
  auto scores = torch::empty({total}, reference.options().dtype(at::kFloat));
  for (int64_t i = 0; i < count; ++i) table[i].scores = scores.data_ptr<float>() + offsets[i];
  const size_t bytes = lrk_scores_from_keys_workspace_bytes(table.data(), count, window, groups);
  TORCH_CHECK(bytes > 0, "scores_from_keys: invalid segments");
  auto workspace = torch::empty({static_cast<int64_t>(bytes)}, reference.options().dtype(at::kByte));
  check_status(lrk_scores_from_keys(table.data(), count, layer_table.data(), static_cast<int64_t>(layers),
                                    query_positions.data_ptr<int64_t>(), window, groups, dim,
                                    static_cast<float>(scale), margin.data_ptr<float>(), static_cast<float>(epsilon),
                                    workspace.data_ptr(), bytes, current_stream()));
  return scores;
}

// Layer-group selection, one radix round on this rank: the histograms of
// request r's score table scores[r] (f32 [n_r], CUDA) per question, given the
// states ([requests, questions, LRK_SELECT_STATE_FIELDS] int64, CUDA).
// Returns [requests, questions, LRK_SELECT_BINS] int32 (the u32 counts' bits).
torch::Tensor select_histogram(std::vector<torch::Tensor> scores, torch::Tensor states, int64_t round) {
  check_cuda(states, states);
  TORCH_CHECK(states.scalar_type() == at::kLong && states.dim() == 3 && states.size(2) == LRK_SELECT_STATE_FIELDS,
              "states must be int64 [requests, questions, LRK_SELECT_STATE_FIELDS]");
  const int64_t requests = states.size(0), questions = states.size(1);
  TORCH_CHECK(static_cast<int64_t>(scores.size()) == requests, "one score table per request");
  std::vector<const float *> pointers(requests);
  std::vector<int64_t> counts(requests);
  for (int64_t r = 0; r < requests; ++r) {
    check_cuda(scores[r], states);
    TORCH_CHECK(scores[r].scalar_type() == at::kFloat && scores[r].dim() == 1, "score tables must be f32 [n]");
    pointers[r] = scores[r].data_ptr<float>();
    counts[r] = scores[r].numel();
  }
  c10::cuda::CUDAGuard guard(states.device());
  auto histograms = torch::empty({requests, questions, LRK_SELECT_BINS}, states.options().dtype(at::kInt));
  check_status(lrk_select_histogram(pointers.data(), counts.data(), requests, questions, static_cast<int>(round),
                                    states.data_ptr<int64_t>(),
                                    reinterpret_cast<uint32_t *>(histograms.data_ptr<int32_t>()), current_stream()));
  return histograms;
}

// Advance the states by one round from the all-gathered histograms
// ([world, requests, questions, LRK_SELECT_BINS] int32, CUDA).  In place.
void select_pick(torch::Tensor gathered, int64_t rank, torch::Tensor states, int64_t round) {
  check_cuda(gathered, states);
  check_cuda(states, states);
  TORCH_CHECK(states.scalar_type() == at::kLong && states.dim() == 3 && states.size(2) == LRK_SELECT_STATE_FIELDS,
              "states must be int64 [requests, questions, LRK_SELECT_STATE_FIELDS]");
  TORCH_CHECK(gathered.scalar_type() == at::kInt && gathered.dim() == 4 && gathered.size(1) == states.size(0) &&
                  gathered.size(2) == states.size(1) && gathered.size(3) == LRK_SELECT_BINS,
              "gathered must be int32 [world, requests, questions, LRK_SELECT_BINS]");
  c10::cuda::CUDAGuard guard(states.device());
  check_status(lrk_select_pick(reinterpret_cast<const uint32_t *>(gathered.data_ptr<int32_t>()), gathered.size(0),
                               rank, states.size(0), states.size(1), static_cast<int>(round),
                               states.data_ptr<int64_t>(), current_stream()));
}

// The KV arena of one cache: keys, values [heads_total, capacity, D] (one
// dtype), positions [heads_total, capacity] f32, lengths [heads_total] i32.
lrk_arena arena_of(const torch::Tensor &keys, const torch::Tensor &values, const torch::Tensor &positions,
                   const torch::Tensor &lengths) {
  for (const auto &tensor : {keys, values, positions, lengths}) check_cuda(tensor, keys);
  TORCH_CHECK(keys.dim() == 3 && keys.sizes() == values.sizes() && keys.scalar_type() == values.scalar_type(),
              "arena keys/values must be [heads, capacity, dimension] of one dtype");
  TORCH_CHECK(positions.scalar_type() == at::kFloat && positions.dim() == 2 && positions.size(0) == keys.size(0) &&
                  positions.size(1) == keys.size(1),
              "arena positions must be float32 [heads, capacity]");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.dim() == 1 && lengths.size(0) == keys.size(0),
              "arena lengths must be int32 [heads]");
  lrk_arena a{};
  a.keys = keys.data_ptr();
  a.values = values.data_ptr();
  a.positions = positions.data_ptr<float>();
  a.lengths = lengths.data_ptr<int32_t>();
  a.heads_total = keys.size(0);
  a.capacity = keys.size(1);
  a.dimension = keys.size(2);
  a.dtype = dtype_code(keys.scalar_type());
  return a;
}

// Recall rows into the arena in place (lrk_arena_insert): plan int64 [touched,
// 3] (head, first entry, count), recalled [entries, 2, D], recalled_positions
// float32 [entries].  check: only the checks.  Returns the device flag (int32 [1]).
torch::Tensor arena_insert(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor lengths,
                           torch::Tensor plan, torch::Tensor recalled, torch::Tensor recalled_positions, bool check) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  for (const auto &t : {plan, recalled, recalled_positions}) check_cuda(t, keys);
  TORCH_CHECK(plan.scalar_type() == at::kLong && plan.dim() == 2 && plan.size(1) == 3, "plan must be int64 [touched, 3]");
  TORCH_CHECK(recalled.scalar_type() == keys.scalar_type() && recalled.dim() == 3 && recalled.size(1) == 2 &&
                  recalled.size(2) == keys.size(2),
              "recalled rows must be [entries, 2, dimension] of the arena dtype");
  TORCH_CHECK(recalled_positions.scalar_type() == at::kFloat && recalled_positions.numel() == recalled.size(0),
              "recalled positions must be float32, one per recalled row");
  c10::cuda::CUDAGuard guard(keys.device());
  auto flag = torch::zeros({1}, lengths.options());
  check_status(lrk_arena_insert(&a, plan.data_ptr<int64_t>(), plan.size(0), recalled.data_ptr(),
                                recalled_positions.data_ptr<float>(), check ? 1 : 0,
                                reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
  return flag;
}

// Append one row per head to heads [first_head, first_head + new_keys.size(0))
// in place; returns the device overflow flag (int32 [1], nonzero if a head
// was full).
torch::Tensor arena_append(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor lengths,
                           int64_t first_head, torch::Tensor new_keys, torch::Tensor new_values, double position) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  check_cuda(new_keys, keys);
  check_cuda(new_values, keys);
  TORCH_CHECK(new_keys.scalar_type() == keys.scalar_type() && new_values.scalar_type() == keys.scalar_type() &&
                  new_keys.numel() == new_values.numel() && new_keys.numel() % keys.size(2) == 0,
              "new rows must be [heads, dimension] of the arena dtype");
  c10::cuda::CUDAGuard guard(keys.device());
  auto flag = torch::zeros({1}, lengths.options());
  check_status(lrk_arena_append(&a, first_head, new_keys.numel() / keys.size(2), new_keys.data_ptr(),
                                new_values.data_ptr(), static_cast<float>(position),
                                reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
  return flag;
}

// In-place eviction: plan int64 [touched, 3] = (head, offset, count) into
// removed (int64, ascending per head).  Returns the device error flag.
torch::Tensor arena_compact(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor lengths,
                            torch::Tensor plan, torch::Tensor removed) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  check_cuda(plan, keys);
  check_cuda(removed, keys);
  TORCH_CHECK(plan.scalar_type() == at::kLong && plan.dim() == 2 && plan.size(1) == 3, "plan must be int64 [n, 3]");
  TORCH_CHECK(removed.scalar_type() == at::kLong && removed.dim() == 1, "removed must be int64 [n]");
  c10::cuda::CUDAGuard guard(keys.device());
  auto flag = torch::zeros({1}, lengths.options());
  check_status(lrk_arena_compact(&a, plan.data_ptr<int64_t>(), plan.size(0), removed.data_ptr<int64_t>(),
                                 reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
  return flag;
}

// In-place eviction by logical position: removed is float32 (ascending per
// head, every position present in its head).  Returns the device error flag.
torch::Tensor arena_compact_positions(torch::Tensor keys, torch::Tensor values, torch::Tensor positions,
                                      torch::Tensor lengths, torch::Tensor plan, torch::Tensor removed) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  check_cuda(plan, keys);
  check_cuda(removed, keys);
  TORCH_CHECK(plan.scalar_type() == at::kLong && plan.dim() == 2 && plan.size(1) == 3, "plan must be int64 [n, 3]");
  TORCH_CHECK(removed.scalar_type() == at::kFloat && removed.dim() == 1, "removed must be float32 [n]");
  c10::cuda::CUDAGuard guard(keys.device());
  auto flag = torch::zeros({1}, lengths.options());
  check_status(lrk_arena_compact_positions(&a, plan.data_ptr<int64_t>(), plan.size(0), removed.data_ptr<float>(),
                                           reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()),
                                           current_stream()));
  return flag;
}

// Lazy eviction batch: heads int64 [n], removed float32 [n] (any order).
// Writes the device error flag into `flag` (int32 [1], the caller's).
void arena_evict(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor lengths,
                 torch::Tensor heads, torch::Tensor removed, torch::Tensor flag) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  for (const auto &tensor : {heads, removed, flag}) check_cuda(tensor, keys);
  TORCH_CHECK(heads.scalar_type() == at::kLong && removed.scalar_type() == at::kFloat && heads.dim() == 1 &&
                  removed.sizes() == heads.sizes(),
              "heads int64 [n] and removed float32 [n]");
  TORCH_CHECK(flag.scalar_type() == at::kInt && flag.numel() >= 1, "flag must be int32");
  c10::cuda::CUDAGuard guard(keys.device());
  check_status(lrk_arena_evict(&a, heads.data_ptr<int64_t>(), removed.data_ptr<float>(), heads.numel(),
                               reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
}

// arena_append writing its overflow flag into the caller's `flag` (no
// allocation per call).
void arena_append_into(torch::Tensor keys, torch::Tensor values, torch::Tensor positions, torch::Tensor lengths,
                       int64_t first_head, torch::Tensor new_keys, torch::Tensor new_values, double position,
                       torch::Tensor flag) {
  const lrk_arena a = arena_of(keys, values, positions, lengths);
  check_cuda(new_keys, keys);
  check_cuda(new_values, keys);
  check_cuda(flag, keys);
  TORCH_CHECK(new_keys.scalar_type() == keys.scalar_type() && new_values.scalar_type() == keys.scalar_type() &&
                  new_keys.numel() == new_values.numel() && new_keys.numel() % keys.size(2) == 0,
              "new rows must be [heads, dimension] of the arena dtype");
  TORCH_CHECK(flag.scalar_type() == at::kInt && flag.numel() >= 1, "flag must be int32");
  c10::cuda::CUDAGuard guard(keys.device());
  check_status(lrk_arena_append(&a, first_head, new_keys.numel() / keys.size(2), new_keys.data_ptr(),
                                new_values.data_ptr(), static_cast<float>(position),
                                reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
}

// Recall merge plans of several layers on the device (recall/planning.py:34-52).
// Per layer: positions (f32, the layer's [rows] or [rows, 1]), head_starts
// (int32 [heads + 1]), recalled positions (f32, sorted by (head, position)),
// their indices among the layer's recalled rows (int64), recalled_starts
// (int32 [heads + 1]).  Returns the mappings (int64 [rows + recalled] each) and
// the device flag (int32 [1]: bit 1 duplicate, bit 2 unsorted head).
std::tuple<std::vector<torch::Tensor>, torch::Tensor> merge_plan(std::vector<torch::Tensor> positions,
                                                                 std::vector<torch::Tensor> head_starts,
                                                                 std::vector<torch::Tensor> recalled_positions,
                                                                 std::vector<torch::Tensor> recalled_index,
                                                                 std::vector<torch::Tensor> recalled_starts) {
  const size_t count = positions.size();
  TORCH_CHECK(count > 0 && head_starts.size() == count && recalled_positions.size() == count &&
                  recalled_index.size() == count && recalled_starts.size() == count,
              "one entry per layer in every list");
  const auto &reference = positions[0];
  const int64_t heads = head_starts[0].numel() - 1;
  std::vector<lrk_plan_layer> table(count);
  std::vector<torch::Tensor> mappings;
  c10::cuda::CUDAGuard guard(reference.device());
  for (size_t i = 0; i < count; ++i) {
    for (const auto &t : {positions[i], head_starts[i], recalled_positions[i], recalled_index[i],
                          recalled_starts[i]})
      check_cuda(t, reference);
    TORCH_CHECK(positions[i].scalar_type() == at::kFloat && recalled_positions[i].scalar_type() == at::kFloat,
                "positions must be float32");
    TORCH_CHECK(head_starts[i].scalar_type() == at::kInt && recalled_starts[i].scalar_type() == at::kInt &&
                    head_starts[i].numel() == heads + 1 && recalled_starts[i].numel() == heads + 1,
                "head_starts and recalled_starts must be int32 [heads + 1]");
    TORCH_CHECK(recalled_index[i].scalar_type() == at::kLong &&
                    recalled_index[i].numel() == recalled_positions[i].numel(),
                "recalled_index must be int64, one per recalled position");
    const int64_t rows = positions[i].numel(), recalled = recalled_positions[i].numel();
    mappings.push_back(torch::empty({rows + recalled}, reference.options().dtype(at::kLong)));
    lrk_plan_layer &l = table[i];
    l.positions = positions[i].data_ptr<float>();
    l.head_starts = head_starts[i].data_ptr<int32_t>();
    l.recalled_positions = recalled_positions[i].data_ptr<float>();
    l.recalled_index = recalled_index[i].data_ptr<int64_t>();
    l.recalled_starts = recalled_starts[i].data_ptr<int32_t>();
    l.rows = rows;
    l.recalled = recalled;
    l.mapping = mappings.back().data_ptr<int64_t>();
  }
  auto flag = torch::zeros({1}, reference.options().dtype(at::kInt));
  check_status(lrk_merge_plan(table.data(), static_cast<int64_t>(count), heads,
                              reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
  return {mappings, flag};
}

// A recall event over several layers in two launches: the merge plan on the
// device (lrk_merge_plan) and the merge (lrk_merge_layers).  recalled [n, 2,
// D] and recalled_positions [n] hold the event's rows sorted by (layer, head,
// position); layer i's are rows firsts[i] .. firsts[i + 1], and
// recalled_starts[i] (int32 [layers, heads + 1], device) bounds its heads
// within them.  Returns the merged keys, values and positions per layer
// (views into one allocation each) and the plan's flag word (int32 [1]),
// which the caller reads before adopting them.
std::tuple<std::vector<torch::Tensor>, std::vector<torch::Tensor>, std::vector<torch::Tensor>, torch::Tensor>
reinsert_layers(std::vector<torch::Tensor> keys, std::vector<torch::Tensor> values,
                std::vector<torch::Tensor> positions, std::vector<torch::Tensor> head_starts, torch::Tensor recalled,
                torch::Tensor recalled_positions, torch::Tensor recalled_starts, std::vector<int64_t> firsts) {
  const size_t n = keys.size();
  TORCH_CHECK(n > 0 && values.size() == n && positions.size() == n && head_starts.size() == n &&
                  firsts.size() == n + 1,
              "reinsert_layers: one tensor of each kind per layer and layers + 1 bounds");
  const int64_t heads = head_starts[0].numel() - 1;
  const auto dimension = keys[0].size(1);
  for (const auto &t : {recalled, recalled_positions, recalled_starts}) check_recall_tensor(t, keys[0]);
  TORCH_CHECK(recalled.dim() == 3 && recalled.size(1) == 2 && recalled.size(2) == dimension &&
                  recalled.scalar_type() == keys[0].scalar_type(),
              "Invalid recalled shape");
  TORCH_CHECK(recalled_positions.scalar_type() == at::kFloat && recalled_positions.numel() == recalled.size(0),
              "Invalid positions");
  TORCH_CHECK(recalled_starts.scalar_type() == at::kInt && recalled_starts.numel() == static_cast<int64_t>(n) * (heads + 1),
              "recalled_starts must be int32 [layers, heads + 1]");
  TORCH_CHECK(firsts[0] == 0 && firsts[n] == recalled.size(0), "firsts must run from 0 to the recalled rows");
  std::vector<lrk_plan_layer> plan(n);
  std::vector<lrk_merge_layer> table(n);
  int64_t total = 0;
  for (size_t i = 0; i < n; ++i) {
    for (const auto &tensor : {keys[i], values[i], positions[i], head_starts[i]}) check_recall_tensor(tensor, keys[0]);
    TORCH_CHECK(keys[i].dim() == 2 && keys[i].size(1) == dimension && keys[i].sizes() == values[i].sizes(),
                "Invalid K/V shape");
    TORCH_CHECK(keys[i].scalar_type() == keys[0].scalar_type() && values[i].scalar_type() == keys[0].scalar_type(),
                "K/V dtypes differ");
    TORCH_CHECK(positions[i].scalar_type() == at::kFloat && positions[i].numel() == keys[i].size(0),
                "Invalid positions");
    TORCH_CHECK(head_starts[i].scalar_type() == at::kInt && head_starts[i].numel() == heads + 1,
                "head_starts must be int32 [heads + 1]");
    TORCH_CHECK(firsts[i] <= firsts[i + 1], "firsts must ascend");
    total += keys[i].size(0) + firsts[i + 1] - firsts[i];
  }
  c10::cuda::CUDAGuard guard(keys[0].device());
  auto mapping = torch::empty({total}, keys[0].options().dtype(at::kLong));
  auto all_keys = torch::empty({total, dimension}, keys[0].options());
  auto all_values = torch::empty_like(all_keys);
  auto all_positions = torch::empty({total, 1}, positions[0].options());
  auto flag = torch::zeros({1}, keys[0].options().dtype(at::kInt));
  const int64_t row_bytes = 2 * dimension * recalled.element_size();
  int64_t first = 0;
  for (size_t i = 0; i < n; ++i) {
    const int64_t rows = keys[i].size(0), count = firsts[i + 1] - firsts[i];
    const float *recalled_at = recalled_positions.data_ptr<float>() + firsts[i];
    plan[i] = {positions[i].data_ptr<float>(), head_starts[i].data_ptr<int32_t>(), recalled_at, nullptr,
               recalled_starts.data_ptr<int32_t>() + i * (heads + 1), rows, count,
               mapping.data_ptr<int64_t>() + first};
    table[i] = {keys[i].data_ptr(), values[i].data_ptr(), positions[i].data_ptr<float>(), rows,
                static_cast<const char *>(recalled.data_ptr()) + firsts[i] * row_bytes, recalled_at, count,
                mapping.data_ptr<int64_t>() + first, rows + count};
    first += rows + count;
  }
  if (total) {
    check_status(lrk_merge_plan(plan.data(), static_cast<int64_t>(n), heads,
                                reinterpret_cast<unsigned int *>(flag.data_ptr<int32_t>()), current_stream()));
    check_status(lrk_merge_layers(table.data(), static_cast<int64_t>(n), dimension, dtype_code(keys[0].scalar_type()),
                                  all_keys.data_ptr(), all_values.data_ptr(), all_positions.data_ptr<float>(),
                                  current_stream()));
  }
  std::vector<torch::Tensor> out_keys, out_values, out_positions;
  first = 0;
  for (size_t i = 0; i < n; ++i) {
    const int64_t rows = keys[i].size(0) + firsts[i + 1] - firsts[i];
    out_keys.push_back(all_keys.narrow(0, first, rows));
    out_values.push_back(all_values.narrow(0, first, rows));
    out_positions.push_back(all_positions.narrow(0, first, rows));
    first += rows;
  }
  return {out_keys, out_values, out_positions, flag};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("temporal_probabilities", &temporal_probabilities);
  module.def("temporal_risk", &temporal_risk);
  module.def("append", &append);
  module.def("compact", &compact);
  module.def("compact_layers", &compact_layers);
  module.def("merge_layers", &merge_layers);
  module.def("scores_from_keys", &scores_from_keys);
  module.def("pool", &pool);
  module.def("merge", &merge);
  module.def("pack", &pack);
  module.def("batch_append", &batch_append);
  module.def("refine", &refine);
  module.def("topk_smallest", &topk_smallest);
  module.def("logits", &logits);
  module.def("logits_heads", &logits_heads, pybind11::arg("queries"), pybind11::arg("keys"), pybind11::arg("heads"),
             pybind11::arg("starts"), pybind11::arg("ends"), pybind11::arg("k_steps"), pybind11::arg("groups") = 0);
  module.def("temporal_scores", &temporal_scores, pybind11::arg("logits"), pybind11::arg("projected_values"),
             pybind11::arg("key_positions"), pybind11::arg("first"), pybind11::arg("last"),
             pybind11::arg("query_positions"), pybind11::arg("margin"), pybind11::arg("scale"),
             pybind11::arg("epsilon"), pybind11::arg("query_chunks") = std::vector<int64_t>{},
             pybind11::arg("probability_stash") = true);
  module.def("project_values", &project_values);
  module.def("select_histogram", &select_histogram);
  module.def("select_pick", &select_pick);
  module.def("arena_append", &arena_append);
  module.def("arena_compact", &arena_compact);
  module.def("arena_insert", &arena_insert);
  module.def("arena_compact_positions", &arena_compact_positions);
  module.def("arena_evict", &arena_evict);
  module.def("arena_append_into", &arena_append_into);
  module.def("merge_plan", &merge_plan);
  module.def("reinsert_layers", &reinsert_layers);
}
