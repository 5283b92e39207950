// Phases of the fused temporal-risk scorer (fused.cu) that other launchers
// reuse (scores_tc.cu): the visible-prefix pre-pass and the risk kernels over
// precomputed row statistics.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "lrk.h"

namespace lrk {

// visible[(s * window) + q] for every segment s (fused.cu: visibility_kernel).
int score_visibility(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window,
                     int32_t *visible, cudaStream_t stream);

// Scores of every segment's candidates from bf16 logits and the row
// statistics stats[(s * window * groups) + row] (fused.cu: risk kernels).
int score_risk_bf16(const lrk_score_segment *segments, int64_t count, const int64_t *qpos, int window, int groups,
                    float scale, const float *margin, float epsilon, const float3 *stats, cudaStream_t stream);

}  // namespace lrk
