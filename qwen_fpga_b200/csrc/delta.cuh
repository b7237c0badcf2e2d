// Host-side entry point of the standalone delta-rule operator (delta.cu).
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace qb {

// The gated delta rule of one 16-head layer on caller buffers
// (S [16][128][128] in place, out [16][128]).
cudaError_t enqueue_delta_rule(const float* q, const float* k, const float* v, const float* g,
                               const float* beta, float* S, float* out, cudaStream_t st);

}  // namespace qb
