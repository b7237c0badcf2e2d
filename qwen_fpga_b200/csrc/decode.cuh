// Host-side entry points of the decode-step kernels (decode.cu).
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace qb {

// Enqueue one decode step (all per-step values come from device memory, so
// the sequence can be captured once into a CUDA graph and replayed).
cudaError_t enqueue_step(const ModelW& Mh, ModelW* Md, const StateW& S, int sm_count,
                         cudaStream_t st);
// Number of argmax partials the head writes.
int head_grid_size(int sm_count);

// The gated delta rule of one 16-head layer on caller buffers
// (S [16][128][128] in place, out [16][128]).
cudaError_t enqueue_delta_rule(const float* q, const float* k, const float* v, const float* g,
                               const float* beta, float* S, float* out, cudaStream_t st);

}  // namespace qb
