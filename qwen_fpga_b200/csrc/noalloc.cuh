// Host-side interface of the allocation-free GEMV + argmax (noalloc.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qb {

constexpr int NA_ROWS_PER_BLOCK = 1024;   // rows per block
constexpr int NA_MAX_BLOCKS = 1024;       // slots of the static scratch
constexpr int NA_MAX_ROWS = NA_ROWS_PER_BLOCK * NA_MAX_BLOCKS;   // 1,048,576
constexpr int NA_MAX_DEVICES = 64;

// y (nullable) = s .* (W x); *argmax = first index of the largest y.  Same
// argument rules as enqueue_gemv's fp32-x kernel plus 1 <= N <= NA_MAX_ROWS
// (checked by the caller).  Calls on one device must not overlap in time.
cudaError_t enqueue_gemv_argmax_noalloc(float* y, int* argmax, const int8_t* w, const float* s,
                                        const float* xf, int N, int K, cudaStream_t st);

}  // namespace qb
