// Host-side entry point of the standalone GEMV kernels (gemv.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qb {

// xq != nullptr selects the int8 x int8 kernel (acc and y each nullable);
// otherwise the fp32-x kernel (xf, y required).  N >= 1, K % 32 == 0,
// 32 <= K <= KMAX, w 32-byte aligned.
cudaError_t enqueue_gemv(float* y, int32_t* acc, const int8_t* w, const float* s, const float* xf,
                         const int8_t* xq, float sx, int N, int K, int sm_count, cudaStream_t st);

}  // namespace qb
