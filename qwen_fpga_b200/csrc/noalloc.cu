// Allocation-free int8 GEMV + argmax (device pointers, no context).
//
// A standalone variant of the head's GEMV + block-argmax (the tied head of
// golden/model.py:266-267 with hls/src/gemv.hpp:63-73 row dots and the strict
// '>' first-index argmax of hls/src/qwen_synth.hpp:86): y = s .* (W x) with
// the arithmetic of k_gemv (gemv.cu), plus the index of the largest y.  The
// per-block maxima and the arrival counter live in a file-scope device array,
// so a call allocates nothing: no cudaMalloc, no library allocator.
#include <mutex>

#include "common.cuh"
#include "noalloc.cuh"

namespace qb {

// [0, NA_MAX_BLOCKS): one packed (value, index) maximum per block, written by
// the block before it arrives (no initial value needed).
// [NA_MAX_BLOCKS]: arrival counter.  It must be zero when a call's kernel
// starts: every call clears it on its stream just before the launch (a memset
// of 8 bytes, no allocation), so a launch that failed part-way cannot leave a
// stale count for the next call; the last block also resets it.
static __device__ __align__(256) unsigned long long g_argmax_scratch[NA_MAX_BLOCKS + 1];

// Block b owns rows [b * NA_ROWS_PER_BLOCK, ...); its 8 warps take 4-row units.
__global__ void __launch_bounds__(256) k_gemv_argmax(float* __restrict__ y, int* __restrict__ argmax,
                                                     const int8_t* __restrict__ w,
                                                     const float* __restrict__ s,
                                                     const float* __restrict__ xf, int N, int K,
                                                     unsigned long long* scratch) {
  constexpr int R = 4;
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  __shared__ unsigned long long wbest[8];
  __shared__ int last;
  for (int i = threadIdx.x; i < K; i += blockDim.x) enc.xf[i] = xf[i];
  __syncthreads();
  encode_x(enc, K, false, red);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int row_lo = blockIdx.x * NA_ROWS_PER_BLOCK;
  const int row_hi = min(N, row_lo + NA_ROWS_PER_BLOCK);
  unsigned long long best = 0ull;
  for (int r0 = row_lo + R * wid; r0 < row_hi; r0 += R * 8) {
    const int8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = w + (size_t)min(r0 + r, N - 1) * K;  // ragged tail re-reads
    int acc[R][3];
    warp_rows_dot<R>(rows, enc, K, acc);
    if (lane < R && r0 + lane < row_hi) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r == lane) { a0 = acc[r][0]; a1 = acc[r][1]; a2 = acc[r][2]; }
      const int o = r0 + lane;
      const float v = finish_row(a0, a1, a2, 3, enc.scale, s[o]);
      if (y) y[o] = v;
      best = umax64(best, am_pack(v, o));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) wbest[wid] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int i = 0; i < 8; ++i) b = umax64(b, wbest[i]);
    scratch[blockIdx.x] = b;
    __threadfence();
    last = (atomicAdd(scratch + NA_MAX_BLOCKS, 1ull) == (unsigned long long)gridDim.x - 1ull);
  }
  __syncthreads();
  if (!last) return;
  // last block: reduce every block's maximum, publish the index, re-arm the counter
  __threadfence();
  unsigned long long b = 0ull;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) b = umax64(b, __ldcg(scratch + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
  if (lane == 0) wbest[wid] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) b = umax64(b, wbest[i]);
    *argmax = am_index(b);
    scratch[NA_MAX_BLOCKS] = 0ull;
  }
}

// Device address of the scratch, resolved once per device (the first call on a
// device does it; that first call must come before any stream capture).
static cudaError_t scratch_for_current_device(unsigned long long** out) {
  static std::mutex mu;
  static unsigned long long* addr[NA_MAX_DEVICES] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= NA_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_argmax_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = static_cast<unsigned long long*>(p);
  }
  *out = addr[dev];
  return cudaSuccess;
}

cudaError_t enqueue_gemv_argmax_noalloc(float* y, int* argmax, const int8_t* w, const float* s,
                                        const float* xf, int N, int K, cudaStream_t st) {
  unsigned long long* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return e;
  const int blocks = (N + NA_ROWS_PER_BLOCK - 1) / NA_ROWS_PER_BLOCK;
  e = cudaMemsetAsync(scratch + NA_MAX_BLOCKS, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess) return e;
  k_gemv_argmax<<<blocks, 256, 0, st>>>(y, argmax, w, s, xf, N, K, scratch);
  return cudaGetLastError();
}

}  // namespace qb
