// Standalone int8-weight GEMV operators of libqwenb200 (device pointers).
//
//   gemv_i8_f32 : y = s .* (W x), fp32 x  -- hls/src/gemv.hpp:28-42
//   gemv_i8_i8  : acc = W xq exactly in int32, y = acc * sx * sw
//                 -- rtl/gemv_i8.sv:13-76 + rtl/dequant.sv:12-29,
//                    scripts/export_gemv_tv.py:49-50
//
// Each CTA owns a contiguous range of rows: it asks L2 for their weights
// (bulk prefetch) before waiting on the previous kernel, stages x (its digit
// image) in shared memory once, then its warps stream R weight rows at a time
// with 32-byte-per-lane loads and reduce the dp4a partial sums with warp
// shuffles into int32 accumulators; the per-row scale is applied in the
// epilogue.
#include "common.cuh"
#include "gemv.cuh"

namespace qb {

// x staging: W8A32 -> three-digit image of fp32 x; W8A8 -> xq copied as digit 0.
template <int R, bool XINT8>
__global__ void __launch_bounds__(256) k_gemv(float* __restrict__ y, int32_t* __restrict__ acc_out,
                                              const int8_t* __restrict__ w,
                                              const float* __restrict__ s, const float* xf,
                                              const int8_t* xq, float sx, int N, int K) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  // This CTA's rows are [r_lo, r_hi) (contiguous).  Their weights do not depend
  // on the previous kernel: ask L2 for them before griddepcontrol.wait, so that
  // under programmatic dependent launch they stream in while it drains.
  const int units_all = (N + R - 1) / R;
  const int upc = (units_all + gridDim.x - 1) / gridDim.x;   // row units per CTA
  const int r_lo = min(N, (int)blockIdx.x * upc * R), r_hi = min(N, r_lo + upc * R);
  if (threadIdx.x < 32) {
    // (at most the first 64 KB: a large GEMV's CTAs together would otherwise
    // ask for more than L2 holds before they reach it)
    const size_t lo = (size_t)r_lo * K;   // K % 32 == 0: 32-byte aligned pieces
    const size_t hi = min((size_t)r_hi * K, lo + (size_t)65536);
    for (size_t off = lo + (size_t)threadIdx.x * 4096; off < hi; off += 32 * 4096) {
      const unsigned bytes = (unsigned)min((size_t)4096, hi - off);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(w + off), "r"(bytes) : "memory");
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (XINT8) {
    int8_t* d0 = &enc.dig[0][0][0];
    for (int i = threadIdx.x; i < K; i += blockDim.x) d0[dig_off(i)] = xq[i];
    if (threadIdx.x == 0) { enc.scale = (double)sx; enc.ndig = 1; enc.K = K; }
    __syncthreads();
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) enc.xf[i] = xf[i];
    __syncthreads();
    encode_x(enc, K, false, red);
  }
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int u = (int)blockIdx.x * upc + wid; u < min(units_all, ((int)blockIdx.x + 1) * upc); u += nw) {
    const int r0 = u * R;
    const int8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int rr = (r0 + r < N) ? (r0 + r) : (N - 1);   // ragged tail re-reads the last row
      rows[r] = w + (size_t)rr * K;
    }
    int acc[R][3];
    warp_rows_dot<R>(rows, enc, K, acc);
    if (lane < R && r0 + lane < N) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r == lane) { a0 = acc[r][0]; a1 = acc[r][1]; a2 = acc[r][2]; }
      const int o = r0 + lane;
      if (XINT8) {
        if (acc_out) acc_out[o] = a0;
        // y = acc * sx * sw in fp32, the dequant order of export_gemv_tv.py:50
        if (y) y[o] = __fmul_rn(__fmul_rn(__int2float_rn(a0), sx), s[o]);
      } else {
        y[o] = finish_row(a0, a1, a2, 3, enc.scale, s[o]);
      }
    }
  }
}

static int grid_for(int N, int R, int sm_count) {
  const int warps_needed = (N + R - 1) / R;
  int g = (warps_needed + 7) / 8;
  const int cap = 4 * sm_count;
  return g < 1 ? 1 : (g > cap ? cap : g);
}

// Launched with programmatic dependent launch: a GEMV's weight prefetch and
// launch overlap the previous kernel in the stream.
template <int R, bool XINT8>
static cudaError_t launch_gemv(int grid, float* y, int32_t* acc, const int8_t* w, const float* s, const float* xf,
                               const int8_t* xq, float sx, int N, int K, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_gemv<R, XINT8>, y, acc, w, s, xf, xq, sx, N, K);
}

cudaError_t enqueue_gemv(float* y, int32_t* acc, const int8_t* w, const float* s, const float* xf,
                         const int8_t* xq, float sx, int N, int K, int sm_count, cudaStream_t st) {
  const bool big = N >= 8 * 8 * sm_count * 4;   // enough rows to give every warp 4-row units
  if (xq) {
    if (big) return launch_gemv<4, true>(grid_for(N, 4, sm_count), y, acc, w, s, xf, xq, sx, N, K, st);
    return launch_gemv<1, true>(grid_for(N, 1, sm_count), y, acc, w, s, xf, xq, sx, N, K, st);
  }
  if (big) return launch_gemv<4, false>(grid_for(N, 4, sm_count), y, acc, w, s, xf, xq, sx, N, K, st);
  return launch_gemv<1, false>(grid_for(N, 1, sm_count), y, acc, w, s, xf, xq, sx, N, K, st);
}

}  // namespace qb
