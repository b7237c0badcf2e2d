// Shared device-side definitions of libqwenb200: model dimensions, the device
// views of the packed weight blob and of the decode state, and the integer
// GEMV building blocks every projection uses.
//
// Arithmetic contract: golden/model.py of allthingssecurity/qwen_fpga.
//
// GEMV numerics.  Every int8-weight projection computes
//     y[o] = s_w[o] * sum_i q[o,i] * x[i]
// with an exact integer inner product:
//   * W8A8 (ACT_INT8, golden/model.py:37-45): x is quantised per vector to
//     int8 (s_x = amax/127, rint half-even, clip +-127); acc = sum q*xq is an
//     exact int32 (rtl/gemv_i8.sv:13-76) and y = acc * s_x * s_w (dequant.sv).
//   * W8A32: x is mapped to a signed fixed-point image X = rint(x * 2^sh),
//     sh = 22 - ceil_log2(max|x|), so |X| <= 2^22; X is split into three int8
//     digits X = D0 + 256*D1 + 65536*D2 (D0, D1 in [-128,127], D2 in [-64,64]);
//     each digit row is dotted with q by dp4a into an exact int32
//     (|sum| <= 3584*127*128 < 2^31), the three sums are recombined exactly in
//     int64 and scaled once in fp64.  The only approximation is x's rounding to
//     the 2^-sh grid (relative 2^-23 of max|x|), which is below the fp32
//     summation error of the golden's BLAS product.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qb {

// ---- model dimensions (hls/src/types.hpp:19-47)
constexpr int HID = 1024;
constexpr int NLAYER = 24;
constexpr int FFN = 3584;
constexpr int VOCAB = 248320;
constexpr int NLIN = 18;
constexpr int NFULL = 6;
constexpr int LH = 16;          // DeltaNet heads
constexpr int LK = 128;         // key head dim
constexpr int LV = 128;         // value head dim
constexpr int KDIM = LH * LK;   // 2048
constexpr int VDIM = LH * LV;   // 2048
constexpr int CONVD = 2 * KDIM + VDIM;  // 6144
constexpr int CONVK = 4;
constexpr int NH = 8;           // attention query heads
constexpr int NKV = 2;          // attention kv heads
constexpr int HD = 256;         // attention head dim
constexpr int QPROJ = NH * HD * 2;  // 4096, per head [query 256 | gate 256]
constexpr int KVPROJ = NKV * HD;    // 512
constexpr int ROT = 64;         // rotated dims (head_dim * 0.25)
constexpr int KMAX = FFN;       // largest GEMV reduction length in the model
constexpr float EPS = 1e-6f;

// The standalone delta-rule operator: each head's 128 value columns in slices of DSLICE.
constexpr int DSLICE = 16;
constexpr int NDSLICE = LV / DSLICE;      // 8
// attention split-KV: at most ATT_MAXCH chunks per kv head; cached positions per attention layer
constexpr int ATT_MAXCH = 64;
constexpr int MAX_CTX = 65536;
constexpr int AM_PARTS = 4096;           // argmax partial slots (>= the grid)

// ---- device view of one layer's tensors inside the uploaded blob
struct LayerW {
  int linear;                 // 1 = gated DeltaNet, 0 = full attention
  int lin_idx, full_idx;      // index among linear / full layers
  const float* in_norm;       // [1024]  (1+w) RMSNorm gain offsets
  const float* post_norm;     // [1024]
  // gated DeltaNet (golden/model.py:135-191)
  const int8_t* qkv_q; const float* qkv_s;   // [6144,1024]
  const int8_t* z_q;   const float* z_s;     // [2048,1024]
  const float* b_w;    const float* a_w;     // [16,1024] fp32
  const float* conv_w;                       // [6144,1,4]
  const float* A_log;  const float* dt_bias; // [16]
  const float* gnorm_w;                      // [128] gain w (not 1+w)
  const int8_t* out_q; const float* out_s;   // [1024,2048]
  // gated full attention (golden/model.py:194-230)
  const int8_t* q_q; const float* q_s;       // [4096,1024]
  const int8_t* k_q; const float* k_s;       // [512,1024]
  const int8_t* v_q; const float* v_s;       // [512,1024]
  const float* qn_w; const float* kn_w;      // [256]
  const int8_t* o_q; const float* o_s;       // [1024,2048]
  // SwiGLU MLP (golden/model.py:233-237)
  const int8_t* gate_q; const float* gate_s; // [3584,1024]
  const int8_t* up_q;   const float* up_s;   // [3584,1024]
  const int8_t* down_q; const float* down_s; // [1024,3584]
  // panel copies for the persistent engine (layout in persist.cuh; null until
  // built): pin = the input projections [qkv | z] or [q | k | v]; pout =
  // out_proj / o_proj; pgu = (gate, up) pair panels; pdown = down_proj
  const int8_t* pin;
  const int8_t* pout;
  const int8_t* pgu;
  const int8_t* pdown;
};

struct ModelW {
  const int8_t* emb_q; const float* emb_s;   // [248320,1024], [248320] (tied head)
  const float* final_norm;                   // [1024]
  LayerW L[NLAYER];
};

// ---- per-step values that change every token; they live in device memory,
// read by each launch of the decode kernel.
struct StepDyn {
  int pos;        // RoPE position of the token being decoded
  int T;          // cached positions per attention layer before this token
  int conv_base;  // ring origin of the conv history (advances by one per step)
  int step;       // steps run since the token program was armed
  int n_prompt;   // tokens taken from `prompt` before switching to greedy feedback
  int act_int8;   // ACT_INT8 switch
  int want_logits;
  int seq;        // launch sequence number (tags of the persistent kernel)
};

// ---- device decode state of one sequence
struct StateW {
  float* conv;       // [18][6144][4] conv history ring
  float* rec;        // [18][16][128][128] DeltaNet state
  float* kcache;     // [6][max_ctx][512] post-RoPE K
  float* vcache;     // [6][max_ctx][512] V
  const float* rope; // [max_ctx][64]: cos[32] | sin[32] (angles pos * inv_freq)
  float* logits;     // [248320]
  unsigned long long* am_part;  // [AM_PARTS] packed (logit, index) maxima
  int* io;           // [2 + max_steps]: step, n_prompt, prompt tokens
  int* ids;          // [max_steps] argmax of every step
  int* err;          // device error word (0 = ok)
  StepDyn* dyn;
  int max_ctx;       // KV slots per attention layer
  int max_rope;      // rows of the RoPE table
  int max_steps;     // capacity of io / ids
};

// device error codes (first one wins)
constexpr int ERR_TOKEN = 1;   // token id outside the vocabulary
constexpr int ERR_CTX = 2;     // KV cache / RoPE table / step log full
constexpr int ERR_WAIT = 3;    // a bounded device wait ran out
constexpr int ERR_CHECK = 4;   // a device-side bounds check failed (site in err[1], value in err[2])

// ---- small helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum / max; `red` is >= 32 floats of shared scratch.  All threads
// of the block must call; returns the result to every thread.  The sum adds
// the per-warp partials in warp order.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < nw; ++w) t += red[w];
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.0f;
  return warp_max(t);
}

// fp32 nonlinearities of golden/model.py:50-60, evaluated without FMA
// contraction so each step rounds like the numpy expression.
__device__ __forceinline__ float silu_f(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}
__device__ __forceinline__ float sigmoid_f(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
}
__device__ __forceinline__ float softplus_f(float x) {
  return x > 20.0f ? x : log1pf(expf(fminf(x, 20.0f)));
}

// Total order on (logit, index): larger logit first, then the smaller index
// (np.argmax and the strict '>' of hls/src/qwen_synth.hpp:86 keep the first).
// -0.0 and +0.0 are one value (np.argmax compares them equal, so the first
// index wins); NaN ranks above every number, so the first NaN wins, as with
// np.argmax.
__device__ __forceinline__ unsigned long long am_pack(float v, int idx) {
  unsigned u = __float_as_uint(v);
  if ((u << 1) == 0u) u = 0u;                          // -0.0 -> +0.0
  u = ((u & 0x7fffffffu) > 0x7f800000u) ? 0xffffffffu  // NaN
      : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
  return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (unsigned)idx);
}
__device__ __forceinline__ int am_index(unsigned long long p) {
  return (int)(0xffffffffu - (unsigned)(p & 0xffffffffull));
}
__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// ---- the encoded GEMV input held in shared memory
//
// Digit layout: element k of digit d lives in dig[d][(k >> 4) & 1][16*(k >> 5) + (k & 15)],
// i.e. each 32-byte lane chunk of a weight row meets its 32 digits as two
// 16-byte pieces in separate half-planes, so a warp's LDS.128 reads are
// contiguous (bank-conflict free) while its weight loads are 32 bytes per lane.
struct XEnc {
  int8_t dig[3][2][KMAX / 2];  // int8 digits (W8A32: 3 digits, W8A8: digit 0 = xq)
  float xf[KMAX];              // fp32 vector the fp32-weight rows multiply
  double scale;                // W8A32: 2^-sh; W8A8: s_x
  int ndig;                    // 3 or 1
  int K;
};

__device__ __forceinline__ int dig_off(int k) { return ((k >> 4) & 1) * (KMAX / 2) + 16 * (k >> 5) + (k & 15); }

// Encode xf[0..K) (already in smem) into `e`.  Block-wide.  act_int8 selects the
// golden _qa quantiser (golden/model.py:37-45); otherwise the 3-digit image.
// `red` >= 32 floats of smem scratch.  K must be a multiple of 32.
__device__ __forceinline__ void encode_x(XEnc& e, int K, bool act_int8, float* red) {
  float m = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(e.xf[i]));
  const float amax = block_max(m, red);
  int8_t* d0p = &e.dig[0][0][0];
  int8_t* d1p = &e.dig[1][0][0];
  int8_t* d2p = &e.dig[2][0][0];
  if (act_int8) {
    if (amax == 0.0f) {
      for (int i = threadIdx.x; i < K; i += blockDim.x) d0p[dig_off(i)] = 0;
      if (threadIdx.x == 0) { e.scale = 1.0; e.ndig = 1; e.K = K; }
    } else {
      const float s = __fdiv_rn(amax, 127.0f);
      for (int i = threadIdx.x; i < K; i += blockDim.x) {
        float q = rintf(__fdiv_rn(e.xf[i], s));
        q = fminf(fmaxf(q, -127.0f), 127.0f);
        d0p[dig_off(i)] = (int8_t)(int)q;
        e.xf[i] = __fmul_rn(q, s);   // the fake-quant value fp32 rows multiply
      }
      if (threadIdx.x == 0) { e.scale = (double)s; e.ndig = 1; e.K = K; }
    }
  } else {
    int ex = 0;
    if (amax > 0.0f) frexpf(amax, &ex);   // amax in [2^(ex-1), 2^ex)
    const int sh = 22 - ex;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      const int X = (amax > 0.0f) ? (int)rintf(ldexpf(e.xf[i], sh)) : 0;
      const int a0 = (int)(int8_t)(X & 0xff);
      const int X1 = (X - a0) >> 8;
      const int a1 = (int)(int8_t)(X1 & 0xff);
      const int a2 = (X1 - a1) >> 8;
      const int o = dig_off(i);
      d0p[o] = (int8_t)a0;
      d1p[o] = (int8_t)a1;
      d2p[o] = (int8_t)a2;
    }
    if (threadIdx.x == 0) { e.scale = ldexp(1.0, -sh); e.ndig = 3; e.K = K; }
  }
  __syncthreads();
}

// Exact int64 recombination of the digit sums and the single fp64 scaling.
__device__ __forceinline__ float finish_row(int a0, int a1, int a2, int ndig, double xscale,
                                            float sw) {
  long long Y = (long long)a0;
  if (ndig == 3) Y += ((long long)a1 << 8) + ((long long)a2 << 16);
  return __double2float_rn((double)Y * xscale * (double)sw);
}

struct W32 { int v[8]; };

// 32 weight bytes per lane, streamed: read once per token, so bypass L1 and
// mark them first to leave L2 (keeps the recurrent state and activations resident).
__device__ __forceinline__ W32 ldg_stream32(const int8_t* p) {
  W32 w;
  asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w.v[0]), "=r"(w.v[1]), "=r"(w.v[2]), "=r"(w.v[3]), "=r"(w.v[4]),
                 "=r"(w.v[5]), "=r"(w.v[6]), "=r"(w.v[7])
               : "l"(p));
  return w;
}

// 32 weights of lane chunk c against digit plane `plane` (layout of dig_off).
__device__ __forceinline__ void dot32(int& a, const W32& w, const int8_t* plane, int c) {
  const int4 x0 = *reinterpret_cast<const int4*>(plane + 16 * c);
  const int4 x1 = *reinterpret_cast<const int4*>(plane + KMAX / 2 + 16 * c);
  a = __dp4a(w.v[0], x0.x, a);
  a = __dp4a(w.v[1], x0.y, a);
  a = __dp4a(w.v[2], x0.z, a);
  a = __dp4a(w.v[3], x0.w, a);
  a = __dp4a(w.v[4], x1.x, a);
  a = __dp4a(w.v[5], x1.y, a);
  a = __dp4a(w.v[6], x1.z, a);
  a = __dp4a(w.v[7], x1.w, a);
}

// One warp: R rows (row pointers rows[r], all of length K, K % 32 == 0,
// 32-byte aligned) dotted with the encoded x.  Returns, in every lane, the
// digit sums of each row in acc[r][0..ndig-1].
template <int R>
__device__ __forceinline__ void warp_rows_dot(const int8_t* const* rows, const XEnc& e, int K,
                                              int (&acc)[R][3]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = acc[r][2] = 0;
  const int nch = K >> 5;          // 32-byte chunks per row
  const int nd = e.ndig;
  for (int c = lane; c < nch; c += 64) {
    const bool two = (c + 32) < nch;
    W32 w0[R], w1[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      w0[r] = ldg_stream32(rows[r] + 32 * c);
      if (two) w1[r] = ldg_stream32(rows[r] + 32 * (c + 32));
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      dot32(acc[r][0], w0[r], &e.dig[0][0][0], c);
      if (two) dot32(acc[r][0], w1[r], &e.dig[0][0][0], c + 32);
      if (nd == 3) {
        dot32(acc[r][1], w0[r], &e.dig[1][0][0], c);
        dot32(acc[r][2], w0[r], &e.dig[2][0][0], c);
        if (two) {
          dot32(acc[r][1], w1[r], &e.dig[1][0][0], c + 32);
          dot32(acc[r][2], w1[r], &e.dig[2][0][0], c + 32);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    acc[r][0] = warp_sum_i(acc[r][0]);
    if (nd == 3) {
      acc[r][1] = warp_sum_i(acc[r][1]);
      acc[r][2] = warp_sum_i(acc[r][2]);
    }
  }
}

// One warp: fp32 row (length K, K % 128 == 0) dotted with e.xf.
__device__ __forceinline__ float warp_row_dot_f32(const float* row, const XEnc& e, int K) {
  const int lane = threadIdx.x & 31;
  float a = 0.0f;
  for (int i = 4 * lane; i < K; i += 128) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(row + i));
    const float4 x = *reinterpret_cast<const float4*>(&e.xf[i]);
    a = fmaf(w.x, x.x, a);
    a = fmaf(w.y, x.y, a);
    a = fmaf(w.z, x.z, a);
    a = fmaf(w.w, x.w, a);
  }
  return warp_sum(a);
}

}  // namespace qb
