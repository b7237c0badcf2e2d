// Batched decode engine: sequences 0 .. nb-1 (nb <= BATCH_MAX) step together,
// each with its own DeltaNet state, conv history and KV cache
// (golden/model.py:86-107, one DecodeState per sequence; decode_step
// golden/model.py:243-267 applied to each).
//
// Per step (one CUDA graph):
//   normq      per token: (1+w) RMSNorm in numpy's pairwise order
//              (golden/model.py:63-75) and the projection input's image --
//              W8A8: the golden per-vector int8 quantiser (golden/model.py:37-45);
//              W8A32: a 23-bit fixed-point image split into three signed int8
//              digit planes; DeltaNet layers also take in_proj_a / in_proj_b
//              (fp32 rows) here.
//   gemm       tcgen05.mma kind::i8, M = 128 weight rows per CTA tile, N = 64
//              tokens x digit planes, K streamed in 128-byte slabs (16 KB of
//              weights + the image slab per stage, cp.async.bulk into a
//              4-stage ring), int32 accumulators in TMEM; optional split-K
//              over CTAs with exact int32 reductions; epilogue: dequant
//              acc * s_x[b] * s_w[row], then store, residual add, or SwiGLU.
//   delta      per (token, DeltaNet head): conv + SiLU, l2norm, gates, the
//              delta rule on the sequence's state, gated RMSNorm
//              (golden/model.py:149-189).
//   attn       split-KV flash-decoding items (token, KV group, 256-position
//              chunk): QK RMSNorm + partial RoPE, cached K / V blocks staged
//              by bulk copies, online softmax, (m, l, o) partials
//              (golden/model.py:194-229); merge + output gate + quantiser per
//              token.
//   quant      per token: the quantiser of an out_proj / o_proj / down_proj input.
//   head       persistent tcgen05 kernel over the tied embedding tiles
//              (N = 64 tokens x 3 digit planes of the final-normed h, held in
//              shared memory), logits, per-token argmax (first index on ties).
//   finish     per token: argmax over CTAs -> ids and the next token.
//
// Every device wait is bounded (2 s) and reports ERR_WAIT; no multicast form
// of any copy is used.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/qwen_b200.h"
#include "batch.cuh"
#include "common.cuh"
#include "tc.cuh"

namespace qb {

namespace {

// ---------------------------------------------------------------- shared helpers

constexpr int NT = 512;   // threads of the per-token kernels
constexpr int NW = NT / 32;

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Fixed-point shift of a vector whose exact max|x| is amax: X = rint(x 2^sh)
// with |X| <= 2^22 (amax in [2^(ex-1), 2^ex) -> sh = 22 - ex).
struct Fix {
  int sh;
  float p2;     // 2^sh when `fast`
  bool fast, live;
};
__device__ __forceinline__ Fix fix_of(float amax) {
  Fix f;
  f.live = amax > 0.0f;
  const unsigned eb = (__float_as_uint(amax) >> 23) & 0xffu;
  f.sh = 22 - ((int)eb - 126);
  f.fast = f.live && eb != 0u && f.sh >= -126 && f.sh <= 127;
  if (f.live && !f.fast) {
    int ex = 0;
    frexpf(amax, &ex);
    f.sh = 22 - ex;
  }
  f.p2 = f.fast ? pow2f(f.sh) : 0.0f;
  return f;
}
__device__ __forceinline__ int fix_val(float v, const Fix& f) {
  if (!f.live) return 0;
  return f.fast ? __float2int_rn(v * f.p2) : (int)rintf(ldexpf(v, f.sh));
}
// X = d0 + 256 d1 + 65536 d2 with d0, d1 in [-128, 127], |d2| <= 64
__device__ __forceinline__ void digits3(int X, int& d0, int& d1, int& d2) {
  d0 = (X << 24) >> 24;
  const int X1 = (X - d0) >> 8;
  d1 = (X1 << 24) >> 24;
  d2 = (X1 - d1) >> 8;
}
// golden _qa: q = clip(rint(x / s), -127, 127) (golden/model.py:37-45)
__device__ __forceinline__ int q8(float x, float s, bool live) {
  if (!live) return 0;
  return (int)fminf(fmaxf(rintf(__fdiv_rn(x, s)), -127.0f), 127.0f);
}

// max over the block's 512 threads (red: >= NW floats); every thread gets it
__device__ __forceinline__ float amax512(float m, float* red) {
  m = warp_max(m);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float a = 0.0f;
#pragma unroll
  for (int w = 0; w < NW; ++w) a = fmaxf(a, red[w]);
  return a;
}

// Write E (2 or 4) consecutive elements k0 .. of token b into the image:
// W8A8 (NPL 1) the int8 codes, W8A32 (NPL 3) the three digit planes.  The
// scale (s_x or 2^-sh) goes to xs[b] from thread 0.  xfq (nullable) gets the
// values the fp32 rows multiply (W8A8: the fake-quantised x, golden
// _qa; W8A32: x).
template <int NPL, int E>
__device__ __forceinline__ void image_store(const float (&x)[E], int k0, int b, float amax, int8_t* X, float* xs,
                                            float (*xfq)[E]) {
  static_assert(E == 2 || E == 4, "group");
  constexpr int NR = 64 * NPL;
  if constexpr (NPL == 1) {
    const bool live = amax > 0.0f;
    const float s = live ? __fdiv_rn(amax, 127.0f) : 1.0f;
    unsigned w = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int q = q8(x[e], s, live);
      w |= ((unsigned)q & 0xffu) << (8 * e);
      if (xfq) (*xfq)[e] = live ? __fmul_rn((float)q, s) : 0.0f;
    }
    int8_t* dst = X + img_off(b, k0, NR);
    if constexpr (E == 2) *reinterpret_cast<unsigned short*>(dst) = (unsigned short)w;
    else *reinterpret_cast<unsigned*>(dst) = w;
    if (threadIdx.x == 0) xs[b] = s;
  } else {
    const Fix f = fix_of(amax);
    unsigned w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      int d0, d1, d2;
      digits3(fix_val(x[e], f), d0, d1, d2);
      w0 |= ((unsigned)d0 & 0xffu) << (8 * e);
      w1 |= ((unsigned)d1 & 0xffu) << (8 * e);
      w2 |= ((unsigned)d2 & 0xffu) << (8 * e);
      if (xfq) (*xfq)[e] = x[e];
    }
    int8_t* p0 = X + img_off(b, k0, NR);
    int8_t* p1 = X + img_off(64 + b, k0, NR);
    int8_t* p2 = X + img_off(128 + b, k0, NR);
    if constexpr (E == 2) {
      *reinterpret_cast<unsigned short*>(p0) = (unsigned short)w0;
      *reinterpret_cast<unsigned short*>(p1) = (unsigned short)w1;
      *reinterpret_cast<unsigned short*>(p2) = (unsigned short)w2;
    } else {
      *reinterpret_cast<unsigned*>(p0) = w0;
      *reinterpret_cast<unsigned*>(p1) = w1;
      *reinterpret_cast<unsigned*>(p2) = w2;
    }
    if (threadIdx.x == 0) xs[b] = f.live ? ldexpf(1.0f, -f.sh) : 0.0f;
  }
}

// ---------------------------------------------------------------- control block

// Per-step values the kernels read (copied from the host before each step).
struct BtCtl {
  int pos[BATCH_MAX];     // RoPE position of the token being decoded
  int T[BATCH_MAX];       // cached positions before this token
  int cbase[BATCH_MAX];   // conv ring origin
  int nb;                 // sequences stepped
  int want_logits;
  int nchmax;             // attention chunks of the longest sequence
  int pad;
};

constexpr int AT_CL = 256;   // positions per attention chunk
constexpr int BT_HEAD_TILES = VOCAB / GT_M;            // tied head tiles (1940)
constexpr int BT_MAXTILES = (CONVD + VDIM) / GT_M;   // most tiles of one layer projection (64)
static_assert(2 * FFN / GT_M <= BT_MAXTILES && (QPROJ + 2 * KVPROJ) / GT_M <= BT_MAXTILES, "split-K scratch");

// ---------------------------------------------------------------- repack

__global__ void k_bt_repack(const int8_t* const* __restrict__ rowptr, int4* __restrict__ out, int nrows, int K) {
  const int nslab = K / GT_KS;
  const size_t total = (size_t)nrows * K / 16;
  for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < total; u += (size_t)gridDim.x * blockDim.x) {
    const size_t slab = u >> 10;   // 1024 16-byte units per slab
    const int w = (int)(u & 1023);
    const int tile = (int)(slab / nslab), j = (int)(slab % nslab);
    const int core = w >> 3;
    const int m = ((core >> 3) << 3) + (w & 7), kc = core & 7;
    out[u] = *reinterpret_cast<const int4*>(rowptr[(size_t)tile * GT_M + m] + (size_t)j * GT_KS + kc * 16);
  }
}

// row-major xq [B][K] -> image of 64 rows (rows >= B zero)
__global__ void k_bt_image(const int8_t* __restrict__ xq, int8_t* __restrict__ X, int B, int K) {
  const int units = K / 16;
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < 64 * units; u += gridDim.x * blockDim.x) {
    const int b = u / units, k = (u % units) * 16;
    int4 v = make_int4(0, 0, 0, 0);
    if (b < B) v = *reinterpret_cast<const int4*>(xq + (size_t)b * K + k);
    *reinterpret_cast<int4*>(X + img_off(b, k, 64)) = v;
  }
}

// ---------------------------------------------------------------- GEMM

enum { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

struct GemmArgs {
  const int8_t* W;     // tiles [ntiles][nslab][16 KB]
  const float* sw;     // per row, tile order
  const int8_t* X;     // image [nslab][64 NPL][128]
  const float* xs;     // per token
  int nslab, kspl;     // slabs of K; slabs per CTA (grid.y = ceil(nslab / kspl))
  int nb;              // live tokens
  int mode;
  float* Y;            // STORE / ADD: Y[b ldy + row]; SWIGLU: Y[b ldy + 64 tile + r]
  int ldy;
  int32_t* part;       // split-K sums [ntiles][64 NPL][128], zero between uses
  int* cnt;            // [ntiles] arrival counters, zero between uses
  int32_t* acc_out;    // nullable (NPL 1): acc[b nrows + row]
  int nrows;
  int* err;
};

template <int NPL>
struct GC {
  static constexpr int NR = 64 * NPL;
  static constexpr int BBYTES = NR * GT_KS;
  static constexpr int STAGE = GT_SLAB + BBYTES;
  static constexpr int NST = 4;
  static constexpr int OFF_BAR = NST * STAGE;
  static constexpr int SMEM = OFF_BAR + 128;   // barriers, TMEM slot, flags
  static constexpr int TCOLS = NPL == 1 ? 64 : 256;
  static constexpr unsigned IDESC = tc::idesc_i8(GT_M, NR);
};

template <int NPL>
__global__ void __launch_bounds__(128) k_bt_gemm(const GemmArgs a) {
  using C = GC<NPL>;
  extern __shared__ __align__(1024) unsigned char sm[];
  const int t = threadIdx.x, wid = t >> 5, lane = t & 31;
  const int tile = blockIdx.x;
  const int j0 = blockIdx.y * a.kspl, j1 = min(a.nslab, j0 + a.kspl), ns = j1 - j0;
  const unsigned bar0 = tc::smem_u32(sm + C::OFF_BAR);
  const unsigned accf = bar0 + 16u * C::NST;
  unsigned* tslot = reinterpret_cast<unsigned*>(sm + C::OFF_BAR + 16 * C::NST + 8);
  int* flag = reinterpret_cast<int*>(tslot + 1);
  if (t == 0) {
    for (int s = 0; s < C::NST; ++s) {
      tc::mbar_init(bar0 + 8u * s, 1);                 // full
      tc::mbar_init(bar0 + 8u * (C::NST + s), 1);      // empty
    }
    tc::mbar_init(accf, 1);
    tc::mbar_init_fence();
    flag[0] = 0;
  }
  tc::grid_wait();
  if (wid == 0) tc::tmem_alloc<C::TCOLS>(tslot);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const unsigned tmem = *tslot;
  int issued = 0, consumed = 0;
  if (t == 0) {
    // producer: weights (read once: evict first) and the image slab (shared by every tile)
    const unsigned long long pw = tc::policy_evict_first(), px = tc::policy_evict_last();
    for (int i = 0; i < ns; ++i) {
      const int s = i % C::NST;
      if (i >= C::NST && !tc::mbar_wait(bar0 + 8u * (C::NST + s), (unsigned)(((i / C::NST) - 1) & 1), a.err, 40, i))
        break;
      const unsigned dst = tc::smem_u32(sm + s * C::STAGE);
      const unsigned fb = bar0 + 8u * s;
      tc::mbar_expect(fb, (unsigned)C::STAGE);
      tc::bulk_g2s(dst, a.W + ((size_t)tile * a.nslab + j0 + i) * GT_SLAB, GT_SLAB, fb, pw);
      tc::bulk_g2s(dst + GT_SLAB, a.X + (size_t)(j0 + i) * C::BBYTES, C::BBYTES, fb, px);
      issued = i + 1;
    }
  } else if (t == 32) {
    // MMA issuer
    for (int i = 0; i < ns; ++i) {
      const int s = i % C::NST;
      if (!tc::mbar_wait(bar0 + 8u * s, (unsigned)((i / C::NST) & 1), a.err, 41, i)) break;
      tc::fence_after();
      const unsigned sa = tc::smem_u32(sm + s * C::STAGE);
      const unsigned long long da = tc::desc(sa, 128u, 1024u), db = tc::desc(sa + GT_SLAB, 128u, 1024u);
#pragma unroll
      for (int kk = 0; kk < GT_KS / 32; ++kk)
        tc::mma_i8(tmem, da + 16ull * kk, db + 16ull * kk, C::IDESC, (unsigned)((i | kk) != 0));
      tc::commit(bar0 + 8u * (C::NST + s));
      consumed = i + 1;
    }
    tc::commit(accf);
  }
  if (t == 0) flag[1] = issued;
  if (t == 32) flag[2] = consumed;
  __syncwarp();
  const bool got = tc::mbar_wait(accf, 0u, a.err, 42, tile);
  const bool ok = __syncthreads_and(got) && flag[2] == ns && flag[1] == ns;
  const int row = 32 * wid + lane;                       // TMEM lane = tile row
  const unsigned taddr = tmem + ((unsigned)(32 * wid) << 16);
  bool last = true;
  if (ok && gridDim.y > 1) {
    // split K: add this CTA's sums into the tile's exact int32 totals; the
    // last CTA to arrive finishes the tile
    tc::fence_after();
    int32_t* P = a.part + (size_t)tile * C::NR * 128;
    for (int c0 = 0; c0 < C::NR; c0 += 16) {
      unsigned r[16];
      tc::tmem_ld16(taddr + c0, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) atomicAdd(P + (size_t)(c0 + e) * 128 + row, (int)r[e]);
    }
    __threadfence();
    __syncthreads();
    if (t == 0) flag[0] = atomicAdd(a.cnt + tile, 1) == (int)gridDim.y - 1;
    __syncthreads();
    last = flag[0] != 0;
    if (last) __threadfence();
  }
  if (ok && last) {
    tc::fence_after();
    const bool split = gridDim.y > 1;
    int32_t* P = a.part + (size_t)tile * C::NR * 128;
    const int grow = tile * GT_M + row;
    const float sw = a.sw[grow];
    float* ub = reinterpret_cast<float*>(sm);   // SWIGLU: up rows [64 tokens][64]
    for (int c0 = 0; c0 < 64; c0 += 16) {
      unsigned r[NPL][16];
#pragma unroll
      for (int p = 0; p < NPL; ++p) {
        if (split) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            int32_t* q = P + (size_t)(64 * p + c0 + e) * 128 + row;
            r[p][e] = (unsigned)__ldcg(q);
            *q = 0;
          }
        } else {
          tc::tmem_ld16(taddr + 64 * p + c0, r[p]);
        }
      }
      if (!split) tc::tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int b = c0 + e;
        float y;
        if constexpr (NPL == 1) {
          y = (float)(int)r[0][e] * (a.xs[b] * sw);
          if (a.acc_out && b < a.nb && grow < a.nrows) a.acc_out[(size_t)b * a.nrows + grow] = (int)r[0][e];
        } else {
          const long long X = (long long)(int)r[0][e] + 256ll * (int)r[1][e] + 65536ll * (int)r[2][e];
          y = (float)((double)X * (double)(a.xs[b] * sw));
        }
        if (b >= a.nb) continue;
        if (a.mode == EPI_STORE) {
          if (grow < a.nrows) a.Y[(size_t)b * a.ldy + grow] = y;
        } else if (a.mode == EPI_ADD) {
          float* h = a.Y + (size_t)b * a.ldy + grow;
          *h = __fadd_rn(*h, y);
        } else if (row >= 64) {
          ub[b * 64 + row - 64] = y;   // up row
        } else {
          r[0][e] = __float_as_uint(y);   // gate row, kept for the SwiGLU below
        }
      }
      if (a.mode == EPI_SWIGLU) {
        __syncthreads();
        if (row < 64) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int b = c0 + e;
            if (b < a.nb)
              a.Y[(size_t)b * a.ldy + 64 * tile + row] = __fmul_rn(silu_f(__uint_as_float(r[0][e])), ub[b * 64 + row]);
          }
        }
        __syncthreads();
      }
    }
    if (split && t == 0) a.cnt[tile] = 0;
  }
  // teardown: copies that were issued but never consumed (only after a wait
  // ran out) are waited for, with the same bound, before the CTA exits
  if (t == 0 && flag[2] < flag[1]) {
    for (int i = flag[2]; i < flag[1]; ++i)
      if (!tc::mbar_wait(bar0 + 8u * (i % C::NST), (unsigned)((i / C::NST) & 1), a.err, 43, i)) break;
  }
  tc::fence_before();
  __syncthreads();
  if (wid == 0) {
    tc::fence_after();
    tc::tmem_free<C::TCOLS>(tmem);
  }
}

// ---------------------------------------------------------------- norm + image

struct NormqArgs {
  float* H;                  // [64][HID] residual stream
  const int* tok;            // layer 0: the tokens (H is written from the embedding)
  const int8_t* emb_q; const float* emb_s;
  const float* gain;         // RMSNorm offsets w: x (1 + w)
  const float* a_w; const float* b_w;   // DeltaNet layer: [16][HID] fp32 rows (else null)
  float* AB;                 // [64][32]: b rows, then a rows
  int8_t* X; float* xs;
  int* err;
};

// One token per CTA, elements 2t, 2t + 1 per thread.
template <int NPL>
__global__ void __launch_bounds__(NT) k_bt_normq(const NormqArgs a) {
  __shared__ float hs[HID];
  __shared__ float red[2 * NW];
  __shared__ float rab[32][NW];
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, wid = t >> 5;
  tc::grid_wait();
  float* hrow = a.H + (size_t)b * HID;
  float2 h2;
  if (a.tok) {
    // the residual stream starts at the dequantised embedding row (golden/model.py:246)
    int tok = a.tok[b];
    if (tok < 0 || tok >= VOCAB) {
      if (t == 0) atomicCAS(a.err, 0, ERR_TOKEN);
      tok = 0;
    }
    const float sc = a.emb_s[tok];
    const int8_t* er = a.emb_q + (size_t)tok * HID;
    h2 = make_float2(__fmul_rn((float)er[2 * t], sc), __fmul_rn((float)er[2 * t + 1], sc));
    *reinterpret_cast<float2*>(hrow + 2 * t) = h2;
  } else {
    h2 = *reinterpret_cast<const float2*>(hrow + 2 * t);
  }
  *reinterpret_cast<float2*>(hs + 2 * t) = h2;
  const float2 g2 = *reinterpret_cast<const float2*>(a.gain + 2 * t);
  __syncthreads();
  // sum of squares in numpy's pairwise order (np.mean(x**2), golden/model.py:74):
  // 8 blocks of 128, each 8 interleaved accumulators of 16 terms, combined
  // ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the blocks as a binary tree
  if (wid < 2) {
    const int ch = lane + 32 * wid;
    const float* p = hs + 128 * (ch >> 3) + (ch & 7);
    float acc = __fmul_rn(p[0], p[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) acc = __fadd_rn(acc, __fmul_rn(p[8 * i], p[8 * i]));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 16));
    if (lane == 0) red[NW + wid] = acc;
  }
  __syncthreads();
  const float tot = __fadd_rn(red[NW], red[NW + 1]);
  // 1 / sqrt(mean + eps): HID is a power of two (the product by 1/HID is the
  // quotient), the reciprocal correctly rounded like numpy's 1.0 / np.sqrt
  const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / HID), EPS)));
  float x[2];
  x[0] = __fmul_rn(__fmul_rn(h2.x, inv), __fadd_rn(1.0f, g2.x));
  x[1] = __fmul_rn(__fmul_rn(h2.y, inv), __fadd_rn(1.0f, g2.y));
  const float amax = amax512(fmaxf(fabsf(x[0]), fabsf(x[1])), red);
  float xf[2];
  image_store<NPL, 2>(x, 2 * t, b, amax, a.X, a.xs, &xf);
  if (a.a_w) {
    // b = in_proj_b . x, a = in_proj_a . x (golden/model.py:146-147; x the
    // fake-quantised input under W8A8), per head: pair products, warp sums,
    // then the warps in order
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
      const float* wr = (r < 16 ? a.b_w + (size_t)r * HID : a.a_w + (size_t)(r - 16) * HID) + 2 * t;
      const float2 w = __ldg(reinterpret_cast<const float2*>(wr));
      const float p = warp_sum(fmaf(w.y, xf[1], __fmul_rn(w.x, xf[0])));
      if (lane == 0) rab[r][wid] = p;
    }
    __syncthreads();
    if (t < 32) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += rab[t][w];
      a.AB[b * 32 + t] = s;
    }
  }
}

// Quantiser of a K-vector per token (K a multiple of 4, <= 4096): src[b lds + k].
template <int NPL>
__global__ void __launch_bounds__(NT) k_bt_quant(const float* __restrict__ src, int lds, int K, int8_t* X, float* xs) {
  __shared__ float red[NW];
  const int b = blockIdx.x, t = threadIdx.x;
  tc::grid_wait();
  const float* s = src + (size_t)b * lds;
  float v[2][4];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int g = t + NT * j;
    if (4 * g < K) {
      const float4 q = *reinterpret_cast<const float4*>(s + 4 * g);
      v[j][0] = q.x; v[j][1] = q.y; v[j][2] = q.z; v[j][3] = q.w;
      m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
    }
  }
  const float amax = amax512(m, red);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int g = t + NT * j;
    if (4 * g < K) image_store<NPL, 4>(v[j], 4 * g, b, amax, X, xs, nullptr);
  }
}

// ---------------------------------------------------------------- DeltaNet mixer

struct DeltaArgs {
  const float* Y; int ldy;     // in-proj outputs: qkv [0, 6144), z [6144, 8192)
  const float* AB;             // [64][32]
  float* conv; float* rec;     // sequence 0's arrays; sequence b at + b * conv_seq / rec_seq
  size_t conv_seq, rec_seq;
  int lin;
  const float* conv_w; const float* A_log; const float* dt_bias; const float* gnorm_w;
  const BtCtl* ctl;
  float* O;                    // [64][VDIM] gated-normed output
};

// One (head, token) per CTA, 512 threads: 0..127 q channels, 128..255 k,
// 256..383 v, 384 the gates; the delta rule maps thread t to value column
// t % 128 and state rows 32 (t / 128) .. +31 (golden/model.py:149-189).
__global__ void __launch_bounds__(NT) k_bt_delta(const DeltaArgs a) {
  __shared__ float qs[LK], ks[LK], vs[LV], wsq[16], ob[LV];
  __shared__ float part[4][LV];
  __shared__ float gbeta, gg, ginv;
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  constexpr int KPG = LK / 4;
  tc::grid_wait();
  const float* y = a.Y + (size_t)b * a.ldy;
  float* cs = a.conv + (size_t)b * a.conv_seq + (size_t)a.lin * CONVD * CONVK;
  float* Sh = a.rec + (size_t)b * a.rec_seq + ((size_t)a.lin * LH + h) * LK * LV;
  const int base = a.ctl->cbase[b];
  const int vi = t & (LV - 1), kg = t / LV;
  float sv[KPG];
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) sv[kk] = Sh[(size_t)(kg * KPG + kk) * LV + vi];
  const int role = (t < 2 * LK) ? 0 : (t < 2 * LK + LV ? 1 : (t == 2 * LK + LV ? 2 : 3));
  int ch = 0;
  if (role == 0) ch = (t < LK) ? (h * LK + t) : (KDIM + h * LK + (t - LK));
  else if (role == 1) ch = 2 * KDIM + h * LV + (t - 2 * LK);
  float x = 0.0f;
  if (role <= 1) {
    // causal conv over [conv1, conv2, conv3, new] (golden/model.py:154-158); the
    // oldest column's slot takes the new value
    float* st = cs + (size_t)ch * CONVK;
    const float s1 = st[(base + 1) & 3], s2 = st[(base + 2) & 3], s3 = st[(base + 3) & 3];
    const float4 w4 = *reinterpret_cast<const float4*>(a.conv_w + (size_t)ch * CONVK);
    const float nv = y[ch];
    float acc = __fmul_rn(s1, w4.x);
    acc = __fadd_rn(acc, __fmul_rn(s2, w4.y));
    acc = __fadd_rn(acc, __fmul_rn(s3, w4.z));
    acc = __fadd_rn(acc, __fmul_rn(nv, w4.w));
    x = silu_f(acc);
    st[base & 3] = nv;
    if (role == 1) vs[t - 2 * LK] = x;
  } else if (role == 2) {
    gbeta = sigmoid_f(a.AB[b * 32 + h]);
    gg = __fmul_rn(-expf(a.A_log[h]), softplus_f(__fadd_rn(a.AB[b * 32 + 16 + h], a.dt_bias[h])));
  }
  // l2norm of q (warps 0-3) and k (warps 4-7); q scaled by 128^-0.5 after it
  const float ss = warp_sum(role == 0 ? x * x : 0.0f);
  if ((t & 31) == 0) wsq[t >> 5] = ss;
  __syncthreads();
  if (role == 0) {
    const int g0 = (t < LK) ? 0 : 4;
    const float tot = ((wsq[g0] + wsq[g0 + 1]) + wsq[g0 + 2]) + wsq[g0 + 3];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(tot, EPS)));
    if (t < LK) qs[t] = __fmul_rn(__fmul_rn(x, inv), 0.08838834764831845f);
    else ks[t - LK] = __fmul_rn(x, inv);
  }
  __syncthreads();
  // S *= exp(g); kv = k^T S; d = (v - kv) beta; S += k (x) d; o = q^T S
  const float gexp = expf(gg);
  float pkv = 0.0f;
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) {
    sv[kk] = __fmul_rn(sv[kk], gexp);
    pkv = fmaf(sv[kk], ks[kg * KPG + kk], pkv);
  }
  part[kg][vi] = pkv;
  __syncthreads();
  float kvv = 0.0f;
#pragma unroll
  for (int g = 0; g < 4; ++g) kvv += part[g][vi];
  const float delta = __fmul_rn(__fsub_rn(vs[vi], kvv), gbeta);
  __syncthreads();
  float po = 0.0f;
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) {
    const int k = kg * KPG + kk;
    const float s2v = __fadd_rn(sv[kk], __fmul_rn(ks[k], delta));
    Sh[(size_t)k * LV + vi] = s2v;
    po = fmaf(s2v, qs[k], po);
  }
  part[kg][vi] = po;
  __syncthreads();
  if (t < LV) {
    float o = 0.0f;
#pragma unroll
    for (int g = 0; g < 4; ++g) o += part[g][t];
    ob[t] = o;
  }
  __syncthreads();
  // gated RMSNorm (golden/model.py:183-189): o / rms(o) * w * silu(z)
  if (t < 32) {
    float s = 0.0f;
    for (int i = t; i < LV; i += 32) s = fmaf(ob[i], ob[i], s);
    s = warp_sum(s);
    if (t == 0) ginv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(s, 1.0f / LV), EPS)));
  }
  __syncthreads();
  if (t < LV) {
    const float z = silu_f(y[CONVD + h * LV + t]);
    const float v = __fmul_rn(__fmul_rn(ob[t], ginv), a.gnorm_w[t]);
    a.O[(size_t)b * VDIM + h * LV + t] = __fmul_rn(v, z);
  }
}

// ---------------------------------------------------------------- attention

constexpr int AT_BLK = 16;                       // positions per staged block
constexpr int AT_NST = 3;                        // staged blocks in flight
constexpr int AT_KROW = HD * 4 + 16;             // padded K row in shared memory (bytes)
constexpr int AT_KB = AT_BLK * AT_KROW;
constexpr int AT_VB = AT_BLK * HD * 4;
constexpr int AT_STAGE = AT_KB + AT_VB;
constexpr int AT_OFF_Q = AT_NST * AT_STAGE;      // qn [4][256]
constexpr int AT_OFF_KN = AT_OFF_Q + 4 * HD * 4; // kn [256]
constexpr int AT_OFF_VN = AT_OFF_KN + HD * 4;    // vn [256]
constexpr int AT_OFF_PART = AT_OFF_VN + HD * 4;  // partial scores [4 quarters][4 heads][16]
constexpr int AT_OFF_SP = AT_OFF_PART + 4 * 4 * AT_BLK * 4;   // probabilities [4][16]
constexpr int AT_OFF_ST = AT_OFF_SP + 4 * AT_BLK * 4;         // m[4], l[4], scale[4]
constexpr int AT_OFF_BAR = AT_OFF_ST + 64;
constexpr int AT_SMEM = AT_OFF_BAR + 8 * AT_NST;
constexpr int AT_PROW = 4 + HD;                  // partial row: m, l, 2 pad, o[256]
static_assert(AT_STAGE % 16 == 0 && AT_KROW % 16 == 0 && AT_OFF_BAR % 8 == 0, "attention smem alignment");

struct AttnArgs {
  const float* Y; int ldy;     // in-proj outputs: [q | gate] per head (4096), k (512), v (512)
  float* kc; float* vc;        // [B][6][NKV][max_ctx][HD]
  int fi, max_ctx;
  const float* qn_w; const float* kn_w; const float* rope;
  const BtCtl* ctl;
  float* part;                 // [B][NKV][maxch][4][AT_PROW]
  int maxch;
  int* err;
};

// QK RMSNorm (1 + w) and partial RoPE of one 256-vector (elements lane + 32 q), by one warp
__device__ __forceinline__ void norm_rope_warp(const float* src, const float* w, float co, float si, float* dst) {
  const int lane = threadIdx.x & 31;
  float v[8];
  float ss = 0.0f;
#pragma unroll
  for (int q = 0; q < 8; ++q) { v[q] = src[lane + 32 * q]; ss = fmaf(v[q], v[q], ss); }
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), EPS)));
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = __fmul_rn(__fmul_rn(v[q], inv), __fadd_rn(1.0f, w[lane + 32 * q]));
  // rotate_half on the first 64 dims: (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin)
  const float x1 = v[0], x2 = v[1];
  v[0] = __fadd_rn(__fmul_rn(x1, co), __fmul_rn(-x2, si));
  v[1] = __fadd_rn(__fmul_rn(x2, co), __fmul_rn(x1, si));
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[lane + 32 * q] = v[q];
}

// Persistent over items (token b, group g, chunk cc); 256 threads.
__global__ void __launch_bounds__(256, 2) k_bt_attn(const AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* qn = reinterpret_cast<float*>(sm + AT_OFF_Q);
  float* kn = reinterpret_cast<float*>(sm + AT_OFF_KN);
  float* vn = reinterpret_cast<float*>(sm + AT_OFF_VN);
  float* part = reinterpret_cast<float*>(sm + AT_OFF_PART);
  float* sp = reinterpret_cast<float*>(sm + AT_OFF_SP);
  float* st = reinterpret_cast<float*>(sm + AT_OFF_ST);
  const unsigned bar0 = tc::smem_u32(sm + AT_OFF_BAR);
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  if (t == 0) {
    for (int s = 0; s < AT_NST; ++s) tc::mbar_init(bar0 + 8u * s, 1);
    tc::mbar_init_fence();
  }
  tc::grid_wait();
  __syncthreads();
  const BtCtl& C = *a.ctl;
  const int nchm = C.nchmax, nitems = C.nb * NKV * nchm;
  const unsigned long long pol = tc::policy_evict_first();
  unsigned nblk_done = 0;   // blocks this CTA consumed so far (stage / parity bookkeeping)
  unsigned nissued = 0, nfail = 0;   // blocks staged so far (warp 0's count); the block whose wait failed
  bool good = true;
  for (int item = blockIdx.x; item < nitems && good; item += gridDim.x) {
    const int cc = item % nchm, g = (item / nchm) % NKV, b = item / (nchm * NKV);
    const int T = C.T[b], pos = C.pos[b], Tn = T + 1;
    const int t0 = cc * AT_CL;
    if (t0 >= Tn) continue;
    const int t1 = min(Tn, t0 + AT_CL), tcache = min(t1, T);
    const int nblk = (t1 - t0 + AT_BLK - 1) / AT_BLK;
    const size_t kvoff = (((size_t)b * NFULL + a.fi) * NKV + g) * (size_t)a.max_ctx * HD;
    const float* kc = a.kc + kvoff;
    const float* vc = a.vc + kvoff;
    // stage the cached rows of block i (warp 0: lane 0 arms the barrier, lanes
    // 0-15 copy one K row each into the padded layout, lane 16 the V rows)
    auto issue = [&](int i) {
      const unsigned n = nblk_done + (unsigned)i, s = n % AT_NST;
      const int s0 = t0 + i * AT_BLK;
      const int nbc = max(0, min(AT_BLK, tcache - s0));
      const unsigned kb = tc::smem_u32(sm + s * AT_STAGE), vb = kb + AT_KB, bar = bar0 + 8u * s;
      if (lane == 0) tc::mbar_expect(bar, (unsigned)(2 * nbc * HD * 4));
      __syncwarp();
      if (lane < nbc) tc::bulk_g2s(kb + lane * AT_KROW, kc + (size_t)(s0 + lane) * HD, HD * 4, bar, pol);
      if (lane == 16 && nbc > 0) tc::bulk_g2s(vb, vc + (size_t)s0 * HD, (unsigned)(nbc * HD * 4), bar, pol);
      nissued = n + 1;
    };
    if (wid == 0) {
      tc::fence_async_smem();
      for (int i = 0; i < AT_NST && i < nblk; ++i) issue(i);
    }
    // this token's q (4 heads of group g), k and v: RMSNorm + RoPE (golden/model.py:203-214)
    const float* y = a.Y + (size_t)b * a.ldy;
    const float* rope = a.rope + (size_t)pos * ROT;
    if (wid < 4) norm_rope_warp(y + (4 * g + wid) * 2 * HD, a.qn_w, rope[lane], rope[32 + lane], qn + wid * HD);
    else if (wid == 4) norm_rope_warp(y + QPROJ + g * HD, a.kn_w, rope[lane], rope[32 + lane], kn);
    else if (wid == 5) for (int e = lane; e < HD; e += 32) vn[e] = y[QPROJ + KVPROJ + g * HD + e];
    if (t < 4) { st[t] = -INFINITY; st[4 + t] = 0.0f; }
    __syncthreads();
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    const int p = t & 15, hq = (t >> 4) & 3, qd = t >> 6;
    for (int i = 0; i < nblk; ++i) {
      const unsigned n = nblk_done + (unsigned)i, s = n % AT_NST;
      if (!tc::mbar_wait(bar0 + 8u * s, (n / AT_NST) & 1u, a.err, 50, item)) good = false;
      if (__syncthreads_or(!good)) {
        good = false;
        nfail = n;
        break;
      }
      const int s0 = t0 + i * AT_BLK;
      const int nbk = min(AT_BLK, t1 - s0), nbc = max(0, min(AT_BLK, tcache - s0));
      unsigned char* kb = sm + s * AT_STAGE;
      float* vb = reinterpret_cast<float*>(kb + AT_KB);
      if (nbk > nbc) {
        // this block holds the new token (position T) at row nbc
        reinterpret_cast<float*>(kb + nbc * AT_KROW)[t] = kn[t];
        vb[nbc * HD + t] = vn[t];
        __syncthreads();
      }
      // scores: thread = (position p, head hq, quarter qd of the 256 dims)
      if (p < nbk) {
        const float4* kr = reinterpret_cast<const float4*>(kb + p * AT_KROW) + qd * 16;
        const float4* qr = reinterpret_cast<const float4*>(qn + hq * HD) + qd * 16;
        float d = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float4 kv = kr[j], qv = qr[j];
          d = fmaf(qv.x, kv.x, d);
          d = fmaf(qv.y, kv.y, d);
          d = fmaf(qv.z, kv.z, d);
          d = fmaf(qv.w, kv.w, d);
        }
        part[(qd * 4 + hq) * AT_BLK + p] = d;
      }
      __syncthreads();
      // online softmax: warp hq < 4 updates head hq (scale 256^-0.5 = 1/16, exact)
      if (wid < 4) {
        const int h4 = wid;
        float sv = -INFINITY;
        if (lane < nbk)
          sv = __fmul_rn(((part[(0 * 4 + h4) * AT_BLK + lane] + part[(1 * 4 + h4) * AT_BLK + lane]) +
                          part[(2 * 4 + h4) * AT_BLK + lane]) + part[(3 * 4 + h4) * AT_BLK + lane], 0.0625f);
        const float mold = st[h4];
        const float mnew = fmaxf(mold, warp_max(sv));
        const float pe = lane < nbk ? expf(sv - mnew) : 0.0f;
        const float ls = warp_sum(pe);
        if (lane < AT_BLK) sp[h4 * AT_BLK + lane] = pe;
        if (lane == 0) {
          const float sc = mold == -INFINITY ? 0.0f : expf(mold - mnew);
          st[8 + h4] = sc;
          st[4 + h4] = fmaf(st[4 + h4], sc, ls);
          st[h4] = mnew;
        }
      }
      __syncthreads();
      // P V: thread = dim t
#pragma unroll
      for (int h4 = 0; h4 < 4; ++h4) o[h4] = __fmul_rn(o[h4], st[8 + h4]);
      for (int j = 0; j < nbk; ++j) {
        const float vv = vb[j * HD + t];
#pragma unroll
        for (int h4 = 0; h4 < 4; ++h4) o[h4] = fmaf(sp[h4 * AT_BLK + j], vv, o[h4]);
      }
      __syncthreads();   // the stage is free
      if (wid == 0 && i + AT_NST < nblk) {
        tc::fence_async_smem();
        issue(i + AT_NST);
      }
    }
    if (!good) break;
    nblk_done += (unsigned)nblk;
    // the chunk's (m, l, o) of its four heads
    float* pr = a.part + ((((size_t)b * NKV + g) * a.maxch + cc) * 4) * AT_PROW;
#pragma unroll
    for (int h4 = 0; h4 < 4; ++h4) pr[h4 * AT_PROW + 4 + t] = o[h4];
    if (t < 4) {
      pr[t * AT_PROW] = st[t];
      pr[t * AT_PROW + 1] = st[4 + t];
    }
    if (t1 == Tn) {
      // roped K and raw V into slot T (golden/model.py:216-217)
      a.kc[kvoff + (size_t)T * HD + t] = kn[t];
      a.vc[kvoff + (size_t)T * HD + t] = vn[t];
    }
    __syncthreads();
  }
  // after a wait that ran out: the stages still in flight, waited for with the same bound
  if (!good && t == 0) {
    for (unsigned u = nfail; u < nissued; ++u)
      if (!tc::mbar_wait(bar0 + 8u * (u % AT_NST), (u / AT_NST) & 1u, a.err, 51, (int)u)) break;
  }
}

// Merge the chunks of every head of token b (online, in chunk order), times
// sigmoid(gate) (golden/model.py:227-229), then the o_proj input's image.
// Thread = head t / 64, dims 4 (t % 64) .. +3.
template <int NPL>
__global__ void __launch_bounds__(NT) k_bt_merge(const float* __restrict__ Y, int ldy, const float* __restrict__ part,
                                                 int maxch, const BtCtl* ctl, int8_t* X, float* xs) {
  __shared__ float red[NW];
  const int b = blockIdx.x, t = threadIdx.x;
  const int hh = t >> 6, d0 = 4 * (t & 63), g = hh >> 2, hq = hh & 3;
  tc::grid_wait();
  const int nch = (ctl->T[b] + 1 + AT_CL - 1) / AT_CL;
  float M = -INFINITY, Ls = 0.0f, O[4] = {0.f, 0.f, 0.f, 0.f};
  for (int cc = 0; cc < nch; ++cc) {
    const float* pr = part + ((((size_t)b * NKV + g) * maxch + cc) * 4 + hq) * AT_PROW;
    const float mq = pr[0], lq = pr[1];
    const float4 oq = *reinterpret_cast<const float4*>(pr + 4 + d0);
    const float Mn = fmaxf(M, mq);
    const float sa = M == -INFINITY ? 0.0f : expf(M - Mn), sb = expf(mq - Mn);
    Ls = fmaf(lq, sb, __fmul_rn(Ls, sa));
    O[0] = fmaf(oq.x, sb, __fmul_rn(O[0], sa));
    O[1] = fmaf(oq.y, sb, __fmul_rn(O[1], sa));
    O[2] = fmaf(oq.z, sb, __fmul_rn(O[2], sa));
    O[3] = fmaf(oq.w, sb, __fmul_rn(O[3], sa));
    M = Mn;
  }
  const float4 gt = *reinterpret_cast<const float4*>(Y + (size_t)b * ldy + hh * 2 * HD + HD + d0);
  float x[4];
  x[0] = __fmul_rn(__fdiv_rn(O[0], Ls), sigmoid_f(gt.x));
  x[1] = __fmul_rn(__fdiv_rn(O[1], Ls), sigmoid_f(gt.y));
  x[2] = __fmul_rn(__fdiv_rn(O[2], Ls), sigmoid_f(gt.z));
  x[3] = __fmul_rn(__fdiv_rn(O[3], Ls), sigmoid_f(gt.w));
  const float amax = amax512(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))), red);
  image_store<NPL, 4>(x, hh * HD + d0, b, amax, X, xs, nullptr);
}

// ---------------------------------------------------------------- head

constexpr int HB_BBYTES = 3 * 64 * GT_KS;             // one K-slab of the head image (192 rows)
constexpr int HB_NSLAB = HID / GT_KS;                 // 8
constexpr int HB_IMG = HB_NSLAB * HB_BBYTES;          // 192 KB, resident
constexpr int HB_NST = 2;
constexpr int HB_OFF_A = HB_IMG;
constexpr int HB_OFF_BAR = HB_OFF_A + HB_NST * GT_SLAB;
// barriers: full[2], empty[2], image, accf[2], acce[2]; TMEM slot; best[4][64]
constexpr int HB_OFF_SLOT = HB_OFF_BAR + 9 * 8;
constexpr int HB_OFF_BEST = HB_OFF_SLOT + 8;
constexpr int HB_SMEM = HB_OFF_BEST + 4 * 64 * 8;
constexpr int HB_THREADS = 320;   // warps 0-7 epilogue, 8 loads, 9 MMAs
static_assert(HB_SMEM <= 227 * 1024, "head shared memory");
static_assert(HB_OFF_BEST % 8 == 0, "alignment");

struct HeadArgs {
  const int8_t* tiles;      // embed_tokens.weight as tiles (repack_head_tiles)
  const float* emb_s;
  const int8_t* HX;         // the head image [8][192][128]
  const float* hxs;         // per token 2^-sh
  const BtCtl* ctl;
  float* logits;            // [64][VOCAB]
  unsigned long long* am;   // [gridDim.x][64]
  int* err;
};

__global__ void __launch_bounds__(HB_THREADS, 1) k_bt_head(const HeadArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const int t = threadIdx.x, wid = t >> 5, lane = t & 31;
  const unsigned bar0 = tc::smem_u32(sm + HB_OFF_BAR);
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (2 + s); };
  const unsigned bimg = bar0 + 32u;
  auto accf = [&](int s) { return bar0 + 8u * (5 + s); };
  auto acce = [&](int s) { return bar0 + 8u * (7 + s); };
  unsigned* tslot = reinterpret_cast<unsigned*>(sm + HB_OFF_SLOT);
  unsigned long long* bestsm = reinterpret_cast<unsigned long long*>(sm + HB_OFF_BEST);
  if (t == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(full(s), 1);
      tc::mbar_init(empty(s), 1);
      tc::mbar_init(accf(s), 1);
      tc::mbar_init(acce(s), 8);
    }
    tc::mbar_init(bimg, 1);
    tc::mbar_init_fence();
  }
  tc::grid_wait();
  if (wid == 0) tc::tmem_alloc<512>(tslot);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const unsigned tmem = *tslot;
  const int ntl = (BT_HEAD_TILES - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // this CTA's tiles
  constexpr unsigned IDESC = tc::idesc_i8(GT_M, 192);
  int fail = 0;
  if (wid == 8) {
    if (lane == 0) {
      const unsigned long long pw = tc::policy_evict_first(), px = tc::policy_evict_last();
      tc::mbar_expect(bimg, (unsigned)HB_IMG);
      for (int j = 0; j < HB_NSLAB; ++j)
        tc::bulk_g2s(tc::smem_u32(sm + j * HB_BBYTES), a.HX + (size_t)j * HB_BBYTES, HB_BBYTES, bimg, px);
      int n = 0;
      for (int lt = 0; lt < ntl && !fail; ++lt) {
        const int tile = (int)blockIdx.x + lt * (int)gridDim.x;
        for (int j = 0; j < HB_NSLAB; ++j, ++n) {
          const int s = n & 1;
          if (n >= 2 && !tc::mbar_wait(empty(s), (unsigned)(((n >> 1) - 1) & 1), a.err, 60, n)) { fail = 1; break; }
          tc::mbar_expect(full(s), (unsigned)GT_SLAB);
          tc::bulk_g2s(tc::smem_u32(sm + HB_OFF_A + s * GT_SLAB), a.tiles + ((size_t)tile * HB_NSLAB + j) * GT_SLAB,
                       GT_SLAB, full(s), pw);
        }
      }
      // drain: the last two stages' MMAs must be done before the CTA exits
      for (int q = max(0, n - 2); q < n; ++q)
        if (!tc::mbar_wait(empty(q & 1), (unsigned)((q >> 1) & 1), a.err, 61, q)) break;
      if (!tc::mbar_wait(bimg, 0u, a.err, 62, 0)) fail = 1;
    }
    __syncwarp();
  } else if (wid == 9) {
    if (lane == 0) {
      if (!tc::mbar_wait(bimg, 0u, a.err, 63, 0)) fail = 1;
      tc::fence_after();
      const unsigned bimg_a = tc::smem_u32(sm);
      int n = 0;
      for (int lt = 0; lt < ntl && !fail; ++lt) {
        const int bf = lt & 1;
        if (lt >= 2) {
          if (!tc::mbar_wait(acce(bf), (unsigned)(((lt - 2) >> 1) & 1), a.err, 64, lt)) { fail = 1; break; }
          tc::fence_after();
        }
        const unsigned dt = tmem + 256u * bf;
        for (int j = 0; j < HB_NSLAB; ++j, ++n) {
          const int s = n & 1;
          if (!tc::mbar_wait(full(s), (unsigned)((n >> 1) & 1), a.err, 65, n)) { fail = 1; break; }
          tc::fence_after();
          const unsigned long long da = tc::desc(tc::smem_u32(sm + HB_OFF_A + s * GT_SLAB), 128u, 1024u);
          const unsigned long long db = tc::desc(bimg_a + j * HB_BBYTES, 128u, 1024u);
#pragma unroll
          for (int kk = 0; kk < GT_KS / 32; ++kk)
            tc::mma_i8(dt, da + 16ull * kk, db + 16ull * kk, IDESC, (unsigned)((j | kk) != 0));
          tc::commit(empty(s));
        }
        if (fail) break;
        tc::commit(accf(bf));
      }
    }
    __syncwarp();
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. (tile rows) and tokens
    // 32 (w / 4) .. +31; lane i keeps the running best of token 32 (w / 4) + i
    const int q = wid & 3, hf = wid >> 2;
    const int nb = a.ctl->nb;
    const bool want = a.ctl->want_logits != 0;
    const float hx = a.hxs[32 * hf + lane];
    unsigned long long best = 0ull;
    for (int lt = 0; lt < ntl; ++lt) {
      const int bf = lt & 1;
      const int tile = (int)blockIdx.x + lt * (int)gridDim.x;
      if (!tc::mbar_wait(accf(bf), (unsigned)((lt >> 1) & 1), a.err, 66, lt)) fail = 1;
      if (__any_sync(0xffffffffu, fail)) { fail = 1; break; }
      tc::fence_after();
      const int row = tile * GT_M + 32 * q + lane;
      const float sw = a.emb_s[row];
      const unsigned ta = tmem + ((unsigned)(32 * q) << 16) + 256u * bf + 32u * hf;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        unsigned r0[16], r1[16], r2[16];
        tc::tmem_ld16(ta + 16 * c, r0);
        tc::tmem_ld16(ta + 64 + 16 * c, r1);
        tc::tmem_ld16(ta + 128 + 16 * c, r2);
        tc::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int tb = 16 * c + e, b = 32 * hf + tb;
          const float xsb = __shfl_sync(0xffffffffu, hx, tb);
          const long long X = (long long)(int)r0[e] + 256ll * (int)r1[e] + 65536ll * (int)r2[e];
          const float yv = (float)((double)X * (double)(xsb * sw));
          if (want && b < nb) a.logits[(size_t)b * VOCAB + row] = yv;
          const unsigned long long key = am_pack(yv, row);
          const unsigned hi = __reduce_max_sync(0xffffffffu, (unsigned)(key >> 32));
          const unsigned lo = __reduce_max_sync(0xffffffffu, (unsigned)(key >> 32) == hi ? (unsigned)key : 0u);
          if (lane == tb) best = umax64(best, (unsigned long long)hi << 32 | lo);
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acce(bf));
    }
    bestsm[q * 64 + 32 * hf + lane] = best;
  }
  __syncthreads();
  if (t < 64) {
    unsigned long long m = 0ull;
#pragma unroll
    for (int q = 0; q < 4; ++q) m = umax64(m, bestsm[q * 64 + t]);
    a.am[(size_t)blockIdx.x * 64 + t] = m;
  }
  tc::fence_before();
  __syncthreads();
  if (wid == 0) {
    tc::fence_after();
    tc::tmem_free<512>(tmem);
  }
}

// argmax over the head CTAs per token -> ids, and the next step's token
__global__ void k_bt_finish(const unsigned long long* __restrict__ am, int G, int* ids, int* tok) {
  const int b = blockIdx.x, lane = threadIdx.x;
  tc::grid_wait();
  unsigned long long m = 0ull;
  for (int c = lane; c < G; c += 32) m = umax64(m, am[(size_t)c * 64 + b]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = umax64(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) {
    const int id = am_index(m);
    ids[b] = id;
    tok[b] = id;
  }
}

}  // namespace

// ---------------------------------------------------------------- host side

cudaError_t repack_tiles(const int8_t* const* rowptr, int8_t* out, int nrows, int K, cudaStream_t st) {
  if (nrows % GT_M || K % GT_KS) return cudaErrorInvalidValue;
  const size_t units = (size_t)nrows * K / 16;
  const int blocks = (int)std::min<size_t>((units + 255) / 256, 65535);
  k_bt_repack<<<blocks, 256, 0, st>>>(rowptr, reinterpret_cast<int4*>(out), nrows, K);
  return cudaGetLastError();
}

namespace {

template <int NPL>
cudaError_t launch_gemm(const GemmArgs& a, int ntiles, cudaStream_t st) {
  const int ny = (a.nslab + a.kspl - 1) / a.kspl;
  k_bt_gemm<NPL><<<dim3(ntiles, ny), 128, GC<NPL>::SMEM, st>>>(a);
  return cudaGetLastError();
}

cudaError_t set_smem_attrs() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_bt_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, GC<1>::SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_bt_gemm<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, GC<3>::SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_bt_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_bt_head, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM))) return e;
  return cudaSuccess;
}

}  // namespace

cudaError_t gemm_i8_i8_batched(int32_t* acc, float* y, const int8_t* w, const float* sw, const int8_t* xq,
                               const float* sx, int N, int K, int B, cudaStream_t st) {
  if (N <= 0 || N % GT_M || K <= 0 || K % GT_KS || K > 4096 || B < 1 || B > BATCH_MAX) return cudaErrorInvalidValue;
  cudaError_t e = set_smem_attrs();
  if (e != cudaSuccess) return e;
  const int ntiles = N / GT_M, nslab = K / GT_KS;
  int8_t* tiles = nullptr;
  int8_t* img = nullptr;
  const int8_t** rows = nullptr;
  float* xs = nullptr;
  int32_t* part = nullptr;
  int* cnt = nullptr;
  int* err = nullptr;
  std::vector<const int8_t*> hrows(N);
  for (int r = 0; r < N; ++r) hrows[r] = w + (size_t)r * K;
  const int kspl = nslab >= 8 ? (nslab + 1) / 2 : nslab;   // two K halves for the long shapes (exercises split K)
  if ((e = cudaMallocAsync((void**)&tiles, (size_t)N * K, st)) ||
      (e = cudaMallocAsync((void**)&img, (size_t)nslab * 64 * GT_KS, st)) ||
      (e = cudaMallocAsync((void**)&rows, N * sizeof(void*), st)) ||
      (e = cudaMallocAsync((void**)&xs, 64 * 4, st)) ||
      (e = cudaMallocAsync((void**)&part, (size_t)ntiles * 64 * 128 * 4, st)) ||
      (e = cudaMallocAsync((void**)&cnt, ntiles * 4 + 16, st)) || (e = cudaMallocAsync((void**)&err, 16, st)))
    return e;
  e = cudaMemcpyAsync(rows, hrows.data(), N * sizeof(void*), cudaMemcpyHostToDevice, st);
  if (!e) e = cudaMemsetAsync(xs, 0, 64 * 4, st);
  if (!e) e = cudaMemcpyAsync(xs, sx, B * 4, cudaMemcpyDeviceToDevice, st);
  if (!e) e = cudaMemsetAsync(part, 0, (size_t)ntiles * 64 * 128 * 4, st);
  if (!e) e = cudaMemsetAsync(cnt, 0, ntiles * 4 + 16, st);
  if (!e) e = cudaMemsetAsync(err, 0, 16, st);
  if (!e) e = repack_tiles(rows, tiles, N, K, st);
  if (!e) {
    k_bt_image<<<64, 256, 0, st>>>(xq, img, B, K);
    e = cudaGetLastError();
  }
  GemmArgs a{};
  a.W = tiles; a.sw = sw; a.X = img; a.xs = xs;
  a.nslab = nslab; a.kspl = kspl; a.nb = B; a.mode = EPI_STORE;
  a.Y = y; a.ldy = N; a.part = part; a.cnt = cnt; a.acc_out = acc; a.nrows = N; a.err = err;
  if (!e) e = launch_gemm<1>(a, ntiles, st);
  int herr[4] = {0, 0, 0, 0};
  if (!e) e = cudaMemcpyAsync(herr, err, 16, cudaMemcpyDeviceToHost, st);
  if (!e) e = cudaStreamSynchronize(st);
  cudaFreeAsync(tiles, st); cudaFreeAsync(img, st); cudaFreeAsync(rows, st); cudaFreeAsync(xs, st);
  cudaFreeAsync(part, st); cudaFreeAsync(cnt, st); cudaFreeAsync(err, st);
  if (!e && herr[0]) e = cudaErrorLaunchTimeout;
  return e;
}

// ---------------------------------------------------------------- the engine

namespace {

struct LayerTiles {
  int8_t* win; float* swin; int nin;    // [qkv | z] or [q | k | v] rows
  int8_t* wout; float* swout;
  int8_t* wgu; float* swgu;             // tile t: gate rows 64 t .., then up rows 64 t ..
  int8_t* wdown; float* swdown;
};

}  // namespace

struct BatchEngine {
  int max_batch = 0, max_ctx = 0, max_rope = 0, maxch = 0, sm_count = 148, head_grid = 148;
  cudaStream_t st = nullptr;
  ModelW M{};
  const int8_t* head_tiles = nullptr;
  const float* rope = nullptr;
  LayerTiles L[NLAYER]{};
  std::vector<void*> allocs;
  // per-sequence state
  float *conv = nullptr, *rec = nullptr, *kc = nullptr, *vc = nullptr;
  size_t conv_seq = 0, rec_seq = 0, kv_seq = 0;
  // step buffers
  float *H = nullptr, *Y = nullptr, *O = nullptr, *AB = nullptr, *xs = nullptr, *hxs = nullptr, *attp = nullptr,
        *logits = nullptr;
  int8_t *X = nullptr, *HX = nullptr;
  int32_t* part = nullptr;
  int* cnt = nullptr;
  unsigned long long* am = nullptr;
  int *tok = nullptr, *ids = nullptr, *err = nullptr;
  BtCtl* dctl = nullptr;
  BtCtl* hctl = nullptr;    // pinned
  int* hbuf = nullptr;      // pinned: tokens in, ids out, err
  // host mirror of the per-sequence scalars
  std::vector<int> pos, T, cbase;
  std::map<int, cudaGraphExec_t> graphs;   // key: nb * 2 + i8
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  // slabs per CTA of each projection (K / 128 slabs; fewer slabs per CTA =
  // more CTAs per tile, reduced exactly in int32)
  int ksplit_in = 4, ksplit_out = 2, ksplit_gu = 4, ksplit_down = 4;
};

namespace {

template <typename T>
cudaError_t balloc(BatchEngine* e, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t r = cudaMalloc(&q, bytes);
  if (r != cudaSuccess) return r;
  e->allocs.push_back(q);
  r = cudaMemset(q, 0, bytes);
  *p = reinterpret_cast<T*>(q);
  return r;
}

#define BCUDA(x)                                                                  \
  do {                                                                            \
    cudaError_t e_ = (x);                                                         \
    if (e_ != cudaSuccess) {                                                      \
      err = std::string(#x) + ": " + cudaGetErrorString(e_);                      \
      return QWEN_ERR_CUDA;                                                       \
    }                                                                             \
  } while (0)

// Enqueue one step of nb sequences with NPL digit planes (1: W8A8, 3: W8A32).
template <int NPL>
cudaError_t enqueue_step(BatchEngine* E, int nb) {
  cudaStream_t st = E->st;
  cudaError_t e = cudaSuccess;
  auto gemm = [&](const int8_t* W, const float* sw, int nrows, int K, int kspl, int mode, float* Y, int ldy) {
    if (e != cudaSuccess) return;
    GemmArgs a{};
    a.W = W; a.sw = sw; a.X = E->X; a.xs = E->xs;
    a.nslab = K / GT_KS; a.kspl = kspl; a.nb = nb; a.mode = mode;
    a.Y = Y; a.ldy = ldy; a.part = E->part; a.cnt = E->cnt; a.acc_out = nullptr; a.nrows = nrows; a.err = E->err;
    e = launch_gemm<NPL>(a, nrows / GT_M, st);
  };
  auto normq = [&](int l, bool embed, bool head) {
    if (e != cudaSuccess) return;
    NormqArgs a{};
    a.H = E->H; a.tok = embed ? E->tok : nullptr; a.emb_q = E->M.emb_q; a.emb_s = E->M.emb_s;
    a.err = E->err;
    if (head) {
      a.gain = E->M.final_norm;
      a.X = E->HX; a.xs = E->hxs;
      k_bt_normq<3><<<nb, NT, 0, st>>>(a);
    } else {
      const LayerW& Lw = E->M.L[l];
      a.gain = Lw.in_norm;
      if (Lw.linear) { a.a_w = Lw.a_w; a.b_w = Lw.b_w; a.AB = E->AB; }
      a.X = E->X; a.xs = E->xs;
      k_bt_normq<NPL><<<nb, NT, 0, st>>>(a);
    }
    e = cudaGetLastError();
  };
  auto post_normq = [&](int l) {
    if (e != cudaSuccess) return;
    NormqArgs a{};
    a.H = E->H; a.gain = E->M.L[l].post_norm; a.X = E->X; a.xs = E->xs; a.err = E->err;
    k_bt_normq<NPL><<<nb, NT, 0, st>>>(a);
    e = cudaGetLastError();
  };
  constexpr int LDY = 8192;
  normq(0, true, false);
  for (int l = 0; l < NLAYER && e == cudaSuccess; ++l) {
    const LayerW& Lw = E->M.L[l];
    const LayerTiles& T = E->L[l];
    gemm(T.win, T.swin, T.nin, HID, E->ksplit_in, EPI_STORE, E->Y, LDY);
    if (Lw.linear) {
      DeltaArgs d{};
      d.Y = E->Y; d.ldy = LDY; d.AB = E->AB; d.conv = E->conv; d.rec = E->rec;
      d.conv_seq = E->conv_seq; d.rec_seq = E->rec_seq; d.lin = Lw.lin_idx;
      d.conv_w = Lw.conv_w; d.A_log = Lw.A_log; d.dt_bias = Lw.dt_bias; d.gnorm_w = Lw.gnorm_w;
      d.ctl = E->dctl; d.O = E->O;
      if (e == cudaSuccess) { k_bt_delta<<<dim3(LH, nb), NT, 0, st>>>(d); e = cudaGetLastError(); }
      if (e == cudaSuccess) { k_bt_quant<NPL><<<nb, NT, 0, st>>>(E->O, VDIM, VDIM, E->X, E->xs); e = cudaGetLastError(); }
    } else {
      AttnArgs at{};
      at.Y = E->Y; at.ldy = LDY; at.kc = E->kc; at.vc = E->vc; at.fi = Lw.full_idx; at.max_ctx = E->max_ctx;
      at.qn_w = Lw.qn_w; at.kn_w = Lw.kn_w; at.rope = E->rope; at.ctl = E->dctl; at.part = E->attp;
      at.maxch = E->maxch; at.err = E->err;
      if (e == cudaSuccess) { k_bt_attn<<<2 * E->sm_count, 256, AT_SMEM, st>>>(at); e = cudaGetLastError(); }
      if (e == cudaSuccess) {
        k_bt_merge<NPL><<<nb, NT, 0, st>>>(E->Y, LDY, E->attp, E->maxch, E->dctl, E->X, E->xs);
        e = cudaGetLastError();
      }
    }
    gemm(T.wout, T.swout, HID, VDIM, E->ksplit_out, EPI_ADD, E->H, HID);
    post_normq(l);
    gemm(T.wgu, T.swgu, 2 * FFN, HID, E->ksplit_gu, EPI_SWIGLU, E->O, FFN);
    if (e == cudaSuccess) { k_bt_quant<NPL><<<nb, NT, 0, st>>>(E->O, FFN, FFN, E->X, E->xs); e = cudaGetLastError(); }
    gemm(T.wdown, T.swdown, HID, FFN, E->ksplit_down, EPI_ADD, E->H, HID);
    if (l + 1 < NLAYER) normq(l + 1, false, false);
  }
  normq(0, false, true);
  if (e == cudaSuccess) {
    HeadArgs h{};
    h.tiles = E->head_tiles; h.emb_s = E->M.emb_s; h.HX = E->HX; h.hxs = E->hxs; h.ctl = E->dctl;
    h.logits = E->logits; h.am = E->am; h.err = E->err;
    k_bt_head<<<E->head_grid, HB_THREADS, HB_SMEM, st>>>(h);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    k_bt_finish<<<nb, 32, 0, st>>>(E->am, E->head_grid, E->ids, E->tok);
    e = cudaGetLastError();
  }
  return e;
}

cudaError_t graph_for(BatchEngine* E, int nb, bool i8, cudaGraphExec_t* out) {
  const int key = nb * 2 + (i8 ? 1 : 0);
  auto it = E->graphs.find(key);
  if (it != E->graphs.end()) { *out = it->second; return cudaSuccess; }
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(E->st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return e;
  cudaError_t el = i8 ? enqueue_step<1>(E, nb) : enqueue_step<3>(E, nb);
  e = cudaStreamEndCapture(E->st, &g);
  if (el != cudaSuccess) { if (g) cudaGraphDestroy(g); return el; }
  if (e != cudaSuccess) return e;
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiate(&x, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return e;
  E->graphs[key] = x;
  *out = x;
  return cudaSuccess;
}

int check_seq(const BatchEngine* E, int seq, std::string& err) {
  if (seq < 0 || seq >= E->max_batch) {
    err = "seq out of range";
    return QWEN_ERR_ARG;
  }
  return QWEN_OK;
}

// Fill the control block for nb sequences; QWEN_ERR_STATE if one is full.
int fill_ctl(BatchEngine* E, int nb, bool want_logits, std::string& err) {
  BtCtl& c = *E->hctl;
  int nchmax = 1;
  for (int b = 0; b < nb; ++b) {
    if (E->T[b] + 1 > E->max_ctx || E->pos[b] >= E->max_rope) {
      err = "sequence " + std::to_string(b) + " is full (max_ctx)";
      return QWEN_ERR_STATE;
    }
    c.pos[b] = E->pos[b];
    c.T[b] = E->T[b];
    c.cbase[b] = E->cbase[b];
    nchmax = std::max(nchmax, (E->T[b] + 1 + AT_CL - 1) / AT_CL);
  }
  c.nb = nb;
  c.want_logits = want_logits ? 1 : 0;
  c.nchmax = nchmax;
  return QWEN_OK;
}

void advance(BatchEngine* E, int nb) {
  for (int b = 0; b < nb; ++b) {
    E->pos[b]++;
    E->T[b]++;
    E->cbase[b]++;
  }
}

int read_err(BatchEngine* E, std::string& err) {
  int* h = E->hbuf + 2 * BATCH_MAX;
  BCUDA(cudaMemcpyAsync(h, E->err, 16, cudaMemcpyDeviceToHost, E->st));
  BCUDA(cudaStreamSynchronize(E->st));
  if (h[0] == 0) return QWEN_OK;
  char buf[160];
  snprintf(buf, sizeof buf, "batched step: device error %d (site %d, value %d)", h[0], h[1], h[2]);
  err = buf;
  const int code = h[0];
  BCUDA(cudaMemsetAsync(E->err, 0, 16, E->st));
  return code == ERR_TOKEN ? QWEN_ERR_ARG : (code == ERR_CTX ? QWEN_ERR_STATE : QWEN_ERR_DEVICE);
}

}  // namespace

BatchEngine* batch_create(const ModelW& M, const int8_t* head_tiles, const float* rope, int max_rope, int max_batch,
                          int max_ctx, int sm_count, cudaStream_t st, std::string& err) {
  if (max_batch < 1 || max_batch > BATCH_MAX) {
    err = "max_batch must be in [1, 64]";
    return nullptr;
  }
  BatchEngine* E = new BatchEngine();
  E->max_batch = max_batch;
  E->max_ctx = max_ctx;
  E->max_rope = max_rope;
  E->maxch = (max_ctx + AT_CL - 1) / AT_CL;
  E->sm_count = sm_count;
  E->head_grid = std::min(sm_count, BT_HEAD_TILES);
  E->st = st;
  E->M = M;
  E->head_tiles = head_tiles;
  E->rope = rope;
  E->pos.assign(BATCH_MAX, 0);
  E->T.assign(BATCH_MAX, 0);
  E->cbase.assign(BATCH_MAX, 0);
  auto bail = [&](const std::string& m) {
    err = m;
    batch_destroy(E);
    return (BatchEngine*)nullptr;
  };
  cudaError_t e = set_smem_attrs();
  if (e != cudaSuccess) return bail(std::string("kernel attributes: ") + cudaGetErrorString(e));
  E->conv_seq = (size_t)NLIN * CONVD * CONVK;
  E->rec_seq = (size_t)NLIN * LH * LK * LV;
  E->kv_seq = (size_t)NFULL * NKV * max_ctx * HD;
  const size_t B = (size_t)max_batch;
  if ((e = balloc(E, &E->conv, B * E->conv_seq * 4)) || (e = balloc(E, &E->rec, B * E->rec_seq * 4)) ||
      (e = balloc(E, &E->kc, B * E->kv_seq * 4)) || (e = balloc(E, &E->vc, B * E->kv_seq * 4)) ||
      (e = balloc(E, &E->H, (size_t)BATCH_MAX * HID * 4)) || (e = balloc(E, &E->Y, (size_t)BATCH_MAX * 8192 * 4)) ||
      (e = balloc(E, &E->O, (size_t)BATCH_MAX * FFN * 4)) || (e = balloc(E, &E->AB, (size_t)BATCH_MAX * 32 * 4)) ||
      (e = balloc(E, &E->xs, 64 * 4)) || (e = balloc(E, &E->hxs, 64 * 4)) ||
      (e = balloc(E, &E->attp, B * NKV * E->maxch * 4 * AT_PROW * 4)) ||
      (e = balloc(E, &E->logits, (size_t)BATCH_MAX * VOCAB * 4)) ||
      (e = balloc(E, &E->X, (size_t)(FFN / GT_KS) * 192 * GT_KS)) || (e = balloc(E, &E->HX, (size_t)HB_IMG)) ||
      (e = balloc(E, &E->part, (size_t)BT_MAXTILES * 192 * 128 * 4)) ||
      (e = balloc(E, &E->cnt, (size_t)BT_MAXTILES * 4)) ||
      (e = balloc(E, &E->am, (size_t)E->head_grid * 64 * 8)) || (e = balloc(E, &E->tok, 64 * 4)) ||
      (e = balloc(E, &E->ids, 64 * 4)) || (e = balloc(E, &E->err, 16)) || (e = balloc(E, &E->dctl, sizeof(BtCtl))))
    return bail(std::string("device memory: ") + cudaGetErrorString(e));
  if (cudaMallocHost((void**)&E->hctl, sizeof(BtCtl)) != cudaSuccess ||
      cudaMallocHost((void**)&E->hbuf, (2 * BATCH_MAX + 4) * sizeof(int)) != cudaSuccess)
    return bail("pinned host buffers");
  memset(E->hctl, 0, sizeof(BtCtl));
  cudaEventCreate(&E->ev0);
  cudaEventCreate(&E->ev1);
  // the layer projections as tensor-core tiles (copies; the row-major blob stays)
  std::vector<const int8_t*> rows;
  const int8_t** drows = nullptr;
  if ((e = balloc(E, &drows, (size_t)8192 * sizeof(void*))))
    return bail(std::string("row table: ") + cudaGetErrorString(e));
  auto pack = [&](int8_t** out, float** sout, const std::vector<std::pair<const int8_t*, const float*>>& segs,
                  const std::vector<int>& nrows, int K) -> cudaError_t {
    rows.clear();
    int total = 0;
    for (size_t i = 0; i < segs.size(); ++i) {
      for (int r = 0; r < nrows[i]; ++r) rows.push_back(segs[i].first + (size_t)r * K);
      total += nrows[i];
    }
    cudaError_t r = balloc(E, out, (size_t)total * K);
    if (r) return r;
    if ((r = balloc(E, sout, (size_t)total * 4))) return r;
    if ((r = cudaMemcpy(drows, rows.data(), rows.size() * sizeof(void*), cudaMemcpyHostToDevice))) return r;
    if ((r = repack_tiles(drows, *out, total, K, st))) return r;
    int off = 0;
    for (size_t i = 0; i < segs.size(); ++i) {
      if ((r = cudaMemcpyAsync(*sout + off, segs[i].second, (size_t)nrows[i] * 4, cudaMemcpyDeviceToDevice, st)))
        return r;
      off += nrows[i];
    }
    return cudaStreamSynchronize(st);
  };
  for (int l = 0; l < NLAYER; ++l) {
    const LayerW& W = M.L[l];
    LayerTiles& T = E->L[l];
    if (W.linear) {
      e = pack(&T.win, &T.swin, {{W.qkv_q, W.qkv_s}, {W.z_q, W.z_s}}, {CONVD, VDIM}, HID);
      T.nin = CONVD + VDIM;
    } else {
      e = pack(&T.win, &T.swin, {{W.q_q, W.q_s}, {W.k_q, W.k_s}, {W.v_q, W.v_s}}, {QPROJ, KVPROJ, KVPROJ}, HID);
      T.nin = QPROJ + 2 * KVPROJ;
    }
    if (!e) e = pack(&T.wout, &T.swout, {{W.linear ? W.out_q : W.o_q, W.linear ? W.out_s : W.o_s}}, {HID}, VDIM);
    if (!e) {
      std::vector<std::pair<const int8_t*, const float*>> segs;
      std::vector<int> nr;
      for (int q = 0; q < FFN / 64; ++q) {
        segs.push_back({W.gate_q + (size_t)q * 64 * HID, W.gate_s + q * 64});
        segs.push_back({W.up_q + (size_t)q * 64 * HID, W.up_s + q * 64});
        nr.push_back(64);
        nr.push_back(64);
      }
      e = pack(&T.wgu, &T.swgu, segs, nr, HID);
    }
    if (!e) e = pack(&T.wdown, &T.swdown, {{W.down_q, W.down_s}}, {HID}, FFN);
    if (e) return bail(std::string("weight tiles: ") + cudaGetErrorString(e));
  }
  return E;
}

void batch_destroy(BatchEngine* E) {
  if (!E) return;
  if (E->st) cudaStreamSynchronize(E->st);
  for (auto& kv : E->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : E->allocs) cudaFree(p);
  if (E->hctl) cudaFreeHost(E->hctl);
  if (E->hbuf) cudaFreeHost(E->hbuf);
  if (E->ev0) cudaEventDestroy(E->ev0);
  if (E->ev1) cudaEventDestroy(E->ev1);
  delete E;
}

int batch_max(const BatchEngine* E) { return E->max_batch; }

int batch_reset(BatchEngine* E, int seq, std::string& err) {
  int b0 = 0, b1 = E->max_batch;
  if (seq >= 0) {
    if (int rc = check_seq(E, seq, err)) return rc;
    b0 = seq;
    b1 = seq + 1;
  }
  for (int b = b0; b < b1; ++b) {
    BCUDA(cudaMemsetAsync(E->conv + (size_t)b * E->conv_seq, 0, E->conv_seq * 4, E->st));
    BCUDA(cudaMemsetAsync(E->rec + (size_t)b * E->rec_seq, 0, E->rec_seq * 4, E->st));
    E->pos[b] = E->T[b] = E->cbase[b] = 0;
  }
  BCUDA(cudaStreamSynchronize(E->st));
  return QWEN_OK;
}

int batch_import(BatchEngine* E, int seq, const float* conv, const float* rec, const float* kc, const float* vc, int T,
                 int pos, std::string& err) {
  if (int rc = check_seq(E, seq, err)) return rc;
  if (!conv || !rec || T < 0 || T > E->max_ctx - 1 || pos < 0 || pos >= E->max_rope || (T > 0 && (!kc || !vc))) {
    err = "state_import: bad arguments (T must be <= max_ctx - 1)";
    return QWEN_ERR_ARG;
  }
  cudaStream_t st = E->st;
  // conv history at ring origin 0: logical column i in slot i
  BCUDA(cudaMemcpyAsync(E->conv + (size_t)seq * E->conv_seq, conv, E->conv_seq * 4, cudaMemcpyHostToDevice, st));
  BCUDA(cudaMemcpyAsync(E->rec + (size_t)seq * E->rec_seq, rec, E->rec_seq * 4, cudaMemcpyHostToDevice, st));
  for (int f = 0; f < NFULL && T > 0; ++f)
    for (int g = 0; g < NKV; ++g) {
      const size_t dst = (size_t)seq * E->kv_seq + ((size_t)f * NKV + g) * E->max_ctx * HD;
      const size_t src = (size_t)f * T * KVPROJ + (size_t)g * HD;
      BCUDA(cudaMemcpy2DAsync(E->kc + dst, HD * 4, kc + src, KVPROJ * 4, HD * 4, T, cudaMemcpyHostToDevice, st));
      BCUDA(cudaMemcpy2DAsync(E->vc + dst, HD * 4, vc + src, KVPROJ * 4, HD * 4, T, cudaMemcpyHostToDevice, st));
    }
  BCUDA(cudaStreamSynchronize(st));
  E->T[seq] = T;
  E->pos[seq] = pos;
  E->cbase[seq] = 0;
  return QWEN_OK;
}

int batch_export(BatchEngine* E, int seq, float* conv, float* rec, float* kc, float* vc, int* T, int* pos,
                 std::string& err) {
  if (int rc = check_seq(E, seq, err)) return rc;
  cudaStream_t st = E->st;
  const int Ts = E->T[seq];
  if (T) *T = Ts;
  if (pos) *pos = E->pos[seq];
  if (conv) {
    // unroll the ring: logical column i lives in slot (cbase + i) & 3
    std::vector<float> ring(E->conv_seq);
    BCUDA(cudaMemcpyAsync(ring.data(), E->conv + (size_t)seq * E->conv_seq, E->conv_seq * 4, cudaMemcpyDeviceToHost, st));
    BCUDA(cudaStreamSynchronize(st));
    const int cb = E->cbase[seq];
    for (size_t r = 0; r < E->conv_seq / CONVK; ++r)
      for (int i = 0; i < CONVK; ++i) conv[r * CONVK + i] = ring[r * CONVK + ((cb + i) & 3)];
  }
  if (rec) BCUDA(cudaMemcpyAsync(rec, E->rec + (size_t)seq * E->rec_seq, E->rec_seq * 4, cudaMemcpyDeviceToHost, st));
  for (int f = 0; f < NFULL && Ts > 0; ++f)
    for (int g = 0; g < NKV; ++g) {
      const size_t src = (size_t)seq * E->kv_seq + ((size_t)f * NKV + g) * E->max_ctx * HD;
      const size_t dst = (size_t)f * Ts * KVPROJ + (size_t)g * HD;
      if (kc) BCUDA(cudaMemcpy2DAsync(kc + dst, KVPROJ * 4, E->kc + src, HD * 4, HD * 4, Ts, cudaMemcpyDeviceToHost, st));
      if (vc) BCUDA(cudaMemcpy2DAsync(vc + dst, KVPROJ * 4, E->vc + src, HD * 4, HD * 4, Ts, cudaMemcpyDeviceToHost, st));
    }
  BCUDA(cudaStreamSynchronize(st));
  return QWEN_OK;
}

int batch_step(BatchEngine* E, const int* tok, int nb, bool act_int8, float* logits_out, int* argmax_out,
               std::string& err) {
  if (nb < 1 || nb > E->max_batch) {
    err = "batch must be in [1, max_batch]";
    return QWEN_ERR_ARG;
  }
  if (tok)
    for (int b = 0; b < nb; ++b)
      if (tok[b] < 0 || tok[b] >= VOCAB) {
        err = "token id out of range";
        return QWEN_ERR_ARG;
      }
  if (int rc = fill_ctl(E, nb, logits_out != nullptr, err)) return rc;
  cudaStream_t st = E->st;
  cudaGraphExec_t g = nullptr;
  BCUDA(graph_for(E, nb, act_int8, &g));
  BCUDA(cudaMemcpyAsync(E->dctl, E->hctl, sizeof(BtCtl), cudaMemcpyHostToDevice, st));
  if (tok) {
    memcpy(E->hbuf, tok, nb * sizeof(int));
    BCUDA(cudaMemcpyAsync(E->tok, E->hbuf, nb * sizeof(int), cudaMemcpyHostToDevice, st));
  }
  BCUDA(cudaGraphLaunch(g, st));
  int* hid = E->hbuf + BATCH_MAX;
  BCUDA(cudaMemcpyAsync(hid, E->ids, nb * sizeof(int), cudaMemcpyDeviceToHost, st));
  if (logits_out) BCUDA(cudaMemcpyAsync(logits_out, E->logits, (size_t)nb * VOCAB * 4, cudaMemcpyDefault, st));
  if (int rc = read_err(E, err)) return rc;
  advance(E, nb);
  if (argmax_out) memcpy(argmax_out, hid, nb * sizeof(int));
  return QWEN_OK;
}

int batch_timed_steps(BatchEngine* E, int nb, bool act_int8, int steps, double* seconds, std::string& err) {
  if (nb < 1 || nb > E->max_batch || steps < 1) {
    err = "batch / steps out of range";
    return QWEN_ERR_ARG;
  }
  cudaStream_t st = E->st;
  cudaGraphExec_t g = nullptr;
  BCUDA(graph_for(E, nb, act_int8, &g));
  // every step reads its scalars from the control block: one copy per step
  // (from its own pinned slot), tokens fed back on the device
  BtCtl* slots = nullptr;
  BCUDA(cudaMallocHost((void**)&slots, sizeof(BtCtl) * steps));
  int rc = QWEN_OK;
  for (int s = 0; s < steps && rc == QWEN_OK; ++s) {
    rc = fill_ctl(E, nb, false, err);
    if (rc == QWEN_OK) {
      slots[s] = *E->hctl;
      advance(E, nb);
    }
  }
  if (rc != QWEN_OK) {
    // roll the mirror back to where it was
    for (int b = 0; b < nb; ++b) { E->pos[b] = slots[0].pos[b]; E->T[b] = slots[0].T[b]; E->cbase[b] = slots[0].cbase[b]; }
    cudaFreeHost(slots);
    return rc;
  }
  cudaError_t e = cudaEventRecord(E->ev0, st);
  for (int s = 0; s < steps && e == cudaSuccess; ++s) {
    e = cudaMemcpyAsync(E->dctl, slots + s, sizeof(BtCtl), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaGraphLaunch(g, st);
  }
  if (e == cudaSuccess) e = cudaEventRecord(E->ev1, st);
  if (e == cudaSuccess) e = cudaEventSynchronize(E->ev1);
  cudaFreeHost(slots);
  if (e != cudaSuccess) {
    err = std::string("timed steps: ") + cudaGetErrorString(e);
    return QWEN_ERR_CUDA;
  }
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, E->ev0, E->ev1);
  if (seconds) *seconds = ms * 1e-3;
  return read_err(E, err);
}

}  // namespace qb
