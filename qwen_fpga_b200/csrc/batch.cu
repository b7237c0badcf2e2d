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
  int nslab, kspl;     // slabs of K; slabs per CTA (grid.y = ceil(nslab / kspl) <= 8: one cluster per tile)
  int nb;              // live tokens
  int mode;
  float* Y;            // STORE / ADD: Y[b ldy + row]; SWIGLU: Y[b ldy + 64 tile + r]
  int ldy;
  int32_t* acc_out;    // nullable (NPL 1): acc[b nrows + row]
  int nrows;
  int* err;
};

template <int NPL>
struct GC {
  static constexpr int NR = 64 * NPL;
  static constexpr int BBYTES = NR * GT_KS;
  static constexpr int STAGE = GT_SLAB + BBYTES;
  // ring depth: W8A8 holds every slab of an unsplit K = 1024 tile in flight
  // (one CTA per SM)
  static constexpr int NST = NPL == 1 ? 8 : 5;
  static constexpr int OFF_BAR = NST * STAGE;
  // W8A32 split-K epilogue (pull): the parked sums (128 rows x (NR + 4) ints)
  // and, after them, the SwiGLU exchange (64 tokens x 128 rows floats), inside the ring
  static constexpr int XCH = ((128 * (NR + 4) * 4 + 1023) / 1024) * 1024;
  static_assert(XCH + 64 * 128 * 4 <= OFF_BAR, "split-K scratch inside the ring");
  // barriers (full[NST], empty[NST], accf), the TMEM slot, three flags
  static constexpr int OFF_SLOT = OFF_BAR + 16 * NST + 8;
  static constexpr int SMEM = OFF_SLOT + 16;
  static constexpr int TCOLS = NPL == 1 ? 64 : 256;
  static constexpr unsigned IDESC = tc::idesc_i8(GT_M, NR);
};
static_assert(GC<1>::SMEM + 1024 <= 227 * 1024 && GC<3>::SMEM + 1024 <= 227 * 1024, "GEMM shared memory");

// W8A8 split-K over a (1, S, 1) cluster (push): tokens are owned in
// contiguous ranges of TPC; every CTA stores its int32 sums of each 4-token
// group straight into the owner's receive buffer (slot = source rank; remote
// 16-byte stores over distributed shared memory, fire and forget), one
// cluster barrier, then each owner adds its S slots from its own shared
// memory.  The receive buffer sits at the end of the ring, beyond the stages
// the CTA's K range uses (checked).
__host__ __device__ constexpr int push_tpc(int S) { return ((64 + S - 1) / S + 3) & ~3; }
__host__ __device__ constexpr int push_rsp(int S) {
  return (push_tpc(S) + 4) % 16 == 0 ? push_tpc(S) + 8 : push_tpc(S) + 4;
}
// ring offset of the receive buffer of an S-CTA cluster
__host__ __device__ constexpr int push_off(int S) { return GC<1>::OFF_BAR - S * 128 * push_rsp(S) * 4; }
template <int S>
struct SplitPush {
  static constexpr int TPC = push_tpc(S);   // tokens per owner
  static constexpr int RSP = push_rsp(S);   // padded row (ints)
  static constexpr int OFF = push_off(S);
  static_assert(OFF > 0, "receive buffer");
};
// W8A8 GEMM split: the most slabs a CTA of an S-CTA cluster may stream (its
// stages must stay clear of the receive buffer)
__host__ __device__ constexpr int push_max_slabs(int S) { return push_off(S) / GC<1>::STAGE; }

// Dequantised output of one token from its digit sums: W8A8 acc * (s_x s_w);
// W8A32 the exact digit recombination, scaled once in fp64.
template <int NPL>
__device__ __forceinline__ float dequant(const int (&v)[NPL], float xs, float sw) {
  if constexpr (NPL == 1) {
    return (float)v[0] * (xs * sw);
  } else {
    const long long X = (long long)v[0] + 256ll * v[1] + 65536ll * v[2];
    return (float)((double)X * (double)(xs * sw));
  }
}

// Split-K epilogue over a (1, S, 1) cluster, one CTA per K range: every CTA
// parks its int32 sums in its own shared memory (row-major, padded rows),
// then CTA r finishes the contiguous tokens [r tpc, (r + 1) tpc): it reads the
// S CTAs' sums of its row over distributed shared memory, 16 bytes at a time,
// all loads of a chunk in flight before the first add (exact integer adds).
// Every CTA takes both cluster barriers, whatever happened before.
template <int NPL, int S, int MODE>
__device__ __forceinline__ void split_epilogue(const GemmArgs& a, unsigned char* sm, const float* xs_s, unsigned taddr,
                                               bool ok, int tile, int row, int grow, float sw0) {
  using C = GC<NPL>;
  constexpr int RS = C::NR + 4;   // padded row stride (ints): conflict-free 16-byte accesses
  int* red = reinterpret_cast<int*>(sm);
  if (ok) {
    tc::fence_after();
    for (int c0 = 0; c0 < C::NR; c0 += 16) {
      unsigned r[16];
      tc::tmem_ld16(taddr + c0, r);
      tc::tmem_ld_wait();
      int4* dst = reinterpret_cast<int4*>(red + row * RS + c0);
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[e] = make_int4((int)r[4 * e], (int)r[4 * e + 1], (int)r[4 * e + 2], (int)r[4 * e + 3]);
    }
  }
  tc::cluster_sync();
  const int rank = (int)tc::cluster_ctarank();
  constexpr int TPC = ((64 + S - 1) / S + 3) & ~3;      // tokens per CTA
  constexpr int LDN = NPL == 1 ? 16 : 8;                 // 16-byte loads in flight per plane
  constexpr int G = LDN / S > 0 ? LDN / S : 1;           // 4-token groups per chunk
  const int bl0 = rank * TPC, bl1 = min(a.nb, bl0 + TPC);
  const unsigned rbase = tc::smem_u32(red) + 4u * (unsigned)(row * RS);
  unsigned rq[S];
#pragma unroll
  for (int q = 0; q < S; ++q) rq[q] = tc::mapa(rbase, (unsigned)q);
  float* xch = reinterpret_cast<float*>(sm + C::XCH);   // SWIGLU: [tokens of this CTA][128 rows]
  float* __restrict__ Yp = a.Y;
  for (int g0 = bl0; g0 < bl1; g0 += 4 * G) {           // (CTA-uniform bounds)
    int4 sum[NPL][G];
#pragma unroll
    for (int p = 0; p < NPL; ++p) {
      int4 v[G][S];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int q = 0; q < S; ++q) {
          v[g][q] = make_int4(0, 0, 0, 0);
          if (ok && g0 + 4 * g < bl1) v[g][q] = tc::ld_dsmem_v4(rq[q] + 4u * (unsigned)(64 * p + g0 + 4 * g));
        }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sum[p][g] = v[g][0];
#pragma unroll
        for (int q = 1; q < S; ++q) {
          sum[p][g].x += v[g][q].x; sum[p][g].y += v[g][q].y; sum[p][g].z += v[g][q].z; sum[p][g].w += v[g][q].w;
        }
      }
    }
    float yv[4 * G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int b = g0 + 4 * g + e;
        int v[NPL];
#pragma unroll
        for (int p = 0; p < NPL; ++p)
          v[p] = e == 0 ? sum[p][g].x : e == 1 ? sum[p][g].y : e == 2 ? sum[p][g].z : sum[p][g].w;
        yv[4 * g + e] = 0.0f;
        if (b < bl1) {
          yv[4 * g + e] = dequant<NPL>(v, xs_s[b], sw0);
          if (NPL == 1 && a.acc_out && grow < a.nrows && ok) a.acc_out[(size_t)b * a.nrows + grow] = v[0];
        }
      }
    }
    const int nt = min(4 * G, bl1 - g0);
    if constexpr (MODE == EPI_SWIGLU) {
      // gate rows 0-63 and up rows 64-127 of the pair tile meet in shared memory
#pragma unroll
      for (int j = 0; j < 4 * G; ++j)
        if (j < nt) xch[(g0 + j - bl0) * 128 + row] = yv[j];
      __syncthreads();
      if (ok && row < 64) {
#pragma unroll
        for (int j = 0; j < 4 * G; ++j)
          if (j < nt)
            Yp[(size_t)(g0 + j) * a.ldy + 64 * tile + row] =
                __fmul_rn(silu_f(xch[(g0 + j - bl0) * 128 + row]), xch[(g0 + j - bl0) * 128 + row + 64]);
      }
      __syncthreads();
    } else if (ok) {
      if constexpr (MODE == EPI_STORE) {
        if (grow < a.nrows) {
#pragma unroll
          for (int j = 0; j < 4 * G; ++j)
            if (j < nt) Yp[(size_t)(g0 + j) * a.ldy + grow] = yv[j];
        }
      } else {
        float h[4 * G];
#pragma unroll
        for (int j = 0; j < 4 * G; ++j) h[j] = j < nt ? Yp[(size_t)(g0 + j) * a.ldy + grow] : 0.0f;
#pragma unroll
        for (int j = 0; j < 4 * G; ++j)
          if (j < nt) Yp[(size_t)(g0 + j) * a.ldy + grow] = __fadd_rn(h[j], yv[j]);
      }
    }
  }
  tc::cluster_sync();   // the other CTAs' sums stay readable until every CTA is done
}

__device__ __forceinline__ void st_dsmem_v4(unsigned addr, int4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1,%2,%3,%4};" :: "r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Outputs of tokens b0 .. b0 + n - 1 (n <= N) of this thread's row: stored,
// added to the residual rows (loads first, then the stores), or, for a SwiGLU
// pair tile, exchanged through xch ([token][128 rows] floats, CTA-uniform
// call) and combined by all 128 threads.
template <int MODE, int N>
__device__ __forceinline__ void emit_rows(const GemmArgs& a, const float (&yv)[N], int b0, int n, int tile, int row,
                                          int grow, float* xch) {
  float* __restrict__ Yp = a.Y;
  if constexpr (MODE == EPI_SWIGLU) {
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < n) xch[j * 128 + row] = yv[j];
    __syncthreads();
    // thread t: row t % 64 of tokens j = t / 64, t / 64 + 2, ...
    const int r = row & 63;
    for (int j = row >> 6; j < n; j += 2)
      Yp[(size_t)(b0 + j) * a.ldy + 64 * tile + r] = __fmul_rn(silu_f(xch[j * 128 + r]), xch[j * 128 + r + 64]);
    __syncthreads();
  } else if constexpr (MODE == EPI_STORE) {
    if (grow < a.nrows) {
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (j < n) Yp[(size_t)(b0 + j) * a.ldy + grow] = yv[j];
    }
  } else {
    float h[N];
#pragma unroll
    for (int j = 0; j < N; ++j) h[j] = j < n ? Yp[(size_t)(b0 + j) * a.ldy + grow] : 0.0f;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < n) Yp[(size_t)(b0 + j) * a.ldy + grow] = __fadd_rn(h[j], yv[j]);
  }
}

template <int S, int MODE>
__device__ __forceinline__ void split_push(const GemmArgs& a, unsigned char* sm, const float* xs_s, unsigned taddr,
                                           bool ok, int ns, int tile, int row, int grow, float sw0) {
  using P = SplitPush<S>;
  const int rank = (int)tc::cluster_ctarank();
  const bool fits = ns * GC<1>::STAGE <= P::OFF;
  if (!fits && threadIdx.x == 0 && atomicCAS(a.err, 0, ERR_CHECK) == 0) { a.err[1] = 44; a.err[2] = ns; }
  const bool go = ok && fits;
  const unsigned recv = tc::smem_u32(sm + P::OFF);
  if (go) {
    tc::fence_after();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      unsigned r[16];
      tc::tmem_ld16(taddr + 16 * c, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int tb = 16 * c + 4 * g, ow = tb / P::TPC, tl = tb - ow * P::TPC;
        const unsigned dst = tc::mapa(recv, (unsigned)ow) + 4u * (unsigned)((rank * 128 + row) * P::RSP + tl);
        st_dsmem_v4(dst, make_int4((int)r[4 * g], (int)r[4 * g + 1], (int)r[4 * g + 2], (int)r[4 * g + 3]));
      }
    }
  }
  tc::cluster_sync();   // every CTA's sums have landed with their owners
  const int bl0 = rank * P::TPC, n = max(0, min(a.nb, bl0 + P::TPC) - bl0);
  if (!go || n == 0) return;
  const int* rv = reinterpret_cast<const int*>(sm + P::OFF);
  float yv[P::TPC];
#pragma unroll
  for (int g = 0; g < P::TPC / 4; ++g) {
    int4 acc = *reinterpret_cast<const int4*>(rv + row * P::RSP + 4 * g);
#pragma unroll
    for (int q = 1; q < S; ++q) {
      const int4 v = *reinterpret_cast<const int4*>(rv + (q * 128 + row) * P::RSP + 4 * g);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const int vv[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = 4 * g + e, b = bl0 + j;
      const int v1[1] = {vv[e]};
      yv[j] = b < a.nb ? dequant<1>(v1, xs_s[b < 64 ? b : 0], sw0) : 0.0f;
      if (a.acc_out && j < n && grow < a.nrows) a.acc_out[(size_t)b * a.nrows + grow] = vv[e];
    }
  }
  // (the stages are free: the SwiGLU exchange may use the ring's start)
  emit_rows<MODE, P::TPC>(a, yv, bl0, n, tile, row, grow, reinterpret_cast<float*>(sm));
}

// One instance per (digit planes, K-split cluster size S, epilogue): each
// launch runs only its own path (a small kernel: its instructions stay in the
// SM's instruction cache).
template <int NPL, int S, int MODE>
__global__ void __launch_bounds__(128, 1) k_bt_gemm(const GemmArgs a) {
  using C = GC<NPL>;
  extern __shared__ __align__(1024) unsigned char sm[];
  const int t = threadIdx.x, wid = t >> 5, lane = t & 31;
  const int tile = blockIdx.x;
  const int j0 = blockIdx.y * a.kspl, j1 = min(a.nslab, j0 + a.kspl), ns = j1 - j0;
  const unsigned bar0 = tc::smem_u32(sm + C::OFF_BAR);
  const unsigned accf = bar0 + 16u * C::NST;
  unsigned* tslot = reinterpret_cast<unsigned*>(sm + C::OFF_SLOT);
  int* flag = reinterpret_cast<int*>(tslot + 1);   // [0] spare, [1] issued, [2] consumed
  if (t == 0) {
    for (int s = 0; s < C::NST; ++s) {
      tc::mbar_init(bar0 + 8u * s, 1);                 // full
      tc::mbar_init(bar0 + 8u * (C::NST + s), 1);      // empty
    }
    tc::mbar_init(accf, 1);
    tc::mbar_init_fence();
    flag[0] = 0;
  }
  // The first stages' weight slabs do not depend on the previous kernel: they
  // are requested before the dependency wait (under programmatic dependent
  // launch they stream in while the previous kernel drains).
  // Slab i of this CTA is K slab j0 + (i + tile) % ns: concurrent tiles stream
  // different offsets of their weights (the int32 sums do not depend on order).
  const int npre = min(ns, C::NST);
  auto slab = [&](int i) { const int j = i + tile % max(ns, 1); return j0 + (j >= ns ? j - ns : j); };
  unsigned long long pw = 0, px = 0;
  if (t == 0) {
    pw = tc::policy_evict_first();
    px = tc::policy_evict_last();
    for (int i = 0; i < npre; ++i) {
      const unsigned fb = bar0 + 8u * i;
      tc::mbar_expect(fb, (unsigned)C::STAGE);
      tc::bulk_g2s(tc::smem_u32(sm + i * C::STAGE), a.W + ((size_t)tile * a.nslab + slab(i)) * GT_SLAB, GT_SLAB, fb, pw);
    }
  }
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
  tc::grid_wait();
  if (wid == 0) tc::tmem_alloc<C::TCOLS>(tslot);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const unsigned tmem = *tslot;
  __shared__ float xs_s[64];   // per-token scales, read in the epilogue
  if (t < 64) xs_s[t] = a.xs[t];
  int issued = 0, consumed = 0;
  if (t == 0) {
    // producer: weights (read once: evict first) and the image slab (shared by every tile)
    for (int i = 0; i < npre; ++i)
      tc::bulk_g2s(tc::smem_u32(sm + i * C::STAGE) + GT_SLAB, a.X + (size_t)slab(i) * C::BBYTES, C::BBYTES,
                   bar0 + 8u * i, px);
    issued = npre;
    for (int i = npre; i < ns; ++i) {
      const int s = i % C::NST;
      if (!tc::mbar_wait(bar0 + 8u * (C::NST + s), (unsigned)(((i / C::NST) - 1) & 1), a.err, 40, i)) break;
      const unsigned dst = tc::smem_u32(sm + s * C::STAGE);
      const unsigned fb = bar0 + 8u * s;
      tc::mbar_expect(fb, (unsigned)C::STAGE);
      tc::bulk_g2s(dst, a.W + ((size_t)tile * a.nslab + slab(i)) * GT_SLAB, GT_SLAB, fb, pw);
      tc::bulk_g2s(dst + GT_SLAB, a.X + (size_t)slab(i) * C::BBYTES, C::BBYTES, fb, px);
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
  const int grow = tile * GT_M + row;
  const float sw0 = a.sw[grow];   // this thread's row scale
  auto yval = [&](int b, const int (&v)[NPL], float sw) -> float { return dequant<NPL>(v, xs_s[b], sw); };
  if constexpr (S > 1) {
    // split K over the cluster's CTAs
    if constexpr (NPL == 1) split_push<S, MODE>(a, sm, xs_s, taddr, ok, ns, tile, row, grow, sw0);
    else split_epilogue<NPL, S, MODE>(a, sm, xs_s, taddr, ok, tile, row, grow, sw0);
  } else if (ok) {
    // one CTA per tile: the sums straight from TMEM, 16 tokens at a time (all
    // planes' loads in flight before the wait)
    tc::fence_after();
    unsigned rall[NPL == 1 ? 64 : 1];   // W8A8: all 64 sums requested before one wait
    if constexpr (NPL == 1) {
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld16(taddr + 16 * c, *reinterpret_cast<unsigned(*)[16]>(rall + 16 * c));
      tc::tmem_ld_wait();
    }
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 16) {
      unsigned r[NPL][16];
      if constexpr (NPL == 1) {
#pragma unroll
        for (int e = 0; e < 16; ++e) r[0][e] = rall[c0 + e];
      } else {
#pragma unroll
        for (int p = 0; p < NPL; ++p) tc::tmem_ld16(taddr + 64 * p + c0, r[p]);
        tc::tmem_ld_wait();
      }
      float yv[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        int v[NPL];
#pragma unroll
        for (int p = 0; p < NPL; ++p) v[p] = (int)r[p][e];
        yv[e] = yval(c0 + e, v, sw0);
        if (NPL == 1 && a.acc_out && c0 + e < a.nb && grow < a.nrows)
          a.acc_out[(size_t)(c0 + e) * a.nrows + grow] = v[0];
      }
      emit_rows<MODE, 16>(a, yv, c0, max(0, min(16, a.nb - c0)), tile, row, grow, reinterpret_cast<float*>(sm));
    }
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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

constexpr int AT_BLK = 32;                        // positions per staged block
constexpr int AT_NST = 3;                         // staged blocks in flight (one CTA per SM)
constexpr int AT_CW = 8;                          // compute warps; one more warp loads
constexpr int AT_U = AT_BLK / AT_CW;              // positions per warp per block
constexpr int AT_THREADS = 32 * (AT_CW + 1);
constexpr int AT_KB = AT_BLK * HD * 4;            // K (or V) rows of a block
constexpr int AT_STAGE = 2 * AT_KB;               // K rows, then V rows
constexpr int AT_PROW = 4 + HD;                   // partial row: m, l, 2 pad, o[256]
constexpr int AT_OFF_Q = AT_NST * AT_STAGE;       // qn [4][256]
constexpr int AT_OFF_KN = AT_OFF_Q + 4 * HD * 4;  // kn [256]
constexpr int AT_OFF_VN = AT_OFF_KN + HD * 4;     // vn [256]
constexpr int AT_OFF_MRG = AT_OFF_VN + HD * 4;    // per-warp partials of four warps [4][4][AT_PROW]
constexpr int AT_OFF_BAR = AT_OFF_MRG + 4 * 4 * AT_PROW * 4;
constexpr int AT_SMEM = AT_OFF_BAR + 16 * AT_NST;
static_assert(AT_STAGE % 1024 == 0 && AT_OFF_BAR % 8 == 0, "attention smem alignment");
static_assert(AT_SMEM <= 227 * 1024, "attention shared memory");

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

__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, %0;" :: "n"(32 * AT_CW) : "memory"); }

// Item (token b, KV group g, chunk cc) of the persistent attention kernel's
// stride loop; false if the chunk is empty.
struct AtItem {
  int b, g, cc, T, pos, t0, t1, tcache, nblk;
};
// The i-th block an item's CTA stages: the chunk's blocks in an order rotated
// by the CTA index, so that concurrent CTAs stream different offsets of their
// chunks (the online softmax does not depend on the order).
__device__ __forceinline__ int at_block(const AtItem& it, int i) {
  const int r = (int)(blockIdx.x * 7u % (unsigned)it.nblk);
  const int j = i + r;
  return j >= it.nblk ? j - it.nblk : j;
}
__device__ __forceinline__ bool at_item(const BtCtl& C, int item, int nchm, AtItem& it) {
  it.cc = item % nchm;
  it.g = (item / nchm) % NKV;
  it.b = item / (nchm * NKV);
  it.T = C.T[it.b];
  it.pos = C.pos[it.b];
  it.t0 = it.cc * AT_CL;
  if (it.t0 >= it.T + 1) return false;
  it.t1 = min(it.T + 1, it.t0 + AT_CL);
  it.tcache = min(it.t1, it.T);
  it.nblk = (it.t1 - it.t0 + AT_BLK - 1) / AT_BLK;
  return true;
}

// Split-KV attention (golden/model.py:194-229), persistent over items (token
// b, KV group g, 256-position chunk cc).  Warp 8 stages the chunk's cached K
// and V rows, 32 positions per block, into a three-block ring (bulk copies);
// the eight compute warps each take positions w, w + 8, ... of every block for
// all four query heads of the group: lane = 8 dims, the four 256-dim scores
// by butterfly sums, an online softmax per warp and head (running max m, sum
// l, output o).  At the chunk's end the warps' (m, l, o) merge, four warps at
// a time through shared memory, in warp order (online: M, L = L a + l_w e,
// O = O a + o_w e) into the chunk's partial.  The new token's key and value (position T) come
// from this CTA's own QK-norm + RoPE; the chunk holding T writes them to
// cache slot T.
__global__ void __launch_bounds__(AT_THREADS, 1) k_bt_attn(const AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  float* qn = reinterpret_cast<float*>(sm + AT_OFF_Q);
  float* kn = reinterpret_cast<float*>(sm + AT_OFF_KN);
  float* vn = reinterpret_cast<float*>(sm + AT_OFF_VN);
  float* mrg = reinterpret_cast<float*>(sm + AT_OFF_MRG);
  const unsigned bar0 = tc::smem_u32(sm + AT_OFF_BAR);   // full[s]; empty[s] at + 8 (NST + s)
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  if (t == 0) {
    for (int s = 0; s < AT_NST; ++s) {
      tc::mbar_init(bar0 + 8u * s, 1);
      tc::mbar_init(bar0 + 8u * (AT_NST + s), AT_CW);
    }
    tc::mbar_init_fence();
  }
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
  tc::grid_wait();
  __syncthreads();
  const BtCtl& C = *a.ctl;
  const int nchm = C.nchmax, nitems = C.nb * NKV * nchm;
  if (wid == AT_CW) {
    // loader: every block of this CTA's items, in order
    if (lane == 0) {
      const unsigned long long pol = tc::policy_evict_first();
      unsigned n = 0;
      bool good = true;
      for (int item = blockIdx.x; item < nitems && good; item += gridDim.x) {
        AtItem it;
        if (!at_item(C, item, nchm, it)) continue;
        const size_t kvoff = (((size_t)it.b * NFULL + a.fi) * NKV + it.g) * (size_t)a.max_ctx * HD;
        for (int i = 0; i < it.nblk; ++i, ++n) {
          const unsigned s = n % AT_NST;
          if (n >= AT_NST && !tc::mbar_wait(bar0 + 8u * (AT_NST + s), ((n / AT_NST) - 1) & 1u, a.err, 52, (int)n)) {
            good = false;
            break;
          }
          const int s0 = it.t0 + at_block(it, i) * AT_BLK;
          const int nbc = max(0, min(AT_BLK, it.tcache - s0));
          const unsigned kb = tc::smem_u32(sm + s * AT_STAGE), fb = bar0 + 8u * s;
          tc::mbar_expect(fb, (unsigned)(2 * nbc * HD * 4));
          if (nbc > 0) {
            tc::bulk_g2s(kb, a.kc + kvoff + (size_t)s0 * HD, (unsigned)(nbc * HD * 4), fb, pol);
            tc::bulk_g2s(kb + AT_KB, a.vc + kvoff + (size_t)s0 * HD, (unsigned)(nbc * HD * 4), fb, pol);
          }
        }
      }
      // every staged block is consumed before the CTA ends (the compute warps'
      // empty arrivals of the last blocks)
      for (unsigned u = n > AT_NST ? n - AT_NST : 0; u < n && good; ++u)
        if (!tc::mbar_wait(bar0 + 8u * (AT_NST + u % AT_NST), (u / AT_NST) & 1u, a.err, 53, (int)u)) break;
    }
    __syncwarp();
  } else {
    unsigned n = 0;
    bool good = true;
    for (int item = blockIdx.x; item < nitems && good; item += gridDim.x) {
      AtItem it;
      if (!at_item(C, item, nchm, it)) continue;
      // this token's q (4 heads of group g), k and v: RMSNorm + RoPE (golden/model.py:203-214)
      const float* y = a.Y + (size_t)it.b * a.ldy;
      const float* rope = a.rope + (size_t)it.pos * ROT;
      if (wid < 4) norm_rope_warp(y + (4 * it.g + wid) * 2 * HD, a.qn_w, rope[lane], rope[32 + lane], qn + wid * HD);
      else if (wid == 4) norm_rope_warp(y + QPROJ + it.g * HD, a.kn_w, rope[lane], rope[32 + lane], kn);
      else if (wid == 5) for (int e = lane; e < HD; e += 32) vn[e] = y[QPROJ + KVPROJ + it.g * HD + e];
      bar_compute();
      float qr[4][8];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float4 u0 = *reinterpret_cast<const float4*>(qn + h * HD + 8 * lane);
        const float4 u1 = *reinterpret_cast<const float4*>(qn + h * HD + 8 * lane + 4);
        qr[h][0] = u0.x; qr[h][1] = u0.y; qr[h][2] = u0.z; qr[h][3] = u0.w;
        qr[h][4] = u1.x; qr[h][5] = u1.y; qr[h][6] = u1.z; qr[h][7] = u1.w;
      }
      // running max / sum of head (lane >> 1) & 3 in every lane; o: every head, this lane's 8 dims
      float mh = -INFINITY, lh = 0.0f, o[4][8];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) o[h][j] = 0.0f;
      for (int i = 0; i < it.nblk; ++i, ++n) {
        const unsigned s = n % AT_NST;
        if (!tc::mbar_wait(bar0 + 8u * s, (n / AT_NST) & 1u, a.err, 50, item)) { good = false; break; }
        const int s0 = it.t0 + at_block(it, i) * AT_BLK;
        const int nbk = min(AT_BLK, it.t1 - s0);
        const float* kb = reinterpret_cast<const float*>(sm + s * AT_STAGE);
        const float* vb = kb + AT_BLK * HD;
        // this warp's two positions of the block
        float sc[AT_U][4], vv[AT_U][8];
#pragma unroll
        for (int u = 0; u < AT_U; ++u) {
          const int p = wid + AT_CW * u;
          const bool live = p < nbk;
          const bool fresh = s0 + p == it.T;   // the new token: k, v from this CTA
          const float* kr = fresh ? kn : kb + p * HD;
          const float* vr = fresh ? vn : vb + p * HD;
          float kk[8];
          if (live) {
            const float4 k0 = *reinterpret_cast<const float4*>(kr + 8 * lane);
            const float4 k1 = *reinterpret_cast<const float4*>(kr + 8 * lane + 4);
            const float4 v0 = *reinterpret_cast<const float4*>(vr + 8 * lane);
            const float4 v1 = *reinterpret_cast<const float4*>(vr + 8 * lane + 4);
            kk[0] = k0.x; kk[1] = k0.y; kk[2] = k0.z; kk[3] = k0.w; kk[4] = k1.x; kk[5] = k1.y; kk[6] = k1.z; kk[7] = k1.w;
            vv[u][0] = v0.x; vv[u][1] = v0.y; vv[u][2] = v0.z; vv[u][3] = v0.w;
            vv[u][4] = v1.x; vv[u][5] = v1.y; vv[u][6] = v1.z; vv[u][7] = v1.w;
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) { kk[j] = 0.0f; vv[u][j] = 0.0f; }
          }
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float d = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) d = fmaf(qr[h][j], kk[j], d);
            sc[u][h] = d;
          }
        }
        // the 16 dot products (AT_U = 4 positions x 4 heads) summed over the
        // lanes by a reduce-scatter: at each level a lane keeps half of its
        // values and adds its partner's; lane 2 i, 2 i + 1 end with sum i
        // (i = 4 u + h)
        static_assert(AT_U == 4, "reduce-scatter of 16 sums");
        float w8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const bool hi = lane & 16;
          const float mine = hi ? sc[(8 + k) >> 2][(8 + k) & 3] : sc[k >> 2][k & 3];
          const float oth = hi ? sc[k >> 2][k & 3] : sc[(8 + k) >> 2][(8 + k) & 3];
          w8[k] = mine + __shfl_xor_sync(0xffffffffu, oth, 16);
        }
        float w4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const bool hi = lane & 8;
          w4[k] = (hi ? w8[4 + k] : w8[k]) + __shfl_xor_sync(0xffffffffu, hi ? w8[k] : w8[4 + k], 8);
        }
        float w2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const bool hi = lane & 4;
          w2[k] = (hi ? w4[2 + k] : w4[k]) + __shfl_xor_sync(0xffffffffu, hi ? w4[k] : w4[2 + k], 4);
        }
        const bool h2 = lane & 2;
        float w1 = (h2 ? w2[1] : w2[0]) + __shfl_xor_sync(0xffffffffu, h2 ? w2[0] : w2[1], 2);
        w1 += __shfl_xor_sync(0xffffffffu, w1, 1);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar0 + 8u * (AT_NST + s));   // (the rows are in registers)
        // this lane's (position u, head h): score scaled by 256^-0.5 = 1/16
        // (exact); the head's max over the warp's four positions (lanes ^ 8,
        // ^ 16), online softmax update of the head's running max / sum
        const int iu = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
        const float sv = wid + AT_CW * iu < nbk ? __fmul_rn(w1, 0.0625f) : -INFINITY;
        float mx = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float mn = fmaxf(mh, mx);
        const float al = mh == -INFINITY ? (mn == -INFINITY ? 1.0f : 0.0f) : expf(mh - mn);
        const float e = sv == -INFINITY ? 0.0f : expf(sv - mn);
        float es = e + __shfl_xor_sync(0xffffffffu, e, 8);
        es += __shfl_xor_sync(0xffffffffu, es, 16);
        lh = fmaf(lh, al, es);
        mh = mn;
        // P V: every lane updates its 8 dims of the four heads
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float ah = __shfl_sync(0xffffffffu, al, 2 * h);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[h][j] = __fmul_rn(o[h][j], ah);
#pragma unroll
          for (int u = 0; u < AT_U; ++u) {
            const float pe = __shfl_sync(0xffffffffu, e, 2 * (4 * u + h));
#pragma unroll
            for (int j = 0; j < 8; ++j) o[h][j] = fmaf(pe, vv[u][j], o[h][j]);
          }
        }
      }
      if (!good) break;
      if (it.t1 == it.T + 1) {
        // roped K and raw V into slot T (golden/model.py:216-217)
        const size_t kvoff = (((size_t)it.b * NFULL + a.fi) * NKV + it.g) * (size_t)a.max_ctx * HD;
        a.kc[kvoff + (size_t)it.T * HD + t] = kn[t];
        a.vc[kvoff + (size_t)it.T * HD + t] = vn[t];
      }
      // the warps' (m, l, o), four warps per round; thread t = dim t of every head
      float M[4], Ls[4], O[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) { M[h] = -INFINITY; Ls[h] = 0.0f; O[h] = 0.0f; }
#pragma unroll
      for (int rnd = 0; rnd < 2; ++rnd) {
        if ((wid >> 2) == rnd) {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float* mw = mrg + ((wid & 3) * 4 + h) * AT_PROW;
            const float m_h = __shfl_sync(0xffffffffu, mh, 2 * h), l_h = __shfl_sync(0xffffffffu, lh, 2 * h);
            if (lane == 0) { mw[0] = m_h; mw[1] = l_h; }
            *reinterpret_cast<float4*>(mw + 4 + 8 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
            *reinterpret_cast<float4*>(mw + 8 + 8 * lane) = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
          }
        }
        bar_compute();
#pragma unroll
        for (int h = 0; h < 4; ++h)
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float* mw = mrg + (w * 4 + h) * AT_PROW;
            const float mq = mw[0];
            if (mq == -INFINITY) continue;   // a warp without positions
            const float Mn = fmaxf(M[h], mq);
            const float sa = M[h] == -INFINITY ? 0.0f : expf(M[h] - Mn), sb = expf(mq - Mn);
            Ls[h] = fmaf(mw[1], sb, __fmul_rn(Ls[h], sa));
            O[h] = fmaf(mw[4 + t], sb, __fmul_rn(O[h], sa));
            M[h] = Mn;
          }
        if (rnd == 0) bar_compute();   // the second merge pass rewrites the buffer
      }
      float* pr = a.part + ((((size_t)it.b * NKV + it.g) * a.maxch + it.cc) * 4) * AT_PROW;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        pr[h * AT_PROW + 4 + t] = O[h];
        if (t == 0) { pr[h * AT_PROW] = M[h]; pr[h * AT_PROW + 1] = Ls[h]; }
      }
    }
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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

// ---------------------------------------------------------------- prefill (one sequence, n tokens)
//
// A prompt chunk of n <= PF_MAX tokens of ONE sequence runs through the
// layers at once: the projections are the batched GEMMs with N = the chunk's
// tokens; the DeltaNet mixer is the chunked delta rule (below); attention
// appends the chunk's keys and values to the cache and attends causally.

constexpr int PF_MAX = 32;   // tokens per prefill chunk

struct PfDeltaArgs {
  const float* Y; int ldy;       // in-proj outputs of the chunk: qkv [0, 6144), z [6144, 8192)
  const float* AB;               // [n][32]: b rows, then a rows
  float* conv; float* rec;       // the sequence's conv ring [18][6144][4] and state [18][16][128][128]
  int lin, base, n;              // linear layer, ring origin before the chunk, tokens
  const float* conv_w; const float* A_log; const float* dt_bias; const float* gnorm_w;
  float* O;                      // [n][VDIM] gated-normed outputs
};
// dynamic shared memory of k_pf_delta (floats)
constexpr int PFD_QS = 0, PFD_KS = PFD_QS + PF_MAX * LK, PFD_VS = PFD_KS + PF_MAX * LK, PFD_U = PFD_VS + PF_MAX * LV,
              PFD_PART = PFD_U + PF_MAX * LV, PFD_A = PFD_PART + 4 * PF_MAX * LV, PFD_QK = PFD_A + PF_MAX * PF_MAX,
              PFD_G = PFD_QK + PF_MAX * PF_MAX, PFD_BETA = PFD_G + PF_MAX, PFD_GL = PFD_BETA + PF_MAX,
              PFD_W = PFD_GL + PF_MAX, PFD_WSQ = PFD_W + PF_MAX, PFD_INV = PFD_WSQ + PF_MAX * 8,
              PFD_GINV = PFD_INV + 2 * PF_MAX, PFD_FLOATS = PFD_GINV + PF_MAX;
constexpr int PFD_SMEM = PFD_FLOATS * 4;

// Chunked gated delta rule of head blockIdx.x over the chunk's n tokens
// (golden/model.py:149-189 for each token, restated in the WY form of the
// recurrence).  With G_t = g_0 + ... + g_t (log decay), Gamma_t = e^{G_t} and
// S the state before the chunk, the recurrence S_t = e^{g_t} S_{t-1} + k_t d_t^T,
// d_t = beta_t (v_t - (e^{g_t} S_{t-1})^T k_t), o_t = S_t^T q_t unrolls to
//   d_t = beta_t (v_t - Gamma_t S^T k_t) - sum_{s<t} beta_t e^{G_t - G_s} (k_t . k_s) d_s
//   o_t = Gamma_t S^T q_t + sum_{s<=t} e^{G_t - G_s} (q_t . k_s) d_s
//   S_n = Gamma_{n-1} S + sum_t e^{G_{n-1} - G_t} k_t d_t^T,
// so the chunk needs one triangular solve for d and a few dense products; the
// state is read and written once.  512 threads: conv + SiLU (threads 0-383,
// one channel each, every token), gates (384 + t), l2norm per token as the
// decode step does it, then the products with thread (v = t % 128, row group
// t / 128) holding 32 state rows of column v.
__global__ void __launch_bounds__(NT) k_pf_delta(const PfDeltaArgs a) {
  extern __shared__ __align__(16) float smf[];
  float* qs = smf + PFD_QS;      // [t][128]
  float* ks = smf + PFD_KS;
  float* vs = smf + PFD_VS;      // v, later o
  float* U = smf + PFD_U;        // d_t
  float* part = smf + PFD_PART;  // [4][t][128]
  float* Am = smf + PFD_A;       // [t][s]
  float* QK = smf + PFD_QK;      // [t][s]
  float* G = smf + PFD_G;
  float* beta = smf + PFD_BETA;
  float* gl = smf + PFD_GL;
  float* wt = smf + PFD_W;       // e^{G_{n-1} - G_t}
  float* wsq = smf + PFD_WSQ;    // [t][8] warp sums of squares
  float* inv = smf + PFD_INV;    // [2][t]
  float* ginv = smf + PFD_GINV;  // [t]
  const int h = blockIdx.x, t = threadIdx.x, n = a.n, lane = t & 31, wid = t >> 5;
  const int vi = t & (LV - 1), kg = t / LV;
  constexpr int KPG = LK / 4;
  tc::grid_launch_dependents();
  tc::grid_wait();
  float* Sh = a.rec + ((size_t)a.lin * LH + h) * LK * LV;
  float sv[KPG];
#pragma unroll
  for (int kk = 0; kk < KPG; ++kk) sv[kk] = Sh[(size_t)(kg * KPG + kk) * LV + vi];
  // conv over [x_{t-3}, x_{t-2}, x_{t-1}, x_t] (history from the ring) + SiLU
  if (t < 3 * LK) {
    const int c = t & (LK - 1);
    const int ch = t < LK ? h * LK + c : (t < 2 * LK ? KDIM + h * LK + c : 2 * KDIM + h * LV + c);
    float* dst = t < LK ? qs : (t < 2 * LK ? ks : vs);
    float* st = a.conv + ((size_t)a.lin * CONVD + ch) * CONVK;
    const int base = a.base;
    float h1 = st[(base + 1) & 3], h2 = st[(base + 2) & 3], h3 = st[(base + 3) & 3];
    const float4 w4 = *reinterpret_cast<const float4*>(a.conv_w + (size_t)ch * CONVK);
    for (int tt = 0; tt < n; ++tt) {
      const float nv = a.Y[(size_t)tt * a.ldy + ch];
      float acc = __fmul_rn(h1, w4.x);
      acc = __fadd_rn(acc, __fmul_rn(h2, w4.y));
      acc = __fadd_rn(acc, __fmul_rn(h3, w4.z));
      acc = __fadd_rn(acc, __fmul_rn(nv, w4.w));
      dst[tt * LK + c] = silu_f(acc);
      h1 = h2; h2 = h3; h3 = nv;
    }
    // the ring as n decode steps leave it: input j in slot (base + j) & 3
    for (int j = max(0, n - 4); j < n; ++j) st[(base + j) & 3] = a.Y[(size_t)j * a.ldy + ch];
  } else if (t < 3 * LK + n) {
    const int tt = t - 3 * LK;
    beta[tt] = sigmoid_f(a.AB[tt * 32 + h]);
    gl[tt] = __fmul_rn(-expf(a.A_log[h]), softplus_f(__fadd_rn(a.AB[tt * 32 + 16 + h], a.dt_bias[h])));
  }
  __syncthreads();
  if (t == 0) {
    float acc = 0.0f;
    for (int tt = 0; tt < n; ++tt) { acc = __fadd_rn(acc, gl[tt]); G[tt] = acc; }
  }
  // l2norm of q (warps 0-3) and k (warps 4-7) per token, as the decode step
  if (t < 2 * LK) {
    const float* src = t < LK ? qs : ks;
    for (int tt = 0; tt < n; ++tt) {
      const float x = src[tt * LK + (t & (LK - 1))];
      const float ss = warp_sum(x * x);
      if (lane == 0) wsq[tt * 8 + wid] = ss;
    }
  }
  __syncthreads();
  if (t < 2 * PF_MAX) {
    const int tt = t % PF_MAX, g0 = t < PF_MAX ? 0 : 4;
    if (tt < n) {
      const float tot = ((wsq[tt * 8 + g0] + wsq[tt * 8 + g0 + 1]) + wsq[tt * 8 + g0 + 2]) + wsq[tt * 8 + g0 + 3];
      inv[(t < PF_MAX ? 0 : PF_MAX) + tt] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(tot, EPS)));
    }
  }
  if (t == 64) for (int tt = 0; tt < n; ++tt) wt[tt] = 0.0f;
  __syncthreads();
  if (t < 2 * LK) {
    float* dst = t < LK ? qs : ks;
    const int c = t & (LK - 1);
    for (int tt = 0; tt < n; ++tt) {
      const float x = dst[tt * LK + c];
      dst[tt * LK + c] = t < LK ? __fmul_rn(__fmul_rn(x, inv[tt]), 0.08838834764831845f)
                                : __fmul_rn(x, inv[PF_MAX + tt]);
    }
  }
  if (t == 64) {
    const float Gl = G[n - 1];
    for (int tt = 0; tt < n; ++tt) wt[tt] = expf(Gl - G[tt]);
  }
  __syncthreads();
  // KK (strictly lower, scaled) and QK (lower with the diagonal): pair (tt, ss)
  // per thread, dims read from a lane-rotated start (no bank conflicts)
  for (int pidx = t; pidx < n * n; pidx += NT) {
    const int tt = pidx / n, ss = pidx - tt * n;
    float kk = 0.0f, qk = 0.0f;
    if (ss <= tt) {
      for (int d0 = 0; d0 < LK; ++d0) {
        const int d = (d0 + lane) & (LK - 1);
        const float ksd = ks[ss * LK + d];
        kk = fmaf(ks[tt * LK + d], ksd, kk);
        qk = fmaf(qs[tt * LK + d], ksd, qk);
      }
    }
    const float dec = ss <= tt ? expf(G[tt] - G[ss]) : 0.0f;
    Am[tt * PF_MAX + ss] = ss < tt ? __fmul_rn(__fmul_rn(beta[tt], dec), kk) : 0.0f;
    QK[tt * PF_MAX + ss] = ss <= tt ? __fmul_rn(dec, qk) : 0.0f;
  }
  // S^T k_t partials over this thread's 32 rows
  for (int tt = 0; tt < n; ++tt) {
    float p = 0.0f;
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk) p = fmaf(sv[kk], ks[tt * LK + kg * KPG + kk], p);
    part[(kg * PF_MAX + tt) * LV + vi] = p;
  }
  __syncthreads();
  // right-hand side beta_t (v_t - Gamma_t S^T k_t)
  for (int tt = kg; tt < n; tt += 4) {
    const float kv = ((part[(0 * PF_MAX + tt) * LV + vi] + part[(1 * PF_MAX + tt) * LV + vi]) +
                      part[(2 * PF_MAX + tt) * LV + vi]) + part[(3 * PF_MAX + tt) * LV + vi];
    U[tt * LV + vi] = __fmul_rn(beta[tt], __fsub_rn(vs[tt * LV + vi], __fmul_rn(expf(G[tt]), kv)));
  }
  __syncthreads();
  // forward substitution: d_t = r_t - sum_{s<t} A[t][s] d_s (threads 0-127, column vi)
  if (t < LV) {
    for (int tt = 1; tt < n; ++tt) {
      float u = U[tt * LV + vi];
      for (int ss = 0; ss < tt; ++ss) u = fmaf(-Am[tt * PF_MAX + ss], U[ss * LV + vi], u);
      U[tt * LV + vi] = u;
    }
  }
  // S^T q_t partials
  for (int tt = 0; tt < n; ++tt) {
    float p = 0.0f;
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk) p = fmaf(sv[kk], qs[tt * LK + kg * KPG + kk], p);
    part[(kg * PF_MAX + tt) * LV + vi] = p;
  }
  __syncthreads();
  // o_t = Gamma_t S^T q_t + sum_{s<=t} QK[t][s] d_s (into vs)
  for (int tt = kg; tt < n; tt += 4) {
    const float sq = ((part[(0 * PF_MAX + tt) * LV + vi] + part[(1 * PF_MAX + tt) * LV + vi]) +
                      part[(2 * PF_MAX + tt) * LV + vi]) + part[(3 * PF_MAX + tt) * LV + vi];
    float o = __fmul_rn(expf(G[tt]), sq);
    for (int ss = 0; ss <= tt; ++ss) o = fmaf(QK[tt * PF_MAX + ss], U[ss * LV + vi], o);
    vs[tt * LV + vi] = o;
  }
  // the state after the chunk
  {
    const float gam = expf(G[n - 1]);
#pragma unroll
    for (int kk = 0; kk < KPG; ++kk) {
      const int k = kg * KPG + kk;
      float sval = __fmul_rn(sv[kk], gam);
      for (int tt = 0; tt < n; ++tt) sval = fmaf(__fmul_rn(wt[tt], ks[tt * LK + k]), U[tt * LV + vi], sval);
      Sh[(size_t)k * LV + vi] = sval;
    }
  }
  __syncthreads();
  // gated RMSNorm per token (golden/model.py:183-189), one warp per token
  for (int tt = wid; tt < n; tt += NW) {
    float s = 0.0f;
    for (int i = lane; i < LV; i += 32) s = fmaf(vs[tt * LV + i], vs[tt * LV + i], s);
    s = warp_sum(s);
    if (lane == 0) ginv[tt] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(s, 1.0f / LV), EPS)));
  }
  __syncthreads();
  for (int tt = kg; tt < n; tt += 4) {
    const float z = silu_f(a.Y[(size_t)tt * a.ldy + CONVD + h * LV + vi]);
    const float v = __fmul_rn(__fmul_rn(vs[tt * LV + vi], ginv[tt]), a.gnorm_w[vi]);
    a.O[(size_t)tt * VDIM + h * LV + vi] = __fmul_rn(v, z);
  }
}

struct PfAttnArgs {
  const float* Y; int ldy;       // in-proj outputs of the chunk: [q | gate] per head, k, v
  float* kc; float* vc;          // the sequence's cache, [6][max_ctx][512] (K after QK-norm + RoPE)
  int fi, max_ctx, T0, pos0, n;  // positions before the chunk; the chunk's first RoPE position
  const float* qn_w; const float* kn_w; const float* rope;
  float* QN;                     // [n][8][256] normed + roped queries
  float* O;                      // [n][VDIM]
};

// QK-norm + RoPE of token blockIdx.x's query heads of group blockIdx.y (warps
// 0-3) and its key (warp 4), value (warp 5) into cache slot T0 + token.
__global__ void __launch_bounds__(192) k_pf_kvprep(const PfAttnArgs a) {
  const int tt = blockIdx.x, g = blockIdx.y, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  tc::grid_launch_dependents();
  tc::grid_wait();
  const float* y = a.Y + (size_t)tt * a.ldy;
  const float* rope = a.rope + (size_t)(a.pos0 + tt) * ROT;
  const size_t row = ((size_t)a.fi * a.max_ctx + a.T0 + tt) * KVPROJ + (size_t)g * HD;
  if (wid < 4) norm_rope_warp(y + (4 * g + wid) * 2 * HD, a.qn_w, rope[lane], rope[32 + lane],
                              a.QN + ((size_t)tt * NH + 4 * g + wid) * HD);
  else if (wid == 4) norm_rope_warp(y + QPROJ + g * HD, a.kn_w, rope[lane], rope[32 + lane], a.kc + row);
  else for (int e = lane; e < HD; e += 32) a.vc[row + e] = y[QPROJ + KVPROJ + g * HD + e];
}

// Causal attention of token blockIdx.x of the chunk over cache positions
// [0, T0 + token], the four query heads of group blockIdx.y: warp w takes
// positions w, w + 8, ..., lane = 8 dims, online softmax per warp and head;
// the warps merge in shared memory (dynamic, 8 x 4 x AT_PROW floats), then
// o / l * sigmoid(gate) (golden/model.py:219-229).
__global__ void __launch_bounds__(256) k_pf_attn(const PfAttnArgs a) {
  extern __shared__ __align__(16) float mrg[];
  const int tt = blockIdx.x, g = blockIdx.y, t = threadIdx.x, lane = t & 31, wid = t >> 5;
  tc::grid_launch_dependents();
  tc::grid_wait();
  float qr[4][8];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float* q = a.QN + ((size_t)tt * NH + 4 * g + h) * HD + 8 * lane;
    const float4 u0 = *reinterpret_cast<const float4*>(q), u1 = *reinterpret_cast<const float4*>(q + 4);
    qr[h][0] = u0.x; qr[h][1] = u0.y; qr[h][2] = u0.z; qr[h][3] = u0.w;
    qr[h][4] = u1.x; qr[h][5] = u1.y; qr[h][6] = u1.z; qr[h][7] = u1.w;
  }
  float m[4], l[4], o[4][8];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[h][j] = 0.0f;
  }
  const int npos = a.T0 + tt + 1;
  const float* kb = a.kc + (size_t)a.fi * a.max_ctx * KVPROJ + (size_t)g * HD + 8 * lane;
  const float* vb = a.vc + (size_t)a.fi * a.max_ctx * KVPROJ + (size_t)g * HD + 8 * lane;
  for (int p = wid; p < npos; p += 8) {
    const float4 k0 = *reinterpret_cast<const float4*>(kb + (size_t)p * KVPROJ);
    const float4 k1 = *reinterpret_cast<const float4*>(kb + (size_t)p * KVPROJ + 4);
    const float4 v0 = *reinterpret_cast<const float4*>(vb + (size_t)p * KVPROJ);
    const float4 v1 = *reinterpret_cast<const float4*>(vb + (size_t)p * KVPROJ + 4);
    const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
    const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float sc[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float d = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) d = fmaf(qr[h][j], kk[j], d);
      sc[h] = d;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int h = 0; h < 4; ++h) sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], off);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float sv = __fmul_rn(sc[h], 0.0625f);
      const float mn = fmaxf(m[h], sv);
      const float al = m[h] == -INFINITY ? 0.0f : expf(m[h] - mn);
      const float e = expf(sv - mn);
      l[h] = fmaf(l[h], al, e);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[h][j] = fmaf(e, vv[j], __fmul_rn(o[h][j], al));
      m[h] = mn;
    }
  }
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    float* mw = mrg + (wid * 4 + h) * AT_PROW;
    if (lane == 0) { mw[0] = m[h]; mw[1] = l[h]; }
    *reinterpret_cast<float4*>(mw + 4 + 8 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
    *reinterpret_cast<float4*>(mw + 8 + 8 * lane) = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
  }
  __syncthreads();
  const float* y = a.Y + (size_t)tt * a.ldy;
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    float M = -INFINITY, L = 0.0f, Ov = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float* mw = mrg + (w * 4 + h) * AT_PROW;
      if (mw[0] == -INFINITY) continue;
      const float Mn = fmaxf(M, mw[0]);
      const float sa = M == -INFINITY ? 0.0f : expf(M - Mn), sb = expf(mw[0] - Mn);
      L = fmaf(mw[1], sb, __fmul_rn(L, sa));
      Ov = fmaf(mw[4 + t], sb, __fmul_rn(Ov, sa));
      M = Mn;
    }
    const float gt = y[(4 * g + h) * 2 * HD + HD + t];
    a.O[(size_t)tt * VDIM + (4 * g + h) * HD + t] = __fmul_rn(__fdiv_rn(Ov, L), sigmoid_f(gt));
  }
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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
  tc::grid_launch_dependents();   // dependents may launch (they wait for this grid before reading)
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

// Launch with programmatic dependent launch (the kernel's prologue may start
// while its predecessor drains; every kernel waits on griddepcontrol.wait
// before it reads what the predecessor wrote) and, for cluster_y > 0, a
// (1, cluster_y, 1) thread-block cluster.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                     int cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  int n = 0;
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 0) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = 1;
    at[n].val.clusterDim.y = (unsigned)cluster_y;
    at[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

using GemmKernel = void (*)(const GemmArgs);

template <int NPL, int MODE>
GemmKernel gemm_kernel_s(int S) {
  switch (S) {
    case 1: return k_bt_gemm<NPL, 1, MODE>;
    case 2: return k_bt_gemm<NPL, 2, MODE>;
    case 4: return k_bt_gemm<NPL, 4, MODE>;
    case 8: return k_bt_gemm<NPL, 8, MODE>;
    default: break;
  }
  if constexpr (MODE != EPI_SWIGLU) {
    switch (S) {
      case 3: return k_bt_gemm<NPL, 3, MODE>;
      case 5: return k_bt_gemm<NPL, 5, MODE>;
      case 6: return k_bt_gemm<NPL, 6, MODE>;
      case 7: return k_bt_gemm<NPL, 7, MODE>;
      default: break;
    }
  }
  return nullptr;
}
// The instance for `mode` and an S-CTA K split (null when not built).
template <int NPL>
GemmKernel gemm_kernel(int mode, int S) {
  if (mode == EPI_STORE) return gemm_kernel_s<NPL, EPI_STORE>(S);
  if (mode == EPI_ADD) return gemm_kernel_s<NPL, EPI_ADD>(S);
  if (mode == EPI_SWIGLU) return gemm_kernel_s<NPL, EPI_SWIGLU>(S);
  return nullptr;
}

template <int NPL>
cudaError_t launch_gemm(const GemmArgs& a, int ntiles, cudaStream_t st, bool pdl = false) {
  const int ny = (a.nslab + a.kspl - 1) / a.kspl;
  if (ny < 1 || ny > 8) return cudaErrorInvalidValue;
  const GemmKernel k = gemm_kernel<NPL>(a.mode, ny);
  if (!k) return cudaErrorInvalidValue;
  return launch_k(k, dim3(ntiles, ny, 1), dim3(128, 1, 1), GC<NPL>::SMEM, st, pdl, ny, a);
}

cudaError_t set_smem_attrs() {
  cudaError_t e;
  for (int mode = 0; mode < 3; ++mode)
    for (int S = 1; S <= 8; ++S) {
      if (GemmKernel k = gemm_kernel<1>(mode, S))
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, GC<1>::SMEM))) return e;
      if (GemmKernel k = gemm_kernel<3>(mode, S))
        if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, GC<3>::SMEM))) return e;
    }
  if ((e = cudaFuncSetAttribute(k_bt_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_bt_head, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_pf_delta, cudaFuncAttributeMaxDynamicSharedMemorySize, PFD_SMEM))) return e;
  if ((e = cudaFuncSetAttribute(k_pf_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4 * AT_PROW * 4))) return e;
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
  int* err = nullptr;
  std::vector<const int8_t*> hrows(N);
  for (int r = 0; r < N; ++r) hrows[r] = w + (size_t)r * K;
  // K split over a cluster: the fewest CTAs (at least two when there are two
  // slabs) whose K ranges fit the ring beside the receive buffer
  int kspl = nslab;
  for (int S = 2; S <= 8 && nslab >= 2; ++S) {
    const int k = (nslab + S - 1) / S;
    if (k <= push_max_slabs(S) && (nslab + k - 1) / k == S) { kspl = k; break; }
  }
  if ((e = cudaMallocAsync((void**)&tiles, (size_t)N * K, st)) ||
      (e = cudaMallocAsync((void**)&img, (size_t)nslab * 64 * GT_KS, st)) ||
      (e = cudaMallocAsync((void**)&rows, N * sizeof(void*), st)) ||
      (e = cudaMallocAsync((void**)&xs, 64 * 4, st)) || (e = cudaMallocAsync((void**)&err, 16, st)))
    return e;
  e = cudaMemcpyAsync(rows, hrows.data(), N * sizeof(void*), cudaMemcpyHostToDevice, st);
  if (!e) e = cudaMemsetAsync(xs, 0, 64 * 4, st);
  if (!e) e = cudaMemcpyAsync(xs, sx, B * 4, cudaMemcpyDeviceToDevice, st);
  if (!e) e = cudaMemsetAsync(err, 0, 16, st);
  if (!e) e = repack_tiles(rows, tiles, N, K, st);
  if (!e) {
    k_bt_image<<<64, 256, 0, st>>>(xq, img, B, K);
    e = cudaGetLastError();
  }
  GemmArgs a{};
  a.W = tiles; a.sw = sw; a.X = img; a.xs = xs;
  a.nslab = nslab; a.kspl = kspl; a.nb = B; a.mode = EPI_STORE;
  a.Y = y; a.ldy = N; a.acc_out = acc; a.nrows = N; a.err = err;
  if (!e) e = launch_gemm<1>(a, ntiles, st);
  int herr[4] = {0, 0, 0, 0};
  if (!e) e = cudaMemcpyAsync(herr, err, 16, cudaMemcpyDeviceToHost, st);
  if (!e) e = cudaStreamSynchronize(st);
  cudaFreeAsync(tiles, st); cudaFreeAsync(img, st); cudaFreeAsync(rows, st); cudaFreeAsync(xs, st);
  cudaFreeAsync(err, st);
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
  int ksplit_in = 8, ksplit_out = 2, ksplit_gu = 8, ksplit_down = 4;
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
    a.Y = Y; a.ldy = ldy; a.acc_out = nullptr; a.nrows = nrows; a.err = E->err;
    const int ny = (a.nslab + kspl - 1) / kspl;
    if (NPL == 1 && ny > 1 && kspl > push_max_slabs(ny)) { e = cudaErrorInvalidValue; return; }
    e = launch_gemm<NPL>(a, nrows / GT_M, st, true);
  };
  auto normq = [&](int l, bool embed, bool head) {
    if (e != cudaSuccess) return;
    NormqArgs a{};
    a.H = E->H; a.tok = embed ? E->tok : nullptr; a.emb_q = E->M.emb_q; a.emb_s = E->M.emb_s;
    a.err = E->err;
    if (head) {
      a.gain = E->M.final_norm;
      a.X = E->HX; a.xs = E->hxs;
      e = launch_k(k_bt_normq<3>, dim3(nb), dim3(NT), 0, st, true, 0, a);
      return;
    } else {
      const LayerW& Lw = E->M.L[l];
      a.gain = Lw.in_norm;
      if (Lw.linear) { a.a_w = Lw.a_w; a.b_w = Lw.b_w; a.AB = E->AB; }
      a.X = E->X; a.xs = E->xs;
      e = launch_k(k_bt_normq<NPL>, dim3(nb), dim3(NT), 0, st, true, 0, a);
    }
  };
  auto post_normq = [&](int l) {
    if (e != cudaSuccess) return;
    NormqArgs a{};
    a.H = E->H; a.gain = E->M.L[l].post_norm; a.X = E->X; a.xs = E->xs; a.err = E->err;
    e = launch_k(k_bt_normq<NPL>, dim3(nb), dim3(NT), 0, st, true, 0, a);
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
      if (e == cudaSuccess) e = launch_k(k_bt_delta, dim3(LH, nb), dim3(NT), 0, st, true, 0, d);
      if (e == cudaSuccess) e = launch_k(k_bt_quant<NPL>, dim3(nb), dim3(NT), 0, st, true, 0, (const float*)E->O, (int)VDIM, (int)VDIM, E->X, E->xs);
    } else {
      AttnArgs at{};
      at.Y = E->Y; at.ldy = LDY; at.kc = E->kc; at.vc = E->vc; at.fi = Lw.full_idx; at.max_ctx = E->max_ctx;
      at.qn_w = Lw.qn_w; at.kn_w = Lw.kn_w; at.rope = E->rope; at.ctl = E->dctl; at.part = E->attp;
      at.maxch = E->maxch; at.err = E->err;
      if (e == cudaSuccess) e = launch_k(k_bt_attn, dim3(E->sm_count), dim3(AT_THREADS), AT_SMEM, st, true, 0, at);
      if (e == cudaSuccess) {
        e = launch_k(k_bt_merge<NPL>, dim3(nb), dim3(NT), 0, st, true, 0, (const float*)E->Y, (int)LDY,
                     (const float*)E->attp, E->maxch, (const BtCtl*)E->dctl, E->X, E->xs);
      }
    }
    gemm(T.wout, T.swout, HID, VDIM, E->ksplit_out, EPI_ADD, E->H, HID);
    post_normq(l);
    gemm(T.wgu, T.swgu, 2 * FFN, HID, E->ksplit_gu, EPI_SWIGLU, E->O, FFN);
    if (e == cudaSuccess) e = launch_k(k_bt_quant<NPL>, dim3(nb), dim3(NT), 0, st, true, 0, (const float*)E->O, (int)FFN, (int)FFN, E->X, E->xs);
    gemm(T.wdown, T.swdown, HID, FFN, E->ksplit_down, EPI_ADD, E->H, HID);
    if (l + 1 < NLAYER) normq(l + 1, false, false);
  }
  normq(0, false, true);
  if (e == cudaSuccess) {
    HeadArgs h{};
    h.tiles = E->head_tiles; h.emb_s = E->M.emb_s; h.HX = E->HX; h.hxs = E->hxs; h.ctl = E->dctl;
    h.logits = E->logits; h.am = E->am; h.err = E->err;
    e = launch_k(k_bt_head, dim3(E->head_grid), dim3(HB_THREADS), HB_SMEM, st, true, 0, h);
  }
  if (e == cudaSuccess) {
    e = launch_k(k_bt_finish, dim3(nb), dim3(32), 0, st, true, 0, (const unsigned long long*)E->am, E->head_grid,
                 E->ids, E->tok);
  }
  return e;
}

// One prefill chunk of n tokens (E->tok) of one sequence whose arrays are
// conv / rec / kc / vc (the batch-1 layouts); head: the last token's logits,
// argmax into E->ids[0] (E->dctl: nb = 1).
template <int NPL>
cudaError_t enqueue_prefill(BatchEngine* E, float* conv, float* rec, float* kc, float* vc, int max_ctx, int base, int T0,
                            int pos0, int n, bool head) {
  cudaStream_t st = E->st;
  cudaError_t e = cudaSuccess;
  constexpr int LDY = 8192;
  auto gemm = [&](const int8_t* W, const float* sw, int nrows, int K, int kspl, int mode, float* Y, int ldy) {
    if (e != cudaSuccess) return;
    GemmArgs a{};
    a.W = W; a.sw = sw; a.X = E->X; a.xs = E->xs;
    a.nslab = K / GT_KS; a.kspl = kspl; a.nb = n; a.mode = mode;
    a.Y = Y; a.ldy = ldy; a.acc_out = nullptr; a.nrows = nrows; a.err = E->err;
    e = launch_gemm<NPL>(a, nrows / GT_M, st, true);
  };
  auto normq = [&](int l, bool embed) {
    if (e != cudaSuccess) return;
    NormqArgs a{};
    const LayerW& Lw = E->M.L[l];
    a.H = E->H; a.tok = embed ? E->tok : nullptr; a.emb_q = E->M.emb_q; a.emb_s = E->M.emb_s; a.err = E->err;
    a.gain = Lw.in_norm;
    if (Lw.linear) { a.a_w = Lw.a_w; a.b_w = Lw.b_w; a.AB = E->AB; }
    a.X = E->X; a.xs = E->xs;
    e = launch_k(k_bt_normq<NPL>, dim3(n), dim3(NT), 0, st, true, 0, a);
  };
  auto quant = [&](const float* src, int K) {
    if (e == cudaSuccess) e = launch_k(k_bt_quant<NPL>, dim3(n), dim3(NT), 0, st, true, 0, src, K, K, E->X, E->xs);
  };
  normq(0, true);
  for (int l = 0; l < NLAYER && e == cudaSuccess; ++l) {
    const LayerW& Lw = E->M.L[l];
    const LayerTiles& T = E->L[l];
    gemm(T.win, T.swin, T.nin, HID, E->ksplit_in, EPI_STORE, E->Y, LDY);
    if (Lw.linear) {
      PfDeltaArgs d{};
      d.Y = E->Y; d.ldy = LDY; d.AB = E->AB; d.conv = conv; d.rec = rec; d.lin = Lw.lin_idx; d.base = base; d.n = n;
      d.conv_w = Lw.conv_w; d.A_log = Lw.A_log; d.dt_bias = Lw.dt_bias; d.gnorm_w = Lw.gnorm_w; d.O = E->O;
      if (e == cudaSuccess) e = launch_k(k_pf_delta, dim3(LH), dim3(NT), PFD_SMEM, st, true, 0, d);
    } else {
      PfAttnArgs at{};
      at.Y = E->Y; at.ldy = LDY; at.kc = kc; at.vc = vc; at.fi = Lw.full_idx; at.max_ctx = max_ctx;
      at.T0 = T0; at.pos0 = pos0; at.n = n; at.qn_w = Lw.qn_w; at.kn_w = Lw.kn_w; at.rope = E->rope;
      at.QN = E->attp; at.O = E->O;
      if (e == cudaSuccess) e = launch_k(k_pf_kvprep, dim3(n, NKV), dim3(192), 0, st, true, 0, at);
      if (e == cudaSuccess)
        e = launch_k(k_pf_attn, dim3(n, NKV), dim3(256), (size_t)8 * 4 * AT_PROW * 4, st, true, 0, at);
    }
    quant(E->O, VDIM);
    gemm(T.wout, T.swout, HID, VDIM, E->ksplit_out, EPI_ADD, E->H, HID);
    if (e == cudaSuccess) {
      NormqArgs a{};
      a.H = E->H; a.gain = Lw.post_norm; a.X = E->X; a.xs = E->xs; a.err = E->err;
      e = launch_k(k_bt_normq<NPL>, dim3(n), dim3(NT), 0, st, true, 0, a);
    }
    gemm(T.wgu, T.swgu, 2 * FFN, HID, E->ksplit_gu, EPI_SWIGLU, E->O, FFN);
    quant(E->O, FFN);
    gemm(T.wdown, T.swdown, HID, FFN, E->ksplit_down, EPI_ADD, E->H, HID);
    if (l + 1 < NLAYER) normq(l + 1, false);
  }
  if (head && e == cudaSuccess) {
    NormqArgs a{};
    a.H = E->H + (size_t)(n - 1) * HID; a.gain = E->M.final_norm; a.X = E->HX; a.xs = E->hxs; a.err = E->err;
    e = launch_k(k_bt_normq<3>, dim3(1), dim3(NT), 0, st, true, 0, a);
    HeadArgs h{};
    h.tiles = E->head_tiles; h.emb_s = E->M.emb_s; h.HX = E->HX; h.hxs = E->hxs; h.ctl = E->dctl;
    h.logits = E->logits; h.am = E->am; h.err = E->err;
    if (e == cudaSuccess) e = launch_k(k_bt_head, dim3(E->head_grid), dim3(HB_THREADS), HB_SMEM, st, true, 0, h);
    if (e == cudaSuccess)
      e = launch_k(k_bt_finish, dim3(1), dim3(32), 0, st, true, 0, (const unsigned long long*)E->am, E->head_grid,
                   E->ids, E->tok);
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
      (e = balloc(E, &E->attp, std::max(B * NKV * E->maxch * 4 * AT_PROW, (size_t)PF_MAX * NH * HD) * 4)) ||
      (e = balloc(E, &E->logits, (size_t)BATCH_MAX * VOCAB * 4)) ||
      (e = balloc(E, &E->X, (size_t)(FFN / GT_KS) * 192 * GT_KS)) || (e = balloc(E, &E->HX, (size_t)HB_IMG)) ||
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

namespace qb {

int batch_prefill(BatchEngine* E, float* conv, float* rec, float* kc, float* vc, int max_ctx, int conv_base, int T0,
                  int pos0, const int* tok, int n, bool act_int8, float* logits_out, int* argmax_out, std::string& err) {
  if (n < 1 || !tok) {
    err = "prefill: need n >= 1 tokens";
    return QWEN_ERR_ARG;
  }
  for (int i = 0; i < n; ++i)
    if (tok[i] < 0 || tok[i] >= VOCAB) {
      err = "prefill: token id out of range";
      return QWEN_ERR_ARG;
    }
  if (T0 + n > max_ctx || pos0 + n > E->max_rope) {
    err = "prefill: the context would overflow max_ctx";
    return QWEN_ERR_STATE;
  }
  cudaStream_t st = E->st;
  memset(E->hctl, 0, sizeof(BtCtl));
  E->hctl->nb = 1;
  E->hctl->want_logits = logits_out ? 1 : 0;
  BCUDA(cudaMemcpyAsync(E->dctl, E->hctl, sizeof(BtCtl), cudaMemcpyHostToDevice, st));
  for (int c0 = 0; c0 < n; c0 += PF_MAX) {
    const int nc = std::min(PF_MAX, n - c0);
    BCUDA(cudaStreamSynchronize(st));   // the pinned token slot is rewritten
    memcpy(E->hbuf, tok + c0, nc * sizeof(int));
    BCUDA(cudaMemcpyAsync(E->tok, E->hbuf, nc * sizeof(int), cudaMemcpyHostToDevice, st));
    const bool last = c0 + nc == n;
    BCUDA(act_int8 ? enqueue_prefill<1>(E, conv, rec, kc, vc, max_ctx, conv_base + c0, T0 + c0, pos0 + c0, nc, last)
                   : enqueue_prefill<3>(E, conv, rec, kc, vc, max_ctx, conv_base + c0, T0 + c0, pos0 + c0, nc, last));
  }
  int* hid = E->hbuf + BATCH_MAX;
  BCUDA(cudaMemcpyAsync(hid, E->ids, sizeof(int), cudaMemcpyDeviceToHost, st));
  if (logits_out) BCUDA(cudaMemcpyAsync(logits_out, E->logits, (size_t)VOCAB * 4, cudaMemcpyDefault, st));
  if (int rc = read_err(E, err)) return rc;
  if (argmax_out) *argmax_out = hid[0];
  return QWEN_OK;
}

}  // namespace qb
