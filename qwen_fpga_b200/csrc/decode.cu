// Decode-step kernels of libqwenb200: one token of the Qwen3.5-0.8B hybrid
// decoder, as a fixed program of phases.  Each phase reads the previous
// phase's outputs from global memory and computes its own GEMV input in a
// prologue (redundantly per CTA, from 4-14 KB of L2-resident data), so no
// phase needs a separate normalisation kernel:
//
//   linear layer  : IN (rmsnorm -> qkv|z|b|a)  DELTA (conv, gates, l2norm, delta
//                   rule)  OUT (gated norm -> out_proj, + residual)
//   full layer    : IN (rmsnorm -> q|k|v)  ATTN (QK-norm, RoPE, KV append,
//                   split-KV softmax, combine)  OPROJ (sigmoid gate -> o_proj, + residual)
//   every layer   : GATEUP (rmsnorm -> silu(gate)*up)  DOWN (down_proj, + residual)
//   head          : HEAD (final rmsnorm -> tied int8 head, block argmax)  FINISH
//
// Sequencer: golden/model.py:243-267 decode_step, hls/src/qwen_synth.hpp:39-92.
#include <cstdio>

#include "common.cuh"
#include "decode.cuh"

namespace qb {

// ---------------------------------------------------------------- prologues

// token of the current step: prompt tokens first, then greedy feedback of the
// previous step's argmax (golden/model.py:270-280).
__device__ __forceinline__ int step_token(const StateW& S) {
  const int step = S.io[0], np = S.io[1];
  int t = (step < np) ? S.io[2 + step] : S.ids[step > 0 ? step - 1 : 0];
  if (t < 0 || t >= VOCAB) {
    if (threadIdx.x == 0) atomicCAS(S.err, 0, ERR_TOKEN);
    t = 0;
  }
  return t;
}

// xf = rmsnorm(src) * (1 + w) over HID (golden/model.py:63-75,
// hls/src/norm.hpp:13-20), src = h or, for the first phase of a step, the
// dequantised embedding row (golden/model.py:246, hls/src/gemv.hpp:76-84).
__device__ void prologue_norm(XEnc& e, float* red, const StateW& S, const float* w,
                              const int8_t* emb_q, const float* emb_s, bool embed) {
  float ss = 0.0f;
  if (embed) {
    const int tok = step_token(S);
    const float sc = emb_s[tok];
    const int8_t* row = emb_q + (size_t)tok * HID;
    for (int i = threadIdx.x; i < HID; i += blockDim.x) {
      const float v = __fmul_rn((float)row[i], sc);
      e.xf[i] = v;
      if (blockIdx.x == 0) S.h[i] = v;   // residual stream starts at the embedding
      ss = fmaf(v, v, ss);
    }
  } else {
    for (int i = threadIdx.x; i < HID; i += blockDim.x) {
      const float v = S.h[i];
      e.xf[i] = v;
      ss = fmaf(v, v, ss);
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)HID), EPS)));
  for (int i = threadIdx.x; i < HID; i += blockDim.x)
    e.xf[i] = __fmul_rn(__fmul_rn(e.xf[i], inv), __fadd_rn(1.0f, w[i]));
  __syncthreads();
}

// xf = gated RMSNorm of the delta-rule output: per head o*rsqrt(mean(o^2)+eps)
// * w * silu(z)  -- gain w, not 1+w (golden/model.py:183-189, hls/src/norm.hpp:25-33).
__device__ void prologue_gnorm(XEnc& e, float* red, const StateW& S, const float* w) {
  __shared__ float inv_h[LH];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int h = wid; h < LH; h += nw) {
    float ss = 0.0f;
    for (int i = lane; i < LV; i += 32) {
      const float v = S.o[h * LV + i];
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0)
      inv_h[h] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)LV), EPS)));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < VDIM; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(S.o[i], inv_h[i / LV]), w[i % LV]);
    e.xf[i] = __fmul_rn(v, silu_f(S.z[i]));
  }
  __syncthreads();
  (void)red;
}

// xf = attention output * sigmoid(gate) (golden/model.py:229); the gate is the
// second half of each head's q_proj block (golden/model.py:201-203).
__device__ void prologue_attn_gate(XEnc& e, const StateW& S) {
  for (int i = threadIdx.x; i < NH * HD; i += blockDim.x) {
    const int h = i / HD, d = i % HD;
    e.xf[i] = __fmul_rn(S.attn_o[i], sigmoid_f(S.qg[h * 2 * HD + HD + d]));
  }
  __syncthreads();
}

__device__ void prologue_copy(XEnc& e, const float* src, int K) {
  for (int i = threadIdx.x; i < K; i += blockDim.x) e.xf[i] = src[i];
  __syncthreads();
}

// ---------------------------------------------------------------- GEMV phases

// Rows of one phase: `nseg` int8 segments handled in units of R rows.
struct Seg {
  const int8_t* q; const float* s; int rows; float* y;
};

// Generic int8 phase body: global warp gw processes units gw, gw+nwarps, ...
template <int R>
__device__ void run_segments(const XEnc& e, const Seg* segs, int nseg, int K) {
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int total = 0;
  for (int s = 0; s < nseg; ++s) total += segs[s].rows / R;
  for (int u = gw; u < total; u += nwarps) {
    int s = 0, uu = u;
    while (uu >= segs[s].rows / R) { uu -= segs[s].rows / R; ++s; }
    const int r0 = uu * R;
    const int8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = segs[s].q + (size_t)(r0 + r) * K;
    int acc[R][3];
    warp_rows_dot<R>(rows, e, K, acc);
    if (lane < R) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r == lane) { a0 = acc[r][0]; a1 = acc[r][1]; a2 = acc[r][2]; }
      segs[s].y[r0 + lane] = finish_row(a0, a1, a2, e.ndig, e.scale, segs[s].s[r0 + lane]);
    }
  }
}

// linear-attention layer input projections: qkv, z (int8) and b, a (fp32).
__global__ void __launch_bounds__(256) k_dn_in(LayerW L, StateW S, const int8_t* emb_q,
                                               const float* emb_s, int embed) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_norm(enc, red, S, L.in_norm, emb_q, emb_s, embed != 0);
  encode_x(enc, HID, S.dyn->act_int8 != 0, red);
  // the fp32 rows (in_proj_b, in_proj_a) go to the first warps of the grid
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int j = gw; j < 2 * LH; j += nwarps) {
    const float* row = (j < LH) ? (L.b_w + (size_t)j * HID) : (L.a_w + (size_t)(j - LH) * HID);
    const float v = warp_row_dot_f32(row, enc, HID);
    if ((threadIdx.x & 31) == 0) S.ab[j] = v;
  }
  Seg segs[2] = {{L.qkv_q, L.qkv_s, CONVD, S.qkv}, {L.z_q, L.z_s, VDIM, S.z}};
  run_segments<2>(enc, segs, 2, HID);
}

// full-attention layer input projections q | k | v.
__global__ void __launch_bounds__(256) k_att_in(LayerW L, StateW S, const int8_t* emb_q,
                                                const float* emb_s, int embed) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_norm(enc, red, S, L.in_norm, emb_q, emb_s, embed != 0);
  encode_x(enc, HID, S.dyn->act_int8 != 0, red);
  Seg segs[3] = {{L.q_q, L.q_s, QPROJ, S.qg},
                 {L.k_q, L.k_s, KVPROJ, S.kvn},
                 {L.v_q, L.v_s, KVPROJ, S.kvn + KVPROJ}};
  run_segments<2>(enc, segs, 3, HID);
}

// Row-parallel projection back to the hidden size with the residual add fused
// into the epilogue: h[o] = h[o] + y[o] (golden/model.py:259,263).
template <int R>
__device__ void run_residual(const XEnc& e, const int8_t* q, const float* s, int K, float* h) {
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int u = gw; u < HID / R; u += nwarps) {
    const int r0 = u * R;
    const int8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = q + (size_t)(r0 + r) * K;
    int acc[R][3];
    warp_rows_dot<R>(rows, e, K, acc);
    if (lane < R) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r == lane) { a0 = acc[r][0]; a1 = acc[r][1]; a2 = acc[r][2]; }
      const float y = finish_row(a0, a1, a2, e.ndig, e.scale, s[r0 + lane]);
      h[r0 + lane] = __fadd_rn(h[r0 + lane], y);
    }
  }
}

__global__ void __launch_bounds__(256) k_dn_out(LayerW L, StateW S) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_gnorm(enc, red, S, L.gnorm_w);
  encode_x(enc, VDIM, S.dyn->act_int8 != 0, red);
  run_residual<1>(enc, L.out_q, L.out_s, VDIM, S.h);
}

__global__ void __launch_bounds__(256) k_att_out(LayerW L, StateW S) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_attn_gate(enc, S);
  encode_x(enc, NH * HD, S.dyn->act_int8 != 0, red);
  run_residual<1>(enc, L.o_q, L.o_s, NH * HD, S.h);
}

// SwiGLU front: gate row j and up row j in one warp, act[j] = silu(g) * u
// (golden/model.py:233-237, hls/src/mlp.hpp:11-19).
__global__ void __launch_bounds__(256) k_gate_up(LayerW L, StateW S) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_norm(enc, red, S, L.post_norm, nullptr, nullptr, false);
  encode_x(enc, HID, S.dyn->act_int8 != 0, red);
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int j = gw; j < FFN; j += nwarps) {
    const int8_t* rows[2] = {L.gate_q + (size_t)j * HID, L.up_q + (size_t)j * HID};
    int acc[2][3];
    warp_rows_dot<2>(rows, enc, HID, acc);
    if (lane == 0) {
      const float g = finish_row(acc[0][0], acc[0][1], acc[0][2], enc.ndig, enc.scale, L.gate_s[j]);
      const float u = finish_row(acc[1][0], acc[1][1], acc[1][2], enc.ndig, enc.scale, L.up_s[j]);
      S.act[j] = __fmul_rn(silu_f(g), u);
    }
  }
}

__global__ void __launch_bounds__(256) k_down(LayerW L, StateW S) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  prologue_copy(enc, S.act, FFN);
  encode_x(enc, FFN, S.dyn->act_int8 != 0, red);
  run_residual<1>(enc, L.down_q, L.down_s, FFN, S.h);
}

// ---------------------------------------------------------------- DeltaNet

// Gated delta rule on columns v0..v0+15 of one head's state Sh[128][128]
// (256 threads: thread -> 8 rows of k, one column):
//   S *= exp(g); kv = k^T S; d = (v - kv) * beta; S += k (x) d; o = q^T S
// with o read from the UPDATED state (golden/model.py:174-178,
// hls/src/deltanet.hpp:58-115).  qs/ks/vs are smem (q pre-scaled).
__device__ void delta_slice(float* Sh, const float* qs, const float* ks, const float* vs,
                            float g, float beta, int v0, float* out, float (*part)[DSLICE + 1]) {
  const int t = threadIdx.x;
  const int vi = t & 15, kg = t >> 4;
  const float gexp = expf(g);
  float sv[8];
  float pkv = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int k = kg * 8 + kk;
    sv[kk] = __fmul_rn(Sh[(size_t)k * LV + v0 + vi], gexp);   // decay
    pkv = fmaf(sv[kk], ks[k], pkv);
  }
  part[kg][vi] = pkv;
  __syncthreads();
  float kvv = 0.0f;
#pragma unroll
  for (int gi = 0; gi < 16; ++gi) kvv += part[gi][vi];
  const float delta = __fmul_rn(__fsub_rn(vs[vi], kvv), beta);
  __syncthreads();
  float po = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int k = kg * 8 + kk;
    const float s2 = __fadd_rn(sv[kk], __fmul_rn(ks[k], delta));   // rank-1 write
    Sh[(size_t)k * LV + v0 + vi] = s2;
    po = fmaf(s2, qs[k], po);                                      // read with the new S
  }
  part[kg][vi] = po;
  __syncthreads();
  if (t < DSLICE) {
    float o = 0.0f;
#pragma unroll
    for (int gi = 0; gi < 16; ++gi) o += part[gi][t];
    out[t] = o;
  }
}

// One (head, value-slice) per CTA (256 threads) on caller buffers: the
// standalone delta_rule_layer operator (inputs already conv'd and normalised).
__global__ void __launch_bounds__(256) k_delta_core(const float* q, const float* k,
                                                    const float* v, const float* g,
                                                    const float* beta, float* S, float* out) {
  const int h = blockIdx.x / NDSLICE, j = blockIdx.x % NDSLICE;
  __shared__ float qs[LK], ks[LK], vs[DSLICE];
  __shared__ float part[16][DSLICE + 1];
  const int t = threadIdx.x;
  if (t < LK) qs[t] = q[h * LK + t];
  else ks[t - LK] = k[h * LK + t - LK];
  if (t < DSLICE) vs[t] = v[h * LV + j * DSLICE + t];
  __syncthreads();
  delta_slice(S + (size_t)h * LK * LV, qs, ks, vs, g[h], beta[h], j * DSLICE,
              out + h * LV + j * DSLICE, part);
}

cudaError_t enqueue_delta_rule(const float* q, const float* k, const float* v, const float* g,
                               const float* beta, float* S, float* out, cudaStream_t st) {
  k_delta_core<<<LH * NDSLICE, 256, 0, st>>>(q, k, v, g, beta, S, out);
  return cudaGetLastError();
}

// One (head, value-slice) of the gated delta rule per CTA (256 threads):
// causal conv + SiLU of this head's q/k channels and of the slice's v channels,
// gates, l2norm, then the state update of the slice's 16 columns of S[h].
// golden/model.py:149-178; hls/src/conv1d.hpp:17-38, deltanet.hpp:58-115,164-169.
__global__ void __launch_bounds__(256) k_delta(LayerW L, StateW S) {
  const int h = blockIdx.x / NDSLICE, j = blockIdx.x % NDSLICE;
  const int t = threadIdx.x;
  const int lin = L.lin_idx;
  const int base = S.dyn->conv_base;
  float* cs = S.conv + (size_t)lin * CONVD * CONVK;
  __shared__ float qs[LK], ks[LK], vs[DSLICE];
  __shared__ float part[16][DSLICE + 1];
  __shared__ float wsum[8];
  __shared__ float gate_g, gate_beta;

  auto conv_ch = [&](int ch, bool owner) -> float {
    const float* w = L.conv_w + (size_t)ch * CONVK;
    float* st = cs + (size_t)ch * CONVK;
    const float s1 = st[(base + 1) & 3], s2 = st[(base + 2) & 3], s3 = st[(base + 3) & 3];
    const float nv = S.qkv[ch];
    float acc = __fmul_rn(s1, w[0]);
    acc = __fadd_rn(acc, __fmul_rn(s2, w[1]));
    acc = __fadd_rn(acc, __fmul_rn(s3, w[2]));
    acc = __fadd_rn(acc, __fmul_rn(nv, w[3]));
    if (owner) st[base & 3] = nv;     // the dead oldest column becomes the newest
    return silu_f(acc);
  };
  // q channels (threads 0..127), k channels (128..255); v slice by threads 0..15
  float x;
  if (t < LK) x = conv_ch(h * LK + t, j == 0);
  else x = conv_ch(KDIM + h * LK + (t - LK), j == 0);
  if (t < DSLICE) vs[t] = conv_ch(2 * KDIM + h * LV + j * DSLICE + t, true);
  if (t == 0) {
    const float b = S.ab[h], a = S.ab[LH + h];
    gate_beta = sigmoid_f(b);
    gate_g = __fmul_rn(-expf(L.A_log[h]), softplus_f(__fadd_rn(a, L.dt_bias[h])));
  }
  // l2norm over each 128-vector (warps 0-3: q, warps 4-7: k)
  float ss = warp_sum(x * x);
  if ((t & 31) == 0) wsum[t >> 5] = ss;
  __syncthreads();
  {
    const int g0 = (t < LK) ? 0 : 4;
    const float tot = ((wsum[g0] + wsum[g0 + 1]) + wsum[g0 + 2]) + wsum[g0 + 3];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(tot, EPS)));
    if (t < LK) qs[t] = __fmul_rn(__fmul_rn(x, inv), 0.08838834764831845f);  // * K^-0.5
    else ks[t - LK] = __fmul_rn(x, inv);
  }
  __syncthreads();
  float* Sh = S.rec + ((size_t)lin * LH + h) * LK * LV;
  delta_slice(Sh, qs, ks, vs, gate_g, gate_beta, j * DSLICE, S.o + h * LV + j * DSLICE, part);
}

// ---------------------------------------------------------------- attention

__device__ __forceinline__ void att_layout(int Tn, int& nch, int& cl) {
  nch = (Tn + ATT_MINLEN - 1) / ATT_MINLEN;
  nch = nch < 1 ? 1 : (nch > ATT_MAXCH ? ATT_MAXCH : nch);
  cl = (Tn + nch - 1) / nch;
}

// QK rmsnorm (1+w) then partial RoPE of one 256-vector held by one warp as
// elements lane + 32*j (golden/model.py:205-214, hls/src/rope.hpp:17-41).
__device__ __forceinline__ void warp_norm_rope(const float* src, const float* w, const float* cs,
                                               float* dst) {
  const int lane = threadIdx.x & 31;
  float v[8];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) { v[j] = src[lane + 32 * j]; ss = fmaf(v[j], v[j], ss); }
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), EPS)));
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], inv), __fadd_rn(1.0f, w[lane + 32 * j]));
  // dims 0..31 pair with 32..63: cos/sin of both halves are equal (emb = [f, f])
  const float c = cs[lane], s = cs[32 + lane];
  const float a = v[0], b = v[1];
  v[0] = __fadd_rn(__fmul_rn(a, c), __fmul_rn(-b, s));
  v[1] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
#pragma unroll
  for (int j = 0; j < 8; ++j) dst[lane + 32 * j] = v[j];
}

// Split-KV GQA decode: CTA = (kv head g, chunk c).  Each CTA re-derives the 4
// query heads of group g and the new K/V, appends them to the cache (chunk 0
// only), runs a stable softmax over its chunk, and the last CTA of the group
// merges the chunk partials (max, sum, o).  Scale 256^-0.5, sigmoid gate later.
// golden/model.py:194-228, hls/src/attention.hpp:25-95.
__global__ void __launch_bounds__(256) k_attn(LayerW L, StateW S) {
  const int g = blockIdx.x % NKV, c = blockIdx.x / NKV;
  const int T = S.dyn->T, pos = S.dyn->pos;
  const int Tn = T + 1;
  int nch, cl;
  att_layout(Tn, nch, cl);
  if (c >= nch) return;
  if (T >= S.max_ctx || cl > ATT_MAXLEN || pos >= S.max_rope) {
    if (threadIdx.x == 0) atomicCAS(S.err, 0, ERR_CTX);
    return;
  }
  const int t0 = c * cl, t1 = min(Tn, t0 + cl), n = t1 - t0;
  const int fi = L.full_idx;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __shared__ __align__(16) float qn[4][HD];
  __shared__ __align__(16) float kn[HD], vn[HD];
  __shared__ float sc[4][ATT_MAXLEN];
  __shared__ float mh[4], lh[4];
  __shared__ int last;
  const float* rope = S.rope + (size_t)pos * ROT;
  if (wid < 4) warp_norm_rope(S.qg + (size_t)(4 * g + wid) * 2 * HD, L.qn_w, rope, qn[wid]);
  else if (wid == 4) warp_norm_rope(S.kvn + g * HD, L.kn_w, rope, kn);
  else if (wid == 5) {
    for (int d = lane; d < HD; d += 32) vn[d] = S.kvn[KVPROJ + g * HD + d];
  }
  __syncthreads();
  float* kc = S.kcache + (size_t)fi * S.max_ctx * KVPROJ;
  float* vc = S.vcache + (size_t)fi * S.max_ctx * KVPROJ;
  if (c == 0) {   // roped K and raw V of this token into slot T (golden/model.py:216-217)
    kc[(size_t)T * KVPROJ + g * HD + threadIdx.x] = kn[threadIdx.x];
    vc[(size_t)T * KVPROJ + g * HD + threadIdx.x] = vn[threadIdx.x];
  }
  // scores: one warp per position, lane holds dims 4*lane..+3 and 128+4*lane..+3
  for (int i = wid; i < n; i += 8) {
    const int tt = t0 + i;
    float4 k0, k1;
    if (tt < T) {
      const float* kp = kc + (size_t)tt * KVPROJ + g * HD;
      k0 = *reinterpret_cast<const float4*>(kp + 4 * lane);
      k1 = *reinterpret_cast<const float4*>(kp + 128 + 4 * lane);
    } else {
      k0 = *reinterpret_cast<const float4*>(&kn[4 * lane]);
      k1 = *reinterpret_cast<const float4*>(&kn[128 + 4 * lane]);
    }
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) {
      const float4 q0 = *reinterpret_cast<const float4*>(&qn[hq][4 * lane]);
      const float4 q1 = *reinterpret_cast<const float4*>(&qn[hq][128 + 4 * lane]);
      float d = q0.x * k0.x + q0.y * k0.y + q0.z * k0.z + q0.w * k0.w;
      d += q1.x * k1.x + q1.y * k1.y + q1.z * k1.z + q1.w * k1.w;
      d = warp_sum(d);
      if (lane == 0) sc[hq][i] = d * 0.0625f;   // 256^-0.5, exact
    }
  }
  __syncthreads();
  if (wid < 4) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[wid][i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      const float p = expf(sc[wid][i] - m);
      sc[wid][i] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) { mh[wid] = m; lh[wid] = l; }
  }
  __syncthreads();
  // o[hq][d] = sum_t p[hq][t] * V[t][d], thread d
  const int d = threadIdx.x;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < n; ++i) {
    const int tt = t0 + i;
    const float v = (tt < T) ? vc[(size_t)tt * KVPROJ + g * HD + d] : vn[d];
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) o[hq] = fmaf(sc[hq][i], v, o[hq]);
  }
  float* part = S.att_part + ((size_t)(g * ATT_MAXCH + c) * 4) * (2 + HD);
#pragma unroll
  for (int hq = 0; hq < 4; ++hq) {
    part[hq * (2 + HD) + 2 + d] = o[hq];
    if (d == 0) { part[hq * (2 + HD)] = mh[hq]; part[hq * (2 + HD) + 1] = lh[hq]; }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&S.att_cnt[g], 1) == nch - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge the chunk partials of the 4 heads of group g
  for (int hq = 0; hq < 4; ++hq) {
    const float* pb = S.att_part + ((size_t)(g * ATT_MAXCH) * 4 + hq) * (2 + HD);
    const size_t stride = 4 * (2 + HD);
    float M = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, __ldcg(pb + cc * stride));
    float Lsum = 0.0f, O = 0.0f;
    for (int cc = 0; cc < nch; ++cc) {
      const float f = expf(__ldcg(pb + cc * stride) - M);
      Lsum = fmaf(__ldcg(pb + cc * stride + 1), f, Lsum);
      O = fmaf(__ldcg(pb + cc * stride + 2 + d), f, O);
    }
    S.attn_o[(4 * g + hq) * HD + d] = __fdiv_rn(O, Lsum);
  }
  if (threadIdx.x == 0) S.att_cnt[g] = 0;
}

// ---------------------------------------------------------------- head

// Tied int8 head over the final-normed hidden state (golden/model.py:266-267),
// always fp32 activations (the golden applies no _qa here), fused with a
// block argmax; logits are written when the step asks for them.
__global__ void __launch_bounds__(256) k_head(ModelW* M, StateW S) {
  __shared__ __align__(16) XEnc enc;
  __shared__ float red[32];
  __shared__ unsigned long long wbest[8];
  prologue_norm(enc, red, S, M->final_norm, nullptr, nullptr, false);
  encode_x(enc, HID, false, red);
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const bool want = S.dyn->want_logits != 0;
  const int8_t* E = M->emb_q;
  const float* Es = M->emb_s;
  constexpr int R = 4;
  unsigned long long best = 0ull;
  for (int u = gw; u < VOCAB / R; u += nwarps) {
    const int r0 = u * R;
    const int8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = E + (size_t)(r0 + r) * HID;
    int acc[R][3];
    warp_rows_dot<R>(rows, enc, HID, acc);
    if (lane < R) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r == lane) { a0 = acc[r][0]; a1 = acc[r][1]; a2 = acc[r][2]; }
      const float y = finish_row(a0, a1, a2, 3, enc.scale, Es[r0 + lane]);
      if (want) S.logits[r0 + lane] = y;
      best = umax64(best, am_pack(y, r0 + lane));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) wbest[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = umax64(b, wbest[w]);
    S.am_part[blockIdx.x] = b;
  }
}

// Reduce the head's block maxima, record the step's argmax, advance the state.
__global__ void k_finish(StateW S, int nparts) {
  __shared__ unsigned long long wb[32];
  unsigned long long b = 0ull;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) b = umax64(b, S.am_part[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) b = umax64(b, wb[w]);
    b = umax64(b, wb[0]);
    const int step = S.io[0];
    if (step < S.max_steps) S.ids[step] = am_index(b);
    else atomicCAS(S.err, 0, ERR_CTX);
    S.io[0] = step + 1;
    S.dyn->pos += 1;
    S.dyn->T += 1;
    S.dyn->conv_base += 1;
  }
}

// ---------------------------------------------------------------- launch

// Enqueue one decode step on `st` (graph-capturable: every per-step value is
// read from device memory).
cudaError_t enqueue_step(const ModelW& Mh, ModelW* Md, const StateW& S, int sm_count,
                         cudaStream_t st) {
  const int in_grid = 2 * sm_count;
  const int out_grid = HID / 8;          // one row per warp, 8 warps per CTA
  for (int li = 0; li < NLAYER; ++li) {
    const LayerW& L = Mh.L[li];
    const int embed = (li == 0);
    if (L.linear) {
      k_dn_in<<<in_grid, 256, 0, st>>>(L, S, Mh.emb_q, Mh.emb_s, embed);
      k_delta<<<LH * NDSLICE, 256, 0, st>>>(L, S);
      k_dn_out<<<out_grid, 256, 0, st>>>(L, S);
    } else {
      k_att_in<<<in_grid, 256, 0, st>>>(L, S, Mh.emb_q, Mh.emb_s, embed);
      k_attn<<<NKV * ATT_MAXCH, 256, 0, st>>>(L, S);
      k_att_out<<<out_grid, 256, 0, st>>>(L, S);
    }
    k_gate_up<<<in_grid, 256, 0, st>>>(L, S);
    k_down<<<out_grid, 256, 0, st>>>(L, S);
  }
  const int head_grid = 4 * sm_count;
  k_head<<<head_grid, 256, 0, st>>>(Md, S);
  k_finish<<<1, 1024, 0, st>>>(S, head_grid);
  return cudaGetLastError();
}

int head_grid_size(int sm_count) { return 4 * sm_count; }

}  // namespace qb
