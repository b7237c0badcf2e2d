// The standalone gated delta-rule operator of libqwenb200
// (qwen_delta_rule_layer): one step of a 16-head DeltaNet layer on caller
// buffers, the operator of hls/src/deltanet.hpp:118-127 (delta_rule_layer)
// and golden/model.py:174-178.  (Inside the decode step the persistent
// kernel runs the delta rule per head on its own CTAs.)
#include "common.cuh"
#include "delta.cuh"

namespace qb {

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

}  // namespace qb
