// Host-side interface of the batched decode engine (batch.cu): up to
// BATCH_MAX independent sequences per step, each with its own DeltaNet state
// and KV cache (golden/model.py:86-107 DecodeState, one per sequence), stepped
// together by golden/model.py:243-267 decode_step.  The projections run as
// tcgen05 int8 GEMMs (M = 128 weight rows per tile, N = the batch's tokens,
// times three digit planes under W8A32), the mixers as per-sequence kernels,
// the tied head as a persistent tcgen05 kernel with a per-sequence argmax.
#pragma once
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "common.cuh"

namespace qb {

constexpr int BATCH_MAX = 64;      // tokens per step (N of the GEMMs, per digit plane)
constexpr int GT_M = 128;          // weight rows per tile
constexpr int GT_KS = 128;         // K bytes per slab
constexpr int GT_SLAB = GT_M * GT_KS;   // 16 KB of weights

// Weight tiles of one projection: tile t (rows 128 t ..), slab j (K 128 j ..)
// is one 16 KB block at (t * K / 128 + j) * 16384 in the canonical K-major
// no-swizzle layout of tcgen05: element (m, k) of a slab at
// ((m / 8) * 8 + k / 16) * 128 + (m % 8) * 16 + k % 16 (the head tiles of
// repack_head_tiles have the same layout).  Row r comes from rowptr[r]
// (device array of K-byte rows); nrows a multiple of 128, K of 128.
cudaError_t repack_tiles(const int8_t* const* rowptr, int8_t* out, int nrows, int K, cudaStream_t st);

// Activation image: the B operand of the GEMMs.  nr rows (digit plane p of
// token b is row 64 p + b), K bytes each, as K / 128 slabs of nr x 128 bytes
// in the same canonical layout.  Byte offset of row r, position k:
__host__ __device__ __forceinline__ size_t img_off(int r, int k, int nr) {
  return (size_t)(k >> 7) * nr * 128 + (size_t)((((r >> 3) << 3) + ((k & 127) >> 4)) << 7) + ((r & 7) << 4) +
         (k & 15);
}

// The operator behind qwen_gemm_i8_i8: acc[b][o] = sum_k w[o][k] xq[b][k]
// (exact int32, tcgen05 kind::i8), y[b][o] = acc * (sx[b] * sw[o]).
// w row-major [N][K], xq row-major [B][K]; scratch is allocated on the stream.
cudaError_t gemm_i8_i8_batched(int32_t* acc, float* y, const int8_t* w, const float* sw, const int8_t* xq,
                               const float* sx, int N, int K, int B, cudaStream_t st);

// ---- the engine
struct BatchEngine;
// Build the engine's weight tiles and per-sequence state for max_batch
// sequences of max_ctx cached positions (rope: the context's RoPE table of
// max_rope rows; head_tiles: the tied head in tile layout).  nullptr + err on
// failure.
BatchEngine* batch_create(const ModelW& M, const int8_t* head_tiles, const float* rope, int max_rope, int max_batch,
                          int max_ctx, int sm_count, cudaStream_t st, std::string& err);
void batch_destroy(BatchEngine* e);
// Return codes below are the library's QWEN_* codes.
int batch_reset(BatchEngine* e, int seq, std::string& err);   // seq -1: every sequence
// Host arrays in the golden layout (conv [18][6144][4], rec [18][16][128][128],
// kc / vc [6][T][2][256]).
int batch_import(BatchEngine* e, int seq, const float* conv, const float* rec, const float* kc, const float* vc, int T,
                 int pos, std::string& err);
int batch_export(BatchEngine* e, int seq, float* conv, float* rec, float* kc, float* vc, int* T, int* pos,
                 std::string& err);
// One step of sequences 0 .. nb-1.  tok: host array of nb ids, or null to
// feed each sequence its previous argmax.  logits_out (nullable): host or
// device, nb x VOCAB floats.  argmax_out (nullable): host, nb ints.
int batch_step(BatchEngine* e, const int* tok, int nb, bool act_int8, float* logits_out, int* argmax_out,
               std::string& err);
// Device time of the last batch_timed_steps call.
int batch_timed_steps(BatchEngine* e, int nb, bool act_int8, int steps, double* seconds, std::string& err);
int batch_max(const BatchEngine* e);
// Prefill: n prompt tokens of ONE sequence through every layer at once (in
// chunks of 32), on that sequence's arrays in the batch-1 layouts (conv ring
// with origin conv_base, rec, kc / vc [6][max_ctx][512] with T0 cached
// positions, first RoPE position pos0): the state afterwards is that of n
// decode steps (the DeltaNet layers by the chunked delta rule).  The last
// token's logits (nullable, host or device) and argmax are returned.  Uses
// the engine's kernels and work buffers (an engine created with max_batch 1
// serves a batch-1 context).
int batch_prefill(BatchEngine* e, float* conv, float* rec, float* kc, float* vc, int max_ctx, int conv_base, int T0,
                  int pos0, const int* tok, int n, bool act_int8, float* logits_out, int* argmax_out,
                  std::string& err);

}  // namespace qb
