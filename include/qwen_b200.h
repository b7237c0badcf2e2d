/* qwen_b200.h -- C ABI of libqwenb200.so, the B200 (sm_100a) int8 decode
 * step of the Qwen3.5-0.8B hybrid text decoder, at batch 1 and batched over up
 * to 64 independent sequences.
 *
 * Every entry point returns an int status (0 = QWEN_OK); a context keeps the
 * message of its last failure (qwen_last_error).  Plain pointers and sizes
 * only.  A context is thread-compatible: use one context per host thread, or
 * lock around it.
 *
 * The reference interfaces each call replaces are cited as file:line inside
 * allthingssecurity/qwen_fpga.
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QWEN_OK 0
#define QWEN_ERR_ARG 1       /* bad argument (null, size, alignment, range) */
#define QWEN_ERR_IO 2        /* blob / index file unreadable or inconsistent */
#define QWEN_ERR_CUDA 3      /* a CUDA runtime call failed */
#define QWEN_ERR_DEVICE 4    /* a kernel reported a bounded wait that ran out */
#define QWEN_ERR_STATE 5     /* context too long, or call out of order */

typedef struct qwen_ctx qwen_ctx;
typedef struct CUstream_st* qwen_stream_t; /* same handle as cudaStream_t */

/* Load a packed int8 blob (scripts/pack_weights.py:28-101 layout) and its
 * index (either the flat weights.idx of scripts/emit_weight_index.py:1-22 or
 * the *.manifest.json of pack_weights.py:93-101) onto the GPU and create
 * max_batch decode states (golden/model.py:86-107 DecodeState, one per
 * sequence) with room for max_ctx cached positions per attention layer each.
 * Replaces the blob mmap + DecodeState set-up of hls/tb/run_hls.cpp:27-52 and
 * golden/model.py:97-107.  n_gpus must be 1; device_ids may be NULL (device
 * 0).  max_batch in [1, 64]: 1 = the batch-1 persistent decode kernel; > 1 =
 * the batched engine (sequences 0 .. max_batch-1, each with its own DeltaNet
 * state, conv history and KV cache; projections as tcgen05 int8 GEMMs over
 * the batch's tokens). */
int qwen_create(const char* blob_path, const char* index_path, int n_gpus,
                const int* device_ids, int max_ctx, int max_batch, qwen_ctx** out);

/* Tensor parallelism over tp_world (1, 2, 4 or 8) GPUs of one node, one
 * process and one context per GPU: the weight sharding of a multi-device
 * decode step (the reference runs one device; the split follows the
 * weights' natural shards).  Rank tp_rank of the job keeps the full weights on device
 * device_id and computes its shard: DeltaNet heads, attention KV groups (all
 * four query heads of each), gate/up rows and down columns in 128-column
 * blocks, out/o columns by head, and a vocab slice of the head.  Row-parallel
 * projections add their partial rows across ranks inside the decode kernel
 * (stores into every rank's exchange buffer over NVLink, then a sum in rank
 * order, so every rank holds the same residual stream bit for bit); the head
 * exchanges (max, index) pairs.
 *
 * Set-up: qwen_create_tp on every rank; qwen_tp_export writes this rank's
 * exchange-buffer handle (QWEN_TP_HANDLE_BYTES bytes, a CUDA IPC handle);
 * the caller gathers every rank's handle in rank order (any host transport)
 * and passes the array to qwen_tp_connect.  Every rank then makes the same
 * decode calls in the same order (like collectives); a rank that stops makes
 * the others' next step fail after the 2 s device wait bound with
 * QWEN_ERR_DEVICE.  Under ACT_INT8 the ranks also exchange the maxima of the
 * row-parallel inputs, so each is quantised with the max over the whole
 * vector as on one GPU.
 * Logits: each rank fills only its vocab slice [lo, hi) of logits_out
 * (qwen_tp_vocab_range).  State import/export move the full arrays; a rank
 * uses and updates only its heads' parts.
 *
 * qwen_tp_plan writes the shard of (tp_rank, tp_world) without a context:
 * QWEN_TP_PLAN_INTS ints = DeltaNet heads [h0, h1), KV groups [g0, g1), OUT
 * input columns [o0, o1), FFN columns [f0, f1), vocab rows [v0, v1). */
#define QWEN_TP_HANDLE_BYTES 64
#define QWEN_TP_PLAN_INTS 10
int qwen_create_tp(const char* blob_path, const char* index_path, int device_id, int tp_rank,
                   int tp_world, int max_ctx, int max_batch, qwen_ctx** out);
int qwen_tp_export(qwen_ctx* ctx, void* handle_out);
int qwen_tp_connect(qwen_ctx* ctx, const void* handles);
int qwen_tp_vocab_range(qwen_ctx* ctx, int* lo, int* hi);
int qwen_tp_plan(int tp_rank, int tp_world, int* out);

/* Pack a Hugging Face safetensors snapshot of the Qwen3.5 text decoder into
 * the blob qwen_create loads (replaces scripts/pack_weights.py:50-101 with its
 * loader golden/loader.py:36-78 and quantiser golden/quant.py:43-49).  Reads
 * snapshot_dir/config.json (text_config) and every *.safetensors file in
 * snapshot_dir (BF16, F16, F32, I32 or I64; "model.language_model." prefixes
 * dropped, vision and MTP tensors skipped); writes out_blob (tensors in
 * decode read order, 4 KiB aligned, int8 rows + fp32 row scales for the GEMV
 * weights, fp32 otherwise) and, beside it, <stem>.manifest.json and
 * <stem>.idx.  Host only, no GPU.  QWEN_ERR_IO (message in
 * qwen_last_error(NULL)) when a tensor is missing or extra for the config's
 * layer_types, or a file cannot be read or written. */
int qwen_pack_blob(const char* snapshot_dir, const char* out_blob);

/* Free every device and host resource of the context. */
int qwen_destroy(qwen_ctx* ctx);

/* Zero the recurrent state, empty the KV cache, pos = 0
 * (hls/src/state.hpp:24-34, golden/model.py:97-107) of sequence seq: 0 on a
 * batch-1 context; 0 .. max_batch-1, or -1 for every sequence, on a batched
 * context. */
int qwen_reset(qwen_ctx* ctx, int seq);

/* Load / read back the decode state of sequence seq (golden/model.py:86-95
 * DecodeState; seq as for qwen_reset, -1 excluded):
 *   conv [18][6144][4]   rec [18][16][128][128]
 *   kc, vc [6][T][2][256] (K after QK-norm and RoPE, V raw)   pos
 * Host pointers.  Import requires T <= max_ctx - 1.  Export writes T and pos
 * through the int pointers; kc/vc may be NULL to skip the cache (a call with
 * both NULL reads T), and when given must each hold 6 * T * 512 floats for the
 * current T. */
int qwen_state_import(qwen_ctx* ctx, int seq, const float* conv, const float* rec,
                      const float* kc, const float* vc, int T, int pos);
int qwen_state_export(qwen_ctx* ctx, int seq, float* conv, float* rec, float* kc,
                      float* vc, int* T, int* pos);

/* ACT_INT8 switch of golden/model.py:34-45: on = every projection input is
 * quantised per vector to int8 (int8 x int8 -> int32 GEMVs); off = fp32
 * activations (W8A32).  The tied head always takes fp32 activations. */
int qwen_set_act_int8(qwen_ctx* ctx, int on);

/* Per-phase tracing of the decode kernel (no counterpart in the reference,
 * which times steps with perf_counter at run_prompt.py:80-98): when on, every
 * step records, per CTA and per phase, %globaltimer stamps [entry, inputs
 * arrived, outputs written, exit] (ns; 0 where a phase has no such point),
 * n_ctas * n_phases * 4 words;
 * then, for the first CTA that runs GEMV panels, per phase and per warp (16),
 * 16 SM-clock stamps of a GEMV phase [entry, inputs in, input encoded, first
 * chunk landed, own tasks done, a task's MMA done, a panel's outputs written,
 * unused, W8A8 encoder: statistics, their barrier, digits written, 5 unused]
 * (0 = not reached), n_phases * 16 * 16 words; this second part is filled
 * only by a library built with QB_WARP_TRACE defined (its stamps cost
 * instructions on the hot path).
 * qwen_trace_read copies the last step's record to host memory; max_words
 * must cover both parts. */
int qwen_trace_enable(qwen_ctx* ctx, int on);
int qwen_trace_read(qwen_ctx* ctx, unsigned long long* out, int max_words, int* n_ctas,
                    int* n_phases);

/* W8A8 arithmetic capture, a test hook (no counterpart in the reference):
 * qwen_capture_phase arms GEMV phase `phase` (5 l + 0 IN, + 2 OUT, + 3 GATEUP,
 * + 4 DOWN of layer l; -1 disarms) of every following ACT_INT8 step on the
 * decode kernel of a single-GPU context.  The step then records, into
 * QWEN_CAPTURE_FLOATS floats that qwen_capture_read copies out: [0, 4096) the
 * phase's fp32 input as the kernel quantises it (IN / GATEUP: the residual
 * stream h before the RMSNorm), [4096, 8192) its int8 activations (golden
 * _qa, golden/model.py:37-45), [8192] s_x, [8193] K, [8194] 1 when captured,
 * and from [8200] the int32 accumulators of the phase's rows as bit patterns
 * (IN: [qkv | z] or [q | k | v] rows; GATEUP: 3584 gate rows then 3584 up
 * rows; OUT / DOWN: 1024 rows) -- the exact integer products of
 * scripts/export_gemv_tv.py:49 that a test recomputes. */
#define QWEN_CAPTURE_FLOATS 16392
int qwen_capture_phase(qwen_ctx* ctx, int phase);
int qwen_capture_read(qwen_ctx* ctx, float* out, int max_floats);

/* One decode step for each of `batch` tokens: embed, 24 layers, final norm,
 * tied head, argmax (first index on ties).  Mirrors golden/model.py:243-267
 * decode_step and hls/src/qwen_synth.hpp:39-92 qwen_top.  A max_batch 1
 * context takes batch 1; a batched context steps sequences 0 .. batch-1
 * (batch <= max_batch) together, tok[b] feeding sequence b.  tok and
 * argmax_out (batch ints) are host pointers; logits_out (nullable) may be a
 * host or device pointer of batch x vocab (248320) floats, sequence-major.
 * On a batched context tok may be NULL: every sequence then takes its own
 * previous argmax (greedy continuation).  On a single-GPU batch-1 context,
 * page-locked host logits (cudaMallocHost, a pinned torch tensor) are written
 * by the decode kernel itself while the head runs; any other pointer gets a
 * copy after the kernel.  The values are the same either way. */
int qwen_decode_step(qwen_ctx* ctx, const int* tok, int batch, float* logits_out,
                     int* argmax_out);

/* Prefill (batch-1 single-GPU context): the n prompt tokens run through every
 * layer at once instead of n decode steps -- the projections as tensor-core
 * GEMMs over the tokens, the DeltaNet layers by the chunked delta rule
 * (the recurrence of golden/model.py:168-178 unrolled over a chunk of up to
 * 32 tokens: one triangular solve and dense products, the state read and
 * written once per chunk), attention causal over the cache and the prompt.
 * The decode state afterwards is that of n qwen_decode_step calls (fp32
 * reassociation aside); logits_out (nullable, host or device, vocab floats)
 * and argmax_out (nullable) get the last token's.  The reference only loops
 * the decode step (golden/model.py:1-7, run_prompt.py:82-83). */
int qwen_prefill(qwen_ctx* ctx, const int* tok, int n, float* logits_out, int* argmax_out);

/* Batched context only: `steps` greedy steps of sequences 0 .. batch-1 (each
 * fed its previous argmax), timed on the device (decode steps only, as
 * run_prompt.py:80-98 times them); seconds receives the device time. */
int qwen_decode_timed(qwen_ctx* ctx, int batch, int steps, double* seconds);

/* Prefill n_prompt tokens one at a time, then n_new greedy steps; out_ids gets
 * the n_new generated ids (golden/model.py:270-280, run_prompt.py:80-98).
 * decode_seconds (nullable) receives the device time of the n_new decode
 * steps only, as run_prompt.py times them. */
int qwen_generate(qwen_ctx* ctx, const int* prompt, int n_prompt, int n_new, int* out_ids,
                  double* decode_seconds);

/* Standalone int8-weight GEMV on device pointers, y[N] = s[o] * W[o,:] . x
 * with fp32 x -- the operator of hls/src/gemv.hpp:28-42 (gemv_i8).  K must be
 * a multiple of 32 in [32, 3584]; w 32-byte aligned.  x is mapped to a
 * 23-bit signed fixed-point image (step 2^-22 of its largest power-of-two
 * bound), split into three int8 digits, and each digit is dotted with the row
 * exactly in int32; the digits are recombined exactly in int64 and scaled once
 * in fp64, so the only error is x's fixed-point rounding (about fp32 round-off
 * of the largest |x|). */
int qwen_gemv_i8_f32(float* y, const int8_t* w, const float* s, const float* x, int N,
                     int K, qwen_stream_t stream);

/* Standalone int8 x int8 GEMV on device pointers: acc[o] = sum_i w[o,i]*xq[i]
 * exactly in int32 (rtl/gemv_i8.sv:13-76, scripts/export_gemv_tv.py:49) and
 * y[o] = acc[o] * sx * sw[o] in fp32, left to right (rtl/dequant.sv:12-29,
 * export_gemv_tv.py:50).  acc and y are each nullable (not both).  Same K /
 * alignment rules as above. */
int qwen_gemv_i8_i8(int32_t* acc, float* y, const int8_t* w, const float* sw,
                    const int8_t* xq, float sx, int N, int K, qwen_stream_t stream);

/* The same operator over a batch of B activation vectors (the projection
 * datapath of a batched context), on device pointers: acc[b*N + o] =
 * sum_i w[o,i]*xq[b*K + i] exactly in int32 on the tensor cores
 * (tcgen05.mma kind::i8, 128 weight rows x B tokens per tile) and
 * y[b*N + o] = acc * (sx[b] * sw[o]) in fp32.  acc and y are each nullable
 * (not both).  N a multiple of 128, K of 128 in [128, 4096], B in [1, 64];
 * w and xq 16-byte aligned.  Allocates its scratch (the weights re-laid as
 * tiles) on the stream and returns after the stream has drained. */
int qwen_gemm_i8_i8(int32_t* acc, float* y, const int8_t* w, const float* sw,
                    const int8_t* xq, const float* sx, int N, int K, int B, qwen_stream_t stream);

/* Allocation-free GEMV + argmax on device pointers (no counterpart in the
 * reference): y = s .* (W x) exactly as qwen_gemv_i8_f32 computes it, and
 * *argmax = the first index of the largest y (the tied-head argmax of
 * golden/model.py:266-267).  For callers that may not allocate device memory
 * while they run, such as a serving loop that has fixed its memory after
 * warm-up or a caller with no qwen_ctx: the call uses no cudaMalloc and no
 * library allocator.  Its per-block maxima and an arrival counter sit in a
 * fixed 8 KiB static device array.
 *   - N must be in [1, 1048576] (the array holds 1024 blocks of 1024 rows);
 *     larger N is rejected with QWEN_ERR_ARG.  K, w alignment as for
 *     qwen_gemv_i8_f32.  y may be NULL; argmax (one int) may not.
 *   - The first call on each device resolves the array's address
 *     (cudaGetSymbolAddress) and keeps it for the life of the process; make
 *     that first call before any stream capture.  Resetting the device
 *     (cudaDeviceReset) after that first call is not supported: the kept
 *     address would be stale.
 *   - Each call clears the array's arrival counter on its stream (an 8-byte
 *     memset) before its kernel starts, so a call whose launch failed
 *     part-way does not disturb the next one.  The per-block maxima need no
 *     clearing: every block writes its slot before it arrives.
 *   - Calls on the same device share the array: two calls whose kernels run at
 *     the same time (different streams, overlapping launches) race and return
 *     wrong argmax values.  Order them (one stream, or events). */
int qwen_gemv_i8_f32_argmax_noalloc(float* y, int* argmax, const int8_t* w, const float* s,
                                    const float* x, int N, int K, qwen_stream_t stream);

/* One gated delta-rule step of a 16-head DeltaNet layer on device pointers,
 * S [16][128][128] updated in place, out [16][128]:
 *   S *= exp(g); kv = k^T S; d = (v - kv) * beta; S += k (x) d; out = q^T S
 * hls/src/deltanet.hpp:118-127 delta_rule_layer, golden/model.py:174-178. */
int qwen_delta_rule_layer(const float* q, const float* k, const float* v, const float* g,
                          const float* beta, float* S, float* out, qwen_stream_t stream);

/* Message of the context's last failure ("" when none).  ctx may be NULL for
 * the last failure of a call that had no context. */
const char* qwen_last_error(qwen_ctx* ctx);

/* Library version string. */
const char* qwen_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_H */
