// Host-side interface of the persistent weight-streaming decode kernel (persist.cu).
#pragma once
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "common.cuh"

namespace qb {

// One weight chunk of a CTA's schedule: nrows rows (or (gate, up) row pairs)
// of segment `seg` of phase `phase`, starting at row0.  A tensor-core chunk
// (seg has CHUNK_MMA set) is one K-slab of a tile instead: row0 = tile index
// within the phase, nrows = slab index.
struct Chunk {
  unsigned short phase;
  unsigned char seg;
  unsigned char nrows;
  unsigned row0;
};
static_assert(sizeof(Chunk) == 8, "Chunk layout");
constexpr unsigned char CHUNK_MMA = 0x80;

// Phases of one decode step: 5 per layer (IN, MIX, OUT, GATEUP, DOWN) + the head.
constexpr int PERSIST_NPHASE = NLAYER * 5 + 1;

// Trace record layout: per CTA and phase, %globaltimer stamps at phase entry,
// inputs arrived (the input wait done), outputs written (a GEMV phase: its
// last panel's; the head: its first slab landed), phase exit; then, for the
// first GEMV CTA (the one after the DeltaNet heads' CTAs) only, per phase and
// warp, clock64 stamps of a GEMV phase: 0 entry, 1 inputs in, 2 digit image
// encoded, 3 first task's chunk landed, 4 own tasks done, 5 a task's MMA done,
// 6 a panel's outputs written by this warp, and inside the W8A8 encoder of a
// normed input 8 norm statistics, 9 their barrier passed, 10 digits written
// (0 = not reached).
constexpr int TRACE_STAMPS = 4;
constexpr int TRACE_WARP_STAMPS = 16;

// Head tiles: embed_tokens.weight [VOCAB, HID] int8 as HEAD_TILES tiles of
// HEAD_TM rows, each cut into HEAD_NSLAB K-slabs of HEAD_KS bytes.  Slab
// (t, j) is one contiguous 16 KB block at (t * HEAD_NSLAB + j) * 16384 in the
// tcgen05 canonical K-major no-swizzle layout: element (m, k) of the slab at
// ((m / 8) * (HEAD_KS / 16) + k / 16) * 128 + (m % 8) * 16 + k % 16.
constexpr int HEAD_TM = 128;
constexpr int HEAD_KS = 128;
constexpr int HEAD_NSLAB = HID / HEAD_KS;
constexpr int HEAD_TILES = VOCAB / HEAD_TM;
static_assert(VOCAB % HEAD_TM == 0 && HID % HEAD_KS == 0, "head tiling");
constexpr size_t HEAD_TILE_BYTES = (size_t)VOCAB * HID;
cudaError_t repack_head_tiles(const int8_t* emb_q, int8_t* tiles, cudaStream_t st);

// Tensor parallelism over tp_world GPUs of one node, one process (and one
// context) per GPU.  Every rank keeps the full weights and the global index
// space of every activation; its schedule covers only its shard:
//   DeltaNet heads [dn_h0, dn_h1) (in_proj_qkv / z / a / b rows, conv, state,
//     gated norm: column-parallel, no exchange inside the mixer);
//   attention KV groups [kv_g0, kv_g1) with all four query heads of each; for
//     tp_world 4 and 8 the ns = tp_world / NKV ranks sharing a group split its
//     cached positions instead: slice j = tp_rank % ns is [j Tn / ns,
//     (j + 1) Tn / ns) of the Tn = T + 1 positions, and the slices' (m, l, o)
//     are exchanged and merged in slice order (flash-decoding combine,
//     golden/model.py:219-229), so the KV bytes each rank reads shrink with
//     the world (every rank of the group still writes slot T of its copy);
//   OUT (out_proj / o_proj) row-parallel over input columns [ok0, ok1) (the
//     rank's heads), DOWN row-parallel over FFN columns [dk0, dk1) (128-column
//     blocks), gate/up column-parallel over the same FFN rows;
//   head tiles [t0, t1) (vocab slice).
// An OUT or DOWN phase adds its partial rows across ranks (P2P stores into
// every rank's exchange buffer, then a fixed-order sum: bit-identical on all
// ranks); the head exchanges each rank's (max, index); under W8A8 the OUT and
// DOWN inputs' maxima are exchanged before they are quantised; an attention
// MIX of a split group exchanges the slices' (m, l, o).
constexpr int TP_MAX = 8;
struct TpPlan {
  int rank = 0, world = 1;
  int dn_h0 = 0, dn_h1 = LH;
  int kv_g0 = 0, kv_g1 = NKV;
  int ok0 = 0, ok1 = VDIM;
  int dk0 = 0, dk1 = FFN;
  int t0 = 0, t1 = HEAD_TILES;
};
// The shard of `rank` among `world` (1, 2, 4 or 8); false (with err) otherwise.
bool tp_plan(int rank, int world, TpPlan& out, std::string& err);
// Exchange buffer of one rank (tagged words): [2 (OUT, DOWN)][TP_MAX source
// ranks][HID] partial rows, then [TP_MAX source ranks][2] head (max, index)
// words, then [2 (OUT, DOWN)][TP_MAX source ranks] input maxima (W8A8: the
// golden quantiser's max over the whole input vector), then the attention
// sequence split: [ATT_SPLIT_MAX position slices][4 heads][2 + HD] (m, l, o)
// of the ranks that share this rank's KV group.
constexpr int ATT_SPLIT_MAX = TP_MAX / NKV;   // ranks per KV group at the largest world
constexpr size_t XB_PART = 0;
constexpr size_t XB_HEAD = 2 * (size_t)TP_MAX * HID;
constexpr size_t XB_AMAX = XB_HEAD + 2 * TP_MAX;
constexpr size_t XB_ATT = XB_AMAX + 2 * TP_MAX;
constexpr size_t XB_WORDS = XB_ATT + (size_t)ATT_SPLIT_MAX * 4 * (2 + HD);

// Everything the persistent kernel reads; tv_* are tagged {value, tag} words.
struct PersistArgs {
  const LayerW* layers;        // [NLAYER] (device copy of ModelW::L)
  const int8_t* emb_q; const float* emb_s; const float* final_norm;
  const int8_t* head_tiles;    // embed_tokens.weight re-tiled for the tensor cores (repack_head_tiles)
  const Chunk* chunks;         // [G][MAXCH]
  const unsigned short* phase_first;  // [G][PERSIST_NPHASE + 1]: a phase's chunks are
                                      // [first[p], first[p + 1]) of the CTA's list
  unsigned long long *tv_h, *tv_qkv, *tv_z, *tv_o, *tv_qg, *tv_kvn, *tv_attn, *tv_act;
  float* conv; float* rec; float* kcache; float* vcache;
  unsigned long long* att_tv;      // [NKV][ATT_MAXCH][4][2 + HD] tagged split-KV partials (m, l, o)
  int* head_cnt;
  unsigned long long* am_part;     // [G]
  const float* rope;
  float* logits;
  int* io; int* ids; int* err; int* abort_flag;
  StepDyn* dyn;
  unsigned long long* trace;       // nullable: the trace record (layout above persist_trace_words)
  // W8A8 capture (qwen_capture_phase): phase dbg_phase (-1: off) of the next
  // step writes its input, int8 image, s_x and int32 accumulators to dbg
  // (layout DBG_*); single-GPU ACT_INT8 instance only.
  int dbg_phase;
  float* dbg;
  int max_ctx, max_rope, max_steps;
  // tensor parallelism (tp_world = 1: none; see TpPlan)
  int tp_rank, tp_world;
  int dn_h0, dn_h1, kv_g0, kv_g1, ok0, ok1, dk0, dk1;
  unsigned long long* xbuf[TP_MAX];   // every rank's exchange buffer, mapped here (rank order)
};

// Layer GEMVs on the warp-level tensor-core MMA (mma.sync m16n8k32 s8): every
// projection is re-laid at load time as panels of 16 rows; inside a panel,
// element (m, k) sits at ((k / 16) * 16 + m) * 16 + k % 16, so one K = 32 step
// of all 16 rows is 512 contiguous bytes (one ldmatrix.x4 = the MMA's A
// fragment).  A chunk is one K-slice of a panel: 16 rows x 1024 bytes of K
// (16 KB; the last slice of a K = 3584 panel is 512 bytes, 8 KB); a task is
// 512 bytes of K of a chunk (8 KB of weights, 16 MMA K-steps).  GATEUP uses
// pair panels: rows 0-7 are gate rows 8q .. 8q+7, rows 8-15 the same up rows,
// so a gate row and its up row finish in neighbouring lanes.
constexpr int PANEL = 16;
constexpr int PANEL_KB = 1024;                  // K bytes per chunk
constexpr int TASK_KB = 512;                    // K bytes per task
constexpr int PAIR_ROWS = 8;                    // gate (and up) rows per pair panel
constexpr unsigned char CHUNK_PANEL = 0x40;     // Chunk.seg flag: row0 = panel, nrows = K-slice
static_assert(CONVD % PANEL == 0 && VDIM % PANEL == 0 && QPROJ % PANEL == 0 &&
              KVPROJ % PANEL == 0 && HID % PANEL == 0 && FFN % PAIR_ROWS == 0, "panels");
static_assert(HID % TASK_KB == 0 && VDIM % TASK_KB == 0 && FFN % TASK_KB == 0, "tasks");
static_assert(VDIM == NH * HD && FFN % 128 == 0 && VDIM % (TP_MAX * 128) == 0, "TP column windows");
static_assert(KDIM == VDIM && LK == LV && LH % TP_MAX == 0 && NH % TP_MAX == 0, "TP head blocks");
// Re-lay nrows rows (row r read from rowptr[r], K bytes each) as 16-row panels
// (for GATEUP the caller orders the rows 8 gate, 8 up per panel).
cudaError_t repack_panels(const int8_t* const* rowptr, int8_t* out, int nrows, int K, cudaStream_t st);

// Capture buffer layout (floats): the phase's fp32 input as the kernel
// quantises it (a normed input: the residual h before the norm) at DBG_X, the
// int8 image (as floats, natural order) at DBG_XQ, s_x at DBG_SX, K at DBG_K,
// a claim word at DBG_FLAG, and the int32 accumulators (bit patterns) of the
// phase's rows at DBG_ACC: IN rows in panel order ([qkv | z] or [q | k | v]),
// GATEUP gate rows then up rows, OUT / DOWN the 1024 hidden rows.
constexpr int DBG_X = 0, DBG_XQ = 4096, DBG_SX = 8192, DBG_K = 8193, DBG_FLAG = 8194, DBG_ACC = 8200;
constexpr int DBG_FLOATS = DBG_ACC + 8192;

int persist_smem_bytes();
int persist_num_phases();
int persist_max_chunks();
size_t persist_trace_words(int G);   // words of the trace record for G CTAs
int persist_max_blocks_per_sm();
bool build_schedule(const ModelW& M, int G, const TpPlan& tp, std::vector<Chunk>& chunks,
                    std::vector<unsigned short>& phase_first, std::string& err);
// i8: the ACT_INT8 instance (must match the step's StepDyn::act_int8).
cudaError_t launch_persistent(const PersistArgs& args, int G, cudaStream_t st, bool i8);

}  // namespace qb
