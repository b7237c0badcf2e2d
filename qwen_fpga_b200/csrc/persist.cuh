// Host-side interface of the persistent weight-streaming decode kernel (persist.cu).
#pragma once
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "common.cuh"

namespace qb {

// One weight chunk of a CTA's schedule: nrows rows (or (gate, up) row pairs)
// of segment `seg` of phase `phase`, starting at row0.
struct Chunk {
  unsigned short phase;
  unsigned char seg;
  unsigned char nrows;
  unsigned row0;
};
static_assert(sizeof(Chunk) == 8, "Chunk layout");

// Everything the persistent kernel reads; tv_* are tagged {value, tag} words.
struct PersistArgs {
  const LayerW* layers;        // [NLAYER] (device copy of ModelW::L)
  const int8_t* emb_q; const float* emb_s; const float* final_norm;
  const Chunk* chunks;         // [G][MAXCH]
  const int* nchunks;          // [G]
  unsigned long long *tv_h, *tv_qkv, *tv_z, *tv_ab, *tv_o, *tv_qg, *tv_kvn, *tv_attn, *tv_act;
  float* conv; float* rec; float* kcache; float* vcache;
  float* att_part; int* att_cnt;   // att_cnt: [NFULL][NKV]
  int* head_cnt;
  unsigned long long* am_part;     // [G]
  const float* rope;
  float* logits;
  int* io; int* ids; int* err; int* abort_flag;
  StepDyn* dyn;
  unsigned long long* trace;       // nullable: [G][NPHASE][4] %globaltimer stamps
  int max_ctx, max_rope, max_steps;
};

// Trace record layout: per CTA and phase, stamps at phase entry, inputs ready
// (prologue done), first weight chunk landed, phase exit.
constexpr int TRACE_STAMPS = 4;

int persist_smem_bytes();
int persist_num_phases();
int persist_max_chunks();
int persist_max_blocks_per_sm();
bool build_schedule(const ModelW& M, int G, std::vector<Chunk>& chunks, std::vector<int>& counts,
                    std::string& err);
cudaError_t launch_persistent(const PersistArgs& args, int G, cudaStream_t st);

}  // namespace qb
