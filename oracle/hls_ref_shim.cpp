// C-ABI shim over the reference's HLS C++ decoder, compiled in place from the
// reference checkout (qwen_fpga hls/src/*.hpp) into oracle/_ref/.
//
// TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline / reference arm load the resulting library as a checker or as
// the timed reference CPU implementation.  The product never links it.
//
// What it wraps (all reference code, unmodified, included by path):
//   qwen_top         hls/src/qwen_synth.hpp:39-92   one token from the packed blob
//   DecodeState      hls/src/state.hpp:18-35        conv / rec / KV / pos
//   delta_rule_layer hls/src/deltanet.hpp:118-127   16-head delta rule
//   gemv_i8          hls/src/gemv.hpp:28-42         int8 x fp32 GEMV
// The HLS attention keeps a static 8192-entry score buffer
// (hls/src/attention.hpp:66), so this oracle only accepts contexts <= 8192.
#include <cstdint>
#include <cstring>

#include "qwen_synth.hpp"

using namespace qwen;

extern "C" {

void* hls_ref_new() {
  DecodeState* st = new DecodeState();
  st->reset();
  return st;
}

void hls_ref_free(void* st) { delete static_cast<DecodeState*>(st); }

void hls_ref_reset(void* st) { static_cast<DecodeState*>(st)->reset(); }

int hls_ref_max_ctx() { return 8192; }

// conv [18][6144][4], rec [18][16][128][128], kc/vc [6][T][2][256] (may be null when T == 0)
int hls_ref_set_state(void* vst, const float* conv, const float* rec, const float* kc,
                      const float* vc, int T, int pos) {
  DecodeState* st = static_cast<DecodeState*>(vst);
  if (T < 0 || T + 1 > hls_ref_max_ctx() || pos < 0) return -1;
  std::memcpy(st->conv, conv, sizeof(st->conv));
  std::memcpy(st->rec, rec, sizeof(st->rec));
  const long per = (long)T * KV_PROJ;
  for (int f = 0; f < N_FULL; ++f) {
    st->kc[f].assign(kc + f * per, kc + (f + 1) * per);
    st->vc[f].assign(vc + f * per, vc + (f + 1) * per);
  }
  st->pos = pos;
  return 0;
}

int hls_ref_pos(void* st) { return static_cast<DecodeState*>(st)->pos; }

// qwen_top writes slot `pos` of the KV cache, so the cache length must equal pos.
int hls_ref_step(const uint8_t* blob, void* vst, int tok, float* logits) {
  DecodeState* st = static_cast<DecodeState*>(vst);
  if (st->pos + 1 > hls_ref_max_ctx()) return -1;
  return qwen_top(blob, *st, tok, logits);
}

void hls_ref_delta_rule_layer(const float* q, const float* k, const float* v, const float* g,
                              const float* beta, float* S, float* out) {
  delta_rule_layer(reinterpret_cast<const float(*)[K]>(q), reinterpret_cast<const float(*)[K]>(k),
                   reinterpret_cast<const float(*)[V]>(v), g, beta,
                   reinterpret_cast<float(*)[K][V]>(S), reinterpret_cast<float(*)[V]>(out));
}

void hls_ref_gemv_i8(float* y, const int8_t* w, const float* s, const float* x, int n, int k) {
  gemv_i8(y, w, s, x, n, k);
}

}  // extern "C"
