// Host runtime and C ABI of libqwenb200 (declared in include/qwen_b200.h).
//
// A context owns one GPU's copy of the packed weight blob (plus the panel and
// head-tile copies the persistent kernel streams), one batch-1 decode state,
// and the kernel's per-CTA schedule.  Per call the host only writes a small
// control block (position, token source) and launches the persistent kernel
// once per step.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/qwen_b200.h"
#include "batch.cuh"
#include "common.cuh"
#include "delta.cuh"
#include "gemv.cuh"
#include "noalloc.cuh"
#include "persist.cuh"

using namespace qb;

static_assert(DBG_FLOATS == QWEN_CAPTURE_FLOATS, "capture layout");

namespace {

thread_local std::string g_last_error;

}  // namespace

namespace qb {
// For the library's host-only entry points in other files (pack.cpp).
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace qb

namespace {

struct TensorEnt {
  uint64_t off = 0, nbytes = 0, soff = 0, snbytes = 0;
  int dtype = 0;  // 1 int8, 0 fp32
  std::vector<long> shape;
};

// ------------------------------------------------------------------ index files

// Flat index, one line per tensor: name off nbytes dtype scale_off scale_nbytes out in
// (scripts/emit_weight_index.py:1-22).
bool parse_idx(const std::string& path, std::map<std::string, TensorEnt>& out, std::string& err) {
  std::ifstream f(path);
  if (!f) { err = "cannot open index " + path; return false; }
  std::string name;
  unsigned long long off, nb, so, sn;
  int dt;
  long o, i;
  while (f >> name >> off >> nb >> dt >> so >> sn >> o >> i) {
    TensorEnt e;
    e.off = off; e.nbytes = nb; e.dtype = dt; e.soff = so; e.snbytes = sn;
    if (o) e.shape.push_back(o);
    if (i) e.shape.push_back(i);
    out[name] = e;
  }
  if (out.empty()) { err = "index " + path + " has no entries"; return false; }
  return true;
}

// Minimal JSON reader for the blob manifest (scripts/pack_weights.py:93-101).
struct JVal {
  enum K { NUL, NUM, STR, ARR, OBJ, BOOL } k = NUL;
  double num = 0;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* key) const {
    for (auto& kv : obj) if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  bool ok = true;
  void ws() { while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(end - p) >= n && strncmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  std::string string() {
    std::string s;
    if (p >= end || *p != '"') { ok = false; return s; }
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) { ++p; s.push_back(*p == 'n' ? '\n' : *p); }
      else s.push_back(*p);
      ++p;
    }
    if (p < end) ++p; else ok = false;
    return s;
  }
  JVal value() {
    JVal v;
    ws();
    if (p >= end) { ok = false; return v; }
    if (*p == '{') {
      v.k = JVal::OBJ; ++p; ws();
      if (p < end && *p == '}') { ++p; return v; }
      while (ok) {
        ws();
        std::string key = string();
        ws();
        if (p >= end || *p != ':') { ok = false; break; }
        ++p;
        v.obj.emplace_back(key, value());
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; break; }
        ok = false;
      }
    } else if (*p == '[') {
      v.k = JVal::ARR; ++p; ws();
      if (p < end && *p == ']') { ++p; return v; }
      while (ok) {
        v.arr.push_back(value());
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; break; }
        ok = false;
      }
    } else if (*p == '"') {
      v.k = JVal::STR; v.str = string();
    } else if (lit("true")) { v.k = JVal::BOOL; v.num = 1; }
    else if (lit("false")) { v.k = JVal::BOOL; v.num = 0; }
    else if (lit("null")) { v.k = JVal::NUL; }
    else {
      char* q = nullptr;
      v.k = JVal::NUM;
      v.num = strtod(p, &q);
      if (q == p) ok = false;
      p = q;
    }
    return v;
  }
};

bool parse_manifest(const std::string& path, std::map<std::string, TensorEnt>& out,
                    std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) { err = "cannot open manifest " + path; return false; }
  std::stringstream ss;
  ss << f.rdbuf();
  const std::string txt = ss.str();
  JParser P{txt.data(), txt.data() + txt.size()};
  JVal root = P.value();
  const JVal* ts = root.get("tensors");
  if (!P.ok || !ts || ts->k != JVal::ARR) { err = "manifest " + path + " unreadable"; return false; }
  for (const JVal& t : ts->arr) {
    const JVal* name = t.get("name");
    const JVal* off = t.get("offset");
    const JVal* nb = t.get("nbytes");
    const JVal* dt = t.get("dtype");
    const JVal* sh = t.get("shape");
    if (!name || !off || !nb || !dt || !sh) { err = "manifest entry incomplete"; return false; }
    TensorEnt e;
    e.off = (uint64_t)off->num;
    e.nbytes = (uint64_t)nb->num;
    e.dtype = dt->str == "int8" ? 1 : 0;
    if (const JVal* so = t.get("scale_offset")) e.soff = (uint64_t)so->num;
    if (const JVal* sn = t.get("scale_nbytes")) e.snbytes = (uint64_t)sn->num;
    for (const JVal& d : sh->arr) e.shape.push_back((long)d.num);
    out[name->str] = e;
  }
  return true;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace

// ------------------------------------------------------------------ context

struct qwen_ctx {
  int dev = 0;
  int sm_count = 148;
  cudaStream_t st = nullptr;
  std::string err;
  uint8_t* d_blob = nullptr;
  size_t blob_bytes = 0;
  ModelW Mh{};
  ModelW* Md = nullptr;
  StateW S{};
  std::vector<void*> allocs;
  int max_ctx = 0, max_rope = 0, max_steps = 0;
  // control block: StepDyn followed by io = [step, n_prompt, tokens...]
  void* d_ctl = nullptr;
  void* h_ctl = nullptr;      // pinned mirror
  int* h_ids = nullptr;       // pinned
  int* h_err = nullptr;       // pinned
  int pos = 0, T = 0, conv_base = 0;
  unsigned seq = 1;           // launch sequence number (tag base of the persistent kernel)
  int act_int8 = 0;
  PersistArgs P{};
  TpPlan tp{};                // tensor-parallel shard of this context (world 1: everything)
  unsigned long long* xbuf = nullptr;   // this rank's exchange buffer (IPC-exported)
  std::vector<void*> ipc_open;          // peers' exchange buffers mapped into this process
  bool tp_ready = true;                 // world 1, or qwen_tp_connect done
  unsigned long long* tv_base = nullptr;
  size_t tv_words = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int max_batch = 1;
  BatchEngine* be = nullptr;            // max_batch > 1: the batched engine owns the sequences
  BatchEngine* pf = nullptr;            // batch 1: kernels and buffers of qwen_prefill (made on first use)
};

namespace {

int fail(qwen_ctx* c, int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  g_last_error = buf;
  return code;
}

#define QCUDA(c, call)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail((c), QWEN_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));   \
  } while (0)

template <class T>
int dalloc(qwen_ctx* c, T** p, size_t bytes) {
  void* q = nullptr;
  QCUDA(c, cudaMalloc(&q, bytes));
  QCUDA(c, cudaMemset(q, 0, bytes));
  c->allocs.push_back(q);
  *p = reinterpret_cast<T*>(q);
  return QWEN_OK;
}

StepDyn* ctl_dyn(qwen_ctx* c) { return reinterpret_cast<StepDyn*>(c->h_ctl); }
int* ctl_io(qwen_ctx* c) { return reinterpret_cast<int*>(reinterpret_cast<char*>(c->h_ctl) + sizeof(StepDyn)); }
size_t ctl_bytes(int max_steps) { return sizeof(StepDyn) + sizeof(int) * (2 + (size_t)max_steps); }

// Expected tensors and their byte sizes (golden/model.py shapes, types.hpp).
int bind_weights(qwen_ctx* c, const std::map<std::string, TensorEnt>& idx) {
  auto i8 = [&](const std::string& n, long out, long in, const int8_t** q, const float** s) -> int {
    auto it = idx.find(n);
    if (it == idx.end()) return fail(c, QWEN_ERR_IO, "tensor %s missing from index", n.c_str());
    const TensorEnt& e = it->second;
    if (e.dtype != 1 || e.nbytes != (uint64_t)out * in || e.snbytes != (uint64_t)out * 4)
      return fail(c, QWEN_ERR_IO, "tensor %s: expected int8 [%ld,%ld]", n.c_str(), out, in);
    if (e.off % 32 || e.soff % 4 || e.off + e.nbytes > c->blob_bytes || e.soff + e.snbytes > c->blob_bytes)
      return fail(c, QWEN_ERR_IO, "tensor %s: offset out of range or misaligned", n.c_str());
    *q = reinterpret_cast<const int8_t*>(c->d_blob + e.off);
    *s = reinterpret_cast<const float*>(c->d_blob + e.soff);
    return QWEN_OK;
  };
  auto f32 = [&](const std::string& n, long count, const float** p) -> int {
    auto it = idx.find(n);
    if (it == idx.end()) return fail(c, QWEN_ERR_IO, "tensor %s missing from index", n.c_str());
    const TensorEnt& e = it->second;
    if (e.dtype != 0 || e.nbytes != (uint64_t)count * 4)
      return fail(c, QWEN_ERR_IO, "tensor %s: expected %ld fp32 values", n.c_str(), count);
    if (e.off % 16 || e.off + e.nbytes > c->blob_bytes)
      return fail(c, QWEN_ERR_IO, "tensor %s: offset out of range or misaligned", n.c_str());
    *p = reinterpret_cast<const float*>(c->d_blob + e.off);
    return QWEN_OK;
  };
  int rc;
  ModelW& M = c->Mh;
  if ((rc = i8("embed_tokens.weight", VOCAB, HID, &M.emb_q, &M.emb_s))) return rc;
  if ((rc = f32("norm.weight", HID, &M.final_norm))) return rc;
  int li = 0, fi = 0;
  for (int l = 0; l < NLAYER; ++l) {
    LayerW& L = M.L[l];
    const std::string p = "layers." + std::to_string(l) + ".";
    L.linear = (l % 4) != 3;   // [linear x3, full] x6 (hls/src/types.hpp:47)
    if ((rc = f32(p + "input_layernorm.weight", HID, &L.in_norm))) return rc;
    if ((rc = f32(p + "post_attention_layernorm.weight", HID, &L.post_norm))) return rc;
    if (L.linear) {
      const std::string a = p + "linear_attn.";
      L.lin_idx = li++;
      L.full_idx = -1;
      if ((rc = i8(a + "in_proj_qkv.weight", CONVD, HID, &L.qkv_q, &L.qkv_s))) return rc;
      if ((rc = i8(a + "in_proj_z.weight", VDIM, HID, &L.z_q, &L.z_s))) return rc;
      if ((rc = f32(a + "in_proj_b.weight", LH * HID, &L.b_w))) return rc;
      if ((rc = f32(a + "in_proj_a.weight", LH * HID, &L.a_w))) return rc;
      if ((rc = f32(a + "conv1d.weight", CONVD * CONVK, &L.conv_w))) return rc;
      if ((rc = f32(a + "A_log", LH, &L.A_log))) return rc;
      if ((rc = f32(a + "dt_bias", LH, &L.dt_bias))) return rc;
      if ((rc = f32(a + "norm.weight", LV, &L.gnorm_w))) return rc;
      if ((rc = i8(a + "out_proj.weight", HID, VDIM, &L.out_q, &L.out_s))) return rc;
    } else {
      const std::string a = p + "self_attn.";
      L.full_idx = fi++;
      L.lin_idx = -1;
      if ((rc = i8(a + "q_proj.weight", QPROJ, HID, &L.q_q, &L.q_s))) return rc;
      if ((rc = i8(a + "k_proj.weight", KVPROJ, HID, &L.k_q, &L.k_s))) return rc;
      if ((rc = i8(a + "v_proj.weight", KVPROJ, HID, &L.v_q, &L.v_s))) return rc;
      if ((rc = f32(a + "q_norm.weight", HD, &L.qn_w))) return rc;
      if ((rc = f32(a + "k_norm.weight", HD, &L.kn_w))) return rc;
      if ((rc = i8(a + "o_proj.weight", HID, NH * HD, &L.o_q, &L.o_s))) return rc;
    }
    if ((rc = i8(p + "mlp.gate_proj.weight", FFN, HID, &L.gate_q, &L.gate_s))) return rc;
    if ((rc = i8(p + "mlp.up_proj.weight", FFN, HID, &L.up_q, &L.up_s))) return rc;
    if ((rc = i8(p + "mlp.down_proj.weight", HID, FFN, &L.down_q, &L.down_s))) return rc;
  }
  return QWEN_OK;
}

// cos/sin of every position for the rotated slice (golden/model.py:113-120):
// inv_i = 1 / 1e7^(2i/64) in float32, angle = float(pos) * inv_i in float32.
void rope_table(std::vector<float>& t, int rows) {
  t.assign((size_t)rows * ROT, 0.0f);
  float inv[ROT / 2];
  for (int i = 0; i < ROT / 2; ++i) inv[i] = 1.0f / powf(10000000.0f, (float)(2 * i) / (float)ROT);
  for (int p = 0; p < rows; ++p)
    for (int i = 0; i < ROT / 2; ++i) {
      const float a = (float)p * inv[i];
      t[(size_t)p * ROT + i] = (float)cos((double)a);
      t[(size_t)p * ROT + ROT / 2 + i] = (float)sin((double)a);
    }
}

int upload_blob(qwen_ctx* c, const char* path) {
  FILE* f = fopen(path, "rb");
  if (!f) return fail(c, QWEN_ERR_IO, "cannot open blob %s", path);
  fseek(f, 0, SEEK_END);
  const long len = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (len <= 0) { fclose(f); return fail(c, QWEN_ERR_IO, "blob %s is empty", path); }
  c->blob_bytes = (size_t)len;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, c->blob_bytes);
  if (e != cudaSuccess) { fclose(f); return fail(c, QWEN_ERR_CUDA, "cudaMalloc blob: %s", cudaGetErrorString(e)); }
  c->allocs.push_back(d);
  c->d_blob = reinterpret_cast<uint8_t*>(d);
  const size_t chunk = 64u << 20;
  void* hb = nullptr;
  e = cudaMallocHost(&hb, chunk);
  if (e != cudaSuccess) { fclose(f); return fail(c, QWEN_ERR_CUDA, "cudaMallocHost: %s", cudaGetErrorString(e)); }
  int rc = QWEN_OK;
  for (size_t off = 0; off < c->blob_bytes; off += chunk) {
    const size_t n = std::min(chunk, c->blob_bytes - off);
    if (fread(hb, 1, n, f) != n) { rc = fail(c, QWEN_ERR_IO, "short read of %s", path); break; }
    e = cudaMemcpy(c->d_blob + off, hb, n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { rc = fail(c, QWEN_ERR_CUDA, "upload: %s", cudaGetErrorString(e)); break; }
  }
  cudaFreeHost(hb);
  fclose(f);
  return rc;
}

// Write the host control block to the device (async on the context stream).
int push_ctl(qwen_ctx* c, int n_io_tokens) {
  QCUDA(c, cudaMemcpyAsync(c->d_ctl, c->h_ctl, sizeof(StepDyn) + sizeof(int) * (2 + n_io_tokens),
                           cudaMemcpyHostToDevice, c->st));
  return QWEN_OK;
}

void fill_dyn(qwen_ctx* c, int want_logits) {
  StepDyn* d = ctl_dyn(c);
  memset(d, 0, sizeof(StepDyn));
  d->pos = c->pos;
  d->T = c->T;
  d->conv_base = c->conv_base;
  d->act_int8 = c->act_int8;
  d->want_logits = want_logits;
  d->seq = (int)c->seq;
}

// Keep launch tags unique: before the sequence number would wrap, clear the
// tagged activation words and restart it.
int ensure_seq_room(qwen_ctx* c, int launches) {
  if (c->seq + (unsigned)launches < (1u << 24)) return QWEN_OK;
  QCUDA(c, cudaMemsetAsync(c->tv_base, 0, c->tv_words * 8, c->st));
  c->seq = 1;
  return QWEN_OK;
}

// One decode step on the context stream: one persistent-kernel launch.
int launch_step(qwen_ctx* c) {
  {
    // a traced step starts from a cleared record (0 = stamp not reached)
    if (c->P.trace) QCUDA(c, cudaMemsetAsync(c->P.trace, 0, persist_trace_words(c->sm_count) * 8, c->st));
    if (c->P.dbg_phase >= 0) QCUDA(c, cudaMemsetAsync(c->P.dbg, 0, DBG_FLOATS * sizeof(float), c->st));
    cudaError_t e = launch_persistent(c->P, c->sm_count, c->st, c->act_int8 != 0);
    if (e != cudaSuccess) return fail(c, QWEN_ERR_CUDA, "persistent launch: %s", cudaGetErrorString(e));
  }
  return QWEN_OK;
}

// Inspect the device error word (already copied into h_err together with the
// argmax log) and clear it on the device when set.
int check_device(qwen_ctx* c) {
  if (*c->h_err != 0) {
    const int code = *c->h_err;
    QCUDA(c, cudaMemset(c->S.err, 0, 4 * sizeof(int)));
    QCUDA(c, cudaMemset(c->P.abort_flag, 0, sizeof(int)));
    QCUDA(c, cudaMemset(c->P.head_cnt, 0, sizeof(int)));
    if (code == ERR_TOKEN) return fail(c, QWEN_ERR_ARG, "token id outside [0, %d)", VOCAB);
    if (code == ERR_CTX) return fail(c, QWEN_ERR_STATE, "context or step capacity exceeded on device");
    if (code == ERR_WAIT)
      return fail(c, QWEN_ERR_DEVICE, "device wait ran out (site %d, value %d, block %d)", c->h_err[1],
                  c->h_err[2], c->h_err[3]);
    if (code == ERR_CHECK)
      return fail(c, QWEN_ERR_DEVICE, "device bounds check failed (site %d, value %d)", c->h_err[1], c->h_err[2]);
    return fail(c, QWEN_ERR_DEVICE, "device reported error %d", code);
  }
  return QWEN_OK;
}

int check_ctx(qwen_ctx* c) {
  if (!c) return fail(nullptr, QWEN_ERR_ARG, "null context");
  c->err.clear();
  QCUDA(c, cudaSetDevice(c->dev));
  return QWEN_OK;
}

}  // namespace

extern "C" {

const char* qwen_version(void) { return "qwen-b200 0.1 (sm_100a)"; }

const char* qwen_last_error(qwen_ctx* ctx) {
  if (ctx) return ctx->err.c_str();
  return g_last_error.c_str();
}

int qwen_destroy(qwen_ctx* c) {
  if (!c) return QWEN_OK;
  cudaSetDevice(c->dev);
  if (c->st) cudaStreamSynchronize(c->st);
  batch_destroy(c->be);
  batch_destroy(c->pf);
  for (void* p : c->ipc_open) cudaIpcCloseMemHandle(p);
  for (void* p : c->allocs) cudaFree(p);
  if (c->h_ctl) cudaFreeHost(c->h_ctl);
  if (c->h_err) cudaFreeHost(c->h_err);
  if (c->ev0) cudaEventDestroy(c->ev0);
  if (c->ev1) cudaEventDestroy(c->ev1);
  if (c->st) cudaStreamDestroy(c->st);
  delete c;
  return QWEN_OK;
}

}  // extern "C"

namespace {

// A context on device `dev` holding tensor-parallel shard (tp_rank, tp_world).
int create_impl(const char* blob_path, const char* index_path, int dev, int tp_rank, int tp_world,
                int max_ctx, int max_batch, qwen_ctx** out) {
  if (!out) return fail(nullptr, QWEN_ERR_ARG, "out is null");
  *out = nullptr;
  if (!blob_path || !index_path) return fail(nullptr, QWEN_ERR_ARG, "blob_path / index_path is null");
  if (max_batch < 1 || max_batch > BATCH_MAX) return fail(nullptr, QWEN_ERR_ARG, "max_batch must be in [1, %d]", BATCH_MAX);
  if (max_batch > 1 && tp_world != 1) return fail(nullptr, QWEN_ERR_ARG, "a batched context runs on one GPU");
  if (max_ctx < 1 || max_ctx > MAX_CTX) return fail(nullptr, QWEN_ERR_ARG, "max_ctx must be in [1, %d]", MAX_CTX);
  TpPlan plan;
  {
    std::string perr;
    if (!tp_plan(tp_rank, tp_world, plan, perr)) return fail(nullptr, QWEN_ERR_ARG, "%s", perr.c_str());
  }
  qwen_ctx* c = new qwen_ctx();
  c->dev = dev;
  c->tp = plan;
  c->tp_ready = tp_world == 1;
  int rc = QWEN_OK;
  auto bail = [&](int code) { std::string m = c->err; qwen_destroy(c); g_last_error = m; return code; };
  {
    cudaError_t e = cudaSetDevice(c->dev);
    if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "cudaSetDevice(%d): %s", c->dev, cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, c->dev);
    e = cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking);
    if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "stream: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
    cudaEventCreate(&c->ev0);
    cudaEventCreate(&c->ev1);
  }
  std::map<std::string, TensorEnt> idx;
  std::string perr;
  const std::string ip(index_path);
  const bool okp = ends_with(ip, ".json") ? parse_manifest(ip, idx, perr) : parse_idx(ip, idx, perr);
  if (!okp) { fail(c, QWEN_ERR_IO, "%s", perr.c_str()); return bail(QWEN_ERR_IO); }
  if ((rc = upload_blob(c, blob_path))) return bail(rc);
  if ((rc = bind_weights(c, idx))) return bail(rc);

  c->max_ctx = max_ctx;
  c->max_rope = max_ctx + 64;
  c->max_steps = 1 << 16;
  StateW& S = c->S;
  S.max_ctx = c->max_ctx;
  S.max_rope = c->max_rope;
  S.max_steps = c->max_steps;
  if ((rc = dalloc(c, &S.conv, (size_t)NLIN * CONVD * CONVK * 4)) ||
      (rc = dalloc(c, &S.rec, (size_t)NLIN * LH * LK * LV * 4)) ||
      (rc = dalloc(c, &S.kcache, (size_t)NFULL * max_ctx * KVPROJ * 4)) ||
      (rc = dalloc(c, &S.vcache, (size_t)NFULL * max_ctx * KVPROJ * 4)) ||
      (rc = dalloc(c, &S.logits, (size_t)VOCAB * 4)) ||
      (rc = dalloc(c, &S.am_part, AM_PARTS * 8)) ||
      (rc = dalloc(c, &S.err, 16 + (size_t)c->max_steps * 4)) ||
      (rc = dalloc(c, &c->d_ctl, ctl_bytes(c->max_steps))) ||
      (rc = dalloc(c, &c->Md, sizeof(ModelW))))
    return bail(rc);
  S.ids = S.err + 4;   // status block: err word, 3 spare words, then the argmax log
  S.dyn = reinterpret_cast<StepDyn*>(c->d_ctl);
  S.io = reinterpret_cast<int*>(reinterpret_cast<char*>(c->d_ctl) + sizeof(StepDyn));
  {
    float* rope = nullptr;
    if ((rc = dalloc(c, &rope, (size_t)c->max_rope * ROT * 4))) return bail(rc);
    std::vector<float> t;
    rope_table(t, c->max_rope);
    cudaError_t e = cudaMemcpy(rope, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "rope upload: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
    S.rope = rope;
    e = cudaMemcpy(c->Md, &c->Mh, sizeof(ModelW), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "model table upload: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
    if (cudaMallocHost(&c->h_ctl, ctl_bytes(c->max_steps)) != cudaSuccess ||
        cudaMallocHost((void**)&c->h_err, 16 + (size_t)c->max_steps * 4) != cudaSuccess) {
      fail(c, QWEN_ERR_CUDA, "pinned host buffers");
      return bail(QWEN_ERR_CUDA);
    }
    memset(c->h_ctl, 0, ctl_bytes(c->max_steps));
    c->h_ids = c->h_err + 4;
  }
  if (c->sm_count > AM_PARTS) { fail(c, QWEN_ERR_STATE, "too many SMs"); return bail(QWEN_ERR_STATE); }
  {
    // persistent engine: tagged activation words, counters, per-CTA schedule
    const size_t words = HID + CONVD + VDIM + VDIM + QPROJ + 2 * KVPROJ + NH * HD + FFN;
    if ((rc = dalloc(c, &c->tv_base, words * 8))) return bail(rc);
    c->tv_words = words;
    PersistArgs& P = c->P;
    unsigned long long* w = c->tv_base;
    P.tv_h = w; w += HID;
    P.tv_qkv = w; w += CONVD;
    P.tv_z = w; w += VDIM;
    P.tv_o = w; w += VDIM;
    P.tv_qg = w; w += QPROJ;
    P.tv_kvn = w; w += 2 * KVPROJ;
    P.tv_attn = w; w += NH * HD;
    P.tv_act = w; w += FFN;
    std::vector<Chunk> chunks;
    std::vector<unsigned short> first;
    std::string serr;
    if (!build_schedule(c->Mh, c->sm_count, c->tp, chunks, first, serr)) {
      fail(c, QWEN_ERR_STATE, "schedule: %s", serr.c_str());
      return bail(QWEN_ERR_STATE);
    }
    Chunk* dch = nullptr;
    unsigned short* dfirst = nullptr;
    if ((rc = dalloc(c, &dch, chunks.size() * sizeof(Chunk))) ||
        (rc = dalloc(c, &dfirst, first.size() * sizeof(unsigned short))) ||
        (rc = dalloc(c, &P.att_tv, (size_t)NKV * ATT_MAXCH * 4 * (2 + HD) * 8)) ||
        (rc = dalloc(c, &P.head_cnt, 64)) || (rc = dalloc(c, &P.abort_flag, 64)))
      return bail(rc);
    if (cudaMemcpy(dch, chunks.data(), chunks.size() * sizeof(Chunk), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dfirst, first.data(), first.size() * sizeof(unsigned short), cudaMemcpyHostToDevice) != cudaSuccess) {
      fail(c, QWEN_ERR_CUDA, "schedule upload failed");
      return bail(QWEN_ERR_CUDA);
    }
    P.chunks = dch;
    P.phase_first = dfirst;
    P.layers = &c->Md->L[0];
    P.emb_q = c->Mh.emb_q;
    P.emb_s = c->Mh.emb_s;
    {
      // the head's weights re-tiled once for the tensor cores (a second copy:
      // the row-major table still serves the embedding lookup)
      int8_t* tiles = nullptr;
      if ((rc = dalloc(c, &tiles, HEAD_TILE_BYTES))) return bail(rc);
      cudaError_t e = repack_head_tiles(c->Mh.emb_q, tiles, c->st);
      if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "head repack: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
      P.head_tiles = tiles;
    }
    {
      // every layer projection re-laid as 16-row panels for the persistent
      // engine (second copies)
      struct Job { std::vector<const int8_t*> rows; int K; const int8_t** slot; };
      std::vector<Job> jobs;
      for (int l = 0; l < NLAYER; ++l) {
        LayerW& L = c->Mh.L[l];
        Job in{{}, HID, &L.pin}, out{{}, VDIM, &L.pout}, gu{{}, HID, &L.pgu}, dn{{}, FFN, &L.pdown};
        auto rows = [](std::vector<const int8_t*>& v, const int8_t* w, int n, int K) {
          for (int r = 0; r < n; ++r) v.push_back(w + (size_t)r * K);
        };
        if (L.linear) { rows(in.rows, L.qkv_q, CONVD, HID); rows(in.rows, L.z_q, VDIM, HID); }
        else { rows(in.rows, L.q_q, QPROJ, HID); rows(in.rows, L.k_q, KVPROJ, HID); rows(in.rows, L.v_q, KVPROJ, HID); }
        rows(out.rows, L.linear ? L.out_q : L.o_q, HID, VDIM);
        for (int q = 0; q < FFN / PAIR_ROWS; ++q) {   // pair panel q: gate rows 8q.., then up rows 8q..
          rows(gu.rows, L.gate_q + (size_t)q * PAIR_ROWS * HID, PAIR_ROWS, HID);
          rows(gu.rows, L.up_q + (size_t)q * PAIR_ROWS * HID, PAIR_ROWS, HID);
        }
        rows(dn.rows, L.down_q, HID, FFN);
        jobs.push_back(std::move(in)); jobs.push_back(std::move(out));
        jobs.push_back(std::move(gu)); jobs.push_back(std::move(dn));
      }
      size_t total = 0, maxrows = 0;
      for (auto& j : jobs) { total += j.rows.size() * (size_t)j.K; maxrows = std::max(maxrows, j.rows.size()); }
      int8_t* pbuf = nullptr;
      const int8_t** drows = nullptr;
      if ((rc = dalloc(c, &pbuf, total))) return bail(rc);
      if (cudaMalloc((void**)&drows, maxrows * sizeof(void*)) != cudaSuccess) {
        fail(c, QWEN_ERR_CUDA, "panel row table");
        return bail(QWEN_ERR_CUDA);
      }
      cudaError_t e = cudaSuccess;
      size_t off = 0;
      for (auto& j : jobs) {
        if (e == cudaSuccess) e = cudaMemcpy(drows, j.rows.data(), j.rows.size() * sizeof(void*), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = repack_panels(drows, pbuf + off, (int)j.rows.size(), j.K, c->st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->st);   // the row table is reused
        *j.slot = pbuf + off;
        off += j.rows.size() * (size_t)j.K;
      }
      cudaFree(drows);
      if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "panel repack: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
      e = cudaMemcpy(c->Md, &c->Mh, sizeof(ModelW), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "model table upload: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
    }
    P.final_norm = c->Mh.final_norm;
    P.conv = S.conv; P.rec = S.rec; P.kcache = S.kcache; P.vcache = S.vcache;
    P.am_part = S.am_part;
    P.rope = S.rope;
    P.logits = S.logits;
    P.io = S.io; P.ids = S.ids; P.err = S.err; P.dyn = S.dyn;
    P.max_ctx = S.max_ctx; P.max_rope = S.max_rope; P.max_steps = S.max_steps;
    P.tp_rank = c->tp.rank;
    P.tp_world = c->tp.world;
    P.dn_h0 = c->tp.dn_h0; P.dn_h1 = c->tp.dn_h1;
    P.kv_g0 = c->tp.kv_g0; P.kv_g1 = c->tp.kv_g1;
    P.ok0 = c->tp.ok0; P.ok1 = c->tp.ok1;
    P.dk0 = c->tp.dk0; P.dk1 = c->tp.dk1;
    P.dbg_phase = -1;
    P.dbg = nullptr;
    if (c->tp.world > 1) {
      // the exchange buffer peers store into (its own allocation: IPC maps whole allocations)
      if ((rc = dalloc(c, &c->xbuf, XB_WORDS * 8))) return bail(rc);
      P.xbuf[c->tp.rank] = c->xbuf;
    }
    if (persist_max_blocks_per_sm() < 1) { fail(c, QWEN_ERR_STATE, "persistent kernel does not fit"); return bail(QWEN_ERR_STATE); }
  }
  c->max_batch = max_batch;
  if (max_batch > 1) {
    std::string berr;
    c->be = batch_create(c->Mh, c->P.head_tiles, c->S.rope, c->max_rope, max_batch, max_ctx, c->sm_count, c->st, berr);
    if (!c->be) { fail(c, QWEN_ERR_CUDA, "batched engine: %s", berr.c_str()); return bail(QWEN_ERR_CUDA); }
  }
  {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { fail(c, QWEN_ERR_CUDA, "create: %s", cudaGetErrorString(e)); return bail(QWEN_ERR_CUDA); }
  }
  *out = c;
  return QWEN_OK;
}

// A batched context's entry points report through the context's error string.
int batch_rc(qwen_ctx* c, int rc, const std::string& err) {
  if (rc != QWEN_OK) return fail(c, rc, "%s", err.c_str());
  return QWEN_OK;
}

// Every entry point that launches a step: a TP context must be connected.
int check_tp(qwen_ctx* c) {
  if (!c->tp_ready) return fail(c, QWEN_ERR_STATE, "tensor-parallel context not connected (qwen_tp_connect)");
  return QWEN_OK;
}

}  // namespace

extern "C" {

int qwen_create(const char* blob_path, const char* index_path, int n_gpus, const int* device_ids,
                int max_ctx, int max_batch, qwen_ctx** out) {
  if (n_gpus != 1)
    return fail(nullptr, QWEN_ERR_ARG, "n_gpus must be 1 (tensor parallelism: qwen_create_tp, one context per GPU)");
  return create_impl(blob_path, index_path, device_ids ? device_ids[0] : 0, 0, 1, max_ctx, max_batch, out);
}

int qwen_create_tp(const char* blob_path, const char* index_path, int device_id, int tp_rank, int tp_world,
                   int max_ctx, int max_batch, qwen_ctx** out) {
  return create_impl(blob_path, index_path, device_id, tp_rank, tp_world, max_ctx, max_batch, out);
}

int qwen_tp_plan(int tp_rank, int tp_world, int* out) {
  if (!out) return fail(nullptr, QWEN_ERR_ARG, "out is null");
  TpPlan t;
  std::string err;
  if (!tp_plan(tp_rank, tp_world, t, err)) return fail(nullptr, QWEN_ERR_ARG, "%s", err.c_str());
  const int v[QWEN_TP_PLAN_INTS] = {t.dn_h0, t.dn_h1, t.kv_g0, t.kv_g1, t.ok0, t.ok1, t.dk0, t.dk1, t.t0 * 128,
                                    t.t1 * 128};
  memcpy(out, v, sizeof v);
  return QWEN_OK;
}

int qwen_tp_export(qwen_ctx* c, void* handle_out) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (!handle_out) return fail(c, QWEN_ERR_ARG, "handle_out is null");
  if (c->tp.world == 1) return fail(c, QWEN_ERR_STATE, "not a tensor-parallel context");
  static_assert(sizeof(cudaIpcMemHandle_t) == QWEN_TP_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  QCUDA(c, cudaIpcGetMemHandle(&h, c->xbuf));
  memcpy(handle_out, &h, sizeof h);
  return QWEN_OK;
}

int qwen_tp_connect(qwen_ctx* c, const void* handles) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (!handles) return fail(c, QWEN_ERR_ARG, "handles is null");
  if (c->tp.world == 1) return fail(c, QWEN_ERR_STATE, "not a tensor-parallel context");
  if (c->tp_ready) return fail(c, QWEN_ERR_STATE, "already connected");
  const char* hb = static_cast<const char*>(handles);
  for (int r = 0; r < c->tp.world; ++r) {
    if (r == c->tp.rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)r * QWEN_TP_HANDLE_BYTES, sizeof h);
    void* p = nullptr;
    QCUDA(c, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->ipc_open.push_back(p);
    c->P.xbuf[r] = static_cast<unsigned long long*>(p);
  }
  c->tp_ready = true;
  return QWEN_OK;
}

int qwen_tp_vocab_range(qwen_ctx* c, int* lo, int* hi) {
  if (!c) return fail(nullptr, QWEN_ERR_ARG, "null context");
  if (lo) *lo = c->tp.t0 * HEAD_TM;
  if (hi) *hi = c->tp.t1 * HEAD_TM;
  return QWEN_OK;
}

int qwen_reset(qwen_ctx* c, int seq) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) {
    std::string err;
    return batch_rc(c, batch_reset(c->be, seq, err), err);
  }
  if (seq != 0) return fail(c, QWEN_ERR_ARG, "seq must be 0 (batch 1)");
  QCUDA(c, cudaMemsetAsync(c->S.conv, 0, (size_t)NLIN * CONVD * CONVK * 4, c->st));
  QCUDA(c, cudaMemsetAsync(c->S.rec, 0, (size_t)NLIN * LH * LK * LV * 4, c->st));
  QCUDA(c, cudaStreamSynchronize(c->st));
  c->pos = c->T = c->conv_base = 0;
  return QWEN_OK;
}

int qwen_set_act_int8(qwen_ctx* c, int on) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  c->act_int8 = on ? 1 : 0;
  return QWEN_OK;
}


int qwen_trace_enable(qwen_ctx* c, int on) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (on && !c->P.trace) {
    const size_t words = persist_trace_words(c->sm_count);
    if ((rc = dalloc(c, &c->P.trace, words * 8))) return rc;
  } else if (!on) {
    c->P.trace = nullptr;   // the buffer stays allocated until qwen_destroy
  }
  return QWEN_OK;
}

int qwen_trace_read(qwen_ctx* c, unsigned long long* out, int max_words, int* n_ctas,
                    int* n_phases) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (!c->P.trace) return fail(c, QWEN_ERR_STATE, "tracing is off");
  const size_t words = persist_trace_words(c->sm_count);
  if (!out || (size_t)max_words < words) return fail(c, QWEN_ERR_ARG, "need %zu words", words);
  QCUDA(c, cudaStreamSynchronize(c->st));
  QCUDA(c, cudaMemcpy(out, c->P.trace, words * 8, cudaMemcpyDeviceToHost));
  if (n_ctas) *n_ctas = c->sm_count;
  if (n_phases) *n_phases = persist_num_phases();
  return QWEN_OK;
}

int qwen_capture_phase(qwen_ctx* c, int phase) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (phase < 0) {
    c->P.dbg_phase = -1;
    return QWEN_OK;
  }
  if (phase >= persist_num_phases() - 1 || phase % 5 == 1)
    return fail(c, QWEN_ERR_ARG, "phase %d is not a GEMV phase (IN, OUT, GATEUP or DOWN of a layer)", phase);
  if (c->tp.world > 1) return fail(c, QWEN_ERR_STATE, "capture is single-GPU only");
  if (!c->P.dbg && (rc = dalloc(c, &c->P.dbg, DBG_FLOATS * sizeof(float)))) return rc;
  c->P.dbg_phase = phase;
  return QWEN_OK;
}

int qwen_capture_read(qwen_ctx* c, float* out, int max_floats) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (!c->P.dbg) return fail(c, QWEN_ERR_STATE, "no capture armed (qwen_capture_phase)");
  if (!out || max_floats < DBG_FLOATS) return fail(c, QWEN_ERR_ARG, "need %d floats", DBG_FLOATS);
  QCUDA(c, cudaStreamSynchronize(c->st));
  QCUDA(c, cudaMemcpy(out, c->P.dbg, DBG_FLOATS * sizeof(float), cudaMemcpyDeviceToHost));
  return QWEN_OK;
}

int qwen_state_import(qwen_ctx* c, int seq, const float* conv, const float* rec, const float* kc,
                      const float* vc, int T, int pos) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) {
    std::string err;
    return batch_rc(c, batch_import(c->be, seq, conv, rec, kc, vc, T, pos, err), err);
  }
  if (seq != 0) return fail(c, QWEN_ERR_ARG, "seq must be 0 (batch 1)");
  if (!conv || !rec) return fail(c, QWEN_ERR_ARG, "conv / rec is null");
  if (T < 0 || T > c->max_ctx - 1) return fail(c, QWEN_ERR_ARG, "T=%d outside [0, %d]", T, c->max_ctx - 1);
  if (pos < 0 || pos >= c->max_rope - 1) return fail(c, QWEN_ERR_ARG, "pos=%d outside the RoPE table", pos);
  if (T > 0 && (!kc || !vc)) return fail(c, QWEN_ERR_ARG, "kc / vc is null with T > 0");
  QCUDA(c, cudaMemcpy(c->S.conv, conv, (size_t)NLIN * CONVD * CONVK * 4, cudaMemcpyHostToDevice));
  QCUDA(c, cudaMemcpy(c->S.rec, rec, (size_t)NLIN * LH * LK * LV * 4, cudaMemcpyHostToDevice));
  if (T > 0) {
    for (int f = 0; f < NFULL; ++f) {
      QCUDA(c, cudaMemcpy(c->S.kcache + (size_t)f * c->max_ctx * KVPROJ, kc + (size_t)f * T * KVPROJ,
                          (size_t)T * KVPROJ * 4, cudaMemcpyHostToDevice));
      QCUDA(c, cudaMemcpy(c->S.vcache + (size_t)f * c->max_ctx * KVPROJ, vc + (size_t)f * T * KVPROJ,
                          (size_t)T * KVPROJ * 4, cudaMemcpyHostToDevice));
    }
  }
  c->T = T;
  c->pos = pos;
  c->conv_base = 0;   // logical column j now sits in ring slot j
  return QWEN_OK;
}

int qwen_state_export(qwen_ctx* c, int seq, float* conv, float* rec, float* kc, float* vc, int* T,
                      int* pos) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) {
    std::string err;
    return batch_rc(c, batch_export(c->be, seq, conv, rec, kc, vc, T, pos, err), err);
  }
  if (seq != 0) return fail(c, QWEN_ERR_ARG, "seq must be 0 (batch 1)");
  QCUDA(c, cudaStreamSynchronize(c->st));
  if (conv) {
    std::vector<float> raw((size_t)NLIN * CONVD * CONVK);
    QCUDA(c, cudaMemcpy(raw.data(), c->S.conv, raw.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t ch = 0; ch < (size_t)NLIN * CONVD; ++ch)
      for (int j = 0; j < CONVK; ++j) conv[ch * CONVK + j] = raw[ch * CONVK + ((c->conv_base + j) & 3)];
  }
  if (rec) QCUDA(c, cudaMemcpy(rec, c->S.rec, (size_t)NLIN * LH * LK * LV * 4, cudaMemcpyDeviceToHost));
  if (kc && vc && c->T > 0) {
    for (int f = 0; f < NFULL; ++f) {
      QCUDA(c, cudaMemcpy(kc + (size_t)f * c->T * KVPROJ, c->S.kcache + (size_t)f * c->max_ctx * KVPROJ,
                          (size_t)c->T * KVPROJ * 4, cudaMemcpyDeviceToHost));
      QCUDA(c, cudaMemcpy(vc + (size_t)f * c->T * KVPROJ, c->S.vcache + (size_t)f * c->max_ctx * KVPROJ,
                          (size_t)c->T * KVPROJ * 4, cudaMemcpyDeviceToHost));
    }
  }
  if (T) *T = c->T;
  if (pos) *pos = c->pos;
  return QWEN_OK;
}

int qwen_decode_step(qwen_ctx* c, const int* tok, int batch, float* logits_out, int* argmax_out) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) {
    std::string err;
    return batch_rc(c, batch_step(c->be, tok, batch, c->act_int8 != 0, logits_out, argmax_out, err), err);
  }
  if (batch != 1) return fail(c, QWEN_ERR_ARG, "batch must be 1 (a context created with max_batch 1)");
  if (!tok) return fail(c, QWEN_ERR_ARG, "tok is null");
  if (tok[0] < 0 || tok[0] >= VOCAB) return fail(c, QWEN_ERR_ARG, "token %d outside [0, %d)", tok[0], VOCAB);
  if ((rc = check_tp(c))) return rc;
  if (c->T + 1 > c->max_ctx || c->pos + 1 >= c->max_rope)
    return fail(c, QWEN_ERR_STATE, "context full (T=%d, max_ctx=%d)", c->T, c->max_ctx);
  if ((rc = ensure_seq_room(c, 1))) return rc;
  fill_dyn(c, logits_out ? 1 : 0);
  int* io = ctl_io(c);
  io[0] = 0;
  io[1] = 1;
  io[2] = tok[0];
  if ((rc = push_ctl(c, 1))) return rc;
  // Page-locked host logits (cudaMallocHost, a pinned torch tensor) are in the
  // device's address space: the head writes them there itself, over the bus
  // while it runs, instead of a copy after the kernel.  Any other pointer gets
  // the copy.  (One GPU only: a TP rank writes its vocab slice.)
  float* direct = nullptr;
  if (logits_out && c->tp.world == 1) {
    cudaPointerAttributes pa;
    void* dp = nullptr;
    if (cudaPointerGetAttributes(&pa, logits_out) == cudaSuccess && pa.type == cudaMemoryTypeHost &&
        cudaHostGetDevicePointer(&dp, logits_out, 0) == cudaSuccess && dp)   // mapped for this device
      direct = static_cast<float*>(dp);
    (void)cudaGetLastError();
  }
  if (direct) c->P.logits = direct;
  rc = launch_step(c);
  c->P.logits = c->S.logits;
  if (rc) return rc;
  QCUDA(c, cudaMemcpyAsync(c->h_err, c->S.err, 16 + sizeof(int), cudaMemcpyDeviceToHost, c->st));
  if (logits_out && !direct)
    QCUDA(c, cudaMemcpyAsync(logits_out, c->S.logits, (size_t)VOCAB * 4, cudaMemcpyDefault, c->st));
  QCUDA(c, cudaStreamSynchronize(c->st));
  c->seq += 1;
  if ((rc = check_device(c))) return rc;
  c->pos += 1;
  c->T += 1;
  c->conv_base += 1;
  if (argmax_out) argmax_out[0] = c->h_ids[0];
  return QWEN_OK;
}

int qwen_generate(qwen_ctx* c, const int* prompt, int n_prompt, int n_new, int* out_ids,
                  double* decode_seconds) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) return fail(c, QWEN_ERR_STATE, "qwen_generate runs batch-1 contexts; a batched context steps with qwen_decode_step");
  if (!prompt || n_prompt < 1 || n_new < 0) return fail(c, QWEN_ERR_ARG, "need n_prompt >= 1, n_new >= 0");
  if ((rc = check_tp(c))) return rc;
  if (n_new > 0 && !out_ids) return fail(c, QWEN_ERR_ARG, "out_ids is null");
  const int total = n_prompt + n_new;
  if (total > c->max_steps) return fail(c, QWEN_ERR_ARG, "n_prompt + n_new > %d", c->max_steps);
  if (c->T + total > c->max_ctx || c->pos + total >= c->max_rope)
    return fail(c, QWEN_ERR_STATE, "context would overflow (T=%d + %d > %d)", c->T, total, c->max_ctx);
  for (int i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= VOCAB) return fail(c, QWEN_ERR_ARG, "prompt token %d out of range", i);
  if ((rc = ensure_seq_room(c, total))) return rc;
  fill_dyn(c, 0);
  int* io = ctl_io(c);
  io[0] = 0;
  io[1] = n_prompt;
  memcpy(io + 2, prompt, sizeof(int) * n_prompt);
  if ((rc = push_ctl(c, n_prompt))) return rc;
  for (int s = 0; s < total; ++s) {
    if (s == n_prompt) QCUDA(c, cudaEventRecord(c->ev0, c->st));
    if ((rc = launch_step(c))) return rc;
  }
  QCUDA(c, cudaEventRecord(c->ev1, c->st));
  QCUDA(c, cudaMemcpyAsync(c->h_err, c->S.err, 16 + sizeof(int) * total, cudaMemcpyDeviceToHost, c->st));
  QCUDA(c, cudaStreamSynchronize(c->st));
  c->seq += total;
  if ((rc = check_device(c))) return rc;
  c->pos += total;
  c->T += total;
  c->conv_base += total;
  for (int j = 0; j < n_new; ++j) out_ids[j] = c->h_ids[n_prompt - 1 + j];
  if (decode_seconds) {
    float ms = 0.0f;
    if (n_new > 0) QCUDA(c, cudaEventElapsedTime(&ms, c->ev0, c->ev1));
    *decode_seconds = ms * 1e-3;
  }
  return QWEN_OK;
}

int qwen_prefill(qwen_ctx* c, const int* tok, int n, float* logits_out, int* argmax_out) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (c->be) return fail(c, QWEN_ERR_STATE, "qwen_prefill runs batch-1 contexts");
  if (c->tp.world != 1) return fail(c, QWEN_ERR_STATE, "qwen_prefill runs single-GPU contexts");
  if (!tok || n < 1) return fail(c, QWEN_ERR_ARG, "need n >= 1 tokens");
  if (c->T + n > c->max_ctx || c->pos + n >= c->max_rope)
    return fail(c, QWEN_ERR_STATE, "context would overflow (T=%d + %d > %d)", c->T, n, c->max_ctx);
  std::string err;
  if (!c->pf) {
    c->pf = batch_create(c->Mh, c->P.head_tiles, c->S.rope, c->max_rope, 1, 64, c->sm_count, c->st, err);
    if (!c->pf) return fail(c, QWEN_ERR_CUDA, "prefill engine: %s", err.c_str());
  }
  QCUDA(c, cudaStreamSynchronize(c->st));
  rc = batch_prefill(c->pf, c->S.conv, c->S.rec, c->S.kcache, c->S.vcache, c->max_ctx, c->conv_base, c->T, c->pos,
                     tok, n, c->act_int8 != 0, logits_out, argmax_out, err);
  if (rc) return fail(c, rc, "%s", err.c_str());
  c->pos += n;
  c->T += n;
  c->conv_base += n;
  return QWEN_OK;
}

int qwen_decode_timed(qwen_ctx* c, int batch, int steps, double* seconds) {
  int rc;
  if ((rc = check_ctx(c))) return rc;
  if (!c->be) return fail(c, QWEN_ERR_STATE, "qwen_decode_timed needs a context created with max_batch > 1");
  std::string err;
  return batch_rc(c, batch_timed_steps(c->be, batch, c->act_int8 != 0, steps, seconds, err), err);
}

// ------------------------------------------------------------------ operators

static int sm_count_current() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

static int gemv_args_ok(const void* w, int N, int K) {
  if (N < 1) return fail(nullptr, QWEN_ERR_ARG, "N must be >= 1");
  if (K < 32 || K > KMAX || K % 32) return fail(nullptr, QWEN_ERR_ARG, "K must be a multiple of 32 in [32, %d]", KMAX);
  if (reinterpret_cast<uintptr_t>(w) % 32) return fail(nullptr, QWEN_ERR_ARG, "w must be 32-byte aligned");
  return QWEN_OK;
}

int qwen_gemv_i8_f32(float* y, const int8_t* w, const float* s, const float* x, int N, int K,
                     qwen_stream_t stream) {
  if (!y || !w || !s || !x) return fail(nullptr, QWEN_ERR_ARG, "null pointer");
  int rc;
  if ((rc = gemv_args_ok(w, N, K))) return rc;
  cudaError_t e = enqueue_gemv(y, nullptr, w, s, x, nullptr, 0.0f, N, K, sm_count_current(),
                               reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(nullptr, QWEN_ERR_CUDA, "gemv_i8_f32 launch: %s", cudaGetErrorString(e));
  return QWEN_OK;
}

int qwen_gemv_i8_i8(int32_t* acc, float* y, const int8_t* w, const float* sw, const int8_t* xq,
                    float sx, int N, int K, qwen_stream_t stream) {
  if (!w || !xq || (!acc && !y) || (y && !sw)) return fail(nullptr, QWEN_ERR_ARG, "null pointer");
  int rc;
  if ((rc = gemv_args_ok(w, N, K))) return rc;
  cudaError_t e = enqueue_gemv(y, acc, w, sw, nullptr, xq, sx, N, K, sm_count_current(),
                               reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(nullptr, QWEN_ERR_CUDA, "gemv_i8_i8 launch: %s", cudaGetErrorString(e));
  return QWEN_OK;
}

int qwen_gemm_i8_i8(int32_t* acc, float* y, const int8_t* w, const float* sw, const int8_t* xq,
                    const float* sx, int N, int K, int B, qwen_stream_t stream) {
  if (!w || !xq || !sx || !sw || (!acc && !y)) return fail(nullptr, QWEN_ERR_ARG, "null pointer");
  if (N < GT_M || N % GT_M) return fail(nullptr, QWEN_ERR_ARG, "N must be a positive multiple of %d", GT_M);
  if (K < GT_KS || K % GT_KS || K > 4096) return fail(nullptr, QWEN_ERR_ARG, "K must be a multiple of %d in [%d, 4096]", GT_KS, GT_KS);
  if (B < 1 || B > BATCH_MAX) return fail(nullptr, QWEN_ERR_ARG, "B must be in [1, %d]", BATCH_MAX);
  if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(xq) % 16)
    return fail(nullptr, QWEN_ERR_ARG, "w and xq must be 16-byte aligned");
  float* yy = y;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!yy && cudaMallocAsync((void**)&yy, (size_t)N * B * 4, st) != cudaSuccess)
    return fail(nullptr, QWEN_ERR_CUDA, "gemm_i8_i8: scratch");
  cudaError_t e = gemm_i8_i8_batched(acc, yy, w, sw, xq, sx, N, K, B, st);
  if (!y) cudaFreeAsync(yy, st);
  if (e != cudaSuccess) return fail(nullptr, QWEN_ERR_CUDA, "gemm_i8_i8: %s", cudaGetErrorString(e));
  return QWEN_OK;
}

int qwen_gemv_i8_f32_argmax_noalloc(float* y, int* argmax, const int8_t* w, const float* s,
                                    const float* x, int N, int K, qwen_stream_t stream) {
  if (!argmax || !w || !s || !x) return fail(nullptr, QWEN_ERR_ARG, "null pointer");
  if (N > NA_MAX_ROWS)
    return fail(nullptr, QWEN_ERR_ARG, "N = %d exceeds the %d rows the static argmax scratch covers", N,
                NA_MAX_ROWS);
  int rc;
  if ((rc = gemv_args_ok(w, N, K))) return rc;
  cudaError_t e = enqueue_gemv_argmax_noalloc(y, argmax, w, s, x, N, K, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(nullptr, QWEN_ERR_CUDA, "gemv_i8_f32_argmax_noalloc: %s", cudaGetErrorString(e));
  return QWEN_OK;
}

int qwen_delta_rule_layer(const float* q, const float* k, const float* v, const float* g,
                          const float* beta, float* S, float* out, qwen_stream_t stream) {
  if (!q || !k || !v || !g || !beta || !S || !out) return fail(nullptr, QWEN_ERR_ARG, "null pointer");
  cudaError_t e = enqueue_delta_rule(q, k, v, g, beta, S, out, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(nullptr, QWEN_ERR_CUDA, "delta_rule launch: %s", cudaGetErrorString(e));
  return QWEN_OK;
}

}  // extern "C"
