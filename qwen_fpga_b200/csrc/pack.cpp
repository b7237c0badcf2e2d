// Blob packer of libqwenb200: a Hugging Face safetensors snapshot of the
// Qwen3.5 text decoder -> the packed int8 blob, its JSON manifest and the flat
// index that qwen_create loads.  The same output as the reference's
// scripts/pack_weights.py:28-101 (tensor order, 4 KiB alignment, int8 rows +
// fp32 row scales, fp32 tensors as-is, manifest fields), with the reference's
// loader rules (golden/loader.py:36-73: BF16 widened by a 16-bit shift, the
// "model.language_model." prefix dropped, vision and MTP tensors skipped) and
// quantiser (golden/quant.py:43-49), written as host C++ so a deployment
// needs no Python to produce its weights.
#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <dirent.h>

#include "../../include/qwen_b200.h"

namespace {

// ---------------------------------------------------------------- minimal JSON
//
// Enough of JSON for config.json and safetensors headers: objects, arrays,
// strings (escapes kept verbatim, names here have none), numbers, literals.
// Every value keeps its source text, so the manifest can copy config values
// through unchanged.
struct JVal {
  enum Kind { OBJ, ARR, STR, NUM, LIT } kind = LIT;
  std::string raw;                                   // source text of the value
  std::string str;                                   // STR: contents
  std::vector<std::pair<std::string, JVal>> obj;     // OBJ: members in order
  std::vector<JVal> arr;                             // ARR
  const JVal* get(const std::string& k) const {
    for (auto& m : obj)
      if (m.first == k) return &m.second;
    return nullptr;
  }
};

struct JParser {
  const std::string& s;
  size_t i = 0;
  std::string err;
  explicit JParser(const std::string& src) : s(src) {}
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool fail(const char* what) {
    if (err.empty()) err = std::string(what) + " at byte " + std::to_string(i);
    return false;
  }
  bool str(std::string& out) {
    if (i >= s.size() || s[i] != '"') return fail("expected string");
    ++i;
    out.clear();
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < s.size()) out += s[i++];
      out += s[i++];
    }
    if (i >= s.size()) return fail("unterminated string");
    ++i;
    return true;
  }
  bool val(JVal& v, int depth = 0) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (i >= s.size()) return fail("unexpected end");
    const size_t b = i;
    const char c = s[i];
    if (c == '{') {
      v.kind = JVal::OBJ;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') { ++i; v.raw = s.substr(b, i - b); return true; }
      for (;;) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') return fail("expected ':'");
        ++i;
        JVal m;
        if (!val(m, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(m));
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == '}') { ++i; break; }
        return fail("expected ',' or '}'");
      }
    } else if (c == '[') {
      v.kind = JVal::ARR;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') { ++i; v.raw = s.substr(b, i - b); return true; }
      for (;;) {
        JVal m;
        if (!val(m, depth + 1)) return false;
        v.arr.push_back(std::move(m));
        ws();
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        if (i < s.size() && s[i] == ']') { ++i; break; }
        return fail("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = JVal::STR;
      if (!str(v.str)) return false;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      v.kind = JVal::NUM;
      while (i < s.size() && (std::strchr("+-.eE", s[i]) || (s[i] >= '0' && s[i] <= '9'))) ++i;
    } else {
      v.kind = JVal::LIT;
      for (const char* lit : {"true", "false", "null"})
        if (s.compare(i, std::strlen(lit), lit) == 0) { i += std::strlen(lit); v.raw = lit; return true; }
      return fail("unexpected character");
    }
    v.raw = s.substr(b, i - b);
    return true;
  }
};

bool parse_json(const std::string& text, JVal& out, std::string& err) {
  JParser p(text);
  if (!p.val(out)) { err = p.err; return false; }
  p.ws();
  if (p.i != text.size()) { err = "trailing bytes after JSON value"; return false; }
  return true;
}

bool read_file(const std::string& path, std::string& out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[1 << 16];
  size_t n;
  out.clear();
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
  std::fclose(f);
  return true;
}

// ---------------------------------------------------------------- the snapshot

struct SrcTensor {
  std::string file;
  std::string dtype;               // BF16, F16, F32, I32, I64
  std::vector<long long> shape;
  unsigned long long lo = 0, hi = 0;   // absolute byte range in the file
};

long long numel(const std::vector<long long>& sh) {
  long long n = 1;
  for (long long d : sh) n *= d;
  return n;
}

// IEEE half -> float (exact).
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  int e = (h >> 10) & 0x1f;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0x1f) {
    bits = sign | 0x7f800000u | (m << 13);
  } else if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {   // subnormal: normalise
      e = 1;
      while (!(m & 0x400u)) { m <<= 1; --e; }
      m &= 0x3ffu;
      bits = sign | (uint32_t)(e + 112) << 23 | (m << 13);
    }
  } else {
    bits = sign | (uint32_t)(e + 112) << 23 | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Tensor t as fp32 (golden/loader.py:28-33, 60-64: BF16 is the top half of an
// fp32, widened by a shift; other types converted value by value).
bool load_f32(const SrcTensor& t, std::vector<float>& out, std::string& err) {
  const long long n = numel(t.shape);
  const int es = t.dtype == "BF16" || t.dtype == "F16" ? 2 : (t.dtype == "F32" || t.dtype == "I32" ? 4 : 8);
  if (t.dtype != "BF16" && t.dtype != "F16" && t.dtype != "F32" && t.dtype != "I32" && t.dtype != "I64") {
    err = "unhandled dtype " + t.dtype;
    return false;
  }
  if ((long long)(t.hi - t.lo) != n * es) { err = "data_offsets do not match the shape"; return false; }
  std::vector<unsigned char> raw((size_t)(t.hi - t.lo));
  FILE* f = std::fopen(t.file.c_str(), "rb");
  if (!f) { err = "cannot open " + t.file; return false; }
  const bool ok = fseeko(f, (off_t)t.lo, SEEK_SET) == 0 && std::fread(raw.data(), 1, raw.size(), f) == raw.size();
  std::fclose(f);
  if (!ok) { err = "short read in " + t.file; return false; }
  out.resize((size_t)n);
  for (long long i = 0; i < n; ++i) {
    const unsigned char* p = raw.data() + i * es;
    if (t.dtype == "BF16") {
      const uint32_t u = (uint32_t)(p[0] | p[1] << 8) << 16;
      std::memcpy(&out[i], &u, 4);
    } else if (t.dtype == "F16") {
      out[i] = half_to_float((uint16_t)(p[0] | p[1] << 8));
    } else if (t.dtype == "F32") {
      std::memcpy(&out[i], p, 4);
    } else if (t.dtype == "I32") {
      int32_t v;
      std::memcpy(&v, p, 4);
      out[i] = (float)v;
    } else {
      int64_t v;
      std::memcpy(&v, p, 8);
      out[i] = (float)v;
    }
  }
  return true;
}

// Every text tensor of the snapshot's *.safetensors files (golden/loader.py:36-73).
bool scan_snapshot(const std::string& dir, std::map<std::string, SrcTensor>& out, std::string& err) {
  std::vector<std::string> files;
  DIR* d = opendir(dir.c_str());
  if (!d) { err = "cannot open snapshot directory " + dir; return false; }
  while (dirent* e = readdir(d)) {
    const std::string n = e->d_name;
    if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(dir + "/" + n);
  }
  closedir(d);
  if (files.empty()) { err = "no .safetensors in " + dir; return false; }
  std::sort(files.begin(), files.end());
  for (const auto& path : files) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) { err = "cannot open " + path; return false; }
    unsigned char lb[8];
    if (std::fread(lb, 1, 8, f) != 8) { std::fclose(f); err = "short header in " + path; return false; }
    unsigned long long hlen = 0;
    for (int k = 7; k >= 0; --k) hlen = hlen << 8 | lb[k];
    if (hlen > (1ull << 30)) { std::fclose(f); err = "implausible header size in " + path; return false; }
    std::string hdr((size_t)hlen, '\0');
    const bool ok = std::fread(&hdr[0], 1, hdr.size(), f) == hdr.size();
    std::fclose(f);
    if (!ok) { err = "short header in " + path; return false; }
    JVal h;
    std::string perr;
    if (!parse_json(hdr, h, perr) || h.kind != JVal::OBJ) { err = path + ": header: " + perr; return false; }
    const unsigned long long base = 8 + hlen;
    for (const auto& m : h.obj) {
      const std::string& name = m.first;
      if (name == "__metadata__") continue;
      if (name.rfind("model.visual", 0) == 0 || name.rfind("mtp.", 0) == 0) continue;
      const JVal* dt = m.second.get("dtype");
      const JVal* sh = m.second.get("shape");
      const JVal* of = m.second.get("data_offsets");
      if (!dt || !sh || !of || sh->kind != JVal::ARR || of->kind != JVal::ARR || of->arr.size() != 2) {
        err = path + ": malformed entry " + name;
        return false;
      }
      SrcTensor t;
      t.file = path;
      t.dtype = dt->str;
      for (const auto& x : sh->arr) t.shape.push_back(std::stoll(x.raw));
      t.lo = base + std::stoull(of->arr[0].raw);
      t.hi = base + std::stoull(of->arr[1].raw);
      std::string key = name;
      const std::string pre = "model.language_model.";
      if (key.compare(0, pre.size(), pre) == 0) key = key.substr(pre.size());
      out[key] = std::move(t);
    }
  }
  return true;
}

// ---------------------------------------------------------------- layout

// The order the decode step reads the weights (scripts/pack_weights.py:28-47).
std::vector<std::string> read_order(const std::vector<std::string>& layer_types) {
  std::vector<std::string> o;
  for (size_t i = 0; i < layer_types.size(); ++i) {
    const std::string p = "layers." + std::to_string(i);
    o.push_back(p + ".input_layernorm.weight");
    if (layer_types[i] == "linear_attention") {
      const std::string a = p + ".linear_attn.";
      for (const char* s : {"in_proj_qkv.weight", "in_proj_z.weight", "in_proj_b.weight", "in_proj_a.weight",
                            "conv1d.weight", "A_log", "dt_bias", "norm.weight", "out_proj.weight"})
        o.push_back(a + s);
    } else {
      const std::string a = p + ".self_attn.";
      for (const char* s : {"q_proj.weight", "k_proj.weight", "v_proj.weight", "q_norm.weight", "k_norm.weight",
                            "o_proj.weight"})
        o.push_back(a + s);
    }
    o.push_back(p + ".post_attention_layernorm.weight");
    for (const char* s : {"mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"})
      o.push_back(p + "." + s);
  }
  o.push_back("norm.weight");
  o.push_back("embed_tokens.weight");
  return o;
}

// The GEMV weights stored as int8 (golden/quant.py:22-40, should_quant).
bool is_quant(const std::string& name) {
  static const char* suf[] = {"in_proj_qkv.weight", "in_proj_z.weight", "linear_attn.out_proj.weight",
                              "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
                              "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                              "self_attn.o_proj.weight", "embed_tokens.weight"};
  for (const char* s : suf) {
    const size_t n = std::strlen(s);
    if (name.size() >= n && name.compare(name.size() - n, n, s) == 0) return true;
  }
  return false;
}

// Per-row symmetric int8 (golden/quant.py:43-49): scale = amax / 127 in fp32
// (1 for an all-zero row), q = clip(rint(w / scale), -127, 127), the quotient
// in fp32 and rint rounding half to even, as numpy does.
void quant_rows(const float* w, long long rows, long long cols, int8_t* q, float* scale) {
  for (long long r = 0; r < rows; ++r) {
    const float* row = w + r * cols;
    float amax = 0.0f;
    for (long long c = 0; c < cols; ++c) amax = std::fmax(amax, std::fabs(row[c]));
    const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
    scale[r] = s;
    for (long long c = 0; c < cols; ++c) {
      float v = std::nearbyint(row[c] / s);
      v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
      q[r * cols + c] = (int8_t)v;
    }
  }
}

std::string shape_json(const std::vector<long long>& sh) {
  std::string o = "[";
  for (size_t k = 0; k < sh.size(); ++k) o += (k ? ", " : "") + std::to_string(sh[k]);
  return o + "]";
}

}  // namespace

namespace qb {
void set_last_error(const std::string& msg);   // runtime.cu: the text qwen_last_error(NULL) returns
}

extern "C" int qwen_pack_blob(const char* snapshot_dir, const char* out_blob) {
  auto bad = [](int code, const std::string& m) { qb::set_last_error(m); return code; };
  if (!snapshot_dir || !out_blob) return bad(QWEN_ERR_ARG, "snapshot_dir / out_blob is null");
  const std::string dir(snapshot_dir), out(out_blob);
  // the text config (golden/loader.py:76-78)
  std::string text, err;
  if (!read_file(dir + "/config.json", text)) return bad(QWEN_ERR_IO, "cannot read " + dir + "/config.json");
  JVal cfgroot;
  if (!parse_json(text, cfgroot, err)) return bad(QWEN_ERR_IO, "config.json: " + err);
  const JVal* cfg = cfgroot.get("text_config");
  if (!cfg || cfg->kind != JVal::OBJ) return bad(QWEN_ERR_IO, "config.json has no text_config object");
  const JVal* lt = cfg->get("layer_types");
  if (!lt || lt->kind != JVal::ARR) return bad(QWEN_ERR_IO, "text_config has no layer_types");
  std::vector<std::string> types;
  for (const auto& x : lt->arr) types.push_back(x.str);
  // the tensors, checked against the read order (scripts/pack_weights.py:59-63)
  std::map<std::string, SrcTensor> W;
  if (!scan_snapshot(dir, W, err)) return bad(QWEN_ERR_IO, err);
  const std::vector<std::string> order = read_order(types);
  std::map<std::string, int> in_order;
  for (const auto& n : order) in_order[n] = 1;
  std::string missing, extra;
  for (const auto& n : order)
    if (!W.count(n) && missing.size() < 200) missing += " " + n;
  for (const auto& kv : W)
    if (!in_order.count(kv.first) && extra.size() < 200) extra += " " + kv.first;
  if (!missing.empty() || !extra.empty())
    return bad(QWEN_ERR_IO, "tensors do not match the read order; missing:" + missing + "; extra:" + extra);
  // blob: every tensor 4 KiB aligned, int8 rows then fp32 scales, or fp32 (pack_weights.py:66-90)
  const unsigned long long ALIGN = 4096;
  FILE* f = std::fopen((out + ".partial").c_str(), "wb");
  if (!f) return bad(QWEN_ERR_IO, "cannot write " + out + ".partial");
  std::string man_t, idx;
  unsigned long long off = 0;
  std::vector<float> w;
  std::vector<int8_t> q;
  std::vector<float> s;
  const std::vector<char> zeros(ALIGN, 0);
  bool ok = true;
  for (size_t k = 0; k < order.size() && ok; ++k) {
    const std::string& name = order[k];
    const SrcTensor& t = W[name];
    const unsigned long long pad = (ALIGN - off % ALIGN) % ALIGN;
    if (pad) { ok = std::fwrite(zeros.data(), 1, pad, f) == pad; off += pad; }
    if (!ok || !load_f32(t, w, err)) { ok = false; break; }
    const long long n = numel(t.shape);
    char line[512];
    if (is_quant(name) && t.shape.size() == 2) {
      const long long rows = t.shape[0], cols = t.shape[1];
      q.resize((size_t)n);
      s.resize((size_t)rows);
      quant_rows(w.data(), rows, cols, q.data(), s.data());
      ok = std::fwrite(q.data(), 1, q.size(), f) == q.size() && std::fwrite(s.data(), 4, s.size(), f) == s.size();
      std::snprintf(line, sizeof line,
                    "{\"name\": \"%s\", \"shape\": %s, \"offset\": %llu, \"dtype\": \"int8\", \"nbytes\": %lld, "
                    "\"scale_offset\": %llu, \"scale_nbytes\": %lld}",
                    name.c_str(), shape_json(t.shape).c_str(), off, n, off + (unsigned long long)n, 4 * rows);
      man_t += std::string(k ? ",\n  " : "  ") + line;
      std::snprintf(line, sizeof line, "%s %llu %lld 1 %llu %lld %lld %lld\n", name.c_str(), off, n,
                    off + (unsigned long long)n, 4 * rows, rows, cols);
      idx += line;
      off += (unsigned long long)n + 4ull * rows;
    } else {
      ok = std::fwrite(w.data(), 4, w.size(), f) == w.size();
      std::snprintf(line, sizeof line, "{\"name\": \"%s\", \"shape\": %s, \"offset\": %llu, \"dtype\": \"fp32\", "
                    "\"nbytes\": %lld}", name.c_str(), shape_json(t.shape).c_str(), off, 4 * n);
      man_t += std::string(k ? ",\n  " : "  ") + line;
      std::snprintf(line, sizeof line, "%s %llu %lld 0 0 0 %lld %lld\n", name.c_str(), off, 4 * n,
                    t.shape.size() > 0 ? t.shape[0] : 0, t.shape.size() > 1 ? t.shape[1] : 0);
      idx += line;
      off += 4ull * (unsigned long long)n;
    }
  }
  if (std::fclose(f) != 0) ok = false;
  if (!ok) {
    std::remove((out + ".partial").c_str());
    return bad(QWEN_ERR_IO, err.empty() ? "write failed: " + std::string(std::strerror(errno)) : err);
  }
  if (std::rename((out + ".partial").c_str(), out.c_str()) != 0) return bad(QWEN_ERR_IO, "cannot rename to " + out);
  // manifest (pack_weights.py:92-101): the kept config keys copied verbatim
  std::string man = "{\"config\": {";
  bool first = true;
  for (const char* key : {"hidden_size", "num_hidden_layers", "layer_types", "head_dim", "num_attention_heads",
                          "num_key_value_heads", "intermediate_size", "vocab_size", "rms_norm_eps",
                          "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim",
                          "linear_conv_kernel_dim", "rope_parameters"}) {
    const JVal* v = cfg->get(key);
    if (!v) return bad(QWEN_ERR_IO, std::string("text_config has no ") + key);
    man += std::string(first ? "" : ", ") + "\"" + key + "\": " + v->raw;
    first = false;
  }
  man += "},\n \"align\": 4096, \"total_bytes\": " + std::to_string(off) + ",\n \"tensors\": [\n" + man_t + "\n ]}\n";
  const size_t dot = out.find_last_of('.');
  const size_t slash = out.find_last_of('/');
  const std::string stem = (dot != std::string::npos && (slash == std::string::npos || dot > slash)) ? out.substr(0, dot) : out;
  FILE* mf = std::fopen((stem + ".manifest.json").c_str(), "wb");
  FILE* xf = std::fopen((stem + ".idx").c_str(), "wb");
  const bool wok = mf && xf && std::fwrite(man.data(), 1, man.size(), mf) == man.size() &&
                   std::fwrite(idx.data(), 1, idx.size(), xf) == idx.size();
  if (mf) std::fclose(mf);
  if (xf) std::fclose(xf);
  if (!wok) return bad(QWEN_ERR_IO, "cannot write " + stem + ".manifest.json / .idx");
  return QWEN_OK;
}
