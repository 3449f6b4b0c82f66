// Host-side file formats: config.json, BF16 safetensors, the `.lsq` quantized file.
// Byte layouts follow src/weights.rs, src/safetensors.rs and src/quant.rs:137-145 of the reference so
// that files written by either implementation are read by the other.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstring>
#include <map>

#include "ls_internal.h"

namespace ls {

// ---- a small JSON reader (objects keep their key order) -----------------------------------------

namespace {

struct J {
  enum K { Null, Bool, Num, Str, Arr, Obj } k = Null;
  bool b = false;
  double n = 0;
  std::string s;
  std::vector<J> a;
  std::vector<std::pair<std::string, J>> o;
  const J* get(const char* key) const {
    if (k != Obj) return nullptr;
    for (auto& kv : o)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  bool u64(uint64_t* out) const {
    if (k != Num || !(n >= 0) || n != std::floor(n) || !(n < 9.0e15)) return false;
    *out = (uint64_t)n;
    return true;
  }
};

struct Parser {
  const std::string& t;
  size_t i = 0;
  [[noreturn]] void fail(const char* w) { LS_THROW(-2, std::string("JSON error at byte ") + std::to_string(i) + ": " + w); }
  void ws() {
    while (i < t.size() && (t[i] == ' ' || t[i] == '\n' || t[i] == '\r' || t[i] == '\t')) i++;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) o += (char)c;
    else if (c < 0x800) { o += (char)(0xC0 | (c >> 6)); o += (char)(0x80 | (c & 63)); }
    else if (c < 0x10000) { o += (char)(0xE0 | (c >> 12)); o += (char)(0x80 | ((c >> 6) & 63)); o += (char)(0x80 | (c & 63)); }
    else { o += (char)(0xF0 | (c >> 18)); o += (char)(0x80 | ((c >> 12) & 63)); o += (char)(0x80 | ((c >> 6) & 63)); o += (char)(0x80 | (c & 63)); }
  }
  uint32_t hex4() {
    if (i + 4 > t.size()) fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; k++) {
      char c = t[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string str() {
    if (i >= t.size() || t[i] != '"') fail("expected a string");
    i++;
    std::string o;
    for (;;) {
      if (i >= t.size()) fail("unterminated string");
      char c = t[i++];
      if (c == '"') return o;
      if (c != '\\') { o += c; continue; }
      if (i >= t.size()) fail("unterminated escape");
      char e = t[i++];
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t c1 = hex4();
          if (c1 >= 0xD800 && c1 < 0xDC00) {
            if (t.compare(i, 2, "\\u") != 0) fail("unpaired surrogate");
            i += 2;
            uint32_t c2 = hex4();
            if (c2 < 0xDC00 || c2 >= 0xE000) fail("unpaired surrogate");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          } else if (c1 >= 0xDC00 && c1 < 0xE000) {
            fail("unpaired surrogate");
          }
          utf8(o, c1);
          break;
        }
        default: fail("unknown escape");
      }
    }
  }
  J val(int depth) {
    if (depth > 64) fail("nesting too deep");
    ws();
    if (i >= t.size()) fail("unexpected end");
    J j;
    char c = t[i];
    if (c == '{') {
      i++;
      j.k = J::Obj;
      ws();
      if (i < t.size() && t[i] == '}') { i++; return j; }
      for (;;) {
        ws();
        std::string key = str();
        ws();
        if (i >= t.size() || t[i] != ':') fail("expected ':'");
        i++;
        j.o.emplace_back(key, val(depth + 1));
        ws();
        if (i < t.size() && t[i] == ',') { i++; continue; }
        if (i < t.size() && t[i] == '}') { i++; return j; }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      i++;
      j.k = J::Arr;
      ws();
      if (i < t.size() && t[i] == ']') { i++; return j; }
      for (;;) {
        j.a.push_back(val(depth + 1));
        ws();
        if (i < t.size() && t[i] == ',') { i++; continue; }
        if (i < t.size() && t[i] == ']') { i++; return j; }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') { j.k = J::Str; j.s = str(); return j; }
    if (t.compare(i, 4, "true") == 0) { i += 4; j.k = J::Bool; j.b = true; return j; }
    if (t.compare(i, 5, "false") == 0) { i += 5; j.k = J::Bool; return j; }
    if (t.compare(i, 4, "null") == 0) { i += 4; return j; }
    size_t s0 = i;
    while (i < t.size() && std::strchr("+-.eE0123456789", t[i]) && t[i]) i++;
    if (i == s0) fail("unexpected character");
    std::string num = t.substr(s0, i - s0);
    char* end = nullptr;
    double v = std::strtod(num.c_str(), &end);
    if (end != num.c_str() + num.size()) fail("bad number");
    j.k = J::Num;
    j.n = v;
    return j;
  }
};

J parse_json(const std::string& text) {
  Parser p{text};
  J v = p.val(0);
  p.ws();
  if (p.i != text.size()) LS_THROW(-2, "JSON: trailing characters");
  return v;
}

std::string quote(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"') o += "\\\"";
    else if (c == '\\') o += "\\\\";
    else if (c == '\n') o += "\\n";
    else if (c == '\r') o += "\\r";
    else if (c == '\t') o += "\\t";
    else if (c < 0x20) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o += (char)c;
    }
  }
  return o + "\"";
}

WeightFormat fmt_from(uint64_t bits, uint64_t group) {
  if (bits > 255 || group > 4096) LS_THROW(-1, "config: implausible layerstream_quant values");
  WeightFormat f;
  f.bits = bits == 16 ? 255 : (int)bits;  // 16 marks bf16 internally; a stored 16 is invalid
  f.group = (int)group;
  return f;
}

void validate(const WeightFormat& f, std::initializer_list<size_t> cols) {
  if (!f.quant()) return;
  if (f.bits != 8 && f.bits != 4) LS_THROW(-1, "quantization supports 8 or 4 bits, not " + std::to_string(f.bits));
  if (f.group < 16 || f.group > 256 || f.group % 16)
    LS_THROW(-1, "group size must be a multiple of 16 between 16 and 256, not " + std::to_string(f.group));
  for (size_t c : cols)
    if (c % (size_t)f.group)
      LS_THROW(-1, "group size " + std::to_string(f.group) + " does not divide a matrix width of " + std::to_string(c));
}

}  // namespace

const char* const kSlotSuffix[N_SLOTS] = {
    "input_layernorm.weight",  "mlp.down_proj.weight",   "mlp.gate_proj.weight",  "mlp.up_proj.weight",
    "post_attention_layernorm.weight", "self_attn.k_proj.bias", "self_attn.k_proj.weight", "self_attn.o_proj.weight",
    "self_attn.q_proj.bias",   "self_attn.q_proj.weight", "self_attn.v_proj.bias", "self_attn.v_proj.weight"};

// src/weights.rs:77-141
Config parse_config(const std::string& text) {
  J j = parse_json(text);
  auto u = [&](const char* k) -> size_t {
    const J* v = j.get(k);
    uint64_t o;
    if (!v || !v->u64(&o)) LS_THROW(-1, std::string("config.json: missing integer ") + k);
    return (size_t)o;
  };
  auto f = [&](const char* k) -> float {
    const J* v = j.get(k);
    if (!v || v->k != J::Num) LS_THROW(-1, std::string("config.json: missing number ") + k);
    return (float)v->n;
  };
  auto is = [&](const char* k, const char* want) {
    const J* v = j.get(k);
    return v && v->k == J::Str && v->s == want;
  };
  if (!is("model_type", "qwen2")) LS_THROW(-1, "only Qwen2-architecture models are supported");
  if (!is("hidden_act", "silu")) LS_THROW(-1, "only SiLU activations are supported");
  const J* tie = j.get("tie_word_embeddings");
  if (!tie || tie->k != J::Bool || !tie->b) LS_THROW(-1, "only models with tied input/output embeddings are supported");
  Config c;
  c.hidden = u("hidden_size");
  c.heads = u("num_attention_heads");
  c.kv_heads = u("num_key_value_heads");
  if (!c.heads || !c.kv_heads || c.hidden % c.heads || c.heads % c.kv_heads) LS_THROW(-1, "inconsistent head configuration");
  c.head_dim = c.hidden / c.heads;
  if (c.head_dim % 2) LS_THROW(-1, "head dimension must be even for rotary embeddings");
  c.inter = u("intermediate_size");
  if (const J* q = j.get("layerstream_quant")) {
    auto get = [&](const char* k) {
      const J* v = q->get(k);
      uint64_t o;
      if (!v || !v->u64(&o)) LS_THROW(-1, std::string("config: layerstream_quant is missing ") + k);
      return o;
    };
    c.format = fmt_from(get("bits"), get("group"));
    bool eb = q->get("embed_bits") != nullptr, eg = q->get("embed_group") != nullptr;
    if (eb != eg) LS_THROW(-1, "config: layerstream_quant needs embed_bits and embed_group together");
    c.embed_format = eb ? fmt_from(get("embed_bits"), get("embed_group")) : c.format;
  }
  validate(c.format, {c.hidden, c.inter});
  validate(c.embed_format, {c.hidden});
  c.layers = u("num_hidden_layers");
  c.vocab = u("vocab_size");
  c.eps = f("rms_norm_eps");
  c.rope_theta = f("rope_theta");
  c.max_pos = u("max_position_embeddings");
  return c;
}

// src/weights.rs:188-199
std::vector<size_t> tensor_shape(int slot, const Config& c) {
  size_t h = c.hidden, i = c.inter, kv = c.kv_dim();
  switch (slot) {
    case T_INPUT_NORM: case T_POST_NORM: case T_Q_B: return {h};
    case T_K_B: case T_V_B: return {kv};
    case T_DOWN: return {h, i};
    case T_GATE: case T_UP: return {i, h};
    case T_K_W: case T_V_W: return {kv, h};
    default: return {h, h};
  }
}

bool matrix_shape(int slot, const Config& c, size_t* rows, size_t* cols) {
  auto s = tensor_shape(slot, c);
  if (s.size() != 2) return false;
  *rows = s[0];
  *cols = s[1];
  return true;
}

// src/weights.rs:215-227
LayerLayout layer_layout_for(const Config& c) {
  LayerLayout L;
  size_t off = 0;
  for (int s = 0; s < N_SLOTS; s++) {
    size_t r, k;
    size_t len = matrix_shape(s, c, &r, &k) ? r * c.format.row_bytes(k) : tensor_shape(s, c)[0] * 2;
    L.off[s] = off;
    L.len[s] = len;
    off += len;
  }
  L.total = off;
  return L;
}

void pread_all(int fd, void* buf, size_t n, uint64_t off) {
  size_t done = 0;
  while (done < n) {
    ssize_t r = ::pread(fd, (char*)buf + done, n - done, (off_t)(off + done));
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) LS_THROW(-2, "read at " + std::to_string(off + done) + " failed");
    done += (size_t)r;
  }
}

namespace {
struct Fd {
  int fd;
  uint64_t len = 0;
  explicit Fd(const std::string& p) : fd(::open(p.c_str(), O_RDONLY)) {
    if (fd < 0) LS_THROW(-2, p + ": " + std::strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) LS_THROW(-2, p + ": stat failed");
    len = (uint64_t)st.st_size;
  }
  ~Fd() { ::close(fd); }
};
}  // namespace

std::string read_file_text(const std::string& path) {
  Fd f(path);
  std::string s(f.len, '\0');
  pread_all(f.fd, &s[0], f.len, 0);
  return s;
}

// src/weights.rs:360-423
LsqFile LsqFile::open(const std::string& path) {
  Fd f(path);
  if (f.len < 8) LS_THROW(-2, "file too short to be a quantized model");
  uint8_t frame[8];
  pread_all(f.fd, frame, 8, 0);
  if (std::memcmp(frame, "LSQ1", 4) != 0) LS_THROW(-2, "not a quantized layerstream model (bad magic bytes)");
  uint32_t len = frame[4] | (frame[5] << 8) | (frame[6] << 16) | ((uint32_t)frame[7] << 24);
  if (len == 0 || len > (1u << 20) || 8 + (uint64_t)len > f.len) LS_THROW(-2, "implausible quantized header length");
  std::string text(len, '\0');
  pread_all(f.fd, &text[0], len, 8);
  J j = parse_json(text);
  const J* fm = j.get("format");
  if (!fm || fm->k != J::Str || fm->s != "layerstream-quant-1") LS_THROW(-2, "unknown quantized file format");
  auto u = [&](const char* k) {
    const J* v = j.get(k);
    uint64_t o;
    if (!v || !v->u64(&o)) LS_THROW(-2, std::string("quantized header: missing ") + k);
    return (size_t)o;
  };
  const J* cj = j.get("config_json");
  if (!cj || cj->k != J::Str) LS_THROW(-2, "quantized header: missing config");
  LsqFile q;
  q.path = path;
  q.config_text = cj->s;
  q.cfg = parse_config(q.config_text);
  if (!q.cfg.format.quant()) LS_THROW(-2, "this file does not describe quantized weights");
  q.layout = layer_layout_for(q.cfg);
  size_t lb = u("layer_bytes");
  q.embed_bytes = u("embed_bytes");
  q.norm_bytes = u("norm_bytes");
  if (q.layout.total != lb || q.cfg.vocab * q.cfg.embed_row_bytes() != q.embed_bytes || q.cfg.hidden * 2 != q.norm_bytes)
    LS_THROW(-2, "quantized header does not match the model's shape");
  q.data_start = 8 + (uint64_t)len;
  q.embed_start = q.data_start + (uint64_t)q.cfg.layers * q.layout.total;
  q.norm_start = q.embed_start + q.embed_bytes;
  if (f.len != q.norm_start + q.norm_bytes)
    LS_THROW(-2, "file is " + std::to_string(f.len) + " bytes but its header implies " + std::to_string(q.norm_start + q.norm_bytes));
  return q;
}

// src/weights.rs:271-324 + src/safetensors.rs:54-119
SafetensorsModel SafetensorsModel::open(const std::string& dir) {
  SafetensorsModel m;
  m.dir = dir;
  m.config_text = read_file_text(dir + "/config.json");
  m.cfg = parse_config(m.config_text);
  m.file = dir + "/model.safetensors";
  Fd f(m.file);
  if (f.len < 8) LS_THROW(-2, "file too short for a safetensors header");
  uint8_t lb[8];
  pread_all(f.fd, lb, 8, 0);
  uint64_t n = 0;
  for (int k = 7; k >= 0; k--) n = (n << 8) | lb[k];
  if (n == 0 || n > 100ull * 1024 * 1024 || 8 + n > f.len) LS_THROW(-2, "implausible safetensors header length");
  std::string text(n, '\0');
  pread_all(f.fd, &text[0], n, 8);
  J j = parse_json(text);
  if (j.k != J::Obj) LS_THROW(-2, "header is not a JSON object");
  struct TI { uint64_t start, end; std::vector<size_t> shape; std::string dtype; };
  std::map<std::string, TI> ts;
  for (auto& kv : j.o) {
    if (kv.first == "__metadata__") continue;
    TI ti;
    const J* d = kv.second.get("dtype");
    const J* sh = kv.second.get("shape");
    const J* of = kv.second.get("data_offsets");
    if (!d || d->k != J::Str || !sh || sh->k != J::Arr || !of || of->k != J::Arr || of->a.size() != 2)
      LS_THROW(-2, kv.first + ": malformed tensor entry");
    ti.dtype = d->s;
    size_t numel = 1;
    for (auto& e : sh->a) {
      uint64_t v;
      if (!e.u64(&v)) LS_THROW(-2, "bad shape entry");
      ti.shape.push_back((size_t)v);
      numel *= (size_t)v;
    }
    uint64_t a, b;
    if (!of->a[0].u64(&a) || !of->a[1].u64(&b)) LS_THROW(-2, "bad offset");
    ti.start = 8 + n + a;
    ti.end = 8 + n + b;
    if (ti.end < ti.start || ti.end > f.len) LS_THROW(-2, kv.first + ": data range is outside the file");
    size_t es = (ti.dtype == "BF16" || ti.dtype == "F16") ? 2 : ti.dtype == "F32" ? 4 : 0;
    if (!es) LS_THROW(-2, kv.first + ": unsupported dtype " + ti.dtype);
    if (ti.end - ti.start != numel * es) LS_THROW(-2, kv.first + ": size does not match shape");
    ts[kv.first] = ti;
  }
  auto bf16 = [&](const std::string& name, const std::vector<size_t>& shape) -> const TI& {
    auto it = ts.find(name);
    if (it == ts.end()) LS_THROW(-2, "tensor " + name + " not found");
    if (it->second.dtype != "BF16") LS_THROW(-2, name + ": expected BF16, found " + it->second.dtype);
    if (it->second.shape != shape) LS_THROW(-2, name + ": unexpected shape");
    return it->second;
  };
  const TI& e = bf16("model.embed_tokens.weight", {m.cfg.vocab, m.cfg.hidden});
  const TI& nm = bf16("model.norm.weight", {m.cfg.hidden});
  bool have = false;
  for (size_t l = 0; l < m.cfg.layers; l++) {
    struct It { int slot; uint64_t s, e; };
    std::vector<It> items;
    for (int s = 0; s < N_SLOTS; s++) {
      const TI& t = bf16("model.layers." + std::to_string(l) + "." + kSlotSuffix[s], tensor_shape(s, m.cfg));
      items.push_back({s, t.start, t.end});
    }
    std::sort(items.begin(), items.end(), [](const It& a, const It& b) { return a.s < b.s; });
    for (size_t k = 1; k < items.size(); k++)
      if (items[k - 1].e != items[k].s) LS_THROW(-2, "layer " + std::to_string(l) + ": tensors are not contiguous in the file");
    LayerLayout L;
    for (auto& it : items) {
      L.off[it.slot] = (size_t)(it.s - items[0].s);
      L.len[it.slot] = (size_t)(it.e - it.s);
    }
    L.total = (size_t)(items.back().e - items[0].s);
    if (!have) {
      m.layout = L;
      have = true;
    } else {
      for (int s = 0; s < N_SLOTS; s++)
        if (L.off[s] != m.layout.off[s] || L.len[s] != m.layout.len[s])
          LS_THROW(-2, "layer " + std::to_string(l) + " is laid out differently from layer 0");
    }
    m.layer_start.push_back(items[0].s);
  }
  if (!have) LS_THROW(-2, "model has no layers");
  m.embed_start = e.start;
  m.embed_len = (size_t)(e.end - e.start);
  m.norm_start = nm.start;
  m.norm_len = (size_t)(nm.end - nm.start);
  return m;
}

// src/quant.rs:137-145
std::string inject_quant(const std::string& cfg, WeightFormat body, WeightFormat embed) {
  size_t end = cfg.rfind('}');
  if (end == std::string::npos) LS_THROW(-1, "config.json has no closing brace");
  std::string head = cfg.substr(0, end);
  while (!head.empty() && std::strchr(" \n\r\t", head.back()) && head.back()) head.pop_back();
  std::string extra = (embed == body) ? std::string()
                                      : ",\"embed_bits\":" + std::to_string(embed.bits) + ",\"embed_group\":" +
                                            std::to_string(embed.group);
  return head + ",\"layerstream_quant\":{\"bits\":" + std::to_string(body.bits) + ",\"group\":" +
         std::to_string(body.group) + extra + "}}";
}

// src/seal.rs:574-591 (SealedLayout::to_json): the header's JSON text, in the same key order and
// string escaping, so that a file sealed here is byte-identical to the reference's for the same key
// and nonce prefix.
std::string sealed_header_json(const std::string& config_text, const LayerLayout& layout, size_t layer_chunk,
                               size_t embed_chunk_rows, size_t final_norm_bytes) {
  std::string ranges;
  for (int s = 0; s < N_SLOTS; s++) {
    if (s) ranges += ",";
    ranges += "[" + std::to_string(layout.off[s]) + "," + std::to_string(layout.len[s]) + "]";
  }
  return "{\"format\":\"layerstream-sealed-1\",\"config_json\":" + quote(config_text) + ",\"layer_bytes\":" +
         std::to_string(layout.total) + ",\"layer_chunk\":" + std::to_string(layer_chunk) + ",\"embed_chunk_rows\":" +
         std::to_string(embed_chunk_rows) + ",\"final_norm_bytes\":" + std::to_string(final_norm_bytes) +
         ",\"layer_layout\":[" + ranges + "]}";
}

bool is_sealed_file(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return false;
  char m[4] = {0, 0, 0, 0};
  const ssize_t r = ::pread(fd, m, 4, 0);
  ::close(fd);
  return r == 4 && std::memcmp(m, "LSS1", 4) == 0;
}

// src/seal.rs:13-27 (layout), 593-627 (SealedLayout::from_json), 860-903 (SealedSource::open)
SealedFile SealedFile::open(const std::string& path) {
  Fd f(path);
  SealedFile sf;
  sf.path = path;
  sf.file_len = f.len;
  uint8_t frame[kSealFrame];
  if (f.len < kSealFrame) LS_THROW(-2, "file too short to be a sealed model");
  pread_all(f.fd, frame, kSealFrame, 0);
  if (std::memcmp(frame, "LSS1", 4) != 0) LS_THROW(-2, "not a sealed layerstream model (bad magic bytes)");
  const uint32_t version = frame[4] | (frame[5] << 8) | (frame[6] << 16) | ((uint32_t)frame[7] << 24);
  if (version != 1) LS_THROW(-2, "unsupported sealed format version " + std::to_string(version));
  std::memcpy(sf.nonce_prefix, frame + 8, 8);
  const uint32_t hl = frame[16] | (frame[17] << 8) | (frame[18] << 16) | ((uint32_t)frame[19] << 24);
  if (hl == 0 || hl > (1u << 20) || kSealFrame + (uint64_t)hl > f.len) LS_THROW(-2, "implausible sealed header length");
  sf.aad_prefix.resize(kSealFrame + hl);
  pread_all(f.fd, sf.aad_prefix.data(), sf.aad_prefix.size(), 0);
  const std::string text(reinterpret_cast<const char*>(sf.aad_prefix.data()) + kSealFrame, hl);
  J j = parse_json(text);
  const J* fm = j.get("format");
  if (!fm || fm->k != J::Str || fm->s != "layerstream-sealed-1") LS_THROW(-2, "unknown sealed format");
  auto u = [&](const char* k) {
    const J* v = j.get(k);
    uint64_t o;
    if (!v || !v->u64(&o)) LS_THROW(-2, std::string("sealed header: missing ") + k);
    return (size_t)o;
  };
  const J* cj = j.get("config_json");
  if (!cj || cj->k != J::Str) LS_THROW(-2, "sealed header: missing config");
  sf.config_text = cj->s;
  sf.cfg = parse_config(sf.config_text);
  const J* lj = j.get("layer_layout");
  if (!lj || lj->k != J::Arr) LS_THROW(-2, "sealed header: missing layout");
  if (lj->a.size() != N_SLOTS) LS_THROW(-2, "sealed header: layout must list 12 tensors");
  size_t total = 0;
  for (int s = 0; s < N_SLOTS; s++) {
    const J& pr = lj->a[s];
    uint64_t o, l;
    if (pr.k != J::Arr || pr.a.size() != 2 || !pr.a[0].u64(&o) || !pr.a[1].u64(&l)) LS_THROW(-2, "sealed header: bad layout entry");
    sf.layout.off[s] = (size_t)o;
    sf.layout.len[s] = (size_t)l;
    total = std::max(total, (size_t)(o + l));
  }
  sf.layout.total = total;
  if (u("layer_bytes") != total) LS_THROW(-2, "sealed header: layer layout does not add up");
  sf.layer_chunk = u("layer_chunk");
  sf.embed_chunk_rows = u("embed_chunk_rows");
  if (sf.layer_chunk == 0 || sf.embed_chunk_rows == 0) LS_THROW(-2, "sealed header: zero chunk size");
  sf.final_norm_bytes = u("final_norm_bytes");
  if (sf.final_norm_bytes != sf.cfg.hidden * 2 || sf.cfg.layers == 0 || sf.cfg.layers > 4096)
    LS_THROW(-2, "sealed header: inconsistent sizes");
  // every tensor of the layer block must be the size the configuration implies
  for (int s = 0; s < N_SLOTS; s++) {
    size_t r, k;
    const size_t want = matrix_shape(s, sf.cfg, &r, &k) ? r * sf.cfg.format.row_bytes(k) : tensor_shape(s, sf.cfg)[0] * 2;
    if (sf.layout.len[s] != want) LS_THROW(-2, "sealed header: a tensor of the layer layout has the wrong size");
  }
  const uint64_t nch = sf.n_chunks();
  sf.tags_off = sf.aad_prefix.size();
  sf.ct_base = sf.tags_off + 16 * nch;
  if (f.len != sf.ct_base + sf.total_plain())
    LS_THROW(-2, "file is " + std::to_string(f.len) + " bytes but its header implies " + std::to_string(sf.ct_base + sf.total_plain()));
  sf.tags.resize(16 * nch);
  pread_all(f.fd, sf.tags.data(), sf.tags.size(), sf.tags_off);
  return sf;
}

// src/weights.rs:345-358
std::string lsq_header_bytes(const std::string& config_text, size_t layer_bytes, size_t embed_bytes, size_t norm_bytes) {
  std::string json = "{\"format\":\"layerstream-quant-1\",\"config_json\":" + quote(config_text) +
                     ",\"layer_bytes\":" + std::to_string(layer_bytes) + ",\"embed_bytes\":" + std::to_string(embed_bytes) +
                     ",\"norm_bytes\":" + std::to_string(norm_bytes) + "}";
  std::string out = "LSQ1";
  uint32_t n = (uint32_t)json.size();
  for (int k = 0; k < 4; k++) out += (char)((n >> (8 * k)) & 0xff);
  return out + json;
}

}  // namespace ls
