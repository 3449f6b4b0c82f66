// ORACLE — test infrastructure, not product code.
//
// A CPU restatement of layerstream's speculative-decode verify path, written in C++ because the
// reference is Rust and no Rust toolchain exists here. It follows the reference's floating-point
// operation order exactly (8-lane accumulators, per-group scale * partial sum, sequential lane sums,
// f64 inv_freq, libm expf/sinf/cosf/pow), so that its logits are bit-comparable with a Linux build
// of the reference. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, and
// only as the checker or the timed CPU baseline, never as the product path.
//
// Parity pinning: the reference ships no golden vectors for random-init weights (its golden.json pins
// the real Qwen checkpoint, which is absent). This restatement is pinned against every known-answer
// and property test the reference holds for the path: src/quant.rs:272-373, src/kernels.rs:285-347,
// src/weights.rs:430-464, src/model.rs:372-376, tests/spec.rs:63-193, tests/quant.rs:75-248 and
// tests/pipeline.rs:170-229, ported to tests/test_oracle_*.py.
//
// Build: g++ -O3 -std=c++17 -ffp-contract=off -fno-fast-math -shared -fPIC (see oracle/Makefile).
// -ffp-contract=off matters: Rust never fuses a*b+c into an FMA, so neither may this file.

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <limits>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <utility>
#include <vector>

namespace orc {

using Err = std::runtime_error;

// ---------------------------------------------------------------------------------------------
// bf16 helpers (src/kernels.rs:7-23, src/quant.rs:25-33)
// ---------------------------------------------------------------------------------------------

static inline float bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

static inline float bf16_at(const uint8_t* bytes, size_t i) {
    return bf16_to_f32((uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8)));
}

static inline uint32_t f2u(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

static inline float u2f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// src/quant.rs:26-33: round to nearest bf16, ties to even; NaN passes through.
float bf16_round(float v) {
    uint32_t bits = f2u(v);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return v;
    uint32_t lsb = (bits >> 16) & 1u;
    return u2f((bits + 0x7fffu + lsb) & 0xffff0000u);
}

// ---------------------------------------------------------------------------------------------
// Weight formats (src/weights.rs:15-55)
// ---------------------------------------------------------------------------------------------

struct WeightFormat {
    int bits = 16;  // 16 = bf16, else 8 or 4
    size_t group = 0;
    bool is_quant() const { return bits != 16; }
    bool operator==(const WeightFormat& o) const { return bits == o.bits && group == o.group; }
    bool operator!=(const WeightFormat& o) const { return !(*this == o); }
    // src/weights.rs:26-31
    size_t row_bytes(size_t cols) const {
        if (!is_quant()) return cols * 2;
        return cols * (size_t)bits / 8 + cols / group * 2;
    }
    // src/weights.rs:34-47
    void validate(const std::vector<size_t>& cols) const {
        if (!is_quant()) return;
        if (bits != 8 && bits != 4) throw Err("quantization supports 8 or 4 bits, not " + std::to_string(bits));
        if (group < 16 || group > 256 || group % 16 != 0)
            throw Err("group size must be a multiple of 16 between 16 and 256, not " + std::to_string(group));
        for (size_t c : cols)
            if (c % group != 0)
                throw Err("group size " + std::to_string(group) + " does not divide a matrix width of " + std::to_string(c));
    }
};

// ---------------------------------------------------------------------------------------------
// Dot products and row dequantisation (src/kernels.rs:25-121)
// ---------------------------------------------------------------------------------------------

// Rust's f32 Sum folds from -0.0 in order.
static inline float sum8(const float* a) {
    float s = -0.0f;
    for (int k = 0; k < 8; k++) s = s + a[k];
    return s;
}

// src/kernels.rs:27-43
float dot_bf16(const uint8_t* w, const float* x, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t full = n / 8;
    for (size_t c = 0; c < full; c++) {
        for (int k = 0; k < 8; k++) acc[k] += bf16_at(w, c * 8 + k) * x[c * 8 + k];
    }
    float sum = sum8(acc);
    for (size_t i = full * 8; i < n; i++) sum += bf16_at(w, i) * x[i];
    return sum;
}

// src/kernels.rs:53-68
float dot_q8(const uint8_t* row, const float* x, size_t cols, size_t group) {
    const uint8_t* data = row;
    const uint8_t* scales = row + cols;
    float total = 0.0f;
    size_t ng = cols / group;
    for (size_t g = 0; g < ng; g++) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const uint8_t* qg = data + g * group;
        const float* xg = x + g * group;
        for (size_t c = 0; c < group / 8; c++)
            for (int k = 0; k < 8; k++) acc[k] += (float)(int8_t)qg[c * 8 + k] * xg[c * 8 + k];
        total += bf16_at(scales, g) * sum8(acc);
    }
    return total;
}

// src/kernels.rs:74-92
float dot_q4(const uint8_t* row, const float* x, size_t cols, size_t group) {
    const uint8_t* data = row;
    const uint8_t* scales = row + cols / 2;
    size_t half = group / 2;
    float total = 0.0f;
    size_t ng = cols / group;
    for (size_t g = 0; g < ng; g++) {
        const uint8_t* bytes = data + g * half;
        const float* lo = x + g * group;
        const float* hi = lo + half;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (size_t c = 0; c < half / 8; c++) {
            for (int k = 0; k < 8; k++) {
                uint8_t b = bytes[c * 8 + k];
                float a = (float)((int)(b & 15) - 8) * lo[c * 8 + k];
                float h = (float)((int)(b >> 4) - 8) * hi[c * 8 + k];
                acc[k] += a + h;
            }
        }
        total += bf16_at(scales, g) * sum8(acc);
    }
    return total;
}

float dot_fmt(const WeightFormat& f, const uint8_t* row, const float* x, size_t cols) {
    if (!f.is_quant()) return dot_bf16(row, x, cols);
    if (f.bits == 8) return dot_q8(row, x, cols, f.group);
    return dot_q4(row, x, cols, f.group);
}

// src/kernels.rs:95-121
void dequant_row(const WeightFormat& f, const uint8_t* raw, size_t cols, float* out) {
    if (!f.is_quant()) {
        for (size_t i = 0; i < cols; i++) out[i] = bf16_at(raw, i);
        return;
    }
    const uint8_t* data = raw;
    const uint8_t* scales = raw + cols * (size_t)f.bits / 8;
    size_t G = f.group;
    for (size_t g = 0; g < cols / G; g++) {
        float s = bf16_at(scales, g);
        if (f.bits == 8) {
            for (size_t j = 0; j < G; j++) out[g * G + j] = (float)(int8_t)data[g * G + j] * s;
        } else {
            size_t half = G / 2;
            for (size_t j = 0; j < half; j++) {
                uint8_t b = data[g * half + j];
                out[g * G + j] = (float)((int)(b & 15) - 8) * s;
                out[g * G + j + half] = (float)((int)(b >> 4) - 8) * s;
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Thread pool (src/pool.rs:77-137): persistent workers pull task indices from an atomic counter;
// the caller works too. Only scheduling — values never depend on it.
// ---------------------------------------------------------------------------------------------

class Pool {
  public:
    explicit Pool(size_t threads) : workers_(threads > 0 ? threads - 1 : 0) {
        for (size_t i = 0; i < workers_; i++) handles_.emplace_back([this] { worker(); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            shutdown_ = true;
        }
        start_.notify_all();
        for (auto& h : handles_) h.join();
    }
    size_t threads() const { return workers_ + 1; }

    void run(size_t n_tasks, const std::function<void(size_t)>& f) {
        if (n_tasks == 0) return;
        if (workers_ == 0 || n_tasks == 1) {
            for (size_t i = 0; i < n_tasks; i++) f(i);
            return;
        }
        std::lock_guard<std::mutex> one(run_lock_);
        std::atomic<size_t> next{0};
        {
            std::lock_guard<std::mutex> g(mu_);
            job_f_ = &f;
            job_n_ = n_tasks;
            job_next_ = &next;
            pending_ = workers_;
            generation_++;
        }
        start_.notify_all();
        run_tasks(&f, n_tasks, &next);
        std::unique_lock<std::mutex> g(mu_);
        done_.wait(g, [this] { return pending_ == 0; });
        job_f_ = nullptr;
    }

  private:
    static void run_tasks(const std::function<void(size_t)>* f, size_t n, std::atomic<size_t>* next) {
        for (;;) {
            size_t i = next->fetch_add(1, std::memory_order_relaxed);
            if (i >= n) break;
            (*f)(i);
        }
    }
    void worker() {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(size_t)>* f;
            size_t n;
            std::atomic<size_t>* next;
            {
                std::unique_lock<std::mutex> g(mu_);
                start_.wait(g, [&] { return shutdown_ || generation_ != seen; });
                if (shutdown_) return;
                seen = generation_;
                f = job_f_;
                n = job_n_;
                next = job_next_;
            }
            run_tasks(f, n, next);
            {
                std::lock_guard<std::mutex> g(mu_);
                if (--pending_ == 0) done_.notify_all();
            }
        }
    }
    size_t workers_;
    std::vector<std::thread> handles_;
    std::mutex mu_, run_lock_;
    std::condition_variable start_, done_;
    bool shutdown_ = false;
    uint64_t generation_ = 0;
    const std::function<void(size_t)>* job_f_ = nullptr;
    size_t job_n_ = 0;
    std::atomic<size_t>* job_next_ = nullptr;
    size_t pending_ = 0;
};

// src/kernels.rs:123-203: y[t][r] = dot(row r, x[t]); rows split into blocks of 16 across the pool.
static const size_t ROW_BLOCK = 16;

void matmul(Pool& pool, const WeightFormat& f, const uint8_t* w, size_t rows, size_t cols, const float* x,
            size_t t, float* y) {
    size_t rb = f.row_bytes(cols);
    size_t n_tasks = (rows + ROW_BLOCK - 1) / ROW_BLOCK;
    pool.run(n_tasks, [&](size_t task) {
        size_t r0 = task * ROW_BLOCK, r1 = std::min(rows, r0 + ROW_BLOCK);
        for (size_t r = r0; r < r1; r++)
            for (size_t tt = 0; tt < t; tt++) y[tt * rows + r] = dot_fmt(f, w + r * rb, x + tt * cols, cols);
    });
}

// src/kernels.rs:206-214
void add_bias_bf16(float* y, const uint8_t* bias, size_t n, size_t t) {
    for (size_t r = 0; r < t; r++)
        for (size_t i = 0; i < n; i++) y[r * n + i] += bf16_at(bias, i);
}

// src/kernels.rs:217-228
void rms_norm_bf16(const float* x, const uint8_t* weight, size_t n, size_t t, float eps, float* out) {
    for (size_t r = 0; r < t; r++) {
        const float* xr = x + r * n;
        float* orow = out + r * n;
        float ss = -0.0f;
        for (size_t i = 0; i < n; i++) ss = ss + xr[i] * xr[i];
        float mean_sq = ss / (float)n;
        float inv = 1.0f / std::sqrt(mean_sq + eps);
        for (size_t i = 0; i < n; i++) orow[i] = xr[i] * inv * bf16_at(weight, i);
    }
}

// src/kernels.rs:231-238
void rms_norm_f32(const float* x, const float* weight, size_t n, float eps, float* out) {
    float ss = -0.0f;
    for (size_t i = 0; i < n; i++) ss = ss + x[i] * x[i];
    float mean_sq = ss / (float)n;
    float inv = 1.0f / std::sqrt(mean_sq + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * weight[i];
}

// src/kernels.rs:242-252: rotate-half RoPE. Rust's sin_cos is (sin(), cos()), each a libm call.
void rope_inplace(float* head, const float* inv_freq, size_t hd, size_t pos) {
    size_t half = hd / 2;
    for (size_t i = 0; i < half; i++) {
        float angle = (float)pos * inv_freq[i];
        float s = sinf(angle), c = cosf(angle);
        float a = head[i], b = head[i + half];
        head[i] = a * c - b * s;
        head[i + half] = b * c + a * s;
    }
}

// src/kernels.rs:254-265
void softmax_inplace(float* v, size_t n) {
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t i = 0; i < n; i++) mx = std::fmax(mx, v[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        v[i] = expf(v[i] - mx);
        sum += v[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) v[i] *= inv;
}

// src/kernels.rs:268-270
static inline float silu(float x) { return x / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------------------------
// Minimal JSON (src/json.rs): objects keep key order.
// ---------------------------------------------------------------------------------------------

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double n = 0;
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const std::string& k) const {
        if (kind != Obj) return nullptr;
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    bool as_u64(uint64_t* out) const {
        if (kind != Num || !(n >= 0.0) || n != std::floor(n) || !(n < 9.0e15)) return false;
        *out = (uint64_t)n;
        return true;
    }
};

struct JsonParser {
    const std::string& t;
    size_t i = 0;
    explicit JsonParser(const std::string& text) : t(text) {}
    [[noreturn]] void fail(const std::string& what) { throw Err("JSON error at byte " + std::to_string(i) + ": " + what); }
    void ws() {
        while (i < t.size() && (t[i] == ' ' || t[i] == '\n' || t[i] == '\r' || t[i] == '\t')) i++;
    }
    bool eat(const char* lit) {
        size_t n = std::strlen(lit);
        if (t.compare(i, n, lit) == 0) {
            i += n;
            return true;
        }
        return false;
    }
    static void put_utf8(std::string& o, uint32_t cp) {
        if (cp < 0x80) o += (char)cp;
        else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) { o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
        else { o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
    }
    uint32_t hex4() {
        if (i + 4 > t.size()) fail("short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; k++) {
            char c = t[i++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail("bad \\u escape");
        }
        return v;
    }
    std::string str() {
        if (t[i] != '"') fail("expected string");
        i++;
        std::string o;
        for (;;) {
            if (i >= t.size()) fail("unterminated string");
            char c = t[i++];
            if (c == '"') break;
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
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00) {
                        if (!eat("\\u")) fail("unpaired surrogate");
                        uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo >= 0xE000) fail("unpaired surrogate");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) fail("unpaired surrogate");
                    put_utf8(o, cp);
                    break;
                }
                default: fail("unknown escape");
            }
        }
        return o;
    }
    Json value(int depth) {
        if (depth > 128) fail("nesting too deep");
        ws();
        if (i >= t.size()) fail("unexpected end");
        Json j;
        char c = t[i];
        if (c == '{') {
            i++;
            j.kind = Json::Obj;
            ws();
            if (i < t.size() && t[i] == '}') { i++; return j; }
            for (;;) {
                ws();
                if (i >= t.size()) fail("unexpected end");
                std::string k = str();
                ws();
                if (i >= t.size() || t[i] != ':') fail("expected ':'");
                i++;
                Json v = value(depth + 1);
                j.obj.emplace_back(std::move(k), std::move(v));
                ws();
                if (i < t.size() && t[i] == ',') { i++; continue; }
                if (i < t.size() && t[i] == '}') { i++; break; }
                fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            i++;
            j.kind = Json::Arr;
            ws();
            if (i < t.size() && t[i] == ']') { i++; return j; }
            for (;;) {
                j.arr.push_back(value(depth + 1));
                ws();
                if (i < t.size() && t[i] == ',') { i++; continue; }
                if (i < t.size() && t[i] == ']') { i++; break; }
                fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            j.kind = Json::Str;
            j.s = str();
        } else if (eat("true")) { j.kind = Json::Bool; j.b = true; }
        else if (eat("false")) { j.kind = Json::Bool; j.b = false; }
        else if (eat("null")) { j.kind = Json::Null; }
        else {
            size_t st = i;
            while (i < t.size() && (std::strchr("-+.eE0123456789", t[i]) != nullptr) && t[i] != 0) i++;
            std::string num = t.substr(st, i - st);
            if (num.empty()) fail("unexpected character");
            char* end = nullptr;
            errno = 0;
            double v = std::strtod(num.c_str(), &end);
            if (end != num.c_str() + num.size()) fail("bad number " + num);
            j.kind = Json::Num;
            j.n = v;
        }
        return j;
    }
    static Json parse(const std::string& text) {
        JsonParser p(text);
        Json v = p.value(0);
        p.ws();
        if (p.i != text.size()) throw Err("trailing characters at byte " + std::to_string(p.i));
        return v;
    }
};

// src/json.rs:79-106 (strings only: used for the .lsq header)
std::string json_quote(const std::string& s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': o += "\\\""; break;
            case '\\': o += "\\\\"; break;
            case '\n': o += "\\n"; break;
            case '\r': o += "\\r"; break;
            case '\t': o += "\\t"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    std::snprintf(b, sizeof b, "\\u%04x", c);
                    o += b;
                } else {
                    o += (char)c;
                }
        }
    }
    return o + "\"";
}

// ---------------------------------------------------------------------------------------------
// Config (src/weights.rs:57-156)
// ---------------------------------------------------------------------------------------------

struct Config {
    WeightFormat format, embed_format;
    size_t hidden = 0, inter = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0, max_pos = 0;
    float eps = 0, rope_theta = 0;
    size_t kv_dim() const { return kv_heads * head_dim; }
    size_t row_bytes() const { return embed_format.row_bytes(hidden); }

    static Config from_json(const Json& j) {
        auto u = [&](const char* k) -> size_t {
            const Json* v = j.get(k);
            uint64_t o;
            if (!v || !v->as_u64(&o)) throw Err(std::string("config.json: missing integer ") + k);
            return (size_t)o;
        };
        auto f = [&](const char* k) -> float {
            const Json* v = j.get(k);
            if (!v || v->kind != Json::Num) throw Err(std::string("config.json: missing number ") + k);
            return (float)v->n;
        };
        auto sv = [&](const char* k) -> std::string {
            const Json* v = j.get(k);
            return (v && v->kind == Json::Str) ? v->s : std::string("\x01");
        };
        if (sv("model_type") != "qwen2") throw Err("only Qwen2-architecture models are supported");
        if (sv("hidden_act") != "silu") throw Err("only SiLU activations are supported");
        const Json* tie = j.get("tie_word_embeddings");
        if (!tie || tie->kind != Json::Bool || !tie->b) throw Err("only models with tied input/output embeddings are supported");
        Config c;
        c.hidden = u("hidden_size");
        c.heads = u("num_attention_heads");
        c.kv_heads = u("num_key_value_heads");
        if (c.heads == 0 || c.kv_heads == 0 || c.hidden % c.heads != 0 || c.heads % c.kv_heads != 0)
            throw Err("inconsistent head configuration");
        c.head_dim = c.hidden / c.heads;
        if (c.head_dim % 2 != 0) throw Err("head dimension must be even for rotary embeddings");
        c.inter = u("intermediate_size");
        const Json* q = j.get("layerstream_quant");
        if (q) {
            auto get = [&](const char* k) -> uint64_t {
                const Json* v = q->get(k);
                uint64_t o;
                if (!v || !v->as_u64(&o)) throw Err(std::string("config: layerstream_quant is missing ") + k);
                return o;
            };
            auto quant = [&](const char* bk, const char* gk) {
                uint64_t b = get(bk), g = get(gk);
                if (b > 255 || g > 4096) throw Err("config: implausible layerstream_quant values");
                WeightFormat w;
                w.bits = (int)b;
                w.group = (size_t)g;
                if (w.bits == 16) w.bits = 255;  // 16 is this file's bf16 marker; keep it invalid
                return w;
            };
            c.format = quant("bits", "group");
            bool eb = q->get("embed_bits") != nullptr, eg = q->get("embed_group") != nullptr;
            if (!eb && !eg) c.embed_format = c.format;
            else if (eb && eg) c.embed_format = quant("embed_bits", "embed_group");
            else throw Err("config: layerstream_quant needs embed_bits and embed_group together");
        }
        c.format.validate({c.hidden, c.inter});
        c.embed_format.validate({c.hidden});
        c.layers = u("num_hidden_layers");
        c.vocab = u("vocab_size");
        c.eps = f("rms_norm_eps");
        c.rope_theta = f("rope_theta");
        c.max_pos = u("max_position_embeddings");
        return c;
    }
};

// Tensor slots inside a layer block (src/weights.rs:158-186)
enum { T_INPUT_NORM = 0, T_DOWN, T_GATE, T_UP, T_POST_NORM, T_K_B, T_K_W, T_O_W, T_Q_B, T_Q_W, T_V_B, T_V_W, N_TENSORS };
static const char* SUFFIX[N_TENSORS] = {
    "input_layernorm.weight", "mlp.down_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
    "post_attention_layernorm.weight", "self_attn.k_proj.bias", "self_attn.k_proj.weight", "self_attn.o_proj.weight",
    "self_attn.q_proj.bias", "self_attn.q_proj.weight", "self_attn.v_proj.bias", "self_attn.v_proj.weight"};

// src/weights.rs:188-199
std::vector<size_t> expected_shape(int slot, const Config& c) {
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

// src/weights.rs:203-211
bool matrix_shape(int slot, const Config& c, size_t* rows, size_t* cols) {
    switch (slot) {
        case T_DOWN: case T_GATE: case T_UP: case T_K_W: case T_O_W: case T_Q_W: case T_V_W: {
            auto s = expected_shape(slot, c);
            *rows = s[0];
            *cols = s[1];
            return true;
        }
        default: return false;
    }
}

struct LayerLayout {
    size_t off[N_TENSORS] = {0}, len[N_TENSORS] = {0};
    size_t total = 0;
    bool operator==(const LayerLayout& o) const {
        if (total != o.total) return false;
        for (int s = 0; s < N_TENSORS; s++)
            if (off[s] != o.off[s] || len[s] != o.len[s]) return false;
        return true;
    }
};

// src/weights.rs:215-227
LayerLayout layer_layout_for(const Config& c) {
    LayerLayout L;
    size_t o = 0;
    for (int s = 0; s < N_TENSORS; s++) {
        size_t rows, cols, len;
        if (matrix_shape(s, c, &rows, &cols)) len = rows * c.format.row_bytes(cols);
        else len = expected_shape(s, c)[0] * 2;
        L.off[s] = o;
        L.len[s] = len;
        o += len;
    }
    L.total = o;
    return L;
}

// ---------------------------------------------------------------------------------------------
// Files: safetensors (src/safetensors.rs), .lsq (src/weights.rs:327-423)
// ---------------------------------------------------------------------------------------------

struct File {
    int fd = -1;
    uint64_t len = 0;
    explicit File(const std::string& path) {
        fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) throw Err(path + ": " + std::strerror(errno));
        struct stat st;
        if (fstat(fd, &st) != 0) throw Err(path + ": stat failed");
        len = (uint64_t)st.st_size;
    }
    ~File() {
        if (fd >= 0) ::close(fd);
    }
    void read_at(uint8_t* buf, size_t n, uint64_t off) const {
        size_t done = 0;
        while (done < n) {
            ssize_t r = ::pread(fd, buf + done, n - done, (off_t)(off + done));
            if (r <= 0) throw Err("read at " + std::to_string(off) + " failed");
            done += (size_t)r;
        }
    }
};

static std::string read_text(const std::string& path) {
    File f(path);
    std::string s(f.len, '\0');
    f.read_at((uint8_t*)s.data(), f.len, 0);
    return s;
}

struct TensorInfo {
    std::string dtype;
    std::vector<size_t> shape;
    uint64_t start = 0, end = 0;
};

// src/safetensors.rs:54-119
struct StHeader {
    std::vector<std::pair<std::string, TensorInfo>> tensors;
    uint64_t data_start = 0;
    static StHeader read(const std::string& path) {
        File f(path);
        if (f.len < 8) throw Err("file too short for a safetensors header");
        uint8_t lb[8];
        f.read_at(lb, 8, 0);
        uint64_t n = 0;
        for (int k = 7; k >= 0; k--) n = (n << 8) | lb[k];
        if (n == 0 || n > 100ull * 1024 * 1024 || 8 + n > f.len) throw Err("implausible safetensors header length");
        std::string text(n, '\0');
        f.read_at((uint8_t*)text.data(), n, 8);
        Json j = JsonParser::parse(text);
        if (j.kind != Json::Obj) throw Err("header is not a JSON object");
        StHeader h;
        h.data_start = 8 + n;
        for (auto& kv : j.obj) {
            if (kv.first == "__metadata__") continue;
            TensorInfo ti;
            const Json* d = kv.second.get("dtype");
            if (!d || d->kind != Json::Str) throw Err("tensor without dtype");
            ti.dtype = d->s;
            const Json* sh = kv.second.get("shape");
            if (!sh || sh->kind != Json::Arr) throw Err("tensor without shape");
            size_t numel = 1;
            for (auto& e : sh->arr) {
                uint64_t v;
                if (!e.as_u64(&v)) throw Err("bad shape entry");
                ti.shape.push_back((size_t)v);
                numel *= (size_t)v;
            }
            const Json* offs = kv.second.get("data_offsets");
            if (!offs || offs->kind != Json::Arr || offs->arr.size() != 2) throw Err(kv.first + ": bad data_offsets");
            uint64_t a, b;
            if (!offs->arr[0].as_u64(&a) || !offs->arr[1].as_u64(&b)) throw Err("bad offset");
            ti.start = h.data_start + a;
            ti.end = h.data_start + b;
            if (ti.end < ti.start || ti.end > f.len) throw Err(kv.first + ": data range is outside the file");
            size_t esz = (ti.dtype == "BF16" || ti.dtype == "F16") ? 2 : (ti.dtype == "F32" ? 4 : 0);
            if (esz == 0) throw Err(kv.first + ": unsupported dtype " + ti.dtype);
            if ((ti.end - ti.start) != numel * esz) throw Err(kv.first + ": size does not match shape");
            h.tensors.emplace_back(kv.first, ti);
        }
        return h;
    }
    const TensorInfo& bf16_tensor(const std::string& name, const std::vector<size_t>& shape) const {
        for (auto& kv : tensors) {
            if (kv.first != name) continue;
            if (kv.second.dtype != "BF16") throw Err(name + ": expected BF16, found " + kv.second.dtype);
            if (kv.second.shape != shape) throw Err(name + ": unexpected shape");
            return kv.second;
        }
        throw Err("tensor " + name + " not found");
    }
};

static const char* QUANT_MAGIC = "LSQ1";
static const char* QUANT_FORMAT = "layerstream-quant-1";

struct QuantHeader {
    std::string config_text;
    size_t layer_bytes = 0, embed_bytes = 0, norm_bytes = 0;
    uint64_t data_start = 0;

    // src/weights.rs:345-358
    std::string to_bytes() const {
        std::string json = std::string("{\"format\":\"") + QUANT_FORMAT + "\",\"config_json\":" + json_quote(config_text) +
                           ",\"layer_bytes\":" + std::to_string(layer_bytes) + ",\"embed_bytes\":" +
                           std::to_string(embed_bytes) + ",\"norm_bytes\":" + std::to_string(norm_bytes) + "}";
        std::string out(QUANT_MAGIC, 4);
        uint32_t n = (uint32_t)json.size();
        for (int k = 0; k < 4; k++) out += (char)((n >> (8 * k)) & 0xff);
        return out + json;
    }

    // src/weights.rs:360-386
    static QuantHeader read(const std::string& path) {
        File f(path);
        if (f.len < 8) throw Err("file too short to be a quantized model");
        uint8_t frame[8];
        f.read_at(frame, 8, 0);
        if (std::memcmp(frame, QUANT_MAGIC, 4) != 0) throw Err("not a quantized layerstream model (bad magic bytes)");
        uint32_t len = (uint32_t)frame[4] | ((uint32_t)frame[5] << 8) | ((uint32_t)frame[6] << 16) | ((uint32_t)frame[7] << 24);
        if (len == 0 || len > (1u << 20)) throw Err("implausible quantized header length");
        if (8 + (uint64_t)len > f.len) throw Err("quantized header: file too short");
        std::string text(len, '\0');
        f.read_at((uint8_t*)text.data(), len, 8);
        Json j = JsonParser::parse(text);
        const Json* fmt = j.get("format");
        if (!fmt || fmt->kind != Json::Str || fmt->s != QUANT_FORMAT) throw Err("unknown quantized file format");
        auto u = [&](const char* k) -> size_t {
            const Json* v = j.get(k);
            uint64_t o;
            if (!v || !v->as_u64(&o)) throw Err(std::string("quantized header: missing ") + k);
            return (size_t)o;
        };
        QuantHeader h;
        const Json* cj = j.get("config_json");
        if (!cj || cj->kind != Json::Str) throw Err("quantized header: missing config");
        h.config_text = cj->s;
        h.layer_bytes = u("layer_bytes");
        h.embed_bytes = u("embed_bytes");
        h.norm_bytes = u("norm_bytes");
        h.data_start = 8 + (uint64_t)len;
        return h;
    }
};

// src/quant.rs:137-145
std::string inject_quant(const std::string& config_text, int bits, size_t group, bool has_embed, int eb, size_t eg) {
    size_t end = config_text.rfind('}');
    if (end == std::string::npos) throw Err("config.json has no closing brace");
    std::string head = config_text.substr(0, end);
    while (!head.empty() && (head.back() == ' ' || head.back() == '\n' || head.back() == '\r' || head.back() == '\t'))
        head.pop_back();
    std::string extra = has_embed ? (",\"embed_bits\":" + std::to_string(eb) + ",\"embed_group\":" + std::to_string(eg)) : "";
    return head + ",\"layerstream_quant\":{\"bits\":" + std::to_string(bits) + ",\"group\":" + std::to_string(group) + extra + "}}";
}

// src/weights.rs:254-325, 389-423
struct ModelFiles {
    Config cfg;
    std::string path;
    LayerLayout layout;
    std::vector<uint64_t> layer_start;
    uint64_t embed_start = 0, norm_start = 0;
    size_t embed_len = 0, norm_len = 0;
    std::vector<float> final_norm;

    static ModelFiles open_dir(const std::string& dir) {
        ModelFiles m;
        m.cfg = Config::from_json(JsonParser::parse(read_text(dir + "/config.json")));
        m.path = dir + "/model.safetensors";
        StHeader h = StHeader::read(m.path);
        const TensorInfo& emb = h.bf16_tensor("model.embed_tokens.weight", {m.cfg.vocab, m.cfg.hidden});
        const TensorInfo& nrm = h.bf16_tensor("model.norm.weight", {m.cfg.hidden});
        bool have = false;
        for (size_t l = 0; l < m.cfg.layers; l++) {
            struct It { int slot; uint64_t s, e; };
            std::vector<It> items;
            for (int s = 0; s < N_TENSORS; s++) {
                const TensorInfo& t = h.bf16_tensor("model.layers." + std::to_string(l) + "." + SUFFIX[s], expected_shape(s, m.cfg));
                items.push_back({s, t.start, t.end});
            }
            std::sort(items.begin(), items.end(), [](const It& a, const It& b) { return a.s < b.s; });
            for (size_t k = 1; k < items.size(); k++)
                if (items[k - 1].e != items[k].s) throw Err("layer " + std::to_string(l) + ": tensors are not contiguous in the file");
            uint64_t span0 = items[0].s, span1 = items.back().e;
            LayerLayout L;
            for (auto& it : items) {
                L.off[it.slot] = (size_t)(it.s - span0);
                L.len[it.slot] = (size_t)(it.e - it.s);
            }
            L.total = (size_t)(span1 - span0);
            if (!have) { m.layout = L; have = true; }
            else if (!(m.layout == L)) throw Err("layer " + std::to_string(l) + " is laid out differently from layer 0");
            m.layer_start.push_back(span0);
        }
        if (!have) throw Err("model has no layers");
        m.embed_start = emb.start;
        m.embed_len = (size_t)(emb.end - emb.start);
        m.norm_start = nrm.start;
        m.norm_len = (size_t)(nrm.end - nrm.start);
        File f(m.path);
        std::vector<uint8_t> raw(m.norm_len);
        f.read_at(raw.data(), raw.size(), m.norm_start);
        m.final_norm.resize(m.cfg.hidden);
        for (size_t i = 0; i < m.cfg.hidden; i++) m.final_norm[i] = bf16_at(raw.data(), i);
        return m;
    }

    static ModelFiles open_quantized(const std::string& path) {
        QuantHeader h = QuantHeader::read(path);
        ModelFiles m;
        m.cfg = Config::from_json(JsonParser::parse(h.config_text));
        if (!m.cfg.format.is_quant()) throw Err("this file does not describe quantized weights");
        m.layout = layer_layout_for(m.cfg);
        if (m.layout.total != h.layer_bytes || m.cfg.vocab * m.cfg.row_bytes() != h.embed_bytes || m.cfg.hidden * 2 != h.norm_bytes)
            throw Err("quantized header does not match the model's shape");
        File f(path);
        m.embed_start = h.data_start + (uint64_t)m.cfg.layers * m.layout.total;
        m.norm_start = m.embed_start + h.embed_bytes;
        if (f.len != m.norm_start + h.norm_bytes) throw Err("file size does not match its header");
        m.embed_len = h.embed_bytes;
        m.norm_len = h.norm_bytes;
        m.path = path;
        for (size_t l = 0; l < m.cfg.layers; l++) m.layer_start.push_back(h.data_start + (uint64_t)l * m.layout.total);
        std::vector<uint8_t> raw(m.norm_len);
        f.read_at(raw.data(), raw.size(), m.norm_start);
        m.final_norm.resize(m.cfg.hidden);
        for (size_t i = 0; i < m.cfg.hidden; i++) m.final_norm[i] = bf16_at(raw.data(), i);
        return m;
    }
};

// ---------------------------------------------------------------------------------------------
// Quantizer (src/quant.rs:35-251)
// ---------------------------------------------------------------------------------------------

static const float CLIPS[9] = {1.0f, 0.95f, 0.9f, 0.85f, 0.8f, 0.75f, 0.7f, 0.65f, 0.6f};

// Rust f32::round: half away from zero == C roundf. clamp(-qmax, qmax) then `as i8`.
static inline float qround(float v, float inv, float qmax) {
    float r = roundf(v * inv);
    if (r < -qmax) r = -qmax;
    if (r > qmax) r = qmax;
    return r;
}

// src/quant.rs:39-75
float quantize_group(int bits, const float* w, size_t n, bool clip_search, int8_t* q, double* err_out) {
    float qmax = bits == 8 ? 127.0f : 7.0f;
    float amax = 0.0f;
    for (size_t i = 0; i < n; i++) amax = std::fmax(amax, std::fabs(w[i]));
    auto zeros = [&]() {
        for (size_t i = 0; i < n; i++) q[i] = 0;
        double e = 0;
        for (size_t i = 0; i < n; i++) e += (double)(w[i] * w[i]);
        *err_out = e;
        return 0.0f;
    };
    if (amax == 0.0f || !std::isfinite(amax)) return zeros();
    size_t nclips = clip_search ? 9 : 1;
    double best_e = std::numeric_limits<double>::infinity();
    float best_s = 0.0f;
    for (size_t ci = 0; ci < nclips; ci++) {
        float s = bf16_round(CLIPS[ci] * amax / qmax);
        if (s == 0.0f) continue;
        float inv = 1.0f / s;
        double err = 0.0;
        for (size_t i = 0; i < n; i++) {
            float d = w[i] - qround(w[i], inv, qmax) * s;
            err += (double)(d * d);
        }
        if (err < best_e) {
            best_e = err;
            best_s = s;
        }
    }
    if (best_s == 0.0f) return zeros();
    float inv = 1.0f / best_s;
    for (size_t i = 0; i < n; i++) q[i] = (int8_t)qround(w[i], inv, qmax);
    *err_out = best_e;
    return best_s;
}

// src/quant.rs:79-104
void quantize_row(const WeightFormat& f, const float* row, size_t cols, bool clip, uint8_t* out, double* err, double* norm) {
    if (!f.is_quant()) throw Err("quantize_row needs a quantized format");
    if (f.group > 256 || cols % f.group != 0) throw Err("row width must be a multiple of the group size");
    uint8_t* data = out;
    uint8_t* scales = out + cols * (size_t)f.bits / 8;
    int8_t q[256];
    double e = 0, nn = 0;
    size_t G = f.group;
    for (size_t g = 0; g < cols / G; g++) {
        const float* wg = row + g * G;
        double ge;
        float s = quantize_group(f.bits, wg, G, clip, q, &ge);
        e += ge;
        double gn = 0;
        for (size_t i = 0; i < G; i++) gn += (double)(wg[i] * wg[i]);
        nn += gn;
        uint16_t sb = (uint16_t)(f2u(s) >> 16);
        scales[2 * g] = (uint8_t)(sb & 0xff);
        scales[2 * g + 1] = (uint8_t)(sb >> 8);
        if (f.bits == 8) {
            for (size_t j = 0; j < G; j++) data[g * G + j] = (uint8_t)q[j];
        } else {
            size_t half = G / 2;
            for (size_t j = 0; j < half; j++)
                data[g * half + j] = (uint8_t)((uint8_t)(q[j] + 8) | (uint8_t)((uint8_t)(q[j + half] + 8) << 4));
        }
    }
    if (err) *err = e;
    if (norm) *norm = nn;
}

// src/quant.rs:109-133
void quantize_matrix(Pool& pool, const uint8_t* src, size_t rows, size_t cols, const WeightFormat& f, bool clip, uint8_t* dst,
                     double* err, double* norm) {
    size_t rb_in = cols * 2, rb_out = f.row_bytes(cols);
    const size_t BLOCK = 8;
    std::mutex mu;
    double e_all = 0, n_all = 0;
    pool.run((rows + BLOCK - 1) / BLOCK, [&](size_t task) {
        size_t r0 = task * BLOCK, r1 = std::min(rows, r0 + BLOCK);
        std::vector<float> fr(cols);
        double e = 0, n = 0;
        for (size_t r = r0; r < r1; r++) {
            for (size_t c = 0; c < cols; c++) fr[c] = bf16_at(src + r * rb_in, c);
            double a, b;
            quantize_row(f, fr.data(), cols, clip, dst + r * rb_out, &a, &b);
            e += a;
            n += b;
        }
        std::lock_guard<std::mutex> g(mu);
        e_all += e;
        n_all += n;
    });
    *err += e_all;
    *norm += n_all;
}

// src/quant.rs:158-251
double quantize_model(const std::string& src_dir, const std::string& out, WeightFormat fmt, WeightFormat efmt, bool clip,
                      size_t threads) {
    if (!fmt.is_quant()) throw Err("quantize needs a quantized target format");
    if (!efmt.is_quant()) throw Err("the embedding table needs a quantized format too");
    ModelFiles files = ModelFiles::open_dir(src_dir);
    if (files.cfg.format.is_quant()) throw Err("the source model is already quantized");
    std::string cfg_text = read_text(src_dir + "/config.json");
    std::string qtext = inject_quant(cfg_text, fmt.bits, fmt.group, !(efmt == fmt), efmt.bits, efmt.group);
    Config qcfg = Config::from_json(JsonParser::parse(qtext));
    LayerLayout dst = layer_layout_for(qcfg);
    QuantHeader h;
    h.config_text = qtext;
    h.layer_bytes = dst.total;
    h.embed_bytes = qcfg.vocab * qcfg.row_bytes();
    h.norm_bytes = qcfg.hidden * 2;
    int fd = ::open(out.c_str(), O_WRONLY | O_CREAT | O_EXCL, 0644);
    if (fd < 0) throw Err(out + ": " + std::strerror(errno) + " (file exists?)");
    auto write_all = [&](const void* p, size_t n) {
        const uint8_t* b = (const uint8_t*)p;
        while (n) {
            ssize_t w = ::write(fd, b, n);
            if (w <= 0) throw Err("write failed");
            b += w;
            n -= (size_t)w;
        }
    };
    std::string hb = h.to_bytes();
    Pool pool(std::max<size_t>(threads, 1));
    double err = 0, norm = 0;
    try {
        write_all(hb.data(), hb.size());
        File src(files.path);
        std::vector<uint8_t> inb(files.layout.total), outb(dst.total);
        for (size_t l = 0; l < qcfg.layers; l++) {
            src.read_at(inb.data(), inb.size(), files.layer_start[l]);
            for (int s = 0; s < N_TENSORS; s++) {
                size_t rows, cols;
                if (!matrix_shape(s, qcfg, &rows, &cols)) {
                    if (files.layout.len[s] != dst.len[s]) throw Err("tensor changed size");
                    std::memcpy(outb.data() + dst.off[s], inb.data() + files.layout.off[s], dst.len[s]);
                } else {
                    quantize_matrix(pool, inb.data() + files.layout.off[s], rows, cols, fmt, clip, outb.data() + dst.off[s], &err, &norm);
                }
            }
            write_all(outb.data(), outb.size());
        }
        size_t rb_in = files.cfg.row_bytes(), rb_out = qcfg.row_bytes();
        size_t rows_per = std::min<size_t>(4096, qcfg.vocab);
        std::vector<uint8_t> ein(rows_per * rb_in), eout(rows_per * rb_out);
        for (size_t first = 0; first < qcfg.vocab;) {
            size_t n = std::min(rows_per, qcfg.vocab - first);
            src.read_at(ein.data(), n * rb_in, files.embed_start + first * rb_in);
            quantize_matrix(pool, ein.data(), n, qcfg.hidden, efmt, clip, eout.data(), &err, &norm);
            write_all(eout.data(), n * rb_out);
            first += n;
        }
        std::vector<uint8_t> fn(files.norm_len);
        src.read_at(fn.data(), fn.size(), files.norm_start);
        write_all(fn.data(), fn.size());
    } catch (...) {
        ::close(fd);
        throw;
    }
    ::close(fd);
    return norm > 0 ? std::sqrt(err / norm) : 0.0;
}

// ---------------------------------------------------------------------------------------------
// Model (src/model.rs:16-299), resident weights
// ---------------------------------------------------------------------------------------------

static const size_t PREFILL_CHUNK = 128;

struct Model {
    ModelFiles files;
    Config cfg;
    LayerLayout layout;
    std::vector<std::vector<uint8_t>> layers;
    std::vector<uint8_t> embed;
    std::unique_ptr<Pool> pool;
    std::vector<std::vector<float>> k_cache, v_cache;
    std::vector<float> inv_freq;
    size_t max_ctx = 0, pos = 0;

    Model(ModelFiles f, size_t threads, size_t max_ctx_) : files(std::move(f)), max_ctx(max_ctx_) {
        cfg = files.cfg;
        layout = files.layout;
        File src(files.path);
        layers.resize(cfg.layers);
        for (size_t l = 0; l < cfg.layers; l++) {
            layers[l].resize(layout.total);
            src.read_at(layers[l].data(), layout.total, files.layer_start[l]);
        }
        embed.resize(cfg.vocab * cfg.row_bytes());
        src.read_at(embed.data(), embed.size(), files.embed_start);
        pool.reset(new Pool(std::max<size_t>(threads, 1)));
        size_t kv = cfg.kv_dim();
        k_cache.assign(cfg.layers, std::vector<float>(max_ctx * kv, 0.0f));
        v_cache.assign(cfg.layers, std::vector<float>(max_ctx * kv, 0.0f));
        size_t half = cfg.head_dim / 2;
        inv_freq.resize(half);
        for (size_t i = 0; i < half; i++)
            inv_freq[i] = (float)(1.0 / std::pow((double)cfg.rope_theta, (double)(2 * i) / (double)cfg.head_dim));
    }

    const uint8_t* t(size_t l, int slot) const { return layers[l].data() + layout.off[slot]; }

    void check_request(const uint32_t* toks, size_t n) const {
        if (n == 0) throw Err("no tokens to process");
        if (pos + n > max_ctx) throw Err("context is full");
        for (size_t i = 0; i < n; i++)
            if (toks[i] >= cfg.vocab) throw Err("token id " + std::to_string(toks[i]) + " is outside the vocabulary");
    }

    // src/model.rs:224-299
    void layer_forward(size_t l, float* x, size_t T, size_t pos0) {
        size_t h = cfg.hidden, kvd = cfg.kv_dim(), hd = cfg.head_dim, inter = cfg.inter;
        size_t group = cfg.heads / cfg.kv_heads;
        std::vector<float> hb(T * h), q(T * h), k(T * kvd), v(T * kvd), attn(T * h), proj(T * h), gate(T * inter), up(T * inter);
        std::vector<float> scores(max_ctx);
        const WeightFormat& f = cfg.format;
        rms_norm_bf16(x, t(l, T_INPUT_NORM), h, T, cfg.eps, hb.data());
        matmul(*pool, f, t(l, T_Q_W), h, h, hb.data(), T, q.data());
        add_bias_bf16(q.data(), t(l, T_Q_B), h, T);
        matmul(*pool, f, t(l, T_K_W), kvd, h, hb.data(), T, k.data());
        add_bias_bf16(k.data(), t(l, T_K_B), kvd, T);
        matmul(*pool, f, t(l, T_V_W), kvd, h, hb.data(), T, v.data());
        add_bias_bf16(v.data(), t(l, T_V_B), kvd, T);
        float* kc = k_cache[l].data();
        float* vc = v_cache[l].data();
        for (size_t i = 0; i < T; i++) {
            size_t p = pos0 + i;
            for (size_t hh = 0; hh < cfg.heads; hh++) rope_inplace(&q[i * h + hh * hd], inv_freq.data(), hd, p);
            for (size_t g = 0; g < cfg.kv_heads; g++) rope_inplace(&k[i * kvd + g * hd], inv_freq.data(), hd, p);
            std::memcpy(kc + p * kvd, &k[i * kvd], kvd * 4);
            std::memcpy(vc + p * kvd, &v[i * kvd], kvd * 4);
        }
        float scale = 1.0f / std::sqrt((float)hd);
        for (size_t i = 0; i < T; i++) {
            size_t ctx = pos0 + i + 1;
            for (size_t hh = 0; hh < cfg.heads; hh++) {
                size_t g = hh / group;
                const float* qh = &q[i * h + hh * hd];
                for (size_t j = 0; j < ctx; j++) {
                    const float* kj = kc + j * kvd + g * hd;
                    float s = -0.0f;
                    for (size_t d = 0; d < hd; d++) s = s + qh[d] * kj[d];
                    scores[j] = s * scale;
                }
                softmax_inplace(scores.data(), ctx);
                float* out = &attn[i * h + hh * hd];
                for (size_t d = 0; d < hd; d++) out[d] = 0.0f;
                for (size_t j = 0; j < ctx; j++) {
                    const float* vj = vc + j * kvd + g * hd;
                    float p = scores[j];
                    for (size_t d = 0; d < hd; d++) out[d] += p * vj[d];
                }
            }
        }
        matmul(*pool, f, t(l, T_O_W), h, h, attn.data(), T, proj.data());
        for (size_t i = 0; i < T * h; i++) x[i] += proj[i];
        rms_norm_bf16(x, t(l, T_POST_NORM), h, T, cfg.eps, hb.data());
        matmul(*pool, f, t(l, T_GATE), inter, h, hb.data(), T, gate.data());
        matmul(*pool, f, t(l, T_UP), inter, h, hb.data(), T, up.data());
        for (size_t i = 0; i < T * inter; i++) gate[i] = silu(gate[i]) * up[i];
        matmul(*pool, f, t(l, T_DOWN), h, inter, gate.data(), T, proj.data());
        for (size_t i = 0; i < T * h; i++) x[i] += proj[i];
    }

    // src/model.rs:161-220; logits for the last n positions are written to out (n * vocab).
    void forward_chunk(const uint32_t* toks, size_t T, size_t n_logits, float* out) {
        size_t h = cfg.hidden;
        size_t pos0 = pos;
        std::vector<float> x(T * h);
        size_t rb = cfg.row_bytes();
        for (size_t i = 0; i < T; i++) dequant_row(cfg.embed_format, embed.data() + (size_t)toks[i] * rb, h, &x[i * h]);
        for (size_t l = 0; l < cfg.layers; l++) layer_forward(l, x.data(), T, pos0);
        if (n_logits > 0) {
            size_t n = n_logits;
            std::vector<float> hf(n * h);
            for (size_t j = 0; j < n; j++) rms_norm_f32(&x[(T - n + j) * h], files.final_norm.data(), h, cfg.eps, &hf[j * h]);
            matmul(*pool, cfg.embed_format, embed.data(), cfg.vocab, h, hf.data(), n, out);
        }
        pos += T;
    }

    // src/model.rs:111-119: logits of the last token (vocab floats)
    void forward(const uint32_t* toks, size_t n, float* logits) {
        check_request(toks, n);
        size_t nchunks = (n + PREFILL_CHUNK - 1) / PREFILL_CHUNK;
        for (size_t c = 0; c < nchunks; c++) {
            size_t a = c * PREFILL_CHUNK, b = std::min(n, a + PREFILL_CHUNK);
            bool last = c + 1 == nchunks;
            forward_chunk(toks + a, b - a, last ? 1 : 0, last ? logits : nullptr);
        }
    }

    // src/model.rs:124-133
    void forward_multi(const uint32_t* toks, size_t T, size_t n, float* logits) {
        check_request(toks, T);
        if (n == 0 || n > T) throw Err("asked for logits at " + std::to_string(n) + " positions of " + std::to_string(T) + " tokens");
        if (T > PREFILL_CHUNK) throw Err("forward_multi takes at most 128 tokens at a time");
        forward_chunk(toks, T, n, logits);
    }

    // src/model.rs:137-140
    void truncate(size_t p) {
        if (p > pos) throw Err("cannot truncate beyond the cached tokens");
        pos = p;
    }
};

// ---------------------------------------------------------------------------------------------
// Greedy speculative decoding (src/spec.rs:41-152)
// ---------------------------------------------------------------------------------------------

// src/spec.rs:41-49: the first maximum (strict >).
uint32_t argmax(const float* v, size_t n) {
    size_t best = 0;
    for (size_t i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return (uint32_t)best;
}

static const size_t MAX_DRAFT = 32;

struct SpecStats {
    uint64_t target_passes = 0, drafted = 0, accepted = 0, draft_forwards = 0;
    double target_secs = 0, draft_secs = 0, first_secs = 0, decode_secs = 0;
};

static double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Prompt-lookup drafter (an addition to the reference, restated here so that the CPU baseline runs
// the same algorithm as the CUDA path): the tokens that followed the most recent earlier
// occurrence of the longest suffix n-gram (n = 3, 2, 1) of the history.
std::vector<uint32_t> lookup_draft(const std::vector<uint32_t>& hist, size_t kk) {
    std::vector<uint32_t> out;
    if (kk == 0 || hist.size() < 2) return out;
    for (size_t n = std::min<size_t>(3, hist.size() - 1); n >= 1; n--) {
        size_t tail = hist.size() - n;
        for (size_t s = tail; s-- > 0;) {
            bool ok = true;
            for (size_t j = 0; j < n && ok; j++) ok = hist[s + j] == hist[tail + j];
            if (!ok) continue;
            for (size_t j = s + n; j < hist.size() && out.size() < kk; j++) out.push_back(hist[j]);
            return out;
        }
    }
    return out;
}

// src/spec.rs:94-149: the decode loop from a state where both models hold `hist0` and `a` is the
// target's greedy token after it. draft == nullptr selects the lookup drafter.
std::vector<uint32_t> spec_continue(Model& target, Model* draft, const uint32_t* hist0, size_t hlen, uint32_t a, size_t max_new,
                                    size_t k, const uint32_t* eos, size_t neos, SpecStats* st) {
    if (k == 0 || k > MAX_DRAFT) throw Err("k must be between 1 and 32, not " + std::to_string(k));
    if (max_new == 0) throw Err("need at least one token to generate");
    if (target.pos != hlen || (draft && draft->pos != hlen)) throw Err("the models must hold exactly the history");
    if (draft && target.cfg.vocab != draft->cfg.vocab) throw Err("the draft and the target must share a vocabulary");
    size_t need = hlen + max_new + k;
    if (need > target.max_ctx || (draft && need > draft->max_ctx)) throw Err("prompt + max_new + k exceed the context limit");
    size_t V = target.cfg.vocab;
    auto is_eos = [&](uint32_t t) {
        for (size_t i = 0; i < neos; i++)
            if (eos[i] == t) return true;
        return false;
    };
    std::vector<uint32_t> out{a};
    std::vector<uint32_t> hist(hist0, hist0 + hlen);
    hist.push_back(a);
    bool stop = is_eos(a);
    double td = now_s();
    std::vector<float> logits, dl(V);
    while (!stop && out.size() < max_new) {
        size_t kk = std::min(k, max_new - out.size() - 1);
        double ts = now_s();
        std::vector<uint32_t> drafts;
        if (draft) {
            uint32_t cur = a;
            for (size_t i = 0; i < kk; i++) {
                draft->forward(&cur, 1, dl.data());
                uint32_t d = argmax(dl.data(), V);
                st->draft_forwards++;
                drafts.push_back(d);
                cur = d;
            }
        } else {
            drafts = lookup_draft(hist, kk);
        }
        st->draft_secs += now_s() - ts;
        std::vector<uint32_t> block;
        block.push_back(a);
        block.insert(block.end(), drafts.begin(), drafts.end());
        size_t p = target.pos;
        ts = now_s();
        logits.resize(block.size() * V);
        target.forward_multi(block.data(), block.size(), block.size(), logits.data());
        st->target_secs += now_s() - ts;
        st->target_passes++;
        size_t m = 0;
        while (m < drafts.size() && argmax(&logits[m * V], V) == drafts[m]) m++;
        uint32_t next = argmax(&logits[m * V], V);
        st->drafted += drafts.size();
        st->accepted += m;
        for (size_t i = 0; i <= m; i++) {
            uint32_t tok = i < m ? drafts[i] : next;
            out.push_back(tok);
            hist.push_back(tok);
            if (is_eos(tok) || out.size() == max_new) {
                stop = true;
                break;
            }
        }
        size_t want = p + m + 1;
        target.truncate(want);
        if (draft) {
            if (draft->pos > want) {
                draft->truncate(want);
            } else if (draft->pos < want) {
                ts = now_s();
                draft->forward(&block[draft->pos - p], m + 1 - (draft->pos - p), dl.data());
                st->draft_forwards++;
                st->draft_secs += now_s() - ts;
            }
        }
        a = next;
    }
    st->decode_secs += now_s() - td;
    return out;
}

std::vector<uint32_t> speculative_greedy(Model& target, Model* draft, const uint32_t* prompt, size_t plen, size_t max_new, size_t k,
                                         const uint32_t* eos, size_t neos, SpecStats* st) {
    if (k == 0 || k > MAX_DRAFT) throw Err("k must be between 1 and 32, not " + std::to_string(k));
    if (plen == 0 || max_new == 0) throw Err("need a prompt and at least one token to generate");
    if (target.pos != 0 || (draft && draft->pos != 0)) throw Err("both models must start with an empty cache");
    if (draft && target.cfg.vocab != draft->cfg.vocab) throw Err("the draft and the target must share a vocabulary");
    size_t need = plen + max_new + k;
    if (need > target.max_ctx || (draft && need > draft->max_ctx)) throw Err("prompt + max_new + k exceed the context limit");
    double t0 = now_s();
    std::vector<float> tl(target.cfg.vocab), dl(target.cfg.vocab);
    target.forward(prompt, plen, tl.data());
    if (draft) draft->forward(prompt, plen, dl.data());
    st->first_secs = now_s() - t0;
    return spec_continue(target, draft, prompt, plen, argmax(tl.data(), target.cfg.vocab), max_new, k, eos, neos, st);
}

}  // namespace orc

// =============================================================================================
// C ABI for the Python test harness (ctypes). Every entry returns 0 on success, -1 on error; the
// message is kept per thread and read with orc_last_error.
// =============================================================================================

using namespace orc;

static thread_local std::string g_err;

template <class F>
static int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

static WeightFormat wf(int bits, size_t group) {
    WeightFormat f;
    f.bits = bits;
    f.group = group;
    return f;
}

extern "C" {

int orc_last_error(char* buf, size_t n) {
    if (n == 0) return (int)g_err.size();
    std::snprintf(buf, n, "%s", g_err.c_str());
    return (int)g_err.size();
}

float orc_bf16_round(float v) { return bf16_round(v); }

uint64_t orc_row_bytes(int bits, uint64_t group, uint64_t cols) { return wf(bits, group).row_bytes(cols); }

int orc_validate_format(int bits, uint64_t group, const uint64_t* cols, uint64_t ncols) {
    return guard([&] {
        std::vector<size_t> c(cols, cols + ncols);
        wf(bits, group).validate(c);
    });
}

int orc_quantize_row(int bits, uint64_t group, const float* row, uint64_t cols, int clip, uint8_t* out, double* err, double* norm) {
    return guard([&] { quantize_row(wf(bits, group), row, cols, clip != 0, out, err, norm); });
}

int orc_dequant_row(int bits, uint64_t group, const uint8_t* raw, uint64_t cols, float* out) {
    return guard([&] { dequant_row(wf(bits, group), raw, cols, out); });
}

float orc_dot(int bits, uint64_t group, const uint8_t* row, const float* x, uint64_t cols) {
    return dot_fmt(wf(bits, group), row, x, cols);
}

int orc_matmul(int bits, uint64_t group, const uint8_t* w, uint64_t rows, uint64_t cols, const float* x, uint64_t t, float* y,
               int threads) {
    return guard([&] {
        Pool p((size_t)std::max(threads, 1));
        matmul(p, wf(bits, group), w, rows, cols, x, t, y);
    });
}

void orc_rms_norm_bf16(const float* x, const uint8_t* w, uint64_t n, uint64_t t, float eps, float* out) {
    rms_norm_bf16(x, w, n, t, eps, out);
}
void orc_rms_norm_f32(const float* x, const float* w, uint64_t n, float eps, float* out) { rms_norm_f32(x, w, n, eps, out); }
void orc_rope(float* head, const float* inv_freq, uint64_t hd, uint64_t pos) { rope_inplace(head, inv_freq, hd, pos); }
void orc_softmax(float* v, uint64_t n) { softmax_inplace(v, n); }
float orc_silu(float x) { return silu(x); }
uint32_t orc_argmax(const float* v, uint64_t n) { return argmax(v, n); }

int orc_inject_quant(const char* cfg, int bits, uint64_t group, int has_embed, int eb, uint64_t eg, char* out, uint64_t cap,
                     uint64_t* len) {
    return guard([&] {
        std::string s = inject_quant(cfg, bits, group, has_embed != 0, eb, eg);
        *len = s.size();
        if (s.size() + 1 > cap) throw Err("buffer too small");
        std::memcpy(out, s.c_str(), s.size() + 1);
    });
}

// Parses a config text; fills [hidden, inter, layers, heads, kv_heads, head_dim, vocab, max_pos,
// bits, group, embed_bits, embed_group] and [eps, rope_theta].
int orc_config_parse(const char* text, uint64_t* ints, float* floats) {
    return guard([&] {
        Config c = Config::from_json(JsonParser::parse(text));
        uint64_t v[12] = {c.hidden, c.inter, c.layers, c.heads, c.kv_heads, c.head_dim, c.vocab, c.max_pos,
                          (uint64_t)c.format.bits, c.format.group, (uint64_t)c.embed_format.bits, c.embed_format.group};
        std::memcpy(ints, v, sizeof v);
        floats[0] = c.eps;
        floats[1] = c.rope_theta;
    });
}

int orc_quantize_model(const char* src_dir, const char* out_path, int bits, uint64_t group, int ebits, uint64_t egroup, int clip,
                       int threads, double* rel_rmse) {
    return guard([&] {
        double r = quantize_model(src_dir, out_path, wf(bits, group), wf(ebits, egroup), clip != 0, (size_t)std::max(threads, 1));
        if (rel_rmse) *rel_rmse = r;
    });
}

// Layer layout of an opened file: 12 offsets, 12 lengths, total.
int orc_open_files(const char* path, int quantized, uint64_t* layout25, uint64_t* embed_start, uint64_t* norm_start) {
    return guard([&] {
        ModelFiles m = quantized ? ModelFiles::open_quantized(path) : ModelFiles::open_dir(path);
        for (int s = 0; s < N_TENSORS; s++) {
            layout25[s] = m.layout.off[s];
            layout25[N_TENSORS + s] = m.layout.len[s];
        }
        layout25[24] = m.layout.total;
        if (embed_start) *embed_start = m.embed_start;
        if (norm_start) *norm_start = m.norm_start;
    });
}

void* orc_model_open(const char* path, int quantized, int threads, uint64_t max_ctx) {
    Model* m = nullptr;
    int rc = guard([&] {
        ModelFiles f = quantized ? ModelFiles::open_quantized(path) : ModelFiles::open_dir(path);
        m = new Model(std::move(f), (size_t)std::max(threads, 1), max_ctx);
    });
    return rc == 0 ? m : nullptr;
}

void orc_model_free(void* m) { delete (Model*)m; }

uint64_t orc_model_pos(void* m) { return ((Model*)m)->pos; }
uint64_t orc_model_vocab(void* m) { return ((Model*)m)->cfg.vocab; }
uint64_t orc_model_hidden(void* m) { return ((Model*)m)->cfg.hidden; }
void orc_model_reset(void* m) { ((Model*)m)->pos = 0; }

int orc_model_truncate(void* m, uint64_t pos) {
    return guard([&] { ((Model*)m)->truncate(pos); });
}

int orc_forward(void* m, const uint32_t* toks, uint64_t n, float* logits) {
    return guard([&] { ((Model*)m)->forward(toks, n, logits); });
}

int orc_forward_multi(void* m, const uint32_t* toks, uint64_t t, uint64_t n, float* logits) {
    return guard([&] { ((Model*)m)->forward_multi(toks, t, n, logits); });
}

// Hidden state after the layers (before the final norm) for t tokens, for layer-level checks.
int orc_forward_hidden(void* m, const uint32_t* toks, uint64_t t, uint64_t n_layers, float* x_out) {
    return guard([&] {
        Model* M = (Model*)m;
        M->check_request(toks, t);
        size_t h = M->cfg.hidden, rb = M->cfg.row_bytes();
        std::vector<float> x(t * h);
        for (size_t i = 0; i < t; i++) dequant_row(M->cfg.embed_format, M->embed.data() + (size_t)toks[i] * rb, h, &x[i * h]);
        size_t L = std::min<size_t>(n_layers, M->cfg.layers);
        for (size_t l = 0; l < L; l++) M->layer_forward(l, x.data(), t, M->pos);
        std::memcpy(x_out, x.data(), x.size() * 4);
        M->pos += t;
    });
}

// stats: [target_passes, drafted, accepted, draft_forwards]; times: [target, draft, first, decode]
int orc_speculative_greedy(void* target, void* draft, const uint32_t* prompt, uint64_t plen, uint64_t max_new, uint64_t k,
                           const uint32_t* eos, uint64_t neos, uint32_t* out, uint64_t* out_len, uint64_t* stats, double* times) {
    return guard([&] {
        SpecStats st;
        auto toks = speculative_greedy(*(Model*)target, (Model*)draft, prompt, plen, max_new, k, eos, neos, &st);
        std::memcpy(out, toks.data(), toks.size() * 4);
        *out_len = toks.size();
        uint64_t s[4] = {st.target_passes, st.drafted, st.accepted, st.draft_forwards};
        std::memcpy(stats, s, sizeof s);
        double t[4] = {st.target_secs, st.draft_secs, st.first_secs, st.decode_secs};
        std::memcpy(times, t, sizeof t);
    });
}

int orc_spec_continue(void* target, void* draft, const uint32_t* hist, uint64_t hlen, uint32_t first, uint64_t max_new, uint64_t k,
                      const uint32_t* eos, uint64_t neos, uint32_t* out, uint64_t* out_len, uint64_t* stats, double* times) {
    return guard([&] {
        SpecStats st;
        auto toks = spec_continue(*(Model*)target, (Model*)draft, hist, hlen, first, max_new, k, eos, neos, &st);
        std::memcpy(out, toks.data(), toks.size() * 4);
        *out_len = toks.size();
        uint64_t s4[4] = {st.target_passes, st.drafted, st.accepted, st.draft_forwards};
        std::memcpy(stats, s4, sizeof s4);
        double t[4] = {st.target_secs, st.draft_secs, st.first_secs, st.decode_secs};
        std::memcpy(times, t, sizeof t);
    });
}

// Greedy token after a forward of n tokens (prefill helper for the CPU baseline).
int orc_forward_argmax(void* m, const uint32_t* toks, uint64_t n, uint32_t* tok) {
    return guard([&] {
        Model* M = (Model*)m;
        std::vector<float> l(M->cfg.vocab);
        M->forward(toks, n, l.data());
        *tok = argmax(l.data(), M->cfg.vocab);
    });
}

}  // extern "C"
