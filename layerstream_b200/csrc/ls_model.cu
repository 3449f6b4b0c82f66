// Host runtime of the verify path: model loading (resident or streamed layer slots), the per-pass
// kernel sequence (captured once per shape in a CUDA graph), the greedy speculative loop and the
// C ABI declared in include/layerstream.h.
//
// Reference counterparts: model::Model (src/model.rs:16-220), provider::{ResidentProvider,
// StreamProvider} (src/provider.rs:61-337), spec::speculative_greedy (src/spec.rs:57-152),
// quant::quantize_model (src/quant.rs:158-251).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <tuple>

#include "layerstream.h"
#include "ls_internal.h"

using namespace ls;

namespace {

constexpr int kPrefillChunk = 128;  // src/model.rs:14
constexpr size_t kPrefillSeqs = 16;  // sequences of a batch prefilled by one pass (<= 2048 rows)
constexpr int kHeadRows = 4096;     // src/provider.rs:21
constexpr int kMaxDraft = 32;       // src/spec.rs:52
constexpr int kMaxT = kPrefillChunk;

thread_local std::string g_err;

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// Page size of the K/V cache: LS_KV_PAGE positions (a power of two, 8 .. 65536), else 64.
int kv_page_shift() {
  int page = 64;
  if (const char* e = getenv("LS_KV_PAGE")) page = atoi(e);
  int sh = 0;
  while ((1 << sh) < page && sh < 16) sh++;
  if ((1 << sh) != page || sh < 3) LS_THROW(LS_ERR_ARG, "LS_KV_PAGE must be a power of two in 8..65536");
  return sh;
}

// Pages of a paged K/V cache (the same page ids index every layer's pool): a LIFO free list, each
// sequence's table of pool pages (a pinned host mirror and the device copy the kernels read), and
// the number of logical pages each sequence holds. A sequence takes pages as it grows (ensure) and
// returns those past its length when it is rolled back (shrink): a rollback is a length, and the
// freed pages serve the next growth of any sequence. Table uploads are stream-ordered before the
// pass that reads them; the host changes the mirror only between passes it has synchronized.
struct PagePool {
  int shift = 6, nseq = 0, max_pages = 0, num_pages = 0;
  std::vector<int32_t> free_list;
  std::vector<int> held;       // logical pages per sequence
  int32_t* h_table = nullptr;  // [nseq][max_pages], pinned
  int32_t* d_table = nullptr;
  uint64_t* h2d = nullptr;     // bytes counter to charge uploads to

  int page() const { return 1 << shift; }
  void init(int seqs, size_t max_ctx, int32_t* host_table, int32_t* dev_table) {
    nseq = seqs;
    max_pages = (int)((max_ctx + page() - 1) >> shift);
    num_pages = nseq * max_pages;
    h_table = host_table;
    d_table = dev_table;
    held.assign(nseq, 0);
    free_list.clear();
    for (int p = num_pages - 1; p >= 0; p--) free_list.push_back(p);  // page 0 handed out first
  }
  // Sequence s holds the pages of positions [0, n).
  void ensure(int s, size_t n, cudaStream_t st) {
    const int need = (int)((n + page() - 1) >> shift);
    if (need <= held[s]) return;
    if (need > max_pages || (int)free_list.size() < need - held[s]) LS_THROW(LS_ERR_ARG, "the K/V page pool is exhausted");
    const int first = held[s];
    for (int i = first; i < need; i++) {
      h_table[(size_t)s * max_pages + i] = free_list.back();
      free_list.pop_back();
    }
    held[s] = need;
    const size_t off = (size_t)s * max_pages + first, bytes = (size_t)(need - first) * 4;
    LS_CUDA(cudaMemcpyAsync(d_table + off, h_table + off, bytes, cudaMemcpyHostToDevice, st));
    if (h2d) *h2d += bytes;
  }
  // Sequence s keeps only the pages of positions [0, n).
  void shrink(int s, size_t n) {
    const int keep = (int)((n + page() - 1) >> shift);
    while (held[s] > keep) free_list.push_back(h_table[(size_t)s * max_pages + --held[s]]);
  }
  int used() const { return num_pages - (int)free_list.size(); }
};

// RoPE (cos, sin) table [n_pos][hd/2] with the float steps of src/model.rs:62-65 and
// src/kernels.rs:242-252: inv_freq in f64 then f32, angle = pos as f32 * inv_freq, libm cosf/sinf.
std::vector<float2> rope_table(float theta, size_t hd, size_t n_pos) {
  const size_t half = hd / 2;
  std::vector<float> inv(half);
  for (size_t i = 0; i < half; i++) inv[i] = (float)(1.0 / std::pow((double)theta, (double)(2 * i) / (double)hd));
  std::vector<float2> tab(n_pos * half);
  for (size_t p = 0; p < n_pos; p++)
    for (size_t i = 0; i < half; i++) {
      const float ang = (float)p * inv[i];
      tab[p * half + i] = make_float2(cosf(ang), sinf(ang));
    }
  return tab;
}

// Device planes of one quantized matrix carved out of a larger allocation.
QMat carve(uint8_t*& p, int rows, int cols, const WeightFormat& f) {
  QMat m;
  m.rows = rows;
  m.rows_pad = pad32(rows);
  m.cols = cols;
  m.bits = f.bits;
  m.group = f.group;
  m.data = p;
  p += align256(m.data_bytes());
  m.scales = reinterpret_cast<uint16_t*>(p);
  p += align256(m.scale_bytes());
  return m;
}

size_t qmat_bytes(int rows, int cols, const WeightFormat& f) {
  QMat m;
  m.rows = rows;
  m.rows_pad = pad32(rows);
  m.cols = cols;
  m.bits = f.bits;
  m.group = f.group;
  return align256(m.data_bytes()) + align256(m.scale_bytes());
}

struct LayerW {
  QMat qkv, o, gu, down;
  uint16_t* in_norm = nullptr;
  uint16_t* post_norm = nullptr;
  uint16_t* qkv_bias = nullptr;  // q_b | k_b | v_b
};

// GEMV path: tensor cores (tcgen05) wherever the format allows, unless LS_GEMV=fma asks for the
// CUDA-core kernel (kept as a cross-check).
bool use_tc(const QMat& w) {
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("LS_GEMV");
    forced = (e && std::string(e) == "fma") ? 1 : 0;
  }
  return forced == 0 && gemv_tc_supported(w);
}

// Tensor-core GEMV: K-split and grid. Aim for ~4 CTAs per SM over (tiles x slices x token groups),
// keep at least two 64-wide K blocks per slice, never fewer slices than shared memory needs.
// The argmax epilogue needs whole dot products (no K split): it narrows the token groups instead
// until one K slice of staged activations fits (max_nt, when given, receives the width).
void choose_tc(const QMat& w, int M, int num_sms, bool argmax, int* ksplit, int* grid_x, int* max_nt = nullptr) {
  int cap = 64;
  if (argmax) {
    while (cap > 16 && gemv_tc_min_ksplit(w, M, cap) > 1) cap -= 16;
    if (gemv_tc_min_ksplit(w, M, cap) > 1) LS_THROW(LS_ERR_ARG, "matrix too wide for the LM-head GEMV");
  }
  if (max_nt) *max_nt = cap;
  const int NT = gemv_tc_nt(M, cap);
  const int tiles128 = (w.rows_pad / 32 + 3) / 4;
  const int nz = (M + NT - 1) / NT;
  const int kb = (w.bits == 4 && w.group > 64) ? w.group : 64;
  const int nblk = w.cols / kb;
  const int target = 4 * num_sms;
  int ks = 1;
  if (!argmax) {
    ks = (target + tiles128 * nz - 1) / (tiles128 * nz);
    ks = std::min(ks, std::max(1, nblk / 2));
    ks = std::min(ks, 32);
  }
  ks = std::max(ks, gemv_tc_min_ksplit(w, M, cap));
  ks = std::min(ks, nblk);
  *ksplit = ks;
  *grid_x = std::max(1, std::min(tiles128, (target + ks * nz - 1) / (ks * nz)));
}

// K-split of a GEMV launch: aim for ~8 warp-tiles per SM, keep at least 8 chunks (one unrolled
// round of loads) per slice, and never less than the staged activations need.
int choose_ksplit(const QMat& w, int M, int num_sms) {
  const int tiles = w.rows_pad / 32, nz = (M + 15) / 16;
  const int U = (w.bits == 4 && w.group >= 32) ? w.group / 32 : 1;
  const int units = w.chunks() / U;
  const int by_work = std::max(1, w.chunks() / 8 / U);
  const int want = std::max(1, (8 * num_sms + tiles * nz - 1) / (tiles * nz));
  return std::max(gemv_min_ksplit(w, M), std::min({want, by_work, units, 32}));
}

void check_gpu_format(const Config& c) {
  if (c.format.quant() != c.embed_format.quant())
    LS_THROW(LS_ERR_ARG, "the CUDA path takes bf16 layers only with a bf16 embedding table");
  for (const WeightFormat* f : {&c.format, &c.embed_format}) {
    if (f->quant() && (f->group & (f->group - 1)))
      LS_THROW(LS_ERR_ARG, "the CUDA path needs a power-of-two group size, not " + std::to_string(f->group));
  }
  if (!c.format.quant() && (c.hidden % 64 || c.inter % 64))
    LS_THROW(LS_ERR_ARG, "bf16 weights need hidden and intermediate sizes that are multiples of 64");
  if (c.head_dim != 16 && c.head_dim != 32 && c.head_dim != 64 && c.head_dim != 128)
    LS_THROW(LS_ERR_ARG, "head dimension " + std::to_string(c.head_dim) + " is not supported by the CUDA path");
  if (c.inter % 16) LS_THROW(LS_ERR_ARG, "intermediate size must be a multiple of 16");
}

}  // namespace

struct LsModel {
  int device = 0;
  LsqFile file;                   // the model's offsets (a .lsq file, or a bf16 safetensors model)
  std::vector<uint64_t> layer_off;  // file offset of each layer's block
  Config cfg;
  int mode = LS_MODE_RESIDENT, slots = 1;
  size_t max_ctx = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr, copy_stream = nullptr;
  std::vector<void*> dev_allocs;
  std::vector<void*> host_allocs;

  std::vector<LayerW> layers;  // resident: one per layer; stream: one per slot
  QMat embed;                  // resident: the whole tiled table (also the LM head)
  std::vector<QMat> head_slot; // stream: head chunk planes per slot
  float* final_norm = nullptr;

  // streaming
  uint8_t* host_model = nullptr;      // pinned copy of the file's data (layers, embedding, norm)
  const uint8_t* host_embed_dev = nullptr;  // device-visible pointer to the embedding in host_model
  std::vector<uint8_t*> raw_slot;
  std::vector<cudaEvent_t> ev_loaded, ev_free;
  size_t raw_slot_bytes = 0;

  // sealed files (src/seal.rs): the ciphertext is copied to the device and opened there (tags
  // checked, then decrypted) before it is repacked; a failed tag leaves *d_bad = chunk + 1
  bool sealed = false;
  SealedFile sfile;
  uint32_t* d_key = nullptr;         // the 32-byte key
  uint8_t* d_aad = nullptr;          // frame + header, the associated data's shared prefix
  AeadChunk* d_layer_desc = nullptr; // stream mode: the messages of layer l in raw slot s, [l][s][chunk]
  AeadChunk* d_desc_stage[2] = {nullptr, nullptr};  // resident load / one-off opens: per staging buffer
  AeadChunk* h_desc_stage[2] = {nullptr, nullptr};
  size_t desc_stage_cap = 0;
  void* aead_scr = nullptr;
  size_t aead_scr_bytes = 0;
  int* d_bad = nullptr;

  // cache, tables and activations
  uint16_t *kc = nullptr, *vc = nullptr;  // page pools of every layer, kv_layer elements apart
  size_t kv_layer = 0;
  PagePool pool;
  float2* rope = nullptr;
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *hbuf = nullptr, *logits = nullptr;
  ArgPart* arg_parts = nullptr;
  unsigned *tickets = nullptr, *arg_ticket = nullptr, *att_tickets = nullptr;
  float *partial = nullptr, *att_part = nullptr;
  size_t partial_floats = 0, att_part_floats = 0;
  int att_slots = 1;
  // passes through separate kernels (prefill chunks, stream mode) run the projections as batched
  // tensor-core GEMMs over all the pass's rows: f16 operands in the bt layout, split-K scratch
  bool use_bg = false;
  uint16_t *bt_a = nullptr, *bt_h = nullptr;
  float* bg_partial = nullptr;
  unsigned* bg_tickets = nullptr;
  Ctl* ctl = nullptr;
  Ctl* ctl_host = nullptr;

  // persistent pass kernel state (resident mode, passes of <= 48 tokens)
  PassLayer* d_pass_layers = nullptr;
  QMaps* d_pass_maps = nullptr;
  long long *x_fix = nullptr, *qkv_fix = nullptr, *gu_fix = nullptr;
  float* pk_att = nullptr;
  unsigned* pk_bar = nullptr;
  ArgPart* pk_parts = nullptr;
  int pk_max_grid = 0;
  cudaEvent_t pk_ev[2] = {nullptr, nullptr};

  std::map<std::tuple<int, int, int, int>, cudaGraphExec_t> graphs;
  size_t pos = 0;
  uint64_t bytes_read = 0, wait_ns = 0, passes = 0, resident_weight_bytes = 0, h2d_bytes = 0, d2h_bytes = 0;

  // live profile: event pairs around the launches of one sampled layer, the head and the pass
  bool prof_on = false;
  bool prof_timeline = false;  // barrier timestamps of the persistent pass kernel
  std::vector<cudaEvent_t> prof_ev;
  struct ProfRec { int cls; double bytes; };
  std::vector<ProfRec> prof_rec;  // filled at enqueue (capture) time, one per event pair
  std::map<std::tuple<int, int, int, int>, std::vector<ProfRec>> prof_recs;  // per graph
  const std::vector<ProfRec>* prof_cur = nullptr;
  bool prof_pending = false;
  LsProfile prof{};
  int prof_layer() const { return (int)cfg.layers / 2; }

  ~LsModel() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    for (auto e : prof_ev) cudaEventDestroy(e);
    for (auto e : pk_ev)
      if (e) cudaEventDestroy(e);
    for (auto e : ev_loaded) cudaEventDestroy(e);
    for (auto e : ev_free) cudaEventDestroy(e);
    for (void* p : dev_allocs) cudaFree(p);
    for (void* p : host_allocs) cudaFreeHost(p);
    if (stream) cudaStreamDestroy(stream);
    if (copy_stream) cudaStreamDestroy(copy_stream);
  }

  template <class T>
  T* dalloc(size_t n) {
    void* p = nullptr;
    LS_CUDA(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)));
    dev_allocs.push_back(p);
    LS_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(n * sizeof(T), 16), stream));
    return reinterpret_cast<T*>(p);
  }
  template <class T>
  T* halloc(size_t n, unsigned flags = cudaHostAllocDefault) {
    void* p = nullptr;
    LS_CUDA(cudaHostAlloc(&p, std::max<size_t>(n * sizeof(T), 16), flags));
    host_allocs.push_back(p);
    return reinterpret_cast<T*>(p);
  }

  size_t layer_plane_bytes() const {
    const size_t h = cfg.hidden, kv = cfg.kv_dim(), I = cfg.inter;
    return qmat_bytes((int)(h + 2 * kv), (int)h, cfg.format) + qmat_bytes((int)h, (int)h, cfg.format) +
           qmat_bytes((int)(2 * I), (int)h, cfg.format) + qmat_bytes((int)h, (int)I, cfg.format) + align256(h * 2) * 2 +
           align256((h + 2 * kv) * 2);
  }

  LayerW carve_layer(uint8_t*& p) {
    const int h = (int)cfg.hidden, kv = (int)cfg.kv_dim(), I = (int)cfg.inter;
    LayerW w;
    w.qkv = carve(p, h + 2 * kv, h, cfg.format);
    w.o = carve(p, h, h, cfg.format);
    w.gu = carve(p, 2 * I, h, cfg.format);
    w.down = carve(p, h, I, cfg.format);
    w.in_norm = reinterpret_cast<uint16_t*>(p);
    p += align256((size_t)h * 2);
    w.post_norm = reinterpret_cast<uint16_t*>(p);
    p += align256((size_t)h * 2);
    w.qkv_bias = reinterpret_cast<uint16_t*>(p);
    p += align256((size_t)(h + 2 * kv) * 2);
    return w;
  }

  // Raw layer block on the device (file layout) -> tiled planes of `w`.
  void repack_layer(const uint8_t* raw, LayerW& w, cudaStream_t s) {
    const LayerLayout& L = file.layout;
    const int h = (int)cfg.hidden, kv = (int)cfg.kv_dim(), I = (int)cfg.inter;
    RepackSrc q;
    q.nseg = 3;
    q.seg[0] = raw + L.off[T_Q_W];
    q.seg_rows[0] = h;
    q.seg[1] = raw + L.off[T_K_W];
    q.seg_rows[1] = kv;
    q.seg[2] = raw + L.off[T_V_W];
    q.seg_rows[2] = kv;
    launch_repack(q, w.qkv.bits, w.qkv.group, h, const_cast<uint8_t*>(w.qkv.data), const_cast<uint16_t*>(w.qkv.scales),
                  w.qkv.rows_pad, s);
    RepackSrc o;
    o.seg[0] = raw + L.off[T_O_W];
    o.seg_rows[0] = h;
    launch_repack(o, w.o.bits, w.o.group, h, const_cast<uint8_t*>(w.o.data), const_cast<uint16_t*>(w.o.scales), w.o.rows_pad, s);
    RepackSrc gu;
    gu.nseg = 2;
    gu.interleave16 = 1;
    gu.seg[0] = raw + L.off[T_GATE];
    gu.seg_rows[0] = I;
    gu.seg[1] = raw + L.off[T_UP];
    gu.seg_rows[1] = I;
    launch_repack(gu, w.gu.bits, w.gu.group, h, const_cast<uint8_t*>(w.gu.data), const_cast<uint16_t*>(w.gu.scales),
                  w.gu.rows_pad, s);
    RepackSrc d;
    d.seg[0] = raw + L.off[T_DOWN];
    d.seg_rows[0] = h;
    launch_repack(d, w.down.bits, w.down.group, I, const_cast<uint8_t*>(w.down.data), const_cast<uint16_t*>(w.down.scales),
                  w.down.rows_pad, s);
    LS_CUDA(cudaMemcpyAsync(w.in_norm, raw + L.off[T_INPUT_NORM], (size_t)h * 2, cudaMemcpyDeviceToDevice, s));
    LS_CUDA(cudaMemcpyAsync(w.post_norm, raw + L.off[T_POST_NORM], (size_t)h * 2, cudaMemcpyDeviceToDevice, s));
    LS_CUDA(cudaMemcpyAsync(w.qkv_bias, raw + L.off[T_Q_B], (size_t)h * 2, cudaMemcpyDeviceToDevice, s));
    LS_CUDA(cudaMemcpyAsync(w.qkv_bias + h, raw + L.off[T_K_B], (size_t)kv * 2, cudaMemcpyDeviceToDevice, s));
    LS_CUDA(cudaMemcpyAsync(w.qkv_bias + h + kv, raw + L.off[T_V_B], (size_t)kv * 2, cudaMemcpyDeviceToDevice, s));
  }

  void repack_embed_rows(const uint8_t* raw_rows, int first, int rows, QMat& dst, cudaStream_t s) {
    // dst holds the whole table (resident) or one chunk (stream, first == 0)
    const int nch = dst.chunks(), ng = dst.groups();
    RepackSrc e;
    e.seg[0] = raw_rows;
    e.seg_rows[0] = rows;
    uint8_t* d = const_cast<uint8_t*>(dst.data) + (size_t)(first / 32) * nch * 512;
    uint16_t* sc = const_cast<uint16_t*>(dst.scales) + (size_t)(first / 32) * ng * 32;
    launch_repack(e, dst.bits, dst.group, dst.cols, d, sc, pad32(rows), s);
  }

  // The AEAD message of sealed chunk idx over len device bytes at data (src/seal.rs:341-350).
  AeadChunk sealed_chunk(size_t idx, uint8_t* data, uint64_t len) const {
    AeadChunk c{};
    c.data = data;
    c.len = len;
    std::memcpy(c.nonce, sfile.nonce_prefix, 8);
    c.nonce[2] = (uint32_t)idx;
    c.tail = (uint32_t)idx;
    c.tail_len = 4;
    std::memcpy(c.tag, &sfile.tags[16 * idx], 16);
    return c;
  }
  // Opens, on stream s, the sealed chunks first_chunk.. that make up the n plaintext bytes copied to
  // data (chunks of clen bytes, the last one shorter), through staging descriptor set k (the caller
  // has waited for the last step that used set k).
  void open_range(int k, size_t first_chunk, uint8_t* data, uint64_t n, uint64_t clen, cudaStream_t s) {
    const size_t nch = (size_t)((n + clen - 1) / clen);
    if (nch > desc_stage_cap) LS_THROW(-1, "sealed open: too many chunks in one step");
    for (size_t i = 0; i < nch; i++)
      h_desc_stage[k][i] = sealed_chunk(first_chunk + i, data + i * clen, std::min<uint64_t>(clen, n - i * clen));
    LS_CUDA(cudaMemcpyAsync(d_desc_stage[k], h_desc_stage[k], nch * sizeof(AeadChunk), cudaMemcpyHostToDevice, s));
    launch_aead(d_desc_stage[k], (int)nch, clen, d_aad, (uint32_t)sfile.aad_prefix.size(), d_key, false, aead_scr, aead_scr_bytes,
                d_bad, s);
  }
  // Throws when a sealed chunk failed its tag (a wrong key, or a modified file).
  void sealed_check() const {
    if (!sealed) return;
    int b = 0;
    LS_CUDA(cudaMemcpy(&b, d_bad, 4, cudaMemcpyDeviceToHost));
    if (b != 0x7fffffff)
      LS_THROW(LS_ERR_IO, "authentication failed for chunk " + std::to_string(b - 1) + ": wrong key, or the file was modified");
  }
  // Device state of a sealed model: key, associated data, descriptor staging, scratch, error word.
  void setup_sealed(const uint8_t* key, size_t embed_step_rows) {
    d_key = dalloc<uint32_t>(8);
    LS_CUDA(cudaMemcpy(d_key, key, 32, cudaMemcpyHostToDevice));
    d_aad = dalloc<uint8_t>(sfile.aad_prefix.size());
    LS_CUDA(cudaMemcpy(d_aad, sfile.aad_prefix.data(), sfile.aad_prefix.size(), cudaMemcpyHostToDevice));
    const size_t rb = cfg.embed_row_bytes(), ecr = sfile.embed_chunk_rows;
    desc_stage_cap = std::max<size_t>({sfile.layer_chunks(), (embed_step_rows + ecr - 1) / ecr, 1});
    for (int k = 0; k < 2; k++) {
      d_desc_stage[k] = dalloc<AeadChunk>(desc_stage_cap);
      h_desc_stage[k] = halloc<AeadChunk>(desc_stage_cap);
    }
    const uint32_t al = (uint32_t)sfile.aad_prefix.size();
    aead_scr_bytes = std::max({aead_scratch_bytes((int)sfile.layer_chunks() * std::max(1, slots), sfile.layer_chunk, al),
                               aead_scratch_bytes((int)desc_stage_cap, ecr * rb, al),
                               aead_scratch_bytes(1, sfile.final_norm_bytes, al)});
    aead_scr = dalloc<uint8_t>(aead_scr_bytes);
    d_bad = dalloc<int>(1);
    const int big = 0x7fffffff;
    LS_CUDA(cudaMemcpy(d_bad, &big, 4, cudaMemcpyHostToDevice));
  }

  void open(const char* path, int dev, uint64_t mctx, int md, int nslots, const uint8_t* key = nullptr) {
    struct stat stt;
    const bool dir = ::stat(path, &stt) == 0 && S_ISDIR(stt.st_mode);
    std::string data_path = path;
    if (dir) {
      // an unquantized (bf16) safetensors model directory, read as the reference's
      // ModelFiles::open does (src/weights.rs:271-324): each layer's tensors one contiguous block
      const SafetensorsModel st = SafetensorsModel::open(path);
      file = LsqFile();
      file.path = st.file;
      file.config_text = st.config_text;
      file.cfg = st.cfg;
      file.layout = st.layout;
      file.data_start = st.layer_start[0];
      file.embed_start = st.embed_start;
      file.norm_start = st.norm_start;
      layer_off = st.layer_start;
      data_path = st.file;
      if (md != LS_MODE_RESIDENT) LS_THROW(LS_ERR_ARG, "streaming reads quantized (.lsq) files; open a bf16 model resident");
    } else if (is_sealed_file(path)) {
      // a sealed file (src/seal.rs:860-903): the plaintext's layers, table and norm lie at ct_base
      if (!key) LS_THROW(LS_ERR_ARG, "a sealed model needs its key (ls_model_open_sealed)");
      sfile = SealedFile::open(path);
      sealed = true;
      file = LsqFile();
      file.path = path;
      file.config_text = sfile.config_text;
      file.cfg = sfile.cfg;
      file.layout = sfile.layout;
      file.data_start = sfile.ct_base;
      file.embed_start = sfile.ct_base + sfile.embed_plain_off();
      file.norm_start = file.embed_start + sfile.embed_bytes();
      file.embed_bytes = sfile.embed_bytes();
      file.norm_bytes = sfile.final_norm_bytes;
      for (size_t l = 0; l < file.cfg.layers; l++) layer_off.push_back(sfile.ct_base + l * file.layout.total);
      if (!file.cfg.format.quant() && md != LS_MODE_RESIDENT)
        LS_THROW(LS_ERR_ARG, "streaming reads quantized weights; open a sealed bf16 model resident");
    } else {
      if (key) LS_THROW(LS_ERR_ARG, "a key was given for a file that is not sealed");
      file = LsqFile::open(path);
      for (size_t l = 0; l < file.cfg.layers; l++) layer_off.push_back(file.data_start + l * file.layout.total);
    }
    cfg = file.cfg;
    check_gpu_format(cfg);
    device = dev;
    LS_CUDA(cudaSetDevice(device));
    if (mctx == 0) LS_THROW(LS_ERR_ARG, "max_ctx must be positive");
    max_ctx = mctx;
    mode = md;
    if (mode != LS_MODE_RESIDENT && mode != LS_MODE_STREAM) LS_THROW(LS_ERR_ARG, "mode must be resident or stream");
    slots = std::max(1, nslots);
    LS_CUDA(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device));
    LS_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    LS_CUDA(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking));

    const size_t h = cfg.hidden, kv = cfg.kv_dim(), I = cfg.inter, V = cfg.vocab, L = cfg.layers;
    const size_t lt = file.layout.total, rb = cfg.embed_row_bytes();
    int fd = ::open(data_path.c_str(), O_RDONLY);
    if (fd < 0) LS_THROW(LS_ERR_IO, data_path + ": cannot open");
    struct FdGuard {
      int fd;
      ~FdGuard() { ::close(fd); }
    } guard{fd};

    // sealed: embedding rows are opened in whole chunks, so a load step takes a multiple of them
    size_t embed_step = std::min<size_t>(kHeadRows, V);
    if (sealed) {
      const size_t ecr = sfile.embed_chunk_rows;
      embed_step = std::min(V, ecr >= kHeadRows ? ecr : kHeadRows / ecr * ecr);
      setup_sealed(key, embed_step);
    }

    // final norm (src/weights.rs:408-411): bf16 -> f32, resident in both modes
    std::vector<uint16_t> nb(h);
    pread_all(fd, nb.data(), h * 2, file.norm_start);
    if (sealed) {  // opening the norm's chunk checks the key up front (src/seal.rs:894-902)
      uint8_t* dn = dalloc<uint8_t>(h * 2);
      LS_CUDA(cudaMemcpyAsync(dn, nb.data(), h * 2, cudaMemcpyHostToDevice, stream));
      open_range(0, sfile.final_chunk(), dn, h * 2, h * 2, stream);
      LS_CUDA(cudaMemcpyAsync(nb.data(), dn, h * 2, cudaMemcpyDeviceToHost, stream));
      LS_CUDA(cudaStreamSynchronize(stream));
      sealed_check();
    }
    std::vector<float> nf(h);
    for (size_t i = 0; i < h; i++) {
      uint32_t u = (uint32_t)nb[i] << 16;
      std::memcpy(&nf[i], &u, 4);
    }
    final_norm = dalloc<float>(h);
    LS_CUDA(cudaMemcpyAsync(final_norm, nf.data(), h * 4, cudaMemcpyHostToDevice, stream));
    LS_CUDA(cudaStreamSynchronize(stream));

    if (mode == LS_MODE_RESIDENT) {
      const size_t per = layer_plane_bytes();
      uint8_t* base = dalloc<uint8_t>(per * L + qmat_bytes((int)V, (int)h, cfg.embed_format));
      resident_weight_bytes = per * L + qmat_bytes((int)V, (int)h, cfg.embed_format);
      uint8_t* p = base;
      for (size_t l = 0; l < L; l++) layers.push_back(carve_layer(p));
      embed = carve(p, (int)V, (int)h, cfg.embed_format);
      // load through two pinned staging buffers and one device raw buffer
      const size_t chunk_rows = embed_step;
      const size_t stage = std::max(lt, chunk_rows * rb);
      uint8_t* hst[2] = {halloc<uint8_t>(stage), halloc<uint8_t>(stage)};
      uint8_t* raw[2] = {dalloc<uint8_t>(stage), dalloc<uint8_t>(stage)};
      cudaEvent_t done[2];
      LS_CUDA(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming));
      LS_CUDA(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming));
      bool used[2] = {false, false};
      int k = 0;
      auto step = [&](uint64_t off, size_t n, const std::function<void(const uint8_t*)>& after) {
        if (used[k]) LS_CUDA(cudaEventSynchronize(done[k]));
        pread_all(fd, hst[k], n, off);
        LS_CUDA(cudaMemcpyAsync(raw[k], hst[k], n, cudaMemcpyHostToDevice, stream));
        after(raw[k]);
        LS_CUDA(cudaEventRecord(done[k], stream));
        used[k] = true;
        k ^= 1;
      };
      for (size_t l = 0; l < L; l++)
        step(layer_off[l], lt, [&](const uint8_t* r) {
          if (sealed) open_range(k, l * sfile.layer_chunks(), const_cast<uint8_t*>(r), lt, sfile.layer_chunk, stream);
          repack_layer(r, layers[l], stream);
        });
      for (size_t first = 0; first < V; first += chunk_rows) {
        const size_t rows = std::min(chunk_rows, V - first);
        step(file.embed_start + first * rb, rows * rb, [&](const uint8_t* r) {
          if (sealed)
            open_range(k, sfile.embed_first_chunk() + first / sfile.embed_chunk_rows, const_cast<uint8_t*>(r), rows * rb,
                       sfile.embed_chunk_rows * rb, stream);
          repack_embed_rows(r, (int)first, (int)rows, embed, stream);
        });
      }
      LS_CUDA(cudaStreamSynchronize(stream));
      sealed_check();
      cudaEventDestroy(done[0]);
      cudaEventDestroy(done[1]);
    } else {
      // pinned, device-mapped host copy of the whole model; HBM holds `slots` layer-sized slots
      const size_t data_bytes = (size_t)(file.norm_start - file.data_start);
      host_model = halloc<uint8_t>(data_bytes, cudaHostAllocMapped);
      const size_t step_bytes = 64ull << 20;
      for (size_t off = 0; off < data_bytes; off += step_bytes)
        pread_all(fd, host_model + off, std::min(step_bytes, data_bytes - off), file.data_start + off);
      void* dp = nullptr;
      LS_CUDA(cudaHostGetDevicePointer(&dp, host_model + (file.embed_start - file.data_start), 0));
      host_embed_dev = reinterpret_cast<const uint8_t*>(dp);
      const size_t chunk_rows = std::min<size_t>(kHeadRows, V);
      raw_slot_bytes = std::max({lt, chunk_rows * rb, sealed ? embed_step * rb : (size_t)0});
      // a slot holds either a layer or a head chunk, so their planes share one region
      const size_t per = std::max(layer_plane_bytes(), qmat_bytes((int)chunk_rows, (int)h, cfg.embed_format));
      for (int s = 0; s < slots; s++) {
        raw_slot.push_back(dalloc<uint8_t>(raw_slot_bytes));
        uint8_t* p = dalloc<uint8_t>(per);
        uint8_t* hp = p;
        layers.push_back(carve_layer(p));
        head_slot.push_back(carve(hp, (int)chunk_rows, (int)h, cfg.embed_format));
        cudaEvent_t a, b;
        LS_CUDA(cudaEventCreateWithFlags(&a, cudaEventDisableTiming));
        LS_CUDA(cudaEventCreateWithFlags(&b, cudaEventDisableTiming));
        ev_loaded.push_back(a);
        ev_free.push_back(b);
      }
      resident_weight_bytes = (size_t)slots * (raw_slot_bytes + per);
      if (sealed) {
        // layer blocks stay sealed in host memory and are opened in their raw slot on every pass:
        // the messages of layer l in slot s, fixed for the model's life
        const size_t lc = sfile.layer_chunks();
        std::vector<AeadChunk> desc(L * slots * lc);
        for (size_t l = 0; l < L; l++)
          for (int s = 0; s < slots; s++)
            for (size_t c = 0; c < lc; c++)
              desc[(l * slots + s) * lc + c] = sealed_chunk(l * lc + c, raw_slot[s] + c * sfile.layer_chunk,
                                                            std::min<uint64_t>(sfile.layer_chunk, lt - c * sfile.layer_chunk));
        d_layer_desc = dalloc<AeadChunk>(desc.size());
        LS_CUDA(cudaMemcpy(d_layer_desc, desc.data(), desc.size() * sizeof(AeadChunk), cudaMemcpyHostToDevice));
        // the embedding table is opened once, in place in host memory: the input rows and the LM
        // head chunks of every pass read it from there
        uint8_t* he = host_model + (file.embed_start - file.data_start);
        for (size_t first = 0; first < V; first += embed_step) {
          const size_t rows = std::min(embed_step, V - first);
          LS_CUDA(cudaMemcpyAsync(raw_slot[0], he + first * rb, rows * rb, cudaMemcpyHostToDevice, stream));
          open_range(0, sfile.embed_first_chunk() + first / sfile.embed_chunk_rows, raw_slot[0], rows * rb,
                     sfile.embed_chunk_rows * rb, stream);
          LS_CUDA(cudaMemcpyAsync(he + first * rb, raw_slot[0], rows * rb, cudaMemcpyDeviceToHost, stream));
          LS_CUDA(cudaStreamSynchronize(stream));
        }
        sealed_check();
      }
    }

    // K/V cache: per layer a pool [kv_heads][pages][page][hd] f16 (src/model.rs:67-68 reserves the
    // same capacity up front) with this sequence's page table; the RoPE table, computed here with the
    // same float steps as src/model.rs:62-65 and src/kernels.rs:242-252 (so the angles match the CPU
    // path)
    {
      const int sh = kv_page_shift();
      const size_t pages = (max_ctx + ((size_t)1 << sh) - 1) >> sh;
      kv_layer = kv * (pages << sh);
      kc = dalloc<uint16_t>(L * kv_layer);
      vc = dalloc<uint16_t>(L * kv_layer);
      pool.shift = sh;
      pool.init(1, max_ctx, halloc<int32_t>(pages), dalloc<int32_t>(pages));
      pool.h2d = &h2d_bytes;
    }
    const size_t half = cfg.head_dim / 2;
    const std::vector<float2> tab = rope_table(cfg.rope_theta, cfg.head_dim, max_ctx);
    rope = dalloc<float2>(max_ctx * half);
    LS_CUDA(cudaMemcpyAsync(rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, stream));

    // activations for up to one prefill chunk
    x = dalloc<float>(kMaxT * h);
    qkv = dalloc<float>(kMaxT * (h + 2 * kv));
    attn = dalloc<float>(kMaxT * h);
    hbuf = dalloc<float>(kMaxT * I);
    logits = dalloc<float>((size_t)(kMaxDraft + 1) * V);
    const size_t vtiles = (size_t)pad32((int)V) / 32;
    arg_parts = dalloc<ArgPart>(vtiles * kMaxT);
    const size_t max_tiles = std::max<size_t>({(size_t)pad32((int)(h + 2 * kv)), (size_t)2 * I, h}) / 32;
    tickets = dalloc<unsigned>(max_tiles * (kMaxT / 16 + 1));
    partial_floats = (size_t)max_tiles * 32 * 16 * 32 * (kMaxT / 16 + 1);
    partial = dalloc<float>(partial_floats);
    setup_bgemm();
    arg_ticket = dalloc<unsigned>(1);
    // context splits of the attention of one sequence: up to 64 (the tensor-core kernel's bound; the
    // CUDA-core kernel takes at most 16), so that long contexts spread over the SMs
    att_slots = (int)std::max<size_t>(1, std::min<size_t>(64, (max_ctx + 63) / 64));
    att_part_floats = cfg.heads * (size_t)att_slots * kMaxT * (cfg.head_dim + 2);
    att_part = dalloc<float>(att_part_floats);
    att_tickets = dalloc<unsigned>(cfg.heads);
    ctl = dalloc<Ctl>(1);
    ctl_host = halloc<Ctl>(1);
    std::memset(ctl_host, 0, sizeof(Ctl));
    if (mode == LS_MODE_RESIDENT) setup_pass_kernel();
    LS_CUDA(cudaStreamSynchronize(stream));
  }

  // Launch plan of the pass kernel for one token tile (16, 32 or 48 tokens): CTAs, attention slots
  // per head, K slices per GEMV phase and dynamic shared memory.
  struct PassPlan {
    int grid = 0, slots = 1, ks_qkv = 1, ks_o = 1, ks_gu = 1, ks_down = 1, kv_off = 0, stages = 0;
    bool xs = false;
    size_t smem = 0;
  };
  PassPlan pk_plan[3];
  static int pk_class(int T) { return T <= 16 ? 0 : T <= 32 ? 1 : 2; }

  // Device table of layer planes, fixed-point accumulators and the launch plans of the pass kernel.
  void setup_pass_kernel() {
    const char* e = getenv("LS_PASS");
    if (e && std::string(e) == "0") return;
    if (!pass_kernel_supported(cfg.format, cfg.embed_format, 1, (int)cfg.head_dim)) return;
    int max_per_sm = 4;
    if (const char* c = getenv("LS_PASS_CTAS")) max_per_sm = std::max(1, std::min(4, atoi(c)));
    const int h = (int)cfg.hidden, kv = (int)cfg.kv_dim(), I = (int)cfg.inter, QS = h + 2 * kv;
    const int kb = (cfg.format.bits == 4 && cfg.format.group > 64) ? cfg.format.group : 64;
    int max_grid = 0;
    for (int c = 0; c < 3; c++) {
      PassPlan& P = pk_plan[c];
      const int T = 16 * (c + 1);
      // items are 256-row tiles x K slices; enough slices to give every CTA about one item, but
      // at least one whole weight-stream stage (nbs K blocks) per item
      const int nbs = pass_kernel_stage_blocks(cfg.format);
      auto plan = [&](const QMat& w, int grid) {
        const int tiles = (w.rows_pad / 32 + 7) / 8, nblk = w.cols / kb;
        return std::max(1, std::min(std::max(1, nblk / nbs), grid / tiles));
      };
      // one CTA per SM (it takes the whole tensor memory); the weight ring takes the shared memory
      // the rest leaves (LS_PASS_STAGES caps it)
      // the staging reads x from the RMS statistics' shared-memory copy when that leaves room for a
      // ring of at least 4 stages (LS_PASS_XS=0 reads it from L2 again)
      P.ks_down = plan(layers[0].down, num_sms);
      const size_t budget = pass_kernel_smem_budget(cfg.format, T);
      const char* xe = getenv("LS_PASS_XS");
      P.xs = !(xe && std::string(xe) == "0") &&
             pass_kernel_stages(cfg.format, T, h, I, (int)cfg.head_dim, P.ks_down, budget, true) >= 4;
      P.stages = pass_kernel_stages(cfg.format, T, h, I, (int)cfg.head_dim, P.ks_down, budget, P.xs);
      if (const char* st = getenv("LS_PASS_STAGES")) P.stages = std::min(P.stages, std::max(2, atoi(st)));
      if (P.stages == 0) continue;
      const size_t smem = pass_kernel_smem(cfg.format, T, h, I, (int)cfg.head_dim, P.ks_down, P.stages, P.xs);
      const int per_sm = pass_kernel_blocks_per_sm(cfg.format, T, smem, max_per_sm);
      if (per_sm < 1) continue;
      P.grid = per_sm * num_sms;
      P.smem = smem;
      P.ks_qkv = plan(layers[0].qkv, P.grid);
      P.ks_o = plan(layers[0].o, P.grid);
      P.ks_gu = plan(layers[0].gu, P.grid);
      P.slots = std::max(1, std::min(kMaxAttSlots, P.grid / (int)cfg.heads));
      P.kv_off = (int)pass_kernel_kv_off(cfg.format, T, h, I, (int)cfg.head_dim, P.ks_down);
      max_grid = std::max(max_grid, P.grid);
    }
    if (getenv("LS_PASS_VERBOSE"))
      for (int c = 0; c < 3; c++)
        fprintf(stderr, "pass plan T<=%d: grid %d slots %d stages %d xs %d ks qkv %d o %d gu %d down %d smem %zu\n",
                16 * (c + 1), pk_plan[c].grid, pk_plan[c].slots, pk_plan[c].stages, (int)pk_plan[c].xs, pk_plan[c].ks_qkv,
                pk_plan[c].ks_o, pk_plan[c].ks_gu, pk_plan[c].ks_down, pk_plan[c].smem);
    if (pk_plan[0].grid == 0) return;
    pk_max_grid = max_grid;
    // TMA descriptors of every matrix: [layer][qkv, o, gate/up, down], then the embedding/head
    std::vector<QMaps> maps(4 * cfg.layers + 1);
    for (size_t l = 0; l < cfg.layers; l++) {
      pass_encode_maps(layers[l].qkv, &maps[4 * l + 0]);
      pass_encode_maps(layers[l].o, &maps[4 * l + 1]);
      pass_encode_maps(layers[l].gu, &maps[4 * l + 2]);
      pass_encode_maps(layers[l].down, &maps[4 * l + 3]);
    }
    pass_encode_maps(embed, &maps[4 * cfg.layers]);
    d_pass_maps = dalloc<QMaps>(maps.size());
    LS_CUDA(cudaMemcpyAsync(d_pass_maps, maps.data(), maps.size() * sizeof(QMaps), cudaMemcpyHostToDevice, stream));
    std::vector<PassLayer> pl(cfg.layers);
    for (size_t l = 0; l < cfg.layers; l++) {
      pl[l].qkv = layers[l].qkv;
      pl[l].o = layers[l].o;
      pl[l].gu = layers[l].gu;
      pl[l].down = layers[l].down;
      pl[l].maps = d_pass_maps + 4 * l;
      pl[l].in_norm = layers[l].in_norm;
      pl[l].post_norm = layers[l].post_norm;
      pl[l].qkv_bias = layers[l].qkv_bias;
    }
    d_pass_layers = dalloc<PassLayer>(cfg.layers);
    LS_CUDA(cudaMemcpyAsync(d_pass_layers, pl.data(), pl.size() * sizeof(PassLayer), cudaMemcpyHostToDevice, stream));
    constexpr int kMaxPassT = 48;
    x_fix = dalloc<long long>((size_t)kMaxPassT * h);
    qkv_fix = dalloc<long long>((size_t)kMaxPassT * QS);
    gu_fix = dalloc<long long>((size_t)kMaxPassT * 2 * I);
    pk_att = dalloc<float>(cfg.heads * (size_t)kMaxAttSlots * kMaxPassT * (cfg.head_dim + 2));
    pk_bar = dalloc<unsigned>(1 + cfg.heads);
    pk_parts = dalloc<ArgPart>((size_t)max_grid * kMaxPassT);
    LS_CUDA(cudaEventCreate(&pk_ev[0]));
    LS_CUDA(cudaEventCreate(&pk_ev[1]));
  }
  static constexpr int kMaxAttSlots = 16;  // equals the kernel's slot bound

  bool use_pass_kernel(int T) const { return T >= 1 && T <= 48 && pk_plan[pk_class(T)].grid > 0; }

  void launch_pass_kernel(int T, int n_logits, bool want_logits) {
    const PassPlan& P = pk_plan[pk_class(T)];
    PassArgs a{};
    a.layers = d_pass_layers;
    a.embed = embed;
    a.embed_maps = d_pass_maps + 4 * cfg.layers;
    a.final_norm = final_norm;
    a.ctl = ctl;
    a.x = x_fix;
    a.qkv = qkv_fix;
    a.gu = gu_fix;
    a.att_part = pk_att;
    a.kc = kc;
    a.vc = vc;
    a.pages = pool.d_table;
    a.kv_layer = kv_layer;
    a.page_shift = pool.shift;
    a.num_pages = pool.num_pages;
    a.rope = rope;
    a.arg_parts = pk_parts;
    a.logits = want_logits ? logits : nullptr;
    a.bar = pk_bar;
    if (prof_timeline && !pk_trace) pk_trace = dalloc<unsigned>(pk_trace_slots() * (size_t)pk_max_grid);
    a.trace = prof_timeline ? pk_trace : nullptr;
    a.trace_sub = (int)pk_trace_sub();
    a.kv_off = P.kv_off;
    a.stages = P.stages;
    a.xs = P.xs ? 1 : 0;
    a.poll_limit = 1u << 21;  // polls of ~0.5 us: about a second
    if (stall_barrier) {      // test hook: one barrier wait runs out after ~5 ms
      a.stall_barrier = stall_barrier;
      a.poll_limit = 1u << 13;
      stall_barrier = 0;
    }
    pk_T = T;
    pk_n_logits = n_logits;
    pk_traced = a.trace != nullptr;
    pk_grid_last = P.grid;
    a.L = (int)cfg.layers;
    a.hidden = (int)cfg.hidden;
    a.inter = (int)cfg.inter;
    a.heads = (int)cfg.heads;
    a.kv_heads = (int)cfg.kv_heads;
    a.hd = (int)cfg.head_dim;
    a.vocab = (int)cfg.vocab;
    a.max_ctx = (int)max_ctx;
    a.T = T;
    a.n_logits = n_logits;
    a.slots = P.slots;
    a.ks_qkv = P.ks_qkv;
    a.ks_o = P.ks_o;
    a.ks_gu = P.ks_gu;
    a.ks_down = P.ks_down;
    a.eps = cfg.eps;
    // the grid barrier's counter starts at zero
    LS_CUDA(cudaMemsetAsync(pk_bar, 0, sizeof(unsigned), stream));
    if (prof_on) LS_CUDA(cudaEventRecord(pk_ev[0], stream));
    launch_pass(a, cfg.format, P.smem, P.grid, stream);
    if (prof_on) {
      LS_CUDA(cudaEventRecord(pk_ev[1], stream));
      pk_pending = true;
    }
  }
  int pk_grid_last = 0;
  int stall_barrier = 0;  // test hook (ls_model_inject_stall): the next pass kernel stalls at this barrier
  bool pk_pending = false;
  unsigned* pk_trace = nullptr;
  int pk_T = 0, pk_n_logits = 0;
  bool pk_traced = false;
  // timeline slots of one pass: start, (arrive, leave) per grid barrier, end
  // plus 4 stamps inside each phase (embedding, 5 per layer, head)
  size_t pk_trace_sub() const { return 2 * (2 + 5 * cfg.layers) + 2; }
  size_t pk_trace_slots() const { return pk_trace_sub() + 4 * (2 + 5 * cfg.layers); }

  // Turns the pass kernel's barrier timestamps into per-class phase spans (averaged over layers).
  void collect_pass_trace() {
    const int G = pk_grid_last, L = (int)cfg.layers, T = pk_T;
    const int nb = 1 + 5 * L + (pk_n_logits > 0 ? 1 : 0);
    std::vector<uint32_t> tr(pk_trace_slots() * (size_t)G);
    LS_CUDA(cudaMemcpy(tr.data(), pk_trace, tr.size() * 4, cudaMemcpyDeviceToHost));
    const int sub0 = (int)pk_trace_sub();
    auto at = [&](int slot, int c) { return tr[(size_t)slot * G + c]; };
    uint32_t t0 = at(0, 0);
    for (int c = 1; c < G; c++)
      if ((int32_t)(at(0, c) - t0) < 0) t0 = at(0, c);
    auto rel = [&](int slot, int c) { return (double)(int32_t)(at(slot, c) - t0) * 1e-6; };  // ms
    double prev_leave = 0;
    const int h = (int)cfg.hidden, kv = (int)cfg.kv_dim(), I = (int)cfg.inter;
    const LayerW& W = layers[cfg.layers / 2];
    for (int b = 1; b <= nb; b++) {
      double leave = -1e30, busy = 0;
      for (int c = 0; c < G; c++) {
        leave = std::max(leave, rel(2 * b, c));
        busy += rel(2 * b - 1, c) - rel(2 * b - 2, c);
      }
      busy /= G;
      // the critical CTA: last to arrive; its own stamps inside the phase (a stamp outside
      // [its previous departure, its arrival] was not written this pass and merges into the next)
      int cc = 0;
      for (int c = 1; c < G; c++)
        if (rel(2 * b - 1, c) > rel(2 * b - 1, cc)) cc = c;
      double seg[6];
      {
        double t = rel(2 * b - 2, cc);
        const double arr = rel(2 * b - 1, cc);
        for (int k = 0; k < 4; k++) {
          const double sk = rel(sub0 + 4 * (b - 1) + k, cc);
          if (sk >= t && sk <= arr) {
            seg[k] = sk - t;
            t = sk;
          } else {
            seg[k] = 0;
          }
        }
        seg[4] = arr - t;
        seg[5] = leave - arr;
      }
      double span = leave - prev_leave;
      prev_leave = leave;
      if (b == 1) continue;  // embedding rows: part of the whole-pass class only
      int cls = 5;
      double scale = 1.0;
      if (b <= 1 + 5 * L) {
        cls = (b - 2) % 5;
        scale = 1.0 / L;
      } else {
        span += rel(2 * nb + 1, 0) - rel(2 * nb, 0);  // argmax merge + acceptance in CTA 0
      }
      prof.ms[cls] += span * scale;
      prof.busy_ms[cls] += busy * scale;
      for (int k = 0; k < 6; k++) prof.crit_ms[cls][k] += seg[k] * scale;
    }
    const double pos0 = ctl_host->pos0;
    const double b_cls[5] = {gemv_bytes(W.qkv, T, h + 2 * kv),
                             (double)T * kv * 2 * 2 + (double)T * (h + 2 * kv) * 4 + (double)T * h * 4 + pos0 * kv * 2 * 2,
                             gemv_bytes(W.o, T, h) + (double)T * h * 4, gemv_bytes(W.gu, T, I),
                             gemv_bytes(W.down, T, h) + (double)T * h * 4};
    for (int c = 0; c < 5; c++) {
      prof.launches[c]++;
      prof.bytes[c] += b_cls[c];
    }
    if (pk_n_logits > 0) {
      prof.launches[5]++;
      prof.bytes[5] += gemv_bytes(embed, pk_n_logits, 0);
    }
  }

  // ---- the pass --------------------------------------------------------------------------------

  // Opens an event pair around the next launch when profiling (returns the pair index or -1).
  int prof_begin(int cls, double bytes, cudaStream_t s) {
    if (!prof_on) return -1;
    const size_t i = prof_rec.size();
    while (prof_ev.size() < 2 * (i + 1)) {
      cudaEvent_t e;
      LS_CUDA(cudaEventCreate(&e));
      prof_ev.push_back(e);
    }
    prof_rec.push_back({cls, bytes});
    // External: inside a stream capture this becomes an event-record node that timestamps every
    // replay of the graph (a plain record would only be a capture dependency)
    LS_CUDA(cudaEventRecordWithFlags(prof_ev[2 * i], s, cudaEventRecordExternal));
    return (int)i;
  }
  void prof_end(int i, cudaStream_t s) {
    if (i >= 0) LS_CUDA(cudaEventRecordWithFlags(prof_ev[2 * i + 1], s, cudaEventRecordExternal));
  }
  double gemv_bytes(const QMat& w, int M, int out_rows) const {
    const double rb = (double)w.cols * w.bits / 8 + (double)w.groups() * 2;
    return (double)w.rows * rb + (double)M * w.cols * 4 + (double)M * out_rows * 4;
  }
  void prof_collect() {
    if (pk_pending) {
      pk_pending = false;
      float ms = 0;
      LS_CUDA(cudaEventElapsedTime(&ms, pk_ev[0], pk_ev[1]));
      // one launch covers the whole pass: weights once + the cached K/V rows read + new rows
      const double wb = (double)cfg.layers * file.layout.total + (double)cfg.vocab * cfg.embed_row_bytes();
      const double kvb = (double)cfg.layers * ((double)ctl_host->pos0 + ctl_host->M) * cfg.kv_dim() * 2 * 2;
      prof.launches[7 - 1]++;
      prof.ms[7 - 1] += ms;
      prof.busy_ms[7 - 1] += ms;
      prof.bytes[7 - 1] += wb + kvb;
      if (pk_trace && pk_traced) collect_pass_trace();
      return;
    }
    if (!prof_pending || !prof_cur) return;
    prof_pending = false;
    for (size_t i = 0; i < prof_cur->size(); i++) {
      float ms = 0;
      LS_CUDA(cudaEventElapsedTime(&ms, prof_ev[2 * i], prof_ev[2 * i + 1]));
      const ProfRec& r = (*prof_cur)[i];
      prof.launches[r.cls]++;
      prof.ms[r.cls] += ms;
      prof.busy_ms[r.cls] += ms;
      // attention also reads the cached K/V rows of this pass (pos0 of the pass, f16 K and V)
      prof.bytes[r.cls] += r.bytes + (r.cls == 1 ? (double)ctl_host->pos0 * cfg.kv_dim() * 2 * 2 : 0.0);
    }
  }

  int pick_ksplit(const QMat& w, int M) const { return choose_ksplit(w, M, num_sms); }

  // The batched GEMM path of passes through separate kernels, when every matrix's format allows it
  // (LS_BGEMM=0 keeps the per-token-group GEMV): operand and scratch buffers for up to kMaxT rows.
  void setup_bgemm() {
    const char* e = getenv("LS_BGEMM");
    const size_t h = cfg.hidden, I = cfg.inter;
    const LayerW& W = layers[0];
    use_bg = !(e && std::string(e) == "0") && (I % 8) == 0;
    for (const QMat* w : {&W.qkv, &W.o, &W.gu, &W.down}) use_bg = use_bg && bgemm_supported(*w);
    if (!use_bg) return;
    size_t bpf = 0, btk = 0, rows_bt = 0;
    for (int rows = 1; rows <= kMaxT; rows++) {
      for (const QMat* w : {&W.qkv, &W.o, &W.gu, &W.down}) {
        const BgemmPlan p = bgemm_plan(*w, rows, num_sms, false);
        bpf = std::max(bpf, p.partial_floats);
        btk = std::max(btk, p.tickets);
      }
      rows_bt = std::max(rows_bt, bt_elems(rows, 1));
    }
    bt_a = dalloc<uint16_t>(rows_bt * h);
    bt_h = dalloc<uint16_t>(rows_bt * I);
    bg_partial = dalloc<float>(bpf);
    bg_tickets = dalloc<unsigned>(btk);
  }
  void bg(const QMat& w, const uint16_t* xin, int M, int epi, float* y, int y_stride, uint16_t* yh, const uint16_t* bias,
          cudaStream_t s) {
    BgemmLaunch g;
    g.w = w;
    g.x = xin;
    g.M = M;
    g.epi = epi;
    g.y = y;
    g.y_stride = y_stride;
    g.yh = yh;
    g.bias = bias;
    g.partial = bg_partial;
    g.tickets = bg_tickets;
    g.err = &ctl->err;
    launch_bgemm(g, bgemm_plan(w, M, num_sms, false), s);
  }

  void gemv(const QMat& w, const float* xin, int x_stride, int M, int epi, float* y, int y_stride, const uint16_t* norm_bf16,
            const float* norm_f32, const uint16_t* bias, cudaStream_t s) {
    GemvLaunch g;
    g.w = w;
    g.x = xin;
    g.x_stride = x_stride;
    g.M = M;
    g.norm_bf16 = norm_bf16;
    g.norm_f32 = norm_f32;
    g.eps = cfg.eps;
    g.epi = epi;
    g.y = y;
    g.y_stride = y_stride;
    g.bias = bias;
    g.partial = partial;
    g.tickets = tickets;
    g.err = &ctl->err;
    if (use_tc(w)) {
      choose_tc(w, M, num_sms, epi == EPI_ARGMAX, &g.ksplit, &g.grid_x, &g.max_nt);
      launch_gemv_tc(g, s);
      return;
    }
    g.ksplit = (epi == EPI_ARGMAX) ? 1 : pick_ksplit(w, M);
    g.grid_x = gemv_grid_x(w, g.ksplit, M, num_sms);
    launch_gemv(g, s);
  }

  // Returns the number of argmax parts (CTAs) the launch writes.
  int head(const QMat& w, const float* xin, int n, bool want_logits, int row_offset, int n_valid, int part_tile_offset,
           int finalize, int n_part_tiles, cudaStream_t s) {
    GemvLaunch g;
    g.w = w;
    g.x = xin;
    g.x_stride = (int)cfg.hidden;
    g.M = n;
    g.norm_f32 = final_norm;
    g.eps = cfg.eps;
    g.epi = EPI_ARGMAX;
    g.arg_parts = arg_parts;
    g.arg_ticket = arg_ticket;
    g.ctl = ctl;
    g.n_valid_rows = n_valid;
    g.row_offset = row_offset;
    g.part_tile_offset = part_tile_offset;
    g.finalize = finalize;
    g.n_part_tiles = n_part_tiles;
    g.logits = want_logits ? logits : nullptr;
    g.logits_stride = (int)cfg.vocab;
    g.err = &ctl->err;
    if (use_tc(w)) {
      choose_tc(w, n, num_sms, true, &g.ksplit, &g.grid_x, &g.max_nt);
      launch_gemv_tc(g, s);
      return g.grid_x;
    }
    g.grid_x = gemv_grid_x(w, 1, n, num_sms);
    launch_gemv(g, s);
    return g.grid_x;
  }

  void layer_compute(const LayerW& W, size_t l, int T, cudaStream_t s) {
    const int h = (int)cfg.hidden, kv = (int)cfg.kv_dim(), I = (int)cfg.inter;
    const bool sample = prof_on && (int)l == prof_layer();
    auto pb = [&](int cls, double b) { return sample ? prof_begin(cls, b, s) : -1; };
    int pi = pb(0, gemv_bytes(W.qkv, T, h + 2 * kv));
    if (use_bg) {
      launch_bt_prep(x, h, T, h, W.in_norm, nullptr, cfg.eps, bt_a, s);
      bg(W.qkv, bt_a, T, EPI_BIAS_STORE, qkv, h + 2 * kv, nullptr, W.qkv_bias, s);
    } else {
      gemv(W.qkv, x, h, T, EPI_BIAS_STORE, qkv, h + 2 * kv, W.in_norm, nullptr, W.qkv_bias, s);
    }
    prof_end(pi, s);
    AttnLaunch a;
    a.qkv = qkv;
    a.qkv_stride = h + 2 * kv;
    a.k_cache = kc + l * kv_layer;
    a.v_cache = vc + l * kv_layer;
    a.pages = pool.d_table;
    a.page_shift = pool.shift;
    a.num_pages = pool.num_pages;
    a.max_pages = pool.max_pages;
    a.rope = rope;
    a.ctl = ctl;
    a.out = attn;
    a.part = att_part;
    a.tickets = att_tickets;
    a.heads = (int)cfg.heads;
    a.kv_heads = (int)cfg.kv_heads;
    a.hd = (int)cfg.head_dim;
    a.max_ctx = (int)max_ctx;
    a.M = T;
    a.max_splits = att_slots;
    a.err = &ctl->err;
    // attention bytes: new K/V rows written (f16) + q|k|v in and out (f32); the cached rows read are
    // added per replay from that pass's pos0 (prof_collect)
    pi = pb(1, (double)T * kv * 2 * 2 + (double)T * (h + 2 * kv) * 4 + (double)T * h * 4);
    if (use_bg && attention_tc_supported(a)) {  // straight into the O GEMM's operand
      int gn = 16, gg = 1;
      bgemm_groups(T, &gn, &gg);
      a.out_h = bt_a;
      a.out_h_n = gn;
    }
    launch_attention(a, s);
    if (use_bg && !a.out_h) launch_bt_prep(attn, h, T, h, nullptr, nullptr, 0.f, bt_a, s);
    prof_end(pi, s);
    if (use_bg) {
      pi = pb(2, gemv_bytes(W.o, T, h) + (double)T * h * 4);
      bg(W.o, bt_a, T, EPI_RESID, x, h, nullptr, nullptr, s);
      prof_end(pi, s);
      pi = pb(3, gemv_bytes(W.gu, T, I));
      launch_bt_prep(x, h, T, h, W.post_norm, nullptr, cfg.eps, bt_a, s);
      bg(W.gu, bt_a, T, EPI_SWIGLU_H, nullptr, 0, bt_h, nullptr, s);
      prof_end(pi, s);
      pi = pb(4, gemv_bytes(W.down, T, h) + (double)T * h * 4);
      bg(W.down, bt_h, T, EPI_RESID, x, h, nullptr, nullptr, s);
      prof_end(pi, s);
      return;
    }
    pi = pb(2, gemv_bytes(W.o, T, h) + (double)T * h * 4);
    gemv(W.o, attn, h, T, EPI_RESID, x, h, nullptr, nullptr, nullptr, s);
    prof_end(pi, s);
    pi = pb(3, gemv_bytes(W.gu, T, I));
    gemv(W.gu, x, h, T, EPI_SWIGLU, hbuf, I, W.post_norm, nullptr, nullptr, s);
    prof_end(pi, s);
    pi = pb(4, gemv_bytes(W.down, T, h) + (double)T * h * 4);
    gemv(W.down, hbuf, I, T, EPI_RESID, x, h, nullptr, nullptr, nullptr, s);
    prof_end(pi, s);
  }

  // Enqueues one pass over T tokens already in ctl->tokens (pos0 in ctl). n_logits > 0 runs the
  // LM head on the last n_logits positions with the device argmax (and the acceptance rule when
  // ctl->mode == 1); otherwise only advances pos0.
  void enqueue_pass(int T, int n_logits, bool want_logits) {
    const int h = (int)cfg.hidden;
    const size_t V = cfg.vocab;
    if (mode == LS_MODE_RESIDENT) {
      const int pp = prof_begin(6, 0, stream);
      launch_embed(embed, ctl, x, h, T, stream);
      for (size_t l = 0; l < cfg.layers; l++) layer_compute(layers[l], l, T, stream);
      if (n_logits > 0) {
        const int ph = prof_begin(5, gemv_bytes(embed, n_logits, 0), stream);
        head(embed, x + (size_t)(T - n_logits) * h, n_logits, want_logits, 0, (int)V, 0, 1, 0, stream);
        prof_end(ph, stream);
      } else {
        launch_advance(ctl, stream);
      }
      prof_end(pp, stream);
      return;
    }
    // streaming (src/provider.rs:234-268)
    launch_embed_raw(host_embed_dev, cfg.embed_row_bytes(), cfg.embed_format.bits, cfg.embed_format.group, ctl, x, h,
                     (int)V, T, stream);
    bytes_read += (uint64_t)T * cfg.embed_row_bytes();
    int part_tiles = 0;
    stream_weights(
        n_logits > 0, stream, [&](const LayerW& W, size_t l) { layer_compute(W, l, T, stream); },
        [&](const QMat& hq, int first, int rows) {
          part_tiles += head(hq, x + (size_t)(T - n_logits) * h, n_logits, want_logits, first, rows, part_tiles, 0, 0, stream);
        });
    if (n_logits > 0) launch_argmax_finalize(arg_parts, part_tiles, n_logits, ctl, stream);
    else launch_advance(ctl, stream);
  }

  // Streams the weights through the HBM slots: items are layers 0..L-1, then (with_head) the LM
  // head in chunks of kHeadRows rows; each slot is refilled by a copy on the side stream once the
  // compute that used it has finished (src/provider.rs:234-268). layer_fn(planes, l) and
  // head_fn(planes, first_row, rows) enqueue the compute on stream cs.
  template <class LF, class HF>
  void stream_weights(bool with_head, cudaStream_t cs, LF layer_fn, HF head_fn) {
    const size_t V = cfg.vocab, L = cfg.layers;
    const size_t chunk_rows = std::min<size_t>(kHeadRows, V);
    const size_t nchunks = with_head ? (V + chunk_rows - 1) / chunk_rows : 0;
    const size_t items = L + nchunks;
    const size_t lt = file.layout.total, rb = cfg.embed_row_bytes();
    size_t issued = 0;
    auto issue = [&](size_t it) {
      const int s = (int)(it % slots);
      LS_CUDA(cudaStreamWaitEvent(copy_stream, ev_free[s], 0));
      const uint8_t* src;
      size_t n;
      if (it < L) {
        src = host_model + it * lt;
        n = lt;
      } else {
        const size_t c = it - L, first = c * chunk_rows, rows = std::min(chunk_rows, V - first);
        src = host_model + (file.embed_start - file.data_start) + first * rb;
        n = rows * rb;
      }
      LS_CUDA(cudaMemcpyAsync(raw_slot[s], src, n, cudaMemcpyHostToDevice, copy_stream));
      LS_CUDA(cudaEventRecord(ev_loaded[s], copy_stream));
      bytes_read += n;
    };
    for (size_t it = 0; it < items; it++) {
      while (issued < items && issued < it + (size_t)slots) issue(issued++);
      const int s = (int)(it % slots);
      LS_CUDA(cudaStreamWaitEvent(cs, ev_loaded[s], 0));
      if (it < L) {
        if (sealed) {  // open the layer's chunks in the slot (src/seal.rs:977-986)
          const size_t lc = sfile.layer_chunks();
          launch_aead(d_layer_desc + (it * slots + s) * lc, (int)lc, sfile.layer_chunk, d_aad, (uint32_t)sfile.aad_prefix.size(),
                      d_key, false, aead_scr, aead_scr_bytes, d_bad, cs);
        }
        repack_layer(raw_slot[s], layers[s], cs);
        LS_CUDA(cudaEventRecord(ev_free[s], cs));  // the raw slot may be refilled now
        layer_fn(layers[s], it);
      } else {
        const size_t c = it - L, first = c * chunk_rows, rows = std::min(chunk_rows, V - first);
        QMat hq = head_slot[s];
        hq.rows = (int)rows;
        hq.rows_pad = pad32((int)rows);
        repack_embed_rows(raw_slot[s], 0, (int)rows, hq, cs);
        LS_CUDA(cudaEventRecord(ev_free[s], cs));
        head_fn(hq, (int)first, (int)rows);
      }
    }
  }

  void run_pass(int T, int n_logits, bool want_logits) {
    passes++;
    if (mode == LS_MODE_RESIDENT && use_pass_kernel(T)) {
      launch_pass_kernel(T, n_logits, want_logits);
      return;
    }
    if (mode != LS_MODE_RESIDENT) {
      prof_rec.clear();
      enqueue_pass(T, n_logits, want_logits);
      return;
    }
    auto key = std::make_tuple(T, n_logits, (int)want_logits, (int)prof_on);
    auto it = graphs.find(key);
    if (it == graphs.end()) {
      cudaGraph_t graph;
      prof_rec.clear();
      LS_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      try {
        enqueue_pass(T, n_logits, want_logits);
      } catch (...) {
        cudaStreamEndCapture(stream, &graph);
        throw;
      }
      LS_CUDA(cudaStreamEndCapture(stream, &graph));
      cudaGraphExec_t exec;
      LS_CUDA(cudaGraphInstantiate(&exec, graph, 0));
      cudaGraphDestroy(graph);
      it = graphs.emplace(key, exec).first;
      prof_recs[key] = prof_rec;
    }
    LS_CUDA(cudaGraphLaunch(it->second, stream));
    if (prof_on) {
      prof_cur = &prof_recs[key];
      prof_pending = true;
    }
  }

  // ---- host API --------------------------------------------------------------------------------

  void check_request(const uint32_t* ids, uint64_t n) const {
    if (n == 0) LS_THROW(LS_ERR_ARG, "no tokens to process");
    if (pos + n > max_ctx)
      LS_THROW(LS_ERR_ARG, "context is full: " + std::to_string(pos) + " cached + " + std::to_string(n) +
                               " new tokens exceeds the limit of " + std::to_string(max_ctx));
    for (uint64_t i = 0; i < n; i++)
      if (ids[i] >= cfg.vocab) LS_THROW(LS_ERR_ARG, "token id " + std::to_string(ids[i]) + " is outside the vocabulary");
  }

  void push_ctl(int T, int n_logits, int md, const uint32_t* ids) {
    pool.ensure(0, pos + T, stream);  // pages for the pass's new rows
    ctl_host->pos0 = (int32_t)pos;
    ctl_host->M = T;
    ctl_host->n_logits = n_logits;
    ctl_host->mode = md;
    std::memcpy(ctl_host->tokens, ids, (size_t)T * 4);
    ctl_host->err = 0;
    LS_CUDA(cudaMemcpyAsync(ctl, ctl_host, sizeof(Ctl), cudaMemcpyHostToDevice, stream));
    h2d_bytes += sizeof(Ctl);
  }

  void fetch_result() {
    LS_CUDA(cudaMemcpyAsync(&ctl_host->argmax, &ctl->argmax, sizeof(Ctl) - offsetof(Ctl, argmax), cudaMemcpyDeviceToHost, stream));
    d2h_bytes += sizeof(Ctl) - offsetof(Ctl, argmax);
    LS_CUDA(cudaStreamSynchronize(stream));
    prof_collect();
    if (mode != LS_MODE_RESIDENT) sealed_check();
    if (ctl_host->err == 1) LS_THROW(LS_ERR_DEVICE, "a tensor-core kernel gave up waiting on an mbarrier (bounded wait)");
    if (ctl_host->err == 3) LS_THROW(LS_ERR_DEVICE, "the pass kernel gave up waiting at a grid barrier (bounded wait)");
    if (ctl_host->err) LS_THROW(LS_ERR_DEVICE, "a kernel rejected a token id outside the vocabulary");
  }

  // src/model.rs:111-119
  uint32_t forward(const uint32_t* ids, uint64_t n, float* logits_out) {
    check_request(ids, n);
    const uint64_t nchunks = (n + kPrefillChunk - 1) / kPrefillChunk;
    uint32_t tok = 0;
    for (uint64_t c = 0; c < nchunks; c++) {
      const uint64_t a = c * kPrefillChunk, b = std::min<uint64_t>(n, a + kPrefillChunk);
      const bool last = c + 1 == nchunks;
      push_ctl((int)(b - a), last ? 1 : 0, 0, ids + a);
      run_pass((int)(b - a), last ? 1 : 0, last && logits_out != nullptr);
      if (last && logits_out) {
        LS_CUDA(cudaMemcpyAsync(logits_out, logits, cfg.vocab * 4, cudaMemcpyDeviceToHost, stream));
        d2h_bytes += cfg.vocab * 4;
      }
      fetch_result();
      pos += b - a;
      tok = ctl_host->next;
    }
    return tok;
  }

  // src/model.rs:124-133
  void forward_multi(const uint32_t* ids, uint64_t t, uint64_t n, float* logits_out) {
    check_request(ids, t);
    if (n == 0 || n > t) LS_THROW(LS_ERR_ARG, "asked for logits at " + std::to_string(n) + " positions of " + std::to_string(t) + " tokens");
    if (t > (uint64_t)kPrefillChunk) LS_THROW(LS_ERR_ARG, "forward_multi takes at most 128 tokens at a time");
    if (n > (uint64_t)kMaxDraft + 1) LS_THROW(LS_ERR_ARG, "forward_multi returns logits for at most 33 positions");
    push_ctl((int)t, (int)n, 0, ids);
    run_pass((int)t, (int)n, logits_out != nullptr);
    if (logits_out) {
      LS_CUDA(cudaMemcpyAsync(logits_out, logits, n * cfg.vocab * 4, cudaMemcpyDeviceToHost, stream));
      d2h_bytes += n * cfg.vocab * 4;
    }
    fetch_result();
    pos += t;
  }

  // the verify step of src/spec.rs:110-139
  void verify(const uint32_t* block, uint64_t n, uint32_t* m_out, uint32_t* next_out) {
    check_request(block, n);
    if (n > (uint64_t)kMaxDraft + 1) LS_THROW(LS_ERR_ARG, "a verify block holds at most 33 tokens");
    push_ctl((int)n, (int)n, 1, block);
    run_pass((int)n, (int)n, false);
    fetch_result();
    pos += (size_t)ctl_host->m + 1;
    pool.shrink(0, pos);  // the rejected rows' pages go back to the pool
    *m_out = (uint32_t)ctl_host->m;
    *next_out = ctl_host->next;
  }

  void truncate(uint64_t p) {
    if (p > pos) LS_THROW(LS_ERR_ARG, "cannot truncate to " + std::to_string(p) + ": only " + std::to_string(pos) + " tokens are cached");
    pos = p;
    pool.shrink(0, pos);
  }
};

// ------------------------------------------------------------------------------------------------
// Greedy speculative decoding (src/spec.rs:57-152)
// ------------------------------------------------------------------------------------------------

namespace {

// Prompt-lookup drafter (an addition to the reference): proposes the tokens that followed the most
// recent earlier occurrence of the longest suffix n-gram (n = 3, 2, 1) of the history.
std::vector<uint32_t> lookup_draft(const std::vector<uint32_t>& hist, size_t kk) {
  std::vector<uint32_t> out;
  if (kk == 0 || hist.size() < 2) return out;
  for (size_t n = std::min<size_t>(3, hist.size() - 1); n >= 1; n--) {
    const size_t tail = hist.size() - n;
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

}  // namespace

static bool contains(const uint32_t* v, uint64_t n, uint32_t t) {
  for (uint64_t i = 0; i < n; i++)
    if (v[i] == t) return true;
  return false;
}

// The decode loop of src/spec.rs:94-149, from a state where both models hold `hist` and `a` is the
// target's greedy token after it. out_tokens[0] = a.
static void spec_continue(LsModel& target, LsModel* draft, const uint32_t* hist0, uint64_t hlen, uint32_t a,
                          uint64_t max_new, uint64_t k, const uint32_t* eos, uint64_t neos, uint32_t* out_tokens,
                          uint64_t* out_len, LsSpecStats* st) {
  if (k == 0 || k > (uint64_t)kMaxDraft) LS_THROW(LS_ERR_ARG, "k must be between 1 and 32, not " + std::to_string(k));
  if (max_new == 0) LS_THROW(LS_ERR_ARG, "need at least one token to generate");
  if (target.pos != hlen || (draft && draft->pos != hlen)) LS_THROW(LS_ERR_ARG, "the models must hold exactly the history");
  if (draft && draft->cfg.vocab != target.cfg.vocab) LS_THROW(LS_ERR_ARG, "the draft and the target must share a vocabulary");
  const uint64_t need = hlen + max_new + k;
  if (need > target.max_ctx || (draft && need > draft->max_ctx))
    LS_THROW(LS_ERR_ARG, "prompt + max_new + k = " + std::to_string(need) + " tokens exceed the context limit");
  std::vector<uint32_t> out{a};
  std::vector<uint32_t> hist(hist0, hist0 + hlen);
  hist.push_back(a);
  bool stop = contains(eos, neos, a);
  const double td = now_s();
  while (!stop && out.size() < max_new) {
    // never ask for more than is still needed: a pass yields at most kk + 1 tokens
    const uint64_t kk = std::min<uint64_t>(k, max_new - out.size() - 1);
    double ts = now_s();
    std::vector<uint32_t> drafts;
    if (draft) {
      uint32_t cur = a;
      for (uint64_t i = 0; i < kk; i++) {
        cur = draft->forward(&cur, 1, nullptr);
        st->draft_forwards++;
        drafts.push_back(cur);
      }
    } else {
      drafts = lookup_draft(hist, kk);
    }
    st->draft_secs += now_s() - ts;
    std::vector<uint32_t> block{a};
    block.insert(block.end(), drafts.begin(), drafts.end());
    const size_t p = target.pos;
    ts = now_s();
    uint32_t m = 0, next = 0;
    target.verify(block.data(), block.size(), &m, &next);
    st->target_secs += now_s() - ts;
    st->target_passes++;
    st->drafted += drafts.size();
    st->accepted += m;
    for (uint32_t i = 0; i <= m; i++) {
      const uint32_t tok = i < m ? drafts[i] : next;
      out.push_back(tok);
      hist.push_back(tok);
      if (contains(eos, neos, tok) || out.size() == max_new) {
        stop = true;
        break;
      }
    }
    // both models now hold exactly [.., a, d_1 .. d_m]
    if (draft) {
      const size_t want = p + m + 1;
      if (draft->pos > want) {
        draft->truncate(want);
      } else if (draft->pos < want) {
        ts = now_s();
        const size_t from = draft->pos - p;
        draft->forward(block.data() + from, m + 1 - from, nullptr);
        st->draft_forwards++;
        st->draft_secs += now_s() - ts;
      }
    }
    a = next;
  }
  st->decode_secs += now_s() - td;
  std::memcpy(out_tokens, out.data(), out.size() * 4);
  *out_len = out.size();
}

static void speculative_greedy(LsModel& target, LsModel* draft, const uint32_t* prompt, uint64_t plen, uint64_t max_new,
                               uint64_t k, const uint32_t* eos, uint64_t neos, uint32_t* out_tokens, uint64_t* out_len,
                               LsSpecStats* st) {
  if (k == 0 || k > (uint64_t)kMaxDraft) LS_THROW(LS_ERR_ARG, "k must be between 1 and 32, not " + std::to_string(k));
  if (plen == 0 || max_new == 0) LS_THROW(LS_ERR_ARG, "need a prompt and at least one token to generate");
  if (target.pos != 0 || (draft && draft->pos != 0)) LS_THROW(LS_ERR_ARG, "both models must start with an empty cache");
  if (draft && draft->cfg.vocab != target.cfg.vocab) LS_THROW(LS_ERR_ARG, "the draft and the target must share a vocabulary");
  const uint64_t need = plen + max_new + k;
  if (need > target.max_ctx || (draft && need > draft->max_ctx))
    LS_THROW(LS_ERR_ARG, "prompt + max_new + k = " + std::to_string(need) + " tokens exceed the context limit");
  std::memset(st, 0, sizeof *st);
  const double t0 = now_s();
  const uint32_t a = target.forward(prompt, plen, nullptr);
  if (draft) draft->forward(prompt, plen, nullptr);
  st->first_secs = now_s() - t0;
  spec_continue(target, draft, prompt, plen, a, max_new, k, eos, neos, out_tokens, out_len, st);
}

// ------------------------------------------------------------------------------------------------
// Batched verify (configs 4 and 5): B independent sequences sharing one resident model's weights.
// A pass runs ns sequences x M rows as one set of GEMV launches (token groups of 64 on the grid's
// z axis, so each weight tile is read once per pass), one attention launch over all sequences and
// a per-sequence acceptance on the device. src/spec.rs:94-149 per sequence; the sequences share
// nothing but the weights, so every sequence's tokens equal its own single-sequence decode.
// ------------------------------------------------------------------------------------------------

struct LsBatch {
  LsModel* m = nullptr;
  size_t B = 0, max_ctx = 0, max_rows = 0, max_block = 0;
  // Per-rank compute dimensions: the whole model, or this rank's tensor-parallel shard (its q
  // heads, the kv heads they read, a slice of the intermediate dimension).
  struct Dims {
    int heads, kv_heads, q_dim, kv_dim, inter;
  } dm{};
  int tp_rank = 0, tp_world = 1, tp_v0 = 0;
  std::vector<LayerW> tp_layers;
  QMat tp_head;  // this rank's vocabulary rows of the tied head (a view into the model's table)
  ncclComm_t comm = nullptr;
  float* ybuf = nullptr;                            // partial sums of row-parallel projections
  // peer-memory reduction of ybuf over NVLink instead of NCCL (LS_TP_P2P=0 keeps NCCL); ybuf then
  // holds two buffers of partials, reduction e of a pass writing buffer e mod 2 (a pass makes an even
  // number of reductions, so the alternation carries across passes and captured graphs)
  bool p2p = false;
  P2PReduce p2pr{};
  std::vector<void*> ipc_maps;  // the peers' buffers mapped into this process
  size_t yhalf = 0;             // floats in one buffer of partials
  int red_idx = 0;              // reductions enqueued in the current pass
  size_t pending = 0;           // elements of a peer reduction deferred into the next operand prep
  float* ycur() const { return p2p ? ybuf + (size_t)(red_idx & 1) * yhalf : ybuf; }
  ArgPart *tp_best = nullptr, *tp_all = nullptr;    // per-row best of this rank / of all ranks
  const LayerW& layer(size_t l) const { return tp_world > 1 ? tp_layers[l] : m->layers[l]; }
  size_t kv_layer = 0;  // elements of one layer's page pool (K or V)
  PagePool pool;        // pages shared by the batch's sequences
  cudaStream_t stream = nullptr;
  std::vector<void*> dev_allocs, host_allocs;
  uint16_t *kc = nullptr, *vc = nullptr;
  float2* rope = nullptr;
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *hbuf = nullptr, *partial = nullptr, *att_part = nullptr;
  unsigned *tickets = nullptr, *att_tickets = nullptr;
  ArgPart* parts = nullptr;
  uint32_t *d_tok = nullptr, *d_argmax = nullptr, *d_m = nullptr, *d_next = nullptr;
  int *d_pos0 = nullptr, *d_err = nullptr;
  float* inv_rms = nullptr;  // [max_rows] 1/rms of the rows a normed GEMV reads
  // batched weight GEMM path: activations as f16 in the bt layout, split-K scratch
  bool use_bg = false;
  uint16_t *bt_a = nullptr, *bt_h = nullptr;  // GEMM inputs (K = hidden or q width) / SwiGLU output (K = inter)
  float* bg_partial = nullptr;
  unsigned* bg_tickets = nullptr;
  bool graphs_on = true;                       // LS_BATCH_GRAPHS=0 launches every pass eagerly
  std::map<int, cudaGraphExec_t> bgraphs;      // decode passes by block length
  uint32_t *h_tok = nullptr, *h_m = nullptr, *h_next = nullptr;
  int *h_pos0 = nullptr, *h_err = nullptr;
  int inject_err = 0;      // test hook: the next pass reports this error code (a host-made fault)
  bool tp_failed = false;  // a tensor-parallel pass reported an error
  std::vector<uint64_t> pos;
  uint64_t passes = 0, h2d_bytes = 0, d2h_bytes = 0;

  // Live profile: an event pair around every launch class of a pass (classes as LsBatchProfile).
  bool prof_on = false;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<std::pair<int, double>> prof_rec;  // (class, algorithmic bytes) per event pair
  LsBatchProfile prof{};
  int prof_begin(int cls, double bytes) {
    if (!prof_on) return -1;
    const size_t i = prof_rec.size();
    while (prof_ev.size() < 2 * (i + 1)) {
      cudaEvent_t e;
      LS_CUDA(cudaEventCreate(&e));
      prof_ev.push_back(e);
    }
    prof_rec.push_back({cls, bytes});
    LS_CUDA(cudaEventRecord(prof_ev[2 * i], stream));
    return (int)i;
  }
  void prof_end(int i) {
    if (i >= 0) LS_CUDA(cudaEventRecord(prof_ev[2 * i + 1], stream));
  }
  void prof_collect() {  // after the pass's stream synchronize
    for (size_t i = 0; i < prof_rec.size(); i++) {
      float ms = 0;
      LS_CUDA(cudaEventElapsedTime(&ms, prof_ev[2 * i], prof_ev[2 * i + 1]));
      const int c = prof_rec[i].first;
      prof.launches[c]++;
      prof.ms[c] += ms;
      prof.bytes[c] += prof_rec[i].second;
    }
    prof_rec.clear();
  }
  static double qbytes(const QMat& w) {
    return (double)w.rows_pad * ((double)w.cols * w.bits / 8 + (double)w.groups() * 2);
  }

  template <class T>
  T* dalloc(size_t n) {
    void* p = nullptr;
    LS_CUDA(cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 16)));
    dev_allocs.push_back(p);
    LS_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(n * sizeof(T), 16), stream));
    return reinterpret_cast<T*>(p);
  }
  template <class T>
  T* halloc(size_t n) {
    void* p = nullptr;
    LS_CUDA(cudaHostAlloc(&p, std::max<size_t>(n * sizeof(T), 16), cudaHostAllocDefault));
    host_allocs.push_back(p);
    return reinterpret_cast<T*>(p);
  }

  // Split-K scratch of the tensor-core GEMV for one launch of M token rows.
  void tc_scratch(const QMat& w, int M, size_t* floats, size_t* tks) const {
    int ks = 1, gx = 1;
    choose_tc(w, M, m->num_sms, false, &ks, &gx);
    const int NT = M <= 16 ? 16 : M <= 32 ? 32 : M <= 48 ? 48 : 64;
    const size_t nz = (M + NT - 1) / NT, tiles32 = w.rows_pad / 32;
    *floats = std::max(*floats, nz * tiles32 * ks * NT * 32);
    *tks = std::max(*tks, nz * tiles32);
  }

  // A slice of a tiled matrix into new planes: row tiles [t0, t0 + nt) x columns [c0, c0 + nc).
  QMat slice(const QMat& src, int t0, int nt, int c0, int nc) {
    WeightFormat f;
    f.bits = src.bits;
    f.group = src.group;
    uint8_t* p = dalloc<uint8_t>(qmat_bytes(nt * 32, nc, f));
    QMat d = carve(p, nt * 32, nc, f);
    const size_t cw = 128 / src.bits;  // columns per 16-byte chunk
    LS_CUDA(cudaMemcpy2DAsync(const_cast<uint8_t*>(d.data), (size_t)d.chunks() * 512,
                              src.data + ((size_t)t0 * src.chunks() + c0 / cw) * 512, (size_t)src.chunks() * 512,
                              (size_t)d.chunks() * 512, nt, cudaMemcpyDeviceToDevice, stream));
    LS_CUDA(cudaMemcpy2DAsync(const_cast<uint16_t*>(d.scales), (size_t)d.groups() * 64,
                              src.scales + ((size_t)t0 * src.groups() + c0 / src.group) * 32, (size_t)src.groups() * 64,
                              (size_t)d.groups() * 64, nt, cudaMemcpyDeviceToDevice, stream));
    return d;
  }
  // Rows [r0, r0 + n) of planes (32-row aligned) appended into d's row tiles from tile dt.
  void copy_rows(QMat& d, int dt, const QMat& src, int r0, int n) {
    const int nt = n / 32, st = r0 / 32;
    LS_CUDA(cudaMemcpyAsync(const_cast<uint8_t*>(d.data) + (size_t)dt * d.chunks() * 512, src.data + (size_t)st * src.chunks() * 512,
                            (size_t)nt * src.chunks() * 512, cudaMemcpyDeviceToDevice, stream));
    LS_CUDA(cudaMemcpyAsync(const_cast<uint16_t*>(d.scales) + (size_t)dt * d.groups() * 32,
                            src.scales + (size_t)st * src.groups() * 32, (size_t)nt * src.groups() * 64, cudaMemcpyDeviceToDevice,
                            stream));
  }

  // This rank's shard of every layer (column-parallel QKV by q heads and gate/up by intermediate
  // slice; row-parallel O and down) and of the head's vocabulary, copied out of the resident
  // planes on the device.
  void make_shard(const uint8_t* nccl_id) {
    const Config& c = m->cfg;
    const int R = tp_world, r = tp_rank, hd = (int)c.head_dim, h = (int)c.hidden;
    if (m->mode != LS_MODE_RESIDENT) LS_THROW(LS_ERR_ARG, "tensor parallelism needs a resident model");
    if (c.heads % R) LS_THROW(LS_ERR_ARG, "the q heads do not split evenly over the ranks");
    const int hl = (int)c.heads / R, group = (int)(c.heads / c.kv_heads);
    int kvl, kv0;
    if (R <= (int)c.kv_heads) {
      if (c.kv_heads % R) LS_THROW(LS_ERR_ARG, "the kv heads do not split evenly over the ranks");
      kvl = (int)c.kv_heads / R;
      kv0 = r * kvl;
    } else {
      if (R % c.kv_heads || group % hl) LS_THROW(LS_ERR_ARG, "each rank's q heads must share one kv head");
      kvl = 1;
      kv0 = r * hl / group;
    }
    const int nb = (int)c.inter / 64;
    const int i0 = 64 * (r * nb / R), i1 = 64 * ((r + 1) * nb / R);
    if (c.inter % 64 || i1 <= i0) LS_THROW(LS_ERR_ARG, "the intermediate dimension does not split over the ranks in 64s");
    dm = Dims{hl, kvl, hl * hd, kvl * hd, i1 - i0};
    if (dm.q_dim % 64) LS_THROW(LS_ERR_ARG, "each rank's q width must be a multiple of 64");
    if (!c.format.quant()) LS_THROW(LS_ERR_ARG, "tensor parallelism takes quantized models");
    const int gq = m->layers[0].o.group;
    if (dm.q_dim % gq || (i1 - i0) % gq || (r * dm.q_dim) % gq || i0 % gq)
      LS_THROW(LS_ERR_ARG, "each rank's column slice of O and down must hold whole quantization groups");
    const int QF = (int)(c.heads * c.head_dim), KVf = (int)c.kv_dim(), QSl = dm.q_dim + 2 * dm.kv_dim;
    tp_layers.resize(c.layers);
    for (size_t l = 0; l < c.layers; l++) {
      const LayerW& F = m->layers[l];
      LayerW& W = tp_layers[l];
      WeightFormat f;
      f.bits = F.qkv.bits;
      f.group = F.qkv.group;
      uint8_t* qp = dalloc<uint8_t>(qmat_bytes(QSl, h, f));
      W.qkv = carve(qp, QSl, h, f);
      copy_rows(W.qkv, 0, F.qkv, r * dm.q_dim, dm.q_dim);
      copy_rows(W.qkv, dm.q_dim / 32, F.qkv, QF + kv0 * hd, dm.kv_dim);
      copy_rows(W.qkv, (dm.q_dim + dm.kv_dim) / 32, F.qkv, QF + KVf + kv0 * hd, dm.kv_dim);
      W.o = slice(F.o, 0, F.o.rows_pad / 32, r * dm.q_dim, dm.q_dim);
      W.o.rows = F.o.rows;
      W.gu = slice(F.gu, i0 / 16, (i1 - i0) / 16, 0, h);  // a tile holds 16 gate rows then the same 16 up rows
      W.gu.rows = 2 * (i1 - i0);
      W.down = slice(F.down, 0, F.down.rows_pad / 32, i0, i1 - i0);
      W.down.rows = F.down.rows;
      W.in_norm = F.in_norm;
      W.post_norm = F.post_norm;
      W.qkv_bias = dalloc<uint16_t>(QSl);
      LS_CUDA(cudaMemcpyAsync(W.qkv_bias, F.qkv_bias + r * dm.q_dim, dm.q_dim * 2, cudaMemcpyDeviceToDevice, stream));
      LS_CUDA(cudaMemcpyAsync(W.qkv_bias + dm.q_dim, F.qkv_bias + QF + kv0 * hd, dm.kv_dim * 2, cudaMemcpyDeviceToDevice, stream));
      LS_CUDA(cudaMemcpyAsync(W.qkv_bias + dm.q_dim + dm.kv_dim, F.qkv_bias + QF + KVf + kv0 * hd, dm.kv_dim * 2,
                              cudaMemcpyDeviceToDevice, stream));
    }
    const int tiles = pad32((int)c.vocab) / 32, t0 = r * tiles / R, t1 = (r + 1) * tiles / R;
    tp_v0 = 32 * t0;
    tp_head = m->embed;
    tp_head.data += (size_t)t0 * m->embed.chunks() * 512;
    tp_head.scales += (size_t)t0 * m->embed.groups() * 32;
    tp_head.rows = std::min((int)c.vocab, 32 * t1) - tp_v0;
    tp_head.rows_pad = 32 * (t1 - t0);
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    nccl_check(nccl_api().comm_init_rank(&comm, R, id, r), "ncclCommInitRank");
  }

  LsBatch(LsModel* model, size_t batch, size_t ctx, size_t block, int rank = 0, int world = 1,
          const uint8_t* nccl_id = nullptr)
      : m(model), B(batch), max_ctx(ctx), max_block(block), tp_rank(rank), tp_world(world) {
    if (B == 0 || B > 4096) LS_THROW(LS_ERR_ARG, "batch must be in 1..4096");
    if (max_block == 0 || max_block > (size_t)kMaxDraft + 1) LS_THROW(LS_ERR_ARG, "the verify block holds 1..33 tokens");
    if (max_ctx < 2 || max_ctx > (1u << 20)) LS_THROW(LS_ERR_ARG, "max_ctx must be in 2..2^20");
    const Config& c = m->cfg;
    if (tp_world < 1 || tp_rank < 0 || tp_rank >= tp_world) LS_THROW(LS_ERR_ARG, "rank must be in 0..world-1");
    if (tp_world > 1 && !nccl_id) LS_THROW(LS_ERR_ARG, "a tensor-parallel batch needs the NCCL unique id");
    // rows of a pass: a verify block of every sequence, or one prefill chunk of up to
    // kPrefillSeqs sequences at a time
    max_rows = std::max<size_t>({(size_t)kMaxT, B * max_block, std::min<size_t>(B, kPrefillSeqs) * kPrefillChunk});
    if (max_rows > 8192) LS_THROW(LS_ERR_ARG, "batch x block exceeds 8192 rows per pass");
    LS_CUDA(cudaSetDevice(m->device));
    LS_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    dm = Dims{(int)c.heads, (int)c.kv_heads, (int)(c.heads * c.head_dim), (int)c.kv_dim(), (int)c.inter};
    if (tp_world > 1) make_shard(nccl_id);
    const size_t L = c.layers, kv = dm.kv_dim, h = c.hidden, I = dm.inter, QS = dm.q_dim + 2 * kv;
    // per layer one page pool for all sequences (as many pages as B full contexts need), handed
    // to the sequences as they grow
    {
      const int sh = kv_page_shift();
      const size_t per_seq = (max_ctx + ((size_t)1 << sh) - 1) >> sh;
      kv_layer = kv * ((B * per_seq) << sh);
      kc = dalloc<uint16_t>(L * kv_layer);
      vc = dalloc<uint16_t>(L * kv_layer);
      pool.shift = sh;
      pool.init((int)B, max_ctx, halloc<int32_t>(B * per_seq), dalloc<int32_t>(B * per_seq));
      pool.h2d = &h2d_bytes;
    }
    const std::vector<float2> tab = rope_table(c.rope_theta, c.head_dim, max_ctx);
    rope = dalloc<float2>(tab.size());
    LS_CUDA(cudaMemcpyAsync(rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, stream));
    x = dalloc<float>(max_rows * h);
    qkv = dalloc<float>(max_rows * QS);
    attn = dalloc<float>(max_rows * dm.q_dim);
    hbuf = dalloc<float>(max_rows * I);
    if (tp_world > 1) {
      ybuf = dalloc<float>(2 * max_rows * h);  // two buffers for the peer-memory path
      tp_best = dalloc<ArgPart>(max_rows);
      tp_all = dalloc<ArgPart>((size_t)tp_world * max_rows);
    }
    size_t pf = 0, tk = 0;
    const LayerW& W = layer(0);
    for (int rows = 1; rows <= (int)max_rows; rows++)
      for (const QMat* w : {&W.qkv, &W.o, &W.gu, &W.down}) tc_scratch(*w, rows, &pf, &tk);
    {
      const char* e = getenv("LS_BGEMM");
      use_bg = !(e && std::string(e) == "0") && (dm.inter % 8) == 0;
      QMat head_fmt;  // the LM head's format (its planes may be streamed)
      head_fmt.bits = c.embed_format.bits;
      head_fmt.group = c.embed_format.group;
      head_fmt.cols = (int)c.hidden;
      head_fmt.rows = head_fmt.rows_pad = 32;
      for (const QMat* w : {&W.qkv, &W.o, &W.gu, &W.down, static_cast<const QMat*>(&head_fmt)})
        use_bg = use_bg && bgemm_supported(*w);
    }
    {
      const char* e = getenv("LS_BATCH_GRAPHS");
      graphs_on = !(e && std::string(e) == "0");
    }
    if (use_bg) {
      size_t bpf = 0, btk = 0;
      for (int rows = 1; rows <= (int)max_rows; rows++)
        for (const QMat* w : {&W.qkv, &W.o, &W.gu, &W.down}) {
          const BgemmPlan p = bgemm_plan(*w, rows, m->num_sms, false);
          bpf = std::max(bpf, p.partial_floats);
          btk = std::max(btk, p.tickets);
        }
      size_t rows_bt = 0;  // padded token-group rows of the largest pass
      for (int rows = 1; rows <= (int)max_rows; rows++) rows_bt = std::max(rows_bt, bt_elems(rows, 1));
      bt_a = dalloc<uint16_t>(rows_bt * std::max((int)h, dm.q_dim));
      bt_h = dalloc<uint16_t>(rows_bt * I);
      bg_partial = dalloc<float>(bpf);
      bg_tickets = dalloc<unsigned>(btk);
    }
    partial = dalloc<float>(pf);
    tickets = dalloc<unsigned>(tk);
    parts = dalloc<ArgPart>((size_t)(pad32((int)c.vocab) / 128 + c.vocab / kHeadRows + 2) * max_rows);
    att_part = dalloc<float>(dm.heads * (size_t)16 * max_rows * (c.head_dim + 2));
    att_tickets = dalloc<unsigned>(B * dm.heads);
    d_tok = dalloc<uint32_t>(max_rows);
    d_argmax = dalloc<uint32_t>(max_rows);
    d_m = dalloc<uint32_t>(B);
    d_next = dalloc<uint32_t>(B);
    d_pos0 = dalloc<int>(B);
    d_err = dalloc<int>(1);
    if (tp_world > 1) setup_p2p();
    inv_rms = dalloc<float>(max_rows);
    h_tok = halloc<uint32_t>(max_rows);
    h_m = halloc<uint32_t>(B);
    h_next = halloc<uint32_t>(B);
    h_pos0 = halloc<int>(B);
    h_err = halloc<int>(1);
    pos.assign(B, 0);
    LS_CUDA(cudaStreamSynchronize(stream));
  }
  ~LsBatch() {
    cudaSetDevice(m->device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto& kv : bgraphs) cudaGraphExecDestroy(kv.second);  // before the communicator its nodes use
    // a failed tensor-parallel pass may leave collectives in flight on a peer: abort, do not wait
    if (comm) (tp_failed ? nccl_api().comm_abort : nccl_api().comm_destroy)(comm);
    for (cudaEvent_t e : prof_ev) cudaEventDestroy(e);
    for (void* p : ipc_maps) cudaIpcCloseMemHandle(p);
    for (void* p : dev_allocs) cudaFree(p);
    for (void* p : host_allocs) cudaFreeHost(p);
    if (stream) cudaStreamDestroy(stream);
  }

  void gemv(const QMat& w, const float* xin, int x_stride, int M, int epi, float* y, int y_stride, const uint16_t* norm_bf16,
            const uint16_t* bias) {
    GemvLaunch g;
    g.w = w;
    g.x = xin;
    g.x_stride = x_stride;
    g.M = M;
    g.norm_bf16 = norm_bf16;
    g.eps = m->cfg.eps;
    g.epi = epi;
    g.y = y;
    g.y_stride = y_stride;
    g.bias = bias;
    g.partial = partial;
    g.tickets = tickets;
    g.err = d_err;
    if (norm_bf16) {  // the row norms once, not in every CTA
      launch_inv_rms(xin, x_stride, M, (int)w.cols, g.eps, inv_rms, stream);
      g.inv_rms = inv_rms;
    }
    if (use_tc(w)) {
      choose_tc(w, M, m->num_sms, false, &g.ksplit, &g.grid_x);
      launch_gemv_tc(g, stream);
      return;
    }
    LS_THROW(LS_ERR_ARG, "batches need a weight format the tensor-core GEMV supports");
  }

  // Argmax parts of the LM head rows [first, first + rows) (planes w) over M rows of x (final
  // RMSNorm folded in), written after part_off earlier parts; returns this launch's CTA count.
  int head(const QMat& w, int first, int rows, const float* xin, int x_stride, int M, int part_off) {
    GemvLaunch g;
    g.w = w;
    g.x = xin;
    g.x_stride = x_stride;
    g.M = M;
    g.norm_f32 = m->final_norm;
    g.eps = m->cfg.eps;
    g.epi = EPI_ARGMAX;
    g.arg_parts = parts;
    g.n_valid_rows = rows;
    g.row_offset = first;
    g.part_tile_offset = part_off;
    g.finalize = 0;
    g.err = d_err;
    if (part_off == 0) launch_inv_rms(xin, x_stride, M, (int)m->cfg.hidden, g.eps, inv_rms, stream);
    g.inv_rms = inv_rms;
    if (!use_tc(w)) LS_THROW(LS_ERR_ARG, "batches need a weight format the tensor-core GEMV supports");
    choose_tc(w, M, m->num_sms, true, &g.ksplit, &g.grid_x, &g.max_nt);
    launch_gemv_tc(g, stream);
    return g.grid_x;
  }

  // Batched weight GEMM of M rows of bt-layout activations xin.
  void bg(const QMat& w, const uint16_t* xin, int M, int epi, float* y, int y_stride, uint16_t* yh, const uint16_t* bias) {
    BgemmLaunch g;
    g.w = w;
    g.x = xin;
    g.M = M;
    g.epi = epi;
    g.y = y;
    g.y_stride = y_stride;
    g.yh = yh;
    g.bias = bias;
    g.partial = bg_partial;
    g.tickets = bg_tickets;
    g.err = d_err;
    launch_bgemm(g, bgemm_plan(w, M, m->num_sms, false), stream);
  }
  // LM head rows [first, first + rows) with the argmax epilogue over M rows of bt_a; returns the
  // number of argmax parts written after part_off.
  int bg_head(const QMat& w, int first, int rows, int M, int part_off) {
    BgemmLaunch g;
    g.w = w;
    g.x = bt_a;
    g.M = M;
    g.epi = EPI_ARGMAX;
    g.arg_parts = parts;
    g.n_valid_rows = rows;
    g.row_offset = first;
    g.part_tile_offset = part_off;
    g.err = d_err;
    launch_bgemm(g, bgemm_plan(w, M, m->num_sms, true), stream);
    return (w.rows_pad / 32 + 3) / 4;
  }

  // One pass over sequences [s0, s0 + ns), M rows each. head_mode 0: advance only; 1: argmax of
  // every row and the acceptance rule per sequence (pos += m + 1); 2: argmax of the last row
  // (prefill of one sequence), pos += M.
  // Sum of the row-parallel partials (ycur()) over the ranks, then the residual add into x. On the
  // peer-memory path with the batched GEMMs the sum is deferred into the next operand prep (prep_x),
  // which every consumer of x on that path is, or into flush_reduce.
  void reduce_into_x(size_t n) {
    if (p2p && use_bg) {
      if (pending) LS_THROW(LS_ERR_ARG, "internal: a peer reduction is already pending");
      pending = n;
      return;
    }
    const int pi = prof_begin(6, (double)n * 4 * 2 * (tp_world - 1) / tp_world);
    if (p2p) {
      launch_p2p_reduce_add(x, p2pr, (size_t)(red_idx & 1) * yhalf, n, m->num_sms, stream);
      red_idx++;
    } else {
      nccl_check(nccl_api().all_reduce(ybuf, ybuf, n, ncclFloat32, ncclSum, comm, stream), "ncclAllReduce");
      launch_add(x, ybuf, n, stream);
    }
    prof_end(pi);
  }
  void flush_reduce() {
    if (!pending) return;
    const size_t n = pending;
    pending = 0;
    const int pi = prof_begin(6, (double)n * 4 * 2 * (tp_world - 1) / tp_world);
    launch_p2p_reduce_add(x, p2pr, (size_t)(red_idx & 1) * yhalf, n, m->num_sms, stream);
    red_idx++;
    prof_end(pi);
  }
  // The batched GEMM's operand from `rows` rows of x (stride hidden), RMSNorm-ed with nb or nf; a
  // pending peer reduction over the same rows is applied first, in the same kernel.
  void prep_x(int rows, const uint16_t* nb, const float* nf) {
    const int h = (int)m->cfg.hidden;
    if (pending && pending == (size_t)rows * h) {
      pending = 0;
      const int pi = prof_begin(6, (double)rows * h * 4 * 2 * (tp_world - 1) / tp_world);
      launch_p2p_reduce_prep(x, p2pr, (size_t)(red_idx & 1) * yhalf, rows, h, nb, nf, m->cfg.eps, bt_a, m->num_sms, stream);
      red_idx++;
      prof_end(pi);
      return;
    }
    flush_reduce();
    launch_bt_prep(x, h, rows, h, nb, nf, m->cfg.eps, bt_a, stream);
  }

  // Maps every rank's partial buffer and flag words into this process (CUDA IPC; the handles are
  // exchanged with an NCCL all-gather) when every rank sits on its own GPU and can reach every
  // peer's memory. A collective call: all ranks take the same decision (the check is reduced over
  // the ranks). LS_TP_P2P=0 keeps the NCCL all-reduce; LS_TP_WAIT_MS bounds each wait of the
  // reduction kernels (default 5000).
  void setup_p2p() {
    const char* pe = getenv("LS_TP_P2P");
    if ((pe && std::string(pe) == "0") || tp_world > kMaxTpWorld) return;
    struct Handles {
      cudaIpcMemHandle_t y, f;
      cudaUUID_t uuid;
    };
    P2PReduce r;
    r.world = tp_world;
    r.rank = tp_rank;
    r.flags = dalloc<unsigned>((size_t)tp_world);
    r.seq = dalloc<unsigned>(1);
    r.ticket = dalloc<unsigned>(1);
    r.arrive = dalloc<unsigned>(1);
    r.err = d_err;
    const char* we = getenv("LS_TP_WAIT_MS");
    const long long wait_ms = we ? std::max(1ll, std::atoll(we)) : 5000;
    r.limit_ns = (unsigned long long)wait_ms * 1000000ull;
    Handles mine{};
    LS_CUDA(cudaIpcGetMemHandle(&mine.y, ybuf));
    LS_CUDA(cudaIpcGetMemHandle(&mine.f, r.flags));
    cudaDeviceProp prop;
    LS_CUDA(cudaGetDeviceProperties(&prop, m->device));
    mine.uuid = prop.uuid;
    auto* dsend = dalloc<uint8_t>(sizeof(Handles));
    auto* drecv = dalloc<uint8_t>(sizeof(Handles) * tp_world);
    LS_CUDA(cudaMemcpyAsync(dsend, &mine, sizeof(Handles), cudaMemcpyHostToDevice, stream));
    nccl_check(nccl_api().all_gather(dsend, drecv, sizeof(Handles), ncclUint8, comm, stream), "ncclAllGather (handles)");
    std::vector<Handles> all(tp_world);
    LS_CUDA(cudaMemcpyAsync(all.data(), drecv, sizeof(Handles) * tp_world, cudaMemcpyDeviceToHost, stream));
    LS_CUDA(cudaStreamSynchronize(stream));
    // every peer on another GPU that this process sees and can reach: ranks that wait on one
    // another must never share a GPU
    int ok = 1, ndev = 0;
    LS_CUDA(cudaGetDeviceCount(&ndev));
    for (int p = 0; p < tp_world && ok; p++) {
      if (p == tp_rank) continue;
      if (std::memcmp(&all[p].uuid, &mine.uuid, sizeof(cudaUUID_t)) == 0) ok = 0;
      int local = -1;
      for (int d = 0; d < ndev && ok; d++) {
        cudaDeviceProp q;
        LS_CUDA(cudaGetDeviceProperties(&q, d));
        if (std::memcmp(&q.uuid, &all[p].uuid, sizeof(cudaUUID_t)) == 0) local = d;
      }
      int can = 0;
      if (local < 0 || cudaDeviceCanAccessPeer(&can, m->device, local) != cudaSuccess || !can) ok = 0;
    }
    auto* dok = dalloc<int>(1);
    LS_CUDA(cudaMemcpyAsync(dok, &ok, 4, cudaMemcpyHostToDevice, stream));
    nccl_check(nccl_api().all_reduce(dok, dok, 1, ncclInt32, ncclMin, comm, stream), "ncclAllReduce (peer access)");
    LS_CUDA(cudaMemcpyAsync(&ok, dok, 4, cudaMemcpyDeviceToHost, stream));
    LS_CUDA(cudaStreamSynchronize(stream));
    if (!ok) return;
    // map the peers' buffers; a failure on any rank sends every rank back to NCCL (a rank that
    // threw here alone would leave the others waiting for it in their first pass)
    for (int p = 0; p < tp_world && ok; p++) {
      if (p == tp_rank) {
        r.peer_y[p] = ybuf;
        r.peer_flags[p] = r.flags;
        continue;
      }
      void *py = nullptr, *pf = nullptr;
      if (cudaIpcOpenMemHandle(&py, all[p].y, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        ok = 0;
        break;
      }
      ipc_maps.push_back(py);
      if (cudaIpcOpenMemHandle(&pf, all[p].f, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        ok = 0;
        break;
      }
      ipc_maps.push_back(pf);
      r.peer_y[p] = static_cast<const float*>(py);
      r.peer_flags[p] = static_cast<unsigned*>(pf);
    }
    if (!ok) cudaGetLastError();  // clear the failed open's error
    LS_CUDA(cudaMemcpyAsync(dok, &ok, 4, cudaMemcpyHostToDevice, stream));
    nccl_check(nccl_api().all_reduce(dok, dok, 1, ncclInt32, ncclMin, comm, stream), "ncclAllReduce (peer mappings)");
    LS_CUDA(cudaMemcpyAsync(&ok, dok, 4, cudaMemcpyDeviceToHost, stream));
    LS_CUDA(cudaStreamSynchronize(stream));
    if (!ok) {
      for (void* q : ipc_maps) cudaIpcCloseMemHandle(q);
      ipc_maps.clear();
      return;
    }
    p2pr = r;
    p2p = true;
    yhalf = max_rows * (size_t)m->cfg.hidden;
  }

  // A sequence's length; the pages past it go back to the pool.
  void set_pos(size_t sq, uint64_t p) {
    pos[sq] = p;
    pool.shrink((int)sq, p);
  }

  void pass(size_t s0, size_t ns, int M, const uint32_t* tokens, int head_mode) {
    const Config& c = m->cfg;
    const int h = (int)c.hidden, kv = dm.kv_dim, I = dm.inter, QS = dm.q_dim + 2 * kv;
    const bool tp = tp_world > 1;
    const size_t T = ns * (size_t)M;
    if (T == 0 || T > max_rows) LS_THROW(LS_ERR_ARG, "pass of " + std::to_string(T) + " rows exceeds the batch's " + std::to_string(max_rows));
    if (s0 + ns > B) LS_THROW(LS_ERR_ARG, "sequence index out of range");
    size_t maxpos = 0;
    for (size_t i = 0; i < ns; i++) {
      if (pos[s0 + i] + M > max_ctx)
        LS_THROW(LS_ERR_ARG, "sequence " + std::to_string(s0 + i) + ": context is full (" + std::to_string(pos[s0 + i]) + " + " +
                                 std::to_string(M) + " > " + std::to_string(max_ctx) + ")");
      maxpos = std::max<size_t>(maxpos, pos[s0 + i]);
      h_pos0[i] = (int)pos[s0 + i];
    }
    for (size_t i = 0; i < T; i++)
      if (tokens[i] >= c.vocab) LS_THROW(LS_ERR_ARG, "token id " + std::to_string(tokens[i]) + " is outside the vocabulary");
    for (size_t i = 0; i < ns; i++) pool.ensure((int)(s0 + i), pos[s0 + i] + M, stream);  // pages for the new rows
    std::memcpy(h_tok, tokens, T * 4);
    h2d_bytes += T * 4 + ns * 4;
    const bool streamed = m->mode != LS_MODE_RESIDENT;
    // A decode pass of every sequence on resident weights replays a captured graph (one per block
    // length): positions and tokens come from the pinned buffers at replay time, the attention is
    // sized for the whole context.
    const bool graphed = graphs_on && !streamed && !prof_on && use_bg && s0 == 0 && ns == B && head_mode == 1 && !inject_err;
    auto enqueue = [&](bool for_graph) {
    red_idx = 0;
    pending = 0;
    LS_CUDA(cudaMemcpyAsync(d_tok, h_tok, T * 4, cudaMemcpyHostToDevice, stream));
    LS_CUDA(cudaMemcpyAsync(d_pos0, h_pos0, ns * 4, cudaMemcpyHostToDevice, stream));
    LS_CUDA(cudaMemsetAsync(d_err, 0, 4, stream));
    if (streamed) {
      launch_embed_raw_tokens(m->host_embed_dev, c.embed_row_bytes(), c.embed_format.bits, c.embed_format.group, d_tok, x, h,
                              (int)c.vocab, (int)T, d_err, stream);
      m->bytes_read += T * c.embed_row_bytes();  // streamed passes are never graphed
    } else {
      launch_embed_tokens(m->embed, d_tok, (int)T, x, h, (int)c.vocab, d_err, stream);
    }
    const size_t span = for_graph ? max_ctx : maxpos + M;  // positions the attention may see
    const int slots = (int)std::max<size_t>(1, std::min<size_t>(16, (span + 63) / 64));
    const int pp = prof_begin(7, 0);
    double kv_rows = 0;  // cached + new positions of the pass's sequences (K/V rows per layer)
    for (size_t i = 0; i < ns; i++) kv_rows += (double)pos[s0 + i] + M;
    const double act = (double)T * 4;
    auto layer_fn = [&](const LayerW& W, size_t l) {
      int pi = prof_begin(0, qbytes(W.qkv) + act * (h + QS));
      if (use_bg) {
        prep_x((int)T, W.in_norm, nullptr);
        bg(W.qkv, bt_a, (int)T, EPI_BIAS_STORE, qkv, QS, nullptr, W.qkv_bias);
      } else {
        gemv(W.qkv, x, h, (int)T, EPI_BIAS_STORE, qkv, QS, W.in_norm, W.qkv_bias);
      }
      prof_end(pi);
      pi = prof_begin(1, kv_rows * kv * 2 * 2 + act * (QS + dm.q_dim));
      AttnLaunch a;
      a.qkv = qkv;
      a.qkv_stride = QS;
      a.k_cache = kc + l * kv_layer;
      a.v_cache = vc + l * kv_layer;
      a.pages = pool.d_table + s0 * pool.max_pages;
      a.page_shift = pool.shift;
      a.num_pages = pool.num_pages;
      a.max_pages = pool.max_pages;
      a.rope = rope;
      a.out = attn;
      a.part = att_part;
      a.tickets = att_tickets;
      a.heads = dm.heads;
      a.kv_heads = dm.kv_heads;
      a.hd = (int)c.head_dim;
      a.max_ctx = (int)max_ctx;
      a.M = M;
      a.max_splits = slots;
      a.nseq = (int)ns;
      a.pos0 = d_pos0;
      a.pdl = use_bg;  // positions come from the pass's host upload, before every kernel
      a.err = d_err;
      a.max_total = (int)span;
      if (use_bg && attention_tc_supported(a)) {  // straight into the O GEMM's operand
        int gn = 16, gg = 1;
        bgemm_groups((int)T, &gn, &gg);
        a.out_h = bt_a;
        a.out_h_n = gn;
      }
      launch_attention(a, stream);
      if (use_bg && !a.out_h) launch_bt_prep(attn, dm.q_dim, (int)T, dm.q_dim, nullptr, nullptr, 0.f, bt_a, stream);
      prof_end(pi);
      pi = prof_begin(2, qbytes(W.o) + act * (dm.q_dim + 2 * h));
      if (use_bg) {
        if (tp) {
          bg(W.o, bt_a, (int)T, EPI_STORE, ycur(), h, nullptr, nullptr);
          prof_end(pi);
          reduce_into_x(T * h);
        } else {
          bg(W.o, bt_a, (int)T, EPI_RESID, x, h, nullptr, nullptr);
          prof_end(pi);
        }
        pi = prof_begin(3, qbytes(W.gu) + act * (h + I));
        prep_x((int)T, W.post_norm, nullptr);
        bg(W.gu, bt_a, (int)T, EPI_SWIGLU_H, nullptr, 0, bt_h, nullptr);
        prof_end(pi);
        pi = prof_begin(4, qbytes(W.down) + act * (I + 2 * h));
        if (tp) {
          bg(W.down, bt_h, (int)T, EPI_STORE, ycur(), h, nullptr, nullptr);
          prof_end(pi);
          reduce_into_x(T * h);
        } else {
          bg(W.down, bt_h, (int)T, EPI_RESID, x, h, nullptr, nullptr);
          prof_end(pi);
        }
        return;
      }
      if (tp) {  // row-parallel O: this rank's heads' share of every output, summed over the ranks
        gemv(W.o, attn, dm.q_dim, (int)T, EPI_STORE, ycur(), h, nullptr, nullptr);
        prof_end(pi);
        reduce_into_x(T * h);
      } else {
        gemv(W.o, attn, dm.q_dim, (int)T, EPI_RESID, x, h, nullptr, nullptr);
        prof_end(pi);
      }
      pi = prof_begin(3, qbytes(W.gu) + act * (h + I));
      gemv(W.gu, x, h, (int)T, EPI_SWIGLU, hbuf, I, W.post_norm, nullptr);
      prof_end(pi);
      pi = prof_begin(4, qbytes(W.down) + act * (I + 2 * h));
      if (tp) {  // row-parallel down over this rank's intermediate slice
        gemv(W.down, hbuf, I, (int)T, EPI_STORE, ycur(), h, nullptr, nullptr);
        prof_end(pi);
        reduce_into_x(T * h);
      } else {
        gemv(W.down, hbuf, I, (int)T, EPI_RESID, x, h, nullptr, nullptr);
        prof_end(pi);
      }
    };
    // head over all T rows (verify) or the last row (prefill end)
    // head rows: every row (verify) or the last row of every sequence (end of a prefill)
    const float* hx = head_mode == 2 ? x + (size_t)(M - 1) * h : x;
    const int hstride = head_mode == 2 ? M * h : h;
    const int hM = head_mode == 2 ? (int)ns : (int)T;
    int nparts = 0;
    auto head_fn = [&](const QMat& w, int first, int rows) {
      const int pi = prof_begin(5, qbytes(w) + (double)hM * h * 4);
      if (use_bg) {
        if (nparts == 0) {
          if (hx == x && hstride == h && hM == (int)T) {
            prep_x(hM, nullptr, m->final_norm);  // with the last layer's pending reduction, if any
          } else {
            flush_reduce();
            launch_bt_prep(hx, hstride, hM, h, nullptr, m->final_norm, m->cfg.eps, bt_a, stream);
          }
        }
        nparts += bg_head(w, first, rows, hM, nparts);
      } else {
        flush_reduce();
        nparts += head(w, first, rows, hx, hstride, hM, nparts);
      }
      prof_end(pi);
    };
    if (streamed) {
      m->stream_weights(head_mode != 0, stream, layer_fn, head_fn);
    } else {
      for (size_t l = 0; l < c.layers; l++) layer_fn(layer(l), l);
      if (head_mode) {
        if (tp) head_fn(tp_head, tp_v0, tp_head.rows);
        else head_fn(m->embed, 0, (int)c.vocab);
      }
    }
    flush_reduce();  // a pass without a head still completes x (and every rank the same reductions)
    if (red_idx & 1) LS_THROW(LS_ERR_ARG, "internal: a pass made an odd number of peer reductions");
    const ArgPart* fparts = parts;
    int fnparts = nparts;
    if (tp && head_mode) {
      // vocabulary-parallel head: each rank's first maximum per row (global ids), gathered from
      // every rank, then reduced with the same first-maximum rule: identical on all ranks
      launch_row_best(parts, nparts, hM, tp_best, stream);
      const int pi = prof_begin(6, (double)hM * 8 * (tp_world - 1));
      nccl_check(nccl_api().all_gather(tp_best, tp_all, (size_t)hM * 2, ncclUint32, comm, stream), "ncclAllGather");
      prof_end(pi);
      fparts = tp_all;
      fnparts = tp_world;
    }
    if (head_mode == 1) launch_batch_accept(fparts, fnparts, (int)T, M, d_tok, d_argmax, d_m, d_next, stream);
    else if (head_mode == 2) launch_batch_accept(fparts, fnparts, hM, 1, d_tok, d_argmax, d_m, d_next, stream);
    if (head_mode) {
      const size_t nres = ns;
      LS_CUDA(cudaMemcpyAsync(h_m, d_m, nres * 4, cudaMemcpyDeviceToHost, stream));
      LS_CUDA(cudaMemcpyAsync(h_next, d_next, nres * 4, cudaMemcpyDeviceToHost, stream));
    }
    prof_end(pp);
    if (inject_err) {  // never captured: an injected pass runs eagerly
      *h_err = inject_err;
      LS_CUDA(cudaMemcpyAsync(d_err, h_err, 4, cudaMemcpyHostToDevice, stream));
      LS_CUDA(cudaStreamSynchronize(stream));
    }
    // tensor parallel: every rank must see every rank's error, so that all of them stop on the same
    // pass (a rank that went on would wait in its next collective for a peer that has stopped)
    if (tp) nccl_check(nccl_api().all_reduce(d_err, d_err, 1, ncclInt32, ncclMax, comm, stream), "ncclAllReduce (error)");
    LS_CUDA(cudaMemcpyAsync(h_err, d_err, 4, cudaMemcpyDeviceToHost, stream));
    };
    if (graphed) {
      auto it = bgraphs.find(M);
      if (it == bgraphs.end()) {
        cudaGraph_t graph;
        LS_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        try {
          enqueue(true);
        } catch (...) {
          cudaStreamEndCapture(stream, &graph);
          throw;
        }
        LS_CUDA(cudaStreamEndCapture(stream, &graph));
        cudaGraphExec_t exec;
        LS_CUDA(cudaGraphInstantiate(&exec, graph, 0));
        cudaGraphDestroy(graph);
        it = bgraphs.emplace(M, exec).first;
      }
      LS_CUDA(cudaGraphLaunch(it->second, stream));
    } else {
      enqueue(false);
    }
    if (head_mode) d2h_bytes += 2 * ns * 4;
    LS_CUDA(cudaStreamSynchronize(stream));
    if (prof_on) prof_collect();
    if (m->mode != LS_MODE_RESIDENT) m->sealed_check();
    passes++;
    inject_err = 0;
    if (*h_err) tp_failed = tp;
    if (*h_err == 1) LS_THROW(LS_ERR_DEVICE, "a tensor-core kernel gave up waiting on an mbarrier (bounded wait)");
    if (*h_err == 4) LS_THROW(LS_ERR_DEVICE, "a pass reported an injected error (test hook)");
    if (*h_err == 5) LS_THROW(LS_ERR_DEVICE, "a peer rank did not answer the tensor-parallel reduction in time (bounded wait)");
    if (*h_err) LS_THROW(LS_ERR_DEVICE, "a kernel rejected a token id outside the vocabulary");
    for (size_t i = 0; i < ns; i++) set_pos(s0 + i, pos[s0 + i] + (head_mode == 1 ? h_m[i] + 1 : (uint64_t)M));
  }

  // src/model.rs:111-119 for one sequence: 128-token chunks; returns the greedy token after them.
  uint32_t prefill(size_t sq, const uint32_t* ids, uint64_t n) {
    if (sq >= B) LS_THROW(LS_ERR_ARG, "sequence index out of range");
    if (n == 0) LS_THROW(LS_ERR_ARG, "no tokens to process");
    if (pos[sq] + n > max_ctx) LS_THROW(LS_ERR_ARG, "context is full");
    for (uint64_t off = 0; off < n; off += kPrefillChunk) {
      const uint64_t len = std::min<uint64_t>(kPrefillChunk, n - off);
      pass(sq, 1, (int)len, ids + off, off + len == n ? 2 : 0);
    }
    return h_next[0];
  }

  // Every sequence's prompt from position 0 (src/model.rs:111-119 per sequence: 128-token chunks):
  // chunk i of up to kPrefillSeqs sequences runs as one pass; returns each sequence's greedy token
  // after its prompt.
  std::vector<uint32_t> prefill_all(const uint32_t* prompts, uint64_t plen) {
    if (plen == 0) LS_THROW(LS_ERR_ARG, "no tokens to process");
    std::vector<uint32_t> firsts(B), chunk;
    for (size_t s0 = 0; s0 < B; s0 += kPrefillSeqs) {
      const size_t ns = std::min<size_t>(kPrefillSeqs, B - s0);
      for (size_t i = 0; i < ns; i++)
        if (pos[s0 + i] + plen > max_ctx) LS_THROW(LS_ERR_ARG, "context is full");
      for (uint64_t off = 0; off < plen; off += kPrefillChunk) {
        const uint64_t len = std::min<uint64_t>(kPrefillChunk, plen - off);
        chunk.resize(ns * len);
        for (size_t i = 0; i < ns; i++) std::memcpy(chunk.data() + i * len, prompts + (s0 + i) * plen + off, len * 4);
        pass(s0, ns, (int)len, chunk.data(), off + len == plen ? 2 : 0);
      }
      for (size_t i = 0; i < ns; i++) firsts[s0 + i] = h_next[i];
    }
    return firsts;
  }

  // The decode loop of src/spec.rs:94-149 for every sequence, with the prompt-lookup drafter; all
  // sequences verify one k+1 block per pass (a sequence that has finished stays in the pass at a
  // frozen position, its results ignored).
  void spec(const uint32_t* prompts, uint64_t plen, uint64_t max_new, uint64_t k, const uint32_t* eos, uint64_t neos,
            uint32_t* out, uint64_t* out_len, LsSpecStats* st) {
    if (k == 0 || k + 1 > max_block) LS_THROW(LS_ERR_ARG, "k must be between 1 and the batch's block length - 1");
    if (plen == 0 || max_new == 0) LS_THROW(LS_ERR_ARG, "need a prompt and at least one token to generate");
    if (plen + max_new + k + 1 > max_ctx) LS_THROW(LS_ERR_ARG, "prompt + max_new + k exceeds the batch's context");
    std::memset(st, 0, sizeof *st);
    for (size_t sq = 0; sq < B; sq++) set_pos(sq, 0);
    const double t0 = now_s();
    std::vector<std::vector<uint32_t>> outs(B), hist(B);
    std::vector<char> active(B, 1);
    std::vector<uint32_t> firsts = prefill_all(prompts, plen);
    for (size_t sq = 0; sq < B; sq++) {
      const uint32_t* p = prompts + sq * plen;
      const uint32_t a = firsts[sq];
      outs[sq].push_back(a);
      hist[sq].assign(p, p + plen);
      hist[sq].push_back(a);
      if (contains(eos, neos, a) || max_new == 1) active[sq] = 0;
    }
    st->first_secs = now_s() - t0;
    const double td = now_s();
    const int M = (int)k + 1;
    std::vector<uint32_t> blocks(B * M);
    std::vector<std::vector<uint32_t>> drafts(B);
    std::vector<uint64_t> frozen(B);
    while (std::find(active.begin(), active.end(), 1) != active.end()) {
      const double ts = now_s();
      for (size_t sq = 0; sq < B; sq++) {
        const uint32_t a = outs[sq].back();
        drafts[sq] = active[sq] ? lookup_draft(hist[sq], k) : std::vector<uint32_t>();
        uint32_t* blk = blocks.data() + sq * M;
        blk[0] = a;
        for (int i = 1; i < M; i++) blk[i] = (size_t)(i - 1) < drafts[sq].size() ? drafts[sq][i - 1] : (i > 1 ? blk[i - 1] : a);
        frozen[sq] = pos[sq];
      }
      st->draft_secs += now_s() - ts;
      const double tv = now_s();
      pass(0, B, M, blocks.data(), 1);
      st->target_secs += now_s() - tv;
      st->target_passes++;
      for (size_t sq = 0; sq < B; sq++) {
        if (!active[sq]) {
          set_pos(sq, frozen[sq]);
          continue;
        }
        const uint32_t mm = h_m[sq], next = h_next[sq];
        const uint32_t* blk = blocks.data() + sq * M;
        st->drafted += drafts[sq].size();
        st->accepted += std::min<uint64_t>(mm, drafts[sq].size());
        for (uint32_t i = 0; i <= mm; i++) {
          const uint32_t tok = i < mm ? blk[i + 1] : next;
          outs[sq].push_back(tok);
          hist[sq].push_back(tok);
          if (contains(eos, neos, tok) || outs[sq].size() == max_new) {
            active[sq] = 0;
            break;
          }
        }
      }
    }
    st->decode_secs = now_s() - td;
    for (size_t sq = 0; sq < B; sq++) {
      out_len[sq] = outs[sq].size();
      std::memset(out + sq * max_new, 0, max_new * 4);
      std::memcpy(out + sq * max_new, outs[sq].data(), outs[sq].size() * 4);
    }
  }
};

// ------------------------------------------------------------------------------------------------
// Quantizer (src/quant.rs:158-251): the group quantization runs on the GPU, the file layout on the host
// ------------------------------------------------------------------------------------------------

static double quantize_model(const char* src_dir, const char* out_path, WeightFormat fmt, WeightFormat efmt, int clip, int dev) {
  if (!fmt.quant()) LS_THROW(LS_ERR_ARG, "quantize needs a quantized target format");
  if (!efmt.quant()) LS_THROW(LS_ERR_ARG, "the embedding table needs a quantized format too");
  LS_CUDA(cudaSetDevice(dev));
  SafetensorsModel src = SafetensorsModel::open(src_dir);
  if (src.cfg.format.quant()) LS_THROW(LS_ERR_ARG, "the source model is already quantized");
  const std::string qtext = inject_quant(src.config_text, fmt, efmt);
  const Config q = parse_config(qtext);
  const LayerLayout dst = layer_layout_for(q);
  const size_t rb_out = q.embed_row_bytes(), rb_in = src.cfg.hidden * 2;
  int ofd = ::open(out_path, O_WRONLY | O_CREAT | O_EXCL, 0644);
  if (ofd < 0) LS_THROW(LS_ERR_IO, std::string(out_path) + ": cannot create (it must not exist already)");
  int ifd = ::open(src.file.c_str(), O_RDONLY);
  if (ifd < 0) {
    ::close(ofd);
    LS_THROW(LS_ERR_IO, src.file + ": cannot open");
  }
  cudaStream_t s;
  LS_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  const size_t erows = std::min<size_t>(kHeadRows, q.vocab);
  const size_t in_max = std::max(src.layout.total, erows * rb_in), out_max = std::max(dst.total, erows * rb_out);
  uint8_t *din = nullptr, *dout = nullptr;
  double* den = nullptr;
  std::vector<uint8_t> hin(in_max), hout(out_max);
  double result = 0;
  try {
    LS_CUDA(cudaMalloc(&din, in_max));
    LS_CUDA(cudaMalloc(&dout, out_max));
    LS_CUDA(cudaMalloc(&den, 16));
    LS_CUDA(cudaMemsetAsync(den, 0, 16, s));
    auto wr = [&](const void* p, size_t n) {
      const char* b = (const char*)p;
      while (n) {
        ssize_t w = ::write(ofd, b, n);
        if (w <= 0) LS_THROW(LS_ERR_IO, "write failed");
        b += w;
        n -= (size_t)w;
      }
    };
    const std::string hb = lsq_header_bytes(qtext, dst.total, q.vocab * rb_out, q.hidden * 2);
    wr(hb.data(), hb.size());
    for (size_t l = 0; l < q.layers; l++) {
      pread_all(ifd, hin.data(), src.layout.total, src.layer_start[l]);
      LS_CUDA(cudaMemcpyAsync(din, hin.data(), src.layout.total, cudaMemcpyHostToDevice, s));
      for (int sl = 0; sl < N_SLOTS; sl++) {
        size_t rows, cols;
        if (matrix_shape(sl, q, &rows, &cols))
          launch_quantize_rows(reinterpret_cast<const uint16_t*>(din + src.layout.off[sl]), (int)rows, (int)cols, fmt.bits,
                               fmt.group, clip, dout + dst.off[sl], den, s);
      }
      LS_CUDA(cudaMemcpyAsync(hout.data(), dout, dst.total, cudaMemcpyDeviceToHost, s));
      LS_CUDA(cudaStreamSynchronize(s));
      for (int sl = 0; sl < N_SLOTS; sl++) {
        size_t rows, cols;
        if (!matrix_shape(sl, q, &rows, &cols)) std::memcpy(hout.data() + dst.off[sl], hin.data() + src.layout.off[sl], dst.len[sl]);
      }
      wr(hout.data(), dst.total);
    }
    for (size_t first = 0; first < q.vocab; first += erows) {
      const size_t n = std::min(erows, q.vocab - first);
      pread_all(ifd, hin.data(), n * rb_in, src.embed_start + first * rb_in);
      LS_CUDA(cudaMemcpyAsync(din, hin.data(), n * rb_in, cudaMemcpyHostToDevice, s));
      launch_quantize_rows(reinterpret_cast<const uint16_t*>(din), (int)n, (int)q.hidden, efmt.bits, efmt.group, clip, dout, den, s);
      LS_CUDA(cudaMemcpyAsync(hout.data(), dout, n * rb_out, cudaMemcpyDeviceToHost, s));
      LS_CUDA(cudaStreamSynchronize(s));
      wr(hout.data(), n * rb_out);
    }
    std::vector<uint8_t> nb(src.norm_len);
    pread_all(ifd, nb.data(), nb.size(), src.norm_start);
    wr(nb.data(), nb.size());
    double en[2];
    LS_CUDA(cudaMemcpy(en, den, 16, cudaMemcpyDeviceToHost));
    result = en[1] > 0 ? std::sqrt(en[0] / en[1]) : 0.0;
  } catch (...) {
    cudaFree(din);
    cudaFree(dout);
    cudaFree(den);
    cudaStreamDestroy(s);
    ::close(ifd);
    ::close(ofd);
    ::unlink(out_path);
    throw;
  }
  cudaFree(din);
  cudaFree(dout);
  cudaFree(den);
  cudaStreamDestroy(s);
  ::close(ifd);
  if (::close(ofd) != 0) LS_THROW(LS_ERR_IO, "close failed");
  return result;
}

// ------------------------------------------------------------------------------------------------
// Kernel-level GEMV entry points
// ------------------------------------------------------------------------------------------------

struct LsQWeights {
  int device = 0;
  QMat w;
  void* mem = nullptr;
  float* partial = nullptr;
  unsigned* tickets = nullptr;
  int* err = nullptr;
  int num_sms = 148;
  ~LsQWeights() {
    cudaFree(mem);
    cudaFree(partial);
    cudaFree(tickets);
    cudaFree(err);
  }
};

static void qweights_upload(LsQWeights* q, int dev, int bits, int group, const uint8_t* raw, uint64_t rows, uint64_t cols) {
  WeightFormat f;
  f.bits = bits;
  f.group = group;
  if (bits == 16) {  // bf16 rows: no groups
    if (cols % 64) LS_THROW(LS_ERR_ARG, "bf16 rows need a multiple of 64 columns");
    f.group = group = 0;
  } else if ((bits != 8 && bits != 4) || group < 16 || group > 256 || (group & (group - 1)) || cols % (uint64_t)group || cols % 32) {
    LS_THROW(LS_ERR_ARG, "unsupported GEMV format or shape");
  }
  q->device = dev;
  LS_CUDA(cudaSetDevice(dev));
  LS_CUDA(cudaDeviceGetAttribute(&q->num_sms, cudaDevAttrMultiProcessorCount, dev));
  const size_t bytes = qmat_bytes((int)rows, (int)cols, f);
  LS_CUDA(cudaMalloc(&q->mem, bytes));
  uint8_t* p = reinterpret_cast<uint8_t*>(q->mem);
  q->w = carve(p, (int)rows, (int)cols, f);
  const size_t rb = f.row_bytes(cols);
  uint8_t* draw = nullptr;
  LS_CUDA(cudaMalloc(&draw, rows * rb));
  LS_CUDA(cudaMemcpy(draw, raw, rows * rb, cudaMemcpyHostToDevice));
  RepackSrc s;
  s.seg[0] = draw;
  s.seg_rows[0] = (int)rows;
  launch_repack(s, bits, group, (int)cols, const_cast<uint8_t*>(q->w.data), const_cast<uint16_t*>(q->w.scales), q->w.rows_pad, 0);
  LS_CUDA(cudaDeviceSynchronize());
  cudaFree(draw);
  const size_t tiles = q->w.rows_pad / 32;
  LS_CUDA(cudaMalloc(&q->partial, tiles * 32 * 16 * 32 * 4 * 3));
  LS_CUDA(cudaMalloc(&q->tickets, tiles * 4 * 3));
  LS_CUDA(cudaMemset(q->tickets, 0, tiles * 4 * 3));
  LS_CUDA(cudaMalloc(&q->err, sizeof(int)));
  LS_CUDA(cudaMemset(q->err, 0, sizeof(int)));
}

static void qgemv_device(const LsQWeights* q, const float* x, uint64_t M, float* y, cudaStream_t s) {
  if (M == 0 || M > 48) LS_THROW(LS_ERR_ARG, "the GEMV takes 1..48 token rows");
  GemvLaunch g;
  g.w = q->w;
  g.x = x;
  g.x_stride = q->w.cols;
  g.M = (int)M;
  g.epi = EPI_STORE;
  g.y = y;
  g.y_stride = q->w.rows;
  g.partial = q->partial;
  g.tickets = q->tickets;
  g.err = q->err;
  if (use_tc(q->w)) {
    choose_tc(q->w, (int)M, q->num_sms, false, &g.ksplit, &g.grid_x);
    launch_gemv_tc(g, s);
    return;
  }
  g.ksplit = choose_ksplit(q->w, (int)M, q->num_sms);
  g.grid_x = gemv_grid_x(q->w, g.ksplit, (int)M, q->num_sms);
  launch_gemv(g, s);
}

static void qweights_check(const LsQWeights* q) {
  int e = 0;
  LS_CUDA(cudaMemcpy(&e, q->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) LS_THROW(LS_ERR_DEVICE, "a tensor-core kernel gave up waiting on an mbarrier (bounded wait)");
}

// ------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------

template <class F>
static int guard(F&& f) {
  try {
    f();
    return LS_OK;
  } catch (const ls::Error& e) {
    g_err = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_err = e.what();
    return LS_ERR_ARG;
  }
}

#define NEED(p)                                                  \
  do {                                                           \
    if (!(p)) LS_THROW(LS_ERR_ARG, #p " must not be NULL");      \
  } while (0)

extern "C" {

int ls_last_error(char* buf, size_t cap) {
  if (buf && cap) std::snprintf(buf, cap, "%s", g_err.c_str());
  return (int)g_err.size();
}

int ls_model_open(const char* path, int device, uint64_t max_ctx, int mode, int slots, LsModel** out) {
  return guard([&] {
    NEED(path);
    NEED(out);
    *out = nullptr;
    std::unique_ptr<LsModel> m(new LsModel);
    m->open(path, device, max_ctx, mode, slots);
    *out = m.release();
  });
}

int ls_model_open_sealed(const char* path, const uint8_t* key, int device, uint64_t max_ctx, int mode, int slots, LsModel** out) {
  return guard([&] {
    NEED(path);
    NEED(key);
    NEED(out);
    *out = nullptr;
    if (!is_sealed_file(path)) LS_THROW(LS_ERR_IO, std::string(path) + ": not a sealed layerstream model (bad magic bytes)");
    std::unique_ptr<LsModel> m(new LsModel);
    m->open(path, device, max_ctx, mode, slots, key);
    *out = m.release();
  });
}

int ls_seal_model(const char* src, const char* out_path, const uint8_t* key, const uint8_t* nonce_prefix, uint64_t layer_chunk,
                  uint64_t embed_chunk_rows, int device, uint64_t* n_chunks) {
  return guard([&] {
    NEED(src);
    NEED(out_path);
    NEED(key);
    NEED(nonce_prefix);
    LS_CUDA(cudaSetDevice(device));
    const size_t n = seal_model_file(src, out_path, key, nonce_prefix, layer_chunk, embed_chunk_rows);
    if (n_chunks) *n_chunks = n;
  });
}

int ls_model_free(LsModel* m) {
  return guard([&] { delete m; });
}

int ls_model_info(const LsModel* m, LsModelInfo* o) {
  return guard([&] {
    NEED(m);
    NEED(o);
    const Config& c = m->cfg;
    o->hidden = c.hidden;
    o->inter = c.inter;
    o->layers = c.layers;
    o->heads = c.heads;
    o->kv_heads = c.kv_heads;
    o->head_dim = c.head_dim;
    o->vocab = c.vocab;
    o->max_ctx = m->max_ctx;
    o->bits = c.format.bits;
    o->group = c.format.group;
    o->embed_bits = c.embed_format.bits;
    o->embed_group = c.embed_format.group;
    o->eps = c.eps;
    o->rope_theta = c.rope_theta;
    o->layer_bytes = m->file.layout.total;
    o->embed_row_bytes = c.embed_row_bytes();
    o->weight_bytes = c.layers * m->file.layout.total + c.vocab * c.embed_row_bytes();
    o->persistent_pass = m->pk_max_grid > 0 ? 1 : 0;
    o->kv_page = m->pool.page();
    o->kv_pages_total = (uint64_t)m->pool.num_pages;
    o->kv_pages_used = (uint64_t)m->pool.used();
  });
}

int ls_model_report(const LsModel* m, LsReport* o) {
  return guard([&] {
    NEED(m);
    NEED(o);
    o->resident_weight_bytes = m->resident_weight_bytes;
    o->bytes_read = m->bytes_read;
    o->wait_ns = m->wait_ns;
    o->passes = m->passes;
    o->h2d_bytes = m->h2d_bytes;
    o->d2h_bytes = m->d2h_bytes;
  });
}

int ls_model_stream(const LsModel* m, void** stream) {
  return guard([&] {
    NEED(m);
    NEED(stream);
    *stream = reinterpret_cast<void*>(m->stream);
  });
}

int ls_model_profile_enable(LsModel* m, int on) {
  return guard([&] {
    NEED(m);
    m->prof_on = on != 0;
    m->prof_timeline = on >= 2;
    m->prof = LsProfile{};
    m->prof_pending = false;
  });
}

int ls_model_profile(const LsModel* m, LsProfile* out) {
  return guard([&] {
    NEED(m);
    NEED(out);
    *out = m->prof;
  });
}

int ls_pos(const LsModel* m, uint64_t* pos) {
  return guard([&] {
    NEED(m);
    NEED(pos);
    *pos = m->pos;
  });
}

int ls_reset(LsModel* m) {
  return guard([&] {
    NEED(m);
    m->pos = 0;
    m->pool.shrink(0, 0);
  });
}

int ls_truncate(LsModel* m, uint64_t pos) {
  return guard([&] {
    NEED(m);
    m->truncate(pos);
  });
}

int ls_forward(LsModel* m, const uint32_t* ids, uint64_t n, float* logits, uint32_t* argmax) {
  return guard([&] {
    NEED(m);
    if (n) NEED(ids);
    LS_CUDA(cudaSetDevice(m->device));
    uint32_t t = m->forward(ids, n, logits);
    if (argmax) *argmax = t;
  });
}

int ls_forward_multi(LsModel* m, const uint32_t* ids, uint64_t t, uint64_t n, float* logits) {
  return guard([&] {
    NEED(m);
    if (t) NEED(ids);
    LS_CUDA(cudaSetDevice(m->device));
    m->forward_multi(ids, t, n, logits);
  });
}

int ls_verify(LsModel* m, const uint32_t* block, uint64_t n, uint32_t* accepted_m, uint32_t* next) {
  return guard([&] {
    NEED(m);
    NEED(accepted_m);
    NEED(next);
    if (n) NEED(block);
    LS_CUDA(cudaSetDevice(m->device));
    m->verify(block, n, accepted_m, next);
  });
}

int ls_speculative_greedy(LsModel* target, LsModel* draft, const uint32_t* prompt, uint64_t plen, uint64_t max_new, uint64_t k,
                          const uint32_t* eos, uint64_t neos, uint32_t* out_tokens, uint64_t* out_len, LsSpecStats* stats) {
  return guard([&] {
    NEED(target);
    NEED(out_tokens);
    NEED(out_len);
    NEED(stats);
    if (plen) NEED(prompt);
    if (neos) NEED(eos);
    LS_CUDA(cudaSetDevice(target->device));
    speculative_greedy(*target, draft, prompt, plen, max_new, k, eos, neos, out_tokens, out_len, stats);
  });
}

int ls_spec_continue(LsModel* target, LsModel* draft, const uint32_t* hist, uint64_t hlen, uint32_t first, uint64_t max_new,
                     uint64_t k, const uint32_t* eos, uint64_t neos, uint32_t* out_tokens, uint64_t* out_len, LsSpecStats* stats) {
  return guard([&] {
    NEED(target);
    NEED(out_tokens);
    NEED(out_len);
    NEED(stats);
    if (hlen) NEED(hist);
    if (neos) NEED(eos);
    LS_CUDA(cudaSetDevice(target->device));
    std::memset(stats, 0, sizeof *stats);
    spec_continue(*target, draft, hist, hlen, first, max_new, k, eos, neos, out_tokens, out_len, stats);
  });
}

int ls_quantize_model(const char* src_dir, const char* out_path, int bits, int group, int embed_bits, int embed_group,
                      int clip_search, int device, double* rel_rmse) {
  return guard([&] {
    NEED(src_dir);
    NEED(out_path);
    WeightFormat f, e;
    f.bits = bits;
    f.group = group;
    e.bits = embed_bits;
    e.group = embed_group;
    double r = quantize_model(src_dir, out_path, f, e, clip_search, device);
    if (rel_rmse) *rel_rmse = r;
  });
}

int ls_qweights_upload(int device, int bits, int group, const uint8_t* rows_raw, uint64_t rows, uint64_t cols, LsQWeights** out) {
  return guard([&] {
    NEED(rows_raw);
    NEED(out);
    std::unique_ptr<LsQWeights> q(new LsQWeights);
    qweights_upload(q.get(), device, bits, group, rows_raw, rows, cols);
    *out = q.release();
  });
}

int ls_qweights_free(LsQWeights* w) {
  return guard([&] { delete w; });
}

int ls_qgemv_device(const LsQWeights* w, const float* x_dev, uint64_t M, float* y_dev, void* stream) {
  return guard([&] {
    NEED(w);
    NEED(x_dev);
    NEED(y_dev);
    LS_CUDA(cudaSetDevice(w->device));
    qgemv_device(w, x_dev, M, y_dev, reinterpret_cast<cudaStream_t>(stream));
  });
}

int ls_aead_host(int seal, const uint8_t* key, const uint8_t* nonce, const uint8_t* aad, uint64_t aad_len, uint8_t* data,
                 uint64_t len, uint64_t chunk_bytes, uint32_t first, uint8_t* tags, int iters, double* ms, int64_t* bad_chunk) {
  return guard([&] {
    NEED(key);
    NEED(nonce);
    NEED(tags);
    if (len && !data) LS_THROW(LS_ERR_ARG, "data must not be NULL");
    if (aad_len && !aad) LS_THROW(LS_ERR_ARG, "aad must not be NULL");
    const int bad = aead_host(seal != 0, key, nonce, chunk_bytes != 0, first, aad, aad_len, data, len, chunk_bytes, tags, iters, ms);
    if (bad_chunk) *bad_chunk = bad;
    if (bad >= 0) LS_THROW(LS_ERR_IO, "authentication failed for chunk " + std::to_string(bad) + ": wrong key, or the data was modified");
  });
}

int ls_tp_reduce_host(const float* x, const float* ys, uint32_t world, uint32_t rank, uint64_t n, int preset, uint32_t wait_ms,
                      int calls, float* x_out, int* status, double* ms, uint32_t K, const float* norm, float eps, uint16_t* op_out) {
  return guard([&] {
    NEED(x);
    NEED(ys);
    NEED(x_out);
    const int e = tp_reduce_host(x, ys, (int)world, (int)rank, n, preset != 0, wait_ms, calls, x_out, ms, K, norm, eps, op_out);
    if (status) *status = e;
    if (e == 5) LS_THROW(LS_ERR_DEVICE, "a peer rank did not answer the tensor-parallel reduction in time (bounded wait)");
    if (e) LS_THROW(LS_ERR_DEVICE, "peer reduction: error " + std::to_string(e));
  });
}

int ls_qgemv_rows_noalloc(int bits, int group, const uint8_t* rows_dev, uint64_t rows, uint64_t cols, const float* x_dev,
                          uint64_t M, float* y_dev, void* stream) {
  return guard([&] { qgemv_rows_noalloc(bits, group, rows_dev, rows, cols, x_dev, M, y_dev, reinterpret_cast<cudaStream_t>(stream)); });
}

int ls_batch_open(LsModel* m, uint64_t batch, uint64_t max_ctx, uint64_t max_block, LsBatch** out) {
  return guard([&] {
    NEED(m);
    NEED(out);
    *out = nullptr;
    LS_CUDA(cudaSetDevice(m->device));
    *out = new LsBatch(m, batch, max_ctx, max_block);
  });
}

int ls_tp_unique_id(uint8_t* out, size_t cap) {
  return guard([&] {
    NEED(out);
    if (cap < sizeof(ncclUniqueId)) LS_THROW(LS_ERR_ARG, "the id needs " + std::to_string(sizeof(ncclUniqueId)) + " bytes");
    ncclUniqueId id;
    nccl_check(nccl_api().get_unique_id(&id), "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof id);
  });
}

int ls_batch_open_tp(LsModel* m, uint64_t batch, uint64_t max_ctx, uint64_t max_block, int rank, int world, const uint8_t* id,
                     LsBatch** out) {
  return guard([&] {
    NEED(m);
    NEED(out);
    *out = nullptr;
    if (world > 1) NEED(id);
    LS_CUDA(cudaSetDevice(m->device));
    *out = new LsBatch(m, batch, max_ctx, max_block, rank, world, id);
  });
}

int ls_batch_free(LsBatch* b) {
  delete b;
  return LS_OK;
}

int ls_batch_pos(const LsBatch* b, uint64_t seq, uint64_t* pos) {
  return guard([&] {
    NEED(b);
    NEED(pos);
    if (seq >= b->B) LS_THROW(LS_ERR_ARG, "sequence index out of range");
    *pos = b->pos[seq];
  });
}

int ls_batch_truncate(LsBatch* b, uint64_t seq, uint64_t pos) {
  return guard([&] {
    NEED(b);
    if (seq >= b->B) LS_THROW(LS_ERR_ARG, "sequence index out of range");
    if (pos > b->pos[seq]) LS_THROW(LS_ERR_ARG, "cannot truncate to a position beyond the cache");
    b->set_pos(seq, pos);
  });
}

int ls_batch_prefill(LsBatch* b, uint64_t seq, const uint32_t* ids, uint64_t n, uint32_t* argmax) {
  return guard([&] {
    NEED(b);
    NEED(ids);
    LS_CUDA(cudaSetDevice(b->m->device));
    const uint32_t a = b->prefill(seq, ids, n);
    if (argmax) *argmax = a;
  });
}

int ls_batch_verify(LsBatch* b, const uint32_t* blocks, uint64_t nseq, uint64_t M, uint32_t* accepted_m, uint32_t* next) {
  return guard([&] {
    NEED(b);
    NEED(blocks);
    NEED(accepted_m);
    NEED(next);
    if (M == 0 || M > b->max_block) LS_THROW(LS_ERR_ARG, "verify blocks hold 1..max_block tokens");
    if (nseq == 0 || nseq > b->B) LS_THROW(LS_ERR_ARG, "nseq must be in 1..batch");
    LS_CUDA(cudaSetDevice(b->m->device));
    b->pass(0, nseq, (int)M, blocks, 1);
    std::memcpy(accepted_m, b->h_m, nseq * 4);
    std::memcpy(next, b->h_next, nseq * 4);
  });
}

int ls_batch_spec(LsBatch* b, const uint32_t* prompts, uint64_t plen, uint64_t max_new, uint64_t k, const uint32_t* eos,
                  uint64_t neos, uint32_t* out_tokens, uint64_t* out_len, LsSpecStats* stats) {
  return guard([&] {
    NEED(b);
    NEED(prompts);
    NEED(out_tokens);
    NEED(out_len);
    if (neos) NEED(eos);
    LsSpecStats local;
    LS_CUDA(cudaSetDevice(b->m->device));
    b->spec(prompts, plen, max_new, k, eos, neos, out_tokens, out_len, stats ? stats : &local);
  });
}

int ls_batch_report(const LsBatch* b, uint64_t* passes, uint64_t* h2d_bytes, uint64_t* d2h_bytes) {
  return guard([&] {
    NEED(b);
    if (passes) *passes = b->passes;
    if (h2d_bytes) *h2d_bytes = b->h2d_bytes;
    if (d2h_bytes) *d2h_bytes = b->d2h_bytes;
  });
}

int ls_batch_profile_enable(LsBatch* b, int on) {
  return guard([&] {
    NEED(b);
    b->prof_on = on != 0;
    b->prof = LsBatchProfile{};
    b->prof_rec.clear();
  });
}

int ls_model_inject_stall(LsModel* m, int barrier) {
  return guard([&] {
    NEED(m);
    if (barrier < 0 || barrier > 1 + 5 * (int)m->cfg.layers + 1) LS_THROW(LS_ERR_ARG, "no such grid barrier in a pass");
    if (barrier && m->pk_max_grid == 0) LS_THROW(LS_ERR_ARG, "this model does not run the persistent pass kernel");
    m->stall_barrier = barrier;
  });
}

int ls_batch_inject_error(LsBatch* b, int code) {
  return guard([&] {
    NEED(b);
    if (code != 0 && code != 4) LS_THROW(LS_ERR_ARG, "the injected error code must be 4 (or 0 to clear)");
    b->inject_err = code;
  });
}

int ls_batch_profile(const LsBatch* b, LsBatchProfile* out) {
  return guard([&] {
    NEED(b);
    NEED(out);
    *out = b->prof;
  });
}

int ls_batch_tp_peer(const LsBatch* b, int* on) {
  return guard([&] {
    NEED(b);
    NEED(on);
    *on = b->p2p ? 1 : 0;
  });
}

namespace {

// One layer's attention through the CUDA kernels on host buffers: the cached rows live in page
// pools (k_pool, v_pool: kv_heads x num_pages x 2^page_shift x hd f16) addressed through `table`
// (the pool page of each logical page of the context); the block's rows are written to the pools,
// which are copied back when k_out / v_out are given.
void attention_host_impl(uint64_t heads, uint64_t kv_heads, uint64_t hd, float rope_theta, uint64_t pos0, uint64_t M,
                         const float* qkv, const uint16_t* k_pool, const uint16_t* v_pool, int page_shift, uint64_t num_pages,
                         const int32_t* table, float* out, int iters, double* ms, uint16_t* k_out, uint16_t* v_out) {
  if (heads == 0 || kv_heads == 0 || heads % kv_heads || heads > 256) LS_THROW(LS_ERR_ARG, "heads must be a multiple of kv_heads");
  if (hd != 16 && hd != 32 && hd != 64 && hd != 128) LS_THROW(LS_ERR_ARG, "head_dim must be 16, 32, 64 or 128");
  if (M == 0 || M > 64) LS_THROW(LS_ERR_ARG, "the attention block takes 1..64 rows");
  if (pos0 + M > (1u << 20)) LS_THROW(LS_ERR_ARG, "context beyond 2^20 positions");
  const size_t ctx = pos0 + M, KV = kv_heads * hd, H = heads * hd, QS = H + 2 * KV, page = (size_t)1 << page_shift;
  const size_t ctx_pages = (ctx + page - 1) / page;
  for (size_t i = 0; i < ctx_pages; i++)
    if (table[i] < 0 || (uint64_t)table[i] >= num_pages) LS_THROW(LS_ERR_ARG, "page table entry outside the pool");
  const size_t pool_elems = kv_heads * num_pages * page * hd;
  cudaStream_t st;
  LS_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  std::vector<void*> owned;
  auto dmalloc = [&](size_t bytes) {
    void* p = nullptr;
    LS_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 16)));
    owned.push_back(p);
    return p;
  };
  struct Cleanup {
    std::vector<void*>& o;
    cudaStream_t s;
    ~Cleanup() {
      cudaStreamSynchronize(s);
      for (void* p : o) cudaFree(p);
      cudaStreamDestroy(s);
    }
  } cleanup{owned, st};
  auto* dq = static_cast<float*>(dmalloc(M * QS * 4));
  auto* dk = static_cast<uint16_t*>(dmalloc(pool_elems * 2));
  auto* dv = static_cast<uint16_t*>(dmalloc(pool_elems * 2));
  auto* dtab = static_cast<int32_t*>(dmalloc(ctx_pages * 4));
  auto* dout = static_cast<float*>(dmalloc(M * H * 4));
  auto* drope = static_cast<float2*>(dmalloc(ctx * (hd / 2) * sizeof(float2)));
  // context splits: up to one per 128-position chunk, at most 160 (two per SM for two kv heads)
  // (the CUDA-core kernel, for head_dim 16 and 32, takes up to 16 slots of 64 positions)
  const int slots = (int)std::max<size_t>(1, std::min<size_t>(160, (ctx + 127) / 128));
  const int simt_slots = (int)std::min<size_t>(16, (ctx + 63) / 64);
  const size_t part_floats = heads * (size_t)std::max(slots, simt_slots) * M * (hd + 2);
  auto* dpart = static_cast<float*>(dmalloc(part_floats * 4));
  auto* dtick = static_cast<unsigned*>(dmalloc(heads * 4));
  auto* dctl = static_cast<Ctl*>(dmalloc(sizeof(Ctl)));
  LS_CUDA(cudaMemsetAsync(dtick, 0, heads * 4, st));
  LS_CUDA(cudaMemcpyAsync(dq, qkv, M * QS * 4, cudaMemcpyHostToDevice, st));
  LS_CUDA(cudaMemcpyAsync(dk, k_pool, pool_elems * 2, cudaMemcpyHostToDevice, st));
  LS_CUDA(cudaMemcpyAsync(dv, v_pool, pool_elems * 2, cudaMemcpyHostToDevice, st));
  LS_CUDA(cudaMemcpyAsync(dtab, table, ctx_pages * 4, cudaMemcpyHostToDevice, st));
  const std::vector<float2> tab = rope_table(rope_theta, hd, ctx);
  LS_CUDA(cudaMemcpyAsync(drope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, st));
  launch_set_ctl(dctl, (int)pos0, (int)M, 0, 0, nullptr, st);
  AttnLaunch a;
  a.qkv = dq;
  a.qkv_stride = (int)QS;
  a.k_cache = dk;
  a.v_cache = dv;
  a.pages = dtab;
  a.page_shift = page_shift;
  a.num_pages = (int)num_pages;
  a.max_pages = (int)ctx_pages;
  a.rope = drope;
  a.ctl = dctl;
  a.out = dout;
  a.part = dpart;
  a.part_floats = part_floats;
  a.tickets = dtick;
  a.heads = (int)heads;
  a.kv_heads = (int)kv_heads;
  a.hd = (int)hd;
  a.max_ctx = (int)ctx;
  a.M = (int)M;
  a.max_splits = simt_slots;
  a.max_total = (int)(pos0 + M);
  a.err = &dctl->err;
  // LS_ATT_TRACE=1 (profiling): the tensor-core kernel's per-CTA timeline of this launch, summarised
  // on stderr as the median and maximum over CTAs of each step
  const bool att_trace = getenv("LS_ATT_TRACE") != nullptr;
  const size_t trace_ctas = (size_t)160 * kv_heads * ((heads / kv_heads * M + 127) / 128);
  if (att_trace) {
    a.trace = static_cast<unsigned*>(dmalloc(trace_ctas * AT_TRACE_SLOTS * 4));
    LS_CUDA(cudaMemsetAsync(a.trace, 0, trace_ctas * AT_TRACE_SLOTS * 4, st));
  }
  launch_attention(a, st);
  if (att_trace) {
    std::vector<unsigned> tr(trace_ctas * AT_TRACE_SLOTS);
    LS_CUDA(cudaMemcpyAsync(tr.data(), a.trace, tr.size() * 4, cudaMemcpyDeviceToHost, st));
    LS_CUDA(cudaStreamSynchronize(st));
    int dev = 0, khz = 1;
    LS_CUDA(cudaGetDevice(&dev));
    LS_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev));
    const char* names[] = {"loads issued + previous kernel", "Q staged", "chunk0 loads landed", "chunk0 scores",
                           "chunk0 softmax", "chunk0 P.V + O", "chunk1 loads landed", "chunk1 scores",
                           "chunk1 softmax", "chunk1 P.V + O"};
    for (int k = 1; k <= 11; k++) {
      if (k == 11) names[0] = "partials written";
      std::vector<double> d;
      for (size_t c = 0; c < trace_ctas; c++) {
        const unsigned* t = &tr[c * AT_TRACE_SLOTS];
        int prev = k == 11 ? (t[10] ? 10 : 6) : k - 1;
        if (t[k] && t[prev]) d.push_back((double)(t[k] - t[prev]) / khz * 1e3);
      }
      if (d.empty()) continue;
      std::sort(d.begin(), d.end());
      fprintf(stderr, "attention trace %-32s ctas %4zu  median %7.3f us  max %7.3f us\n", names[k == 11 ? 0 : k - 1],
              d.size(), d[d.size() / 2], d.back());
    }
    a.trace = nullptr;
  }
  if (k_out) LS_CUDA(cudaMemcpyAsync(k_out, dk, pool_elems * 2, cudaMemcpyDeviceToHost, st));
  if (v_out) LS_CUDA(cudaMemcpyAsync(v_out, dv, pool_elems * 2, cudaMemcpyDeviceToHost, st));
  if (iters > 1) {
    // Timing: back-to-back launches (one CUDA graph, so that host launch costs stay out), each over
    // its own replica of the K/V pools, the replicas together at least 256 MB (twice L2), so that
    // every launch reads its cached rows from HBM as a layer of a pass does; ms = the events' span /
    // launches.
    const size_t pool_bytes = pool_elems * 2;
    const size_t reps = std::min<size_t>(4096, std::max<size_t>((size_t)iters, (((size_t)256 << 20) / (2 * pool_bytes)) + 1));
    auto* rk = static_cast<uint8_t*>(dmalloc(reps * pool_bytes));
    auto* rv = static_cast<uint8_t*>(dmalloc(reps * pool_bytes));
    LS_CUDA(cudaMemcpyAsync(rk, dk, pool_bytes, cudaMemcpyDeviceToDevice, st));
    LS_CUDA(cudaMemcpyAsync(rv, dv, pool_bytes, cudaMemcpyDeviceToDevice, st));
    for (size_t have = 1; have < reps;) {  // doubling copies
      const size_t n = std::min(have, reps - have);
      LS_CUDA(cudaMemcpyAsync(rk + have * pool_bytes, rk, n * pool_bytes, cudaMemcpyDeviceToDevice, st));
      LS_CUDA(cudaMemcpyAsync(rv + have * pool_bytes, rv, n * pool_bytes, cudaMemcpyDeviceToDevice, st));
      have += n;
    }
    auto launch_rep = [&](size_t i) {
      AttnLaunch r = a;
      r.k_cache = reinterpret_cast<uint16_t*>(rk + i * pool_bytes);
      r.v_cache = reinterpret_cast<uint16_t*>(rv + i * pool_bytes);
      launch_attention(r, st);
    };
    cudaGraph_t graph;
    LS_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    try {
      for (size_t i = 0; i < reps; i++) launch_rep(i);
    } catch (...) {
      cudaStreamEndCapture(st, &graph);
      throw;
    }
    LS_CUDA(cudaStreamEndCapture(st, &graph));
    cudaGraphExec_t exec;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    LS_CUDA(ie);
    struct ExecGuard {
      cudaGraphExec_t e;
      ~ExecGuard() { cudaGraphExecDestroy(e); }
    } exec_guard{exec};
    LS_CUDA(cudaGraphLaunch(exec, st));  // warm-up: every replica once
    cudaEvent_t e0, e1;
    LS_CUDA(cudaEventCreate(&e0));
    LS_CUDA(cudaEventCreate(&e1));
    LS_CUDA(cudaEventRecord(e0, st));
    LS_CUDA(cudaGraphLaunch(exec, st));
    LS_CUDA(cudaEventRecord(e1, st));
    LS_CUDA(cudaEventSynchronize(e1));
    float t = 0;
    LS_CUDA(cudaEventElapsedTime(&t, e0, e1));
    if (ms) *ms = (double)t / (double)reps;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  } else if (ms) {
    *ms = 0;
  }
  LS_CUDA(cudaMemcpyAsync(out, dout, M * H * 4, cudaMemcpyDeviceToHost, st));
  int herr = 0;
  LS_CUDA(cudaMemcpyAsync(&herr, &dctl->err, 4, cudaMemcpyDeviceToHost, st));
  LS_CUDA(cudaStreamSynchronize(st));
  if (herr == 1) LS_THROW(LS_ERR_DEVICE, "the tensor-core attention gave up waiting on an mbarrier (bounded wait)");
}

}  // namespace

int ls_attention_host(uint64_t heads, uint64_t kv_heads, uint64_t hd, float rope_theta, uint64_t pos0, uint64_t M,
                      const float* qkv, const uint16_t* k_cache, const uint16_t* v_cache, float* out, int iters, double* ms) {
  return guard([&] {
    NEED(qkv);
    NEED(out);
    if (pos0 && (!k_cache || !v_cache)) LS_THROW(LS_ERR_ARG, "k_cache and v_cache must not be NULL when pos0 > 0");
    if (kv_heads == 0 || hd == 0) LS_THROW(LS_ERR_ARG, "heads must be a multiple of kv_heads");
    // the dense cache as a pool of 64-position pages in order (the identity page table)
    const int sh = 6;
    const size_t page = (size_t)1 << sh, ctx = pos0 + M, np = (ctx + page - 1) / page;
    std::vector<uint16_t> kp(kv_heads * np * page * hd, 0), vp(kp.size(), 0);
    for (uint64_t g = 0; g < kv_heads && pos0; g++) {
      std::memcpy(kp.data() + g * np * page * hd, k_cache + g * pos0 * hd, pos0 * hd * 2);
      std::memcpy(vp.data() + g * np * page * hd, v_cache + g * pos0 * hd, pos0 * hd * 2);
    }
    std::vector<int32_t> table(np);
    for (size_t i = 0; i < np; i++) table[i] = (int32_t)i;
    attention_host_impl(heads, kv_heads, hd, rope_theta, pos0, M, qkv, kp.data(), vp.data(), sh, np, table.data(), out, iters, ms,
                        nullptr, nullptr);
  });
}

int ls_attention_paged_host(uint64_t heads, uint64_t kv_heads, uint64_t hd, float rope_theta, uint64_t pos0, uint64_t M,
                            const float* qkv, uint16_t* k_pool, uint16_t* v_pool, uint64_t num_pages, uint64_t page,
                            const int32_t* table, float* out, int iters, double* ms) {
  return guard([&] {
    NEED(qkv);
    NEED(out);
    NEED(k_pool);
    NEED(v_pool);
    NEED(table);
    int sh = 0;
    while (((uint64_t)1 << sh) < page && sh < 16) sh++;
    if (((uint64_t)1 << sh) != page || sh < 3) LS_THROW(LS_ERR_ARG, "page must be a power of two in 8..65536");
    if (num_pages == 0 || num_pages > (1u << 24)) LS_THROW(LS_ERR_ARG, "num_pages must be in 1..2^24");
    attention_host_impl(heads, kv_heads, hd, rope_theta, pos0, M, qkv, k_pool, v_pool, sh, num_pages, table, out, iters, ms,
                        k_pool, v_pool);
  });
}

int ls_qgemv_host(int bits, int group, const uint8_t* rows_raw, uint64_t rows, uint64_t cols, const float* x, uint64_t M, float* y,
                  int iters, double* ms) {
  return guard([&] {
    NEED(rows_raw);
    NEED(x);
    NEED(y);
    int dev = 0;
    LS_CUDA(cudaGetDevice(&dev));
    std::unique_ptr<LsQWeights> q(new LsQWeights);
    qweights_upload(q.get(), dev, bits, group, rows_raw, rows, cols);
    float *dx = nullptr, *dy = nullptr;
    LS_CUDA(cudaMalloc(&dx, M * cols * 4));
    LS_CUDA(cudaMalloc(&dy, M * rows * 4));
    std::unique_ptr<float, decltype(&cudaFree)> gx(dx, &cudaFree), gy(dy, &cudaFree);
    LS_CUDA(cudaMemcpy(dx, x, M * cols * 4, cudaMemcpyHostToDevice));
    qgemv_device(q.get(), dx, M, dy, 0);
    LS_CUDA(cudaDeviceSynchronize());
    if (iters > 1 && ms) {
      // Timing: back-to-back launches (one CUDA graph), each over its own device replica of the
      // weight planes, at least `iters` of them and together at least 256 MB (twice L2), so that
      // every launch streams its weights from HBM; ms = the events' span / launches.
      const size_t bytes = qmat_bytes((int)rows, (int)cols, WeightFormat{q->w.bits, q->w.group});
      const size_t reps = std::min<size_t>(4096, std::max<size_t>((size_t)iters, ((size_t)256 << 20) / bytes + 1));
      uint8_t* rep = nullptr;
      LS_CUDA(cudaMalloc(&rep, reps * bytes));
      std::unique_ptr<uint8_t, decltype(&cudaFree)> grep(rep, &cudaFree);
      cudaStream_t st;
      LS_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
      struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() {
          cudaStreamSynchronize(s);
          cudaStreamDestroy(s);
        }
      } sg{st};
      const uint8_t* base = static_cast<const uint8_t*>(q->mem);
      for (size_t i = 0; i < reps; i++)
        LS_CUDA(cudaMemcpyAsync(rep + i * bytes, base, bytes, cudaMemcpyDeviceToDevice, st));
      std::vector<LsQWeights> views(reps);
      for (size_t i = 0; i < reps; i++) {  // the replica's planes at the same offsets (not owned)
        LsQWeights& v = views[i];
        v.device = q->device;
        v.w = q->w;
        v.w.data = rep + i * bytes + (q->w.data - base);
        v.w.scales = reinterpret_cast<const uint16_t*>(rep + i * bytes + (reinterpret_cast<const uint8_t*>(q->w.scales) - base));
        v.partial = q->partial;
        v.tickets = q->tickets;
        v.err = q->err;
        v.num_sms = q->num_sms;
      }
      struct ViewGuard {  // the views own nothing
        std::vector<LsQWeights>& v;
        ~ViewGuard() {
          for (auto& w : v) w.mem = w.partial = nullptr, w.tickets = nullptr, w.err = nullptr;
        }
      } vg{views};
      cudaGraph_t graph;
      LS_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      try {
        for (size_t i = 0; i < reps; i++) qgemv_device(&views[i], dx, M, dy, st);
      } catch (...) {
        cudaStreamEndCapture(st, &graph);
        throw;
      }
      LS_CUDA(cudaStreamEndCapture(st, &graph));
      cudaGraphExec_t exec;
      const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      LS_CUDA(ie);
      struct ExecGuard {
        cudaGraphExec_t e;
        ~ExecGuard() { cudaGraphExecDestroy(e); }
      } eg{exec};
      LS_CUDA(cudaGraphLaunch(exec, st));  // warm-up
      cudaEvent_t a, b;
      LS_CUDA(cudaEventCreate(&a));
      LS_CUDA(cudaEventCreate(&b));
      LS_CUDA(cudaEventRecord(a, st));
      LS_CUDA(cudaGraphLaunch(exec, st));
      LS_CUDA(cudaEventRecord(b, st));
      LS_CUDA(cudaEventSynchronize(b));
      float t = 0;
      LS_CUDA(cudaEventElapsedTime(&t, a, b));
      *ms = (double)t / (double)reps;
      cudaEventDestroy(a);
      cudaEventDestroy(b);
    }
    LS_CUDA(cudaMemcpy(y, dy, M * rows * 4, cudaMemcpyDeviceToHost));
    qweights_check(q.get());
  });
}

int ls_bgemm_host(int bits, int group, const uint8_t* rows_raw, uint64_t rows, uint64_t cols, const float* x, uint64_t M, float* y,
                  int iters, double* ms) {
  return guard([&] {
    NEED(rows_raw);
    NEED(x);
    NEED(y);
    if (M == 0 || M > 8192) LS_THROW(LS_ERR_ARG, "1..8192 token rows");
    if (cols % 8) LS_THROW(LS_ERR_ARG, "cols must be a multiple of 8");
    int dev = 0, nsm = 0;
    LS_CUDA(cudaGetDevice(&dev));
    LS_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    std::unique_ptr<LsQWeights> q(new LsQWeights);
    qweights_upload(q.get(), dev, bits, group, rows_raw, rows, cols);
    if (!bgemm_supported(q->w)) LS_THROW(LS_ERR_ARG, "format not supported by the batched GEMM");
    const BgemmPlan p = bgemm_plan(q->w, (int)M, nsm, false);
    std::vector<void*> bufs;
    auto dal = [&](size_t bytes) {
      void* d = nullptr;
      LS_CUDA(cudaMalloc(&d, std::max<size_t>(bytes, 16)));
      bufs.push_back(d);
      LS_CUDA(cudaMemset(d, 0, std::max<size_t>(bytes, 16)));
      return d;
    };
    struct Free {
      std::vector<void*>* b;
      ~Free() {
        for (void* d : *b) cudaFree(d);
      }
    } fr{&bufs};
    auto* dx = static_cast<float*>(dal(M * cols * 4));
    auto* dxh = static_cast<uint16_t*>(dal(bt_elems((int)M, (int)cols) * 2));
    auto* dy = static_cast<float*>(dal(M * rows * 4));
    auto* dpart = static_cast<float*>(dal(p.partial_floats * 4));
    auto* dtick = static_cast<unsigned*>(dal(p.tickets * 4));
    auto* derr = static_cast<int*>(dal(4));
    LS_CUDA(cudaMemcpy(dx, x, M * cols * 4, cudaMemcpyHostToDevice));
    launch_bt_prep(dx, (int)cols, (int)M, (int)cols, nullptr, nullptr, 0.f, dxh, 0);
    BgemmLaunch g;
    g.w = q->w;
    g.x = dxh;
    g.M = (int)M;
    g.epi = EPI_STORE;
    g.y = dy;
    g.y_stride = (int)rows;
    g.partial = dpart;
    g.tickets = dtick;
    g.err = derr;
    launch_bgemm(g, p, 0);
    LS_CUDA(cudaDeviceSynchronize());
    if (getenv("LS_BG_TRACE")) {
      // profiling: one more launch with the pipeline timeline, summarised on stderr (CTA 0's events
      // per K block relative to its start; every CTA's duration)
      const int ctas = ((q->w.rows_pad / 32 + 3) / 4) * p.ngroups * p.ks;
      auto* dtr = static_cast<unsigned*>(dal(((size_t)BG_TRACE_CTA + 2 * ctas) * 4));
      BgemmLaunch gt = g;
      gt.trace = dtr;
      launch_bgemm(gt, p, 0);
      LS_CUDA(cudaDeviceSynchronize());
      std::vector<unsigned> tr((size_t)BG_TRACE_CTA + 2 * ctas);
      LS_CUDA(cudaMemcpy(tr.data(), dtr, tr.size() * 4, cudaMemcpyDeviceToHost));
      int khz = 1;
      LS_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev));
      const unsigned t0 = tr[BG_TRACE_CTA];
      fprintf(stderr, "bgemm trace: N %d groups %d ks %d stages %d kstage %d abuf %d issuers %d tmem %d smem %zu\n", p.N,
              p.ngroups, p.ks, p.stages, p.kstage, p.abuf, p.niss, p.tmem_cols, p.smem);
      const char* kinds[] = {"produced", "A written", "MMAs issued", "data seen", "A store", "A stored", "issuer waits"};
      for (int kb = 0; kb < 64; kb++) {
        bool any = false;
        char line[512];
        int o = std::snprintf(line, sizeof line, "  block %2d:", kb);
        for (int k = 0; k < 7; k++) {
          const unsigned t = tr[k * 64 + kb];
          if (!t) continue;
          any = true;
          o += std::snprintf(line + o, sizeof line - o, " %s %.2f", kinds[k], (double)(int)(t - t0) / khz * 1e3);
        }
        if (any) fprintf(stderr, "%s us\n", line);
      }
      fprintf(stderr, "  epilogue %.2f -> %.2f us\n", (double)(int)(tr[7 * 64] - t0) / khz * 1e3,
              (double)(int)(tr[7 * 64 + 1] - t0) / khz * 1e3);
      std::vector<double> d;
      for (int c = 0; c < ctas; c++)
        d.push_back((double)(tr[BG_TRACE_CTA + 2 * c + 1] - tr[BG_TRACE_CTA + 2 * c]) / khz * 1e3);
      std::sort(d.begin(), d.end());
      fprintf(stderr, "  CTA durations: min %.2f median %.2f max %.2f us over %d CTAs\n", d.front(), d[d.size() / 2], d.back(), ctas);
    }
    if (iters > 1 && ms) {
      cudaEvent_t a, b;
      LS_CUDA(cudaEventCreate(&a));
      LS_CUDA(cudaEventCreate(&b));
      LS_CUDA(cudaEventRecord(a, 0));
      for (int i = 0; i < iters; i++) launch_bgemm(g, p, 0);
      LS_CUDA(cudaEventRecord(b, 0));
      LS_CUDA(cudaEventSynchronize(b));
      float t = 0;
      LS_CUDA(cudaEventElapsedTime(&t, a, b));
      *ms = t / iters;
      cudaEventDestroy(a);
      cudaEventDestroy(b);
    }
    int herr = 0;
    LS_CUDA(cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost));
    if (herr) LS_THROW(LS_ERR_DEVICE, "the batched GEMM gave up waiting on an mbarrier (bounded wait)");
    LS_CUDA(cudaMemcpy(y, dy, M * rows * 4, cudaMemcpyDeviceToHost));
  });
}

int ls_dequant_rows_host(int bits, int group, const uint8_t* rows_raw, uint64_t rows, uint64_t cols, const uint32_t* ids,
                         uint64_t n, float* out) {
  return guard([&] {
    NEED(rows_raw);
    NEED(ids);
    NEED(out);
    if (n == 0 || n > 128) LS_THROW(LS_ERR_ARG, "1..128 rows per call");
    for (uint64_t i = 0; i < n; i++)
      if (ids[i] >= rows) LS_THROW(LS_ERR_ARG, "row id out of range");
    int dev = 0;
    LS_CUDA(cudaGetDevice(&dev));
    std::unique_ptr<LsQWeights> q(new LsQWeights);
    qweights_upload(q.get(), dev, bits, group, rows_raw, rows, cols);
    Ctl* ctl = nullptr;
    float* dx = nullptr;
    LS_CUDA(cudaMalloc(&ctl, sizeof(Ctl)));
    std::unique_ptr<Ctl, decltype(&cudaFree)> gc(ctl, &cudaFree);
    LS_CUDA(cudaMalloc(&dx, n * cols * 4));
    std::unique_ptr<float, decltype(&cudaFree)> gx(dx, &cudaFree);
    LS_CUDA(cudaMemset(ctl, 0, sizeof(Ctl)));
    LS_CUDA(cudaMemcpy(ctl->tokens, ids, n * 4, cudaMemcpyHostToDevice));
    launch_embed(q->w, ctl, dx, (int)cols, (int)n, 0);
    LS_CUDA(cudaMemcpy(out, dx, n * cols * 4, cudaMemcpyDeviceToHost));
  });
}

uint64_t ls_qgemv_bytes(int bits, int group, uint64_t rows, uint64_t cols, uint64_t M) {
  const uint64_t scale_bytes = (bits == 16 || group == 0) ? 0 : cols / (uint64_t)group * 2;  // bf16 rows: none
  return rows * (cols * (uint64_t)bits / 8 + scale_bytes) + M * cols * 4 + M * rows * 4;
}

}  // extern "C"
