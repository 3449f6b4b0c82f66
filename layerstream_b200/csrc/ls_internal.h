// Internal declarations shared by the host code and the CUDA kernels of layerstream_b200.
#pragma once

#include <cuda.h>
#include <nccl.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <vector>

namespace ls {

// ---- errors ----------------------------------------------------------------------------------

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define LS_THROW(code, msg) throw ::ls::Error((code), (msg))
#define LS_CUDA(expr)                                                                                   \
  do {                                                                                                  \
    cudaError_t _e = (expr);                                                                            \
    if (_e != cudaSuccess)                                                                              \
      throw ::ls::Error(-3, std::string(#expr) + ": " + cudaGetErrorString(_e) + " (" __FILE__ ":" +   \
                                std::to_string(__LINE__) + ")");                                        \
  } while (0)

// ---- formats (src/weights.rs) ----------------------------------------------------------------

struct WeightFormat {
  int bits = 16;  // 16 = bf16; 8 or 4 = grouped symmetric integers with bf16 scales
  int group = 0;
  bool quant() const { return bits != 16; }
  bool operator==(const WeightFormat& o) const { return bits == o.bits && group == o.group; }
  // src/weights.rs:26-31
  size_t row_bytes(size_t cols) const {
    return quant() ? cols * (size_t)bits / 8 + cols / (size_t)group * 2 : cols * 2;
  }
};

struct Config {
  WeightFormat format, embed_format;
  size_t hidden = 0, inter = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0, max_pos = 0;
  float eps = 0, rope_theta = 0;
  size_t kv_dim() const { return kv_heads * head_dim; }
  size_t embed_row_bytes() const { return embed_format.row_bytes(hidden); }
};

// Tensor slots inside a stored layer block (src/weights.rs:158-171).
enum Slot { T_INPUT_NORM = 0, T_DOWN, T_GATE, T_UP, T_POST_NORM, T_K_B, T_K_W, T_O_W, T_Q_B, T_Q_W, T_V_B, T_V_W, N_SLOTS };

struct LayerLayout {
  size_t off[N_SLOTS] = {0}, len[N_SLOTS] = {0};
  size_t total = 0;
};

Config parse_config(const std::string& json_text);
LayerLayout layer_layout_for(const Config& c);
bool matrix_shape(int slot, const Config& c, size_t* rows, size_t* cols);
std::vector<size_t> tensor_shape(int slot, const Config& c);
extern const char* const kSlotSuffix[N_SLOTS];

// A `.lsq` file opened for reading (src/weights.rs:327-423).
struct LsqFile {
  std::string path;
  std::string config_text;
  Config cfg;
  LayerLayout layout;
  uint64_t data_start = 0, embed_start = 0, norm_start = 0;
  size_t embed_bytes = 0, norm_bytes = 0;
  static LsqFile open(const std::string& path);
};

// A BF16 safetensors model directory (src/weights.rs:271-324).
struct SafetensorsModel {
  std::string dir, file, config_text;
  Config cfg;
  LayerLayout layout;
  std::vector<uint64_t> layer_start;
  uint64_t embed_start = 0, norm_start = 0;
  size_t embed_len = 0, norm_len = 0;
  static SafetensorsModel open(const std::string& dir);
};

// A sealed model file (src/seal.rs:13-27): frame (magic "LSS1", version 1, 8-byte nonce prefix,
// header length), JSON header, 16-byte tags (one per chunk), then the ciphertext of every layer
// block, the embedding table and the final norm. Layer blocks are cut into layer_chunk-byte chunks,
// the table into embed_chunk_rows-row chunks, the norm is one chunk; chunk i's message has nonce
// prefix || le32(i) and associated data = frame + header || le32(i).
constexpr size_t kSealFrame = 20;
struct SealedFile {
  std::string path, config_text;
  Config cfg;
  LayerLayout layout;  // from the header
  size_t layer_chunk = 0, embed_chunk_rows = 0, final_norm_bytes = 0;
  uint8_t nonce_prefix[8] = {0};
  std::vector<uint8_t> aad_prefix;  // frame + header bytes
  std::vector<uint8_t> tags;        // 16 x n_chunks
  uint64_t tags_off = 0, ct_base = 0, file_len = 0;
  size_t layer_chunks() const { return (layout.total + layer_chunk - 1) / layer_chunk; }
  size_t embed_bytes() const { return cfg.vocab * cfg.embed_row_bytes(); }
  size_t embed_chunks() const { return (cfg.vocab + embed_chunk_rows - 1) / embed_chunk_rows; }
  size_t embed_first_chunk() const { return cfg.layers * layer_chunks(); }
  size_t final_chunk() const { return embed_first_chunk() + embed_chunks(); }
  size_t n_chunks() const { return final_chunk() + 1; }
  uint64_t embed_plain_off() const { return (uint64_t)cfg.layers * layout.total; }
  uint64_t total_plain() const { return embed_plain_off() + embed_bytes() + final_norm_bytes; }
  static SealedFile open(const std::string& path);
};
std::string sealed_header_json(const std::string& config_text, const LayerLayout& layout, size_t layer_chunk,
                               size_t embed_chunk_rows, size_t final_norm_bytes);
bool is_sealed_file(const std::string& path);  // starts with the magic bytes "LSS1"
// Seals the model at src (a .lsq file or a bf16 safetensors directory) into a new file at out
// (src/seal.rs:726-827, seal_model), the cipher on the GPU; returns the number of chunks.
size_t seal_model_file(const std::string& src, const std::string& out, const uint8_t* key, const uint8_t* nonce_prefix,
                       size_t layer_chunk, size_t embed_chunk_rows);

std::string inject_quant(const std::string& config_text, WeightFormat body, WeightFormat embed);
std::string lsq_header_bytes(const std::string& config_text, size_t layer_bytes, size_t embed_bytes, size_t norm_bytes);
std::string read_file_text(const std::string& path);
void pread_all(int fd, void* buf, size_t n, uint64_t off);

// ---- device layout of a quantized matrix --------------------------------------------------------
//
// A matrix of R rows x C columns is stored on the device as two planes, both tiled by 32 rows so
// that one warp (lane = row) reads 512 contiguous bytes per step:
//   data  : tile-major [R/32][C*bits/128 chunks][32 rows][16 B]  (the row's packed ints, unchanged)
//   scales: tile-major [R/32][C/G groups][32 rows] bf16
// R is padded up to a multiple of 32 with zero rows. Byte values are the file's, only moved.

struct QMat {
  const uint8_t* data = nullptr;    // tiled data plane
  const uint16_t* scales = nullptr; // tiled scale plane (bf16 bits)
  int rows = 0, rows_pad = 0, cols = 0, bits = 8, group = 64;
  __host__ __device__ size_t data_bytes() const { return (size_t)rows_pad * cols * bits / 8; }
  __host__ __device__ size_t scale_bytes() const { return (size_t)rows_pad * groups() * 2; }
  __host__ __device__ int chunks() const { return cols * bits / 128; }
  __host__ __device__ int groups() const { return bits == 16 ? 0 : cols / group; }  // bf16: no scales
};

inline int pad32(int r) { return (r + 31) / 32 * 32; }

// Row sources of a repacked matrix: up to 3 stacked segments (e.g. q | k | v), optionally with
// rows interleaved in blocks of 16 between two segments (gate/up, for the SwiGLU epilogue).
struct RepackSrc {
  const uint8_t* seg[3] = {nullptr, nullptr, nullptr};
  int seg_rows[3] = {0, 0, 0};
  int nseg = 1;
  int interleave16 = 0;  // 1: dest tile of 32 = 16 rows of seg0 then the same 16 rows of seg1
};

// ---- kernels (ls_kernels.cu) -------------------------------------------------------------------

enum Epilogue { EPI_STORE = 0, EPI_BIAS_STORE = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4, EPI_SWIGLU_H = 5 };

// Argmax partial: value then index, combined so that a larger value wins and, on equal values,
// the smaller index wins (src/spec.rs:41-49 first-maximum rule).
struct ArgPart {
  float v;
  uint32_t i;
};

// Device control block of one model: the token block and position, and the verify result.
struct Ctl {
  int32_t pos0;         // tokens already in the cache
  int32_t M;            // tokens in this pass
  int32_t n_logits;     // positions whose logits/argmax are wanted (the last n_logits)
  int32_t mode;         // 0 = forward (pos += M), 1 = verify (pos += m + 1)
  uint32_t tokens[128]; // the block (max PREFILL_CHUNK)
  // results
  uint32_t argmax[128]; // greedy token at each wanted position
  int32_t m;            // accepted prefix length (verify)
  uint32_t next;        // argmax at position m (verify) / at the last position (forward)
  int32_t err;          // nonzero if a kernel detected a bad input
  int32_t pad;
};

struct GemvLaunch {
  QMat w;
  const float* x = nullptr;  // [M][x_stride] f32
  int x_stride = 0;
  int M = 0;
  int m_base = 0;  // first token row of x for this launch (token groups)
  // optional RMSNorm prologue over the full row of x (K == hidden)
  const uint16_t* norm_bf16 = nullptr;
  const float* norm_f32 = nullptr;
  float eps = 0;
  const float* inv_rms = nullptr;  // [M] 1/rms of every row, computed once (else per CTA)
  // epilogue
  int epi = EPI_STORE;
  float* y = nullptr;          // output [M][y_stride]
  int y_stride = 0;
  const uint16_t* bias = nullptr;
  // argmax epilogue
  ArgPart* arg_parts = nullptr;  // [n_row_ctas][M]
  unsigned* arg_ticket = nullptr;
  Ctl* ctl = nullptr;            // accept/advance target of the last CTA
  int n_valid_rows = 0;          // valid rows of this matrix (ignores padding)
  int row_offset = 0;            // vocabulary id of row 0 (head streamed in chunks)
  int part_tile_offset = 0;      // first arg_parts tile of this launch
  int finalize = 1;              // 1: the last CTA reduces all parts and applies the acceptance rule
  int n_part_tiles = 0;          // tiles over all launches of this pass (finalize)
  float* logits = nullptr;       // optional full logits [M][logits_stride]
  int logits_stride = 0;
  // grid: CTAs along the row tiles (0 = one warp per tile)
  int grid_x = 0;
  int* err = nullptr;  // set to nonzero by a kernel whose bounded wait gave up
  // split-K
  int ksplit = 1;
  int max_nt = 64;           // tensor-core GEMV: widest token group (16, 32, 48 or 64)
  float* partial = nullptr;  // [row_ctas][ksplit][M][32]
  unsigned* tickets = nullptr;
};

void launch_gemv(const GemvLaunch& g, cudaStream_t s);
// inv[t] = 1 / sqrt(mean(x[t]^2) + eps) for M rows of `cols` floats (the GEMV norm prologue's sum)
void launch_inv_rms(const float* x, int x_stride, int M, int cols, float eps, float* inv, cudaStream_t s);
// Smallest K-split whose staged activations fit in shared memory.
int gemv_min_ksplit(const QMat& w, int M);
int gemv_grid_x(const QMat& w, int ksplit, int M, int num_sms);
int gemv_mt(int M);
// tensor-core (tcgen05) GEMV
bool gemv_tc_supported(const QMat& w);
int gemv_tc_min_ksplit(const QMat& w, int M, int max_nt = 64);
int gemv_tc_nt(int M, int max_nt);
void launch_gemv_tc(const GemvLaunch& g, cudaStream_t s);
void launch_repack(const RepackSrc& src, int bits, int group, int cols, uint8_t* data, uint16_t* scales, int rows_pad,
                   cudaStream_t s);
void launch_embed(const QMat& e, const Ctl* ctl, float* x, int hidden, int M, cudaStream_t s);
// Streaming mode: rows read in the file layout through a mapped pinned-host pointer.
void launch_embed_raw(const uint8_t* table, size_t row_bytes, int bits, int group, const Ctl* ctl, float* x, int hidden,
                      int vocab, int M, cudaStream_t s);
void launch_advance(Ctl* ctl, cudaStream_t s);
// Reads `bytes` (a multiple of 16, more than L2 holds) so that L2 holds only clean lines of it.
void launch_l2_evict(const void* buf, size_t bytes, unsigned* sink, cudaStream_t s);
void launch_argmax_finalize(const ArgPart* parts, int nparts, int M, Ctl* ctl, cudaStream_t s);

// ---- paged K/V cache ----
//
// Per layer a pool of pages for K and one for V, [kv_heads][num_pages][page][hd] f16; a sequence's
// position p lives in pool page table[p >> page_shift] at row p & (page - 1). Pages are handed out
// as a sequence grows and returned when it is rolled back or reset, so sequences of a batch share
// one pool. With the identity table the pool is the dense [kv_heads][max_ctx][hd] layout.
__host__ __device__ inline size_t kv_row(const int32_t* table, int page_shift, int num_pages, int g, int p) {
  return ((size_t)((size_t)g * num_pages + table[p >> page_shift]) << page_shift) + (size_t)(p & ((1 << page_shift) - 1));
}

struct AttnLaunch {
  const float* qkv = nullptr;  // [M][qkv_stride] f32: q | k | v (pre-RoPE, bias added)
  int qkv_stride = 0;
  uint16_t* k_cache = nullptr;  // this layer's page pool [kv_heads][num_pages][page][hd] f16 bits
  uint16_t* v_cache = nullptr;
  const int32_t* pages = nullptr;  // [nseq][max_pages] page table (sequence s at pages + s * max_pages)
  int page_shift = 6, num_pages = 0, max_pages = 0;
  const float2* rope = nullptr;  // [max_ctx][hd/2] (cos, sin)
  const Ctl* ctl = nullptr;
  float* out = nullptr;  // [M][heads*hd]
  float* part = nullptr; // split partials
  size_t part_floats = 0; // their capacity (tensor-core kernel: bounds its splits; 0 = max_splits bounds them)
  unsigned* tickets = nullptr;
  int heads = 0, kv_heads = 0, hd = 0, max_ctx = 0, M = 0, split = 64, max_splits = 0;
  // batches: grid.z = nseq sequences of M rows each (rows s*M .. s*M+M-1 of qkv and out); sequence
  // s has its page table row s, its position pos0[s], its partials and tickets after those of
  // sequences < s. pos0 == nullptr: one sequence at ctl->pos0.
  int nseq = 1;
  const int* pos0 = nullptr;
  bool pdl = true;  // false: plain launch (positions written by the previous kernel are read early)
  int* err = nullptr;  // set to 1 when a bounded wait of the tensor-core kernel gives up
  int max_total = 0;   // largest pos0 + M over the sequences when the host knows it (0: max_ctx)
  uint16_t* out_h = nullptr;  // tensor-core kernel: output as f16 in the bt layout (K = heads * hd) instead of out
  int out_h_n = 0;            // its token-group rows
  // profiling (tensor-core kernel): clock() stamps of thread 0 of every CTA, AT_TRACE_SLOTS per CTA
  // (CTA index = x + gridDim.x (y + gridDim.y z)); null = off
  unsigned* trace = nullptr;
};
constexpr int AT_TRACE_SLOTS = 16;
void launch_attention(const AttnLaunch& a, cudaStream_t s);
bool attention_tc_supported(const AttnLaunch& a);  // ls_attn_tc.cu
void launch_attention_tc(const AttnLaunch& a, cudaStream_t s);

void launch_set_ctl(Ctl* ctl, int pos0, int M, int n_logits, int mode, const uint32_t* tokens_dev_or_null, cudaStream_t s);
void launch_quantize_rows(const uint16_t* src_bf16, int rows, int cols, int bits, int group, int clip, uint8_t* dst,
                          double* err_norm, cudaStream_t s);

// ---- batched weight GEMM (ls_bgemm.cu) ----

// Activations in the tensor-core B-operand layout ("bt") of a GEMM whose token groups hold N rows:
// group g = t / N, 16-byte K chunk c = k / 8, element (t, k) at halves
// ((g * (K / 8) + c) * N + t % N) * 8 + k % 8. Every K range of a group is one contiguous block of
// 16-byte rows (chunk-major, token-minor), which the GEMM copies into shared memory with a single
// bulk copy and reads as K-major core matrices (8 tokens x 16 bytes). Buffers hold ngroups * N
// rows.
__host__ __device__ inline size_t bt_off(int t, int k, int K, int N) {
  const int g = t / N;
  return (((size_t)g * (K >> 3) + (k >> 3)) * N + (t - g * N)) * 8 + (k & 7);
}

struct BgemmLaunch {
  QMat w;
  const uint16_t* x = nullptr;  // activations, bt layout with K = w.cols, M rows
  int M = 0;
  int epi = EPI_STORE;          // STORE / BIAS_STORE / RESID into y, SWIGLU_H into yh, ARGMAX
  float* y = nullptr;
  int y_stride = 0;
  uint16_t* yh = nullptr;       // EPI_SWIGLU_H: f16 bt layout with K = rows / 2
  const uint16_t* bias = nullptr;
  ArgPart* arg_parts = nullptr; // EPI_ARGMAX: [part][M]
  int n_valid_rows = 0, row_offset = 0, part_tile_offset = 0;
  float* partial = nullptr;     // split-K scratch
  unsigned* tickets = nullptr;
  int* err = nullptr;
  // profiling: clock() stamps of pipeline events of CTA (0, 0, 0), [kind 0..7][K block 0..63], then
  // every CTA's start and end at BG_TRACE_CTA + 2 * cta; null = off
  unsigned* trace = nullptr;
};
constexpr int BG_TRACE_CTA = 8 * 64;
struct BgemmPlan {
  int N = 16, ngroups = 1, ks = 1, stages = 2, kstage = 1, tmem_cols = 256;
  int abuf = 4, niss = 2;  // A buffers in tensor memory (2 or 4); MMA issuers, each with its own accumulator (1 or 2)
  int n0 = 0;              // > 0: the two issuers split the token columns (n0 and N - n0) of one accumulator
  size_t smem = 0, partial_floats = 0, tickets = 0;
};
// token groups of a pass of M rows (every GEMM of the pass uses the same): N rows each, ngroups
void bgemm_groups(int M, int* N, int* ngroups);
bool bgemm_supported(const QMat& w);
BgemmPlan bgemm_plan(const QMat& w, int M, int num_sms, bool argmax);
void launch_bgemm(const BgemmLaunch& g, const BgemmPlan& p, cudaStream_t s);
// x (f32 rows) -> bt layout f16, with the RMSNorm folded in when a norm weight is given (x * inv *
// w); rows M .. pad8(M) are zero.
void launch_bt_prep(const float* x, int x_stride, int M, int K, const uint16_t* norm_bf16, const float* norm_f32,
                    float eps, uint16_t* out, cudaStream_t s);
// halves of a bt buffer of M rows and K columns (its token groups padded)
size_t bt_elems(int M, int K);

// ---- persistent pass kernel (ls_pass.cu) ----

// TMA descriptors of one matrix's planes for the pass kernel's weight stream: data as
// [row group][16-byte chunk][128 x u32], scales as [row group][group][32 x bf16].
struct QMaps {
  CUtensorMap data, scales;
};

struct PassLayer {
  QMat qkv, o, gu, down;
  const QMaps* maps;  // device [4]: qkv, o, gate/up, down
  const uint16_t* in_norm;
  const uint16_t* post_norm;
  const uint16_t* qkv_bias;
};

struct PassArgs {
  const PassLayer* layers;
  QMat embed;
  const QMaps* embed_maps;  // device
  const float* final_norm;
  Ctl* ctl;
  long long* x;     // [T][h] residual stream, fixed point
  long long* qkv;   // [T][h + 2 kv] q|k|v sums (bias included), fixed point
  long long* gu;    // [T][2 I] gate/up sums in the interleaved row order, fixed point
  float* att_part;  // [heads][slots][T][hd + 2] slot states (m, l, acc)
  uint16_t* kc;     // [L] page pools [kv_heads][num_pages][page][hd] f16 (layer stride kv_layer)
  uint16_t* vc;
  const int32_t* pages;  // the sequence's page table
  size_t kv_layer;
  int page_shift, num_pages;
  const float2* rope;
  ArgPart* arg_parts;  // [gridDim][T]
  float* logits;       // optional [n_logits][vocab]
  unsigned* bar;
  unsigned* trace;     // optional globaltimer stamps (profiling): [2 * barriers + 2][gridDim] at the
                       // barriers, then [phases][4][gridDim] inside the phases from slot trace_sub on
  int trace_sub;
  int kv_off;  // byte offset of the attention K/V region from the B-operand region
  int stall_barrier;    // test hook: this grid barrier (1-based) never completes, 0 = none
  unsigned poll_limit;  // polls of a grid-barrier wait before the CTA gives up with error 3
  int stages;  // weight-stream ring depth
  int xs;      // 1: x rows (f32) and the norm weights stay in shared memory after the RMS statistics
  int L, hidden, inter, heads, kv_heads, hd, vocab, max_ctx, T, n_logits, slots;
  int ks_qkv, ks_o, ks_gu, ks_down;
  float eps;
};

// ---- batched verify (ls_batch.cu): B sequences x M rows per pass ----
// Embedding rows of T tokens (err = 2 on an id >= vocab), bit-exact with embed_kernel.
void launch_embed_tokens(const QMat& e, const uint32_t* tokens, int T, float* x, int hidden, int vocab, int* err,
                         cudaStream_t s);
// argmax[t] over the nparts per-CTA parts of every row t (first-maximum rule); then for every
// sequence of M rows the acceptance rule of src/spec.rs:121-125: m = longest prefix with
// argmax[i] == tokens[i+1], next = argmax[m].
// best[t] = first maximum of row t over nparts parts; x += y over n floats.
void launch_row_best(const ArgPart* parts, int nparts, int T, ArgPart* best, cudaStream_t s);
void launch_add(float* x, const float* y, size_t n, cudaStream_t s);
// The same from a host-mapped table of stored rows (streaming models).
void launch_embed_raw_tokens(const uint8_t* table, size_t row_bytes, int bits, int group, const uint32_t* tokens, float* x,
                             int hidden, int vocab, int T, int* err, cudaStream_t s);
void launch_batch_accept(const ArgPart* parts, int nparts, int T, int M, const uint32_t* tokens, uint32_t* argmax,
                         uint32_t* m_out, uint32_t* next_out, cudaStream_t s);

// ---- ChaCha20-Poly1305 on the GPU (ls_seal.cu), the cipher of sealed model files ----
// One AEAD message (RFC 8439 2.8): data in device memory, opened (tag checked, then decrypted) or
// sealed (encrypted, then tagged) in place; its associated data = a prefix shared by the launch's
// chunks followed by tail_len (0..4) bytes of `tail` (little-endian).
struct AeadChunk {
  uint8_t* data;
  uint64_t len;
  uint32_t nonce[3];
  uint32_t tail, tail_len;
  uint32_t tag[4];
};
size_t aead_scratch_bytes(int nchunks, uint64_t max_len, uint32_t aad_len);
// d_chunks, d_aad, d_key (8 words) in device memory; opening: *d_bad (preset to INT_MAX by the
// caller) becomes min(failing chunk + 1) and the failing chunks stay untouched; sealing writes the
// tags into d_chunks.
void launch_aead(AeadChunk* d_chunks, int nchunks, uint64_t max_len, const uint8_t* d_aad, uint32_t aad_len, const uint32_t* d_key,
                 bool seal, void* scratch, size_t scratch_bytes, int* d_bad, cudaStream_t s);
int aead_host(bool seal, const uint8_t* key, const uint8_t* nonce12, bool indexed, uint32_t first, const uint8_t* aad,
              uint64_t aad_len, uint8_t* data, uint64_t len, uint64_t chunk_bytes, uint8_t* tags, int iters, double* ms);

// ---- tensor-parallel reduction through peer memory (ls_p2p.cu) ----
constexpr int kMaxTpWorld = 8;
struct P2PReduce {
  int world = 0, rank = 0;
  const float* peer_y[kMaxTpWorld] = {};    // every rank's partial rows (this rank's own at [rank])
  unsigned* peer_flags[kMaxTpWorld] = {};   // every rank's ready flags, mapped into this process
  unsigned* flags = nullptr;   // this rank's [world] ready epochs, by rank
  unsigned* seq = nullptr;     // reductions this rank has completed
  unsigned* ticket = nullptr;  // last-CTA election
  unsigned* arrive = nullptr;  // first-CTA election (who signals ready)
  int* err = nullptr;          // error word (5: a peer did not answer in time)
  unsigned long long limit_ns = 0;  // how long one wait may take before it gives up
};
// x[i] += sum over the ranks of y_r[off + i], i < n (all ranks in order).
void launch_p2p_reduce_add(float* x, const P2PReduce& r, size_t off, size_t n, int num_sms, cudaStream_t s);
// The same over M rows of K, fused with the RMSNorm (norm_bf16 or norm_f32 weights) and f16 packing
// into the batched GEMM's operand layout, as launch_bt_prep(x, K, M, K, ...) after the add.
void launch_p2p_reduce_prep(float* x, const P2PReduce& r, size_t off, int M, int K, const uint16_t* norm_bf16, const float* norm_f32,
                            float eps, uint16_t* out, int num_sms, cudaStream_t s);
// One process, one GPU: the reduction as rank `rank` of an emulated world whose peers' partials
// (ys: world x n, this rank's own at [rank]) sit in this GPU's memory. preset: the peers' flags are
// set before the launches, so no wait happens; otherwise nothing sets them and the first wait runs
// out after wait_ms. Returns the error word (0 or 5); x_out = x + calls x the sum of ys. K > 0: the
// fused form over n / K rows of K, op_out = the f16 operand (RMSNorm with norm, or none when NULL)
// in row order.
int tp_reduce_host(const float* x, const float* ys, int world, int rank, uint64_t n, bool preset, uint32_t wait_ms, int calls,
                   float* x_out, double* ms, uint32_t K, const float* norm, float eps, uint16_t* op_out);

// ---- NCCL, loaded at run time (ls_nccl.cpp) ----
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;  // for a communicator left in a failed state
  const char* (*error_string)(ncclResult_t) = nullptr;
};
const NcclApi& nccl_api();  // throws when libnccl.so.2 cannot be loaded
void nccl_check(ncclResult_t r, const char* what);

// ---- allocation-free GEMV (ls_noalloc.cu) ----
void qgemv_rows_noalloc(int bits, int group, const uint8_t* rows_dev, uint64_t rows, uint64_t cols, const float* x_dev,
                        uint64_t M, float* y_dev, cudaStream_t s);

int pass_kernel_nt(int T);
bool pass_kernel_supported(const WeightFormat& body, const WeightFormat& embed, int T, int hd);
// xs: the launch keeps the RMS-normalised rows' source (x as f32, and the norm weights) in shared
// memory for the staging (pass_kernel_xs_bytes more shared memory)
size_t pass_kernel_smem(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down, int stages, bool xs);
int pass_kernel_stages(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down, size_t budget, bool xs);
size_t pass_kernel_xs_bytes(int T, int hidden);
size_t pass_kernel_kv_off(const WeightFormat& f, int T, int hidden, int inter, int hd, int ks_down);
void launch_pass(const PassArgs& a, const WeightFormat& f, size_t smem, int grid, cudaStream_t s);
int pass_kernel_blocks_per_sm(const WeightFormat& f, int T, size_t smem, int max_per_sm);
size_t pass_kernel_smem_budget(const WeightFormat& f, int T);
// K blocks of 64 columns per weight-stream stage of the pass kernel, and the descriptors.
int pass_kernel_stage_blocks(const WeightFormat& f);
void pass_encode_maps(const QMat& w, QMaps* out);
// 3-D tiled tensor maps of a matrix's planes (x = one 16-byte chunk of 32 rows / one group of 32
// scales, y = chunk / group, z = 32-row group) with the given box.
void encode_qmat_maps(const QMat& w, int box_chunks, int box_groups, int box_rowgroups, QMaps* out);

}  // namespace ls
