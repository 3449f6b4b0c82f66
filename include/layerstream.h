/*
 * layerstream_b200 — C ABI of the B200-native speculative-decode verify path.
 *
 * This is the boundary a host in the reference's language binds (a Rust `extern "C"` block, or
 * ctypes). Every entry point takes plain pointers and sizes, returns 0 on success and a negative
 * status on error (never aborts, never throws across the boundary), and leaves a message that
 * ls_last_error() returns. Errors are values, as in the reference, where every fallible call
 * returns Result<_, String>.
 *
 * Threading: one caller thread per LsModel at a time (the reference's Model is `&mut self`).
 * Device memory is owned by the LsModel; host buffers passed in are copied and not retained.
 *
 * Reference interfaces replaced (paths inside themaker00001/layerstream):
 *   LsModel                      <- model::Model (src/model.rs:16-26) + provider::Provider (src/provider.rs:39-55)
 *   ls_model_open                <- weights::ModelFiles::open_quantized (src/weights.rs:391-423)
 *                                   + provider::ResidentProvider::load (src/provider.rs:69-81)
 *                                   / provider::StreamProvider::new (src/provider.rs:182-223)
 *                                   + model::Model::new (src/model.rs:58-77)
 *   ls_forward                   <- model::Model::forward (src/model.rs:111-119)
 *   ls_forward_multi             <- model::Model::forward_multi (src/model.rs:124-133)
 *   ls_verify                    <- the verify step of spec::speculative_greedy (src/spec.rs:110-139):
 *                                   forward_multi + argmax + longest-prefix acceptance + truncate
 *   ls_truncate / ls_pos / ls_reset <- model::Model::truncate / pos / reset (src/model.rs:84-103,137-140)
 *   ls_speculative_greedy        <- spec::speculative_greedy (src/spec.rs:57-152)
 *   ls_quantize_model            <- quant::quantize_model (src/quant.rs:158-251)
 *   ls_model_report              <- provider::ProviderReport (src/provider.rs:29-37) + source::IoStats (src/source.rs:13-21)
 *
 * The K/V cache (src/model.rs:67-68: [max_ctx x kv_dim] per layer, rolled back by a length,
 * src/model.rs:137-140) is paged here: per layer a pool of pages of kv_page positions shared by the
 * sequences of a model or batch, a page table per sequence, pages taken as a sequence grows and
 * returned when it is truncated or reset.
 */
#ifndef LAYERSTREAM_B200_H
#define LAYERSTREAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct LsModel LsModel;

/* Status codes. */
#define LS_OK 0
#define LS_ERR_ARG -1      /* bad request: the reference's Err(String) cases */
#define LS_ERR_IO -2       /* file missing, damaged or of the wrong format */
#define LS_ERR_CUDA -3     /* a CUDA call failed */
#define LS_ERR_DEVICE -4   /* a kernel reported an error status (e.g. a bounded wait gave up) */

/* Residency modes (src/provider.rs): every layer in HBM, or N HBM slots filled per pass from
 * pinned host memory by cudaMemcpyAsync on a side stream. */
#define LS_MODE_RESIDENT 0
#define LS_MODE_STREAM 1

typedef struct LsModelInfo {
  uint64_t hidden, inter, layers, heads, kv_heads, head_dim, vocab, max_ctx;
  int32_t bits, group, embed_bits, embed_group; /* bits 16 = bf16 */
  float eps, rope_theta;
  uint64_t layer_bytes;        /* bytes of one stored layer block */
  uint64_t embed_row_bytes;    /* bytes of one stored embedding row */
  uint64_t weight_bytes;       /* layers * layer_bytes + vocab * embed_row_bytes */
  int32_t persistent_pass;     /* 1: passes of 1..48 tokens run as one persistent kernel launch */
  int32_t kv_page;             /* positions per page of the paged K/V cache (LS_KV_PAGE, default 64) */
  uint64_t kv_pages_total;     /* pages in the model's pool */
  uint64_t kv_pages_used;      /* pages its sequence holds now (ceil(pos / kv_page)) */
} LsModelInfo;

/* src/provider.rs:29-37, src/source.rs:13-21 */
typedef struct LsReport {
  uint64_t resident_weight_bytes; /* device bytes holding weights */
  uint64_t bytes_read;            /* bytes moved host->device for weights since open */
  uint64_t wait_ns;               /* host time blocked on streamed data */
  uint64_t passes;                /* forward passes run */
  uint64_t h2d_bytes;             /* token blocks and control data copied host->device since open */
  uint64_t d2h_bytes;             /* results (tokens, counts, logits) copied device->host since open */
} LsReport;

/* Live kernel timing (on the model's stream), enabled by ls_model_profile_enable. Classes: 0 QKV
 * GEMV, 1 attention, 2 O GEMV, 3 gate/up GEMV, 4 down GEMV (one layer per pass), 5 LM head GEMV +
 * argmax, 6 the whole pass.
 * Separate kernels: CUDA events around each launch; classes 0-4 sample one middle layer.
 * Persistent pass kernel: class 6 from CUDA events around the launch; classes 0-5 from device
 * timestamps taken at its grid barriers, ms = phase span (departure of the last CTA from the
 * previous barrier to departure of the last CTA from this one) averaged over the layers, busy_ms =
 * the part of it the average CTA spends working rather than waiting at the barrier.
 * bytes = algorithmic bytes of the timed work (weights + scales + activations in and out; for
 * attention the K/V cache rows read plus the new rows written). */
#define LS_PROF_CLASSES 7
typedef struct LsProfile {
  uint64_t launches[LS_PROF_CLASSES];
  double ms[LS_PROF_CLASSES];
  double bytes[LS_PROF_CLASSES];
  double busy_ms[LS_PROF_CLASSES];
  /* Persistent pass kernel only: the phase's critical CTA (the last to arrive at the barrier that
   * closes it), its time split into 0 preparation (RMS statistics; attention: query rows staged),
   * 1 staging of its first item (attention: first context tile in shared memory), 2 the first
   * item's K loop and epilogue (attention: scores, values, slot state published), 3 its further
   * items (attention: the slot merge), 4 from its last item to its arrival at the barrier, 5 from
   * that arrival until the last CTA left the barrier; averaged over the layers like ms. */
  double crit_ms[LS_PROF_CLASSES][6];
} LsProfile;

/* Live profile of a batch: CUDA-event time of every launch class of its passes. Classes: 0 QKV,
 * 1 attention, 2 O, 3 gate/up, 4 down, 5 LM head (argmax epilogue), 6 collectives of a
 * tensor-parallel batch (all-reduce + residual add, all-gather), 7 the whole pass. bytes =
 * algorithmic bytes (weights + scales + activations; attention: K/V rows read and written;
 * collectives: bytes each rank sends). */
#define LS_BATCH_PROF_CLASSES 8
typedef struct LsBatchProfile {
  uint64_t launches[LS_BATCH_PROF_CLASSES];
  double ms[LS_BATCH_PROF_CLASSES];
  double bytes[LS_BATCH_PROF_CLASSES];
} LsBatchProfile;

/* src/spec.rs:16-39 */
typedef struct LsSpecStats {
  uint64_t target_passes, drafted, accepted, draft_forwards;
  double target_secs, draft_secs, first_secs, decode_secs;
} LsSpecStats;

/* Copies the last error message of this thread into buf (NUL-terminated); returns its length. */
int ls_last_error(char *buf, size_t cap);

/* Opens a quantized `.lsq` file (src/weights.rs:327-423 format) on CUDA device `device`.
 * mode: LS_MODE_RESIDENT or LS_MODE_STREAM; slots: HBM layer slots when streaming (>= 1).
 * max_ctx: KV-cache capacity in tokens, reserved up front (src/model.rs:67-68). */
int ls_model_open(const char *lsq_path, int device, uint64_t max_ctx, int mode, int slots, LsModel **out);
int ls_model_free(LsModel *m);

/* A sealed model file (src/seal.rs: SealedSource::open + ResidentProvider::load / StreamProvider):
 * ChaCha20-Poly1305 per chunk, key = 32 bytes. The ciphertext is copied to the GPU and opened
 * there (tags checked, then decrypted) before the weights are repacked: resident mode opens every
 * chunk once at load; stream mode opens each layer block in its HBM slot on every pass (the
 * embedding table is opened once, into the pinned host copy the passes read). Opening checks the
 * key on the final norm's chunk (LS_ERR_IO: "authentication failed", as src/seal.rs:894-902); a
 * modified chunk fails the load (resident) or the pass that streams it (LS_ERR_IO). */
int ls_model_open_sealed(const char *path, const uint8_t *key, int device, uint64_t max_ctx, int mode, int slots,
                         LsModel **out);
/* seal_model (src/seal.rs:726-827): seals the model at src (a .lsq file or a bf16 model directory)
 * into a new file out_path (which must not exist) under key (32 bytes) and nonce_prefix (8 bytes),
 * layer blocks cut into layer_chunk-byte chunks and the table into embed_chunk_rows-row chunks
 * (the reference's defaults: 1 MiB and 512), the cipher run on GPU `device`. The file is
 * byte-identical to the reference's for the same inputs. *n_chunks (optional): chunks written. */
int ls_seal_model(const char *src, const char *out_path, const uint8_t *key, const uint8_t *nonce_prefix,
                  uint64_t layer_chunk, uint64_t embed_chunk_rows, int device, uint64_t *n_chunks);
int ls_model_info(const LsModel *m, LsModelInfo *out);
int ls_model_report(const LsModel *m, LsReport *out);

/* The CUDA stream (cudaStream_t) every kernel of this model is launched on, for callers that time
 * the model's work with their own CUDA events. */
int ls_model_stream(const LsModel *m, void **stream);

/* on: 0 off, 1 CUDA-event timing, 2 also the persistent pass kernel's barrier timeline (which
 * adds a few % to the pass); also clears the counters */
int ls_model_profile_enable(LsModel *m, int on);
int ls_model_profile(const LsModel *m, LsProfile *out);

int ls_pos(const LsModel *m, uint64_t *pos);
int ls_reset(LsModel *m);
int ls_truncate(LsModel *m, uint64_t pos);

/* Pushes n tokens (prefill, 128-token chunks) and returns the last position's logits (vocab
 * floats, may be NULL) and its greedy token (first maximum; may be NULL). */
int ls_forward(LsModel *m, const uint32_t *ids, uint64_t n, float *logits, uint32_t *argmax);

/* One pass over t <= 128 tokens returning the logits at the last n positions (n * vocab floats). */
int ls_forward_multi(LsModel *m, const uint32_t *ids, uint64_t t, uint64_t n, float *logits);

/* The verify step. block = [a, d_1 .. d_k] (n = k + 1 <= 33 tokens). One pass over the weights,
 * the greedy token at every position computed on the device, then m = the longest prefix with
 * argmax(pos i) == d_{i+1}, next = argmax(pos m). The cache keeps exactly [a, d_1 .. d_m]
 * (pos advances by m + 1). Only (m, next) cross back to the host. */
int ls_verify(LsModel *m, const uint32_t *block, uint64_t n, uint32_t *accepted_m, uint32_t *next);

/* spec::speculative_greedy: generates up to max_new tokens with `target`, `draft` guessing k at a
 * time. Both models must be fresh and share a vocabulary. out_tokens holds max_new entries.
 * draft may be NULL: then a prompt-lookup drafter (longest recent n-gram match in the token
 * history, an addition to the reference) proposes the guesses. */
int ls_speculative_greedy(LsModel *target, LsModel *draft, const uint32_t *prompt, uint64_t plen, uint64_t max_new,
                          uint64_t k, const uint32_t *eos, uint64_t neos, uint32_t *out_tokens, uint64_t *out_len,
                          LsSpecStats *stats);

/* The decode loop of spec::speculative_greedy (src/spec.rs:94-149) from an already prefilled state:
 * target (and draft, if any) hold exactly the hlen tokens of `hist`, and `first` is the target's
 * greedy token after them (ls_forward's argmax). out_tokens[0] = first. speculative_greedy is
 * ls_forward(prompt) on both models followed by this call. */
int ls_spec_continue(LsModel *target, LsModel *draft, const uint32_t *hist, uint64_t hlen, uint32_t first,
                     uint64_t max_new, uint64_t k, const uint32_t *eos, uint64_t neos, uint32_t *out_tokens,
                     uint64_t *out_len, LsSpecStats *stats);

/* quant::quantize_model: reads a BF16 safetensors model directory (config.json +
 * model.safetensors) and writes a new `.lsq` file (must not exist). The group quantization with
 * its clip search runs on CUDA device `device`; bytes equal the reference's quantizer's. */
int ls_quantize_model(const char *src_dir, const char *out_path, int bits, int group, int embed_bits, int embed_group,
                      int clip_search, int device, double *rel_rmse);

/* ---- batches of independent sequences (configs 4 and 5) -------------------------------------- */

/* B sequences sharing one resident model's weights, each with its own K/V cache of max_ctx
 * positions; a verify pass takes one block of M <= max_block tokens per sequence ([B][M] blocks)
 * and runs all B*M rows through the model at once. */
typedef struct LsBatch LsBatch;
int ls_batch_open(LsModel *m, uint64_t batch, uint64_t max_ctx, uint64_t max_block, LsBatch **out);
/* Tensor parallelism (config 5b), one model split over `world` GPUs: rank `rank`
 * (one process or thread per GPU, its model opened resident on its own device) keeps its q heads
 * (and the kv heads they read), a 64-column-aligned slice of the intermediate dimension and a slice
 * of the vocabulary; O and down are row-parallel with a sum all-reduce, the LM head is
 * vocabulary-parallel with an all-gather of each rank's (max, first index) per row. Every rank
 * makes the same calls with the same inputs and gets the same tokens. The ranks share one NCCL
 * unique id (ls_tp_unique_id on one rank, passed to the others by the host); opening is
 * collective. NCCL (libnccl.so.2) is loaded at the first tensor-parallel call. */
int ls_tp_unique_id(uint8_t *out, size_t cap); /* cap >= 128 */
int ls_batch_open_tp(LsModel *m, uint64_t batch, uint64_t max_ctx, uint64_t max_block, int rank, int world,
                     const uint8_t *id, LsBatch **out);
int ls_batch_free(LsBatch *b);
int ls_batch_pos(const LsBatch *b, uint64_t seq, uint64_t *pos);
int ls_batch_truncate(LsBatch *b, uint64_t seq, uint64_t pos);
/* src/model.rs:111-119 for sequence `seq`: pushes n tokens, returns the greedy token after them. */
int ls_batch_prefill(LsBatch *b, uint64_t seq, const uint32_t *ids, uint64_t n, uint32_t *argmax);
/* ls_verify for sequences 0..nseq-1 in one pass: blocks [nseq][M]; per sequence the accepted
 * count m (src/spec.rs:121-125) and the next token; each sequence's position advances by m + 1. */
int ls_batch_verify(LsBatch *b, const uint32_t *blocks, uint64_t nseq, uint64_t M, uint32_t *accepted_m, uint32_t *next);
/* spec::speculative_greedy (src/spec.rs:57-152) for all B sequences with the prompt-lookup drafter:
 * prompts [B][plen] (caches must be empty or are reset), out_tokens [B][max_new], out_len [B];
 * every sequence's tokens equal its own greedy decode. stats sums over sequences. */
int ls_batch_spec(LsBatch *b, const uint32_t *prompts, uint64_t plen, uint64_t max_new, uint64_t k, const uint32_t *eos,
                  uint64_t neos, uint32_t *out_tokens, uint64_t *out_len, LsSpecStats *stats);
int ls_batch_report(const LsBatch *b, uint64_t *passes, uint64_t *h2d_bytes, uint64_t *d2h_bytes);
/* Test hook, no reference counterpart: the model's next persistent-pass launch (passes of 1..48
 * tokens, resident mode) makes grid barrier `barrier` (1-based: 1 closes the embedding phase, then 5
 * per layer and 1 after the LM head) wait for an arrival that never comes, with a short poll limit
 * (about 5 ms): its bounded wait runs out, the kernel releases its tensor memory and returns, and the
 * call fails with LS_ERR_DEVICE. Nothing faults on the GPU; the model stays usable. 0 clears it. */
int ls_model_inject_stall(LsModel *m, int barrier);

/* Test hook, no reference counterpart (the reference's failure tests inject I/O errors through a
 * failing Source, tests/pipeline.rs:170-198): the batch's next pass reports error code 4 from the
 * device as a failed kernel would, without any fault on the GPU. On a tensor-parallel batch the
 * error word is reduced over the ranks, so injecting on one rank makes every rank's pass fail with
 * LS_ERR_DEVICE; a batch whose pass failed releases its communicator with ncclCommAbort. code 0
 * clears a pending injection. */
int ls_batch_inject_error(LsBatch *b, int code);
/* on: 0 off, 1 an event pair around every launch class of each pass; also clears the counters */
int ls_batch_profile_enable(LsBatch *b, int on);
int ls_batch_profile(const LsBatch *b, LsBatchProfile *out);
/* *on = 1 when a tensor-parallel batch sums its row-parallel projections through the peers' memory
 * (every rank on its own GPU, each peer reachable; environment LS_TP_P2P=0 turns it off), 0 when
 * it uses the NCCL all-reduce or the batch is not tensor-parallel. */
int ls_batch_tp_peer(const LsBatch *b, int *on);

/* ---- kernel-level entry points (microbenchmarks and parity tests) ---------------------------- */

/* y[t][r] = dot(stored row r, x[t]) for t < M, with W given as `rows` stored rows in the .lsq
 * row format (packed ints then bf16 scales, src/weights.rs:26-31). Host buffers; the call
 * uploads, repacks, runs the verify-path GEMV kernel and copies y back. Mirrors
 * kernels::matmul (src/kernels.rs:196-203). iters > 1 repeats the kernel and returns the mean
 * kernel time in *ms (may be NULL). */
int ls_qgemv_host(int bits, int group, const uint8_t *rows_raw, uint64_t rows, uint64_t cols, const float *x, uint64_t M,
                  float *y, int iters, double *ms);
/* The batched weight GEMM of the verify / prefill pass (tensor cores, all M rows per weight tile):
 * y[M][rows] = x[M][cols] . W^T for stored rows (the `.lsq` row format) on the current device;
 * iters > 1 also times the GEMM alone (ms per launch). No reference counterpart: it is the kernel
 * behind ls_batch_verify's projections, exposed for parity tests and timing. */
int ls_bgemm_host(int bits, int group, const uint8_t *rows_raw, uint64_t rows, uint64_t cols, const float *x, uint64_t M,
                  float *y, int iters, double *ms);

/* One layer's causal GQA attention (src/model.rs:261-282, src/kernels.rs:242-265) through the
 * CUDA attention kernel of the verify path: the block's M rows at positions pos0..pos0+M-1
 * (qkv: M x (heads + 2 kv_heads) * hd f32, q | k | v before RoPE, bias added) attend over the pos0
 * cached rows (k_cache, v_cache: kv_heads x pos0 x hd, f16 bits, keys already rotated) and their
 * own rows; row i sees pos0 + i + 1 positions. The block's K/V rows are rotated (theta =
 * rope_theta) and rounded to f16 as the cache stores them. out: M x heads * hd f32. Host buffers;
 * iters > 1 repeats the kernel, each launch timed alone after a read that evicts L2 (so K/V come
 * from HBM), and returns its mean time in *ms (may be NULL). */
int ls_attention_host(uint64_t heads, uint64_t kv_heads, uint64_t hd, float rope_theta, uint64_t pos0, uint64_t M,
                      const float *qkv, const uint16_t *k_cache, const uint16_t *v_cache, float *out, int iters, double *ms);

/* The same attention through a paged K/V cache given by the caller: k_pool, v_pool are kv_heads x
 * num_pages x page x hd f16 (page a power of two, 8..65536); table[i] is the pool page holding
 * positions [i * page, (i + 1) * page) of the context, for every page of the pos0 + M positions. The
 * block's rows are rotated, rounded to f16 and written into their pages, and both pools are copied
 * back. No reference counterpart beyond src/model.rs:261-282: the page table is this build's cache
 * layout. */
int ls_attention_paged_host(uint64_t heads, uint64_t kv_heads, uint64_t hd, float rope_theta, uint64_t pos0, uint64_t M,
                            const float *qkv, uint16_t *k_pool, uint16_t *v_pool, uint64_t num_pages, uint64_t page,
                            const int32_t *table, float *out, int iters, double *ms);

/* The tensor-parallel reduction kernel of the row-parallel projections (O and down), run on one GPU
 * as rank `rank` of an emulated world of 2..8 ranks whose partials ys (world x n f32, this rank's own
 * at [rank]) all sit in this GPU's memory: x_out = x + calls x (ys[0] + ... + ys[world-1]), summed
 * in rank order as every rank sums them. preset = 1: the peers' ready flags are set before the
 * launches, so no launch waits; preset = 0: nothing sets them, the kernel's first wait runs out
 * after wait_ms, *status = 5 and LS_ERR_DEVICE is returned (the bounded-wait path). *ms = device
 * time per call. K > 0: the fused form the batch uses before every batched GEMM, over n / K rows of
 * K (K a multiple of 8): after the sum, op_out (n f16 values, row order) = f16(x_out * inv_rms * norm),
 * inv_rms = 1 / sqrt(mean(x_out^2) + eps) per row (norm NULL: no normalisation). In a
 * tensor-parallel batch the peers' partials and flags are the other ranks' buffers mapped over
 * NVLink; the kernel replaces an all-reduce of the projections' partial sums before the residual
 * adds after O and down (src/model.rs:283-297, on one device in the reference). */
int ls_tp_reduce_host(const float *x, const float *ys, uint32_t world, uint32_t rank, uint64_t n, int preset, uint32_t wait_ms,
                      int calls, float *x_out, int *status, double *ms, uint32_t K, const float *norm, float eps, uint16_t *op_out);

/* ChaCha20-Poly1305 (RFC 8439 section 2.8) on the GPU: the cipher of sealed model files
 * (src/seal.rs:340-400, seal_in_place / open_in_place). data: len bytes in host memory. seal = 1:
 * encrypted in place, tags written; seal = 0: every tag is checked, then the data decrypted in
 * place; LS_ERR_IO when a tag does not match (*bad_chunk = the lowest failing chunk, whose bytes are
 * left as they were). chunk_bytes = 0: one message under nonce[12] and aad. chunk_bytes > 0: chunks
 * of chunk_bytes (the last one shorter), chunk i under nonce[0..8) || le32(first + i) with
 * associated data aad || le32(first + i): the sealed file's per-chunk messages
 * (src/seal.rs:25-27); tags holds 16 bytes per chunk. iters > 1 (seal only): *ms = the device time of
 * one call over all chunks, averaged over iters launches. */
int ls_aead_host(int seal, const uint8_t *key, const uint8_t *nonce, const uint8_t *aad, uint64_t aad_len, uint8_t *data,
                 uint64_t len, uint64_t chunk_bytes, uint32_t first, uint8_t *tags, int iters, double *ms,
                 int64_t *bad_chunk);

/* The same GEMV on device buffers prepared once by ls_qweights_upload (for timing loops). */
typedef struct LsQWeights LsQWeights;
int ls_qweights_upload(int device, int bits, int group, const uint8_t *rows_raw, uint64_t rows, uint64_t cols,
                       LsQWeights **out);
int ls_qweights_free(LsQWeights *w);
/* x_dev: M x cols f32, y_dev: M x rows f32, both device pointers; stream: a cudaStream_t or NULL. */
int ls_qgemv_device(const LsQWeights *w, const float *x_dev, uint64_t M, float *y_dev, void *stream);

/* No counterpart in the reference. The GEMV above for hosts that cannot let this library allocate
 * device memory (their device memory belongs to another allocator, or to a fixed budget, so a
 * cudaMalloc here could fail, escape their accounting or synchronize the device mid-pipeline):
 * y_dev[t][r] = dot(stored row r, x_dev[t]) for t < M, the `rows` stored rows (.lsq row format,
 * rows x row_bytes) already in device memory the caller owns; x_dev M x cols f32, y_dev M x rows
 * f32 (rows_dev 2-byte, x_dev and y_dev 4-byte aligned), all on the current device; stream: a
 * cudaStream_t or NULL. The K-split partial sums go to a fixed 4 MiB array in the library's device
 * memory that every GPU loading the library holds until exit; requests beyond it (M > 16 or
 * M x rows > 262144) fail with LS_ERR_ARG. The first call on a device looks up that array's
 * address (once per device, kept for the life of the process), so make it before any stream
 * capture, and do not use the entry point on a device after cudaDeviceReset (the address kept
 * would belong to the context that was reset). All calls on a GPU share the array, and every
 * call overwrites what it reads: calls that overlap on the GPU (other streams, other threads)
 * race and must be serialized by the caller. */
int ls_qgemv_rows_noalloc(int bits, int group, const uint8_t *rows_dev, uint64_t rows, uint64_t cols, const float *x_dev,
                          uint64_t M, float *y_dev, void *stream);

/* Embedding gather + dequantisation of n stored rows (ids index `rows` stored rows in the .lsq row
 * format) into out (n x cols floats), through the same repack and gather kernels the model uses.
 * Mirrors kernels::dequant_row (src/kernels.rs:95-121); the result is bit-exact. */
int ls_dequant_rows_host(int bits, int group, const uint8_t *rows_raw, uint64_t rows, uint64_t cols, const uint32_t *ids,
                         uint64_t n, float *out);

/* Device bytes a kernel of this library reads per GEMV call (weights + scales + x + y). */
uint64_t ls_qgemv_bytes(int bits, int group, uint64_t rows, uint64_t cols, uint64_t M);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* LAYERSTREAM_B200_H */
