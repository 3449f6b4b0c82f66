// ChaCha20-Poly1305 (RFC 8439) on the GPU: the cipher of sealed model files (src/seal.rs), run
// on the ciphertext after it is copied to the device, so that streaming a sealed model is bound by
// the copy, not by host cores.
//
// A sealed file cuts its plaintext into chunks; every chunk is its own AEAD message (key, nonce =
// 8-byte file prefix || le32(chunk index), associated data = the file's frame and header ||
// le32(chunk index), 16-byte tag; src/seal.rs:13-27, 340-400). Opening a batch of chunks runs:
//
//   mac_partial_kernel   grid (segments, chunks): the Poly1305 sum of one segment of a chunk's
//                        MAC input (aad || pad || ciphertext || pad || le64 lengths), every thread
//                        a Horner run over its own blocks, combined with powers of r
//   mac_finish_kernel    one thread per chunk: the segments' sums added mod 2^130 - 5, plus s,
//                        compared with the stored tag (or written, when sealing)
//   chacha_xor_kernel    one thread per 64-byte block: keystream block (counter from 1) xor data,
//                        only for chunks whose tag matched (opening) or before the MAC (sealing)
//
// Poly1305 arithmetic: numbers mod p = 2^130 - 5 in five 26-bit limbs; a product's limbs are sums
// of 32 x 32 -> 64-bit products, the bits above 2^130 folded back times 5 (2^130 = 5 mod p).
// Integer arithmetic mod p is exact and associative, so the split into segments does not change
// the tag.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <vector>

#include "layerstream.h"
#include "ls_device.cuh"
#include "ls_internal.h"

namespace ls {

namespace {

// ---- ChaCha20 block function (RFC 8439 section 2.3) ----

__device__ __forceinline__ uint32_t rotl(uint32_t x, int n) { return __funnelshift_l(x, x, n); }

__device__ __forceinline__ void quarter(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  a += b;
  d = rotl(d ^ a, 16);
  c += d;
  b = rotl(b ^ c, 12);
  a += b;
  d = rotl(d ^ a, 8);
  c += d;
  b = rotl(b ^ c, 7);
}

// Keystream block `counter` of (key, nonce) as 16 little-endian words.
__device__ __forceinline__ void chacha_block(const uint32_t* key, uint32_t counter, const uint32_t* nonce, uint32_t* out) {
  uint32_t x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key[0], key[1],  key[2],  key[3],
                    key[4],      key[5],      key[6],      key[7],      counter, nonce[0], nonce[1], nonce[2]};
  uint32_t s[16];
#pragma unroll
  for (int i = 0; i < 16; i++) s[i] = x[i];
#pragma unroll
  for (int r = 0; r < 10; r++) {
    quarter(x[0], x[4], x[8], x[12]);
    quarter(x[1], x[5], x[9], x[13]);
    quarter(x[2], x[6], x[10], x[14]);
    quarter(x[3], x[7], x[11], x[15]);
    quarter(x[0], x[5], x[10], x[15]);
    quarter(x[1], x[6], x[11], x[12]);
    quarter(x[2], x[7], x[8], x[13]);
    quarter(x[3], x[4], x[9], x[14]);
  }
#pragma unroll
  for (int i = 0; i < 16; i++) out[i] = x[i] + s[i];
}

// ---- arithmetic mod 2^130 - 5 in five 26-bit limbs ----

struct P130 {
  uint32_t v[5];
};

__device__ __forceinline__ P130 p_zero() { return P130{{0, 0, 0, 0, 0}}; }
__device__ __forceinline__ P130 p_one() { return P130{{1, 0, 0, 0, 0}}; }

// Carry the 64-bit limb sums d into 26-bit limbs; the carry out of limb 4 (weight 2^130) re-enters
// limb 0 times 5. The result's limbs are < 2^26 except limb 1 (< 2^26 + small).
__device__ __forceinline__ P130 p_carry(uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t d4) {
  P130 h;
  d1 += d0 >> 26;
  h.v[0] = (uint32_t)d0 & 0x3ffffffu;
  d2 += d1 >> 26;
  h.v[1] = (uint32_t)d1 & 0x3ffffffu;
  d3 += d2 >> 26;
  h.v[2] = (uint32_t)d2 & 0x3ffffffu;
  d4 += d3 >> 26;
  h.v[3] = (uint32_t)d3 & 0x3ffffffu;
  const uint64_t c = d4 >> 26;
  h.v[4] = (uint32_t)d4 & 0x3ffffffu;
  const uint64_t t = (uint64_t)h.v[0] + c * 5;
  h.v[0] = (uint32_t)t & 0x3ffffffu;
  h.v[1] += (uint32_t)(t >> 26);
  return h;
}

// a * b mod p (not fully reduced: < 2^130 + small)
__device__ __forceinline__ P130 p_mul(const P130& a, const P130& b) {
  const uint64_t a0 = a.v[0], a1 = a.v[1], a2 = a.v[2], a3 = a.v[3], a4 = a.v[4];
  const uint64_t b0 = b.v[0], b1 = b.v[1], b2 = b.v[2], b3 = b.v[3], b4 = b.v[4];
  const uint64_t s1 = b1 * 5, s2 = b2 * 5, s3 = b3 * 5, s4 = b4 * 5;
  const uint64_t d0 = a0 * b0 + a1 * s4 + a2 * s3 + a3 * s2 + a4 * s1;
  const uint64_t d1 = a0 * b1 + a1 * b0 + a2 * s4 + a3 * s3 + a4 * s2;
  const uint64_t d2 = a0 * b2 + a1 * b1 + a2 * b0 + a3 * s4 + a4 * s3;
  const uint64_t d3 = a0 * b3 + a1 * b2 + a2 * b1 + a3 * b0 + a4 * s4;
  const uint64_t d4 = a0 * b4 + a1 * b3 + a2 * b2 + a3 * b1 + a4 * b0;
  return p_carry(d0, d1, d2, d3, d4);
}

__device__ __forceinline__ P130 p_add(const P130& a, const P130& b) {
  return p_carry((uint64_t)a.v[0] + b.v[0], (uint64_t)a.v[1] + b.v[1], (uint64_t)a.v[2] + b.v[2],
                 (uint64_t)a.v[3] + b.v[3], (uint64_t)a.v[4] + b.v[4]);
}

// r^e mod p by squaring
__device__ __forceinline__ P130 p_pow(P130 r, uint64_t e) {
  P130 acc = p_one();
  while (e) {
    if (e & 1) acc = p_mul(acc, r);
    e >>= 1;
    if (e) r = p_mul(r, r);
  }
  return acc;
}

// A 16-byte little-endian block (four words) plus `hibit` (2^128 for a full block) as limbs.
__device__ __forceinline__ P130 p_block(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t hibit) {
  P130 m;
  m.v[0] = w0 & 0x3ffffffu;
  m.v[1] = ((w0 >> 26) | (w1 << 6)) & 0x3ffffffu;
  m.v[2] = ((w1 >> 20) | (w2 << 12)) & 0x3ffffffu;
  m.v[3] = ((w2 >> 14) | (w3 << 18)) & 0x3ffffffu;
  m.v[4] = (w3 >> 8) | hibit;
  return m;
}

// The fully reduced value's low 128 bits plus s (mod 2^128) as four words: the tag.
__device__ __forceinline__ void p_tag(P130 h, const uint32_t* s, uint32_t* tag) {
  // canonical limbs (each < 2^26, value < 2^130): carry through, folding the carry out of limb 4
  // back times 5; twice, then once more without a fold (nothing is left to fold by then)
  for (int pass = 0; pass < 3; pass++) {
    uint32_t c = 0;
    for (int i = 0; i < 5; i++) {
      const uint32_t t = h.v[i] + c;
      h.v[i] = t & 0x3ffffffu;
      c = t >> 26;
    }
    if (pass < 2) h.v[0] += c * 5;
  }
  // then subtract p if h >= p
  uint32_t g[5];
  uint32_t c = 5;
  for (int i = 0; i < 5; i++) {
    const uint32_t t = h.v[i] + c;
    g[i] = t & 0x3ffffffu;
    c = t >> 26;
  }
  // g = h + 5; h >= p exactly when g reaches 2^130 (the carry out of limb 4)
  const bool ge = c != 0;
  uint32_t f[5];
  for (int i = 0; i < 5; i++) f[i] = ge ? g[i] : h.v[i];
  const uint32_t w0 = f[0] | (f[1] << 26), w1 = (f[1] >> 6) | (f[2] << 20), w2 = (f[2] >> 12) | (f[3] << 14),
                 w3 = (f[3] >> 18) | (f[4] << 8);
  uint64_t t = (uint64_t)w0 + s[0];
  tag[0] = (uint32_t)t;
  t = (uint64_t)w1 + s[1] + (t >> 32);
  tag[1] = (uint32_t)t;
  t = (uint64_t)w2 + s[2] + (t >> 32);
  tag[2] = (uint32_t)t;
  t = (uint64_t)w3 + s[3] + (t >> 32);
  tag[3] = (uint32_t)t;
}

// ---- kernels ----

constexpr int SEAL_THREADS = 256;
constexpr int SEAL_SEG_BLOCKS = 4096;  // MAC blocks (16 bytes) per segment CTA: 64 KB of a chunk

// Word w (0..3) of MAC-input block j of chunk c: aad || pad16 || ciphertext || pad16 || le64(aad
// length) || le64(ciphertext length), the aad being the shared prefix followed by the chunk's tail.
struct MacInput {
  const AeadChunk* ch;
  const uint8_t* aad;
  uint32_t aad_len;
  __device__ uint32_t aad_total() const { return aad_len + ch->tail_len; }
  __device__ uint32_t aad_blocks() const { return (aad_total() + 15) / 16; }
  __device__ uint64_t ct_blocks() const { return (ch->len + 15) / 16; }
  __device__ uint64_t blocks() const { return aad_blocks() + ct_blocks() + 1; }
  __device__ uint8_t aad_byte(uint32_t i) const {
    if (i < aad_len) return aad[i];
    const uint32_t k = i - aad_len;
    return k < ch->tail_len ? (uint8_t)(ch->tail >> (8 * k)) : 0;
  }
  __device__ void block(uint64_t j, uint32_t* w) const {
    const uint32_t na = aad_blocks();
    if (j < na) {
      const uint32_t base = (uint32_t)j * 16;
      if (base + 16 <= aad_len && ((reinterpret_cast<uintptr_t>(aad) + base) & 15) == 0) {
        const uint4 v = *reinterpret_cast<const uint4*>(aad + base);
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
        return;
      }
      for (int q = 0; q < 4; q++)
        w[q] = (uint32_t)aad_byte(base + 4 * q) | ((uint32_t)aad_byte(base + 4 * q + 1) << 8) |
               ((uint32_t)aad_byte(base + 4 * q + 2) << 16) | ((uint32_t)aad_byte(base + 4 * q + 3) << 24);
      return;
    }
    const uint64_t jc = j - na;
    if (jc < ct_blocks()) {
      const uint64_t base = jc * 16;
      const uint8_t* d = ch->data;
      if (base + 16 <= ch->len && ((reinterpret_cast<uintptr_t>(d) + base) & 15) == 0) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(d + base));
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
        return;
      }
      for (int q = 0; q < 4; q++) {
        uint32_t x = 0;
        for (int e = 0; e < 4; e++) {
          const uint64_t i = base + 4 * q + e;
          if (i < ch->len) x |= (uint32_t)d[i] << (8 * e);
        }
        w[q] = x;
      }
      return;
    }
    const uint64_t al = aad_total(), cl = ch->len;
    w[0] = (uint32_t)al, w[1] = (uint32_t)(al >> 32), w[2] = (uint32_t)cl, w[3] = (uint32_t)(cl >> 32);
  }
};

// The Poly1305 key of chunk c: the first 32 bytes of keystream block 0; r clamped (RFC 8439 2.5).
__device__ void poly_key(const uint32_t* key, const uint32_t* nonce, P130* r, uint32_t* s) {
  uint32_t b[16];
  chacha_block(key, 0, nonce, b);
  const uint32_t t0 = b[0] & 0x0fffffffu, t1 = b[1] & 0x0ffffffcu, t2 = b[2] & 0x0ffffffcu, t3 = b[3] & 0x0ffffffcu;
  *r = p_block(t0, t1, t2, t3, 0);
  s[0] = b[4], s[1] = b[5], s[2] = b[6], s[3] = b[7];
}

// Segment sums: CTA (seg, c) covers MAC blocks [seg * SEAL_SEG_BLOCKS, +SEAL_SEG_BLOCKS) of chunk c;
// thread k a contiguous run of them (Horner: h = (h + m) r), weighted by r^(blocks after its run);
// the CTA's threads' terms summed mod p into part[c][seg].
__global__ void __launch_bounds__(SEAL_THREADS) mac_partial_kernel(const AeadChunk* chunks, const uint8_t* aad, uint32_t aad_len,
                                                                     const uint32_t* key, P130* part, int max_segs) {
  __shared__ P130 s_r;
  __shared__ P130 s_sum[SEAL_THREADS / 32];
  const int c = blockIdx.y, seg = blockIdx.x;
  MacInput in{&chunks[c], aad, aad_len};
  const uint64_t n = in.blocks();
  const uint64_t b0 = (uint64_t)seg * SEAL_SEG_BLOCKS;
  if (b0 >= n) {  // this chunk has fewer segments: an empty sum
    if (threadIdx.x == 0) part[(size_t)c * max_segs + seg] = p_zero();
    return;
  }
  if (threadIdx.x == 0) {
    uint32_t s[4];
    poly_key(key, in.ch->nonce, &s_r, s);
  }
  __syncthreads();
  const P130 r = s_r;
  const uint64_t b1 = min(n, b0 + SEAL_SEG_BLOCKS), nb = b1 - b0;
  const uint64_t lo = b0 + nb * threadIdx.x / SEAL_THREADS, hi = b0 + nb * (threadIdx.x + 1) / SEAL_THREADS;
  P130 h = p_zero();
  for (uint64_t j = lo; j < hi; j++) {
    uint32_t w[4];
    in.block(j, w);
    h = p_mul(p_add(h, p_block(w[0], w[1], w[2], w[3], 1u << 24)), r);
  }
  if (hi > lo) h = p_mul(h, p_pow(r, n - hi));
  // sum over the warp, then over the warps, mod p (exact: the order does not matter)
  for (int o = 16; o > 0; o >>= 1) {
    P130 t;
    for (int q = 0; q < 5; q++) t.v[q] = __shfl_xor_sync(0xffffffffu, h.v[q], o);
    h = p_add(h, t);
  }
  if ((threadIdx.x & 31) == 0) s_sum[threadIdx.x >> 5] = h;
  __syncthreads();
  if (threadIdx.x == 0) {
    P130 t = s_sum[0];
    for (int w = 1; w < SEAL_THREADS / 32; w++) t = p_add(t, s_sum[w]);
    part[(size_t)c * max_segs + seg] = t;
  }
}

// One thread per chunk: the tag of its segment sums; open: ok[c] = (tag == stored tag), a mismatch
// records the lowest failing chunk + 1 in *bad (atomicMin over a value preset to INT_MAX); seal:
// the tag is stored and ok[c] = 1.
__global__ void mac_finish_kernel(AeadChunk* chunks, int nchunks, const uint32_t* key, const P130* part, int max_segs,
                                  int seal, uint32_t* ok, int* bad) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= nchunks) return;
  P130 r;
  uint32_t s[4], tag[4];
  poly_key(key, chunks[c].nonce, &r, s);
  P130 h = p_zero();
  for (int g = 0; g < max_segs; g++) h = p_add(h, part[(size_t)c * max_segs + g]);
  p_tag(h, s, tag);
  if (seal) {
    for (int q = 0; q < 4; q++) chunks[c].tag[q] = tag[q];
    ok[c] = 1;
    return;
  }
  const uint32_t diff = (tag[0] ^ chunks[c].tag[0]) | (tag[1] ^ chunks[c].tag[1]) | (tag[2] ^ chunks[c].tag[2]) |
                        (tag[3] ^ chunks[c].tag[3]);
  ok[c] = diff == 0;
  if (diff) atomicMin(bad, c + 1);
}

// Keystream xor: thread = one 64-byte block of a chunk (counter 1 + block), grid.y = chunk; only
// chunks with ok[c] (opening: their tag matched); ok == nullptr: every chunk (sealing).
__global__ void __launch_bounds__(SEAL_THREADS) chacha_xor_kernel(const AeadChunk* chunks, const uint32_t* key, const uint32_t* ok) {
  const int c = blockIdx.y;
  if (ok && !ok[c]) return;
  const AeadChunk& ch = chunks[c];
  const uint64_t nblk = (ch.len + 63) / 64;
  for (uint64_t b = (uint64_t)blockIdx.x * SEAL_THREADS + threadIdx.x; b < nblk; b += (uint64_t)gridDim.x * SEAL_THREADS) {
    uint32_t ks[16];
    chacha_block(key, (uint32_t)(1 + b), ch.nonce, ks);
    uint8_t* d = ch.data + b * 64;
    const uint64_t n = min((uint64_t)64, ch.len - b * 64);
    if (n == 64 && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
      uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        uint4 v = d4[q];
        v.x ^= ks[4 * q], v.y ^= ks[4 * q + 1], v.z ^= ks[4 * q + 2], v.w ^= ks[4 * q + 3];
        d4[q] = v;
      }
    } else {  // the chunk's last, partial block (or an unaligned one)
#pragma unroll
      for (int q = 0; q < 16; q++)
#pragma unroll
        for (int e = 0; e < 4; e++)
          if ((uint64_t)(4 * q + e) < n) d[4 * q + e] ^= (uint8_t)(ks[q] >> (8 * e));
    }
  }
}

}  // namespace

size_t aead_scratch_bytes(int nchunks, uint64_t max_len, uint32_t aad_len) {
  const uint64_t blocks = (aad_len + 4 + 15) / 16 + (max_len + 15) / 16 + 1;
  const uint64_t segs = (blocks + SEAL_SEG_BLOCKS - 1) / SEAL_SEG_BLOCKS;
  return (size_t)nchunks * segs * sizeof(P130) + (size_t)nchunks * 4;
}

void launch_aead(AeadChunk* d_chunks, int nchunks, uint64_t max_len, const uint8_t* d_aad, uint32_t aad_len, const uint32_t* d_key,
                 bool seal, void* scratch, size_t scratch_bytes, int* d_bad, cudaStream_t s) {
  if (nchunks <= 0) return;
  const uint64_t blocks = (aad_len + 4 + 15) / 16 + (max_len + 15) / 16 + 1;
  const int segs = (int)((blocks + SEAL_SEG_BLOCKS - 1) / SEAL_SEG_BLOCKS);
  if (aead_scratch_bytes(nchunks, max_len, aad_len) > scratch_bytes) LS_THROW(-1, "AEAD scratch too small");
  if (nchunks > 65535) LS_THROW(-1, "too many AEAD chunks in one launch");
  P130* part = static_cast<P130*>(scratch);
  uint32_t* ok = reinterpret_cast<uint32_t*>(part + (size_t)nchunks * segs);
  // a 64-byte keystream block per thread: enough CTAs for the longest chunk, at most 1024 per chunk
  const int xblocks = (int)std::min<uint64_t>(1024, ((max_len + 63) / 64 + SEAL_THREADS - 1) / SEAL_THREADS);
  if (seal) {
    chacha_xor_kernel<<<dim3(std::max(1, xblocks), nchunks), SEAL_THREADS, 0, s>>>(d_chunks, d_key, nullptr);
    LS_CUDA(cudaGetLastError());
  }
  mac_partial_kernel<<<dim3(segs, nchunks), SEAL_THREADS, 0, s>>>(d_chunks, d_aad, aad_len, d_key, part, segs);
  LS_CUDA(cudaGetLastError());
  mac_finish_kernel<<<(nchunks + 127) / 128, 128, 0, s>>>(d_chunks, nchunks, d_key, part, segs, seal ? 1 : 0, ok, d_bad);
  LS_CUDA(cudaGetLastError());
  if (!seal) {
    chacha_xor_kernel<<<dim3(std::max(1, xblocks), nchunks), SEAL_THREADS, 0, s>>>(d_chunks, d_key, ok);
    LS_CUDA(cudaGetLastError());
  }
}

// Host-buffer AEAD (test and timing entry): `data` (len bytes) cut into chunks of chunk_bytes (0:
// one message); indexed: chunk i uses nonce = nonce12[0..8) || le32(first + i) and the aad tail
// le32(first + i) (the sealed-file convention), else the one message uses nonce12 and aad alone.
// tags: n x 16 bytes, read (open) or written (seal). Returns the lowest failing chunk, or -1.
// iters > 1 (seal only): ms = the device time of one seal of all chunks, averaged over iters
// back-to-back launches on the device copy (the result returned is the first one's).
int aead_host(bool seal, const uint8_t* key, const uint8_t* nonce12, bool indexed, uint32_t first, const uint8_t* aad,
              uint64_t aad_len, uint8_t* data, uint64_t len, uint64_t chunk_bytes, uint8_t* tags, int iters, double* ms) {
  if (aad_len > (64u << 20)) LS_THROW(LS_ERR_ARG, "associated data above 64 MiB");
  if (chunk_bytes == 0 || chunk_bytes > len) chunk_bytes = std::max<uint64_t>(len, 1);
  const uint64_t n64 = len == 0 ? 1 : (len + chunk_bytes - 1) / chunk_bytes;
  if (!indexed && n64 != 1) LS_THROW(LS_ERR_ARG, "several chunks need per-chunk nonces (indexed)");
  if (n64 > 65535) LS_THROW(LS_ERR_ARG, "at most 65535 chunks per call");
  const int n = (int)n64;
  std::vector<void*> owned;
  auto dmal = [&](size_t b) {
    void* p = nullptr;
    LS_CUDA(cudaMalloc(&p, std::max<size_t>(b, 16)));
    owned.push_back(p);
    return p;
  };
  struct Free {
    std::vector<void*>& o;
    ~Free() {
      cudaDeviceSynchronize();
      for (void* p : o) cudaFree(p);
    }
  } fr{owned};
  auto* dd = static_cast<uint8_t*>(dmal(len));
  auto* da = static_cast<uint8_t*>(dmal(aad_len));
  auto* dk = static_cast<uint32_t*>(dmal(32));
  auto* dc = static_cast<AeadChunk*>(dmal(sizeof(AeadChunk) * n));
  auto* dbad = static_cast<int*>(dmal(4));
  const size_t scratch = aead_scratch_bytes(n, chunk_bytes, (uint32_t)aad_len);
  void* dscr = dmal(scratch);
  std::vector<AeadChunk> ch(n);
  uint32_t kw[8], nw[3];
  std::memcpy(kw, key, 32);
  std::memcpy(nw, nonce12, 12);
  for (int i = 0; i < n; i++) {
    AeadChunk& c = ch[i];
    c.data = dd + (uint64_t)i * chunk_bytes;
    c.len = std::min<uint64_t>(chunk_bytes, len - std::min<uint64_t>(len, (uint64_t)i * chunk_bytes));
    c.nonce[0] = nw[0], c.nonce[1] = nw[1], c.nonce[2] = indexed ? first + (uint32_t)i : nw[2];
    c.tail = first + (uint32_t)i;
    c.tail_len = indexed ? 4 : 0;
    std::memcpy(c.tag, tags + (size_t)16 * i, 16);
  }
  const int big = 0x7fffffff;
  if (len) LS_CUDA(cudaMemcpy(dd, data, len, cudaMemcpyHostToDevice));
  if (aad_len) LS_CUDA(cudaMemcpy(da, aad, aad_len, cudaMemcpyHostToDevice));
  LS_CUDA(cudaMemcpy(dk, kw, 32, cudaMemcpyHostToDevice));
  LS_CUDA(cudaMemcpy(dc, ch.data(), sizeof(AeadChunk) * n, cudaMemcpyHostToDevice));
  LS_CUDA(cudaMemcpy(dbad, &big, 4, cudaMemcpyHostToDevice));
  launch_aead(dc, n, chunk_bytes, da, (uint32_t)aad_len, dk, seal, dscr, scratch, dbad, 0);
  LS_CUDA(cudaDeviceSynchronize());
  int bad = big;
  LS_CUDA(cudaMemcpy(&bad, dbad, 4, cudaMemcpyDeviceToHost));
  if (len) LS_CUDA(cudaMemcpy(data, dd, len, cudaMemcpyDeviceToHost));
  LS_CUDA(cudaMemcpy(ch.data(), dc, sizeof(AeadChunk) * n, cudaMemcpyDeviceToHost));
  if (seal)
    for (int i = 0; i < n; i++) std::memcpy(tags + (size_t)16 * i, ch[i].tag, 16);
  if (ms) *ms = 0;
  if (seal && iters > 1 && ms) {
    cudaEvent_t e0, e1;
    LS_CUDA(cudaEventCreate(&e0));
    LS_CUDA(cudaEventCreate(&e1));
    LS_CUDA(cudaEventRecord(e0, 0));
    for (int it = 0; it < iters; it++) launch_aead(dc, n, chunk_bytes, da, (uint32_t)aad_len, dk, true, dscr, scratch, dbad, 0);
    LS_CUDA(cudaEventRecord(e1, 0));
    LS_CUDA(cudaEventSynchronize(e1));
    float t = 0;
    LS_CUDA(cudaEventElapsedTime(&t, e0, e1));
    *ms = (double)t / iters;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  return bad == big ? -1 : bad - 1;
}

size_t seal_model_file(const std::string& src, const std::string& out, const uint8_t* key, const uint8_t* nonce_prefix,
                       size_t layer_chunk, size_t embed_chunk_rows) {
  if (layer_chunk == 0 || embed_chunk_rows == 0) LS_THROW(LS_ERR_ARG, "chunk sizes must be positive");
  // the plaintext: every layer block, the embedding table, the final norm (src/seal.rs:726-827)
  std::string config_text, data_path;
  Config cfg;
  LayerLayout layout;
  std::vector<uint64_t> layer_start;
  uint64_t embed_start = 0, norm_start = 0;
  struct stat st;
  if (::stat(src.c_str(), &st) == 0 && S_ISDIR(st.st_mode)) {
    const SafetensorsModel m = SafetensorsModel::open(src);
    config_text = m.config_text, data_path = m.file, cfg = m.cfg, layout = m.layout, layer_start = m.layer_start;
    embed_start = m.embed_start, norm_start = m.norm_start;
  } else {
    const LsqFile q = LsqFile::open(src);
    config_text = q.config_text, data_path = q.path, cfg = q.cfg, layout = q.layout;
    for (size_t l = 0; l < cfg.layers; l++) layer_start.push_back(q.data_start + l * layout.total);
    embed_start = q.embed_start, norm_start = q.norm_start;
  }
  const size_t rb = cfg.embed_row_bytes(), norm_bytes = cfg.hidden * 2;
  const std::string header = sealed_header_json(config_text, layout, layer_chunk, embed_chunk_rows, norm_bytes);
  std::vector<uint8_t> frame(kSealFrame);
  std::memcpy(frame.data(), "LSS1", 4);
  const uint32_t ver = 1, hl = (uint32_t)header.size();
  std::memcpy(frame.data() + 4, &ver, 4);
  std::memcpy(frame.data() + 8, nonce_prefix, 8);
  std::memcpy(frame.data() + 16, &hl, 4);
  frame.insert(frame.end(), header.begin(), header.end());
  const size_t lc = (layout.total + layer_chunk - 1) / layer_chunk, ec = (cfg.vocab + embed_chunk_rows - 1) / embed_chunk_rows;
  const size_t n_chunks = cfg.layers * lc + ec + 1;
  std::vector<uint8_t> tags(16 * n_chunks, 0);

  const int in = ::open(data_path.c_str(), O_RDONLY);
  if (in < 0) LS_THROW(LS_ERR_IO, data_path + ": cannot open");
  const int fo = ::open(out.c_str(), O_WRONLY | O_CREAT | O_EXCL, 0644);
  if (fo < 0) {
    ::close(in);
    LS_THROW(LS_ERR_IO, out + ": " + std::strerror(errno));
  }
  struct Files {
    int a, b;
    ~Files() {
      ::close(a);
      ::close(b);
    }
  } files{in, fo};
  auto write_all = [&](const uint8_t* p, size_t n, uint64_t off) {
    size_t done = 0;
    while (done < n) {
      const ssize_t w = ::pwrite(fo, p + done, n - done, (off_t)(off + done));
      if (w < 0 && errno == EINTR) continue;
      if (w <= 0) LS_THROW(LS_ERR_IO, out + ": write failed");
      done += (size_t)w;
    }
  };
  write_all(frame.data(), frame.size(), 0);
  write_all(tags.data(), tags.size(), frame.size());
  uint64_t wpos = frame.size() + tags.size();

  // one section at a time through one host and one device buffer: a layer block, up to 16 chunks of
  // table rows, the norm
  const size_t erows = embed_chunk_rows * 16;
  const size_t buf_bytes = std::max({layout.total, std::min(erows, cfg.vocab) * rb, norm_bytes});
  std::vector<uint8_t> hbuf(buf_bytes);
  uint8_t *dbuf = nullptr, *daad = nullptr;
  uint32_t* dkey = nullptr;
  AeadChunk* dch = nullptr;
  void* scr = nullptr;
  const size_t max_ch = std::max<size_t>({lc, 16, 1});
  const size_t scr_bytes = std::max({aead_scratch_bytes((int)max_ch, layer_chunk, (uint32_t)frame.size()),
                                     aead_scratch_bytes((int)max_ch, embed_chunk_rows * rb, (uint32_t)frame.size()),
                                     aead_scratch_bytes(1, norm_bytes, (uint32_t)frame.size())});
  LS_CUDA(cudaMalloc(&dbuf, buf_bytes));
  LS_CUDA(cudaMalloc(&daad, frame.size()));
  LS_CUDA(cudaMalloc(&dkey, 32));
  LS_CUDA(cudaMalloc(&dch, max_ch * sizeof(AeadChunk)));
  LS_CUDA(cudaMalloc(&scr, scr_bytes));
  struct Dev {
    void* p[5];
    ~Dev() {
      cudaDeviceSynchronize();
      for (void* q : p) cudaFree(q);
    }
  } dev{{dbuf, daad, dkey, dch, scr}};
  LS_CUDA(cudaMemcpy(daad, frame.data(), frame.size(), cudaMemcpyHostToDevice));
  LS_CUDA(cudaMemcpy(dkey, key, 32, cudaMemcpyHostToDevice));
  // seals n plaintext bytes read at file offset `off` as chunks first.. of clen bytes
  auto seal_section = [&](uint64_t off, size_t n, size_t first, size_t clen) {
    pread_all(in, hbuf.data(), n, off);
    const size_t nch = (n + clen - 1) / clen;
    std::vector<AeadChunk> ch(nch);
    for (size_t i = 0; i < nch; i++) {
      AeadChunk& c = ch[i];
      c = AeadChunk{};
      c.data = dbuf + i * clen;
      c.len = std::min<uint64_t>(clen, n - i * clen);
      std::memcpy(c.nonce, nonce_prefix, 8);
      c.nonce[2] = (uint32_t)(first + i);
      c.tail = (uint32_t)(first + i);
      c.tail_len = 4;
    }
    LS_CUDA(cudaMemcpy(dbuf, hbuf.data(), n, cudaMemcpyHostToDevice));
    LS_CUDA(cudaMemcpy(dch, ch.data(), nch * sizeof(AeadChunk), cudaMemcpyHostToDevice));
    launch_aead(dch, (int)nch, clen, daad, (uint32_t)frame.size(), dkey, true, scr, scr_bytes, nullptr, 0);
    LS_CUDA(cudaMemcpy(hbuf.data(), dbuf, n, cudaMemcpyDeviceToHost));
    LS_CUDA(cudaMemcpy(ch.data(), dch, nch * sizeof(AeadChunk), cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < nch; i++) std::memcpy(&tags[16 * (first + i)], ch[i].tag, 16);
    write_all(hbuf.data(), n, wpos);
    wpos += n;
  };
  for (size_t l = 0; l < cfg.layers; l++) seal_section(layer_start[l], layout.total, l * lc, layer_chunk);
  for (size_t first = 0; first < cfg.vocab; first += erows) {
    const size_t rows = std::min(erows, cfg.vocab - first);
    seal_section(embed_start + first * rb, rows * rb, cfg.layers * lc + first / embed_chunk_rows, embed_chunk_rows * rb);
  }
  seal_section(norm_start, norm_bytes, n_chunks - 1, norm_bytes);
  write_all(tags.data(), tags.size(), frame.size());
  if (::fsync(fo) != 0) LS_THROW(LS_ERR_IO, out + ": fsync failed");
  return n_chunks;
}

}  // namespace ls
