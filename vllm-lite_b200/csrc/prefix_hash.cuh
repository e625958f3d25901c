// Content hash of a full KV block, bit-identical to vllm-lite's hash_block
// (vllmlite/block.py:34-40):
//   blake2b(digest_size=16) over  [prev_hex] "|" ",".join(str(t) for t in tokens)
// returned as 32 lowercase hex characters; the previous block's hex digest is
// left out when there is none (the first block of a sequence). The chain of a
// sequence's full blocks feeds each digest into the next block's message
// (block_manager.py:98-120).
//
// BLAKE2b follows its published specification (RFC 7693): 64-bit words, 12
// rounds of the G mixing function over a 16-word working vector, 128-byte
// message blocks counted in bytes, the last block zero-padded and flagged,
// parameter word 0x01010000 ^ digest length for an unkeyed hash. Everything
// is plain integer arithmetic written as __host__ __device__ code, so the same
// functions run in the kernel and, compiled by a host compiler, in the CPU
// tests that compare them with hashlib.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__
#ifndef __host__
#define __host__
#endif
#ifndef __device__
#define __device__
#endif
#endif

namespace vllt {
namespace blake2b {

__host__ __device__ inline uint64_t rotr(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

// initialisation vector (RFC 7693 section 2.6)
__host__ __device__ inline uint64_t iv(int i) {
  switch (i) {
    case 0: return 0x6a09e667f3bcc908ull;
    case 1: return 0xbb67ae8584caa73bull;
    case 2: return 0x3c6ef372fe94f82bull;
    case 3: return 0xa54ff53a5f1d36f1ull;
    case 4: return 0x510e527fade682d1ull;
    case 5: return 0x9b05688c2b3e6c1full;
    case 6: return 0x1f83d9abfb41bd6bull;
    default: return 0x5be0cd19137e2179ull;
  }
}

// message schedule of round r (RFC 7693 section 2.7), packed 4 bits per entry
__host__ __device__ inline int sigma(int r, int i) {
  // rows 0..9; rounds 10 and 11 repeat rows 0 and 1
  const uint64_t rows[10] = {
      0xfedcba9876543210ull, 0x357b20c16df984aeull, 0x491763eadf250c8bull, 0x8f04a562ebcd1397ull,
      0xd386cb1efa427509ull, 0x91ef57d438b0a6c2ull, 0xb8293670a4def15cull, 0xa2684f05931ce7bdull,
      0x5a417d2c803b9ef6ull, 0x0dc3e9bf5167482aull};
  return (int)((rows[r % 10] >> (4 * i)) & 15);
}

__host__ __device__ inline void g(uint64_t* v, int a, int b, int c, int d, uint64_t x, uint64_t y) {
  v[a] = v[a] + v[b] + x;
  v[d] = rotr(v[d] ^ v[a], 32);
  v[c] = v[c] + v[d];
  v[b] = rotr(v[b] ^ v[c], 24);
  v[a] = v[a] + v[b] + y;
  v[d] = rotr(v[d] ^ v[a], 16);
  v[c] = v[c] + v[d];
  v[b] = rotr(v[b] ^ v[c], 63);
}

// Compression function F (RFC 7693 section 3.2) of one 128-byte block.
__host__ __device__ inline void compress(uint64_t* h, const uint8_t* block, uint64_t t, bool last) {
  uint64_t m[16], v[16];
  for (int i = 0; i < 16; ++i) {
    uint64_t w = 0;
    for (int k = 7; k >= 0; --k) w = (w << 8) | block[8 * i + k];  // little-endian words
    m[i] = w;
  }
  for (int i = 0; i < 8; ++i) {
    v[i] = h[i];
    v[i + 8] = iv(i);
  }
  v[12] ^= t;  // byte counter, low word (messages here are far below 2^64 bytes)
  if (last) v[14] = ~v[14];
  for (int r = 0; r < 12; ++r) {
    g(v, 0, 4, 8, 12, m[sigma(r, 0)], m[sigma(r, 1)]);
    g(v, 1, 5, 9, 13, m[sigma(r, 2)], m[sigma(r, 3)]);
    g(v, 2, 6, 10, 14, m[sigma(r, 4)], m[sigma(r, 5)]);
    g(v, 3, 7, 11, 15, m[sigma(r, 6)], m[sigma(r, 7)]);
    g(v, 0, 5, 10, 15, m[sigma(r, 8)], m[sigma(r, 9)]);
    g(v, 1, 6, 11, 12, m[sigma(r, 10)], m[sigma(r, 11)]);
    g(v, 2, 7, 8, 13, m[sigma(r, 12)], m[sigma(r, 13)]);
    g(v, 3, 4, 9, 14, m[sigma(r, 14)], m[sigma(r, 15)]);
  }
  for (int i = 0; i < 8; ++i) h[i] ^= v[i] ^ v[i + 8];
}

// Streaming unkeyed BLAKE2b with a 16-byte digest. A block is compressed
// only when the next byte arrives, so the last block is known at finish().
struct State {
  uint64_t h[8];
  uint8_t buf[128];
  int n;       // bytes in buf
  uint64_t t;  // bytes compressed so far

  __host__ __device__ void init() {
    for (int i = 0; i < 8; ++i) h[i] = iv(i);
    h[0] ^= 0x01010000ull ^ 16ull;  // digest length 16, no key, fanout 1, depth 1
    n = 0;
    t = 0;
  }
  __host__ __device__ void put(uint8_t c) {
    if (n == 128) {
      t += 128;
      compress(h, buf, t, false);
      n = 0;
    }
    buf[n++] = c;
  }
  // 32 lowercase hex characters of the 16-byte digest
  __host__ __device__ void finish(uint8_t* hex) {
    t += (uint64_t)n;
    for (int i = n; i < 128; ++i) buf[i] = 0;
    compress(h, buf, t, true);
    const char* digits = "0123456789abcdef";
    for (int i = 0; i < 16; ++i) {
      const uint8_t b = (uint8_t)(h[i >> 3] >> (8 * (i & 7)));
      hex[2 * i] = (uint8_t)digits[b >> 4];
      hex[2 * i + 1] = (uint8_t)digits[b & 15];
    }
  }
};

}  // namespace blake2b

// Decimal digits of a token id, as Python's str(int) writes them.
__host__ __device__ inline void put_decimal(blake2b::State& s, int32_t v) {
  uint8_t d[11];
  int k = 0;
  int64_t x = v;
  if (x < 0) {
    s.put('-');
    x = -x;
  }
  do {
    d[k++] = (uint8_t)('0' + x % 10);
    x /= 10;
  } while (x);
  while (k) s.put(d[--k]);
}

// hash_block(prev, tokens): prev_hex is 32 hex characters, or NULL / a first
// byte of 0 for "no previous block" (block.py:36-37 skips a falsy prev_hash).
__host__ __device__ inline void hash_block(const uint8_t* prev_hex, const int32_t* tokens, int n, uint8_t* out_hex) {
  blake2b::State s;
  s.init();
  if (prev_hex && prev_hex[0])
    for (int i = 0; i < 32; ++i) s.put(prev_hex[i]);
  s.put('|');
  for (int i = 0; i < n; ++i) {
    if (i) s.put(',');
    put_decimal(s, tokens[i]);
  }
  s.finish(out_hex);
}

// One sequence's chain: n_blocks full blocks of block_size tokens, each
// block's digest the next block's prev (block_manager.py:109-120).
__host__ __device__ inline void hash_chain(const uint8_t* prev_hex, const int32_t* tokens, int n_blocks,
                                           int block_size, uint8_t* out_hex) {
  const uint8_t* prev = prev_hex;
  for (int b = 0; b < n_blocks; ++b) {
    hash_block(prev, tokens + (int64_t)b * block_size, block_size, out_hex + 32 * b);
    prev = out_hex + 32 * b;
  }
}

}  // namespace vllt
