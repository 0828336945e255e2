// SHA-256 compression for sm_100a, integer-only, registers-only.
//
// FIPS 180-4 SHA-256 -- the function of the `sha2` crate v0.10.9 that
// verilm-core hashes with (crates/verilm-core/Cargo.toml:7).  Digests are kept
// as eight 32-bit words in SHA-256's own (big-endian) word order; in memory a
// digest is the 32 output bytes, i.e. each word stored big-endian.
#pragma once
#include <cstdint>

namespace vc {

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// Round constants (FIPS 180-4 section 4.2.2).
struct U32x64 { uint32_t v[64]; };

constexpr U32x64 kRoundK = {{
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u}};


constexpr uint32_t c_rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

// K[t] + W[t] for a block whose 16 message words are known at compile time;
// used for the all-padding second block of a 64-byte message
// (0x80000000, 0 x 14, bit length 512).
constexpr U32x64 make_const_block_kw(uint32_t w0, uint32_t w15) {
  U32x64 w{};
  for (int i = 0; i < 16; ++i) w.v[i] = 0;
  w.v[0] = w0;
  w.v[15] = w15;
  for (int t = 16; t < 64; ++t) {
    uint32_t s0 = c_rotr(w.v[t - 15], 7) ^ c_rotr(w.v[t - 15], 18) ^ (w.v[t - 15] >> 3);
    uint32_t s1 = c_rotr(w.v[t - 2], 17) ^ c_rotr(w.v[t - 2], 19) ^ (w.v[t - 2] >> 10);
    w.v[t] = w.v[t - 16] + s0 + w.v[t - 7] + s1;
  }
  U32x64 kw{};
  for (int t = 0; t < 64; ++t) kw.v[t] = kRoundK.v[t] + w.v[t];
  return kw;
}
// Device copies.  Indexed only with unrolled (compile-time) round numbers, so
// they become constant-bank operands of the adds.
static __constant__ U32x64 c_K = kRoundK;
static __constant__ U32x64 c_Pad64KW = make_const_block_kw(0x80000000u, 512u);

__device__ __forceinline__ uint32_t Sig0(uint32_t a) { return rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22); }
__device__ __forceinline__ uint32_t Sig1(uint32_t e) { return rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25); }
__device__ __forceinline__ uint32_t sig0(uint32_t x) { return rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3); }
__device__ __forceinline__ uint32_t sig1(uint32_t x) { return rotr(x, 17) ^ rotr(x, 19) ^ (x >> 10); }
__device__ __forceinline__ uint32_t Ch(uint32_t e, uint32_t f, uint32_t g) { return (e & f) ^ (~e & g); }
__device__ __forceinline__ uint32_t Maj(uint32_t a, uint32_t b, uint32_t c) { return (a & b) | (c & (a | b)); }

#define VC_SHA_ROUND(a, b, c, d, e, f, g, h, kw)                 \
  do {                                                           \
    uint32_t t1_ = (h) + Sig1(e) + Ch((e), (f), (g)) + (kw);     \
    uint32_t t2_ = Sig0(a) + Maj((a), (b), (c));                 \
    (d) += t1_;                                                  \
    (h) = t1_ + t2_;                                             \
  } while (0)

// One compression of the 16 message words w (consumed: w is overwritten by
// the message schedule).  Words set to literal zeros by the caller fold away
// once inlined.
__device__ __forceinline__ void compress(uint32_t st[8], uint32_t w[16]) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int t = 0; t < 64; t += 8) {
    if (t >= 16) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = (t + i) & 15;
        w[j] += sig1(w[(j + 14) & 15]) + w[(j + 9) & 15] + sig0(w[(j + 1) & 15]);
      }
    }
    const int j = t & 15;
    VC_SHA_ROUND(a, b, c, d, e, f, g, h, c_K.v[t + 0] + w[j + 0]);
    VC_SHA_ROUND(h, a, b, c, d, e, f, g, c_K.v[t + 1] + w[j + 1]);
    VC_SHA_ROUND(g, h, a, b, c, d, e, f, c_K.v[t + 2] + w[j + 2]);
    VC_SHA_ROUND(f, g, h, a, b, c, d, e, c_K.v[t + 3] + w[j + 3]);
    VC_SHA_ROUND(e, f, g, h, a, b, c, d, c_K.v[t + 4] + w[j + 4]);
    VC_SHA_ROUND(d, e, f, g, h, a, b, c, c_K.v[t + 5] + w[j + 5]);
    VC_SHA_ROUND(c, d, e, f, g, h, a, b, c_K.v[t + 6] + w[j + 6]);
    VC_SHA_ROUND(b, c, d, e, f, g, h, a, c_K.v[t + 7] + w[j + 7]);
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

// Compression of the constant padding block of a 64-byte message.
__device__ __forceinline__ void compress_pad64(uint32_t st[8]) {
  const U32x64& kw = c_Pad64KW;
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int t = 0; t < 64; t += 8) {
    VC_SHA_ROUND(a, b, c, d, e, f, g, h, kw.v[t + 0]);
    VC_SHA_ROUND(h, a, b, c, d, e, f, g, kw.v[t + 1]);
    VC_SHA_ROUND(g, h, a, b, c, d, e, f, kw.v[t + 2]);
    VC_SHA_ROUND(f, g, h, a, b, c, d, e, kw.v[t + 3]);
    VC_SHA_ROUND(e, f, g, h, a, b, c, d, kw.v[t + 4]);
    VC_SHA_ROUND(d, e, f, g, h, a, b, c, kw.v[t + 5]);
    VC_SHA_ROUND(c, d, e, f, g, h, a, b, kw.v[t + 6]);
    VC_SHA_ROUND(b, c, d, e, f, g, h, a, kw.v[t + 7]);
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

__device__ __forceinline__ void sha_init(uint32_t st[8]) {
  st[0] = 0x6a09e667u; st[1] = 0xbb67ae85u; st[2] = 0x3c6ef372u; st[3] = 0xa54ff53au;
  st[4] = 0x510e527fu; st[5] = 0x9b05688cu; st[6] = 0x1f83d9abu; st[7] = 0x5be0cd19u;
}

// merkle.rs:118-123 hash_pair: SHA256(left || right), a 64-byte message.
__device__ __forceinline__ void hash_pair(const uint32_t l[8], const uint32_t r[8], uint32_t out[8]) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) { w[i] = l[i]; w[8 + i] = r[i]; }
  sha_init(out);
  compress(out, w);
  compress_pad64(out);
}

// Digest <-> memory (32 bytes, SHA-256 output byte order).
__device__ __forceinline__ void store_digest(uint8_t* p, const uint32_t h[8]) {
  uint4 lo = make_uint4(bswap32(h[0]), bswap32(h[1]), bswap32(h[2]), bswap32(h[3]));
  uint4 hi = make_uint4(bswap32(h[4]), bswap32(h[5]), bswap32(h[6]), bswap32(h[7]));
  reinterpret_cast<uint4*>(p)[0] = lo;
  reinterpret_cast<uint4*>(p)[1] = hi;
}

__device__ __forceinline__ void load_digest(const uint8_t* p, uint32_t h[8]) {
  uint4 lo = reinterpret_cast<const uint4*>(p)[0];
  uint4 hi = reinterpret_cast<const uint4*>(p)[1];
  h[0] = bswap32(lo.x); h[1] = bswap32(lo.y); h[2] = bswap32(lo.z); h[3] = bswap32(lo.w);
  h[4] = bswap32(hi.x); h[5] = bswap32(hi.y); h[6] = bswap32(hi.z); h[7] = bswap32(hi.w);
}

// L1-bypassing load, for digests written by other CTAs of the same grid.
__device__ __forceinline__ void load_digest_cg(const uint8_t* p, uint32_t h[8]) {
  uint4 lo = __ldcg(reinterpret_cast<const uint4*>(p));
  uint4 hi = __ldcg(reinterpret_cast<const uint4*>(p) + 1);
  h[0] = bswap32(lo.x); h[1] = bswap32(lo.y); h[2] = bswap32(lo.z); h[3] = bswap32(lo.w);
  h[4] = bswap32(hi.x); h[5] = bswap32(hi.y); h[6] = bswap32(hi.z); h[7] = bswap32(hi.w);
}

}  // namespace vc
