// SHA-256 compression with its work split between the ALU and FMA pipes.
//
// On sm_100a the funnel shifts, 3-input logic ops and 3-input adds of a
// plain SHA-256 round all issue to the integer ALU pipe, which accepts one
// warp instruction every other cycle per SM sub-partition, while the FMA
// pipe (IMAD) stays idle.  Here some of the work is written as IMAD forms:
//   a + b             = mad.lo(a, one, b)
//   x >> n            = mul.hi(x, 2^(32-n))
//   rotr(x, n)        = mad.lo(x, 2^(32-n), mul.hi(x, 2^(32-n)))   (disjoint bits)
// The multipliers come from a kernel parameter (Opq), so the compiler cannot
// see their values and fold the IMADs back into ALU shifts and adds.
// Which operations move is chosen by the template flags; the arithmetic is
// FIPS 180-4 SHA-256 either way.
#pragma once
#include "sha256_core.cuh"
#include "sha256_opq.h"

namespace vc {

__device__ __forceinline__ uint32_t fadd(uint32_t a, uint32_t b, uint32_t one) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(one), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t fshr(uint32_t x, uint32_t m) {
  uint32_t r;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(m));
  return r;
}
__device__ __forceinline__ uint32_t frotr(uint32_t x, uint32_t m) {
  uint32_t hi, r;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(hi) : "r"(x), "r"(m));
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(m), "r"(hi));
  return r;
}
__device__ __forceinline__ uint32_t lop_xor3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x96;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Flags: which operations go to the FMA pipe.
enum : int {
  kAddRound = 1,     // the 4 add groups of a round (7 IMADs instead of 4 IADD3)
  kAddSched = 2,     // the schedule's 4-term add (3 IMADs instead of 2 IADD)
  kShrSched = 4,     // sigma0's shr 3 and sigma1's shr 10 as mul.hi
  kRotS0a = 8,       // one rotation of Sigma0 (rotr 2)
  kRotS0b = 16,      // a second rotation of Sigma0 (rotr 13)
  kRotS1a = 32,      // one rotation of Sigma1 (rotr 6)
  kAddHalf = 64,     // round: only G1 (h+K+W) and G3 (d += t1) as IMAD
  kRotSched = 128,   // one rotation of each schedule sigma (rotr 7, rotr 17)
};

template <int F>
__device__ __forceinline__ uint32_t bSig0(uint32_t a, const Opq& o) {
  const uint32_t r2 = (F & kRotS0a) ? frotr(a, o.m2) : rotr(a, 2);
  const uint32_t r13 = (F & kRotS0b) ? frotr(a, o.m13) : rotr(a, 13);
  return lop_xor3(r2, r13, rotr(a, 22));
}
template <int F>
__device__ __forceinline__ uint32_t bSig1(uint32_t e, const Opq& o) {
  const uint32_t r6 = (F & kRotS1a) ? frotr(e, o.m6) : rotr(e, 6);
  return lop_xor3(r6, rotr(e, 11), rotr(e, 25));
}
template <int F>
__device__ __forceinline__ uint32_t bsig0(uint32_t x, const Opq& o) {
  const uint32_t s = (F & kShrSched) ? fshr(x, o.m3) : (x >> 3);
  const uint32_t r7 = (F & kRotSched) ? frotr(x, o.m7) : rotr(x, 7);
  return lop_xor3(r7, rotr(x, 18), s);
}
template <int F>
__device__ __forceinline__ uint32_t bsig1(uint32_t x, const Opq& o) {
  const uint32_t s = (F & kShrSched) ? fshr(x, o.m10) : (x >> 10);
  const uint32_t r17 = (F & kRotSched) ? frotr(x, o.m17) : rotr(x, 17);
  return lop_xor3(r17, rotr(x, 19), s);
}

template <int F>
__device__ __forceinline__ void bround(uint32_t a, uint32_t b, uint32_t c, uint32_t& d, uint32_t e, uint32_t f,
                                       uint32_t g, uint32_t& h, uint32_t k, uint32_t w, const Opq& o) {
  const uint32_t s1 = bSig1<F>(e, o);
  const uint32_t s0 = bSig0<F>(a, o);
  const uint32_t ch = Ch(e, f, g);
  const uint32_t mj = Maj(a, b, c);
  if (F & kAddRound) {
    const uint32_t hk = fadd(fadd(h, w, o.one), k, o.one);   // G1: h + W + K
    const uint32_t t1 = fadd(fadd(hk, s1, o.one), ch, o.one);
    d = fadd(d, t1, o.one);
    h = fadd(fadd(t1, s0, o.one), mj, o.one);
  } else if (F & kAddHalf) {
    const uint32_t hk = fadd(fadd(h, w, o.one), k, o.one);   // G1 on FMA
    const uint32_t t1 = hk + s1 + ch;                       // IADD3
    d = fadd(d, t1, o.one);                                 // G3 on FMA
    h = t1 + s0 + mj;                                       // IADD3
  } else {
    const uint32_t t1 = h + s1 + ch + k + w;
    d += t1;
    h = t1 + s0 + mj;
  }
}

// bround with a flag for a known-zero message word (skips the W add).
template <int F>
__device__ __forceinline__ void bround_z(uint32_t a, uint32_t b, uint32_t c, uint32_t& d, uint32_t e, uint32_t f,
                                         uint32_t g, uint32_t& h, uint32_t k, uint32_t w, bool wzero, const Opq& o) {
  const uint32_t s1 = bSig1<F>(e, o);
  const uint32_t s0 = bSig0<F>(a, o);
  const uint32_t ch = Ch(e, f, g);
  const uint32_t mj = Maj(a, b, c);
  if (F & (kAddRound | kAddHalf)) {
    const uint32_t hk = wzero ? fadd(h, k, o.one) : fadd(fadd(h, w, o.one), k, o.one);
    uint32_t t1;
    if (F & kAddRound) t1 = fadd(fadd(hk, s1, o.one), ch, o.one);
    else t1 = hk + s1 + ch;
    d = fadd(d, t1, o.one);
    if (F & kAddRound) h = fadd(fadd(t1, s0, o.one), mj, o.one);
    else h = t1 + s0 + mj;
  } else {
    const uint32_t t1 = h + s1 + ch + k + (wzero ? 0u : w);
    d += t1;
    h = t1 + s0 + mj;
  }
}

// compress() with the chosen split.  w is consumed (message schedule).
// ZM: bit i set = message word i is known to be zero (the IMAD forms are
// opaque to the compiler, so known zeros are skipped here explicitly).
template <int F, uint32_t ZM = 0>
__device__ __forceinline__ void compress_bal(uint32_t st[8], uint32_t w[16], const Opq& o) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
#pragma unroll
  for (int t = 0; t < 64; t += 8) {
    if (t >= 16) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int tt = t + i;
        const int j = tt & 15;
        // inputs W[tt-16], W[tt-15], W[tt-7], W[tt-2]; original words may be known zeros
        const bool z16 = tt - 16 < 16 && ((ZM >> (tt - 16)) & 1u);
        const bool z15 = tt - 15 < 16 && ((ZM >> (tt - 15)) & 1u);
        const bool z7 = tt - 7 < 16 && ((ZM >> (tt - 7)) & 1u);
        const bool z2 = tt - 2 < 16 && ((ZM >> (tt - 2)) & 1u);
        uint32_t acc = z16 ? 0u : w[j];
        bool have = !z16;
        if (!z2) {
          const uint32_t s1 = bsig1<F>(w[(j + 14) & 15], o);
          acc = have ? ((F & kAddSched) ? fadd(acc, s1, o.one) : acc + s1) : s1;
          have = true;
        }
        if (!z7) {
          acc = have ? ((F & kAddSched) ? fadd(acc, w[(j + 9) & 15], o.one) : acc + w[(j + 9) & 15]) : w[(j + 9) & 15];
          have = true;
        }
        if (!z15) {
          const uint32_t s0 = bsig0<F>(w[(j + 1) & 15], o);
          acc = have ? ((F & kAddSched) ? fadd(acc, s0, o.one) : acc + s0) : s0;
          have = true;
        }
        w[j] = have ? acc : 0u;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int tt = t + i;
      const bool zw = tt < 16 && ((ZM >> tt) & 1u);
      const uint32_t wv = zw ? 0u : w[tt & 15];
      // rotate the working variables by renaming: round tt uses (a..h) shifted by i
      switch (i) {
        case 0: bround_z<F>(a, b, c, d, e, f, g, h, c_K.v[tt], wv, zw, o); break;
        case 1: bround_z<F>(h, a, b, c, d, e, f, g, c_K.v[tt], wv, zw, o); break;
        case 2: bround_z<F>(g, h, a, b, c, d, e, f, c_K.v[tt], wv, zw, o); break;
        case 3: bround_z<F>(f, g, h, a, b, c, d, e, c_K.v[tt], wv, zw, o); break;
        case 4: bround_z<F>(e, f, g, h, a, b, c, d, c_K.v[tt], wv, zw, o); break;
        case 5: bround_z<F>(d, e, f, g, h, a, b, c, c_K.v[tt], wv, zw, o); break;
        case 6: bround_z<F>(c, d, e, f, g, h, a, b, c_K.v[tt], wv, zw, o); break;
        default: bround_z<F>(b, c, d, e, f, g, h, a, c_K.v[tt], wv, zw, o); break;
      }
    }
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

}  // namespace vc
