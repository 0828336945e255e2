// Per-thread streaming SHA-256 for messages built from fields at arbitrary
// byte offsets (the retained-state leaf of merkle.rs:144-161 has 4101-byte
// layer records, so its a_i8 rows start at every alignment mod 4).
//
// Whole blocks inside a field are assembled straight from global memory in
// registers (4-byte loads, one byte-permute per word realigns and byte-swaps).
// The partial blocks where fields meet go through a 16-word block buffer in
// shared memory, word-major across the CTA (word k of thread tid at
// buf[k * NT]), so every access of a warp is one conflict-free wavefront.
// All threads of a warp hash messages of the same layout, so the fill
// position -- and every branch on it -- is warp-uniform.
#pragma once
#include <type_traits>

#include "sha256_bal.cuh"
#include "sha256_core.cuh"

namespace vc {

// BAL: the split of compress_bal (sha256_bal.cuh) to use, 0 for the plain
// compression; with BAL != 0, opq must point at the opaque multipliers.
// PF: blocks of prefetch in direct_blocks.  Two keep a lone warp's loads
// ahead of HBM latency when few threads hash (measured on one 4 096-token
// request: trace leaves 25.5 -> 23.5 ms); with many threads per SM the
// second 17-word buffer costs more in registers than it hides (C4: 129.8 ->
// 144.2 ms), so the busy configurations keep one.
// Sink: when not void, every completed 64-byte block goes to sink->push(w)
// instead of into this stream's own compression (h is then unused): the
// producer half of a split compression.
template <int NT, int BAL = 0, int PF = 1, class Sink = void>
struct Sha256Stream {
  uint32_t h[8];
  const Opq* opq = nullptr;
  Sink* sink = nullptr;
  uint32_t* buf;    // this thread's column of the CTA's [16][NT] buffer
  uint32_t fill;    // bytes of the current block, pending partial word included (0..63)
  uint32_t carry;   // the fill % 4 pending bytes, left-aligned big-endian
  uint64_t total;   // message bytes appended

  __device__ __forceinline__ void init(uint32_t* column) {
    sha_init(h);
    buf = column;
    fill = 0;
    carry = 0;
    total = 0;
  }

  __device__ __forceinline__ void cmp(uint32_t w[16]) {
    if constexpr (!std::is_void_v<Sink>)
      sink->push(w);
    else if constexpr (BAL == 0)
      compress(h, w);
    else
      compress_bal<BAL>(h, w, *opq);
  }

  __device__ __forceinline__ void block() {
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) w[k] = buf[k * NT];
    cmp(w);
  }

  // Append 4 bytes given as a big-endian word.
  __device__ __forceinline__ void put_be(uint32_t wbe) {
    const uint32_t r = fill & 3u;
    const uint32_t k = fill >> 2;
    if (r == 0) {
      buf[k * NT] = wbe;
    } else {
      buf[k * NT] = carry | (wbe >> (8u * r));
      carry = wbe << (32u - 8u * r);
    }
    fill += 4;
    total += 4;
    if (fill >= 64) {
      block();
      fill -= 64;
    }
  }

  // Append 4 bytes in memory order (a little-endian 32-bit load).
  __device__ __forceinline__ void put_le(uint32_t x) { put_be(bswap32(x)); }

  // Append n (1..3) bytes, left-aligned in v (big-endian), low bytes zero.
  __device__ __forceinline__ void put_small(uint32_t v, uint32_t n) {
    const uint32_t r = fill & 3u;
    if (r + n < 4) {
      carry |= v >> (8u * r);
    } else {
      buf[(fill >> 2) * NT] = carry | (v >> (8u * r));
      carry = v << (8u * (4u - r));   // r >= 1 here, so the shift is < 32
    }
    fill += n;
    total += n;
    if (fill >= 64) {
      block();
      fill -= 64;
    }
  }

  __device__ __forceinline__ void put_byte(uint32_t b) { put_small(b << 24, 1); }

  // Append the 8 words of a digest (32 bytes).
  __device__ __forceinline__ void put_digest(const uint32_t d[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) put_be(d[i]);
  }

  // Append len bytes from p (any alignment).  Whole blocks inside the field
  // are assembled in registers; only the partial blocks at its ends go
  // through the shared-memory buffer.
  __device__ __forceinline__ void put_array(const uint8_t* p, int64_t len) {
    // head: up to the next block boundary of the message
    if (fill != 0) {
      const int64_t head = 64 - fill;
      if (len <= head + 68) {
        put_array_buffered(p, len);
        return;
      }
      put_array_buffered(p, head);
      p += head;
      len -= head;
    }
    // interior: the buffer is empty here; keep 4 bytes of margin so the
    // last word load of a misaligned block stays inside the field
    const int64_t nblk = len >= 68 ? (len - 4) >> 6 : 0;
    if (nblk > 0) {
      direct_blocks(p, nblk);
      p += nblk * 64;
      len -= nblk * 64;
      total += uint64_t(nblk) * 64;
    }
    if (len > 0) put_array_buffered(p, len);
  }

  // nblk whole 64-byte blocks from p (any alignment), straight from global
  // memory into the compression, PF blocks of prefetch.  The buffer must be
  // empty (fill == 0).  Reads bytes [p & ~3, p + 64 * nblk + 3).
  __device__ __forceinline__ void direct_blocks(const uint8_t* p, int64_t nblk) {
    const uint32_t s = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3u);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - s);
    // message word j = bytes s..s+3 of (x[j], x[j+1]), most significant first
    const uint32_t sel = (s << 12) | ((s + 1) << 8) | ((s + 2) << 4) | (s + 3);
    uint32_t x[17];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __ldg(q + j);
    x[16] = s ? __ldg(q + 16) : 0u;
    if constexpr (PF == 1) {
      for (int64_t b = 0; b < nblk; ++b) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = __byte_perm(x[j], x[j + 1], sel);
        if (b + 1 < nblk) {
          // the next block's loads are in flight during this compression
          const uint32_t* qn = q + 16 * (b + 1);
#pragma unroll
          for (int j = 0; j < 16; ++j) x[j] = __ldg(qn + j);
          x[16] = s ? __ldg(qn + 16) : 0u;
        }
        cmp(w);
      }
    } else {
      // y holds block b + 1 while block b compresses; block b + 2 is loaded
      uint32_t y[17] = {};
      if (nblk > 1) {
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = __ldg(q + 16 + j);
        y[16] = s ? __ldg(q + 32) : 0u;
      }
      for (int64_t b = 0; b < nblk; ++b) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = __byte_perm(x[j], x[j + 1], sel);
#pragma unroll
        for (int j = 0; j < 17; ++j) x[j] = y[j];
        if (b + 2 < nblk) {
          const uint32_t* qn = q + 16 * (b + 2);
#pragma unroll
          for (int j = 0; j < 16; ++j) y[j] = __ldg(qn + j);
          y[16] = s ? __ldg(qn + 16) : 0u;
        }
        cmp(w);
      }
    }
  }

  // Append len bytes from p through the shared-memory block buffer.
  __device__ __forceinline__ void put_array_buffered(const uint8_t* p, int64_t len) {
    while (len > 0 && (reinterpret_cast<uintptr_t>(p) & 3u) != 0) {
      put_byte(__ldg(p));
      ++p;
      --len;
    }
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
    int64_t nw = len >> 2;
    // Reach 16-byte alignment with single words.
    while (nw > 0 && (reinterpret_cast<uintptr_t>(q) & 15u) != 0) {
      put_le(__ldg(q));
      ++q;
      --nw;
    }
    const uint4* v = reinterpret_cast<const uint4*>(q);
    int64_t nv = nw >> 2;
    uint4 nxt = make_uint4(0, 0, 0, 0);
    if (nv > 0) nxt = __ldg(v);
    for (int64_t i = 0; i < nv; ++i) {
      const uint4 cur = nxt;
      if (i + 1 < nv) nxt = __ldg(v + i + 1);
      if (fill + 16 < 64) {
        // The 16 bytes stay inside the current block.
        const uint32_t r = fill & 3u;
        const uint32_t k = fill >> 2;
        const uint32_t a = bswap32(cur.x), b = bswap32(cur.y), c = bswap32(cur.z), d = bswap32(cur.w);
        if (r == 0) {
          buf[(k + 0) * NT] = a;
          buf[(k + 1) * NT] = b;
          buf[(k + 2) * NT] = c;
          buf[(k + 3) * NT] = d;
        } else {
          const uint32_t sr = 8u * r, sl = 32u - 8u * r;
          buf[(k + 0) * NT] = carry | (a >> sr);
          buf[(k + 1) * NT] = (a << sl) | (b >> sr);
          buf[(k + 2) * NT] = (b << sl) | (c >> sr);
          buf[(k + 3) * NT] = (c << sl) | (d >> sr);
          carry = d << sl;
        }
        fill += 16;
        total += 16;
      } else {
        put_le(cur.x);
        put_le(cur.y);
        put_le(cur.z);
        put_le(cur.w);
      }
    }
    q += nv << 2;
    for (int64_t i = 0; i < (nw & 3); ++i) put_le(__ldg(q + i));
    q += nw & 3;
    const uint32_t tail = static_cast<uint32_t>(len & 3);
    if (tail) {
      // Read the last bytes one at a time: the word holding them may end
      // past the caller's buffer.
      const uint8_t* t = reinterpret_cast<const uint8_t*>(q);
      uint32_t v = 0;
      for (uint32_t i = 0; i < tail; ++i) v |= static_cast<uint32_t>(__ldg(t + i)) << (24 - 8 * i);
      put_small(v, tail);
    }
  }

  // FIPS 180-4 padding and length; the digest lands in h.
  __device__ __forceinline__ void finish() {
    const uint64_t bits = total * 8ull;
    put_byte(0x80);
    if (fill & 3u) {
      buf[(fill >> 2) * NT] = carry;
      fill = (fill + 3u) & ~3u;
      carry = 0;
    }
    if (fill > 56) {
      for (uint32_t k = fill >> 2; k < 16; ++k) buf[k * NT] = 0;
      block();
      fill = 0;
    }
    for (uint32_t k = fill >> 2; k < 14; ++k) buf[k * NT] = 0;
    buf[14 * NT] = static_cast<uint32_t>(bits >> 32);
    buf[15 * NT] = static_cast<uint32_t>(bits);
    block();
    fill = 0;
  }

  // Append an ASCII tag (domain separator) byte by byte.
  __device__ __forceinline__ void put_tag(const char* s, int n) {
    for (int i = 0; i < n; ++i) put_byte(static_cast<uint8_t>(s[i]));
  }
};

}  // namespace vc
