// Retained-state ("trace") leaves, the IO hash chain, and small tagged hashes.
#include "sha256_core.cuh"
#include "sha256_stream.cuh"
#include "tc05.cuh"
#include "vc_internal.h"

namespace vc {

constexpr int kTraceThreads = 128;
// Compression split of the retained-state leaves: the round's adds, the
// schedule's adds and its two plain shifts go to the FMA pipe as IMADs
// (kAddRound | kAddSched | kShrSched), the rotates and logic ops stay on the
// ALU.  Measured on the C4 workload (256 x 512 tokens with logits): 136.0 ->
// 125.4 ms; the KV kernel, whose messages are half zero words, keeps the
// plain compression (the split measured slower there).
constexpr int kTraceSplit = kAddRound | kAddSched | kShrSched;
// With few tokens (few CTAs per SM) each thread's hash is latency-bound and
// the split's extra instructions cost more than the ALU relief gains: below
// this many CTAs per SM the plain compression is used.  Measured (C4 message
// shape, ms plain / split): 256 tokens 27.4 / 34.5, 1 CTA per SM 28.1 / 35.7,
// 2 per SM 41.9 / 42.0, 4 per SM 81.9 / 74.3, 7 per SM 136.2 / 124.0.
constexpr int kTraceSplitMinCtasPerSm = 3;

// Domain separators (ASCII), merkle.rs:147, 179, 206, 233, 251, 555, 563, 574.
__device__ const char kTagRetained[] = "vi-retained-v3";
__device__ const char kTagFr[] = "vi-retained-fr-v1";
__device__ const char kTagLp[] = "vi-retained-lp-v1";
__device__ const char kTagLogits[] = "vi-retained-logits-v1";
__device__ const char kTagPrompt[] = "vi-prompt-v1";
__device__ const char kTagSeed[] = "vi-seed-v1";
__device__ const char kTagGenesis[] = "vi-io-genesis-v4";

// One thread per token: hash_retained_state_direct (merkle.rs:144-161), then
// the optional wraps of hash_retained_with_captured_logits (merkle.rs:170-241).
template <int SPLIT>
__global__ void __launch_bounds__(kTraceThreads) trace_leaf_kernel(const __grid_constant__ TraceArgs a) {
  __shared__ uint32_t sbuf[16 * kTraceThreads];
  const int t = blockIdx.x * kTraceThreads + threadIdx.x;
  if (t >= a.n_tokens) return;
  const int32_t* tk = a.tok + 5 * int64_t(t);
  const int f = tk[0];
  const int64_t row = tk[1];
  Sha256Stream<kTraceThreads, SPLIT, SPLIT == 0 ? 2 : 1> s;
  s.opq = &a.opq;  // parameter space (__grid_constant__): read as constant operands
  s.init(sbuf + threadIdx.x);
  s.put_tag(kTagRetained, 14);
  for (int l = 0; l < a.n_layers; ++l) {
    const int64_t fl = int64_t(f) * a.n_layers + l;
    const uint8_t* arow = static_cast<const uint8_t*>(a.a_rows[fl]) + row * a.hidden;
    s.put_array(arow, a.hidden);
    s.put_le(__ldg(static_cast<const uint32_t*>(a.scale_a[fl]) + row * a.scale_stride));
    if (a.x_rows) {
      s.put_byte(1);
      const uint8_t* xrow = static_cast<const uint8_t*>(a.x_rows[fl]) + row * a.hidden;
      s.put_array(xrow, a.hidden);
      s.put_le(__ldg(static_cast<const uint32_t*>(a.scale_x[fl]) + row * a.scale_x_stride));
    } else {
      s.put_byte(0);
    }
  }
  s.finish();
  uint32_t d[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) d[w] = s.h[w];
  if (tk[2] >= 0) {
    s.init(sbuf + threadIdx.x);
    s.put_tag(kTagFr, 17);
    s.put_digest(d);
    s.put_array(a.fr + int64_t(tk[2]) * a.fr_stride * 4, int64_t(a.fr_dim) * 4);
    s.finish();
#pragma unroll
    for (int w = 0; w < 8; ++w) d[w] = s.h[w];
  }
  if (tk[3] >= 0) {
    s.init(sbuf + threadIdx.x);
    s.put_tag(kTagLp, 17);
    s.put_digest(d);
    s.put_array(a.lp + int64_t(tk[3]) * a.lp_stride * 2, int64_t(a.lp_dim) * 2);
    s.finish();
#pragma unroll
    for (int w = 0; w < 8; ++w) d[w] = s.h[w];
  }
  if (tk[4] >= 0) {
    s.init(sbuf + threadIdx.x);
    s.put_tag(kTagLogits, 21);
    s.put_digest(d);
    s.put_array(a.logits + int64_t(tk[4]) * a.logits_stride * 4, int64_t(a.vocab) * 4);
    s.finish();
#pragma unroll
    for (int w = 0; w < 8; ++w) d[w] = s.h[w];
  }
  store_digest(a.leaves + int64_t(t) * 32, d);
}

// The same leaves when few tokens are hashed (a request or a decode step):
// each of them is one long serial chain (10 068 blocks for a Llama-8B token
// with its logits), so time is one thread's latency per block, and a lone
// warp issues at most one instruction every other cycle.  A CTA of two warps
// splits each compression: lane l of warp 1 walks token l's message (the
// same field streaming as trace_leaf_kernel) and, for every block, writes
// K[t] + W[t] of all 64 rounds (message schedule included) into a 4-slot ring
// in shared memory; lane l of warp 0 runs the rounds of token l from it.
// Each lane has its own mbarriers (full / empty per slot, count 1), so lanes
// move independently and no barrier depends on the warp being converged; a
// wrap message starts with the previous digest, which warp 0 hands back
// through shared memory and a third per-lane mbarrier.  Every wait gives up
// after 1 s of %globaltimer and sets the context's error flag to 2.
constexpr int kSplitSlots = 4;
constexpr int kSplitLanes = 32;
constexpr uint64_t kSplitWaitNs = 1000000000ull;
// at most this many two-warp CTAs per SM; above it the one-thread kernel's
// throughput wins
constexpr int kSplitMaxPairsPerSm = 2;

struct SplitSmem {
  uint4 kw[kSplitSlots][16][kSplitLanes];   // K + W of a block: [slot][rounds / 4][lane], 4 rounds per uint4
  uint32_t dig[8][kSplitLanes];             // digest handed from warp 0 to warp 1
  uint32_t sbuf[16 * kSplitLanes];          // warp 1's block buffer (Sha256Stream)
  uint64_t full[kSplitSlots][kSplitLanes];
  uint64_t empty[kSplitSlots][kSplitLanes];
  uint64_t dready[kSplitLanes];
};

// Warp 1's sink: the schedule of each completed block into the lane's ring.
struct KwSink {
  SplitSmem* sm;
  int* err;
  uint32_t lane;
  uint32_t k;     // blocks pushed
  bool ok;
  __device__ __forceinline__ void push(uint32_t w[16]) {
    if (!ok) return;
    const uint32_t slot = k % kSplitSlots, u = k / kSplitSlots;
    if (u > 0 && !tc05::mbar_wait(tc05::smem_u32(&sm->empty[slot][lane]), (u - 1) & 1u, kSplitWaitNs)) {
      atomicExch(err, 2);
      ok = false;
      return;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      sm->kw[slot][q][lane] = make_uint4(c_K.v[4 * q] + w[4 * q], c_K.v[4 * q + 1] + w[4 * q + 1],
                                         c_K.v[4 * q + 2] + w[4 * q + 2], c_K.v[4 * q + 3] + w[4 * q + 3]);
#pragma unroll
    for (int q = 4; q < 16; ++q) {
      uint32_t v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = 4 * q + i, j = t & 15;
        w[j] += sig1(w[(j + 14) & 15]) + w[(j + 9) & 15] + sig0(w[(j + 1) & 15]);
        v[i] = c_K.v[t] + w[j];
      }
      sm->kw[slot][q][lane] = make_uint4(v[0], v[1], v[2], v[3]);
    }
    tc05::mbar_arrive(tc05::smem_u32(&sm->full[slot][lane]));
    ++k;
  }
};

__device__ __forceinline__ int64_t sha_blocks_of(int64_t len) { return (len + 9 + 63) / 64; }

__global__ void __launch_bounds__(2 * kSplitLanes) trace_leaf_split_kernel(const __grid_constant__ TraceArgs a) {
  __shared__ SplitSmem sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kSplitLanes + lane;
  if (warp == 0) {
    for (int sl = 0; sl < kSplitSlots; ++sl) {
      tc05::mbar_init(tc05::smem_u32(&sm.full[sl][lane]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.empty[sl][lane]), 1);
    }
    tc05::mbar_init(tc05::smem_u32(&sm.dready[lane]), 1);
  }
  __syncthreads();
  if (t >= a.n_tokens) return;    // per lane: this lane's token does not exist, and its pair skips it too
  const int32_t* tk = a.tok + 5 * int64_t(t);
  // the lane's messages: the retained state, then the wraps it has, in order
  const int64_t len0 = 14 + int64_t(a.n_layers) * (a.hidden + 5 + (a.x_rows ? a.hidden + 4 : 0));
  const bool has[3] = {tk[2] >= 0, tk[3] >= 0, tk[4] >= 0};
  const int64_t wlen[3] = {17 + 32 + int64_t(a.fr_dim) * 4, 17 + 32 + int64_t(a.lp_dim) * 2,
                           21 + 32 + int64_t(a.vocab) * 4};
  const int n_wraps = int(has[0]) + int(has[1]) + int(has[2]);
  if (warp == 0) {
    // ------------------------------------------------------------------ rounds
    uint32_t k = 0, handed = 0;
    uint32_t d[8];
    bool ok = true;
    for (int m = 0; m < 4 && ok; ++m) {
      if (m > 0 && !has[m - 1]) continue;
      const int64_t nb = sha_blocks_of(m == 0 ? len0 : wlen[m - 1]);
      uint32_t st[8];
      sha_init(st);
      for (int64_t b = 0; b < nb; ++b, ++k) {
        const uint32_t slot = k % kSplitSlots, u = k / kSplitSlots;
        if (!tc05::mbar_wait(tc05::smem_u32(&sm.full[slot][lane]), u & 1u, kSplitWaitNs)) {
          atomicExch(a.err, 2);
          ok = false;
          break;
        }
        uint4 kv[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) kv[q] = sm.kw[slot][q][lane];
        tc05::mbar_arrive(tc05::smem_u32(&sm.empty[slot][lane]));
        const uint32_t* kw = reinterpret_cast<const uint32_t*>(kv);
        uint32_t a_ = st[0], b_ = st[1], c_ = st[2], d_ = st[3], e_ = st[4], f_ = st[5], g_ = st[6], h_ = st[7];
#pragma unroll
        for (int r = 0; r < 64; r += 8) {
          VC_SHA_ROUND(a_, b_, c_, d_, e_, f_, g_, h_, kw[r + 0]);
          VC_SHA_ROUND(h_, a_, b_, c_, d_, e_, f_, g_, kw[r + 1]);
          VC_SHA_ROUND(g_, h_, a_, b_, c_, d_, e_, f_, kw[r + 2]);
          VC_SHA_ROUND(f_, g_, h_, a_, b_, c_, d_, e_, kw[r + 3]);
          VC_SHA_ROUND(e_, f_, g_, h_, a_, b_, c_, d_, kw[r + 4]);
          VC_SHA_ROUND(d_, e_, f_, g_, h_, a_, b_, c_, kw[r + 5]);
          VC_SHA_ROUND(c_, d_, e_, f_, g_, h_, a_, b_, kw[r + 6]);
          VC_SHA_ROUND(b_, c_, d_, e_, f_, g_, h_, a_, kw[r + 7]);
        }
        st[0] += a_; st[1] += b_; st[2] += c_; st[3] += d_;
        st[4] += e_; st[5] += f_; st[6] += g_; st[7] += h_;
      }
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = st[w];
      if (ok && int(handed) < n_wraps) {
        // the next message of this lane starts with this digest
#pragma unroll
        for (int w = 0; w < 8; ++w) sm.dig[w][lane] = d[w];
        tc05::mbar_arrive(tc05::smem_u32(&sm.dready[lane]));
        ++handed;
      }
    }
    if (ok) store_digest(a.leaves + int64_t(t) * 32, d);
  } else {
    // ------------------------------------------------------ message + schedule
    KwSink sink{&sm, a.err, uint32_t(lane), 0u, true};
    Sha256Stream<kSplitLanes, 0, 2, KwSink> s;
    s.sink = &sink;
    const int f = tk[0];
    const int64_t row = tk[1];
    s.init(sm.sbuf + lane);
    s.put_tag(kTagRetained, 14);
    for (int l = 0; l < a.n_layers; ++l) {
      const int64_t fl = int64_t(f) * a.n_layers + l;
      const uint8_t* arow = static_cast<const uint8_t*>(a.a_rows[fl]) + row * a.hidden;
      s.put_array(arow, a.hidden);
      s.put_le(__ldg(static_cast<const uint32_t*>(a.scale_a[fl]) + row * a.scale_stride));
      if (a.x_rows) {
        s.put_byte(1);
        const uint8_t* xrow = static_cast<const uint8_t*>(a.x_rows[fl]) + row * a.hidden;
        s.put_array(xrow, a.hidden);
        s.put_le(__ldg(static_cast<const uint32_t*>(a.scale_x[fl]) + row * a.scale_x_stride));
      } else {
        s.put_byte(0);
      }
    }
    s.finish();
    uint32_t waited = 0;
    for (int wi = 0; wi < 3 && sink.ok; ++wi) {
      if (!has[wi]) continue;
      if (!tc05::mbar_wait(tc05::smem_u32(&sm.dready[lane]), waited & 1u, kSplitWaitNs)) {
        atomicExch(a.err, 2);
        break;
      }
      ++waited;
      uint32_t d[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = sm.dig[w][lane];
      s.init(sm.sbuf + lane);
      if (wi == 0) {
        s.put_tag(kTagFr, 17);
        s.put_digest(d);
        s.put_array(a.fr + int64_t(tk[2]) * a.fr_stride * 4, int64_t(a.fr_dim) * 4);
      } else if (wi == 1) {
        s.put_tag(kTagLp, 17);
        s.put_digest(d);
        s.put_array(a.lp + int64_t(tk[3]) * a.lp_stride * 2, int64_t(a.lp_dim) * 2);
      } else {
        s.put_tag(kTagLogits, 21);
        s.put_digest(d);
        s.put_array(a.logits + int64_t(tk[4]) * a.logits_stride * 4, int64_t(a.vocab) * 4);
      }
      s.finish();
    }
  }
}

// IO chain (prover/src/lib.rs:403-410):
//   prev = io_genesis_v4(prompt_hash)  = SHA256("vi-io-genesis-v4" || ph)
//   io_t = io_hash_v4(leaf_t, tok_t, prev) = SHA256("vi-io-v4" || leaf || u32le tok || prev)
// The 76-byte message is two blocks: [tag(2) leaf(8) tok(1) prev0..4] and
// [prev5..7, 0x80000000, 0 x 11, 608].  The chain is serial, and a lone warp
// issues at most one instruction every other cycle, so each sequence gets a
// CTA of two warps that split every compression: warp 1 computes the message
// schedules of both blocks (K[t] + W[t], t = 16..63) into shared memory in
// 8-word chunks as soon as the previous chain value is known, and warp 0 runs
// the rounds, taking each chunk as it is published (named barriers 2-7 for
// block 1, 8-13 for block 2; barrier 1: warp 0 has published the chain
// value).  Both warps walk the same tokens, and every barrier is executed by
// whole warps (all lanes compute the same values, lane 0 stores them).
// Measured as a microbenchmark: 2 364 instead of 3 201 cycles per chained
// block; in this kernel, a 4 096-token chain: 15.5 -> 13.1 ms.
// prev_io (optional): the chain continues from prev_io[s] instead of the
// genesis, and the last value is written back there (online extension).
constexpr int kIoBarPrev = 1, kIoBarS1 = 2, kIoBarS2 = 8, kIoThreads = 64;

__device__ __forceinline__ void io_bar_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(kIoThreads) : "memory");
}
__device__ __forceinline__ void io_bar_arrive(int id) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "n"(kIoThreads) : "memory");
}

// Rounds t .. t+7 with kw[t..t+7] = K[t] + W[t].
#define VC_ROUNDS8(kw, t)                                  \
  do {                                                     \
    VC_SHA_ROUND(a, b, c, d, e, f, g, h, (kw)[(t) + 0]);  \
    VC_SHA_ROUND(h, a, b, c, d, e, f, g, (kw)[(t) + 1]);  \
    VC_SHA_ROUND(g, h, a, b, c, d, e, f, (kw)[(t) + 2]);  \
    VC_SHA_ROUND(f, g, h, a, b, c, d, e, (kw)[(t) + 3]);  \
    VC_SHA_ROUND(e, f, g, h, a, b, c, d, (kw)[(t) + 4]);  \
    VC_SHA_ROUND(d, e, f, g, h, a, b, c, (kw)[(t) + 5]);  \
    VC_SHA_ROUND(c, d, e, f, g, h, a, b, (kw)[(t) + 6]);  \
    VC_SHA_ROUND(b, c, d, e, f, g, h, a, (kw)[(t) + 7]);  \
  } while (0)

// Warp 0's half of one compression: rounds 0-15 from the message words w,
// rounds 16-63 from the schedule chunks warp 1 publishes at barriers bar0..bar0+5.
__device__ __forceinline__ void io_rounds(uint32_t st[8], const uint32_t w[16], const uint32_t* kw, int bar0) {
  uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
  uint32_t k0[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) k0[t] = c_K.v[t] + w[t];
  VC_ROUNDS8(k0, 0);
  VC_ROUNDS8(k0, 8);
#pragma unroll
  for (int ch = 0; ch < 6; ++ch) {
    io_bar_sync(bar0 + ch);
    VC_ROUNDS8(kw, 16 + 8 * ch);
  }
  st[0] += a; st[1] += b; st[2] += c; st[3] += d;
  st[4] += e; st[5] += f; st[6] += g; st[7] += h;
}

// Warp 1's half: the schedule of message w, K + W of rounds 16-63 into kw, one
// barrier arrival per 8 words.
__device__ __forceinline__ void io_schedule(uint32_t w[16], uint32_t* kw, int bar0, bool store) {
#pragma unroll
  for (int ch = 0; ch < 6; ++ch) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int t = 16 + 8 * ch + q;
      const int j = t & 15;
      w[j] += sig1(w[(j + 14) & 15]) + w[(j + 9) & 15] + sig0(w[(j + 1) & 15]);
      if (store) kw[t] = c_K.v[t] + w[j];
    }
    __syncwarp();
    io_bar_arrive(bar0 + ch);
  }
}

__global__ void __launch_bounds__(kIoThreads) io_chain_kernel(int n_seqs, const int64_t* tok_off,
                                                              const uint8_t* leaves, const uint32_t* token_ids,
                                                              const uint8_t* prompt_hash, uint8_t* io,
                                                              uint8_t* prev_io) {
  __shared__ uint32_t kw1[64], kw2[64];   // K + W of each block's rounds 16-63
  __shared__ uint32_t sprev[8];           // the chain value the current token extends
  const int s = blockIdx.x;
  if (s >= n_seqs) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = tok_off[s], t1 = tok_off[s + 1];
  if (t0 >= t1) return;   // nothing appended: prev_io keeps its value
  uint32_t leaf[8], tok;
  load_digest(leaves + t0 * 32, leaf);
  tok = token_ids[t0];
  if (warp == 0) {
    uint32_t prev[8];
    if (prev_io) {
      load_digest(prev_io + int64_t(s) * 32, prev);
    } else {
      uint32_t ph[8];
      load_digest(prompt_hash + int64_t(s) * 32, ph);
      uint32_t w[16] = {0x76692d69u, 0x6f2d6765u, 0x6e657369u, 0x732d7634u,  // "vi-io-genesis-v4"
                        ph[0], ph[1], ph[2], ph[3], ph[4], ph[5], ph[6], ph[7],
                        0x80000000u, 0u, 0u, 384u};
      sha_init(prev);
      compress(prev, w);
    }
    for (int64_t t = t0; t < t1; ++t) {
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) sprev[i] = prev[i];
      }
      __syncwarp();
      io_bar_arrive(kIoBarPrev);
      // the next token's inputs do not depend on the chain: fetch them now
      uint32_t nleaf[8], ntok = 0;
      if (t + 1 < t1) {
        load_digest(leaves + (t + 1) * 32, nleaf);
        ntok = token_ids[t + 1];
      }
      const uint32_t w1[16] = {0x76692d69u, 0x6f2d7634u,  // "vi-io-v4"
                               leaf[0], leaf[1], leaf[2], leaf[3], leaf[4], leaf[5], leaf[6], leaf[7],
                               bswap32(tok), prev[0], prev[1], prev[2], prev[3], prev[4]};
      uint32_t st[8];
      sha_init(st);
      io_rounds(st, w1, kw1, kIoBarS1);
      const uint32_t w2[16] = {prev[5], prev[6], prev[7], 0x80000000u, 0u, 0u, 0u, 0u,
                               0u, 0u, 0u, 0u, 0u, 0u, 0u, 608u};
      io_rounds(st, w2, kw2, kIoBarS2);
      if (lane == 0) store_digest(io + t * 32, st);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 8; ++i) { prev[i] = st[i]; leaf[i] = nleaf[i]; }
      tok = ntok;
    }
    if (prev_io && lane == 0) store_digest(prev_io + int64_t(s) * 32, prev);
  } else {
    for (int64_t t = t0; t < t1; ++t) {
      uint32_t nleaf[8], ntok = 0;
      if (t + 1 < t1) {
        load_digest(leaves + (t + 1) * 32, nleaf);
        ntok = token_ids[t + 1];
      }
      io_bar_sync(kIoBarPrev);
      uint32_t p[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) p[i] = sprev[i];
      uint32_t w1[16] = {0x76692d69u, 0x6f2d7634u,
                         leaf[0], leaf[1], leaf[2], leaf[3], leaf[4], leaf[5], leaf[6], leaf[7],
                         bswap32(tok), p[0], p[1], p[2], p[3], p[4]};
      io_schedule(w1, kw1, kIoBarS1, lane == 0);
      uint32_t w2[16] = {p[5], p[6], p[7], 0x80000000u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 608u};
      io_schedule(w2, kw2, kIoBarS2, lane == 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) leaf[i] = nleaf[i];
      tok = ntok;
    }
  }
}

// SHA256(tag || data_i), one thread per message.  tag 0: "vi-prompt-v1"
// over [off[i], off[i+1]) (hash_prompt, merkle.rs:561-566); tag 1:
// "vi-seed-v1" over 32 bytes at data + 32 i (hash_seed, merkle.rs:553-558);
// tag 2: "vi-io-genesis-v4" over a 32-byte prompt hash (io_genesis_v4,
// merkle.rs:572-577).
__global__ void __launch_bounds__(kTraceThreads) tagged_hash_kernel(int n, int tag, const uint8_t* data,
                                                                     const int64_t* off, int64_t fixed_len,
                                                                     uint8_t* out) {
  __shared__ uint32_t sbuf[16 * kTraceThreads];
  const int i = blockIdx.x * kTraceThreads + threadIdx.x;
  if (i >= n) return;
  const int64_t b = off ? off[i] : int64_t(i) * fixed_len;
  const int64_t len = off ? off[i + 1] - off[i] : fixed_len;
  Sha256Stream<kTraceThreads> s;
  s.init(sbuf + threadIdx.x);
  if (tag == 0) s.put_tag(kTagPrompt, 12);
  else if (tag == 1) s.put_tag(kTagSeed, 10);
  else s.put_tag(kTagGenesis, 16);
  if (len > 0) s.put_array(data + b, len);
  s.finish();
  store_digest(out + int64_t(i) * 32, s.h);
}

cudaError_t launch_trace_leaves(const TraceArgs& a, int n_sm, cudaStream_t s) {
  if (a.n_tokens == 0) return cudaSuccess;
  const int grid = (a.n_tokens + kTraceThreads - 1) / kTraceThreads;
  const int pairs = (a.n_tokens + kSplitLanes - 1) / kSplitLanes;
  if (grid >= kTraceSplitMinCtasPerSm * n_sm)
    trace_leaf_kernel<kTraceSplit><<<grid, kTraceThreads, 0, s>>>(a);
  else if (pairs <= kSplitMaxPairsPerSm * n_sm)
    trace_leaf_split_kernel<<<pairs, 2 * kSplitLanes, 0, s>>>(a);
  else
    trace_leaf_kernel<0><<<grid, kTraceThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_io_chain(int n_seqs, const int64_t* tok_off_dev, const uint8_t* leaves,
                            const uint32_t* token_ids, const uint8_t* prompt_hash, uint8_t* io, uint8_t* prev_io,
                            cudaStream_t s) {
  if (n_seqs == 0) return cudaSuccess;
  io_chain_kernel<<<n_seqs, kIoThreads, 0, s>>>(n_seqs, tok_off_dev, leaves, token_ids, prompt_hash, io, prev_io);
  return cudaGetLastError();
}

cudaError_t launch_tagged_hash(int n, int tag, const uint8_t* data, const int64_t* off_dev,
                               int64_t fixed_len, uint8_t* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  tagged_hash_kernel<<<(n + kTraceThreads - 1) / kTraceThreads, kTraceThreads, 0, s>>>(n, tag, data, off_dev,
                                                                                   fixed_len, out);
  return cudaGetLastError();
}

}  // namespace vc
