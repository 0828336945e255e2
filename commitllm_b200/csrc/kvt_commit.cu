// KV transcript and its KV trees in one pass: compute_kv_transcript
// (crates/verilm-prover/src/lib.rs:207-329) fused with hot loop C of
// commit_minimal (lib.rs:449-482).
//
// The f64 K/V values never reach memory.  A unit is 128 positions of one
// layer; its 2 * kv_dim channels leave the tensor cores as 128-channel tiles
// in message order (K heads, then V heads), and the thread that owns a
// position absorbs them straight into that position's SHA-256 state:
//   hash_kv_entry = SHA256("vi-kv-v1" || u32le layer || u32le pos ||
//                          f64le K[kv_dim] || f64le V[kv_dim])  (merkle.rs:285-293)
// The 16-byte prefix shifts the f64 slots by two, so every 64-byte block is the
// two values carried from the previous eight plus six new ones.  Each unit's
// 128 leaves are one 128-leaf chunk of its layer's tree: the group reduces it
// in shared memory and the group that completes a tree's last chunk builds the
// levels above (merkle_tree.cuh), as kv_commit_kernel does.
//
// CTA layout (one persistent CTA per SM, 640 threads):
//   warp 0      TMA: x_attn rows (A, 128 x 128 B) and weight rows (B, 128 x 128 B)
//               per 128-byte K-step into a 4-stage mbarrier ring, no multicast;
//   warp 1      tcgen05.mma kind::i8, M 128 x N 128 x K 32, into the
//               accumulator (128 TMEM columns) of one of four groups;
//   warps 2-3   idle (warps 0-3 are one warpgroup, which gives most of its
//               registers to the hashing warps, below);
//   warps 4-19  four epilogue groups of four warps (one per TMEM lane
//               quarter): tcgen05.ld 8 columns, dequantise / rotate in f64
//               (each operation rounded on its own, in the reference's order),
//               compress.  Sixteen hashing warps per SM keep the integer pipe
//               busy while any of them waits on TMEM, a table load or an MMA.
// Registers: the launch gives every thread 96 (20 warps, at most five per SM
// sub-partition: 16384 / (5 x 32) = 102, allocated in steps of 8);
// setmaxnreg moves the control warpgroup to 32 and the four epilogue
// warpgroups to 112: (96 - 32) x 128 = 4 x (112 - 96) x 128.  The launch
// checks the compiled register count against that sum first.
// Early release: a group copies the accumulator columns its tile's last
// blocks need (the last 32 columns of a plain tile, the 16 + 16 columns of the
// last 16 RoPE outputs) to shared memory when the tile starts, and releases
// the accumulator after its last direct TMEM load, so the MMAs of its next
// tile overlap the hashing of those blocks.  Measured on the Llama-8B
// transcript (4 096 positions x 32 layers): 3.68 -> 3.49 ms.
// Every wait is bounded (1 s of %globaltimer); a wait that runs out sets the
// context's error flag to 2, and the CTA drains its copies and MMAs and frees
// its TMEM before it returns.
#include <cuda.h>

#include <algorithm>

#include "merkle_tree.cuh"
#include "sha256_core.cuh"
#include "tc05.cuh"
#include "vc_internal.h"

namespace vc {

namespace {

constexpr int kBM = 128;                         // positions per unit (TMEM lanes)
constexpr int kBN = 128;                         // channels per tile (accumulator columns)
constexpr int kBK = 128;                         // bytes of hidden per stage
constexpr int kStages = 4;
constexpr int kGroups = 4;                       // epilogue groups, one accumulator each
constexpr int kEpiWarps = 4 * kGroups;
constexpr int kThreads = 128 + 32 * kEpiWarps;   // 640: a control warpgroup + four epilogue groups
constexpr int kLaunchRegs = 96;                   // what 20 warps per CTA leave a thread (see above)
constexpr int kCtlRegs = 32;                      // setmaxnreg of the control warpgroup
constexpr int kEpiRegs = 112;                     // setmaxnreg of each epilogue warpgroup
static_assert((kLaunchRegs - kCtlRegs) >= kGroups * (kEpiRegs - kLaunchRegs),
              "the epilogue warpgroups take more registers than the control warpgroup gives back");
constexpr uint32_t kStageA = kBM * kBK;
constexpr uint32_t kStageB = kBN * kBK;
constexpr uint32_t kIdesc = tc05::idesc_i8_s32(kBM, kBN);
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr int kErrTimeout = 2;
constexpr int kStep = 8;                         // channels per TMEM load
constexpr int kStgRope = 16;   // outputs of a RoPE tile hashed after the accumulator is released
constexpr int kStgPlain = 32;  // columns of a plain tile hashed after the accumulator is released
constexpr int kStgWords = (2 * kStgRope > kStgPlain ? 2 * kStgRope : kStgPlain);

struct Smem {
  uint8_t a[kStages][kStageA];
  uint8_t b[kStages][kStageB];
  uint32_t sd[kGroups][8][kBM];
  uint32_t stg[kGroups][kStgWords][kBM];    // accumulator columns copied for early release
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[kGroups];
  uint64_t acc_empty[kGroups];
  uint64_t final_mma;
  uint32_t tmem;
  int32_t abort;
  int s_last[kGroups];
  int stop[kGroups];
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory above the 227 KB a CTA may have");

__device__ __forceinline__ bool aborted(const Smem& sm) {
  return *reinterpret_cast<const volatile int32_t*>(&sm.abort) != 0;
}

__device__ __forceinline__ void set_abort(Smem& sm, int* err) {
  atomicExch(&sm.abort, 1);
  atomicExch(err, kErrTimeout);
}

// Dequantisation (rope.rs:107-138, lib.rs:283-316), per tile: toy clamp,
// per-tensor scale, or per-channel scale and/or bias.
enum { kModeToy = 0, kModeTensor = 1, kModeGeneral = 2 };

struct Deq {
  const float* ch;
  const float* bias;
  double sx, scale;
};

template <int MODE>
__device__ __forceinline__ double dq(int32_t acc, int c, const Deq& q) {
  if (MODE == kModeToy) return double(min(127, max(-128, acc)));
  if (MODE == kModeTensor) return __dmul_rn(double(acc), q.scale);
  double f = q.ch ? __dmul_rn(__dmul_rn(double(acc), double(__ldg(q.ch + c))), q.sx) : __dmul_rn(double(acc), q.scale);
  if (q.bias) f = __dadd_rn(f, double(__ldg(q.bias + c)));
  return f;
}

// One SHA-256 block of the leaf message is the two f64 values carried from
// the previous load (w[0..3]) and the first six of the current eight
// (w[4..15]); the last two are carried on.  An f64 d is the message words
// bswap(lo32(d)), bswap(hi32(d)).
__device__ __forceinline__ void put(uint32_t w[16], uint32_t nc[4], int j, double d) {
  const uint32_t lo = bswap32(uint32_t(__double2loint(d)));
  const uint32_t hi = bswap32(uint32_t(__double2hiint(d)));
  if (j < 6) {
    w[4 + 2 * j] = lo;
    w[5 + 2 * j] = hi;
  } else {
    nc[2 * (j - 6)] = lo;
    nc[2 * (j - 6) + 1] = hi;
  }
}

__device__ __forceinline__ void begin_block(uint32_t w[16], const uint32_t carry[4]) {
  w[0] = carry[0];
  w[1] = carry[1];
  w[2] = carry[2];
  w[3] = carry[3];
}

// The accumulator of this group may be overwritten once all four warps have
// read their last columns of it.
__device__ __forceinline__ void release_acc(Smem& sm, int g, int lane) {
  tc05::fence_before_sync();
  __syncwarp();
  if (lane == 0) tc05::mbar_arrive(tc05::smem_u32(&sm.acc_empty[g]));
}

// K tile with RoPE (rope.rs:48-57): per head, out[i] = k[i] c - k[i+half] s
// for i < half, then out[i+half] = k[i+half] c + k[i] s; the accumulator
// columns of each pair are read again for the second half, so the outputs
// leave in channel order.
template <int MODE, int HD>
__device__ __forceinline__ void tile_rope(const KvtArgs& a, Smem& sm, int g, int lane, int p, uint32_t ta, int c0,
                                          int pos_c, const Deq& q, uint32_t st[8], uint32_t carry[4]) {
  constexpr int half = HD / 2;
  constexpr int hb_last = kBN - HD;
  constexpr int j_stg = half - kStgRope;          // pass 1 of the last head from this j0 on reads the copy
  // copy the columns the last kStgRope outputs need, so the accumulator can be released earlier
#pragma unroll
  for (int j0 = j_stg; j0 < half; j0 += kStep) {
    uint32_t lo[kStep], hi[kStep];
    tc05::tmem_ld2_wait<kStep>(ta + hb_last + j0, ta + hb_last + half + j0, lo, hi);
#pragma unroll
    for (int j = 0; j < kStep; ++j) {
      sm.stg[g][j0 - j_stg + j][p] = lo[j];
      sm.stg[g][kStgRope + j0 - j_stg + j][p] = hi[j];
    }
  }
#pragma unroll 1
  for (int hb = 0; hb < kBN; hb += HD) {
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll 1
      for (int j0 = 0; j0 < half; j0 += kStep) {
        uint32_t lo[kStep], hi[kStep];
        if (hb == hb_last && pass == 1 && j0 >= j_stg) {
#pragma unroll
          for (int j = 0; j < kStep; ++j) {
            lo[j] = sm.stg[g][j0 - j_stg + j][p];
            hi[j] = sm.stg[g][kStgRope + j0 - j_stg + j][p];
          }
        } else {
          tc05::tmem_ld2_wait<kStep>(ta + hb + j0, ta + hb + half + j0, lo, hi);
          if (hb == hb_last && pass == 1 && j0 == j_stg - kStep) release_acc(sm, g, lane);
        }
        const double2* cs = a.rope + int64_t(j0) * a.rope_rows + pos_c;
        uint32_t w[16];
        begin_block(w, carry);
#pragma unroll
        for (int j = 0; j < kStep; ++j) {
          const int c = c0 + hb + j0 + j;
          const double kl = dq<MODE>(int32_t(lo[j]), c, q);
          const double kh = dq<MODE>(int32_t(hi[j]), c + half, q);
          const double2 cw = __ldg(cs + int64_t(j) * a.rope_rows);
          put(w, carry, j, pass == 0 ? __dsub_rn(__dmul_rn(kl, cw.x), __dmul_rn(kh, cw.y))
                                     : __dadd_rn(__dmul_rn(kh, cw.x), __dmul_rn(kl, cw.y)));
        }
        compress(st, w);
      }
    }
  }
}

// V tile, or any tile of the toy path: channels in order.
template <int MODE>
__device__ __forceinline__ void tile_plain(Smem& sm, int g, int lane, int p, uint32_t ta, int c0, const Deq& q,
                                           uint32_t st[8], uint32_t carry[4]) {
  constexpr int kDirect = kBN - kStgPlain;
#pragma unroll
  for (int j0 = kDirect; j0 < kBN; j0 += kStep) {
    uint32_t r[kStep];
    tc05::tmem_ld_wait<kStep>(ta + j0, r);
#pragma unroll
    for (int j = 0; j < kStep; ++j) sm.stg[g][j0 - kDirect + j][p] = r[j];
  }
#pragma unroll 1
  for (int j0 = 0; j0 < kBN; j0 += kStep) {
    uint32_t r[kStep];
    if (j0 >= kDirect) {
#pragma unroll
      for (int j = 0; j < kStep; ++j) r[j] = sm.stg[g][j0 - kDirect + j][p];
    } else {
      tc05::tmem_ld_wait<kStep>(ta + j0, r);
      if (j0 == kDirect - kStep) release_acc(sm, g, lane);
    }
    uint32_t w[16];
    begin_block(w, carry);
#pragma unroll
    for (int j = 0; j < kStep; ++j) put(w, carry, j, dq<MODE>(int32_t(r[j]), c0 + j0 + j, q));
    compress(st, w);
  }
}

struct UnitOf {
  int layer, m0, mb;
};

__device__ __forceinline__ UnitOf unit_of(const KvtArgs& a, int u) {
  UnitOf r;
  r.layer = u / a.m_tiles;
  r.mb = u % a.m_tiles;
  r.m0 = r.mb * kBM;
  return r;
}

// Units are dealt to CTAs round-robin; the j-th unit of a CTA goes to group
// j % kGroups.  Both the TMA producer and the MMA issuer walk the tiles in one
// order: for each round k, tile t, group g -- tile t of group g's k-th unit.
__device__ __forceinline__ int n_local_units(int n_units) {
  return n_units > int(blockIdx.x) ? (n_units - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) kvt_commit_kernel(const KvtcArgs A) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const KvtArgs& a = A.t;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (a.hidden + kBK - 1) / kBK;
  const int tpm = a.kv_dim / kBN;                 // tiles per matrix
  const int n_tiles = 2 * tpm;                    // tiles per unit
  const int nj = n_local_units(A.n_units);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc05::mbar_init(tc05::smem_u32(&sm.full[s]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.empty[s]), 1);
    }
    for (int g = 0; g < kGroups; ++g) {
      tc05::mbar_init(tc05::smem_u32(&sm.acc_full[g]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.acc_empty[g]), 4);
    }
    tc05::mbar_init(tc05::smem_u32(&sm.final_mma), 1);
    sm.abort = 0;
    tc05::mbar_init_fence();
  }
  if (warp == 0) tc05::tmem_alloc(tc05::smem_u32(&sm.tmem), kGroups * kBN);
  tc05::fence_before_sync();
  __syncthreads();
  tc05::fence_after_sync();
  const uint32_t tmem = sm.tmem;

  if (warp < 4) {
  // the control warpgroup (TMA, MMA, two idle warps) returns registers
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kCtlRegs));
  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- TMA producer
      int64_t kb_total = 0;
      bool ok = true;
      for (int k = 0; kGroups * k < nj && ok; ++k) {
        for (int t = 0; t < n_tiles && ok; ++t) {
          for (int g = 0; g < kGroups && ok; ++g) {
            const int j = kGroups * k + g;
            if (j >= nj) continue;
            const UnitOf un = unit_of(a, int(blockIdx.x) + j * int(gridDim.x));
            const int mat = t / tpm, c0 = (t % tpm) * kBN;
            const CUtensorMap* map_a = a.maps + 3 * un.layer;
            const CUtensorMap* map_b = a.maps + 3 * un.layer + 1 + mat;
            tc05::tensormap_acquire(map_a);
            tc05::tensormap_acquire(map_b);
            for (int kb = 0; kb < nk; ++kb, ++kb_total) {
              const int s = int(kb_total % kStages);
              const int64_t u = kb_total / kStages;
              if (u > 0 && !tc05::mbar_wait(tc05::smem_u32(&sm.empty[s]), uint32_t((u - 1) & 1), kWaitLimitNs)) {
                set_abort(sm, a.err);
                ok = false;
                break;
              }
              if (aborted(sm)) {
                ok = false;
                break;
              }
              const uint32_t full = tc05::smem_u32(&sm.full[s]);
              tc05::mbar_arrive_expect_tx(full, kStageA + kStageB);
              tc05::tma_load_2d(tc05::smem_u32(sm.a[s]), map_a, kb * kBK, un.m0, full);
              tc05::tma_load_2d(tc05::smem_u32(sm.b[s]), map_b, kb * kBK, c0, full);
            }
          }
        }
      }
      if (!ok) {
        // the copies already issued must land before the CTA exits
        for (int64_t k = kb_total - 1; k >= 0 && k >= kb_total - kStages; --k)
          tc05::mbar_wait(tc05::smem_u32(&sm.full[k % kStages]), uint32_t((k / kStages) & 1), kWaitLimitNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int64_t kb_total = 0;
      uint32_t issued = 0;   // bit g: group g has had a tile
      uint32_t parity = 0;   // bit g: parity of the next acc_empty phase of group g
      bool ok = true;
      for (int k = 0; kGroups * k < nj && ok; ++k) {
        for (int t = 0; t < n_tiles && ok; ++t) {
          for (int g = 0; g < kGroups && ok; ++g) {
            if (kGroups * k + g >= nj) continue;
            if (((issued >> g) & 1u) &&
                !tc05::mbar_wait(tc05::smem_u32(&sm.acc_empty[g]), (parity >> g) & 1u, kWaitLimitNs)) {
              set_abort(sm, a.err);
              ok = false;
              break;
            }
            if (aborted(sm)) {
              ok = false;
              break;
            }
            tc05::fence_after_sync();
            const uint32_t d = tmem + uint32_t(g * kBN);
            for (int kb = 0; kb < nk; ++kb, ++kb_total) {
              const int s = int(kb_total % kStages);
              const int64_t u = kb_total / kStages;
              if (!tc05::mbar_wait(tc05::smem_u32(&sm.full[s]), uint32_t(u & 1), kWaitLimitNs) || aborted(sm)) {
                set_abort(sm, a.err);
                ok = false;
                break;
              }
              tc05::fence_after_sync();
              const uint64_t ad = tc05::sw128_kmajor_desc(tc05::smem_u32(sm.a[s]));
              const uint64_t bd = tc05::sw128_kmajor_desc(tc05::smem_u32(sm.b[s]));
#pragma unroll
              for (int kk = 0; kk < kBK / 32; ++kk) tc05::mma_i8(d, ad + 2 * kk, bd + 2 * kk, kIdesc, (kb | kk) != 0);
              tc05::mma_commit(tc05::smem_u32(&sm.empty[s]));  // frees the stage when these MMAs finish
            }
            if (!ok) break;
            tc05::mma_commit(tc05::smem_u32(&sm.acc_full[g]));  // the group's tile is ready
            if ((issued >> g) & 1u) parity ^= 1u << g;   // the wait above consumed that phase
            issued |= 1u << g;
          }
        }
      }
      // every MMA of this thread has finished before the CTA can free TMEM
      tc05::mma_commit(tc05::smem_u32(&sm.final_mma));
      tc05::mbar_wait(tc05::smem_u32(&sm.final_mma), 0, kWaitLimitNs);
    }
  }
  } else {
    // each epilogue warpgroup takes its share of them
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kEpiRegs));
    // --------------------------------------------------------------- epilogue
    const int e = warp - 4;
    const int g = e >> 2;                       // this warp's group
    const int quarter = warp & 3;               // TMEM lanes 32 * quarter .. + 31
    const int p_local = 32 * quarter + lane;    // the position this thread hashes, in its unit
    const GroupSync gsync{1 + g, 128};
    const uint32_t ta0 = tmem + uint32_t(g * kBN) + (uint32_t(32 * quarter) << 16);
    const TreeMeta& m = A.meta;
    const int c_leaf = 1 << m.log2_chunk;
    uint32_t phase = 0;
    bool live = true;   // warp-uniform: false once a wait ran out or the CTA aborted
    for (int k = 0; kGroups * k + g < nj; ++k) {
      const UnitOf un = unit_of(a, int(blockIdx.x) + (kGroups * k + g) * int(gridDim.x));
      const int pos = un.m0 + p_local;
      const bool valid = pos < a.n_tokens;
      const int pos_c = valid ? pos : 0;        // table rows of padding positions are never used
      const KvtLayer& L = a.layers[un.layer];
      const double sx = (a.use_rope && valid)
                            ? double(__ldg(a.scale_x + int64_t(pos) * a.sx_t + int64_t(un.layer) * a.sx_l))
                            : 0.0;
      uint32_t st[8];
      sha_init(st);
      uint32_t carry[4] = {0x76692d6bu, 0x762d7631u, bswap32(uint32_t(A.layer_base + un.layer)),
                           bswap32(uint32_t(pos))};   // "vi-kv-v1" || u32le layer || u32le pos
#pragma unroll 1
      for (int t = 0; t < n_tiles && live; ++t) {
        if (__shfl_sync(0xffffffffu, aborted(sm) ? 1 : 0, 0)) {
          live = false;
          break;
        }
        bool got = false;
        if (lane == 0) got = tc05::mbar_wait(tc05::smem_u32(&sm.acc_full[g]), phase, kWaitLimitNs);
        got = __shfl_sync(0xffffffffu, got, 0);
        phase ^= 1u;
        if (!got) {
          if (lane == 0) set_abort(sm, a.err);
          live = false;
          break;
        }
        tc05::fence_after_sync();
        const int mat = t / tpm, c0 = (t % tpm) * kBN;
        Deq q;
        q.ch = mat ? L.ch[1] : L.ch[0];
        q.bias = mat ? L.bias[1] : L.bias[0];
        q.sx = sx;
        q.scale = __dmul_rn(double(mat ? L.sw[1] : L.sw[0]), sx);
        if (!a.use_rope) {
          tile_plain<kModeToy>(sm, g, lane, p_local, ta0, c0, q, st, carry);
        } else if (!q.ch && !q.bias) {
          if (mat == 0)
            tile_rope<kModeTensor, HD>(a, sm, g, lane, p_local, ta0, c0, pos_c, q, st, carry);
          else
            tile_plain<kModeTensor>(sm, g, lane, p_local, ta0, c0, q, st, carry);
        } else {
          if (mat == 0)
            tile_rope<kModeGeneral, HD>(a, sm, g, lane, p_local, ta0, c0, pos_c, q, st, carry);
          else
            tile_plain<kModeGeneral>(sm, g, lane, p_local, ta0, c0, q, st, carry);
        }
      }
      // last block: the two carried values, 0x80, zeros, the bit length
      {
        uint32_t w[16];
        w[0] = carry[0];
        w[1] = carry[1];
        w[2] = carry[2];
        w[3] = carry[3];
        w[4] = 0x80000000u;
#pragma unroll
        for (int i = 5; i < 15; ++i) w[i] = 0;
        w[15] = uint32_t(16 + 16 * a.kv_dim) * 8u;
        compress(st, w);
      }
      if (!valid) {
#pragma unroll
        for (int w = 0; w < 8; ++w) st[w] = 0;   // zero leaf: level-0 padding of build_tree
      }
      if (p_local < c_leaf) {
#pragma unroll
        for (int w = 0; w < 8; ++w) sm.sd[g][w][p_local] = st[w];
        if (A.out.nodes)
          store_digest(A.out.nodes + (m.node_base + int64_t(un.layer) * m.node_stride + pos) * 32, st);
      }
      // Every warp of the group reaches these barriers for every unit, whatever
      // its waits did (after an abort the digests are void, not missing).
      gsync();
      chunk_tail<kBM>(sm.sd[g], m, un.layer, un.mb, A.out, p_local, gsync, &sm.s_last[g]);
      // stop together: one thread reads the abort flag between two barriers
      gsync();
      if (p_local == 0) sm.stop[g] = (aborted(sm) || !live) ? 1 : 0;
      gsync();
      if (sm.stop[g]) break;
    }
  }

  tc05::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc05::fence_after_sync();
    tc05::tmem_dealloc(tmem, kGroups * kBN);
  }
}

template <int HD>
cudaError_t launch_hd(const KvtcArgs& a, int n_sm, cudaStream_t s) {
  const size_t smem = sizeof(Smem) + 1024;
  // setmaxnreg.inc waits until the registers it asks for are free: refuse a
  // build whose launch register count cannot cover the epilogue's share
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, kvt_commit_kernel<HD>);
  if (e != cudaSuccess) return e;
  if ((fa.numRegs - kCtlRegs) * 128 < kGroups * 128 * (kEpiRegs - fa.numRegs)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kvt_commit_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const int grid = std::max(1, std::min(a.n_units, n_sm));
  kvt_commit_kernel<HD><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool kvt_commit_supported(int head_dim, int kv_dim) {
  return (head_dim == 64 || head_dim == 128) && kv_dim % kBN == 0;
}

cudaError_t launch_kvt_commit(const KvtcArgs& a, int n_sm, cudaStream_t s) {
  return a.t.head_dim == 64 ? launch_hd<64>(a, n_sm, s) : launch_hd<128>(a, n_sm, s);
}

}  // namespace vc
