// Merkle reduction of one chunk of leaves and the levels above the chunks,
// shared by the kernels that hash leaves (merkle.cu, kvt_commit.cu).
//
// Tree semantics follow crates/verilm-core/src/merkle.rs: build_tree (11-48)
// pads level 0 with zero leaves to the next power of two; parent =
// hash_pair(left, right) (118-123); nodes are stored level-concatenated
// bottom-up, root last.
//
// The threads that run these functions are a "group" of NT threads with its
// own barrier: the whole CTA (CtaSync) or a 128-thread named-barrier group of a
// warp-specialised kernel (GroupSync).
#pragma once
#include "sha256_core.cuh"
#include "vc_internal.h"

namespace vc {

struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// bar.sync on named barrier `id` (1..15) for `count` threads (a multiple of 32).
struct GroupSync {
  int id, count;
  __device__ __forceinline__ void operator()() const {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
  }
};

__host__ __device__ __forceinline__ int64_t level_off(int lp, int k) {
  // Nodes before level k in a tree with 2^lp leaves: sum_{i<k} 2^(lp-i).
  return (int64_t(2) << lp) - (int64_t(2) << (lp - k));
}

__device__ __forceinline__ void store_z(uint8_t* p, const uint32_t* z) {
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = z[i];
  store_digest(p, h);
}

// Subtree of one chunk, in shared memory.  sd[w][i] is word w of leaf i; tid
// is the thread's index in its group.
template <int NT, class Sync>
__device__ __forceinline__ void chunk_reduce(uint32_t (*sd)[NT], int kc, uint8_t* tnodes, int lp, int64_t chunk,
                                             int tid, Sync sync) {
  for (int k = 0; k < kc; ++k) {
    const int half = 1 << (kc - k - 1);
    uint32_t out[8];
    if (tid < half) {
      uint32_t l[8], r[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) { l[w] = sd[w][2 * tid]; r[w] = sd[w][2 * tid + 1]; }
      hash_pair(l, r, out);
    }
    sync();
    if (tid < half) {
#pragma unroll
      for (int w = 0; w < 8; ++w) sd[w][tid] = out[w];
      if (tnodes) store_digest(tnodes + (level_off(lp, k + 1) + (chunk << (kc - k - 1)) + tid) * 32, out);
    }
    sync();
  }
}

// Levels above the chunks, run by the group that finished a tree's last chunk.
// tnodes: the tree's node array (nullptr in roots-only mode, where tcroot
// holds the chunk roots and is reduced in place).
template <int NT, class Sync>
__device__ void finish_tree(uint8_t* tnodes, uint8_t* tcroot, int64_t n, int lp, int kc, int n_chunks,
                            const uint32_t* Z, uint8_t* root_out, int tid, Sync sync) {
  if (tnodes) {
    // Zero-padding chunks: every node of theirs at levels 0..kc is Z_k.
    const int64_t m = int64_t(1) << (lp - kc);
    for (int k = 0; k <= kc; ++k) {
      const int64_t per = int64_t(1) << (kc - k);
      uint8_t* lvl = tnodes + level_off(lp, k) * 32;
      for (int64_t i = int64_t(n_chunks) * per + tid; i < m * per; i += NT) store_z(lvl + i * 32, Z + 8 * k);
    }
  }
  for (int k = kc; k < lp; ++k) {
    const int64_t real_k = (n + (int64_t(1) << k) - 1) >> k;
    const int64_t real_k1 = (n + (int64_t(1) << (k + 1)) - 1) >> (k + 1);
    const int64_t half = int64_t(1) << (lp - k - 1);
    const uint8_t* src = tnodes ? tnodes + level_off(lp, k) * 32 : tcroot;
    uint8_t* dst = tnodes ? tnodes + level_off(lp, k + 1) * 32 : tcroot;
    const int64_t lim = tnodes ? half : real_k1;
    for (int64_t base = 0; base < lim; base += NT) {
      const int64_t i = base + tid;
      uint32_t out[8];
      const bool have = i < lim;
      if (have) {
        if (i < real_k1) {
          uint32_t l[8], r[8];
          load_digest_cg(src + (2 * i) * 32, l);
          if (2 * i + 1 < real_k) {
            load_digest_cg(src + (2 * i + 1) * 32, r);
          } else {
#pragma unroll
            for (int w = 0; w < 8; ++w) r[w] = Z[8 * k + w];
          }
          hash_pair(l, r, out);
        } else {
#pragma unroll
          for (int w = 0; w < 8; ++w) out[w] = Z[8 * (k + 1) + w];
        }
      }
      sync();  // in-place mode: every read of this pass precedes the writes
      if (have) store_digest(dst + i * 32, out);
    }
    sync();
  }
  if (tid == 0) {
    uint32_t r[8];
    load_digest_cg(tnodes ? tnodes + level_off(lp, lp) * 32 : tcroot, r);
    store_digest(root_out, r);
  }
}

// Common tail of a chunk: reduce, publish, and finish the tree if this group
// completed its last chunk (threadfence reduction on a per-tree counter, no
// waiting).  s_last: one shared int per group.
template <int NT, class Sync>
__device__ __forceinline__ void chunk_tail(uint32_t (*sd)[NT], const TreeMeta& m, int layer, int64_t chunk,
                                           const TreeOut& o, int tid, Sync sync, int* s_last) {
  const int lp = m.log2_pad, kc = m.log2_chunk;
  uint8_t* tnodes = o.nodes ? o.nodes + (m.node_base + int64_t(layer) * m.node_stride) * 32 : nullptr;
  uint8_t* tcroot = o.nodes ? nullptr : o.croots + (m.croot_base + int64_t(layer) * m.croot_stride) * 32;
  const int tree = m.tree_base + layer;
  chunk_reduce<NT>(sd, kc, tnodes, lp, chunk, tid, sync);
  if (!tnodes && tid == 0) {
    uint32_t r[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) r[w] = sd[w][0];
    store_digest(tcroot + chunk * 32, r);
  }
  if (m.n_chunks == 1) {
    finish_tree<NT>(tnodes, tcroot, m.n_leaves, lp, kc, 1, o.zero_roots, o.roots + int64_t(tree) * 32, tid, sync);
    return;
  }
  __threadfence();
  sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(o.counters + tree, 1u);
    *s_last = (prev == unsigned(m.n_chunks - 1));
  }
  sync();
  if (*s_last) {
    __threadfence();
    finish_tree<NT>(tnodes, tcroot, m.n_leaves, lp, kc, m.n_chunks, o.zero_roots, o.roots + int64_t(tree) * 32,
                    tid, sync);
    if (tid == 0) o.counters[tree] = 0u;
  }
}

}  // namespace vc
