// Merkle kernels: KV leaves fused with their subtree reduction, generic trees
// over given leaves, and openings.
//
// Tree semantics follow crates/verilm-core/src/merkle.rs:
//   build_tree (11-48): level 0 is the leaves zero-padded to the next power of
//   two; parent = hash_pair(left, right) = SHA256(left || right) (118-123);
//   nodes are stored level-concatenated bottom-up, root last.
//   prove (79-99): siblings bottom-up, sibling = idx ^ 1 at each level.
//
// Work split: a CTA owns an aligned chunk of up to 128 leaves of one tree
// (one thread per leaf).  It hashes the leaves, reduces the chunk to its
// subtree root in shared memory, and counts itself done on the tree's
// counter; the CTA that completes a tree's last chunk finishes the levels
// above the chunks (threadfence reduction, no waiting anywhere).  Chunks that
// hold only zero padding are never launched: their subtree root is the
// constant Z_k (Z_0 = 0^32, Z_{k+1} = hash_pair(Z_k, Z_k)), which is exactly
// what build_tree computes for them.
#include "merkle_tree.cuh"
#include "sha256_core.cuh"
#include "sha256_stream.cuh"
#include "vc_internal.h"

#include <cstring>

namespace vc {

// ---------------------------------------------------------------------------
// f64 widening.  The message of hash_kv_entry holds f64le values
// (merkle.rs:274-293); a K/V row of bf16 or f32 is widened exactly.
// For an f64 d the two message words are bswap(lo32(d)), bswap(hi32(d)).
// ---------------------------------------------------------------------------

// Exact f32 -> f64 bit widening, every class: normal, zero, subnormal
// (renormalised), infinity, NaN (payload kept, quiet bit set).
__device__ __forceinline__ void f32_to_f64_bits(uint32_t f, uint32_t& hi, uint32_t& lo) {
  const uint32_t s = f & 0x80000000u, a = f & 0x7FFFFFFFu;
  const uint32_t e = a >> 23, m = a & 0x7FFFFFu;
  if (e - 1u < 254u) {
    hi = s | ((a >> 3) + 0x38000000u);
    lo = m << 29;
  } else if (a == 0) {
    hi = s;
    lo = 0;
  } else if (e == 0) {
    const int p = 31 - __clz(m);  // f32 subnormal m * 2^-149 = 2^(p-149) * 1.xxx
    const uint64_t mant = (uint64_t(m) << (52 - p)) & 0xFFFFFFFFFFFFFull;
    const uint64_t d = (uint64_t(p + 874) << 52) | mant;
    hi = s | uint32_t(d >> 32);
    lo = uint32_t(d);
  } else {
    hi = s | 0x7FF00000u | (m >> 3) | (m ? 0x80000u : 0u);
    lo = m << 29;
  }
}

// bf16 pair (two elements in one little-endian word) -> the big-endian
// message word of hi32(f64) of each (lo32 is 0 for every bf16 value).  The
// hardware f32 -> f64 conversion is exact for every bf16 bit pattern --
// zeros, subnormals, infinities, and NaNs (payload kept, quiet bit set) --
// which was checked against f32_to_f64_bits over all 65 536 patterns on
// sm_100a; it runs outside the integer ALU pipe the compression saturates.
__device__ __forceinline__ void bf16x2_words(uint32_t x, uint32_t& w0, uint32_t& w1) {
  const double d0 = double(__uint_as_float(x << 16));
  const double d1 = double(__uint_as_float(x & 0xFFFF0000u));
  w0 = bswap32(uint32_t(__double2hiint(d0)));
  w1 = bswap32(uint32_t(__double2hiint(d1)));
}

// Walks the 8-element chunks of a K/V row pair: K heads then V heads, each
// head contiguous, heads stride_head apart.
struct RowCursor {
  const char* kb;
  const char* vb;
  int64_t hs;     // bytes between heads
  int cb;         // bytes per chunk
  int cph;        // chunks per head
  int nh;
  int sel, h, ci;
  __device__ __forceinline__ const char* next() {
    const char* p = (sel ? vb : kb) + int64_t(h) * hs + int64_t(ci) * cb;
    if (++ci == cph) {
      ci = 0;
      if (++h == nh) {
        h = 0;
        sel = 1;
      }
    }
    return p;
  }
};

template <int DT> struct Chunk;
template <> struct Chunk<0> {  // bf16: 8 elements = 16 bytes
  uint4 q;
  __device__ __forceinline__ void load(const char* p) { q = __ldg(reinterpret_cast<const uint4*>(p)); }
};
template <> struct Chunk<1> {  // f32: 32 bytes
  uint4 q[2];
  __device__ __forceinline__ void load(const char* p) {
    q[0] = __ldg(reinterpret_cast<const uint4*>(p));
    q[1] = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  }
};
template <> struct Chunk<2> {  // f64: 64 bytes
  uint4 q[4];
  __device__ __forceinline__ void load(const char* p) {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __ldg(reinterpret_cast<const uint4*>(p) + i);
  }
};

// Message words of element i (0..7) of a chunk: w[2j] = bswap(lo32),
// w[2j+1] = bswap(hi32).  `out` receives elements [e0, e0+n).
__device__ __forceinline__ void chunk_words(const Chunk<0>& c, int e0, int n, uint32_t* out) {
  const uint32_t x[4] = {c.q.x, c.q.y, c.q.z, c.q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (2 * j + 1 < e0 || 2 * j >= e0 + n) continue;
    uint32_t w0, w1;
    bf16x2_words(x[j], w0, w1);
    if (2 * j >= e0) { out[2 * (2 * j - e0)] = 0; out[2 * (2 * j - e0) + 1] = w0; }
    if (2 * j + 1 < e0 + n) { out[2 * (2 * j + 1 - e0)] = 0; out[2 * (2 * j + 1 - e0) + 1] = w1; }
  }
}
__device__ __forceinline__ void chunk_words(const Chunk<1>& c, int e0, int n, uint32_t* out) {
  const uint32_t x[8] = {c.q[0].x, c.q[0].y, c.q[0].z, c.q[0].w, c.q[1].x, c.q[1].y, c.q[1].z, c.q[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < e0 || i >= e0 + n) continue;
    uint32_t hi, lo;
    f32_to_f64_bits(x[i], hi, lo);
    out[2 * (i - e0)] = bswap32(lo);
    out[2 * (i - e0) + 1] = bswap32(hi);
  }
}
__device__ __forceinline__ void chunk_words(const Chunk<2>& c, int e0, int n, uint32_t* out) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < e0 || i >= e0 + n) continue;
    const uint4& q = c.q[i >> 1];
    const uint32_t lo = (i & 1) ? q.z : q.x;
    const uint32_t hi = (i & 1) ? q.w : q.y;
    out[2 * (i - e0)] = bswap32(lo);
    out[2 * (i - e0) + 1] = bswap32(hi);
  }
}

// One block = the last 2 elements of the previous chunk + the first 6 of
// the current one (the 16-byte leaf prefix shifts f64 slots by two).
template <int DT>
__device__ __forceinline__ void block_words(const Chunk<DT>& prev, const Chunk<DT>& cur, uint32_t w[16]) {
  chunk_words(prev, 6, 2, w);
  chunk_words(cur, 0, 6, w + 4);
}

// hash_kv_entry (merkle.rs:285-293) of one (layer, position) with
// kv_dim % 8 == 0 and head_dim % 8 == 0.
template <int DT>
__device__ __forceinline__ void kv_leaf(uint32_t st[8], uint32_t layer, uint32_t pos, RowCursor rc,
                                        int n_chunks, uint32_t bitlen) {
  sha_init(st);
  uint32_t w[16];
  Chunk<DT> cur, nxt, prev;
  cur.load(rc.next());
  nxt.load(rc.next());
  // Block 0: "vi-kv-v1" || u32le layer || u32le pos || elements 0..5.
  w[0] = 0x76692d6bu;  // "vi-k"
  w[1] = 0x762d7631u;  // "v-v1"
  w[2] = bswap32(layer);
  w[3] = bswap32(pos);
  chunk_words(cur, 0, 6, w + 4);
  compress(st, w);
  for (int b = 1; b < n_chunks; ++b) {
    prev = cur;
    cur = nxt;
    if (b + 1 < n_chunks) nxt.load(rc.next());
    block_words<DT>(prev, cur, w);
    compress(st, w);
  }
  // Last block: elements 2*kv-2, 2*kv-1, then 0x80, zeros, bit length.
  chunk_words(cur, 6, 2, w);
  w[4] = 0x80000000u;
#pragma unroll
  for (int i = 5; i < 15; ++i) w[i] = 0;
  w[15] = bitlen;
  compress(st, w);
}

// Element offset of the row of position p, or -1 (error flagged) when the
// row does not lie inside the cache buffer.
__device__ __forceinline__ int64_t kv_row(const KvArgs& a, const TreeMeta& m, int64_t p) {
  int64_t off;
  if (a.paged) {
    const int32_t page = __ldg(a.block_tables + int64_t(m.seq) * a.max_blocks + p / a.block_size);
    off = int64_t(page) * a.stride_page + (p % a.block_size) * a.stride_row;
    if (page < 0) off = -1;
  } else {
    off = (m.src_off + p) * a.stride_row;
  }
  if (off < 0 || off + a.row_span > a.cache_elems) {
    atomicExch(a.err, 1);
    return -1;
  }
  return off;
}

template <int DT>
__global__ void __launch_bounds__(kTreeThreads) kv_commit_kernel(KvArgs a) {
  __shared__ uint32_t sd[8][kTreeThreads];
  __shared__ int s_last;
  const int2 it = a.items[blockIdx.x];
  const TreeMeta m = a.meta[it.x];
  const int layer = blockIdx.y;
  const int tid = threadIdx.x;
  const int c = 1 << m.log2_chunk;
  const int64_t chunk = it.y;
  const int64_t p = chunk * c + tid;
  if (tid < c) {
    uint32_t d[8];
    const int64_t row = p < m.n_leaves ? kv_row(a, m, p) : -1;
    if (row >= 0) {
      constexpr int esz = DT == 0 ? 2 : (DT == 1 ? 4 : 8);
      const int64_t off = row * esz;
      RowCursor rc;
      rc.kb = static_cast<const char*>(a.k_layers[layer]) + off;
      rc.vb = static_cast<const char*>(a.v_layers[layer]) + off;
      rc.hs = a.stride_head * esz;
      rc.cb = 8 * esz;
      rc.cph = a.head_dim >> 3;
      rc.nh = a.n_heads;
      rc.sel = 0; rc.h = 0; rc.ci = 0;
      const int kv = a.n_heads * a.head_dim;
      kv_leaf<DT>(d, uint32_t(a.layer_base + layer), uint32_t(m.pos_base + p), rc, kv >> 2,
                  uint32_t(16 + 16 * kv) * 8u);
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = 0;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) sd[w][tid] = d[w];
    if (a.out.nodes) store_digest(a.out.nodes + (m.node_base + int64_t(layer) * m.node_stride + p) * 32, d);
  }
  __syncthreads();
  chunk_tail<kTreeThreads>(sd, m, layer, chunk, a.out, tid, CtaSync(), &s_last);
}

// Generic path for any kv_dim / head_dim: the stream engine, element by element.
template <int DT>
__global__ void __launch_bounds__(kTreeThreads) kv_commit_generic_kernel(KvArgs a) {
  __shared__ uint32_t sd[8][kTreeThreads];
  __shared__ int s_last;
  __shared__ uint32_t sbuf[16 * kTreeThreads];
  const int2 it = a.items[blockIdx.x];
  const TreeMeta m = a.meta[it.x];
  const int layer = blockIdx.y;
  const int tid = threadIdx.x;
  const int c = 1 << m.log2_chunk;
  const int64_t chunk = it.y;
  const int64_t p = chunk * c + tid;
  if (tid < c) {
    uint32_t d[8];
    const int64_t row = p < m.n_leaves ? kv_row(a, m, p) : -1;
    if (row >= 0) {
      constexpr int esz = DT == 0 ? 2 : (DT == 1 ? 4 : 8);
      const int64_t off = row * esz;
      Sha256Stream<kTreeThreads> s;
      s.init(sbuf + tid);
      s.put_be(0x76692d6bu);
      s.put_be(0x762d7631u);
      s.put_be(bswap32(uint32_t(a.layer_base + layer)));
      s.put_be(bswap32(uint32_t(m.pos_base + p)));
      for (int sel = 0; sel < 2; ++sel) {
        const char* row = static_cast<const char*>(sel ? a.v_layers[layer] : a.k_layers[layer]) + off;
        for (int h = 0; h < a.n_heads; ++h) {
          const char* hp = row + int64_t(h) * a.stride_head * esz;
          for (int i = 0; i < a.head_dim; ++i) {
            uint32_t hi, lo;
            if (DT == 0) {
              f32_to_f64_bits(uint32_t(__ldg(reinterpret_cast<const uint16_t*>(hp) + i)) << 16, hi, lo);
            } else if (DT == 1) {
              f32_to_f64_bits(__ldg(reinterpret_cast<const uint32_t*>(hp) + i), hi, lo);
            } else {
              const uint2 v = __ldg(reinterpret_cast<const uint2*>(hp) + i);
              lo = v.x;
              hi = v.y;
            }
            s.put_be(bswap32(lo));
            s.put_be(bswap32(hi));
          }
        }
      }
      s.finish();
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = s.h[w];
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = 0;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) sd[w][tid] = d[w];
    if (a.out.nodes) store_digest(a.out.nodes + (m.node_base + int64_t(layer) * m.node_stride + p) * 32, d);
  }
  __syncthreads();
  chunk_tail<kTreeThreads>(sd, m, layer, chunk, a.out, tid, CtaSync(), &s_last);
}

__global__ void __launch_bounds__(kTreeThreads) tree_commit_kernel(TreeArgs a) {
  __shared__ uint32_t sd[8][kTreeThreads];
  __shared__ int s_last;
  const int2 it = a.items[blockIdx.x];
  const TreeMeta m = a.meta[it.x];
  const int tid = threadIdx.x;
  const int c = 1 << m.log2_chunk;
  const int64_t chunk = it.y;
  const int64_t p = chunk * c + tid;
  if (tid < c) {
    uint32_t d[8];
    if (p < m.n_leaves) {
      load_digest(a.leaves + (m.src_off + p) * 32, d);
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = 0;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) sd[w][tid] = d[w];
    if (a.out.nodes) store_digest(a.out.nodes + (m.node_base + p) * 32, d);
  }
  __syncthreads();
  chunk_tail<kTreeThreads>(sd, m, 0, chunk, a.out, tid, CtaSync(), &s_last);
}

__global__ void zero_roots_kernel(uint32_t* z) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint32_t cur[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int k = 0; k <= kMaxTreeHeight; ++k) {
#pragma unroll
    for (int w = 0; w < 8; ++w) z[8 * k + w] = cur[w];
    uint32_t nxt[8];
    hash_pair(cur, cur, nxt);
#pragma unroll
    for (int w = 0; w < 8; ++w) cur[w] = nxt[w];
  }
}

// merkle::prove (merkle.rs:79-99): one thread per (opening, level).
__global__ void prove_kernel(const uint8_t* nodes, const ProveReq* reqs, int n, int max_depth,
                             uint8_t* siblings) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= int64_t(n) * max_depth) return;
  const int r = int(gid / max_depth);
  const int k = int(gid % max_depth);
  const ProveReq q = reqs[r];
  if (k >= q.log2_pad) return;
  const int64_t sib = int64_t((q.leaf >> k) ^ 1u);
  const uint4* src = reinterpret_cast<const uint4*>(nodes + (q.node_base + level_off(q.log2_pad, k) + sib) * 32);
  uint4* dst = reinterpret_cast<uint4*>(siblings + gid * 32);
  dst[0] = src[0];
  dst[1] = src[1];
}


// ---------------------------------------------------------------------------
// Allocation-free KV commit: vc_kv_commit_noalloc.
//
// Some callers cannot allocate device memory at the moment they commit: a
// serving engine that reserves all free HBM for its KV cache at start-up, an
// allocator-less embedding, or code running where a cudaMalloc would stall
// the device.  This variant of kv_commit_kernel needs no allocation at all:
// its scratch (per-tree completion counters and per-chunk subtree roots) and
// its padding-root table live in file-scope device arrays that every GPU
// which loads the library holds until the process exits, and its descriptor
// tables travel as one kernel argument.  The caller passes inputs and outputs
// exactly as for vc_kv_commit; no tree nodes are kept (roots only).
// ---------------------------------------------------------------------------
constexpr int kNoAllocMaxSeqs = 64;
constexpr int kNoAllocMaxLayers = 256;
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr size_t kNoAllocErrBytes = 256;                   // internal bounds flag

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(16) uint32_t g_noalloc_zero[(kMaxTreeHeight + 1) * 8];

struct NoAllocArgs {
  KvArgs kv;                                 // meta, items, k_layers, v_layers unused
  TreeMeta meta[kNoAllocMaxSeqs];
  int32_t chunk_off[kNoAllocMaxSeqs + 1];    // first chunk of each sequence in the grid
  int32_t n_seqs;
  const void* k_layers[kNoAllocMaxLayers];
  const void* v_layers[kNoAllocMaxLayers];
};

template <int DT>
__global__ void __launch_bounds__(kTreeThreads) kv_commit_noalloc_kernel(const __grid_constant__ NoAllocArgs na) {
  __shared__ uint32_t sd[8][kTreeThreads];
  __shared__ int s_last;
  const KvArgs& a = na.kv;
  int sq = 0;
  while (sq + 1 < na.n_seqs && na.chunk_off[sq + 1] <= int(blockIdx.x)) ++sq;
  const TreeMeta m = na.meta[sq];
  const int layer = blockIdx.y;
  const int tid = threadIdx.x;
  const int c = 1 << m.log2_chunk;
  const int64_t chunk = int64_t(blockIdx.x) - na.chunk_off[sq];
  const int64_t p = chunk * c + tid;
  if (tid < c) {
    uint32_t d[8];
    const int64_t row = p < m.n_leaves ? kv_row(a, m, p) : -1;
    if (row >= 0) {
      constexpr int esz = DT == 0 ? 2 : (DT == 1 ? 4 : 8);
      const int64_t off = row * esz;
      RowCursor rc;
      rc.kb = static_cast<const char*>(na.k_layers[layer]) + off;
      rc.vb = static_cast<const char*>(na.v_layers[layer]) + off;
      rc.hs = a.stride_head * esz;
      rc.cb = 8 * esz;
      rc.cph = a.head_dim >> 3;
      rc.nh = a.n_heads;
      rc.sel = 0; rc.h = 0; rc.ci = 0;
      const int kv = a.n_heads * a.head_dim;
      kv_leaf<DT>(d, uint32_t(a.layer_base + layer), uint32_t(m.pos_base + p), rc, kv >> 2,
                  uint32_t(16 + 16 * kv) * 8u);
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) d[w] = 0;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) sd[w][tid] = d[w];
  }
  __syncthreads();
  chunk_tail<kTreeThreads>(sd, m, layer, chunk, a.out, tid, CtaSync(), &s_last);
}

}  // namespace vc

#include <mutex>
#include "../../include/vcommit.h"

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
bool g_noalloc_ready[kNoAllocMaxDevices];
unsigned char* g_noalloc_scratch_ptr[kNoAllocMaxDevices];
uint32_t* g_noalloc_zero_ptr[kNoAllocMaxDevices];

// First call on a device: host code cannot use the arrays' names as device
// addresses, so look the addresses up (with that device current) and fill
// the padding-root table.  Synchronises the stream once.
vc_status noalloc_setup(int dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ready[dev]) return VC_OK;
  void* sp = nullptr;
  void* zp = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&sp, vc::g_noalloc_scratch);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&zp, vc::g_noalloc_zero);
  if (e != cudaSuccess) return vc::set_error(VC_ECUDA, "vc_kv_commit_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  e = vc::launch_zero_roots(static_cast<uint32_t*>(zp), stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return vc::set_error(VC_ECUDA, "vc_kv_commit_noalloc: set-up: %s", cudaGetErrorString(e));
  g_noalloc_scratch_ptr[dev] = static_cast<unsigned char*>(sp);
  g_noalloc_zero_ptr[dev] = static_cast<uint32_t*>(zp);
  g_noalloc_ready[dev] = true;
  return VC_OK;
}

}  // namespace

extern "C" vc_status vc_kv_commit_noalloc(const vc_kv_desc* d, uint8_t* kv_roots_dev, int32_t* err_flag_dev,
                                          void* stream_) {
  using namespace vc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (!d || !kv_roots_dev) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: NULL argument");
  if (d->n_layers < 1 || d->n_seqs < 1 || d->n_kv_heads < 1 || d->head_dim < 1)
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: n_layers, n_seqs, n_kv_heads, head_dim must be >= 1");
  if (d->n_seqs > kNoAllocMaxSeqs || d->n_layers > kNoAllocMaxLayers)
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: at most %d sequences and %d layers per call (got %d, %d)",
                     kNoAllocMaxSeqs, kNoAllocMaxLayers, d->n_seqs, d->n_layers);
  if (d->dtype < VC_DTYPE_BF16 || d->dtype > VC_DTYPE_F64) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: bad dtype");
  if (!d->seq_lens || !d->k_layers || !d->v_layers) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: NULL table");
  if (d->pos_base || d->tree_log2 != 0)
    return set_error(VC_ENOTSUP, "vc_kv_commit_noalloc: split trees (pos_base, tree_log2) are not supported");
  if (d->cache_elems <= 0 || d->stride_row < 0 || d->stride_head < 0 || d->stride_page < 0)
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: cache_elems must be > 0 and strides >= 0");
  const int64_t kv = int64_t(d->n_kv_heads) * d->head_dim;
  const int esz = d->dtype == VC_DTYPE_BF16 ? 2 : (d->dtype == VC_DTYPE_F32 ? 4 : 8);
  const bool paged = d->block_tables != nullptr;
  if (paged && (d->block_size < 1 || d->max_blocks_per_seq < 1))
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: paged layout needs block_size and max_blocks_per_seq >= 1");
  // A page id from the device block table is only checked on the GPU; without
  // a flag to report a bad one, its leaf would hash as zeros and the call
  // would return a wrong root as success.
  if (paged && !err_flag_dev)
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: a paged layout needs err_flag_dev (bad page ids are "
                                "only detected on the device)");
  bool fast = kv % 8 == 0 && d->head_dim % 8 == 0 && (d->stride_row * esz) % 16 == 0 &&
              (d->stride_head * esz) % 16 == 0 && (!paged || (d->stride_page * esz) % 16 == 0);
  for (int l = 0; l < d->n_layers && fast; ++l)
    fast = d->k_layers[l] && d->v_layers[l] && reinterpret_cast<uintptr_t>(d->k_layers[l]) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(d->v_layers[l]) % 16 == 0;
  if (!fast)
    return set_error(VC_ENOTSUP, "vc_kv_commit_noalloc: needs kv_dim and head_dim multiples of 8 and 16-byte aligned "
                                 "rows (use vc_kv_commit otherwise)");
  const int64_t row_span = int64_t(d->n_kv_heads - 1) * d->stride_head + d->head_dim;

  NoAllocArgs na;
  std::memset(&na, 0, sizeof(na));
  int64_t acc = 0, croots = 0;
  int32_t chunks = 0;
  for (int s = 0; s < d->n_seqs; ++s) {
    const int64_t n = d->seq_lens[s];
    if (n < 1) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: seq_lens[%d] = %lld (need at least one leaf)", s, (long long)n);
    const int64_t r0 = d->seq_row_offset ? d->seq_row_offset[s] : acc;
    if (paged) {
      if ((n + d->block_size - 1) / d->block_size > d->max_blocks_per_seq)
        return set_error(VC_EINVAL, "vc_kv_commit_noalloc: seq %d needs more than max_blocks_per_seq pages", s);
    } else if (r0 < 0 || (r0 + n - 1) * d->stride_row + row_span > d->cache_elems) {
      return set_error(VC_EINVAL, "vc_kv_commit_noalloc: rows of seq %d exceed cache_elems", s);
    }
    TreeMeta& m = na.meta[s];
    int lp = 0;
    while ((int64_t(1) << lp) < n) ++lp;
    const int kc = lp < kLog2TreeThreads ? lp : kLog2TreeThreads;
    m.n_leaves = n;
    m.log2_pad = lp;
    m.log2_chunk = kc;
    m.n_chunks = int32_t((n + (int64_t(1) << kc) - 1) >> kc);
    m.node_stride = 0;
    m.node_base = 0;
    m.croot_stride = (int64_t(1) << lp) >> kc;
    m.croot_base = croots;
    croots += int64_t(d->n_layers) * m.croot_stride;
    m.src_off = r0;
    m.tree_base = s * d->n_layers;
    m.seq = s;
    na.chunk_off[s] = chunks;
    if (int64_t(chunks) + m.n_chunks > 0x7FFFFFFF) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: too many chunks");
    chunks += m.n_chunks;
    acc += n;
  }
  na.chunk_off[d->n_seqs] = chunks;
  na.n_seqs = d->n_seqs;
  const int n_trees = d->n_seqs * d->n_layers;
  const size_t counters_bytes = (size_t(n_trees) * 4 + 255) / 256 * 256;
  const size_t need = kNoAllocErrBytes + counters_bytes + size_t(croots) * 32;
  if (need > kNoAllocScratchBytes)
    return set_error(VC_EINVAL, "vc_kv_commit_noalloc: needs %zu bytes of scratch, the fixed maximum is %zu bytes "
                                "(commit fewer sequences or layers per call)", need, kNoAllocScratchBytes);
  for (int l = 0; l < d->n_layers; ++l) {
    na.k_layers[l] = d->k_layers[l];
    na.v_layers[l] = d->v_layers[l];
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(VC_ECUDA, "vc_kv_commit_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(VC_EINVAL, "vc_kv_commit_noalloc: device %d", dev);
  vc_status st = noalloc_setup(dev, stream);
  if (st) return st;
  unsigned char* scratch = g_noalloc_scratch_ptr[dev];
  KvArgs& a = na.kv;
  a.block_tables = d->block_tables;
  a.stride_page = d->stride_page;
  a.stride_row = d->stride_row;
  a.stride_head = d->stride_head;
  a.block_size = paged ? d->block_size : 1;
  a.max_blocks = d->max_blocks_per_seq;
  a.n_heads = d->n_kv_heads;
  a.head_dim = d->head_dim;
  a.layer_base = d->layer_base;
  a.paged = paged ? 1 : 0;
  a.cache_elems = d->cache_elems;
  a.row_span = row_span;
  // Contiguous rows were all checked above, so the internal word is never set for them.
  a.err = err_flag_dev ? err_flag_dev : reinterpret_cast<int*>(scratch);
  a.out.nodes = nullptr;
  a.out.counters = reinterpret_cast<uint32_t*>(scratch + kNoAllocErrBytes);
  a.out.croots = scratch + kNoAllocErrBytes + counters_bytes;
  a.out.roots = kv_roots_dev;
  a.out.zero_roots = g_noalloc_zero_ptr[dev];
  // The counters must start at zero; a call that failed part-way may have
  // left some set, so clear them (and the internal flag) every time.
  e = cudaMemsetAsync(scratch, 0, kNoAllocErrBytes + counters_bytes, stream);
  if (e == cudaSuccess) {
    dim3 grid(chunks, d->n_layers);
    switch (d->dtype) {
      case VC_DTYPE_BF16: kv_commit_noalloc_kernel<0><<<grid, kTreeThreads, 0, stream>>>(na); break;
      case VC_DTYPE_F32: kv_commit_noalloc_kernel<1><<<grid, kTreeThreads, 0, stream>>>(na); break;
      default: kv_commit_noalloc_kernel<2><<<grid, kTreeThreads, 0, stream>>>(na); break;
    }
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return set_error(VC_ECUDA, "vc_kv_commit_noalloc launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

namespace vc {

// KvEntry {k_roped, v_deq} of every (selected layer, position): the rows the
// leaves hashed, widened to f64 exactly as the leaf kernel widens them.  One
// CTA per (layer, position), threads stride over the kv_dim elements.
template <int DT>
__global__ void kv_entries_kernel(KvOpenArgs a) {
  const int sel = blockIdx.x / a.n_pos;
  const int pos = blockIdx.x % a.n_pos;
  const int layer = a.layers[sel];
  const int64_t row = kv_row(a.kv, a.seq, pos);
  double* out = a.out + (int64_t(sel) * a.n_pos + pos) * 2 * a.kv_dim;
  for (int e = threadIdx.x; e < 2 * a.kv_dim; e += blockDim.x) {
    double v = 0.0;
    if (row >= 0) {
      const int sel_v = e >= a.kv_dim;
      const int i = sel_v ? e - a.kv_dim : e;
      const int h = i / a.kv.head_dim, dd = i % a.kv.head_dim;
      const int64_t off = row + int64_t(h) * a.kv.stride_head + dd;
      const void* base = sel_v ? a.kv.v_layers[layer] : a.kv.k_layers[layer];
      if (DT == 0) {
        v = double(__uint_as_float(uint32_t(__ldg(static_cast<const uint16_t*>(base) + off)) << 16));
      } else if (DT == 1) {
        uint32_t hi, lo;
        f32_to_f64_bits(__ldg(static_cast<const uint32_t*>(base) + off), hi, lo);
        v = __hiloint2double(int(hi), int(lo));
      } else {
        v = __ldg(static_cast<const double*>(base) + off);
      }
    }
    out[e] = v;
  }
}

cudaError_t launch_kv_entries(const KvOpenArgs& a, int dtype, cudaStream_t s) {
  const int64_t n = int64_t(a.n_sel) * a.n_pos;
  if (n == 0) return cudaSuccess;
  switch (dtype) {
    case 0: kv_entries_kernel<0><<<int(n), 128, 0, s>>>(a); break;
    case 1: kv_entries_kernel<1><<<int(n), 128, 0, s>>>(a); break;
    default: kv_entries_kernel<2><<<int(n), 128, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

// One CTA per (empty subtree, layer): every node at level k is Z_k.
__global__ void empty_tree_kernel(const TreeMeta* meta, const int32_t* which, TreeOut o) {
  const TreeMeta m = meta[which[blockIdx.x]];
  const int layer = blockIdx.y;
  const int lp = m.log2_pad;
  if (o.nodes) {
    uint8_t* t = o.nodes + (m.node_base + int64_t(layer) * m.node_stride) * 32;
    for (int k = 0; k <= lp; ++k) {
      const int64_t cnt = int64_t(1) << (lp - k);
      uint8_t* lvl = t + level_off(lp, k) * 32;
      for (int64_t i = threadIdx.x; i < cnt; i += blockDim.x) store_z(lvl + i * 32, o.zero_roots + 8 * k);
    }
  }
  if (threadIdx.x == 0) store_z(o.roots + int64_t(m.tree_base + layer) * 32, o.zero_roots + 8 * lp);
}

cudaError_t launch_empty_trees(const TreeMeta* meta, const int32_t* which, int n_empty, int n_layers,
                               const TreeOut& o, cudaStream_t s) {
  if (n_empty == 0) return cudaSuccess;
  empty_tree_kernel<<<dim3(n_empty, n_layers), kTreeThreads, 0, s>>>(meta, which, o);
  return cudaGetLastError();
}

cudaError_t launch_zero_roots(uint32_t* z, cudaStream_t s) {
  zero_roots_kernel<<<1, 32, 0, s>>>(z);
  return cudaGetLastError();
}

cudaError_t launch_kv_commit(const KvArgs& a, int n_items, int n_layers, int dtype, bool fast,
                             cudaStream_t s) {
  dim3 grid(n_items, n_layers);
  if (fast) {
    switch (dtype) {
      case 0: kv_commit_kernel<0><<<grid, kTreeThreads, 0, s>>>(a); break;
      case 1: kv_commit_kernel<1><<<grid, kTreeThreads, 0, s>>>(a); break;
      default: kv_commit_kernel<2><<<grid, kTreeThreads, 0, s>>>(a); break;
    }
  } else {
    switch (dtype) {
      case 0: kv_commit_generic_kernel<0><<<grid, kTreeThreads, 0, s>>>(a); break;
      case 1: kv_commit_generic_kernel<1><<<grid, kTreeThreads, 0, s>>>(a); break;
      default: kv_commit_generic_kernel<2><<<grid, kTreeThreads, 0, s>>>(a); break;
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_tree_commit(const TreeArgs& a, int n_items, cudaStream_t s) {
  tree_commit_kernel<<<n_items, kTreeThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_prove(const uint8_t* nodes, const ProveReq* reqs, int n, int max_depth,
                         uint8_t* siblings, cudaStream_t s) {
  const int64_t total = int64_t(n) * max_depth;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  prove_kernel<<<int((total + threads - 1) / threads), threads, 0, s>>>(nodes, reqs, n, max_depth, siblings);
  return cudaGetLastError();
}

}  // namespace vc
