// C ABI of libvcommit.so (include/vcommit.h): argument validation, work
// planning, device staging of descriptor tables, and kernel launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/vcommit.h"
#include "vc_internal.h"

using namespace vc;

namespace {

thread_local std::string g_last_error;

vc_status fail(vc_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

#define VC_CUDA(call)                                                                   \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) return fail(VC_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

int ilog2_ceil(int64_t n) {
  int lp = 0;
  while ((int64_t(1) << lp) < n) ++lp;
  return lp;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

int32_t vc::set_error(int32_t status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

namespace {

// Node storage of released tree sets, kept for the next tree set of a
// similar size so a steady commit loop allocates nothing.  Shared by a
// context and the tree sets it made, so either may go first.  Blocks are
// stream-ordered: a block released on the context's stream is reused by
// later work on that stream only.
struct NodePool {
  std::mutex mu;
  bool closed = false;
  size_t cached = 0;
  std::multimap<size_t, uint8_t*> free_blocks;   // capacity -> block
  static constexpr size_t kMaxCached = size_t(16) << 30;
};

constexpr int kStageSlots = 16;  // descriptor uploads in flight before the host waits

// One pinned staging buffer and the event that says its copy has been read.
struct StageSlot {
  char* p = nullptr;
  size_t cap = 0;
  cudaEvent_t done = nullptr;
  bool pending = false;
};

}  // namespace

struct vc_tree_set {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint8_t* nodes = nullptr;
  size_t bytes = 0;                 // capacity of `nodes`
  std::shared_ptr<NodePool> pool;   // where `nodes` returns, or null
  std::vector<int64_t> node_base;   // per tree
  std::vector<int64_t> n_leaves;
  std::vector<int32_t> log2_pad;
};

struct vc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t* zero_roots = nullptr;   // device [kMaxTreeHeight + 1][8]
  int* err = nullptr;               // device error flag
  uint8_t* scratch = nullptr;       // device, grow-only
  size_t scratch_cap = 0;
  StageSlot stage[kStageSlots];     // host staging of descriptor tables, a ring
  int stage_next = 0;
  char* dargs = nullptr;            // device copy of the staged tables (stream-ordered reuse)
  size_t dargs_cap = 0;
  std::shared_ptr<NodePool> pool;
  int n_sm = 0;
  double* rope = nullptr;           // device (cos, sin) table of the last RoPE frequencies
  int64_t rope_rows = 0;            // positions held
  std::vector<double> rope_inv;     // the frequencies it was built for
};

namespace {

// Collects host tables into one staging image; upload() copies it to the
// device (stream-ordered) and returns the device base.
struct Stager {
  std::vector<char> img;
  size_t add(const void* p, size_t n, size_t align = 16) {
    const size_t off = align_up(img.size(), align);
    img.resize(off + n);
    if (n) std::memcpy(img.data() + off, p, n);
    return off;
  }
};

vc_status ensure_scratch(vc_ctx* c, size_t bytes) {
  if (bytes <= c->scratch_cap) return VC_OK;
  VC_CUDA(cudaStreamSynchronize(c->stream));
  if (c->scratch) cudaFree(c->scratch);
  c->scratch = nullptr;
  c->scratch_cap = 0;
  const size_t cap = std::max(bytes, size_t(1) << 20);
  if (cudaMalloc(&c->scratch, cap) != cudaSuccess) return fail(VC_ENOMEM, "scratch allocation of %zu bytes failed", cap);
  c->scratch_cap = cap;
  return VC_OK;
}

// Copies the staged tables to the device argument buffer on the context's
// stream.  The host copy goes through a ring of pinned slots, so the host
// only waits when kStageSlots earlier uploads have not yet been read by the
// GPU; the device buffer itself is reused in stream order.
vc_status upload(vc_ctx* c, const Stager& st, char** dev) {
  const size_t n = std::max<size_t>(st.img.size(), 16);
  StageSlot& sl = c->stage[c->stage_next];
  c->stage_next = (c->stage_next + 1) % kStageSlots;
  if (sl.pending) {
    VC_CUDA(cudaEventSynchronize(sl.done));
    sl.pending = false;
  }
  if (n > sl.cap) {
    if (sl.p) cudaFreeHost(sl.p);
    sl.p = nullptr;
    sl.cap = 0;
    const size_t cap = std::max(n, size_t(1) << 16);
    if (cudaMallocHost(&sl.p, cap) != cudaSuccess) return fail(VC_ENOMEM, "pinned staging of %zu bytes failed", cap);
    sl.cap = cap;
  }
  if (n > c->dargs_cap) {
    VC_CUDA(cudaStreamSynchronize(c->stream));
    if (c->dargs) cudaFree(c->dargs);
    c->dargs = nullptr;
    c->dargs_cap = 0;
    const size_t cap = std::max(n, size_t(1) << 16);
    if (cudaMalloc(&c->dargs, cap) != cudaSuccess) return fail(VC_ENOMEM, "argument buffer of %zu bytes failed", cap);
    c->dargs_cap = cap;
  }
  if (!st.img.empty()) std::memcpy(sl.p, st.img.data(), st.img.size());
  VC_CUDA(cudaMemcpyAsync(c->dargs, sl.p, n, cudaMemcpyHostToDevice, c->stream));
  VC_CUDA(cudaEventRecord(sl.done, c->stream));
  sl.pending = true;
  *dev = c->dargs;
  return VC_OK;
}

// Work plan of a set of trees (one TreeMeta per leaf group, one item per
// non-padding chunk).
struct Plan {
  std::vector<TreeMeta> meta;
  std::vector<int2> items;
  int64_t nodes = 0;
  int64_t croots = 0;
  int32_t n_trees = 0;
};

// lp_fixed > 0: a subtree of 2^lp_fixed leaves (split trees), n of them real.
void plan_group(Plan& p, int64_t n, int n_layers, int64_t src_off, int seq, int64_t pos_base = 0,
                int lp_fixed = 0) {
  TreeMeta m{};
  const int lp = lp_fixed > 0 ? lp_fixed : ilog2_ceil(n);
  const int kc = std::min(lp, kLog2TreeThreads);
  const int64_t pad = int64_t(1) << lp;
  m.n_leaves = n;
  m.log2_pad = lp;
  m.log2_chunk = kc;
  m.n_chunks = int32_t((n + (int64_t(1) << kc) - 1) >> kc);
  m.node_stride = 2 * pad - 1;
  m.node_base = p.nodes;
  p.nodes += int64_t(n_layers) * m.node_stride;
  m.croot_stride = pad >> kc;
  m.croot_base = p.croots;
  p.croots += int64_t(n_layers) * m.croot_stride;
  m.src_off = src_off;
  m.tree_base = p.n_trees;
  m.seq = seq;
  m.pos_base = pos_base;
  p.n_trees += n_layers;
  const int mi = int(p.meta.size());
  p.meta.push_back(m);
  for (int j = 0; j < m.n_chunks; ++j) p.items.push_back(make_int2(mi, j));
}

// Node storage for a tree set: a released block of the context's pool whose
// capacity is within 2x of the need, else a new stream-ordered allocation.
vc_status make_tree_set(vc_ctx* c, const Plan& p, int n_layers, vc_tree_set** out) {
  auto* ts = new (std::nothrow) vc_tree_set();
  if (!ts) return fail(VC_ENOMEM, "tree set allocation failed");
  ts->device = c->device;
  ts->stream = c->stream;
  ts->pool = c->pool;
  const size_t need = std::max<size_t>(size_t(p.nodes) * 32, 256);
  {
    std::lock_guard<std::mutex> lk(c->pool->mu);
    auto it = c->pool->free_blocks.lower_bound(need);
    if (it != c->pool->free_blocks.end() && it->first <= 2 * need) {
      ts->nodes = it->second;
      ts->bytes = it->first;
      c->pool->cached -= it->first;
      c->pool->free_blocks.erase(it);
    }
  }
  if (!ts->nodes) {
    if (cudaMallocAsync(reinterpret_cast<void**>(&ts->nodes), need, c->stream) != cudaSuccess) {
      delete ts;
      return fail(VC_ENOMEM, "tree node storage of %zu bytes failed", need);
    }
    ts->bytes = need;
  }
  for (const TreeMeta& m : p.meta) {
    for (int l = 0; l < n_layers; ++l) {
      ts->node_base.push_back(m.node_base + int64_t(l) * m.node_stride);
      ts->n_leaves.push_back(m.n_leaves);
      ts->log2_pad.push_back(m.log2_pad);
    }
  }
  *out = ts;
  return VC_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

int32_t vc_abi_version(void) { return VC_ABI_VERSION; }

size_t vc_last_error(char* buf, size_t buf_len) {
  const size_t n = g_last_error.size();
  if (buf && buf_len) {
    const size_t k = std::min(n, buf_len - 1);
    std::memcpy(buf, g_last_error.data(), k);
    buf[k] = 0;
  }
  return n;
}

vc_status vc_ctx_create(int32_t device, void* stream, vc_ctx** out) {
  if (!out) return fail(VC_EINVAL, "vc_ctx_create: out is NULL");
  int n_dev = 0;
  VC_CUDA(cudaGetDeviceCount(&n_dev));
  if (device < 0 || device >= n_dev) return fail(VC_EINVAL, "vc_ctx_create: device %d of %d", device, n_dev);
  DeviceGuard g(device);
  VC_CUDA(cudaSetDevice(device));
  auto* c = new (std::nothrow) vc_ctx();
  if (!c) return fail(VC_ENOMEM, "context allocation failed");
  c->device = device;
  c->stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaDeviceGetAttribute(&c->n_sm, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaMalloc(&c->zero_roots, sizeof(uint32_t) * 8 * (kMaxTreeHeight + 1));
  if (e == cudaSuccess) e = cudaMalloc(&c->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemsetAsync(c->err, 0, sizeof(int), c->stream);
  for (int i = 0; i < kStageSlots && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->stage[i].done, cudaEventDisableTiming);
  if (e == cudaSuccess) {
    c->pool = std::make_shared<NodePool>();
    if (!c->pool) e = cudaErrorMemoryAllocation;
  }
  if (e == cudaSuccess) e = launch_zero_roots(c->zero_roots, c->stream);
  if (e == cudaSuccess) {
    // Tree sets come from the stream-ordered pool: keep freed blocks cached.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t thr = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
  }
  if (e != cudaSuccess) {
    vc_ctx_destroy(c);
    return fail(VC_ECUDA, "vc_ctx_create: %s", cudaGetErrorString(e));
  }
  *out = c;
  return VC_OK;
}

vc_status vc_ctx_destroy(vc_ctx* c) {
  if (!c) return VC_OK;
  DeviceGuard g(c->device);
  cudaStreamSynchronize(c->stream);
  if (c->zero_roots) cudaFree(c->zero_roots);
  if (c->err) cudaFree(c->err);
  if (c->scratch) cudaFree(c->scratch);
  if (c->dargs) cudaFree(c->dargs);
  for (StageSlot& sl : c->stage) {
    if (sl.p) cudaFreeHost(sl.p);
    if (sl.done) cudaEventDestroy(sl.done);
  }
  if (c->pool) {
    // Cached blocks go back now; tree sets still alive free their own later.
    std::lock_guard<std::mutex> lk(c->pool->mu);
    c->pool->closed = true;
    for (auto& kv : c->pool->free_blocks) cudaFree(kv.second);
    c->pool->free_blocks.clear();
    c->pool->cached = 0;
  }
  if (c->rope) cudaFree(c->rope);
  delete c;
  return VC_OK;
}

vc_status vc_ctx_sync(vc_ctx* c, int32_t timeout_ms) {
  if (!c) return fail(VC_EINVAL, "vc_ctx_sync: ctx is NULL");
  DeviceGuard g(c->device);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(c->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return fail(VC_ECUDA, "vc_ctx_sync: %s", cudaGetErrorString(e));
    if (timeout_ms > 0) {
      const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
      if (ms >= timeout_ms) return fail(VC_ETIMEDOUT, "vc_ctx_sync: stream still busy after %d ms", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int flag = 0;
  VC_CUDA(cudaMemcpy(&flag, c->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) {
    VC_CUDA(cudaMemset(c->err, 0, sizeof(int)));
    if (flag == 2) return fail(VC_ETIMEDOUT, "a bounded wait inside a kernel ran out (results of that launch are void)");
    return fail(VC_ERANGE, "a K/V row addressed through the block table lies outside cache_elems");
  }
  return VC_OK;
}

// --------------------------------------------------------------- KV commit

vc_status vc_kv_commit(vc_ctx* c, const vc_kv_desc* d, uint8_t* kv_roots_dev, vc_tree_set** trees_out) {
  if (!c || !d || !kv_roots_dev) return fail(VC_EINVAL, "vc_kv_commit: NULL argument");
  if (d->n_layers < 1 || d->n_seqs < 1 || d->n_kv_heads < 1 || d->head_dim < 1)
    return fail(VC_EINVAL, "vc_kv_commit: n_layers, n_seqs, n_kv_heads, head_dim must be >= 1");
  if (d->dtype < VC_DTYPE_BF16 || d->dtype > VC_DTYPE_F64) return fail(VC_EINVAL, "vc_kv_commit: bad dtype %d", d->dtype);
  if (!d->seq_lens || !d->k_layers || !d->v_layers) return fail(VC_EINVAL, "vc_kv_commit: NULL table");
  if (d->cache_elems <= 0) return fail(VC_EINVAL, "vc_kv_commit: cache_elems must be > 0");
  if (d->stride_row < 0 || d->stride_head < 0 || d->stride_page < 0) return fail(VC_EINVAL, "vc_kv_commit: negative stride");
  const int64_t kv = int64_t(d->n_kv_heads) * d->head_dim;
  if (16 + 16 * kv > 0xFFFFFFFFll / 8) return fail(VC_EINVAL, "vc_kv_commit: kv_dim %lld too large", (long long)kv);
  const int esz = d->dtype == VC_DTYPE_BF16 ? 2 : (d->dtype == VC_DTYPE_F32 ? 4 : 8);
  const bool paged = d->block_tables != nullptr;
  if (paged && (d->block_size < 1 || d->max_blocks_per_seq < 1))
    return fail(VC_EINVAL, "vc_kv_commit: paged layout needs block_size and max_blocks_per_seq >= 1");
  const int64_t row_span = int64_t(d->n_kv_heads - 1) * d->stride_head + d->head_dim;
  if (d->tree_log2 < 0 || d->tree_log2 > kMaxTreeHeight)
    return fail(VC_EINVAL, "vc_kv_commit: tree_log2 %d out of range", d->tree_log2);
  int64_t acc = 0;
  for (int s = 0; s < d->n_seqs; ++s) {
    const int64_t n = d->seq_lens[s];
    const int64_t pb = d->pos_base ? d->pos_base[s] : 0;
    if (d->tree_log2 > 0) {
      if (n < 0 || n > (int64_t(1) << d->tree_log2))
        return fail(VC_EINVAL, "vc_kv_commit: seq_lens[%d] = %lld does not fit a subtree of 2^%d leaves", s,
                    (long long)n, d->tree_log2);
      if (n == 0) continue;
    } else if (n < 1) {
      return fail(VC_EINVAL, "vc_kv_commit: seq_lens[%d] = %lld (need at least one leaf)", s, (long long)n);
    }
    if (pb < 0 || pb + n > (int64_t(1) << 32))
      return fail(VC_EINVAL, "vc_kv_commit: positions of seq %d do not fit the u32 position field", s);
    if (paged) {
      if ((n + d->block_size - 1) / d->block_size > d->max_blocks_per_seq)
        return fail(VC_EINVAL, "vc_kv_commit: seq %d needs more than max_blocks_per_seq pages", s);
    } else {
      const int64_t r0 = d->seq_row_offset ? d->seq_row_offset[s] : acc;
      if (r0 < 0 || (r0 + n - 1) * d->stride_row + row_span > d->cache_elems)
        return fail(VC_EINVAL, "vc_kv_commit: rows of seq %d exceed cache_elems", s);
    }
    acc += n;
  }
  for (int l = 0; l < d->n_layers; ++l)
    if (!d->k_layers[l] || !d->v_layers[l]) return fail(VC_EINVAL, "vc_kv_commit: NULL K/V pointer of layer %d", l);

  // Fast path: 16-byte vector loads of 8-element chunks within a head.
  bool fast = kv % 8 == 0 && d->head_dim % 8 == 0;
  const int64_t vec = 16;
  for (int l = 0; l < d->n_layers && fast; ++l) {
    fast = (reinterpret_cast<uintptr_t>(d->k_layers[l]) % vec == 0) &&
           (reinterpret_cast<uintptr_t>(d->v_layers[l]) % vec == 0);
  }
  fast = fast && (d->stride_row * esz) % vec == 0 && (d->stride_head * esz) % vec == 0 &&
         (!paged || (d->stride_page * esz) % vec == 0);
  if (!fast) {
    for (int l = 0; l < d->n_layers; ++l)
      if (reinterpret_cast<uintptr_t>(d->k_layers[l]) % esz || reinterpret_cast<uintptr_t>(d->v_layers[l]) % esz)
        return fail(VC_EINVAL, "vc_kv_commit: K/V base of layer %d not aligned to its element size", l);
  }

  DeviceGuard g(c->device);
  Plan p;
  std::vector<int32_t> empty;   // groups of subtrees without a real leaf
  acc = 0;
  for (int s = 0; s < d->n_seqs; ++s) {
    const int64_t r0 = d->seq_row_offset ? d->seq_row_offset[s] : acc;
    if (d->tree_log2 > 0 && d->seq_lens[s] == 0) empty.push_back(int32_t(p.meta.size()));
    plan_group(p, d->seq_lens[s], d->n_layers, r0, s, d->pos_base ? d->pos_base[s] : 0, d->tree_log2);
    acc += d->seq_lens[s];
  }
  if (p.items.size() > 0x7FFFFFFFull) return fail(VC_EINVAL, "vc_kv_commit: too many chunks");

  Stager st;
  const size_t o_meta = st.add(p.meta.data(), p.meta.size() * sizeof(TreeMeta));
  const size_t o_items = st.add(p.items.data(), p.items.size() * sizeof(int2));
  const size_t o_empty = st.add(empty.data(), empty.size() * sizeof(int32_t));
  const size_t o_k = st.add(d->k_layers, sizeof(void*) * d->n_layers);
  const size_t o_v = st.add(d->v_layers, sizeof(void*) * d->n_layers);
  vc_tree_set* ts = nullptr;
  if (trees_out) {
    vc_status r = make_tree_set(c, p, d->n_layers, &ts);
    if (r) return r;
  }
  const size_t counters_bytes = align_up(sizeof(uint32_t) * p.n_trees, 256);
  const size_t croot_bytes = ts ? 0 : size_t(p.croots) * 32;
  vc_status r = ensure_scratch(c, counters_bytes + croot_bytes);
  if (!r) {
    char* dev = nullptr;
    r = upload(c, st, &dev);
    if (!r) {
      KvArgs a{};
      a.meta = reinterpret_cast<const TreeMeta*>(dev + o_meta);
      a.items = reinterpret_cast<const int2*>(dev + o_items);
      a.k_layers = reinterpret_cast<const void* const*>(dev + o_k);
      a.v_layers = reinterpret_cast<const void* const*>(dev + o_v);
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
      a.err = c->err;
      a.out.nodes = ts ? ts->nodes : nullptr;
      a.out.counters = reinterpret_cast<uint32_t*>(c->scratch);
      a.out.croots = c->scratch + counters_bytes;
      a.out.roots = kv_roots_dev;
      a.out.zero_roots = c->zero_roots;
      cudaError_t e = cudaMemsetAsync(c->scratch, 0, counters_bytes, c->stream);
      if (e == cudaSuccess && !p.items.empty())
        e = launch_kv_commit(a, int(p.items.size()), d->n_layers, d->dtype, fast, c->stream);
      if (e == cudaSuccess)
        e = launch_empty_trees(a.meta, reinterpret_cast<const int32_t*>(dev + o_empty), int(empty.size()),
                               d->n_layers, a.out, c->stream);
      if (e != cudaSuccess) r = fail(VC_ECUDA, "vc_kv_commit launch: %s", cudaGetErrorString(e));
    }
  }
  if (r) {
    if (ts) vc_tree_set_free(ts);
    return r;
  }
  if (trees_out) *trees_out = ts;
  return VC_OK;
}

// ------------------------------------------------------------ Merkle trees

vc_status vc_build_trees(vc_ctx* c, int32_t n_trees, const int64_t* leaf_off, const uint8_t* leaves_dev,
                         uint8_t* roots_dev, vc_tree_set** trees_out) {
  if (!c || !leaf_off || !leaves_dev || !roots_dev) return fail(VC_EINVAL, "vc_build_trees: NULL argument");
  if (n_trees < 1) return fail(VC_EINVAL, "vc_build_trees: n_trees must be >= 1");
  if (reinterpret_cast<uintptr_t>(leaves_dev) % 16) return fail(VC_EINVAL, "vc_build_trees: leaves_dev not 16-byte aligned");
  for (int i = 0; i < n_trees; ++i)
    if (leaf_off[i + 1] - leaf_off[i] < 1 || leaf_off[i] < 0)
      return fail(VC_EINVAL, "vc_build_trees: tree %d has no leaves (build_tree needs at least one)", i);
  DeviceGuard g(c->device);
  Plan p;
  for (int i = 0; i < n_trees; ++i) plan_group(p, leaf_off[i + 1] - leaf_off[i], 1, leaf_off[i], i);
  Stager st;
  const size_t o_meta = st.add(p.meta.data(), p.meta.size() * sizeof(TreeMeta));
  const size_t o_items = st.add(p.items.data(), p.items.size() * sizeof(int2));
  vc_tree_set* ts = nullptr;
  if (trees_out) {
    vc_status r = make_tree_set(c, p, 1, &ts);
    if (r) return r;
  }
  const size_t counters_bytes = align_up(sizeof(uint32_t) * p.n_trees, 256);
  const size_t croot_bytes = ts ? 0 : size_t(p.croots) * 32;
  vc_status r = ensure_scratch(c, counters_bytes + croot_bytes);
  if (!r) {
    char* dev = nullptr;
    r = upload(c, st, &dev);
    if (!r) {
      TreeArgs a{};
      a.meta = reinterpret_cast<const TreeMeta*>(dev + o_meta);
      a.items = reinterpret_cast<const int2*>(dev + o_items);
      a.leaves = leaves_dev;
      a.out.nodes = ts ? ts->nodes : nullptr;
      a.out.counters = reinterpret_cast<uint32_t*>(c->scratch);
      a.out.croots = c->scratch + counters_bytes;
      a.out.roots = roots_dev;
      a.out.zero_roots = c->zero_roots;
      cudaError_t e = cudaMemsetAsync(c->scratch, 0, counters_bytes, c->stream);
      if (e == cudaSuccess) e = launch_tree_commit(a, int(p.items.size()), c->stream);
      if (e != cudaSuccess) r = fail(VC_ECUDA, "vc_build_trees launch: %s", cudaGetErrorString(e));
    }
  }
  if (r) {
    if (ts) vc_tree_set_free(ts);
    return r;
  }
  if (trees_out) *trees_out = ts;
  return VC_OK;
}

vc_status vc_prove(vc_ctx* c, const vc_tree_set* ts, int32_t n, const int32_t* tree, const uint32_t* leaf,
                   uint8_t* siblings_dev, int32_t max_depth, int32_t* depth_out) {
  if (!c || !ts || (n > 0 && (!tree || !leaf || !siblings_dev || !depth_out)))
    return fail(VC_EINVAL, "vc_prove: NULL argument");
  if (n < 0 || max_depth < 0) return fail(VC_EINVAL, "vc_prove: negative count");
  std::vector<ProveReq> reqs(n);
  for (int i = 0; i < n; ++i) {
    const int t = tree[i];
    if (t < 0 || t >= int(ts->node_base.size())) return fail(VC_ERANGE, "vc_prove: tree %d of %zu", t, ts->node_base.size());
    if (int64_t(leaf[i]) >= ts->n_leaves[t])
      return fail(VC_ERANGE, "vc_prove: leaf index %u out of range (n_leaves=%lld)", leaf[i], (long long)ts->n_leaves[t]);
    if (ts->log2_pad[t] > max_depth)
      return fail(VC_EINVAL, "vc_prove: max_depth %d < proof length %d", max_depth, ts->log2_pad[t]);
    reqs[i].node_base = ts->node_base[t];
    reqs[i].leaf = leaf[i];
    reqs[i].log2_pad = ts->log2_pad[t];
    depth_out[i] = ts->log2_pad[t];
  }
  if (n == 0) return VC_OK;
  DeviceGuard g(c->device);
  Stager st;
  const size_t o = st.add(reqs.data(), reqs.size() * sizeof(ProveReq));
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  const cudaError_t e = launch_prove(ts->nodes, reinterpret_cast<const ProveReq*>(dev + o), n, max_depth,
                                     siblings_dev, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_prove launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_kv_open(vc_ctx* c, const vc_kv_desc* d, const vc_tree_set* ts, int32_t seq, int32_t n_sel,
                     const int32_t* layers, int32_t n_positions, double* entries_dev, uint8_t* siblings_dev,
                     int32_t max_depth, int32_t* depth_out) {
  if (!c || !d || !ts || !layers || (n_sel > 0 && n_positions > 0 && (!entries_dev || !siblings_dev)))
    return fail(VC_EINVAL, "vc_kv_open: NULL argument");
  if (n_sel < 0 || n_positions < 0) return fail(VC_EINVAL, "vc_kv_open: negative count");
  if (seq < 0 || seq >= d->n_seqs) return fail(VC_ERANGE, "vc_kv_open: seq %d of %d", seq, d->n_seqs);
  if (int64_t(d->n_seqs) * d->n_layers != int64_t(ts->node_base.size()))
    return fail(VC_EINVAL, "vc_kv_open: tree set does not match the descriptor (%zu trees, %d x %d)",
                ts->node_base.size(), d->n_seqs, d->n_layers);
  if (n_positions > d->seq_lens[seq])
    return fail(VC_ERANGE, "vc_kv_open: %d positions of a %d-token sequence", n_positions, d->seq_lens[seq]);
  if (!d->k_layers || !d->v_layers || d->cache_elems <= 0) return fail(VC_EINVAL, "vc_kv_open: bad descriptor");
  for (int i = 0; i < n_sel; ++i)
    if (layers[i] < 0 || layers[i] >= d->n_layers) return fail(VC_ERANGE, "vc_kv_open: layer %d of %d", layers[i], d->n_layers);
  if (n_sel == 0 || n_positions == 0) return VC_OK;
  const int64_t n = int64_t(n_sel) * n_positions;
  if (n > 0x7FFFFFFF) return fail(VC_EINVAL, "vc_kv_open: too many openings");
  // proofs: the batched merkle::prove of every (layer, position)
  std::vector<int32_t> tree(n);
  std::vector<uint32_t> leaf(n);
  for (int i = 0; i < n_sel; ++i)
    for (int p = 0; p < n_positions; ++p) {
      tree[int64_t(i) * n_positions + p] = seq * d->n_layers + layers[i];
      leaf[int64_t(i) * n_positions + p] = uint32_t(p);
    }
  std::vector<int32_t> depth(n);
  vc_status r = vc_prove(c, ts, int32_t(n), tree.data(), leaf.data(), siblings_dev, max_depth, depth.data());
  if (r) return r;
  if (depth_out) *depth_out = depth[0];
  // entries: the rows widened to f64
  int64_t r0 = 0;
  if (!d->block_tables) {
    if (d->seq_row_offset) {
      r0 = d->seq_row_offset[seq];
    } else {
      for (int s = 0; s < seq; ++s) r0 += d->seq_lens[s];
    }
  }
  DeviceGuard g(c->device);
  Stager st;
  const size_t o_k = st.add(d->k_layers, sizeof(void*) * d->n_layers);
  const size_t o_v = st.add(d->v_layers, sizeof(void*) * d->n_layers);
  const size_t o_l = st.add(layers, sizeof(int32_t) * n_sel);
  char* dev = nullptr;
  r = upload(c, st, &dev);
  if (r) return r;
  KvOpenArgs a{};
  a.kv.k_layers = reinterpret_cast<const void* const*>(dev + o_k);
  a.kv.v_layers = reinterpret_cast<const void* const*>(dev + o_v);
  a.kv.block_tables = d->block_tables;
  a.kv.stride_page = d->stride_page;
  a.kv.stride_row = d->stride_row;
  a.kv.stride_head = d->stride_head;
  a.kv.block_size = d->block_tables ? d->block_size : 1;
  a.kv.max_blocks = d->max_blocks_per_seq;
  a.kv.n_heads = d->n_kv_heads;
  a.kv.head_dim = d->head_dim;
  a.kv.paged = d->block_tables ? 1 : 0;
  a.kv.cache_elems = d->cache_elems;
  a.kv.row_span = int64_t(d->n_kv_heads - 1) * d->stride_head + d->head_dim;
  a.kv.err = c->err;
  a.seq.seq = seq;
  a.seq.src_off = r0;
  a.layers = reinterpret_cast<const int32_t*>(dev + o_l);
  a.n_sel = n_sel;
  a.n_pos = n_positions;
  a.kv_dim = d->n_kv_heads * d->head_dim;
  a.out = entries_dev;
  const cudaError_t e = launch_kv_entries(a, d->dtype, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_kv_open launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

int32_t vc_tree_set_count(const vc_tree_set* ts) { return ts ? int32_t(ts->node_base.size()) : 0; }

vc_status vc_tree_nodes(const vc_tree_set* ts, int32_t tree, const uint8_t** nodes_dev, int64_t* n_leaves,
                        int64_t* padded_size) {
  if (!ts) return fail(VC_EINVAL, "vc_tree_nodes: NULL tree set");
  if (tree < 0 || tree >= int32_t(ts->node_base.size())) return fail(VC_ERANGE, "vc_tree_nodes: tree %d", tree);
  if (nodes_dev) *nodes_dev = ts->nodes + ts->node_base[tree] * 32;
  if (n_leaves) *n_leaves = ts->n_leaves[tree];
  if (padded_size) *padded_size = int64_t(1) << ts->log2_pad[tree];
  return VC_OK;
}

vc_status vc_tree_set_free(vc_tree_set* ts) {
  if (!ts) return VC_OK;
  DeviceGuard g(ts->device);
  if (ts->nodes) {
    bool kept = false;
    if (ts->pool) {
      std::lock_guard<std::mutex> lk(ts->pool->mu);
      if (!ts->pool->closed && ts->pool->cached + ts->bytes <= NodePool::kMaxCached) {
        ts->pool->free_blocks.emplace(ts->bytes, ts->nodes);
        ts->pool->cached += ts->bytes;
        kept = true;
      }
    }
    if (!kept) cudaFreeAsync(ts->nodes, ts->stream);
  }
  delete ts;
  return VC_OK;
}

// ---------------------------------------------------------- trace leaves

vc_status vc_trace_leaves(vc_ctx* c, const vc_trace_desc* d, uint8_t* leaves_dev) {
  if (!c || !d || !leaves_dev) return fail(VC_EINVAL, "vc_trace_leaves: NULL argument");
  if (d->n_tokens < 0 || d->n_layers < 0 || d->hidden < 0 || d->n_fwd < 0)
    return fail(VC_EINVAL, "vc_trace_leaves: negative size");
  if (d->n_tokens == 0) return VC_OK;
  if (!d->tok_fwd || !d->tok_row || !d->fwd_rows) return fail(VC_EINVAL, "vc_trace_leaves: NULL token table");
  if (d->n_layers > 0 && (!d->a_rows || !d->scale_a)) return fail(VC_EINVAL, "vc_trace_leaves: NULL a_rows/scale_a");
  if ((d->x_attn_rows == nullptr) != (d->scale_x_attn == nullptr))
    return fail(VC_EINVAL, "vc_trace_leaves: x_attn_rows and scale_x_attn must be given together");
  const size_t nfl = size_t(d->n_fwd) * d->n_layers;
  for (size_t i = 0; i < nfl; ++i) {
    if (!d->a_rows[i] || !d->scale_a[i]) return fail(VC_EINVAL, "vc_trace_leaves: NULL a_rows/scale_a entry %zu", i);
    if (reinterpret_cast<uintptr_t>(d->scale_a[i]) % 4) return fail(VC_EINVAL, "vc_trace_leaves: scale_a entry %zu not f32-aligned", i);
    if (d->x_attn_rows && (!d->x_attn_rows[i] || !d->scale_x_attn[i]))
      return fail(VC_EINVAL, "vc_trace_leaves: NULL x_attn entry %zu", i);
    if (d->x_attn_rows && reinterpret_cast<uintptr_t>(d->scale_x_attn[i]) % 4)
      return fail(VC_EINVAL, "vc_trace_leaves: scale_x_attn entry %zu not f32-aligned", i);
  }
  struct Wrap { const void* p; int32_t dim, rows; int64_t stride; const int32_t* tok; int esz; const char* name; };
  const Wrap wraps[3] = {{d->final_residual, d->fr_dim, d->fr_rows, d->fr_stride, d->tok_fr_row, 4, "final_residual"},
                         {d->lp_hidden, d->lp_dim, d->lp_rows, d->lp_stride, d->tok_lp_row, 2, "lp_hidden"},
                         {d->logits, d->vocab, d->logits_rows, d->logits_stride, d->tok_logits_row, 4, "logits"}};
  for (const Wrap& w : wraps) {
    if (!w.tok) continue;
    if (!w.p || w.dim < 0 || w.rows < 0 || w.stride < w.dim)
      return fail(VC_EINVAL, "vc_trace_leaves: bad %s buffer", w.name);
    if (reinterpret_cast<uintptr_t>(w.p) % w.esz) return fail(VC_EINVAL, "vc_trace_leaves: %s not aligned", w.name);
  }
  std::vector<int32_t> tok(size_t(d->n_tokens) * 5);
  for (int t = 0; t < d->n_tokens; ++t) {
    const int f = d->tok_fwd[t], row = d->tok_row[t];
    if (f < 0 || f >= d->n_fwd) return fail(VC_EINVAL, "vc_trace_leaves: tok_fwd[%d] = %d of %d", t, f, d->n_fwd);
    if (row < 0 || row >= d->fwd_rows[f]) return fail(VC_EINVAL, "vc_trace_leaves: tok_row[%d] = %d of %d", t, row, d->fwd_rows[f]);
    tok[size_t(t) * 5 + 0] = f;
    tok[size_t(t) * 5 + 1] = row;
    for (int k = 0; k < 3; ++k) {
      int32_t r = -1;
      if (wraps[k].tok) {
        r = wraps[k].tok[t];
        if (r >= wraps[k].rows) return fail(VC_EINVAL, "vc_trace_leaves: %s row %d of %d for token %d", wraps[k].name, r, wraps[k].rows, t);
        if (r < -1) return fail(VC_EINVAL, "vc_trace_leaves: %s row %d for token %d", wraps[k].name, r, t);
      }
      tok[size_t(t) * 5 + 2 + k] = r;
    }
  }
  DeviceGuard g(c->device);
  Stager st;
  const size_t o_tok = st.add(tok.data(), tok.size() * sizeof(int32_t));
  const size_t o_a = st.add(d->a_rows, nfl * sizeof(void*));
  const size_t o_s = st.add(d->scale_a, nfl * sizeof(void*));
  const size_t o_x = d->x_attn_rows ? st.add(d->x_attn_rows, nfl * sizeof(void*)) : 0;
  const size_t o_sx = d->x_attn_rows ? st.add(d->scale_x_attn, nfl * sizeof(void*)) : 0;
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  TraceArgs a{};
  a.opq = make_opq();
  a.n_tokens = d->n_tokens;
  a.n_layers = d->n_layers;
  a.hidden = d->hidden;
  a.tok = reinterpret_cast<const int32_t*>(dev + o_tok);
  a.a_rows = reinterpret_cast<const void* const*>(dev + o_a);
  a.scale_a = reinterpret_cast<const void* const*>(dev + o_s);
  a.scale_stride = d->scale_stride;
  a.x_rows = d->x_attn_rows ? reinterpret_cast<const void* const*>(dev + o_x) : nullptr;
  a.scale_x = d->x_attn_rows ? reinterpret_cast<const void* const*>(dev + o_sx) : nullptr;
  a.scale_x_stride = d->scale_x_stride;
  a.fr = static_cast<const uint8_t*>(d->final_residual);
  a.fr_dim = d->fr_dim;
  a.fr_stride = d->fr_stride;
  a.lp = static_cast<const uint8_t*>(d->lp_hidden);
  a.lp_dim = d->lp_dim;
  a.lp_stride = d->lp_stride;
  a.logits = static_cast<const uint8_t*>(d->logits);
  a.vocab = d->vocab;
  a.logits_stride = d->logits_stride;
  a.leaves = leaves_dev;
  a.err = c->err;
  if (reinterpret_cast<uintptr_t>(leaves_dev) % 16) return fail(VC_EINVAL, "vc_trace_leaves: leaves_dev not 16-byte aligned");
  const cudaError_t e = launch_trace_leaves(a, c->n_sm, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_trace_leaves launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

// ---------------------------------------------------------------- IO chain

vc_status vc_io_chain(vc_ctx* c, int32_t n_seqs, const int64_t* tok_off, const uint8_t* leaves_dev,
                      const uint32_t* token_ids_dev, const uint8_t* prompt_hash_dev, uint8_t* io_dev) {
  if (!c || !tok_off || !leaves_dev || !token_ids_dev || !prompt_hash_dev || !io_dev)
    return fail(VC_EINVAL, "vc_io_chain: NULL argument");
  if (n_seqs < 1) return fail(VC_EINVAL, "vc_io_chain: n_seqs must be >= 1");
  for (int s = 0; s < n_seqs; ++s)
    if (tok_off[s] < 0 || tok_off[s + 1] < tok_off[s]) return fail(VC_EINVAL, "vc_io_chain: tok_off not ascending at %d", s);
  for (const void* p : {(const void*)leaves_dev, (const void*)prompt_hash_dev, (const void*)io_dev})
    if (reinterpret_cast<uintptr_t>(p) % 16) return fail(VC_EINVAL, "vc_io_chain: digest arrays must be 16-byte aligned");
  DeviceGuard g(c->device);
  Stager st;
  const size_t o = st.add(tok_off, sizeof(int64_t) * (n_seqs + 1));
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  const cudaError_t e = launch_io_chain(n_seqs, reinterpret_cast<const int64_t*>(dev + o), leaves_dev, token_ids_dev,
                                        prompt_hash_dev, io_dev, nullptr, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_io_chain launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_io_extend(vc_ctx* c, int32_t n_seqs, const int64_t* tok_off, const uint8_t* leaves_dev,
                       const uint32_t* token_ids_dev, uint8_t* prev_io_dev, uint8_t* io_dev) {
  if (!c || !tok_off || !prev_io_dev || (tok_off[n_seqs] > tok_off[0] && (!leaves_dev || !token_ids_dev || !io_dev)))
    return fail(VC_EINVAL, "vc_io_extend: NULL argument");
  if (n_seqs < 1) return fail(VC_EINVAL, "vc_io_extend: n_seqs must be >= 1");
  for (int s = 0; s < n_seqs; ++s)
    if (tok_off[s] < 0 || tok_off[s + 1] < tok_off[s]) return fail(VC_EINVAL, "vc_io_extend: tok_off not ascending at %d", s);
  for (const void* p : {(const void*)leaves_dev, (const void*)prev_io_dev, (const void*)io_dev})
    if (p && reinterpret_cast<uintptr_t>(p) % 16) return fail(VC_EINVAL, "vc_io_extend: digest arrays must be 16-byte aligned");
  DeviceGuard g(c->device);
  Stager st;
  const size_t o = st.add(tok_off, sizeof(int64_t) * (n_seqs + 1));
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  const cudaError_t e = launch_io_chain(n_seqs, reinterpret_cast<const int64_t*>(dev + o), leaves_dev, token_ids_dev,
                                        nullptr, io_dev, prev_io_dev, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_io_extend launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_io_genesis(vc_ctx* c, int32_t n, const uint8_t* prompt_hash_dev, uint8_t* out_dev) {
  if (!c || (n > 0 && (!prompt_hash_dev || !out_dev))) return fail(VC_EINVAL, "vc_io_genesis: NULL argument");
  if (n < 0) return fail(VC_EINVAL, "vc_io_genesis: negative count");
  if (n > 0 && reinterpret_cast<uintptr_t>(out_dev) % 16) return fail(VC_EINVAL, "vc_io_genesis: out_dev not 16-byte aligned");
  if (n == 0) return VC_OK;
  DeviceGuard g(c->device);
  const cudaError_t e = launch_tagged_hash(n, 2, prompt_hash_dev, nullptr, 32, out_dev, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_io_genesis launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_prompt_hash(vc_ctx* c, int32_t n, const uint8_t* prompts_dev, const int64_t* off, uint8_t* out_dev) {
  if (!c || !off || !out_dev || (!prompts_dev && n > 0 && off[n] > off[0])) return fail(VC_EINVAL, "vc_prompt_hash: NULL argument");
  if (n < 0) return fail(VC_EINVAL, "vc_prompt_hash: negative count");
  if (reinterpret_cast<uintptr_t>(out_dev) % 16) return fail(VC_EINVAL, "vc_prompt_hash: out_dev not 16-byte aligned");
  for (int i = 0; i < n; ++i)
    if (off[i] < 0 || off[i + 1] < off[i]) return fail(VC_EINVAL, "vc_prompt_hash: offsets not ascending at %d", i);
  if (n == 0) return VC_OK;
  DeviceGuard g(c->device);
  Stager st;
  const size_t o = st.add(off, sizeof(int64_t) * (n + 1));
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  const cudaError_t e = launch_tagged_hash(n, 0, prompts_dev, reinterpret_cast<const int64_t*>(dev + o), 0, out_dev, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_prompt_hash launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_seed_commitment(vc_ctx* c, int32_t n, const uint8_t* seeds_dev, uint8_t* out_dev) {
  if (!c || (n > 0 && (!seeds_dev || !out_dev))) return fail(VC_EINVAL, "vc_seed_commitment: NULL argument");
  if (n < 0) return fail(VC_EINVAL, "vc_seed_commitment: negative count");
  if (reinterpret_cast<uintptr_t>(out_dev) % 16) return fail(VC_EINVAL, "vc_seed_commitment: out_dev not 16-byte aligned");
  if (n == 0) return VC_OK;
  DeviceGuard g(c->device);
  const cudaError_t e = launch_tagged_hash(n, 1, seeds_dev, nullptr, 32, out_dev, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_seed_commitment launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

// ------------------------------------------------------- measurement aid

// ------------------------------------------------------------ KV transcript

}  // extern "C"

namespace {

// Argument checks of the transcript entry points (n_tokens >= 0).
vc_status check_kvt(const vc_kvt_desc* d, const char* fn) {
  if (d->n_tokens < 0 || d->n_layers < 1 || d->n_kv_heads < 1)
    return fail(VC_EINVAL, "%s: n_tokens >= 0, n_layers and n_kv_heads >= 1 required", fn);
  if (d->hidden < 16 || d->hidden % 16) return fail(VC_EINVAL, "%s: hidden %d must be a positive multiple of 16", fn, d->hidden);
  if (d->head_dim < 2 || d->head_dim % 2 || d->head_dim > 256)
    return fail(VC_EINVAL, "%s: head_dim %d must be even and <= 256", fn, d->head_dim);
  const int64_t kv = int64_t(d->n_kv_heads) * d->head_dim;
  if (kv > (int64_t(1) << 24)) return fail(VC_EINVAL, "%s: kv_dim too large", fn);
  if (d->n_tokens == 0) return VC_OK;
  if (d->x_row_stride < d->hidden || d->x_row_stride % 16)
    return fail(VC_EINVAL, "%s: x_row_stride must be >= hidden and a multiple of 16", fn);
  if (!d->x_layers || !d->wk_layers || !d->wv_layers) return fail(VC_EINVAL, "%s: NULL layer table", fn);
  if (d->use_rope && !d->scale_x) return fail(VC_EINVAL, "%s: scale_x is NULL", fn);
  for (int l = 0; l < d->n_layers; ++l) {
    const void* p[3] = {d->x_layers[l], d->wk_layers[l], d->wv_layers[l]};
    for (const void* q : p)
      if (!q || reinterpret_cast<uintptr_t>(q) % 16)
        return fail(VC_EINVAL, "%s: x/Wk/Wv pointer of layer %d is NULL or not 16-byte aligned", fn, l);
  }
  return VC_OK;
}

// The context's (cos, sin) table for these frequencies and >= n_tokens
// positions (host C library cos/sin), then the per-layer tensor maps (x_attn
// boxes of 128 rows, weight boxes of w_box_rows rows) and scale/bias tables,
// staged to the device; fills every field of *a except out[] and err.
vc_status prepare_kvt(vc_ctx* c, const vc_kvt_desc* d, int w_box_rows, KvtArgs* a, const char* fn) {
  const int64_t kv = int64_t(d->n_kv_heads) * d->head_dim;
  if (d->use_rope) {
    const std::vector<double> inv =
        kvt_inv_freq(d->head_dim, d->rope_theta, d->rope_scaling, d->rope_factor, d->rope_low_freq_factor,
                     d->rope_high_freq_factor, d->rope_original_max_position_embeddings);
    const bool same = inv.size() == c->rope_inv.size() &&
                      std::memcmp(inv.data(), c->rope_inv.data(), inv.size() * sizeof(double)) == 0;
    if (!same || c->rope_rows < d->n_tokens) {
      const int64_t rows = std::max<int64_t>(d->n_tokens, same ? 2 * c->rope_rows : 0);
      std::vector<double> tab(size_t(rows) * inv.size() * 2);
      kvt_rope_table(inv, rows, tab.data());
      VC_CUDA(cudaStreamSynchronize(c->stream));
      if (c->rope) cudaFree(c->rope);
      c->rope = nullptr;
      c->rope_rows = 0;
      c->rope_inv.clear();
      if (cudaMalloc(&c->rope, tab.size() * sizeof(double)) != cudaSuccess)
        return fail(VC_ENOMEM, "%s: RoPE table of %zu bytes", fn, tab.size() * sizeof(double));
      VC_CUDA(cudaMemcpy(c->rope, tab.data(), tab.size() * sizeof(double), cudaMemcpyHostToDevice));
      c->rope_rows = rows;
      c->rope_inv = inv;
    }
  }
  std::vector<CUtensorMap> maps(size_t(d->n_layers) * 3);
  std::vector<KvtLayer> layers(d->n_layers);
  for (int l = 0; l < d->n_layers; ++l) {
    int r = kvt_encode_map(&maps[3 * l], d->x_layers[l], d->hidden, d->n_tokens, d->x_row_stride, 128);
    if (!r) r = kvt_encode_map(&maps[3 * l + 1], d->wk_layers[l], d->hidden, kv, d->hidden, w_box_rows);
    if (!r) r = kvt_encode_map(&maps[3 * l + 2], d->wv_layers[l], d->hidden, kv, d->hidden, w_box_rows);
    if (r) return fail(VC_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d) for layer %d", fn, r, l);
    KvtLayer& L = layers[l];
    std::memset(&L, 0, sizeof(L));
    L.ch[0] = d->ch_k ? d->ch_k[l] : nullptr;
    L.ch[1] = d->ch_v ? d->ch_v[l] : nullptr;
    L.bias[0] = d->bias_k ? d->bias_k[l] : nullptr;
    L.bias[1] = d->bias_v ? d->bias_v[l] : nullptr;
    L.sw[0] = d->sw_k ? d->sw_k[l] : 0.0f;
    L.sw[1] = d->sw_v ? d->sw_v[l] : 0.0f;
  }
  Stager st;
  const size_t om = st.add(maps.data(), maps.size() * sizeof(CUtensorMap), 128);
  const size_t ol = st.add(layers.data(), layers.size() * sizeof(KvtLayer));
  char* dev = nullptr;
  vc_status r = upload(c, st, &dev);
  if (r) return r;
  std::memset(a, 0, sizeof(*a));
  a->maps = reinterpret_cast<const CUtensorMap*>(dev + om);
  a->layers = reinterpret_cast<const KvtLayer*>(dev + ol);
  a->scale_x = d->scale_x;
  a->sx_t = d->sx_tstride;
  a->sx_l = d->sx_lstride;
  a->rope = d->use_rope ? reinterpret_cast<const double2*>(c->rope) : nullptr;
  a->rope_rows = c->rope_rows;
  a->n_tokens = d->n_tokens;
  a->hidden = d->hidden;
  a->kv_dim = int32_t(kv);
  a->head_dim = d->head_dim;
  a->use_rope = d->use_rope != 0;
  a->err = c->err;
  a->m_tiles = (d->n_tokens + 127) / 128;
  return VC_OK;
}

}  // namespace

extern "C" {

vc_status vc_kv_transcript(vc_ctx* c, const vc_kvt_desc* d, double* k_out, double* v_out) {
  if (!c || !d) return fail(VC_EINVAL, "vc_kv_transcript: NULL argument");
  vc_status r = check_kvt(d, "vc_kv_transcript");
  if (r || d->n_tokens == 0) return r;
  if (!k_out || !v_out) return fail(VC_EINVAL, "vc_kv_transcript: NULL output");
  if (reinterpret_cast<uintptr_t>(k_out) % 32 || reinterpret_cast<uintptr_t>(v_out) % 32)
    return fail(VC_EINVAL, "vc_kv_transcript: outputs must be 32-byte aligned");
  DeviceGuard g(c->device);
  KvtArgs a;
  r = prepare_kvt(c, d, 256, &a, "vc_kv_transcript");
  if (r) return r;
  a.out[0] = k_out;
  a.out[1] = v_out;
  a.tile_cols = (256 / d->head_dim) * d->head_dim;
  a.tiles_per_mat = int32_t((int64_t(a.kv_dim) + a.tile_cols - 1) / a.tile_cols);
  const int64_t n_tiles = int64_t(d->n_layers) * a.m_tiles * 2 * a.tiles_per_mat;
  if (n_tiles > 0x7FFFFFFF) return fail(VC_EINVAL, "vc_kv_transcript: too many tiles");
  a.n_tiles = int32_t(n_tiles);
  const cudaError_t e = launch_kv_transcript(a, c->n_sm, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_kv_transcript launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

vc_status vc_kv_transcript_commit(vc_ctx* c, const vc_kvt_desc* d, int32_t layer_base, uint8_t* kv_roots_dev,
                                  vc_tree_set** trees_out) {
  if (!c || !d || !kv_roots_dev) return fail(VC_EINVAL, "vc_kv_transcript_commit: NULL argument");
  vc_status r = check_kvt(d, "vc_kv_transcript_commit");
  if (r) return r;
  if (d->n_tokens < 1) return fail(VC_EINVAL, "vc_kv_transcript_commit: need at least one position (build_tree)");
  if (layer_base < 0 || int64_t(layer_base) + d->n_layers > 0x7FFFFFFF)
    return fail(VC_EINVAL, "vc_kv_transcript_commit: layer_base %d out of range", layer_base);
  DeviceGuard g(c->device);
  const int64_t kv = int64_t(d->n_kv_heads) * d->head_dim;
  if (!kvt_commit_supported(d->head_dim, int(kv))) {
    // Other head sizes: the transcript's f64 rows through device scratch, then their trees.
    const size_t bytes = size_t(d->n_layers) * size_t(d->n_tokens) * size_t(kv) * sizeof(double);
    double* kbuf = nullptr;
    double* vbuf = nullptr;
    if (cudaMallocAsync(reinterpret_cast<void**>(&kbuf), bytes, c->stream) != cudaSuccess ||
        cudaMallocAsync(reinterpret_cast<void**>(&vbuf), bytes, c->stream) != cudaSuccess) {
      if (kbuf) cudaFreeAsync(kbuf, c->stream);
      return fail(VC_ENOMEM, "vc_kv_transcript_commit: f64 rows of %zu bytes", 2 * bytes);
    }
    r = vc_kv_transcript(c, d, kbuf, vbuf);
    if (!r) {
      std::vector<const void*> kl(d->n_layers), vl(d->n_layers);
      for (int l = 0; l < d->n_layers; ++l) {
        kl[l] = kbuf + size_t(l) * d->n_tokens * kv;
        vl[l] = vbuf + size_t(l) * d->n_tokens * kv;
      }
      const int32_t n = d->n_tokens;
      vc_kv_desc kd{};
      kd.n_layers = d->n_layers;
      kd.layer_base = layer_base;
      kd.n_kv_heads = 1;
      kd.head_dim = int32_t(kv);
      kd.dtype = VC_DTYPE_F64;
      kd.n_seqs = 1;
      kd.seq_lens = &n;
      kd.stride_row = kv;
      kd.stride_head = kv;
      kd.cache_elems = int64_t(n) * kv;
      kd.k_layers = kl.data();
      kd.v_layers = vl.data();
      r = vc_kv_commit(c, &kd, kv_roots_dev, trees_out);
    }
    cudaFreeAsync(kbuf, c->stream);
    cudaFreeAsync(vbuf, c->stream);
    return r;
  }
  KvtcArgs A;
  std::memset(&A, 0, sizeof(A));
  r = prepare_kvt(c, d, 128, &A.t, "vc_kv_transcript_commit");
  if (r) return r;
  const int64_t n_units = int64_t(d->n_layers) * A.t.m_tiles;
  if (n_units > 0x7FFFFFFF) return fail(VC_EINVAL, "vc_kv_transcript_commit: too many units");
  A.n_units = int32_t(n_units);
  A.layer_base = layer_base;
  Plan p;
  plan_group(p, d->n_tokens, d->n_layers, 0, 0);
  A.meta = p.meta[0];
  vc_tree_set* ts = nullptr;
  if (trees_out) {
    r = make_tree_set(c, p, d->n_layers, &ts);
    if (r) return r;
  }
  const size_t counters_bytes = align_up(sizeof(uint32_t) * p.n_trees, 256);
  const size_t croot_bytes = ts ? 0 : size_t(p.croots) * 32;
  r = ensure_scratch(c, counters_bytes + croot_bytes);
  if (!r) {
    A.out.nodes = ts ? ts->nodes : nullptr;
    A.out.counters = reinterpret_cast<uint32_t*>(c->scratch);
    A.out.croots = c->scratch + counters_bytes;
    A.out.roots = kv_roots_dev;
    A.out.zero_roots = c->zero_roots;
    cudaError_t e = cudaMemsetAsync(c->scratch, 0, counters_bytes, c->stream);
    if (e == cudaSuccess) e = launch_kvt_commit(A, c->n_sm, c->stream);
    if (e != cudaSuccess) r = fail(VC_ECUDA, "vc_kv_transcript_commit launch: %s", cudaGetErrorString(e));
  }
  if (r) {
    if (ts) vc_tree_set_free(ts);
    return r;
  }
  if (trees_out) *trees_out = ts;
  return VC_OK;
}

vc_status vc_int_peak(vc_ctx* c, int32_t variant, int64_t iters, double* ops_per_s) {
  if (!c || !ops_per_s || iters < 1 || variant < 0 || variant > 3) return fail(VC_EINVAL, "vc_int_peak: bad argument");
  DeviceGuard g(c->device);
  const size_t sink_bytes = size_t(c->n_sm) * 4 * 256 * sizeof(uint32_t);
  vc_status r = ensure_scratch(c, sink_bytes);
  if (r) return r;
  cudaEvent_t e0, e1;
  VC_CUDA(cudaEventCreate(&e0));
  VC_CUDA(cudaEventCreate(&e1));
  double ops = 0;
  cudaError_t e = launch_int_peak(variant, iters, c->n_sm, reinterpret_cast<uint32_t*>(c->scratch), c->stream, &ops);  // warm-up
  if (e == cudaSuccess) e = cudaEventRecord(e0, c->stream);
  if (e == cudaSuccess) e = launch_int_peak(variant, iters, c->n_sm, reinterpret_cast<uint32_t*>(c->scratch), c->stream, &ops);
  if (e == cudaSuccess) e = cudaEventRecord(e1, c->stream);
  if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  float ms = 0;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_int_peak: %s", cudaGetErrorString(e));
  *ops_per_s = ops / (double(ms) * 1e-3);
  return VC_OK;
}

vc_status vc_wait_probe(vc_ctx* c, int64_t limit_ns) {
  if (!c || limit_ns < 1 || limit_ns > 2000000000) return fail(VC_EINVAL, "vc_wait_probe: limit_ns must be in [1, 2e9]");
  DeviceGuard g(c->device);
  const cudaError_t e = launch_wait_probe(uint64_t(limit_ns), c->err, c->stream);
  if (e != cudaSuccess) return fail(VC_ECUDA, "vc_wait_probe launch: %s", cudaGetErrorString(e));
  return VC_OK;
}

}  // extern "C"
