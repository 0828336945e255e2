// Internal declarations shared by the CUDA translation units of libvcommit.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <vector>

#include "sha256_opq.h"

namespace vc {

constexpr int kTreeThreads = 128;  // leaves per CTA of the Merkle kernels (chunk cap)
constexpr int kLog2TreeThreads = 7;
constexpr int kMaxTreeHeight = 62; // zero-subtree table size - 1

// One leaf group: a tree (generic) or all n_layers trees of one sequence (KV).
struct TreeMeta {
  int64_t n_leaves;
  int64_t node_base;     // index (in 32-byte nodes) of layer 0's tree
  int64_t node_stride;   // nodes between consecutive layers' trees
  int64_t croot_base;    // roots-only mode: chunk-root slot of layer 0
  int64_t croot_stride;  // roots-only mode: slots between layers
  int64_t src_off;       // KV contiguous layout: row of position 0; generic: first leaf
  int32_t log2_pad;
  int32_t log2_chunk;
  int32_t n_chunks;      // chunks holding at least one real leaf
  int32_t tree_base;     // tree index of layer 0 (tree = tree_base + layer)
  int32_t seq;           // KV: block-table row
  int32_t pad_;
  int64_t pos_base;      // KV: leaf position of local row 0 (split trees; 0 otherwise)
};

struct TreeOut {
  uint8_t* nodes;            // full node arrays, or nullptr (roots only)
  uint8_t* croots;           // chunk-root scratch, used when nodes == nullptr
  uint32_t* counters;        // [n_trees] finished-chunk counters, zero on entry and on exit
  uint8_t* roots;            // [n_trees][32]
  const uint32_t* zero_roots;// [kMaxTreeHeight + 1][8] Z_k words
};

struct KvArgs {
  const TreeMeta* meta;
  const int2* items;         // (meta index, chunk index) per CTA column
  const void* const* k_layers;
  const void* const* v_layers;
  const int32_t* block_tables;
  int64_t stride_page, stride_row, stride_head;  // elements
  int32_t block_size, max_blocks;
  int32_t n_heads, head_dim;
  int32_t layer_base;
  int32_t paged;
  int64_t cache_elems;       // every row must lie inside [0, cache_elems) elements
  int64_t row_span;          // (n_heads - 1) * stride_head + head_dim: extent of one row
  int* err;                  // set to 1 when a row falls outside the cache
  TreeOut out;
};

struct TreeArgs {
  const TreeMeta* meta;
  const int2* items;
  const uint8_t* leaves;
  TreeOut out;
};

struct ProveReq {
  int64_t node_base;   // first node of the tree
  uint32_t leaf;
  int32_t log2_pad;
};

// KvEntry materialisation for openings: (layer sel, position) -> f64 K row, f64 V row.
struct KvOpenArgs {
  KvArgs kv;               // addressing of the committed transcript (k_layers/v_layers device tables)
  TreeMeta seq;            // the opened sequence (seq index, src_off)
  const int32_t* layers;   // [n_sel] layer indices (within the call's layers)
  int32_t n_sel, n_pos, kv_dim;
  double* out;             // [n_sel][n_pos][2][kv_dim]
};

cudaError_t launch_zero_roots(uint32_t* z, cudaStream_t s);
cudaError_t launch_kv_entries(const KvOpenArgs& a, int dtype, cudaStream_t s);
cudaError_t launch_kv_commit(const KvArgs& a, int n_items, int n_layers, int dtype, bool fast,
                             cudaStream_t s);
cudaError_t launch_tree_commit(const TreeArgs& a, int n_items, cudaStream_t s);
// Subtrees without a real leaf (split trees past the sequence's end): nodes Z_k, root Z_lp.
cudaError_t launch_empty_trees(const TreeMeta* meta, const int32_t* which, int n_empty, int n_layers,
                               const TreeOut& o, cudaStream_t s);
cudaError_t launch_prove(const uint8_t* nodes, const ProveReq* reqs, int n, int max_depth,
                         uint8_t* siblings, cudaStream_t s);

// trace.cu
struct TraceArgs {
  int32_t n_tokens, n_layers, hidden;
  const int32_t* tok;           // [n_tokens][5]: fwd, row, fr_row, lp_row, logits_row
  const void* const* a_rows;    // [n_fwd * n_layers]
  const void* const* scale_a;
  int64_t scale_stride;
  const void* const* x_rows;    // or nullptr
  const void* const* scale_x;
  int64_t scale_x_stride;
  const uint8_t* fr; int32_t fr_dim; int64_t fr_stride;
  const uint8_t* lp; int32_t lp_dim; int64_t lp_stride;
  const uint8_t* logits; int32_t vocab; int64_t logits_stride;
  uint8_t* leaves;
  Opq opq;                      // multipliers of the balanced compression (make_opq())
  int* err;                     // the context's error flag (2: a bounded wait ran out)
};
cudaError_t launch_trace_leaves(const TraceArgs& a, int n_sm, cudaStream_t s);
cudaError_t launch_io_chain(int n_seqs, const int64_t* tok_off_dev, const uint8_t* leaves,
                            const uint32_t* token_ids, const uint8_t* prompt_hash, uint8_t* io, uint8_t* prev_io,
                            cudaStream_t s);
cudaError_t launch_tagged_hash(int n, int tag, const uint8_t* data, const int64_t* off_dev,
                               int64_t fixed_len, uint8_t* out, cudaStream_t s);

// api.cu: record the calling thread's error text (read by vc_last_error).
int32_t set_error(int32_t status, const char* fmt, ...);

// kv_transcript.cu
struct KvtLayer {
  const float* ch[2];     // per-channel weight scales of Wk, Wv ([kv_dim]) or nullptr
  const float* bias[2];   // K, V projection biases ([kv_dim]) or nullptr
  float sw[2];            // per-tensor weight scales (0 when absent)
  int32_t pad_[2];
};

struct KvtArgs {
  const CUtensorMap* maps;     // [n_layers][3]: x_attn, Wk, Wv (64-byte aligned, device)
  const KvtLayer* layers;      // [n_layers]
  const float* scale_x;        // scale_x_attn of (t, l) at t * sx_t + l * sx_l
  int64_t sx_t, sx_l;
  const double2* rope;         // [head_dim / 2][rope_rows] (cos, sin), or nullptr (toy path)
  int64_t rope_rows;           // positions in the table (>= n_tokens)
  double* out[2];              // K, V: [n_layers][n_tokens][kv_dim]
  int32_t n_tokens, hidden, kv_dim, head_dim;
  int32_t tile_cols;           // channels stored per tile: whole heads, <= 256
  int32_t tiles_per_mat;
  int32_t m_tiles;             // ceil(n_tokens / 128)
  int32_t n_tiles;             // n_layers * m_tiles * 2 * tiles_per_mat
  int32_t use_rope;
  int* err;                    // set to 2 when a bounded wait ran out
};
int kvt_group_width(int head_dim);
size_t kvt_smem_bytes();
std::vector<double> kvt_inv_freq(int head_dim, double theta, int scaling_type, double factor, double low_ff,
                                 double high_ff, int64_t orig_max_pos);
void kvt_rope_table(const std::vector<double>& inv, int64_t n_pos, double* out);
int kvt_encode_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t row_stride,
                   int box_rows);
cudaError_t launch_kv_transcript(const KvtArgs& a, int n_sm, cudaStream_t s);

// kvt_commit.cu: the transcript and its KV trees in one pass (no f64 rows in memory)
struct KvtcArgs {
  KvtArgs t;                   // transcript (weight tensor maps with 128-row boxes; out[] unused)
  TreeMeta meta;               // the n_layers trees over positions 0..n_tokens-1
  TreeOut out;
  int32_t layer_base;          // leaf layer index = layer_base + layer
  int32_t n_units;             // n_layers * m_tiles units of 128 positions
};
bool kvt_commit_supported(int head_dim, int kv_dim);
cudaError_t launch_kvt_commit(const KvtcArgs& a, int n_sm, cudaStream_t s);

// int_peak.cu
cudaError_t launch_int_peak(int variant, int64_t iters, int n_sm, uint32_t* sink, cudaStream_t s,
                            double* ops_per_launch);
cudaError_t launch_wait_probe(uint64_t limit_ns, int* err, cudaStream_t s);

}  // namespace vc
