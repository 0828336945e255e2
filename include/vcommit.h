/*
 * vcommit.h -- C ABI of libvcommit.so, the B200 trace-commitment library.
 *
 * It replaces the hashing half of CommitLLM's provider-side commit
 * (crates/verilm-prover/src/lib.rs:336-544, commit_minimal; 753-964,
 * commit_minimal_packed) and the SHA-256 Merkle primitives it calls
 * (crates/verilm-core/src/merkle.rs:11-123, 144-293, 553-577).  Every digest,
 * root, opening and chain value is bit-identical to those functions on the
 * same inputs, so the existing verifier accepts the receipts unchanged.
 *
 * Conventions
 *   - Plain C: pointers, sizes, status codes.  No CUDA or torch types; a
 *     stream is passed as `void*` (a cudaStream_t, NULL = legacy default).
 *   - Pointers documented DEVICE are read/written in place in HBM; HOST
 *     arrays are small descriptor tables copied by the library.
 *   - Every call is stream-ordered and asynchronous on its context's stream,
 *     returns a vc_status and never aborts.  vc_last_error() gives the text.
 *   - Errors: VC_EINVAL where the reference raises PyValueError or panics on
 *     an assert (verilm-py/src/lib.rs:843-893, prover/src/lib.rs:347-351,
 *     766-802); VC_ERANGE where merkle::prove asserts an index
 *     (merkle.rs:80).
 *   - Threading: one context per stream; distinct contexts may be used from
 *     distinct host threads concurrently.
 *   - Digests are 32 bytes in SHA-256 output byte order ([u8; 32]).
 */
#ifndef VCOMMIT_H
#define VCOMMIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VC_ABI_VERSION 2

#if defined(__GNUC__)
#define VC_API __attribute__((visibility("default")))
#else
#define VC_API
#endif

typedef int32_t vc_status;
#define VC_OK 0
#define VC_EINVAL 1     /* invalid argument */
#define VC_ENOMEM 2     /* device or host allocation failed */
#define VC_ECUDA 3      /* a CUDA runtime call failed */
#define VC_ETIMEDOUT 4  /* a bounded wait ran out */
#define VC_ERANGE 5     /* index out of range */
#define VC_ENOTSUP 6    /* layout not supported */

/* Element type of K/V rows. */
#define VC_DTYPE_BF16 0 /* raw bf16 bits, widened exactly to f64 before hashing */
#define VC_DTYPE_F32 1  /* f32, widened exactly to f64 */
#define VC_DTYPE_F64 2  /* f64 as the reference's KvEntry holds it */

typedef struct vc_ctx vc_ctx;           /* per-stream context (scratch, staging) */
typedef struct vc_tree_set vc_tree_set; /* device-resident Merkle trees */

/* ---------------------------------------------------------------- context */

/* Version of this ABI (VC_ABI_VERSION). */
VC_API int32_t vc_abi_version(void);

/* Text of the last error raised on the calling host thread. Returns the
 * length of the message (excluding the NUL), truncating to buf_len-1. */
VC_API size_t vc_last_error(char* buf, size_t buf_len);

/* Create a context bound to CUDA device `device` and stream `stream`. */
VC_API vc_status vc_ctx_create(int32_t device, void* stream, vc_ctx** out);
VC_API vc_status vc_ctx_destroy(vc_ctx* ctx);
/* Wait for the context's stream, polling, for at most timeout_ms
 * milliseconds (<= 0: no limit). VC_ETIMEDOUT when the limit is reached.
 * VC_ERANGE if a kernel of this context found a device-side index out of
 * range since the last sync (its output is then unspecified). */
VC_API vc_status vc_ctx_sync(vc_ctx* ctx, int32_t timeout_ms);

/* ------------------------------------------------------------- KV commit */

/*
 * Where the K and V rows live.  The row of (layer l, sequence s, position p)
 * is the kv_dim = n_kv_heads * head_dim elements
 *
 *   base_l + page * stride_page + slot * stride_row + h * stride_head + d
 *
 * for head h in [0, n_kv_heads), d in [0, head_dim), with
 *   paged      (block_tables != NULL): page = block_tables[s * max_blocks_per_seq
 *              + p / block_size], slot = p % block_size;
 *   contiguous (block_tables == NULL): page = 0, slot = seq_row_offset[s] + p.
 * Strides are in elements.  vLLM's flash layout [pages, block, heads, dim] is
 * stride_page = block*kv_dim, stride_row = kv_dim, stride_head = head_dim.
 *
 * K concatenates heads head-major, the order rope.rs:95-98 uses for
 * kv_dim = h * d_head + i, and so does V.
 */
typedef struct vc_kv_desc {
    int32_t n_layers;      /* layers in this call */
    int32_t layer_base;    /* leaf layer index = layer_base + l (layer sharding) */
    int32_t n_kv_heads;
    int32_t head_dim;
    int32_t dtype;         /* VC_DTYPE_* */
    int32_t n_seqs;
    const int32_t* seq_lens;          /* HOST [n_seqs], each >= 1 */
    const int64_t* seq_row_offset;    /* HOST [n_seqs], contiguous layout; NULL = prefix sum of seq_lens */
    const int32_t* block_tables;      /* DEVICE [n_seqs * max_blocks_per_seq] or NULL */
    int32_t block_size;
    int32_t max_blocks_per_seq;
    int64_t stride_page;
    int64_t stride_row;
    int64_t stride_head;
    int64_t cache_elems;              /* elements in each layer's K (and V) buffer, > 0:
                                         every row is bounds-checked against it (rows
                                         of a paged cache on the device; a bad page id
                                         is reported by vc_ctx_sync as VC_ERANGE) */
    const void* const* k_layers;      /* HOST [n_layers] DEVICE base pointers */
    const void* const* v_layers;      /* HOST [n_layers] DEVICE base pointers */
    /* Split trees: one request's trees spread over G GPUs, each holding the
     * aligned range [r * 2^tree_log2, (r + 1) * 2^tree_log2) of positions
     * (n_pad = G * 2^tree_log2, G a power of two).  Each GPU commits its
     * subtrees; the all-gathered subtree roots, as the G leaves of one
     * vc_build_trees tree per layer, give the merkle::build_tree roots
     * (merkle.rs:11-48), since build_tree pads only level 0 with zeros. */
    const int64_t* pos_base;          /* HOST [n_seqs] or NULL (0): position of the sequence's local row 0,
                                         the u32 position hashed into hash_kv_entry */
    int32_t tree_log2;                /* 0: every tree padded to the next power of two of seq_lens[s]
                                         (build_tree); > 0: every tree is the subtree of 2^tree_log2 leaves,
                                         the first seq_lens[s] real (0 allowed: a subtree of zero leaves,
                                         root Z_tree_log2), the rest zero */
} vc_kv_desc;

/*
 * Per-layer KV Merkle roots: hot loop C of commit_minimal
 * (crates/verilm-prover/src/lib.rs:449-482).  Leaf (l, p) is
 * merkle::hash_kv_entry(layer_base + l, p, f64(K row), f64(V row))
 * (merkle.rs:285-293); each (sequence, layer) gets one merkle::build_tree
 * (merkle.rs:11-48) over positions 0..seq_lens[s].
 *
 * kv_roots_dev: DEVICE [n_seqs][n_layers][32] -- sequence s's kv_roots are the
 *   n_layers consecutive roots, the layout of BatchCommitment.kv_roots
 *   (types.rs:1753-1758).
 * trees_out: if non-NULL, receives every node of every tree (for openings);
 *   tree index = s * n_layers + l.  Free with vc_tree_set_free.
 */
VC_API vc_status vc_kv_commit(vc_ctx* ctx, const vc_kv_desc* desc, uint8_t* kv_roots_dev,
                       vc_tree_set** trees_out);

/*
 * Allocation-free variant of vc_kv_commit.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory when they commit
 * (an engine that has reserved all free HBM for its KV cache, or code that
 * must not stall the device in cudaMalloc).  It calls no cudaMalloc,
 * cudaFree or allocating library routine and needs no context: its scratch
 * is a fixed 8 MiB device array inside the library (plus a small padding-root
 * table), held by every GPU that loads the library until the process exits.
 *
 * Same descriptor and output as vc_kv_commit (without split trees: pos_base
 * and tree_log2 must be NULL / 0, VC_ENOTSUP otherwise), roots only (no tree set), on
 * the given stream (NULL = legacy default stream) of the current device.
 * Limits: at most 64 sequences and 256 layers per call, kv_dim and head_dim
 * multiples of 8, 16-byte aligned rows (VC_ENOTSUP otherwise), and
 * 256 + 4 * n_trees (rounded up to 256) + 32 * (sum over trees of
 * padded_size / 128) bytes of scratch <= 8 MiB (VC_EINVAL otherwise).
 * err_flag_dev: DEVICE int set to 1 when a paged row (a negative page id or
 * one past cache_elems in the device block table) falls outside the cache;
 * the caller clears it before the call and reads it after.  The roots of a
 * call that set it are void.  Required for a paged layout (VC_EINVAL when
 * NULL); contiguous rows are checked on the host, and may pass NULL.
 * The first call on a device looks up the scratch address and fills the
 * padding-root table, synchronising the stream once: make that first call
 * before any stream capture.  Every call shares the one scratch array, so
 * calls whose kernels overlap on the GPU race: serialise them (one stream,
 * or events).
 */
VC_API vc_status vc_kv_commit_noalloc(const vc_kv_desc* desc, uint8_t* kv_roots_dev, int32_t* err_flag_dev,
                                      void* stream);

/* ----------------------------------------------------------- trace leaves */

/*
 * Retained-state ("trace") leaves, hot loop A of commit_minimal
 * (prover/src/lib.rs:367-393): per token
 *   base = hash_retained_state_direct  (merkle.rs:144-161)
 *   then the optional wraps of merkle.rs:170-241, each applied when the
 *   token's row index for it is >= 0:
 *     "vi-retained-fr-v1"     || base || f32le[final_residual]
 *     "vi-retained-lp-v1"     || prev || u16le[lp_hidden_bf16]
 *     "vi-retained-logits-v1" || prev || f32le[captured_logits]
 *
 * Token t's activation rows come from forward pass tok_fwd[t], batch row
 * tok_row[t]: a_i8 of layer l at a_rows[f * n_layers + l] + row * hidden, and
 * scale_a at scale_a[f * n_layers + l][row * scale_stride].  This covers both
 * reference layouts: the per-(fwd, layer) buffers of
 * commit_minimal_from_captures (verilm-py/src/lib.rs:800-885) and
 * commit_minimal_packed's packed_a / packed_scales (prover/src/lib.rs:601-605).
 *
 * x_attn_rows / scale_x_attn non-NULL binds the optional "0x01 || x_attn_i8 ||
 * f32le(scale_x_attn)" field; NULL hashes the 0x00 marker, as the
 * reference's production path does (prover/src/lib.rs:162-167).
 */
typedef struct vc_trace_desc {
    int32_t n_tokens;
    int32_t n_layers;
    int32_t hidden;                      /* bytes per a_i8 (and x_attn) row */
    int32_t n_fwd;
    const int32_t* fwd_rows;             /* HOST [n_fwd]: batch rows of each forward pass */
    const int32_t* tok_fwd;              /* HOST [n_tokens] */
    const int32_t* tok_row;              /* HOST [n_tokens] */
    const void* const* a_rows;           /* HOST [n_fwd * n_layers] DEVICE i8 */
    const void* const* scale_a;          /* HOST [n_fwd * n_layers] DEVICE f32 */
    int64_t scale_stride;                /* f32 elements between batch rows */
    const void* const* x_attn_rows;      /* HOST [n_fwd * n_layers] DEVICE i8, or NULL */
    const void* const* scale_x_attn;     /* HOST [n_fwd * n_layers] DEVICE f32, or NULL */
    int64_t scale_x_stride;
    /* optional wraps: DEVICE row-major arrays of *_rows rows (stride in
     * elements) + HOST per-token row index (-1: not bound for that token) */
    const void* final_residual;  int32_t fr_dim;  int32_t fr_rows;     int64_t fr_stride;
    const int32_t* tok_fr_row;
    const void* lp_hidden;       int32_t lp_dim;  int32_t lp_rows;     int64_t lp_stride;
    const int32_t* tok_lp_row;
    const void* logits;          int32_t vocab;   int32_t logits_rows; int64_t logits_stride;
    const int32_t* tok_logits_row;
} vc_trace_desc;

/* leaves_dev: DEVICE [n_tokens][32]. */
VC_API vc_status vc_trace_leaves(vc_ctx* ctx, const vc_trace_desc* desc, uint8_t* leaves_dev);

/* ---------------------------------------------------------------- IO chain */

/*
 * IO chains (prover/src/lib.rs:403-410): for each sequence s over its tokens
 * t in [tok_off[s], tok_off[s+1]):
 *   prev = io_genesis_v4(prompt_hash[s])                   (merkle.rs:572-577)
 *   io[t] = io_hash_v4(leaves[t], token_ids[t], prev)      (merkle.rs:250-257)
 * tok_off: HOST [n_seqs + 1]; leaves_dev, io_dev: DEVICE [n_tokens][32];
 * token_ids_dev: DEVICE u32 [n_tokens]; prompt_hash_dev: DEVICE [n_seqs][32].
 */
VC_API vc_status vc_io_chain(vc_ctx* ctx, int32_t n_seqs, const int64_t* tok_off,
                      const uint8_t* leaves_dev, const uint32_t* token_ids_dev,
                      const uint8_t* prompt_hash_dev, uint8_t* io_dev);

/*
 * Online extension of IO chains (the same loop as vc_io_chain, resumed):
 * sequence s appends the tokens [tok_off[s], tok_off[s+1]) -- leaves_dev,
 * token_ids_dev and io_dev indexed by token as in vc_io_chain -- starting
 * from prev_io_dev[s] (its last io value, or its genesis), and
 * prev_io_dev[s] receives the new last value.  A sequence with no tokens
 * keeps its value.  prev_io_dev: DEVICE [n_seqs][32].
 */
VC_API vc_status vc_io_extend(vc_ctx* ctx, int32_t n_seqs, const int64_t* tok_off, const uint8_t* leaves_dev,
                              const uint32_t* token_ids_dev, uint8_t* prev_io_dev, uint8_t* io_dev);

/* io_genesis_v4 (merkle.rs:572-577) of n prompt hashes: DEVICE [n][32] -> [n][32]. */
VC_API vc_status vc_io_genesis(vc_ctx* ctx, int32_t n, const uint8_t* prompt_hash_dev, uint8_t* out_dev);

/* hash_prompt (merkle.rs:561-566) of n prompts; prompt i is the bytes
 * [off[i], off[i+1]) of prompts_dev.  off: HOST [n + 1]; out: DEVICE [n][32]. */
VC_API vc_status vc_prompt_hash(vc_ctx* ctx, int32_t n, const uint8_t* prompts_dev,
                         const int64_t* off, uint8_t* out_dev);

/* hash_seed (merkle.rs:553-558) of n 32-byte seeds: DEVICE [n][32] -> [n][32]. */
VC_API vc_status vc_seed_commitment(vc_ctx* ctx, int32_t n, const uint8_t* seeds_dev,
                             uint8_t* out_dev);

/* ------------------------------------------------------------- Merkle trees */

/*
 * merkle::build_tree (merkle.rs:11-48) over n_trees independent leaf ranges:
 * tree i has the leaves [leaf_off[i], leaf_off[i+1]) of leaves_dev (>= 1 leaf).
 * leaf_off: HOST [n_trees + 1]; roots_dev: DEVICE [n_trees][32];
 * trees_out: optional, as for vc_kv_commit.
 */
VC_API vc_status vc_build_trees(vc_ctx* ctx, int32_t n_trees, const int64_t* leaf_off,
                         const uint8_t* leaves_dev, uint8_t* roots_dev,
                         vc_tree_set** trees_out);

/*
 * merkle::prove (merkle.rs:79-99) for n openings (tree[i], leaf[i]), HOST
 * arrays.  siblings_dev: DEVICE [n][max_depth][32], bottom-up, the order of
 * MerkleProof.siblings (merkle.rs:303-307); depth_out: HOST [n], the number
 * of siblings of each proof (log2 of the tree's padded size).
 * VC_ERANGE if a leaf index is >= the tree's leaf count or a tree is unknown.
 */
VC_API vc_status vc_prove(vc_ctx* ctx, const vc_tree_set* trees, int32_t n, const int32_t* tree,
                   const uint32_t* leaf, uint8_t* siblings_dev, int32_t max_depth,
                   int32_t* depth_out);

/*
 * KV openings of one sequence, as open_v4 returns them
 * (crates/verilm-prover/src/lib.rs:1564-1588): for each selected layer
 * (layers[i], HOST, indices into desc's layers) and every position
 * p in 0..n_positions-1 (the challenged token index + 1):
 *   entries_dev[i][p] = KvEntry { k_roped: f64[kv_dim], v_deq: f64[kv_dim] }
 *     (types.rs:1244-1251), the rows the leaf hashed, widened as hashed;
 *     DEVICE f64 [n_sel][n_positions][2][kv_dim];
 *   siblings_dev[i][p] = merkle::prove(kv_tree[layer], p).siblings
 *     (merkle.rs:79-99), DEVICE [n_sel][n_positions][max_depth][32].
 * trees: the tree set vc_kv_commit returned for the same descriptor.
 * *depth_out: the proof length (log2 of the sequence's padded length).
 */
VC_API vc_status vc_kv_open(vc_ctx* ctx, const vc_kv_desc* desc, const vc_tree_set* trees, int32_t seq,
                            int32_t n_sel, const int32_t* layers, int32_t n_positions, double* entries_dev,
                            uint8_t* siblings_dev, int32_t max_depth, int32_t* depth_out);

/* Shape of a tree set: number of trees. */
VC_API int32_t vc_tree_set_count(const vc_tree_set* trees);
/*
 * The node array of one tree, laid out as MerkleTree.nodes (merkle.rs:16-39):
 * level 0 (padded_size leaves, zero padded), then each parent level, root
 * last; 2 * padded_size - 1 nodes of 32 bytes.  *nodes_dev is DEVICE memory
 * owned by the tree set.
 */
VC_API vc_status vc_tree_nodes(const vc_tree_set* trees, int32_t tree, const uint8_t** nodes_dev,
                        int64_t* n_leaves, int64_t* padded_size);
VC_API vc_status vc_tree_set_free(vc_tree_set* trees);

/* ------------------------------------------------------------ KV transcript */

/* Rope scaling of ModelConfig (crates/verilm-core/src/constants.rs:126-156). */
#define VC_ROPE_NONE 0
#define VC_ROPE_LLAMA3 1
#define VC_ROPE_LINEAR 2

typedef struct vc_kvt_desc {
    int32_t n_tokens;        /* positions 0..n_tokens-1 (token order of captured_x_attn) */
    int32_t n_layers;
    int32_t hidden;          /* hidden_dim: multiple of 16 */
    int32_t n_kv_heads;
    int32_t head_dim;        /* d_head: even, <= 256 */
    int32_t use_rope;        /* 0: toy path (clamp to i8, lib.rs:307-316); 1: dequant + bias + RoPE */
    const int8_t* const* x_layers;   /* HOST [n_layers] DEVICE: row t of layer l at x_layers[l] + t * x_row_stride */
    int64_t x_row_stride;            /* bytes, multiple of 16, >= hidden */
    const int8_t* const* wk_layers;  /* HOST [n_layers] DEVICE [kv_dim][hidden] row-major (Wk) */
    const int8_t* const* wv_layers;  /* HOST [n_layers] DEVICE [kv_dim][hidden] row-major (Wv) */
    const float* scale_x;            /* DEVICE: scale_x_attn of (t, l) at scale_x[t * sx_tstride + l * sx_lstride] */
    int64_t sx_tstride, sx_lstride;
    const float* sw_k;               /* HOST [n_layers] per-tensor scales of Wk, or NULL (0.0) */
    const float* sw_v;               /* HOST [n_layers] per-tensor scales of Wv, or NULL (0.0) */
    const float* const* ch_k;        /* HOST [n_layers] of DEVICE [kv_dim] per-channel scales, or NULL;
                                        a NULL entry falls back to the per-tensor scale */
    const float* const* ch_v;
    const float* const* bias_k;      /* HOST [n_layers] of DEVICE [kv_dim] biases, or NULL / NULL entries */
    const float* const* bias_v;
    double rope_theta;
    int32_t rope_scaling;            /* VC_ROPE_* */
    int32_t rope_original_max_position_embeddings;
    double rope_factor, rope_low_freq_factor, rope_high_freq_factor;
} vc_kvt_desc;

/*
 * verilm_prover::compute_kv_transcript (crates/verilm-prover/src/lib.rs:207-329):
 * the committed KV values from captured x_attn and the Wk/Wv weights, on the
 * tensor cores.  k_acc = Wk x_attn, v_acc = Wv x_attn (exact i32, matmul.rs:12-22);
 * use_rope: per-channel ((acc * cw[c]) * sx, rope.rs:124-138) when the layer has
 * a per-channel table, else acc * (sw * sx) (rope.rs:107-112); + bias; K rotated
 * per head with scaled_inv_freq (constants.rs:253-297) and the C library's
 * cos/sin (rope.rs:38-60, 88-100).  Every f64 operation is rounded on its own.
 * k_out_dev / v_out_dev: DEVICE f64 [n_layers][n_tokens][kv_dim] (32-byte
 * aligned): KvEntry.k_roped / v_deq of (layer, position), ready for
 * vc_kv_commit with VC_DTYPE_F64 and stride_row = kv_dim.
 * Weights and x_attn base pointers must be 16-byte aligned (VC_EINVAL).
 * A wait that runs out inside the kernel is reported by vc_ctx_sync as VC_ETIMEDOUT.
 */
VC_API vc_status vc_kv_transcript(vc_ctx* ctx, const vc_kvt_desc* desc, double* k_out_dev, double* v_out_dev);

/*
 * compute_kv_transcript and hot loop C of commit_minimal in one pass
 * (crates/verilm-prover/src/lib.rs:207-329 then 449-482; the pair
 * verilm-py/src/lib.rs:941-975 runs): per layer l, the kv_root of
 * merkle::build_tree over hash_kv_entry(layer_base + l, p, K[l][p], V[l][p])
 * for p in 0..n_tokens-1, with K/V exactly the f64 rows vc_kv_transcript
 * writes.  The rows are hashed as they leave the tensor cores and never stored,
 * so the kv_roots (and trees) equal vc_kv_transcript followed by vc_kv_commit
 * (VC_DTYPE_F64) bit for bit, without the 16 bytes per K/V element pair of
 * HBM traffic in between.  Openings re-derive the rows they reveal with
 * vc_kv_transcript over the opened positions.
 * kv_roots_dev: DEVICE [n_layers][32]; trees_out: optional, as for
 * vc_kv_commit (tree index = l).  head_dim 64 or 128 with kv_dim a multiple of
 * 128 run fused; other shapes run the two calls through device scratch.
 * n_tokens >= 1.
 */
VC_API vc_status vc_kv_transcript_commit(vc_ctx* ctx, const vc_kvt_desc* desc, int32_t layer_base,
                                         uint8_t* kv_roots_dev, vc_tree_set** trees_out);

/* --------------------------------------------------------- measurement aid */

/*
 * Integer-ALU peak probe: runs a register-only loop of 32-bit funnel shifts,
 * 3-input logic ops and 3-input adds in SHA-256's proportions across the whole
 * device for `iters` iterations and reports executed 32-bit ops per second
 * (device-timed).  variant 0: SHA-256 mix; 1: funnel shift only;
 * 2: lop3 only; 3: iadd3 only.
 */
VC_API vc_status vc_int_peak(vc_ctx* ctx, int32_t variant, int64_t iters, double* ops_per_s);

/*
 * Bounded-wait probe (no reference counterpart; the reference has no device
 * waits): launches one thread that waits on an mbarrier nothing arrives at.
 * Its wait gives up after limit_ns (1 .. 2e9) nanoseconds and sets the
 * context's error flag, exactly as a bounded wait of the commit kernels does
 * when the work it waits for never lands; the next vc_ctx_sync then returns
 * VC_ETIMEDOUT and clears the flag, and the context stays usable.  Lets a
 * caller check that failure path without faulting or hanging a GPU.
 */
VC_API vc_status vc_wait_probe(vc_ctx* ctx, int64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* VCOMMIT_H */
