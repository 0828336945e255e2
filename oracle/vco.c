/*
 * vco.c -- the oracle's C restatement of CommitLLM's commitment hashing.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for large cases and the timed CPU
 * baseline.  Nothing in the product (commitllm_b200/) links or loads it.
 *
 * It restates, on the host CPU:
 *   merkle::hash_kv_entry      crates/verilm-core/src/merkle.rs:285-293
 *   merkle::build_tree         merkle.rs:11-48 (nodes level-concatenated)
 *   merkle::compute_root       merkle.rs:55-76
 *   hash_retained_state_direct merkle.rs:144-161, wraps 170-241
 *   io_hash_v4 / io_genesis_v4 / hash_prompt  merkle.rs:250-257, 561-577
 *   the KV-tree loop of commit_minimal  crates/verilm-prover/src/lib.rs:449-482
 *   compute_kv_transcript      crates/verilm-prover/src/lib.rs:207-329 (per-tensor / toy)
 * SHA-256 is OpenSSL's (FIPS 180-4, SHA-NI when the CPU has it), standing in
 * for the sha2 0.10.9 crate the reference uses (Cargo.lock:783-784), which
 * also dispatches to SHA-NI at run time.
 *
 * Threading: vco_kv_commit with n_threads == 1 is the reference's sequential
 * per-layer loop; n_threads > 1 hashes distinct trees on distinct threads.
 */
#define _GNU_SOURCE
#include <math.h>
#include <openssl/sha.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/vcommit.h"

#pragma GCC diagnostic ignored "-Wdeprecated-declarations"

static void hash_pair(const uint8_t* l, const uint8_t* r, uint8_t* out) {
  uint8_t buf[64];
  memcpy(buf, l, 32);
  memcpy(buf + 32, r, 32);
  SHA256(buf, 64, out);
}

static int ilog2_ceil(int64_t n) {
  int lp = 0;
  while (((int64_t)1 << lp) < n) ++lp;
  return lp;
}

/* build_tree: nodes_out has room for 2*pad-1 nodes; returns the root in nodes[2*pad-2]. */
void vco_build_tree(const uint8_t* leaves, int64_t n, uint8_t* nodes_out) {
  const int64_t pad = (int64_t)1 << ilog2_ceil(n);
  memcpy(nodes_out, leaves, (size_t)n * 32);
  memset(nodes_out + n * 32, 0, (size_t)(pad - n) * 32);
  int64_t start = 0, size = pad, w = pad;
  while (size > 1) {
    for (int64_t i = 0; i < size; i += 2) {
      hash_pair(nodes_out + (start + i) * 32, nodes_out + (start + i + 1) * 32, nodes_out + w * 32);
      ++w;
    }
    start += size;
    size /= 2;
  }
}

/* compute_root: in-place over a scratch copy. */
void vco_compute_root(const uint8_t* leaves, int64_t n, uint8_t* root) {
  const int64_t pad = (int64_t)1 << ilog2_ceil(n);
  uint8_t* lvl = (uint8_t*)malloc((size_t)pad * 32);
  memcpy(lvl, leaves, (size_t)n * 32);
  memset(lvl + n * 32, 0, (size_t)(pad - n) * 32);
  for (int64_t size = pad; size > 1; size /= 2)
    for (int64_t i = 0; i < size; i += 2) hash_pair(lvl + i * 32, lvl + (i + 1) * 32, lvl + (i / 2) * 32);
  memcpy(root, lvl, 32);
  free(lvl);
}

/* Widen one K/V element to f64 (exact; x86 quiets signalling NaNs). */
static double widen(const uint8_t* p, int dtype) {
  if (dtype == VC_DTYPE_BF16) {
    uint16_t b;
    memcpy(&b, p, 2);
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
  }
  if (dtype == VC_DTYPE_F32) {
    float f;
    memcpy(&f, p, 4);
    return (double)f;
  }
  double d;
  memcpy(&d, p, 8);
  return d;
}

static int esize(int dtype) { return dtype == VC_DTYPE_BF16 ? 2 : (dtype == VC_DTYPE_F32 ? 4 : 8); }

/* Element offset of the row of (seq s, position p) in a layer buffer. */
static int64_t kv_row(const vc_kv_desc* d, int s, int64_t p, const int64_t* row0) {
  if (d->block_tables) {
    const int32_t page = d->block_tables[(int64_t)s * d->max_blocks_per_seq + p / d->block_size];
    return (int64_t)page * d->stride_page + (p % d->block_size) * d->stride_row;
  }
  return (row0[s] + p) * d->stride_row;
}

/* hash_kv_entry of one (layer, position); msg has room for 16 + 16*kv bytes. */
static void kv_leaf(const vc_kv_desc* d, int l, int s, int64_t p, const int64_t* row0, uint8_t* msg, uint8_t* out) {
  const int es = esize(d->dtype);
  const int64_t kv = (int64_t)d->n_kv_heads * d->head_dim;
  const uint32_t layer = (uint32_t)(d->layer_base + l), pos = (uint32_t)p;
  memcpy(msg, "vi-kv-v1", 8);
  memcpy(msg + 8, &layer, 4);
  memcpy(msg + 12, &pos, 4);
  const int64_t off = kv_row(d, s, p, row0);
  double* dst = (double*)(msg + 16);
  for (int sel = 0; sel < 2; ++sel) {
    const uint8_t* base = (const uint8_t*)(sel ? d->v_layers[l] : d->k_layers[l]) + off * es;
    for (int h = 0; h < d->n_kv_heads; ++h) {
      const uint8_t* hp = base + (int64_t)h * d->stride_head * es;
      for (int i = 0; i < d->head_dim; ++i) {
        const double v = widen(hp + (int64_t)i * es, d->dtype);
        memcpy(dst++, &v, 8);
      }
    }
  }
  SHA256(msg, (size_t)(16 + 16 * kv), out);
}

void vco_kv_leaf(const vc_kv_desc* d, int32_t layer, int32_t seq, int64_t pos, uint8_t* out) {
  int64_t* row0 = (int64_t*)calloc((size_t)d->n_seqs, sizeof(int64_t));
  int64_t acc = 0;
  for (int s = 0; s < d->n_seqs; ++s) {
    row0[s] = d->seq_row_offset ? d->seq_row_offset[s] : acc;
    acc += d->seq_lens[s];
  }
  const int64_t kv = (int64_t)d->n_kv_heads * d->head_dim;
  uint8_t* msg = (uint8_t*)malloc((size_t)(16 + 16 * kv));
  kv_leaf(d, layer, seq, pos, row0, msg, out);
  free(msg);
  free(row0);
}

typedef struct {
  const vc_kv_desc* d;
  const int64_t* row0;
  uint8_t* roots;
  uint8_t* nodes;        /* optional: per-tree node arrays at node_off */
  const int64_t* node_off;
  int64_t next;          /* next tree to take (atomic) */
  int64_t n_trees;
} kv_job;

static void* kv_worker(void* arg) {
  kv_job* j = (kv_job*)arg;
  const vc_kv_desc* d = j->d;
  const int64_t kv = (int64_t)d->n_kv_heads * d->head_dim;
  uint8_t* msg = (uint8_t*)malloc((size_t)(16 + 16 * kv));
  int64_t max_n = 1;
  for (int s = 0; s < d->n_seqs; ++s)
    if (d->seq_lens[s] > max_n) max_n = d->seq_lens[s];
  uint8_t* leaves = (uint8_t*)malloc((size_t)max_n * 32);
  for (;;) {
    const int64_t t = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (t >= j->n_trees) break;
    const int s = (int)(t / d->n_layers), l = (int)(t % d->n_layers);
    const int64_t n = d->seq_lens[s];
    for (int64_t p = 0; p < n; ++p) kv_leaf(d, l, s, p, j->row0, msg, leaves + p * 32);
    if (j->nodes) {
      uint8_t* nodes = j->nodes + j->node_off[t] * 32;
      vco_build_tree(leaves, n, nodes);
      const int64_t pad = (int64_t)1 << ilog2_ceil(n);
      memcpy(j->roots + t * 32, nodes + (2 * pad - 2) * 32, 32);
    } else {
      vco_compute_root(leaves, n, j->roots + t * 32);
    }
  }
  free(leaves);
  free(msg);
  return NULL;
}

/* kv_roots of every (sequence, layer): roots [n_seqs][n_layers][32].  With
 * nodes != NULL each tree's build_tree nodes go to nodes + node_off[t]*32,
 * t = s*n_layers + l.  All pointers in d are host pointers. */
int vco_kv_commit(const vc_kv_desc* d, uint8_t* roots, uint8_t* nodes, const int64_t* node_off, int n_threads) {
  if (!d || !roots || d->n_layers < 1 || d->n_seqs < 1) return VC_EINVAL;
  int64_t* row0 = (int64_t*)calloc((size_t)d->n_seqs, sizeof(int64_t));
  int64_t acc = 0;
  for (int s = 0; s < d->n_seqs; ++s) {
    if (d->seq_lens[s] < 1) {
      free(row0);
      return VC_EINVAL;
    }
    row0[s] = d->seq_row_offset ? d->seq_row_offset[s] : acc;
    acc += d->seq_lens[s];
  }
  kv_job j = {d, row0, roots, nodes, node_off, 0, (int64_t)d->n_seqs * d->n_layers};
  if (n_threads < 1) n_threads = 1;
  if (n_threads == 1) {
    kv_worker(&j);
  } else {
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, kv_worker, &j);
    for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
    free(th);
  }
  free(row0);
  return VC_OK;
}

/* --- retained leaves and IO chain (host pointers; same table layout as vc_trace_desc) --- */

static void retained_leaf(const vc_trace_desc* d, int t, uint8_t* out) {
  SHA256_CTX c;
  SHA256_Init(&c);
  SHA256_Update(&c, "vi-retained-v3", 14);
  const int f = d->tok_fwd[t];
  const int64_t row = d->tok_row[t];
  for (int l = 0; l < d->n_layers; ++l) {
    const int64_t fl = (int64_t)f * d->n_layers + l;
    SHA256_Update(&c, (const uint8_t*)d->a_rows[fl] + row * d->hidden, (size_t)d->hidden);
    SHA256_Update(&c, (const float*)d->scale_a[fl] + row * d->scale_stride, 4);
    if (d->x_attn_rows) {
      SHA256_Update(&c, "\x01", 1);
      SHA256_Update(&c, (const uint8_t*)d->x_attn_rows[fl] + row * d->hidden, (size_t)d->hidden);
      SHA256_Update(&c, (const float*)d->scale_x_attn[fl] + row * d->scale_x_stride, 4);
    } else {
      SHA256_Update(&c, "\x00", 1);
    }
  }
  uint8_t base[32];
  SHA256_Final(base, &c);
  struct { const char* tag; int tl; const void* p; int32_t dim; int64_t stride; const int32_t* tok; int es; } w[3] = {
      {"vi-retained-fr-v1", 17, d->final_residual, d->fr_dim, d->fr_stride, d->tok_fr_row, 4},
      {"vi-retained-lp-v1", 17, d->lp_hidden, d->lp_dim, d->lp_stride, d->tok_lp_row, 2},
      {"vi-retained-logits-v1", 21, d->logits, d->vocab, d->logits_stride, d->tok_logits_row, 4}};
  for (int k = 0; k < 3; ++k) {
    if (!w[k].tok || w[k].tok[t] < 0) continue;
    SHA256_Init(&c);
    SHA256_Update(&c, w[k].tag, (size_t)w[k].tl);
    SHA256_Update(&c, base, 32);
    SHA256_Update(&c, (const uint8_t*)w[k].p + (int64_t)w[k].tok[t] * w[k].stride * w[k].es, (size_t)w[k].dim * w[k].es);
    SHA256_Final(base, &c);
  }
  memcpy(out, base, 32);
}

typedef struct {
  const vc_trace_desc* d;
  uint8_t* leaves;
  int64_t next;
} trace_job;

static void* trace_worker(void* arg) {
  trace_job* j = (trace_job*)arg;
  for (;;) {
    const int64_t t = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (t >= j->d->n_tokens) break;
    retained_leaf(j->d, (int)t, j->leaves + t * 32);
  }
  return NULL;
}

/* Hot loop A of commit_minimal (rayon par_iter over tokens): leaves [n_tokens][32]. */
int vco_trace_leaves(const vc_trace_desc* d, uint8_t* leaves, int n_threads) {
  trace_job j = {d, leaves, 0};
  if (n_threads <= 1) {
    trace_worker(&j);
    return VC_OK;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
  for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, trace_worker, &j);
  for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
  free(th);
  return VC_OK;
}

/* IO chain (prover/src/lib.rs:403-410) for one sequence of n tokens. */
void vco_io_chain(const uint8_t* leaves, const uint32_t* token_ids, int64_t n, const uint8_t* prompt,
                  int64_t prompt_len, uint8_t* io_out) {
  uint8_t ph[32], prev[32], msg[76];
  SHA256_CTX c;
  SHA256_Init(&c);
  SHA256_Update(&c, "vi-prompt-v1", 12);
  SHA256_Update(&c, prompt, (size_t)prompt_len);
  SHA256_Final(ph, &c);
  SHA256_Init(&c);
  SHA256_Update(&c, "vi-io-genesis-v4", 16);
  SHA256_Update(&c, ph, 32);
  SHA256_Final(prev, &c);
  for (int64_t t = 0; t < n; ++t) {
    memcpy(msg, "vi-io-v4", 8);
    memcpy(msg + 8, leaves + t * 32, 32);
    memcpy(msg + 40, &token_ids[t], 4);
    memcpy(msg + 44, prev, 32);
    SHA256(msg, 76, prev);
    memcpy(io_out + t * 32, prev, 32);
  }
}

/* Raw SHA-256 throughput probe: n messages of len bytes each, on n_threads. */
typedef struct { const uint8_t* buf; int64_t len, n, next; } sha_job;
static void* sha_worker(void* arg) {
  sha_job* j = (sha_job*)arg;
  uint8_t out[32];
  for (;;) {
    const int64_t i = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (i >= j->n) break;
    SHA256(j->buf, (size_t)j->len, out);
  }
  return NULL;
}
void vco_sha_probe(const uint8_t* buf, int64_t len, int64_t n, int n_threads) {
  sha_job j = {buf, len, n, 0};
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)(n_threads > 0 ? n_threads : 1));
  for (int i = 0; i < n_threads; ++i) pthread_create(&th[i], NULL, sha_worker, &j);
  for (int i = 0; i < n_threads; ++i) pthread_join(th[i], NULL);
  free(th);
}

/* compute_kv_transcript (crates/verilm-prover/src/lib.rs:207-329), per-tensor
 * scales or the toy path, on one thread as the reference runs it.  For each
 * position t and layer l: k_acc / v_acc = matmul_i32 (matmul.rs:12-22, one i32
 * dot product per output row), then acc * (sw * sx) (rope.rs:107-112) and, for
 * K, RoPE per head with the C library's cos/sin (rope.rs:38-60); toy path
 * (sw == NULL): clamp to i8 (verilm-core/src/lib.rs:22-24).
 * x: [n_tok][n_layers][hidden]; wk[l], wv[l]: [kv][hidden]; scale_x:
 * [n_tok][n_layers]; sw: [n_layers][2] (K, V) or NULL; inv_freq: [head_dim/2].
 * Outputs [n_layers][n_tok][kv]. */
void vco_kv_transcript(int32_t n_tok, int32_t n_layers, int32_t hidden, int32_t n_heads, int32_t head_dim,
                       const int8_t* x, const int8_t* const* wk, const int8_t* const* wv, const float* scale_x,
                       const float* sw, const double* inv_freq, double* k_out, double* v_out) {
    const int64_t kv = (int64_t)n_heads * head_dim;
    const int half = head_dim / 2;
    double* kf = (double*)malloc(sizeof(double) * kv);
    for (int32_t t = 0; t < n_tok; ++t) {
        for (int32_t l = 0; l < n_layers; ++l) {
            const int8_t* xr = x + ((int64_t)t * n_layers + l) * hidden;
            double* ko = k_out + ((int64_t)l * n_tok + t) * kv;
            double* vo = v_out + ((int64_t)l * n_tok + t) * kv;
            for (int m = 0; m < 2; ++m) {
                const int8_t* w = m ? wv[l] : wk[l];
                double* dst = m ? vo : kf;
                const double scale = sw ? (double)sw[2 * l + m] * (double)scale_x[(int64_t)t * n_layers + l] : 0.0;
                for (int64_t r = 0; r < kv; ++r) {
                    const int8_t* wr = w + r * hidden;
                    int32_t acc = 0;
                    for (int32_t c = 0; c < hidden; ++c) acc += (int32_t)wr[c] * (int32_t)xr[c];
                    if (!sw) dst[r] = (double)(acc < -128 ? -128 : acc > 127 ? 127 : acc);
                    else dst[r] = (double)acc * scale;
                }
            }
            if (!sw) {
                memcpy(ko, kf, sizeof(double) * kv);
                continue;
            }
            for (int h = 0; h < n_heads; ++h) {
                const double* hv = kf + (int64_t)h * head_dim;
                double* o = ko + (int64_t)h * head_dim;
                for (int i = 0; i < half; ++i) {
                    const double a = (double)t * inv_freq[i];
                    const double c = cos(a), s = sin(a);
                    o[i] = hv[i] * c - hv[i + half] * s;
                    o[i + half] = hv[i + half] * c + hv[i] * s;
                }
            }
        }
    }
    free(kf);
}
