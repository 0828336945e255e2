// KV transcript from captured x_attn on the tensor cores:
// compute_kv_transcript (crates/verilm-prover/src/lib.rs:207-329).
//
// For every layer l and position t:
//   k_acc = Wk[l] x_attn[t][l],  v_acc = Wv[l] x_attn[t][l]      (exact i32)
//   value = dequant(acc) (+ bias), K additionally rotated by RoPE (f64)
// A tile is 128 positions x 256 channels of one layer's K or V projection:
// TMA brings 128-byte K-slices of x_attn (A, 128 rows) and of the weight rows
// (B, 256 rows) into shared memory (128-byte swizzle), one thread issues
// tcgen05.mma kind::i8 into a 128 x 256 s32 accumulator in TMEM, and eight
// epilogue warps read it back (one position per thread, two warps per TMEM
// lane quarter) for the f64 values.
// i8 x i8 products summed in s32 are exact in any order, so the accumulators
// equal matmul_i32 (crates/verilm-core/src/matmul.rs:12-22).  The epilogue
// rounds every f64 operation separately (__dmul_rn / __dadd_rn: no fused
// multiply-add), in the reference's order; cos/sin come from a host table.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "tc05.cuh"
#include "vc_internal.h"

namespace vc {

namespace {

constexpr int kBM = 128;       // positions per tile (TMEM lanes)
constexpr int kBN = 256;       // accumulator columns per tile
constexpr int kBK = 128;       // bytes of K per stage (one swizzle row)
constexpr int kStages = 3;
constexpr int kEpiWarps = 8;                   // two per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0: TMA, warp 1: MMA, warps 2-9: epilogue
constexpr uint32_t kStageA = kBM * kBK;
constexpr uint32_t kStageB = kBN * kBK;
constexpr uint32_t kIdesc = tc05::idesc_i8_s32(kBM, kBN);
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int kErrTimeout = 2;
constexpr int kStep = 16;                      // accumulator columns per TMEM load in the epilogue

struct Smem {
  uint8_t a[kStages][kStageA];
  uint8_t b[kStages][kStageB];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t final_mma;
  uint32_t tmem;
  int32_t abort;
};

__device__ __forceinline__ double deq(int32_t acc, int c, const float* ch, double sx, double scale,
                                      const float* bias) {
  double f;
  if (ch)
    f = __dmul_rn(__dmul_rn(double(acc), double(__ldg(ch + c))), sx);  // rope.rs:134-137
  else
    f = __dmul_rn(double(acc), scale);                                 // rope.rs:107-112
  if (bias) f = __dadd_rn(f, double(__ldg(bias + c)));                 // lib.rs:283-302
  return f;
}

__device__ __forceinline__ bool aborted(const Smem& sm) {
  return *reinterpret_cast<const volatile int32_t*>(&sm.abort) != 0;
}

__device__ __forceinline__ void set_abort(Smem& sm, int* err) {
  atomicExch(&sm.abort, 1);
  atomicExch(err, kErrTimeout);
}

struct Tile {
  int layer, m0, mat, c0, nvalid;
};

// Tile order: channels fastest, then positions, then layers, so that the CTAs
// working at one time share one layer's weights and one block of x_attn in L2.
__device__ __forceinline__ Tile tile_of(const KvtArgs& a, int idx) {
  Tile t;
  const int n_tiles_n = 2 * a.tiles_per_mat;
  const int n = idx % n_tiles_n;
  const int rest = idx / n_tiles_n;
  t.m0 = (rest % a.m_tiles) * kBM;
  t.layer = rest / a.m_tiles;
  t.mat = n / a.tiles_per_mat;
  t.c0 = (n % a.tiles_per_mat) * a.tile_cols;
  t.nvalid = min(a.tile_cols, a.kv_dim - t.c0);
  return t;
}

// 32-byte store of four f64 (one full sector per lane); p 32-byte aligned.
__device__ __forceinline__ void st_v4(double* p, const double (&v)[4]) {
  asm volatile("st.global.v4.f64 [%0], {%1, %2, %3, %4};" ::"l"(p), "d"(v[0]), "d"(v[1]), "d"(v[2]), "d"(v[3])
               : "memory");
}

// Dequantisation modes, fixed per tile: toy clamp (lib.rs:307-316), per-tensor
// scale without bias, or per-channel scales and/or bias.
enum { kModeToy = 0, kModeTensor = 1, kModeGeneral = 2 };

template <int MODE>
__device__ __forceinline__ double dq(int32_t acc, int c, const float* ch, double sx, double scale,
                                     const float* bias) {
  if (MODE == kModeToy) return double(min(127, max(-128, acc)));
  if (MODE == kModeTensor) return __dmul_rn(double(acc), scale);
  return deq(acc, c, ch, sx, scale, bias);
}

// Epilogue of one tile for one thread (position pos) of one of the two column
// groups: 16-column steps alternate between the groups.  Every f64 operation
// is rounded on its own, in the reference's order.  head_dim is a multiple of
// 64 here, so the tile holds whole heads and every step is 16 columns of one
// half-head; results leave as 32-byte stores of four consecutive channels.
template <int MODE>
__device__ __forceinline__ void epilogue_fast(const KvtArgs& a, const Tile& t, uint32_t tbase, int group, int pos,
                                              bool valid, double* out, const float* ch, const float* bias, double sx,
                                              double scale) {
  const int half = a.head_dim >> 1;
  if (MODE != kModeToy && t.mat == 0) {
    // K: per head, out[i] = k[i] c - k[i+half] s, out[i+half] = k[i+half] c + k[i] s (rope.rs:48-57)
    int step = 0;
    for (int hb = 0; hb < t.nvalid; hb += a.head_dim) {
      for (int q = 0; q < half; q += kStep, ++step) {
        if ((step & 1) != group) continue;
        uint32_t lo[kStep], hi[kStep];
        tc05::tmem_ld2_wait<kStep>(tbase + hb + q, tbase + hb + half + q, lo, hi);
        if (valid) {
          const double2* cs = a.rope + int64_t(q) * a.rope_rows + pos;
#pragma unroll
          for (int j = 0; j < kStep; j += 4) {
            double olo[4], ohi[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int c = t.c0 + hb + q + j + u;
              const double kl = dq<MODE>(int32_t(lo[j + u]), c, ch, sx, scale, bias);
              const double kh = dq<MODE>(int32_t(hi[j + u]), c + half, ch, sx, scale, bias);
              const double2 w = __ldg(cs + int64_t(j + u) * a.rope_rows);
              olo[u] = __dsub_rn(__dmul_rn(kl, w.x), __dmul_rn(kh, w.y));
              ohi[u] = __dadd_rn(__dmul_rn(kh, w.x), __dmul_rn(kl, w.y));
            }
            st_v4(out + hb + q + j, olo);
            st_v4(out + hb + half + q + j, ohi);
          }
        }
      }
    }
  } else {
    for (int cb = kStep * group; cb < t.nvalid; cb += 2 * kStep) {
      uint32_t r[kStep];
      tc05::tmem_ld_wait<kStep>(tbase + cb, r);
      if (valid) {
#pragma unroll
        for (int j = 0; j < kStep; j += 4) {
          double o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) o[u] = dq<MODE>(int32_t(r[j + u]), t.c0 + cb + j + u, ch, sx, scale, bias);
          st_v4(out + cb + j, o);
        }
      }
    }
  }
}

// One persistent CTA per SM walks the tiles (layer, 128 positions, 256 channels
// of K or V).  Warp 0 streams A/B stages with TMA, warp 1 issues the MMAs into
// one of two TMEM accumulators, warps 2-9 turn the other accumulator into f64
// rows, so the epilogue of one tile overlaps the MMAs of the next.
// FAST: head_dim a multiple of 64 (epilogue_fast); otherwise RoPE pairs are
// read in groups of G columns and stored one f64 at a time.
template <int G, bool FAST>
__global__ void __launch_bounds__(kThreads, 1) kv_transcript_kernel(const KvtArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (a.hidden + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc05::mbar_init(tc05::smem_u32(&sm.full[s]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc05::mbar_init(tc05::smem_u32(&sm.acc_full[b]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.acc_empty[b]), kEpiWarps);
    }
    tc05::mbar_init(tc05::smem_u32(&sm.final_mma), 1);
    sm.abort = 0;
    tc05::mbar_init_fence();
  }
  if (warp == 0) tc05::tmem_alloc(tc05::smem_u32(&sm.tmem), 2 * kBN);
  tc05::fence_before_sync();
  __syncthreads();
  tc05::fence_after_sync();
  const uint32_t tmem = sm.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- TMA producer
      int64_t kb_total = 0;  // stage uses so far (all tiles)
      bool ok = true;
      for (int idx = blockIdx.x; idx < a.n_tiles && ok; idx += gridDim.x) {
        const Tile t = tile_of(a, idx);
        const CUtensorMap* map_a = a.maps + 3 * t.layer;
        const CUtensorMap* map_b = a.maps + 3 * t.layer + 1 + t.mat;
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
          if (aborted(sm)) { ok = false; break; }
          const uint32_t full = tc05::smem_u32(&sm.full[s]);
          tc05::mbar_arrive_expect_tx(full, kStageA + kStageB);
          tc05::tma_load_2d(tc05::smem_u32(sm.a[s]), map_a, kb * kBK, t.m0, full);
          tc05::tma_load_2d(tc05::smem_u32(sm.b[s]), map_b, kb * kBK, t.c0, full);
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
      int it = 0;
      for (int idx = blockIdx.x; idx < a.n_tiles; idx += gridDim.x, ++it) {
        const int buf = it & 1, use = it >> 1;
        if (use > 0 &&
            !tc05::mbar_wait(tc05::smem_u32(&sm.acc_empty[buf]), uint32_t((use - 1) & 1), kWaitLimitNs)) {
          set_abort(sm, a.err);
          break;
        }
        if (aborted(sm)) break;
        tc05::fence_after_sync();
        const uint32_t d = tmem + uint32_t(buf * kBN);
        bool ok = true;
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
          for (int k = 0; k < kBK / 32; ++k) tc05::mma_i8(d, ad + 2 * k, bd + 2 * k, kIdesc, (kb | k) != 0);
          tc05::mma_commit(tc05::smem_u32(&sm.empty[s]));  // frees the stage when these MMAs finish
        }
        if (!ok) break;
        tc05::mma_commit(tc05::smem_u32(&sm.acc_full[buf]));  // accumulator ready for the epilogue
      }
      // every MMA of this thread has finished before the CTA can free TMEM
      tc05::mma_commit(tc05::smem_u32(&sm.final_mma));
      tc05::mbar_wait(tc05::smem_u32(&sm.final_mma), 0, kWaitLimitNs);
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int e = warp - 2;
    const int quarter = warp & 3;  // this warp may read TMEM lanes 32 * quarter .. + 31
    const int group = e >> 2;      // which column steps of the tile (two warps per quarter)
    int it = 0;
    for (int idx = blockIdx.x; idx < a.n_tiles; idx += gridDim.x, ++it) {
      const int buf = it & 1, use = it >> 1;
      bool ok = false;
      if (lane == 0) ok = tc05::mbar_wait(tc05::smem_u32(&sm.acc_full[buf]), uint32_t(use & 1), kWaitLimitNs);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) set_abort(sm, a.err);
        break;
      }
      if (__shfl_sync(0xffffffffu, aborted(sm) ? 1 : 0, 0)) break;
      tc05::fence_after_sync();
      const Tile t = tile_of(a, idx);
      const int pos = t.m0 + 32 * quarter + lane;  // this thread's position
      const bool valid = pos < a.n_tokens;
      const uint32_t tbase = tmem + uint32_t(buf * kBN) + (uint32_t(32 * quarter) << 16);
      double* out_mine = (t.mat ? a.out[1] : a.out[0]) + (int64_t(t.layer) * a.n_tokens + (valid ? pos : 0)) * a.kv_dim + t.c0;
      const KvtLayer& L = a.layers[t.layer];
      const float* ch = t.mat ? L.ch[1] : L.ch[0];
      const float* bias = t.mat ? L.bias[1] : L.bias[0];
      const double sx =
          (a.use_rope && valid) ? double(__ldg(a.scale_x + int64_t(pos) * a.sx_t + int64_t(t.layer) * a.sx_l)) : 0.0;
      const double scale = __dmul_rn(double(t.mat ? L.sw[1] : L.sw[0]), sx);
      const bool rope_k = a.use_rope && t.mat == 0;
      const int half = a.head_dim >> 1;

      if (FAST) {
        if (!a.use_rope)
          epilogue_fast<kModeToy>(a, t, tbase, group, pos, valid, out_mine, ch, bias, sx, scale);
        else if (!ch && !bias)
          epilogue_fast<kModeTensor>(a, t, tbase, group, pos, valid, out_mine, ch, bias, sx, scale);
        else
          epilogue_fast<kModeGeneral>(a, t, tbase, group, pos, valid, out_mine, ch, bias, sx, scale);
      } else {
        if (rope_k) {
          int step = 0;
          for (int hb = 0; hb < t.nvalid; hb += a.head_dim) {
            for (int q = 0; q < half; q += G, ++step) {
              if ((step & 1) != group) continue;
              uint32_t lo[G], hi[G];
              tc05::tmem_ld2_wait<G>(tbase + hb + q, tbase + hb + half + q, lo, hi);
              if (valid) {
                const double2* cs = a.rope + int64_t(q) * a.rope_rows + pos;
#pragma unroll
                for (int j = 0; j < G; ++j) {
                  const int c = t.c0 + hb + q + j;
                  const double kl = deq(int32_t(lo[j]), c, ch, sx, scale, bias);
                  const double kh = deq(int32_t(hi[j]), c + half, ch, sx, scale, bias);
                  const double2 w = __ldg(cs + int64_t(j) * a.rope_rows);
                  out_mine[hb + q + j] = __dsub_rn(__dmul_rn(kl, w.x), __dmul_rn(kh, w.y));
                  out_mine[hb + half + q + j] = __dadd_rn(__dmul_rn(kh, w.x), __dmul_rn(kl, w.y));
                }
              }
            }
          }
        } else {
          for (int cb = 32 * group; cb < t.nvalid; cb += 64) {
            uint32_t r[32];
            tc05::tmem_ld_wait<32>(tbase + cb, r);
            if (valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (cb + j < t.nvalid)
                  out_mine[cb + j] = a.use_rope ? deq(int32_t(r[j]), t.c0 + cb + j, ch, sx, scale, bias)
                                                : double(min(127, max(-128, int32_t(r[j]))));
            }
          }
        }
      }
      // this accumulator may now be overwritten by the MMAs of the tile after next
      tc05::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc05::mbar_arrive(tc05::smem_u32(&sm.acc_empty[buf]));
    }
  }

  tc05::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc05::fence_after_sync();
    tc05::tmem_dealloc(tmem, 2 * kBN);
  }
}

template <int G, bool FAST>
cudaError_t launch_g(const KvtArgs& a, int n_sm, cudaStream_t s) {
  const size_t smem = sizeof(Smem) + 1024;
  const cudaError_t e =
      cudaFuncSetAttribute(kv_transcript_kernel<G, FAST>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const int grid = std::max(1, std::min(a.n_tiles, n_sm));
  kv_transcript_kernel<G, FAST><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

__attribute__((noinline)) void fill_cos(double* out, const std::vector<double>& inv, int64_t n_pos) {
  for (size_t i = 0; i < inv.size(); ++i)
    for (int64_t p = 0; p < n_pos; ++p) out[2 * (int64_t(i) * n_pos + p)] = std::cos(double(p) * inv[i]);
}

__attribute__((noinline)) void fill_sin(double* out, const std::vector<double>& inv, int64_t n_pos) {
  for (size_t i = 0; i < inv.size(); ++i)
    for (int64_t p = 0; p < n_pos; ++p) out[2 * (int64_t(i) * n_pos + p) + 1] = std::sin(double(p) * inv[i]);
}

}  // namespace

int kvt_group_width(int head_dim) {
  const int half = head_dim / 2;
  int g = 32;
  while (g > 1 && half % g) g >>= 1;
  return g;
}

size_t kvt_smem_bytes() { return sizeof(Smem) + 1024; }

// ModelConfig::scaled_inv_freq (crates/verilm-core/src/constants.rs:253-297).
std::vector<double> kvt_inv_freq(int head_dim, double theta, int scaling_type, double factor, double low_ff,
                                 double high_ff, int64_t orig_max_pos) {
  const int half = head_dim / 2;
  std::vector<double> f(half);
  for (int k = 0; k < half; ++k) f[k] = 1.0 / std::pow(theta, double(2 * k) / double(head_dim));
  if (scaling_type == 1) {  // "llama3"
    const double old_ctx = double(orig_max_pos);
    const double low_wl = old_ctx / low_ff;
    const double high_wl = old_ctx / high_ff;
    const double two_pi = 2.0 * 3.141592653589793;  // 2.0 * std::f64::consts::PI, rounded alike
    for (double& x : f) {
      const double wl = two_pi / x;
      if (wl > low_wl) {
        x = x / factor;                                   // low frequency: full scaling
      } else if (!(wl < high_wl)) {
        const double smooth = (old_ctx / wl - low_ff) / (high_ff - low_ff);
        x = x * ((1.0 - smooth) / factor + smooth);       // medium band: interpolation
      }                                                   // high frequency: unchanged
    }
  } else if (scaling_type == 2) {  // "linear"
    for (double& x : f) x = x / factor;
  }
  return f;
}

// (cos, sin) of position * inv_freq[i] for positions [0, n_pos), laid out
// [half][n_pos][2] (a warp's 32 positions are contiguous), with the C
// library's cos and sin (rope.rs:48-52).
void kvt_rope_table(const std::vector<double>& inv, int64_t n_pos, double* out) {
  fill_cos(out, inv, n_pos);
  fill_sin(out, inv, n_pos);
}

// x: [rows][row_stride bytes] int8, tiles of 128 rows x 128 bytes; w: [rows][hidden]
// int8, tiles of 256 rows x 128 bytes.  Both with the 128-byte swizzle and zero fill.
int kvt_encode_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t row_stride,
                   int box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return -1;
  const cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(row_stride)};
  const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : int(r);
}

cudaError_t launch_kv_transcript(const KvtArgs& a, int n_sm, cudaStream_t s) {
  if (a.head_dim % 64 == 0) return launch_g<32, true>(a, n_sm, s);
  switch (kvt_group_width(a.head_dim)) {
    case 1: return launch_g<1, false>(a, n_sm, s);
    case 2: return launch_g<2, false>(a, n_sm, s);
    case 4: return launch_g<4, false>(a, n_sm, s);
    case 8: return launch_g<8, false>(a, n_sm, s);
    case 16: return launch_g<16, false>(a, n_sm, s);
    default: return launch_g<32, false>(a, n_sm, s);
  }
}

}  // namespace vc
