// KV transcript from captured x_attn on the tensor cores:
// compute_kv_transcript (crates/verilm-prover/src/lib.rs:207-329).
//
// For every layer l and position t:
//   k_acc = Wk[l] x_attn[t][l],  v_acc = Wv[l] x_attn[t][l]      (exact i32)
//   value = dequant(acc) (+ bias), K additionally rotated by RoPE (f64)
// One CTA computes a 128-position x 256-channel tile of one layer's K or V
// projection: TMA brings 128-byte K-slices of x_attn (A, 128 rows) and of the
// weight rows (B, 256 rows) into shared memory (128-byte swizzle), one thread
// issues tcgen05.mma kind::i8 into a 128 x 256 s32 accumulator in TMEM, and
// the four warps read it back (one position per thread) for the f64 epilogue.
// i8 x i8 products summed in s32 are exact in any order, so the accumulators
// equal matmul_i32 (crates/verilm-core/src/matmul.rs:12-22).  The epilogue
// rounds every f64 operation separately (__dmul_rn / __dadd_rn: no fused
// multiply-add), in the reference's order; cos/sin come from a host table.
#include <cuda.h>

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
constexpr int kStages = 2;
constexpr int kThreads = 128;
constexpr uint32_t kStageA = kBM * kBK;
constexpr uint32_t kStageB = kBN * kBK;
constexpr uint32_t kIdesc = tc05::idesc_i8_s32(kBM, kBN);
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait
constexpr int kErrTimeout = 2;

struct Smem {
  uint8_t a[kStages][kStageA];
  uint8_t b[kStages][kStageB];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t done;
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

// G: columns per TMEM load in the RoPE epilogue = largest power of two <= 32
// dividing head_dim / 2.
template <int G>
__global__ void __launch_bounds__(kThreads, 1) kv_transcript_kernel(const KvtArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int layer = blockIdx.z;
  const int m0 = blockIdx.y * kBM;
  const int mat = blockIdx.x / a.tiles_per_mat;                 // 0 = K, 1 = V
  const int c0 = (blockIdx.x % a.tiles_per_mat) * a.tile_cols;  // first channel of the tile
  const int nvalid = min(a.tile_cols, a.kv_dim - c0);
  const int nk = (a.hidden + kBK - 1) / kBK;
  const CUtensorMap* map_a = a.maps + 3 * layer;
  const CUtensorMap* map_b = a.maps + 3 * layer + 1 + mat;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc05::mbar_init(tc05::smem_u32(&sm.full[s]), 1);
      tc05::mbar_init(tc05::smem_u32(&sm.empty[s]), 1);
    }
    tc05::mbar_init(tc05::smem_u32(&sm.done), 1);
    sm.abort = 0;
    tc05::mbar_init_fence();
  }
  if (warp == 0) tc05::tmem_alloc(tc05::smem_u32(&sm.tmem), kBN);
  tc05::fence_before_sync();
  __syncthreads();
  tc05::fence_after_sync();
  const uint32_t tmem = sm.tmem;

  if (warp == 0 && lane == 0) {
    // producer: one stage = A[128 x 128 B] + B[256 x 128 B]
    tc05::tensormap_acquire(map_a);
    tc05::tensormap_acquire(map_b);
    int issued = 0;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages, u = kb / kStages;
      if (u > 0 && !tc05::mbar_wait(tc05::smem_u32(&sm.empty[s]), (u - 1) & 1, kWaitLimitNs)) {
        ok = false;
        break;
      }
      if (*reinterpret_cast<volatile int32_t*>(&sm.abort)) break;
      const uint32_t full = tc05::smem_u32(&sm.full[s]);
      tc05::mbar_arrive_expect_tx(full, kStageA + kStageB);
      tc05::tma_load_2d(tc05::smem_u32(sm.a[s]), map_a, kb * kBK, m0, full);
      tc05::tma_load_2d(tc05::smem_u32(sm.b[s]), map_b, kb * kBK, c0, full);
      issued = kb + 1;
    }
    if (!ok) {
      atomicExch(&sm.abort, 1);
      atomicExch(a.err, kErrTimeout);
      // let the copies already issued land before the CTA can exit
      for (int kb = max(0, issued - kStages); kb < issued; ++kb)
        tc05::mbar_wait(tc05::smem_u32(&sm.full[kb % kStages]), (kb / kStages) & 1, kWaitLimitNs);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: 4 x (128 x 256 x 32) per stage
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages, u = kb / kStages;
      if (!tc05::mbar_wait(tc05::smem_u32(&sm.full[s]), u & 1, kWaitLimitNs) ||
          *reinterpret_cast<volatile int32_t*>(&sm.abort)) {
        atomicExch(&sm.abort, 1);
        atomicExch(a.err, kErrTimeout);
        break;
      }
      tc05::fence_after_sync();
      const uint64_t ad = tc05::sw128_kmajor_desc(tc05::smem_u32(sm.a[s]));
      const uint64_t bd = tc05::sw128_kmajor_desc(tc05::smem_u32(sm.b[s]));
#pragma unroll
      for (int k = 0; k < kBK / 32; ++k)
        tc05::mma_i8(tmem, ad + 2 * k, bd + 2 * k, kIdesc, (kb | k) != 0);
      tc05::mma_commit(tc05::smem_u32(&sm.empty[s]));  // frees the stage when these MMAs finish
    }
    tc05::mma_commit(tc05::smem_u32(&sm.done));        // all MMAs of this thread finished
  }
  __syncwarp();

  // epilogue: thread = TMEM lane = position m0 + 32 warp + lane
  bool ok = false;
  if (lane == 0) ok = tc05::mbar_wait(tc05::smem_u32(&sm.done), 0, kWaitLimitNs);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok && lane == 0) atomicExch(a.err, kErrTimeout);
  tc05::fence_after_sync();
  ok = ok && !*reinterpret_cast<volatile int32_t*>(&sm.abort);
  ok = __shfl_sync(0xffffffffu, ok, 0);

  if (ok) {
    const int t = m0 + warp * 32 + lane;
    const bool valid = t < a.n_tokens;
    const uint32_t tbase = tmem + (uint32_t(warp * 32) << 16);
    double* out = (mat ? a.out[1] : a.out[0]) + (int64_t(layer) * a.n_tokens + (valid ? t : 0)) * a.kv_dim + c0;
    if (!a.use_rope) {
      // toy path: requantize (clamp to i8), as f64 (lib.rs:307-316; verilm-core/src/lib.rs:22-24)
      for (int cb = 0; cb < nvalid; cb += 32) {
        uint32_t r[32];
        tc05::tmem_ld_wait<32>(tbase + cb, r);
        if (valid) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (cb + j < nvalid) out[cb + j] = double(min(127, max(-128, int32_t(r[j]))));
        }
      }
    } else {
      const KvtLayer& L = a.layers[layer];
      const float* ch = mat ? L.ch[1] : L.ch[0];
      const float* bias = mat ? L.bias[1] : L.bias[0];
      const double sx = valid ? double(__ldg(a.scale_x + int64_t(t) * a.sx_t + int64_t(layer) * a.sx_l)) : 0.0;
      const double scale = __dmul_rn(double(mat ? L.sw[1] : L.sw[0]), sx);
      if (mat == 1) {
        for (int cb = 0; cb < nvalid; cb += 32) {
          uint32_t r[32];
          tc05::tmem_ld_wait<32>(tbase + cb, r);
          if (valid) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cb + j < nvalid) out[cb + j] = deq(int32_t(r[j]), c0 + cb + j, ch, sx, scale, bias);
          }
        }
      } else {
        // K: per head, out[i] = k[i] c - k[i+half] s, out[i+half] = k[i+half] c + k[i] s
        // (rope.rs:48-57); the tile holds whole heads.
        const int half = a.head_dim >> 1;
        const double2* cs_row = a.rope + int64_t(valid ? t : 0) * half;
        for (int hb = 0; hb < nvalid; hb += a.head_dim) {
          for (int q = 0; q < half; q += G) {
            uint32_t lo[G], hi[G];
            tc05::tmem_ld2_wait<G>(tbase + hb + q, tbase + hb + half + q, lo, hi);
            if (valid) {
#pragma unroll
              for (int j = 0; j < G; ++j) {
                const int c = c0 + hb + q + j;
                const double kl = deq(int32_t(lo[j]), c, ch, sx, scale, bias);
                const double kh = deq(int32_t(hi[j]), c + half, ch, sx, scale, bias);
                const double2 w = cs_row[q + j];
                out[hb + q + j] = __dsub_rn(__dmul_rn(kl, w.x), __dmul_rn(kh, w.y));
                out[hb + half + q + j] = __dadd_rn(__dmul_rn(kh, w.x), __dmul_rn(kl, w.y));
              }
            }
          }
        }
      }
    }
  }

  tc05::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc05::fence_after_sync();
    tc05::tmem_dealloc(tmem, kBN);
  }
}

template <int G>
cudaError_t launch_g(const KvtArgs& a, int n_layers, cudaStream_t s) {
  const size_t smem = sizeof(Smem) + 1024;
  const cudaError_t e =
      cudaFuncSetAttribute(kv_transcript_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid(2 * a.tiles_per_mat, (a.n_tokens + kBM - 1) / kBM, n_layers);
  kv_transcript_kernel<G><<<grid, kThreads, smem, s>>>(a);
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
  const size_t h = inv.size();
  for (int64_t p = 0; p < n_pos; ++p)
    for (size_t i = 0; i < h; ++i) out[2 * (p * h + i)] = std::cos(double(p) * inv[i]);
}

__attribute__((noinline)) void fill_sin(double* out, const std::vector<double>& inv, int64_t n_pos) {
  const size_t h = inv.size();
  for (int64_t p = 0; p < n_pos; ++p)
    for (size_t i = 0; i < h; ++i) out[2 * (p * h + i) + 1] = std::sin(double(p) * inv[i]);
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

// (cos, sin) of position * inv_freq[i] for positions [0, n_pos), interleaved
// [n_pos][half][2], with the C library's cos and sin (rope.rs:48-52).
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

cudaError_t launch_kv_transcript(const KvtArgs& a, int n_layers, cudaStream_t s) {
  switch (kvt_group_width(a.head_dim)) {
    case 1: return launch_g<1>(a, n_layers, s);
    case 2: return launch_g<2>(a, n_layers, s);
    case 4: return launch_g<4>(a, n_layers, s);
    case 8: return launch_g<8>(a, n_layers, s);
    case 16: return launch_g<16>(a, n_layers, s);
    default: return launch_g<32>(a, n_layers, s);
  }
}

}  // namespace vc
