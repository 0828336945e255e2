// Integer-ALU peak probe: register-only loops of 32-bit funnel shifts,
// 3-input logic ops and adds, with 8 independent chains per thread so that
// throughput, not latency, bounds them.  The SHA-256 mix reproduces one
// compression round's operation counts (6 rotates, 4 LOP3, 4 adds): the
// denominator of the hash roofline.
#include <cstdint>

#include "tc05.cuh"
#include "vc_internal.h"

namespace vc {

__device__ __forceinline__ uint32_t shf_r(uint32_t x, uint32_t n) {
  uint32_t r;
  asm("shf.r.wrap.b32 %0, %1, %1, %2;" : "=r"(r) : "r"(x), "r"(n));
  return r;
}
template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return r;
}

constexpr int kChains = 8;
constexpr int kPeakThreads = 256;

template <int V>
__global__ void __launch_bounds__(kPeakThreads) int_peak_kernel(int64_t iters, uint32_t rot, uint32_t* sink) {
  uint32_t a[kChains], b[kChains], c[kChains], d[kChains];
  const uint32_t seed = blockIdx.x * kPeakThreads + threadIdx.x;
#pragma unroll
  for (int j = 0; j < kChains; ++j) {
    a[j] = seed * 0x9E3779B9u + j;
    b[j] = a[j] ^ 0x85EBCA6Bu;
    c[j] = a[j] + 0xC2B2AE35u;
    d[j] = a[j] * 3u;
  }
  // Rotation counts come from a kernel argument so that nothing folds.
  const uint32_t r1 = rot, r2 = rot + 5, r3 = rot + 19, r4 = rot - 4, r5 = rot + 7, r6 = rot + 16;
  for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
    for (int j = 0; j < kChains; ++j) {
      if (V == 0) {
        // One SHA-256 round's operations: 6 SHF, 4 LOP3, 4 adds.
        const uint32_t s1 = lop3<0x96>(shf_r(a[j], r1), shf_r(a[j], r2), shf_r(a[j], r3));
        const uint32_t s0 = lop3<0x96>(shf_r(b[j], r4), shf_r(b[j], r5), shf_r(b[j], r6));
        const uint32_t ch = lop3<0xCA>(a[j], b[j], c[j]);
        const uint32_t mj = lop3<0xE8>(b[j], c[j], d[j]);
        uint32_t t1 = d[j] + s1 + ch;
        t1 = t1 + c[j] + 0x428a2f98u;
        const uint32_t na = t1 + s0 + mj;
        const uint32_t nc = b[j] + t1;
        d[j] = c[j];
        c[j] = nc;
        b[j] = a[j];
        a[j] = na;
      } else if (V == 1) {
#pragma unroll
        for (int k = 0; k < 14; ++k) a[j] = shf_r(a[j], r1 + k);
      } else if (V == 2) {
#pragma unroll
        for (int k = 0; k < 14; ++k) {
          const uint32_t n = lop3<0x96>(a[j], b[j], c[j]);
          c[j] = b[j];
          b[j] = a[j];
          a[j] = n;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 14; ++k) {
          const uint32_t n = a[j] + b[j] + c[j];
          c[j] = b[j];
          b[j] = a[j];
          a[j] = n;
        }
      }
    }
  }
  uint32_t x = 0;
#pragma unroll
  for (int j = 0; j < kChains; ++j) x ^= a[j] ^ b[j] ^ c[j] ^ d[j];
  sink[seed] = x;
}

cudaError_t launch_int_peak(int variant, int64_t iters, int n_sm, uint32_t* sink, cudaStream_t s,
                            double* ops_per_launch) {
  const int blocks = n_sm * 4;  // 1024 resident threads per SM
  switch (variant) {
    case 0: int_peak_kernel<0><<<blocks, kPeakThreads, 0, s>>>(iters, 6u, sink); break;
    case 1: int_peak_kernel<1><<<blocks, kPeakThreads, 0, s>>>(iters, 6u, sink); break;
    case 2: int_peak_kernel<2><<<blocks, kPeakThreads, 0, s>>>(iters, 6u, sink); break;
    default: int_peak_kernel<3><<<blocks, kPeakThreads, 0, s>>>(iters, 6u, sink); break;
  }
  *ops_per_launch = double(blocks) * kPeakThreads * double(iters) * kChains * 14.0;
  return cudaGetLastError();
}

// The library's bounded wait with nothing to wait for: one thread waits on an
// mbarrier that no thread arrives at.  The wait gives up after limit_ns of
// %globaltimer and sets the context's error flag to 2, as every bounded wait of
// the commit kernels does; the kernel then returns normally.
__global__ void wait_probe_kernel(uint64_t limit_ns, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) tc05::mbar_init(tc05::smem_u32(&bar), 1);
  __syncthreads();
  if (threadIdx.x == 0 && !tc05::mbar_wait(tc05::smem_u32(&bar), 0, limit_ns)) atomicExch(err, 2);
}

cudaError_t launch_wait_probe(uint64_t limit_ns, int* err, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(limit_ns, err);
  return cudaGetLastError();
}

}  // namespace vc
