// Multipliers for the pipe-balanced SHA-256 compression (sha256_bal.cuh):
// one, and 2^(32-n) for each rotate/shift amount n of the round and schedule
// functions.  They reach the kernels as a parameter, so the compiler cannot
// see their values and fold the IMAD forms back into ALU shifts and adds.
#pragma once
#include <cstdint>

namespace vc {

struct Opq {
  uint32_t one;
  uint32_t m2, m13, m22;    // Sigma0: rotr 2, 13, 22
  uint32_t m6, m11, m25;    // Sigma1: rotr 6, 11, 25
  uint32_t m7, m18, m3;     // sigma0: rotr 7, 18, shr 3
  uint32_t m17, m19, m10;   // sigma1: rotr 17, 19, shr 10
};

inline Opq make_opq() {
  Opq o;
  o.one = 1;
  o.m2 = 1u << 30; o.m13 = 1u << 19; o.m22 = 1u << 10;
  o.m6 = 1u << 26; o.m11 = 1u << 21; o.m25 = 1u << 7;
  o.m7 = 1u << 25; o.m18 = 1u << 14; o.m3 = 1u << 29;
  o.m17 = 1u << 15; o.m19 = 1u << 13; o.m10 = 1u << 22;
  return o;
}

}  // namespace vc
