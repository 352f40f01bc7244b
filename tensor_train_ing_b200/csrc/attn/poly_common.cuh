// Shared pieces of the tcgen05 polynomial-attention kernels.
//
// Layout contract: q1, k1, q2, k2, v live in one token-major bf16 buffer qkv[B*T, ld]; the
// columns of head h of projection p start at col_p + h*d.  Every operand tile is a TMA box of
// 64 feature columns (one 128-byte swizzle row) x R token rows, so a tile is both the K-major
// operand "rows x features" and the MN-major operand "features x rows" of the tensor core.
#pragma once

#include "../common/sm100.cuh"
#include "params.h"

namespace ttb {
namespace attn {



// A(s1, s2) for the three polynomial kinds
template <int KIND>
__device__ __forceinline__ float poly(float s1, float s2, const float (&c)[4]) {
  if (KIND == 0) return s1 * s2;
  if (KIND == 1) {
    const float t = s1 + c[0];
    return t * t;
  }
  return c[0] + c[1] * s1 + c[2] * s2 + c[3] * s1 * s2;
}

// K-major SW128 descriptor for a tile made of 64-column boxes of `rows` rows, at K-step k (16 elems).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int rows, int k) {
  return smem_desc(base + (k >> 2) * rows * 128 + (k & 3) * 32, 16, 1024, 2);
}
// MN-major SW128 descriptor: MN atoms are the 64-column boxes (rows*128 bytes apart), K = rows.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int rows, int k) {
  return smem_desc(base + k * 2048, rows * 128, 1024, 2);
}

}  // namespace attn
}  // namespace ttb
