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



// Persistent kernels take tiles from a device counter pair {next, finished CTAs}.  Thread 0 of each
// CTA calls this after its final barrier; the last CTA to finish returns both counters to zero for
// the next launch, so launches of one kernel must be ordered on a stream (they are: one compute
// stream per device).
__device__ __forceinline__ void sched_finish(unsigned int* sched) {
  __threadfence();
  if (atomicAdd(sched + 1, 1u) == gridDim.x - 1) {
    atomicExch(sched, 0u);
    atomicExch(sched + 1, 0u);
  }
}

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

__device__ __forceinline__ void store32_scaled(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(dst + q * 8) = u;
  }
}

// Drain one accumulator row of width W from TMEM (columns tacc..tacc+W) to global bf16 memory,
// scaled by `scale`, 16 columns at a time (few live registers: the epilogue warps run at the launch
// register count while the tensor pipe works on the next tile).
template <int W>
__device__ __forceinline__ void store_row_lean(uint32_t tacc, __nv_bfloat16* dst, bool valid, float scale) {
#pragma unroll 1
  for (int cc = 0; cc < W / 16; ++cc) {
    uint32_t a[16];
    tmem_ld16(tacc + cc * 16, a);
    tmem_ld_wait();
    if (valid) {
      uint32_t u[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        u[q] = pack_bf16(__uint_as_float(a[2 * q]) * scale, __uint_as_float(a[2 * q + 1]) * scale);
      *reinterpret_cast<uint4*>(dst + cc * 16) = make_uint4(u[0], u[1], u[2], u[3]);
      *reinterpret_cast<uint4*>(dst + cc * 16 + 8) = make_uint4(u[4], u[5], u[6], u[7]);
    }
  }
}

// Rotary tables of one row, 16 pairs (chunk cc) at a time.
__device__ __forceinline__ void rope_fetch16(const float* ct, const float* st, int cc, float (&cs)[16],
                                             float (&sn)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(ct + cc * 16) + q);
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(st + cc * 16) + q);
    cs[q * 4 + 0] = c4.x; cs[q * 4 + 1] = c4.y; cs[q * 4 + 2] = c4.z; cs[q * 4 + 3] = c4.w;
    sn[q * 4 + 0] = s4.x; sn[q * 4 + 1] = s4.y; sn[q * 4 + 2] = s4.z; sn[q * 4 + 3] = s4.w;
  }
}

// Drain N accumulator rows of width W that share one position (dQ1/dQ2, or dK1/dK2), rotating the
// pairs (i, i + W/2) back: g1 = a cos + b sin, g2 = -a sin + b cos.  On entry cs/sn hold chunk 0 of
// the row's tables (fetched before the accumulators were ready); each step fetches the next chunk
// before draining the current one, so the table latency overlaps TMEM loads and stores.
template <int W, int N>
__device__ __forceinline__ void store_rows_rope(const uint32_t (&tacc)[N], __nv_bfloat16* const (&dst)[N], bool valid,
                                                float scale, const float* ct, const float* st, float (&cs)[16],
                                                float (&sn)[16]) {
#pragma unroll 1
  for (int cc = 0; cc < W / 32; ++cc) {
    float ncs[16], nsn[16];
    if (cc + 1 < W / 32) rope_fetch16(ct, st, cc + 1, ncs, nsn);
#pragma unroll
    for (int n = 0; n < N; ++n) {
      uint32_t a[16], b[16];
      tmem_ld16(tacc[n] + cc * 16, a);
      tmem_ld16(tacc[n] + W / 2 + cc * 16, b);
      tmem_ld_wait();
      if (valid) {
        uint32_t g1[8], g2[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float x1 = __uint_as_float(a[e]) * scale, x2 = __uint_as_float(b[e]) * scale;
          const float y1 = __uint_as_float(a[e + 1]) * scale, y2 = __uint_as_float(b[e + 1]) * scale;
          g1[e / 2] = pack_bf16(x1 * cs[e] + x2 * sn[e], y1 * cs[e + 1] + y2 * sn[e + 1]);
          g2[e / 2] = pack_bf16(x2 * cs[e] - x1 * sn[e], y2 * cs[e + 1] - y1 * sn[e + 1]);
        }
        __nv_bfloat16* d = dst[n];
        *reinterpret_cast<uint4*>(d + cc * 16) = make_uint4(g1[0], g1[1], g1[2], g1[3]);
        *reinterpret_cast<uint4*>(d + cc * 16 + 8) = make_uint4(g1[4], g1[5], g1[6], g1[7]);
        *reinterpret_cast<uint4*>(d + W / 2 + cc * 16) = make_uint4(g2[0], g2[1], g2[2], g2[3]);
        *reinterpret_cast<uint4*>(d + W / 2 + cc * 16 + 8) = make_uint4(g2[4], g2[5], g2[6], g2[7]);
      }
    }
    if (cc + 1 < W / 32) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        cs[e] = ncs[e];
        sn[e] = nsn[e];
      }
    }
  }
}

}  // namespace attn
}  // namespace ttb
