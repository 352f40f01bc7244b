// Row-wise and elementwise kernels: (group) RMSNorm forward/backward with a fused residual-grad
// accumulation, rotary embedding (forward / inverse) on the fused QKV buffer, deterministic
// embedding backward, and the small reductions that finish them.
#include <cuda_bf16.h>

#include "../common/host.h"
#include "../common/sm100.cuh"
#include "rowops.h"

#include <type_traits>

namespace ttb {
namespace {

constexpr int kRowThreads = 256;
constexpr int kVec = 4;
constexpr int kMaxChunks = 8;  // d <= 8192
constexpr int kMaxGroups = 8;

__device__ __forceinline__ float block_sum(float v, float* red) {
  // red: >= 32 floats of shared memory
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x / 32;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 u = *reinterpret_cast<const float4*>(p);
  v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
}

// y = bf16(x * rstd_g * w),  rstd_g = 1/sqrt(mean_{group}(x^2) + eps).  One CTA per row.
__global__ void __launch_bounds__(kRowThreads) rmsnorm_fwd_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 __nv_bfloat16* __restrict__ y,
                                                                 float* __restrict__ rstd, int N, int d, int G,
                                                                 float eps) {
  __shared__ float red[32];
  const int gsize = d / G;
  for (int row = blockIdx.x; row < N; row += gridDim.x) {
    const float* xr = x + static_cast<long long>(row) * d;
    float v[kMaxChunks][4];
    float part[kMaxGroups];
#pragma unroll
    for (int g = 0; g < kMaxGroups; ++g) part[g] = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (c * kRowThreads + threadIdx.x) * kVec;
      if (j < d) {
        load4(xr + j, v[c]);
        const float s = v[c][0] * v[c][0] + v[c][1] * v[c][1] + v[c][2] * v[c][2] + v[c][3] * v[c][3];
        const int g = j / gsize;
#pragma unroll
        for (int q = 0; q < kMaxGroups; ++q)
          if (q == g) part[q] += s;
      }
    }
    float inv[kMaxGroups];
    for (int g = 0; g < G; ++g) {
      const float tot = block_sum(part[g], red);
      inv[g] = rsqrtf(tot / gsize + eps);
    }
    if (threadIdx.x < G) rstd[static_cast<long long>(row) * G + threadIdx.x] = inv[threadIdx.x];
    __nv_bfloat16* yr = y + static_cast<long long>(row) * d;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (c * kRowThreads + threadIdx.x) * kVec;
      if (j < d) {
        const int g = j / gsize;
        float r = inv[0];
#pragma unroll
        for (int q = 1; q < kMaxGroups; ++q)
          if (q == g) r = inv[q];
        float wv[4];
        load4(w + j, wv);
        uint2 o;
        o.x = pack_bf16(v[c][0] * r * wv[0], v[c][1] * r * wv[1]);
        o.y = pack_bf16(v[c][2] * r * wv[2], v[c][3] * r * wv[3]);
        *reinterpret_cast<uint2*>(yr + j) = o;
      }
    }
  }
}

// Backward of y = x * rstd * w (rstd depends on x):
//   g = dy * w;  dx = rstd * (g - xhat * mean_group(g * xhat));  dw += dy * xhat
// dx is added into dres (the fp32 residual-stream gradient) when accumulate != 0, else written.
// dw partial sums per CTA go to dw_part[blockIdx.x][d] (reduced by dw_reduce_kernel).
template <typename TDY>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_bwd_kernel(const TDY* __restrict__ dy,
                                                                 const float* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ rstd,
                                                                 float* __restrict__ dres, int accumulate,
                                                                 float* __restrict__ dw_part, int N, int d, int G,
                                                                 __nv_bfloat16* __restrict__ out16, float scale16) {
  __shared__ float red[32];
  const int gsize = d / G;
  float dw[kMaxChunks][4];
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
    for (int k = 0; k < 4; ++k) dw[c][k] = 0.f;
  for (int row = blockIdx.x; row < N; row += gridDim.x) {
    const long long base = static_cast<long long>(row) * d;
    float xh[kMaxChunks][4], gg[kMaxChunks][4];
    float part[kMaxGroups];
#pragma unroll
    for (int g = 0; g < kMaxGroups; ++g) part[g] = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (c * kRowThreads + threadIdx.x) * kVec;
      if (j < d) {
        const int g = j / gsize;
        const float r = rstd[static_cast<long long>(row) * G + g];
        float xv[4], dv[4], wv[4];
        load4(x + base + j, xv);
        load4(dy + base + j, dv);
        load4(w + j, wv);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          xh[c][k] = xv[k] * r;
          gg[c][k] = dv[k] * wv[k];
          dw[c][k] += dv[k] * xh[c][k];
          s += gg[c][k] * xh[c][k];
        }
#pragma unroll
        for (int q = 0; q < kMaxGroups; ++q)
          if (q == g) part[q] += s;
      }
    }
    float mean[kMaxGroups];
    for (int g = 0; g < G; ++g) mean[g] = block_sum(part[g], red) / gsize;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int j = (c * kRowThreads + threadIdx.x) * kVec;
      if (j < d) {
        const int g = j / gsize;
        const float r = rstd[static_cast<long long>(row) * G + g];
        float m = mean[0];
#pragma unroll
        for (int q = 1; q < kMaxGroups; ++q)
          if (q == g) m = mean[q];
        float4 o;
        o.x = r * (gg[c][0] - xh[c][0] * m);
        o.y = r * (gg[c][1] - xh[c][1] * m);
        o.z = r * (gg[c][2] - xh[c][2] * m);
        o.w = r * (gg[c][3] - xh[c][3] * m);
        float4* dst = reinterpret_cast<float4*>(dres + base + j);
        if (accumulate) {
          const float4 prev = *dst;
          o.x += prev.x; o.y += prev.y; o.z += prev.z; o.w += prev.w;
        }
        *dst = o;
        if (out16 != nullptr)
          *reinterpret_cast<uint2*>(out16 + base + j) =
              make_uint2(pack_bf16(o.x * scale16, o.y * scale16), pack_bf16(o.z * scale16, o.w * scale16));
      }
    }
  }
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int j = (c * kRowThreads + threadIdx.x) * kVec;
    if (j < d)
      *reinterpret_cast<float4*>(dw_part + static_cast<long long>(blockIdx.x) * d + j) =
          make_float4(dw[c][0], dw[c][1], dw[c][2], dw[c][3]);
  }
}

// ---------------------------------------------------------------------------------------------
// Warp-per-row variants for d <= 4096: each lane keeps CH float4 of the row in registers, so the
// row is read once and reduced with shuffles only.  GROUPED=false is plain RMSNorm (one group).
template <bool GROUPED>
__device__ __forceinline__ int group_of(int j, int gsize) {
  return GROUPED ? j / gsize : 0;
}

template <int CH, bool GROUPED>
__global__ void __launch_bounds__(256) rmsnorm_fwd_warp_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                              int N, int d, int G, float eps) {
  constexpr int NG = GROUPED ? kMaxGroups : 1;
  const int lane = threadIdx.x % 32;
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= N) return;
  const int gsize = d / G;
  const bool whole = (CH * 128 == d);
  const float* xr = x + static_cast<long long>(row) * d;
  float v[CH][4];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int j = (c * 32 + lane) * 4;
    if (whole || j < d)
      load4(xr + j, v[c]);
    else
      v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
  }
  float part[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) part[g] = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int j = (c * 32 + lane) * 4;
    const float sq = v[c][0] * v[c][0] + v[c][1] * v[c][1] + v[c][2] * v[c][2] + v[c][3] * v[c][3];
    const int g = group_of<GROUPED>(j, gsize);
#pragma unroll
    for (int q = 0; q < NG; ++q)
      if (q == g) part[q] += sq;
  }
  float inv[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float t = part[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    inv[g] = rsqrtf(t / gsize + eps);
  }
#pragma unroll
  for (int g = 0; g < NG; ++g)
    if (lane == g && g < G) rstd[static_cast<long long>(row) * G + g] = inv[g];
  __nv_bfloat16* yr = y + static_cast<long long>(row) * d;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int j = (c * 32 + lane) * 4;
    if (whole || j < d) {
      const int g = group_of<GROUPED>(j, gsize);
      float r = inv[0];
#pragma unroll
      for (int q = 1; q < NG; ++q)
        if (q == g) r = inv[q];
      float wv[4];
      load4(w + j, wv);
      uint2 o;
      o.x = pack_bf16(v[c][0] * r * wv[0], v[c][1] * r * wv[1]);
      o.y = pack_bf16(v[c][2] * r * wv[2], v[c][3] * r * wv[3]);
      *reinterpret_cast<uint2*>(yr + j) = o;
    }
  }
}

// Two passes over the row (the second re-reads x and dy, which are still in L1) keep the register
// footprint at one row of partial weight gradients, so several CTAs stay resident per SM.
template <int CH, bool GROUPED, typename TDY, bool WITH_DW>
__global__ void __launch_bounds__(256) rmsnorm_bwd_warp_kernel(const TDY* __restrict__ dy, const float* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ rstd, float* __restrict__ dres,
                                                              int accumulate, float* __restrict__ dw_part, int N,
                                                              int d, int G, __nv_bfloat16* __restrict__ out16,
                                                              float scale16) {
  constexpr int NG = GROUPED ? kMaxGroups : 1;
  extern __shared__ float acc[];  // d floats
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32, nw = blockDim.x / 32;
  const int gsize = d / G;
  const bool whole = (CH * 128 == d);
  float dwl[CH][4];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int k = 0; k < 4; ++k) dwl[c][k] = 0.f;
  for (int row = blockIdx.x * nw + wid; row < N; row += gridDim.x * nw) {
    const long long base = static_cast<long long>(row) * d;
    float rg[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) rg[g] = (g < G) ? rstd[static_cast<long long>(row) * G + g] : 0.f;
    float part[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) part[g] = 0.f;
    // pass 1: sum of (dy w) xhat per group; weight-gradient partials
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int j = (c * 32 + lane) * 4;
      if (whole || j < d) {
        const int g = group_of<GROUPED>(j, gsize);
        float r = rg[0];
#pragma unroll
        for (int q = 1; q < NG; ++q)
          if (q == g) r = rg[q];
        float xv[4], dv[4], wv[4];
        load4(x + base + j, xv);
        load4(dy + base + j, dv);
        load4(w + j, wv);
        float sacc = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float xh = xv[k] * r;
          if (WITH_DW) dwl[c][k] += dv[k] * xh;
          sacc += dv[k] * wv[k] * xh;
        }
#pragma unroll
        for (int q = 0; q < NG; ++q)
          if (q == g) part[q] += sacc;
      }
    }
    float mean[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      float t = part[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      mean[g] = t / gsize;
    }
    // pass 2: dx = rstd (dy w - xhat mean)
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int j = (c * 32 + lane) * 4;
      if (whole || j < d) {
        const int g = group_of<GROUPED>(j, gsize);
        float r = rg[0], m = mean[0];
#pragma unroll
        for (int q = 1; q < NG; ++q)
          if (q == g) {
            r = rg[q];
            m = mean[q];
          }
        float xv[4], dv[4], wv[4];
        load4(x + base + j, xv);
        load4(dy + base + j, dv);
        load4(w + j, wv);
        float4 o = make_float4(r * (dv[0] * wv[0] - xv[0] * r * m), r * (dv[1] * wv[1] - xv[1] * r * m),
                               r * (dv[2] * wv[2] - xv[2] * r * m), r * (dv[3] * wv[3] - xv[3] * r * m));
        float4* dst = reinterpret_cast<float4*>(dres + base + j);
        if (accumulate) {
          const float4 prev = *dst;
          o.x += prev.x; o.y += prev.y; o.z += prev.z; o.w += prev.w;
        }
        *dst = o;
        if (out16 != nullptr)
          *reinterpret_cast<uint2*>(out16 + base + j) =
              make_uint2(pack_bf16(o.x * scale16, o.y * scale16), pack_bf16(o.z * scale16, o.w * scale16));
      }
    }
  }
  if (!WITH_DW) return;
  // deterministic CTA reduction: warps add their partials into shared memory in warp order
  for (int ww = 0; ww < nw; ++ww) {
    __syncthreads();
    if (wid == ww) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int j = (c * 32 + lane) * 4;
        if (whole || j < d) {
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[j + k] = (ww == 0 ? 0.f : acc[j + k]) + dwl[c][k];
        }
      }
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) dw_part[static_cast<long long>(blockIdx.x) * d + j] = acc[j];
}

// Single-pass RMSNorm backward for one group (G == 1) and d = 256 * 4 * C: dx, the bf16 copy and the
// weight-gradient partials from ONE read of x and dy.  Thread t owns the float4 chunks t, t + 256,
// ... (every load and store coalesced) and keeps its columns of w and of the partial dw in registers.
// CTA b walks rows b, b + gridDim.x, ... R at a time with all loads of those rows issued before any is
// used; the row sums go through a double-buffered shared array, one barrier per step.  The partial
// row b of dw_part is this CTA's sum over its rows in row order: deterministic.
template <int C, int R, typename TDY>
__global__ void __launch_bounds__(256) rmsnorm_bwd_fused_kernel(const TDY* __restrict__ dy, const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ rstd, float* __restrict__ dres,
                                                               int accumulate, float* __restrict__ dw_part, int N,
                                                               __nv_bfloat16* __restrict__ out16, float scale16) {
  constexpr int d = 256 * 4 * C;
  __shared__ float red[2][R][8];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float wv[C][4], dwl[C][4];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    load4(w + (c * 256 + tid) * 4, wv[c]);
#pragma unroll
    for (int k = 0; k < 4; ++k) dwl[c][k] = 0.f;
  }
  int it = 0;
  for (int row0 = blockIdx.x; row0 < N; row0 += R * gridDim.x, ++it) {
    float xv[R][C][4], dv[R][C][4], pv[R][C][4], r[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = row0 + i * gridDim.x;
      const bool live = row < N;
      const long long base = static_cast<long long>(live ? row : row0) * d;
      r[i] = live ? rstd[live ? row : row0] : 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const long long off = base + (c * 256 + tid) * 4;
        load4(x + off, xv[i][c]);
        load4(dy + off, dv[i][c]);
        if (accumulate) load4(dres + off, pv[i][c]);
      }
    }
    float s[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      s[i] = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k) s[i] += dv[i][c][k] * wv[c][k] * xv[i][c][k];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s[i] += __shfl_xor_sync(0xffffffffu, s[i], o);
      if (lane == 0) red[it & 1][i][wid] = s[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = row0 + i * gridDim.x;
      if (row >= N) break;
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) t += red[it & 1][i][q];
      const float m = t * r[i] / d;  // mean over the row of (dy w) xhat
      const long long base = static_cast<long long>(row) * d;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const long long off = base + (c * 256 + tid) * 4;
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float xh = xv[i][c][k] * r[i];
          o[k] = r[i] * (dv[i][c][k] * wv[c][k] - xh * m) + (accumulate ? pv[i][c][k] : 0.f);
          dwl[c][k] += dv[i][c][k] * xh;
        }
        *reinterpret_cast<float4*>(dres + off) = make_float4(o[0], o[1], o[2], o[3]);
        if (out16 != nullptr)
          *reinterpret_cast<uint2*>(out16 + off) =
              make_uint2(pack_bf16(o[0] * scale16, o[1] * scale16), pack_bf16(o[2] * scale16, o[3] * scale16));
      }
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c)
    *reinterpret_cast<float4*>(dw_part + static_cast<long long>(blockIdx.x) * d + (c * 256 + tid) * 4) =
        make_float4(dwl[c][0], dwl[c][1], dwl[c][2], dwl[c][3]);
}

// out[j] (+)= sum_p part[p][j].  Block = 32 columns x 8 row groups: warp g sums rows p = g, g+8, ...
// in order, then warp 0 adds the 8 group sums in order (a fixed tree: deterministic).
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ part, int P, int d,
                                                     float* __restrict__ out, int accumulate) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x % 32, g = threadIdx.x / 32;
  const int j = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (j < d)
    for (int p = g; p < P; p += 8) s += part[static_cast<long long>(p) * d + j];
  red[g][lane] = s;
  __syncthreads();
  if (g == 0 && j < d) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += red[q][lane];
    out[j] = accumulate ? out[j] + t : t;
  }
}

// Weight-gradient partials of the (group) RMSNorm backward: part[p][j] = sum over the rows of chunk
// p of dy[row][j] * x[row][j] * rstd[row][group(j)].  Threads own 4 consecutive columns and walk
// their chunk's rows in order (coalesced rows, deterministic sums).
template <typename TDY>
__global__ void __launch_bounds__(256) rmsnorm_dw_kernel(const TDY* __restrict__ dy, const float* __restrict__ x,
                                                         const float* __restrict__ rstd, float* __restrict__ part,
                                                         int N, int d, int G, int rows_per_chunk) {
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (j >= d) return;
  const int p = blockIdx.y;
  const int r0 = p * rows_per_chunk;
  const int r1 = min(N, r0 + rows_per_chunk);
  const int g = j / (d / G);
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int row = r0; row < r1; ++row) {
    const long long base = static_cast<long long>(row) * d + j;
    float xv[4], dv[4];
    load4(x + base, xv);
    load4(dy + base, dv);
    const float r = rstd[static_cast<long long>(row) * G + g];
    a0 += dv[0] * xv[0] * r;
    a1 += dv[1] * xv[1] * r;
    a2 += dv[2] * xv[2] * r;
    a3 += dv[3] * xv[3] * r;
  }
  *reinterpret_cast<float4*>(part + static_cast<long long>(p) * d + j) = make_float4(a0, a1, a2, a3);
}

// Rotary embedding on the leading `rope_cols` columns of a [N, ld] bf16 buffer, in place.
// Heads of width dk; pair (i, i + dk/2) of a head is rotated by angle pos * inv_freq[i].
// inverse != 0 rotates by the negative angle (the backward of the forward rotation).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ buf, long long ld, int N, int rope_cols, int dk,
                            const int* __restrict__ pos, const float* __restrict__ inv_freq, int inverse) {
  const int half = dk / 2;
  const long long pairs_per_row = rope_cols / 2;
  const long long total = static_cast<long long>(N) * pairs_per_row;
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(t / pairs_per_row);
    const int pr = static_cast<int>(t % pairs_per_row);
    const int head = pr / half;
    const int i = pr % half;
    const float ang = static_cast<float>(pos[row]) * inv_freq[i];
    float s, c;
    sincosf(ang, &s, &c);
    if (inverse) s = -s;
    __nv_bfloat16* p = buf + row * ld + static_cast<long long>(head) * dk + i;
    const float a = __bfloat162float(p[0]);
    const float b = __bfloat162float(p[half]);
    p[0] = __float2bfloat16_rn(a * c - b * s);
    p[half] = __float2bfloat16_rn(a * s + b * c);
  }
}

// x[t, :] = W[idx[t], :]   (fp32 rows; d multiple of 4).  An id outside [0, V) is recorded in the
// status word and its row is written as zeros instead of being read from outside the table.
__global__ void embed_fwd_kernel(const long long* __restrict__ idx, const float* __restrict__ W,
                                 float* __restrict__ x, int N, int d, long long V, uint32_t* status) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < N; t += gridDim.x * warps) {
    const long long id = idx[t];
    float4* dst = reinterpret_cast<float4*>(x + static_cast<long long>(t) * d);
    if (id < 0 || id >= V) {
      if (lane == 0) record_error(status, kErrBadIndex);
      for (int j = lane; j < d / 4; j += 32) dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    const float4* src = reinterpret_cast<const float4*>(W + id * static_cast<long long>(d));
    for (int j = lane; j < d / 4; j += 32) dst[j] = src[j];
  }
}

// Deterministic embedding backward over tokens sorted by id (stable sort, so equal ids keep
// their original order): the first position of each run sums the run's gradient rows in order.
// Ids outside [0, V) are recorded in the status word and their gradient rows dropped.
__global__ void embed_bwd_kernel(const long long* __restrict__ sorted_ids, const long long* __restrict__ order,
                                 const float* __restrict__ dx, float* __restrict__ dW, int N, int d, long long V,
                                 uint32_t* status) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int s = blockIdx.x * warps + threadIdx.x / 32; s < N; s += gridDim.x * warps) {
    const long long id = sorted_ids[s];
    if (s > 0 && sorted_ids[s - 1] == id) continue;
    if (id < 0 || id >= V) {
      if (lane == 0) record_error(status, kErrBadIndex);
      continue;
    }
    int e = s + 1;
    while (e < N && sorted_ids[e] == id) ++e;
    float* dst = dW + id * static_cast<long long>(d);
    for (int j = lane * 4; j < d; j += 128) {
      float4 acc = *reinterpret_cast<float4*>(dst + j);
      for (int q = s; q < e; ++q) {
        const float4 g = *reinterpret_cast<const float4*>(dx + order[q] * static_cast<long long>(d) + j);
        acc.x += g.x; acc.y += g.y; acc.z += g.z; acc.w += g.w;
      }
      *reinterpret_cast<float4*>(dst + j) = acc;
    }
  }
}

}  // namespace

int rmsnorm_bwd_partials(int N) {
  const int g = 4 * num_sms();
  const int warp_ctas = (N + 7) / 8;
  return warp_ctas < g ? warp_ctas : g;  // one partial row per CTA (8 rows per CTA pass)
}

namespace {
template <typename F>
bool with_chunks(int d, int max_ch, F&& f) {
  const int need = (d + 127) / 128;
  if (need > max_ch) return false;
  if (need <= 1) return f(std::integral_constant<int, 1>{});
  if (need <= 2) return f(std::integral_constant<int, 2>{});
  if (need <= 4) return f(std::integral_constant<int, 4>{});
  if (need <= 6) return f(std::integral_constant<int, 6>{});
  if (need <= 8) return f(std::integral_constant<int, 8>{});
  if (need <= 12) return f(std::integral_constant<int, 12>{});
  if (need <= 16) return f(std::integral_constant<int, 16>{});
  if (need <= 24) return f(std::integral_constant<int, 24>{});
  if (need <= 32) return f(std::integral_constant<int, 32>{});
  return false;
}
}  // namespace

void rmsnorm_fwd(const float* x, const float* w, void* y, float* rstd, int N, int d, int G, float eps,
                 cudaStream_t stream) {
  TTB_CHECK(d % 4 == 0 && d <= kRowThreads * kVec * kMaxChunks, "rmsnorm: d must be a multiple of 4 and <= 8192");
  TTB_CHECK(G >= 1 && G <= kMaxGroups && d % G == 0 && (d / G) % 4 == 0, "rmsnorm: bad group count");
  const bool done = with_chunks(d, 32, [&](auto ch) {
    constexpr int CH = decltype(ch)::value;
    if (G == 1)
      rmsnorm_fwd_warp_kernel<CH, false><<<(N + 7) / 8, 256, 0, stream>>>(x, w, static_cast<__nv_bfloat16*>(y), rstd,
                                                                          N, d, G, eps);
    else
      rmsnorm_fwd_warp_kernel<CH, true><<<(N + 7) / 8, 256, 0, stream>>>(x, w, static_cast<__nv_bfloat16*>(y), rstd,
                                                                         N, d, G, eps);
    return true;
  });
  if (!done) {
    const int grid = N < 8 * num_sms() ? N : 8 * num_sms();
    rmsnorm_fwd_kernel<<<grid, kRowThreads, 0, stream>>>(x, w, static_cast<__nv_bfloat16*>(y), rstd, N, d, G, eps);
  }
  TTB_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(const void* dy, bool dy_f32, const float* x, const float* w, const float* rstd, float* dres,
                 bool accumulate, float* dw_part, float* dw, bool dw_accumulate, int N, int d, int G,
                 cudaStream_t stream) {
  rmsnorm_bwd_ex(dy, dy_f32, x, w, rstd, dres, accumulate, dw_part, dw, dw_accumulate, N, d, G, nullptr, 1.f, stream);
}

void rmsnorm_bwd_ex(const void* dy, bool dy_f32, const float* x, const float* w, const float* rstd, float* dres,
                    bool accumulate, float* dw_part, float* dw, bool dw_accumulate, int N, int d, int G,
                    void* out16_, float scale16, cudaStream_t stream) {
  __nv_bfloat16* out16 = static_cast<__nv_bfloat16*>(out16_);
  TTB_CHECK(d % 4 == 0 && d <= kRowThreads * kVec * kMaxChunks, "rmsnorm: d must be a multiple of 4 and <= 8192");
  const int grid = rmsnorm_bwd_partials(N);
  if (G == 1 && (d == 1024 || d == 2048 || d == 4096)) {
    auto fused = [&](auto c, auto r) {
      constexpr int C = decltype(c)::value, R = decltype(r)::value;
      if (dy_f32)
        rmsnorm_bwd_fused_kernel<C, R, float><<<grid, 256, 0, stream>>>(
            static_cast<const float*>(dy), x, w, rstd, dres, accumulate, dw_part, N, out16, scale16);
      else
        rmsnorm_bwd_fused_kernel<C, R, __nv_bfloat16><<<grid, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(dy), x, w, rstd, dres, accumulate, dw_part, N, out16, scale16);
    };
    if (d == 1024)
      fused(std::integral_constant<int, 1>{}, std::integral_constant<int, 2>{});
    else if (d == 2048)
      fused(std::integral_constant<int, 2>{}, std::integral_constant<int, 2>{});
    else
      fused(std::integral_constant<int, 4>{}, std::integral_constant<int, 1>{});
    TTB_CUDA_CHECK(cudaGetLastError());
    colsum_kernel<<<(d + 31) / 32, 256, 0, stream>>>(dw_part, grid, d, dw, dw_accumulate);
    TTB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const bool done = with_chunks(d, 32, [&](auto ch) {
    constexpr int CH = decltype(ch)::value;
    const size_t smem = static_cast<size_t>(d) * sizeof(float);
    // dx pass without weight-gradient accumulators (low register use, more warps per SM), then a
    // coalesced column-reduction pass for dw into the same [grid, d] partials.
    const int dx_grid = (N + 7) / 8 < 8 * num_sms() ? (N + 7) / 8 : 8 * num_sms();
    auto launch = [&](auto grouped) {
      constexpr bool GR = decltype(grouped)::value;
      if (dy_f32)
        rmsnorm_bwd_warp_kernel<CH, GR, float, false><<<dx_grid, 256, 0, stream>>>(
            static_cast<const float*>(dy), x, w, rstd, dres, accumulate, dw_part, N, d, G, out16, scale16);
      else
        rmsnorm_bwd_warp_kernel<CH, GR, __nv_bfloat16, false><<<dx_grid, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(dy), x, w, rstd, dres, accumulate, dw_part, N, d, G, out16, scale16);
      (void)smem;
    };
    if (G == 1)
      launch(std::false_type{});
    else
      launch(std::true_type{});
    return true;
  });
  if (!done) {
    if (dy_f32)
      rmsnorm_bwd_kernel<float><<<grid, kRowThreads, 0, stream>>>(static_cast<const float*>(dy), x, w, rstd, dres,
                                                                  accumulate, dw_part, N, d, G, out16, scale16);
    else
      rmsnorm_bwd_kernel<__nv_bfloat16><<<grid, kRowThreads, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(dy), x, w, rstd, dres, accumulate, dw_part, N, d, G, out16, scale16);
  }
  TTB_CUDA_CHECK(cudaGetLastError());
  if (done) {
    const int rows_per_chunk = (N + grid - 1) / grid;
    const dim3 dgrid((d / 4 + 255) / 256, grid);
    if (dy_f32)
      rmsnorm_dw_kernel<float><<<dgrid, 256, 0, stream>>>(static_cast<const float*>(dy), x, rstd, dw_part, N, d, G,
                                                          rows_per_chunk);
    else
      rmsnorm_dw_kernel<__nv_bfloat16><<<dgrid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(dy), x, rstd,
                                                                  dw_part, N, d, G, rows_per_chunk);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
  colsum_kernel<<<(d + 31) / 32, 256, 0, stream>>>(dw_part, grid, d, dw, dw_accumulate);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void rope_apply(void* buf, long long ld, int N, int rope_cols, int dk, const int* pos, const float* inv_freq,
                bool inverse, cudaStream_t stream) {
  TTB_CHECK(dk % 2 == 0 && rope_cols % dk == 0, "rope: bad head layout");
  const long long total = static_cast<long long>(N) * (rope_cols / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > 16LL * num_sms()) blocks = 16LL * num_sms();
  if (blocks < 1) blocks = 1;
  rope_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(buf), ld, N, rope_cols, dk,
                                                             pos, inv_freq, inverse ? 1 : 0);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void embed_fwd(const long long* idx, const float* W, float* x, int N, int d, long long V, cudaStream_t stream) {
  TTB_CHECK(d % 4 == 0, "embedding: d must be a multiple of 4");
  const int grid = (N + 7) / 8 < 4 * num_sms() ? (N + 7) / 8 : 4 * num_sms();
  embed_fwd_kernel<<<grid, 256, 0, stream>>>(idx, W, x, N, d, V, status_ptr());
  TTB_CUDA_CHECK(cudaGetLastError());
}

void embed_bwd(const long long* sorted_ids, const long long* order, const float* dx, float* dW, int N, int d,
               long long V, cudaStream_t stream) {
  TTB_CHECK(d % 4 == 0, "embedding: d must be a multiple of 4");
  const int grid = (N + 7) / 8 < 4 * num_sms() ? (N + 7) / 8 : 4 * num_sms();
  embed_bwd_kernel<<<grid, 256, 0, stream>>>(sorted_ids, order, dx, dW, N, d, V, status_ptr());
  TTB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ttb
