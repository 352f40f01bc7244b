// Row-normalisation variants (declared in norm_variants.h).
//
// Forward and the dx part of the backward run one warp per row (eight rows per 256-thread block,
// grid-stride over rows): a first pass over the row reduces the sum of squares (forward) or
// sum_j x w dy (backward) in fp32, a second pass writes the outputs with 16-byte accesses; the
// second read of the row comes from L1/L2. For every mode the backward is
//     dx = dy (a_n w + b w2) - K_n x,   K_n = f r_n^-3 / d * sum_j x w dy - dr_n / (d r_n)
// with f = 1 (rms), g (taper) or 0 (lagged, whose divisor does not depend on x).
// Weight gradients are column sums: a column pass writes per-row-chunk partials, and a second
// pass adds the partials in chunk order, so the result is the same on every run.
#include <cuda_bf16.h>

#include <cstdint>

#include "../common/host.h"
#include "norm_variants.h"

namespace ttb {
namespace {

constexpr int kWarps = 8;
constexpr int kRowsPerChunk = 64;

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 load_dy(const void* dy, bool f32, long long i4) {
  if (f32) return reinterpret_cast<const float4*>(dy)[i4];
  const uint2 raw = reinterpret_cast<const uint2*>(dy)[i4];
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float row_coef(const NormVariantArgs& a, float r) {
  return a.mode == kNormLagged ? *a.a_dev : (a.mode == kNormTaper ? a.g / r : 1.f / r);
}

__global__ void __launch_bounds__(256) nv_fwd_kernel(NormVariantArgs a, const float* __restrict__ x,
                                                     const float* __restrict__ resid, float alpha,
                                                     __nv_bfloat16* __restrict__ y16, float* __restrict__ y32,
                                                     float* __restrict__ r_out, float* __restrict__ msq_out) {
  const int lane = threadIdx.x % 32;
  const int d4 = a.d / 4;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  const float4* v4 = reinterpret_cast<const float4*>(a.w2);
  for (long long row = blockIdx.x * kWarps + threadIdx.x / 32; row < a.N; row += gridDim.x * kWarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * a.d);
    float ss = 0.f;
    for (int j = lane; j < d4; j += 32) {
      const float4 v = xr[j];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    const float msq = warp_sum(ss) / a.d;
    const float r = sqrtf(msq + a.eps);
    if (lane == 0) {
      if (r_out != nullptr) r_out[row] = r;
      if (msq_out != nullptr) msq_out[row] = msq;
    }
    const float an = row_coef(a, r);
    for (int j = lane; j < d4; j += 32) {
      const float4 v = xr[j], w = w4[j];
      float4 c = make_float4(an * w.x, an * w.y, an * w.z, an * w.w);
      if (a.b != 0.f) {
        const float4 u = v4[j];
        c.x += a.b * u.x; c.y += a.b * u.y; c.z += a.b * u.z; c.w += a.b * u.w;
      }
      float4 y = make_float4(v.x * c.x, v.y * c.y, v.z * c.z, v.w * c.w);
      const long long i4 = row * d4 + j;
      if (y16 != nullptr) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
        uint2 packed;
        packed.x = *reinterpret_cast<const uint32_t*>(&lo);
        packed.y = *reinterpret_cast<const uint32_t*>(&hi);
        reinterpret_cast<uint2*>(y16)[i4] = packed;
      }
      if (y32 != nullptr) {
        if (resid != nullptr) {
          const float4 res = reinterpret_cast<const float4*>(resid)[i4];
          y = make_float4(res.x + alpha * y.x, res.y + alpha * y.y, res.z + alpha * y.z, res.w + alpha * y.w);
        }
        reinterpret_cast<float4*>(y32)[i4] = y;
      }
    }
  }
}

__global__ void __launch_bounds__(256) nv_bwd_dx_kernel(NormVariantArgs a, const void* __restrict__ dy, int dy_f32,
                                                        float dy_scale, const float* __restrict__ x,
                                                        const float* __restrict__ r_row,
                                                        const float* __restrict__ dr_row, float* __restrict__ dx,
                                                        int accumulate) {
  const int lane = threadIdx.x % 32;
  const int d4 = a.d / 4;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  const float4* v4 = reinterpret_cast<const float4*>(a.w2);
  const float f = a.mode == kNormRms ? 1.f : (a.mode == kNormTaper ? a.g : 0.f);
  for (long long row = blockIdx.x * kWarps + threadIdx.x / 32; row < a.N; row += gridDim.x * kWarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * a.d);
    const float r = r_row != nullptr ? r_row[row] : 1.f;
    float k = 0.f;
    if (f != 0.f) {
      float dot = 0.f;
      for (int j = lane; j < d4; j += 32) {
        const float4 v = xr[j], w = w4[j], g = load_dy(dy, dy_f32, row * d4 + j);
        dot += v.x * w.x * g.x + v.y * w.y * g.y + v.z * w.z * g.z + v.w * w.w * g.w;
      }
      const float rinv = 1.f / r;
      k = f * rinv * rinv * rinv / a.d * warp_sum(dot) * dy_scale;
    }
    if (dr_row != nullptr) k -= dr_row[row] / (a.d * r);
    const float an = row_coef(a, r);
    for (int j = lane; j < d4; j += 32) {
      const float4 v = xr[j], w = w4[j];
      float4 g = load_dy(dy, dy_f32, row * d4 + j);
      g = make_float4(g.x * dy_scale, g.y * dy_scale, g.z * dy_scale, g.w * dy_scale);
      float4 c = make_float4(an * w.x, an * w.y, an * w.z, an * w.w);
      if (a.b != 0.f) {
        const float4 u = v4[j];
        c.x += a.b * u.x; c.y += a.b * u.y; c.z += a.b * u.z; c.w += a.b * u.w;
      }
      float4 out = make_float4(g.x * c.x - k * v.x, g.y * c.y - k * v.y, g.z * c.z - k * v.z, g.w * c.w - k * v.w);
      float4* dst = reinterpret_cast<float4*>(dx) + row * d4 + j;
      if (accumulate) {
        const float4 o = *dst;
        out.x += o.x; out.y += o.y; out.z += o.z; out.w += o.w;
      }
      *dst = out;
    }
  }
}

// partial[c][j] = sum over rows of chunk c of dy x a_n (and dy x into partial2 for w2)
__global__ void __launch_bounds__(256) nv_bwd_dw_kernel(NormVariantArgs a, const void* __restrict__ dy, int dy_f32,
                                                        float dy_scale, const float* __restrict__ x,
                                                        const float* __restrict__ r_row, float* __restrict__ part,
                                                        float* __restrict__ part2) {
  const int d4 = a.d / 4;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d4) return;
  const long long n0 = static_cast<long long>(blockIdx.y) * kRowsPerChunk;
  const long long n1 = n0 + kRowsPerChunk < a.N ? n0 + kRowsPerChunk : a.N;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f), s2 = s;
  for (long long n = n0; n < n1; ++n) {
    const float4 v = reinterpret_cast<const float4*>(x)[n * d4 + j];
    const float4 g = load_dy(dy, dy_f32, n * d4 + j);
    const float an = row_coef(a, r_row != nullptr ? r_row[n] : 1.f);
    const float4 p = make_float4(g.x * v.x, g.y * v.y, g.z * v.z, g.w * v.w);
    s.x += an * p.x; s.y += an * p.y; s.z += an * p.z; s.w += an * p.w;
    s2.x += p.x; s2.y += p.y; s2.z += p.z; s2.w += p.w;
  }
  const long long o = static_cast<long long>(blockIdx.y) * d4 + j;
  reinterpret_cast<float4*>(part)[o] = make_float4(s.x * dy_scale, s.y * dy_scale, s.z * dy_scale, s.w * dy_scale);
  if (part2 != nullptr)
    reinterpret_cast<float4*>(part2)[o] =
        make_float4(s2.x * dy_scale * a.b, s2.y * dy_scale * a.b, s2.z * dy_scale * a.b, s2.w * dy_scale * a.b);
}

__global__ void __launch_bounds__(256) nv_colsum_kernel(const float* __restrict__ part, int chunks, int d,
                                                        float* __restrict__ out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += part[static_cast<long long>(c) * d + j];
  out[j] = s;
}

void check_args(const NormVariantArgs& a) {
  TTB_CHECK(a.N > 0 && a.d > 0 && a.d % 4 == 0, "norm variant: need N > 0 and d a positive multiple of 4");
  TTB_CHECK(a.mode == kNormLagged || a.mode == kNormTaper || a.mode == kNormRms, "norm variant: unknown mode");
  TTB_CHECK(a.mode != kNormLagged || a.a_dev != nullptr, "norm variant: the lagged mode needs its scale");
  TTB_CHECK(a.b == 0.f || a.w2 != nullptr, "norm variant: a nonzero b needs w2");
}

int row_grid(int N) {
  const long long blocks = (static_cast<long long>(N) + kWarps - 1) / kWarps;
  const long long cap = 8LL * num_sms();
  return static_cast<int>(blocks < cap ? blocks : cap);
}

}  // namespace

int norm_variant_partials(int N) { return (N + kRowsPerChunk - 1) / kRowsPerChunk; }

void norm_variant_fwd(const NormVariantArgs& a, const float* x, const float* resid, float alpha, void* y16,
                      float* y32, float* r_out, float* msq_out, cudaStream_t stream) {
  check_args(a);
  nv_fwd_kernel<<<row_grid(a.N), 256, 0, stream>>>(a, x, resid, alpha, static_cast<__nv_bfloat16*>(y16), y32, r_out,
                                                   msq_out);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void norm_variant_bwd(const NormVariantArgs& a, const void* dy, bool dy_f32, float dy_scale, const float* x,
                      const float* r_row, const float* dr_row, float* dx, bool dx_accumulate, float* dw, float* dw2,
                      float* partials, cudaStream_t stream) {
  check_args(a);
  TTB_CHECK(a.mode == kNormLagged || r_row != nullptr, "norm variant: the backward needs the forward's r");
  if (dx != nullptr) {
    nv_bwd_dx_kernel<<<row_grid(a.N), 256, 0, stream>>>(a, dy, dy_f32 ? 1 : 0, dy_scale, x, r_row, dr_row, dx,
                                                        dx_accumulate ? 1 : 0);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
  if (dw == nullptr && dw2 == nullptr) return;
  TTB_CHECK(partials != nullptr, "norm variant: weight gradients need partial scratch");
  const int chunks = norm_variant_partials(a.N);
  float* part2 = dw2 != nullptr ? partials + static_cast<long long>(chunks) * a.d : nullptr;
  const dim3 grid((a.d / 4 + 255) / 256, chunks);
  nv_bwd_dw_kernel<<<grid, 256, 0, stream>>>(a, dy, dy_f32 ? 1 : 0, dy_scale, x, r_row, partials, part2);
  TTB_CUDA_CHECK(cudaGetLastError());
  if (dw != nullptr) {
    nv_colsum_kernel<<<(a.d + 255) / 256, 256, 0, stream>>>(partials, chunks, a.d, dw);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
  if (dw2 != nullptr) {
    nv_colsum_kernel<<<(a.d + 255) / 256, 256, 0, stream>>>(part2, chunks, a.d, dw2);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace ttb
