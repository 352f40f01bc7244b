// Spectral (sigma-reparameterised) linear maps W_eff = gamma * W / s, s = max(|u^T W v|, floor):
//
//   spectral_cast        sigma = u^T W v and bf16(W_eff), the operand the GEMMs read
//   spectral_grad        dW = (gamma / s) dW_eff - k u v^T,  dgamma = <dW_eff, W> / s,
//                        k = gamma sign(sigma) <dW_eff, W> / s^2 (0 while |sigma| < floor)
//   spectral_power_step  v <- W^T u / |W^T u|, then u <- W v / |W v|; a vector whose norm is not
//                        finite or at most `floor` keeps its previous value
//
// Every reduction is written as per-block partials that a later pass adds in block order, so the
// results are identical from run to run. Row dot products take one warp per row with 16-byte
// loads; W^T u takes column blocks over row chunks.
#include <cuda_bf16.h>

#include <cstdint>

#include "../common/host.h"
#include "spectral.h"

namespace ttb {
namespace {

constexpr int kWarps = 8;
constexpr int kRowChunk = 64;

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over warps of a 256-thread block, written by thread 0 (fixed order).
__device__ __forceinline__ void block_partial(float v, float* red, float* out) {
  v = warp_sum(v);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < kWarps; ++w) s += red[w];
    *out = s;
  }
}

__device__ __forceinline__ float ordered_sum(const float* __restrict__ part, int n, float* red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += part[i];
  s = warp_sum(s);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kWarps; ++w) t += red[w];
  return t;
}

// part[b] = sum over the rows block b handles of  scale_i * (A_i . B_i)   (A, B rows of length cols)
// with scale_i = u[i] (or 1 when u is null); B is a matrix when b_ld > 0, else the vector `vec`.
__global__ void __launch_bounds__(256) row_dot_partials(const float* __restrict__ A, long long a_ld,
                                                        const float* __restrict__ B, long long b_ld,
                                                        const float* __restrict__ vec, const float* __restrict__ u,
                                                        int rows, int cols, float* __restrict__ part) {
  __shared__ float red[kWarps];
  const int lane = threadIdx.x % 32;
  float acc = 0.f;
  for (int row = blockIdx.x * kWarps + threadIdx.x / 32; row < rows; row += gridDim.x * kWarps) {
    const float4* a = reinterpret_cast<const float4*>(A + row * a_ld);
    const float4* b = reinterpret_cast<const float4*>(b_ld > 0 ? B + row * b_ld : vec);
    float s = 0.f;
    for (int j = lane; j < cols / 4; j += 32) {
      const float4 x = a[j], y = b[j];
      s += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    }
    acc += (u != nullptr ? u[row] : 1.f) * s;
  }
  block_partial(acc, red, part + blockIdx.x);
}

__global__ void __launch_bounds__(256) cast_kernel(const float* __restrict__ W, int rows, int cols,
                                                   const float* __restrict__ gamma, const float* __restrict__ part,
                                                   int n_part, float floor_, float* __restrict__ sigma_out,
                                                   __nv_bfloat16* __restrict__ out, long long ld) {
  __shared__ float red[kWarps];
  const float sigma = ordered_sum(part, n_part, red);
  if (blockIdx.x == 0 && threadIdx.x == 0) *sigma_out = sigma;
  const float s = fabsf(sigma) > floor_ ? fabsf(sigma) : floor_;
  const float coef = *gamma / s;
  const long long n4 = static_cast<long long>(rows) * cols / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = 4 * i, r = e / cols, c = e % cols;
    const float4 w = reinterpret_cast<const float4*>(W)[i];
    const __nv_bfloat162 lo = __floats2bfloat162_rn(w.x * coef, w.y * coef), hi = __floats2bfloat162_rn(w.z * coef, w.w * coef);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&lo);
    packed.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + r * ld + c) = packed;
  }
}

__global__ void __launch_bounds__(256) grad_kernel(const float* __restrict__ dWe, long long ld, const float* __restrict__ W,
                                                   int rows, int cols, const float* __restrict__ gamma,
                                                   const float* __restrict__ u, const float* __restrict__ v,
                                                   const float* __restrict__ sigma_p, const float* __restrict__ part,
                                                   int n_part, float floor_, float* __restrict__ dW,
                                                   float* __restrict__ dgamma) {
  __shared__ float red[kWarps];
  const float dot = ordered_sum(part, n_part, red);
  const float sigma = *sigma_p;
  const bool live = fabsf(sigma) >= floor_;
  const float s = live ? fabsf(sigma) : floor_;
  const float g = *gamma;
  const float coef = g / s;
  const float k = live ? g * (sigma > 0.f ? 1.f : (sigma < 0.f ? -1.f : 0.f)) * dot / (s * s) : 0.f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *dgamma = dot / s;
  const long long n4 = static_cast<long long>(rows) * cols / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = 4 * i, r = e / cols, c = e % cols;
    const float4 g4 = *reinterpret_cast<const float4*>(dWe + r * ld + c);
    const float4 vv = *reinterpret_cast<const float4*>(v + c);
    const float ku = k * u[r];
    reinterpret_cast<float4*>(dW)[i] =
        make_float4(coef * g4.x - ku * vv.x, coef * g4.y - ku * vv.y, coef * g4.z - ku * vv.z, coef * g4.w - ku * vv.w);
  }
}

// part[chunk][j] = sum over the chunk's rows of W[i, j] u[i]
__global__ void __launch_bounds__(256) col_partials(const float* __restrict__ W, int rows, int cols,
                                                    const float* __restrict__ u, float* __restrict__ part) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= cols) return;
  const int r0 = blockIdx.y * kRowChunk, r1 = min(r0 + kRowChunk, rows);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += W[static_cast<long long>(r) * cols + j] * u[r];
  part[static_cast<long long>(blockIdx.y) * cols + j] = s;
}

// One block: t[j] = sum_c part[c][j] (n_chunks > 0) or t = part itself; vec <- t / |t| unless |t|
// is not finite or at most floor.
__global__ void __launch_bounds__(256) normalize_into(const float* __restrict__ part, int n_chunks, int n,
                                                      float* __restrict__ tbuf, float floor_, float* __restrict__ vec) {
  __shared__ float red[kWarps];
  __shared__ float norm_s;
  float ss = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float t;
    if (n_chunks > 0) {
      t = 0.f;
      for (int c = 0; c < n_chunks; ++c) t += part[static_cast<long long>(c) * n + j];
      tbuf[j] = t;
    } else {
      t = part[j];
    }
    ss += t * t;
  }
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < kWarps; ++w) s += red[w];
    norm_s = sqrtf(s);
  }
  __syncthreads();
  const float nrm = norm_s;
  if (!(isfinite(nrm) && nrm > floor_)) return;
  const float* src = n_chunks > 0 ? tbuf : part;
  for (int j = threadIdx.x; j < n; j += blockDim.x) vec[j] = src[j] / nrm;
}

// s[i] = W_i . v (one warp per row)
__global__ void __launch_bounds__(256) row_dots(const float* __restrict__ W, int rows, int cols,
                                                const float* __restrict__ v, float* __restrict__ s) {
  const int lane = threadIdx.x % 32;
  for (int row = blockIdx.x * kWarps + threadIdx.x / 32; row < rows; row += gridDim.x * kWarps) {
    const float4* a = reinterpret_cast<const float4*>(W + static_cast<long long>(row) * cols);
    const float4* b = reinterpret_cast<const float4*>(v);
    float acc = 0.f;
    for (int j = lane; j < cols / 4; j += 32) {
      const float4 x = a[j], y = b[j];
      acc += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    }
    acc = warp_sum(acc);
    if (lane == 0) s[row] = acc;
  }
}

int row_blocks(int rows) {
  const int blocks = (rows + kWarps - 1) / kWarps;
  const int cap = kSpectralMaxPartials;
  return blocks < cap ? blocks : cap;
}

int elem_blocks(long long n4) {
  const long long blocks = (n4 + 255) / 256, cap = 8LL * num_sms();
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

void check_shape(int rows, int cols) {
  TTB_CHECK(rows > 0 && cols > 0 && cols % 4 == 0, "spectral: need rows > 0 and cols a positive multiple of 4");
}

}  // namespace

long long spectral_scratch_floats(int rows, int cols) {
  const long long chunks = (rows + kRowChunk - 1) / kRowChunk;
  const long long pass = chunks * cols + cols + rows;  // column partials, W^T u, W v
  return pass > kSpectralMaxPartials ? pass : kSpectralMaxPartials;
}

void spectral_cast(const float* W, int rows, int cols, const float* gamma, const float* u, const float* v, float floor_,
                   float* sigma_out, float* partials, __nv_bfloat16* out, long long ld, cudaStream_t stream) {
  check_shape(rows, cols);
  const int nb = row_blocks(rows);
  row_dot_partials<<<nb, 256, 0, stream>>>(W, cols, nullptr, 0, v, u, rows, cols, partials);
  TTB_CUDA_CHECK(cudaGetLastError());
  cast_kernel<<<elem_blocks(static_cast<long long>(rows) * cols / 4), 256, 0, stream>>>(
      W, rows, cols, gamma, partials, nb, floor_, sigma_out, out, ld);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void spectral_grad(const float* dWe, long long ld, const float* W, int rows, int cols, const float* gamma,
                   const float* u, const float* v, const float* sigma, float floor_, float* partials, float* dW,
                   float* dgamma, cudaStream_t stream) {
  check_shape(rows, cols);
  TTB_CHECK(ld % 4 == 0, "spectral: dW_eff row stride must be a multiple of 4");
  const int nb = row_blocks(rows);
  row_dot_partials<<<nb, 256, 0, stream>>>(dWe, ld, W, cols, nullptr, nullptr, rows, cols, partials);
  TTB_CUDA_CHECK(cudaGetLastError());
  grad_kernel<<<elem_blocks(static_cast<long long>(rows) * cols / 4), 256, 0, stream>>>(
      dWe, ld, W, rows, cols, gamma, u, v, sigma, partials, nb, floor_, dW, dgamma);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void spectral_power_step(const float* W, int rows, int cols, float* u, float* v, float floor_, float* scratch,
                         cudaStream_t stream) {
  check_shape(rows, cols);
  const int chunks = (rows + kRowChunk - 1) / kRowChunk;
  float* part = scratch;
  float* t = scratch + static_cast<long long>(chunks) * cols;
  float* s = t + cols;
  col_partials<<<dim3((cols + 255) / 256, chunks), 256, 0, stream>>>(W, rows, cols, u, part);
  TTB_CUDA_CHECK(cudaGetLastError());
  normalize_into<<<1, 256, 0, stream>>>(part, chunks, cols, t, floor_, v);
  TTB_CUDA_CHECK(cudaGetLastError());
  row_dots<<<row_blocks(rows), 256, 0, stream>>>(W, rows, cols, v, s);
  TTB_CUDA_CHECK(cudaGetLastError());
  normalize_into<<<1, 256, 0, stream>>>(s, 0, rows, nullptr, floor_, u);
  TTB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ttb
