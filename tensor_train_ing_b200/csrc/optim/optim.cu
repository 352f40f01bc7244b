// Optimizer update kernels (declared in optim_api.h).
//
// AdamW: one launch per parameter group covers every tensor of the group. A tiny kernel first adds
// one to each tensor's step counter (device scalars, so the update needs no host round trip), then
// the update kernel walks fixed 16 Ki-element chunks; a block finds its tensor by binary search
// over the descriptors' chunk prefix. The clip coefficient multiplies the gradient as it is read.
//
// Muon: the element-wise work around the Newton-Schulz GEMMs is three bandwidth-bound passes:
// prepare (clip scale, momentum lerp, Nesterov lerp, bf16 operand in the orientation the
// iteration wants, sum of squares), normalize (divide by the bf16 Frobenius norm) and apply
// (decoupled decay, scaled update, bf16 weight copy for the next forward's GEMMs). Transposes go
// through 32 x 32 shared-memory tiles so global reads and writes stay coalesced. The lerps use the
// two-sided form (start + w (end - start) for |w| < 1/2, end - (end - start)(1 - w) otherwise), the
// form PyTorch's lerp uses, so momentum buffers track torch.optim.Muon's closely.
#include <cuda_bf16.h>

#include <cstdint>

#include "../common/host.h"
#include "optim_api.h"

namespace ttb {
namespace {

__device__ __forceinline__ float lerp2(float start, float end, float w) {
  return fabsf(w) < 0.5f ? start + w * (end - start) : end - (end - start) * (1.f - w);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32 + (threadIdx.y * blockDim.x) / 32;
  const int lane = (threadIdx.y * blockDim.x + threadIdx.x) % 32;
  const int nwarps = blockDim.x * blockDim.y / 32;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (warp == 0) {
    s = lane < nwarps ? red[lane] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  }
  return s;  // valid in warp 0
}

// ------------------------------------------------------------------------------------ AdamW
__global__ void adamw_count_kernel(const AdamwTensor* __restrict__ list, int count) {
  for (int i = threadIdx.x; i < count; i += blockDim.x) *list[i].step += 1.f;
}

struct AdamwScalars {
  float lr, b1, b2, eps, wd;
};

__device__ __forceinline__ void adamw_one(float& p, float g, float& m, float& v, const AdamwScalars& s,
                                          float step_size, float bc2_sqrt) {
  p -= s.lr * s.wd * p;
  m = s.b1 * m + (1.f - s.b1) * g;
  v = s.b2 * v + (1.f - s.b2) * g * g;
  const float denom = sqrtf(v) / bc2_sqrt + s.eps;
  p -= step_size * m / denom;
}

__global__ void __launch_bounds__(256) adamw_kernel(const AdamwTensor* __restrict__ list, int count,
                                                    long long total_chunks, AdamwScalars s,
                                                    const float* __restrict__ grad_scale) {
  const float scale = grad_scale != nullptr ? *grad_scale : 1.f;
  for (long long c = blockIdx.x; c < total_chunks; c += gridDim.x) {
    int lo = 0, hi = count - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (list[mid].first_chunk <= c) lo = mid; else hi = mid - 1;
    }
    const AdamwTensor t = list[lo];
    const long long begin = (c - t.first_chunk) * kAdamwChunk;
    const long long end = begin + kAdamwChunk < t.n ? begin + kAdamwChunk : t.n;
    const float step = *t.step;
    const float step_size = s.lr / (1.f - powf(s.b1, step));
    const float bc2_sqrt = sqrtf(1.f - powf(s.b2, step));
    const bool vec = ((reinterpret_cast<uintptr_t>(t.p) | reinterpret_cast<uintptr_t>(t.g) |
                       reinterpret_cast<uintptr_t>(t.exp_avg) | reinterpret_cast<uintptr_t>(t.exp_avg_sq)) & 15) == 0 &&
                     (t.cache == nullptr || (reinterpret_cast<uintptr_t>(t.cache) & 7) == 0) && (t.n & 3) == 0;
    if (vec) {
      for (long long i = begin + 4 * threadIdx.x; i < end; i += 4 * blockDim.x) {
        float4 p = *reinterpret_cast<const float4*>(t.p + i);
        const float4 g = *reinterpret_cast<const float4*>(t.g + i);
        float4 m = *reinterpret_cast<const float4*>(t.exp_avg + i);
        float4 v = *reinterpret_cast<const float4*>(t.exp_avg_sq + i);
        adamw_one(p.x, g.x * scale, m.x, v.x, s, step_size, bc2_sqrt);
        adamw_one(p.y, g.y * scale, m.y, v.y, s, step_size, bc2_sqrt);
        adamw_one(p.z, g.z * scale, m.z, v.z, s, step_size, bc2_sqrt);
        adamw_one(p.w, g.w * scale, m.w, v.w, s, step_size, bc2_sqrt);
        *reinterpret_cast<float4*>(t.p + i) = p;
        *reinterpret_cast<float4*>(t.exp_avg + i) = m;
        *reinterpret_cast<float4*>(t.exp_avg_sq + i) = v;
        if (t.cache != nullptr) {
          __nv_bfloat162 lo2 = __floats2bfloat162_rn(p.x, p.y), hi2 = __floats2bfloat162_rn(p.z, p.w);
          uint2 packed;
          packed.x = *reinterpret_cast<uint32_t*>(&lo2);
          packed.y = *reinterpret_cast<uint32_t*>(&hi2);
          *reinterpret_cast<uint2*>(t.cache + i) = packed;
        }
      }
    } else {
      for (long long i = begin + threadIdx.x; i < end; i += blockDim.x) {
        float p = t.p[i], m = t.exp_avg[i], v = t.exp_avg_sq[i];
        adamw_one(p, t.g[i] * scale, m, v, s, step_size, bc2_sqrt);
        t.p[i] = p;
        t.exp_avg[i] = m;
        t.exp_avg_sq[i] = v;
        if (t.cache != nullptr) t.cache[i] = __float2bfloat16_rn(p);
      }
    }
  }
}

// ------------------------------------------------------------------------------------ Muon
constexpr int kTile = 32;
constexpr int kRowsPerThread = 4;  // blockDim = (32, 8)

__global__ void __launch_bounds__(256) muon_prepare_kernel(const float* __restrict__ g, float* __restrict__ buf,
                                                           __nv_bfloat16* __restrict__ x, float* __restrict__ partial,
                                                           int rows, int cols, float w_buf, float w_nest, int nesterov,
                                                           int transpose, const float* __restrict__ grad_scale) {
  __shared__ __nv_bfloat16 tile[kTile][kTile + 2];
  __shared__ float red[8];
  const float scale = grad_scale != nullptr ? *grad_scale : 1.f;
  const int tiles_c = (cols + kTile - 1) / kTile;
  const long long tiles = static_cast<long long>(tiles_c) * ((rows + kTile - 1) / kTile);
  float ss = 0.f;
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = static_cast<int>(t / tiles_c) * kTile, c0 = static_cast<int>(t % tiles_c) * kTile;
    const int c = c0 + threadIdx.x;
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) {
      const int rr = threadIdx.y + 8 * k, r = r0 + rr;
      if (r < rows && c < cols) {
        const long long i = static_cast<long long>(r) * cols + c;
        const float gi = g[i] * scale;
        const float b = lerp2(buf[i], gi, w_buf);
        buf[i] = b;
        const __nv_bfloat16 xb = __float2bfloat16_rn(nesterov ? lerp2(gi, b, w_nest) : b);
        const float xf = __bfloat162float(xb);
        ss += xf * xf;
        if (transpose) tile[rr][threadIdx.x] = xb; else x[i] = xb;
      }
    }
    if (transpose) {
      __syncthreads();
      const int orow_base = c0, ocol = r0 + threadIdx.x;  // x is [cols, rows]
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) {
        const int cc = threadIdx.y + 8 * k, orow = orow_base + cc;
        if (orow < cols && ocol < rows) x[static_cast<long long>(orow) * rows + ocol] = tile[threadIdx.x][cc];
      }
      __syncthreads();
    }
  }
  const float total = block_sum(ss, red);
  if (threadIdx.x == 0 && threadIdx.y == 0) partial[blockIdx.x] = total;
}

__global__ void __launch_bounds__(256) muon_normalize_kernel(__nv_bfloat16* __restrict__ x, long long n,
                                                             const float* __restrict__ partial, int n_partial,
                                                             float eps) {
  __shared__ float divisor;
  if (threadIdx.x < 32) {
    float s = 0.f;
    for (int i = threadIdx.x; i < n_partial; i += 32) s += partial[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) {
      const float norm = __bfloat162float(__float2bfloat16_rn(sqrtf(s)));
      const float floor_ = __bfloat162float(__float2bfloat16_rn(eps));
      divisor = norm > floor_ ? norm : floor_;
    }
  }
  __syncthreads();
  const float d = divisor;
  const long long pairs = n / 2;
  __nv_bfloat162* x2 = reinterpret_cast<__nv_bfloat162*>(x);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float2 f = __bfloat1622float2(x2[i]);
    x2[i] = __floats2bfloat162_rn(f.x / d, f.y / d);
  }
  if ((n & 1) && blockIdx.x == 0 && threadIdx.x == 0) x[n - 1] = __float2bfloat16_rn(__bfloat162float(x[n - 1]) / d);
}

__global__ void __launch_bounds__(256) muon_apply_kernel(float* __restrict__ p, const __nv_bfloat16* __restrict__ o,
                                                         int rows, int cols, int transposed, float decay, float alpha,
                                                         __nv_bfloat16* __restrict__ cache, long long cache_ld) {
  __shared__ __nv_bfloat16 tile[kTile][kTile + 2];
  const int tiles_c = (cols + kTile - 1) / kTile;
  const long long tiles = static_cast<long long>(tiles_c) * ((rows + kTile - 1) / kTile);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = static_cast<int>(t / tiles_c) * kTile, c0 = static_cast<int>(t % tiles_c) * kTile;
    if (transposed) {  // o is [cols, rows]: stage o[c0.., r0..] so tile[cc][rr] = o[c0 + cc][r0 + rr]
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) {
        const int cc = threadIdx.y + 8 * k, oc = c0 + cc, orr = r0 + threadIdx.x;
        if (oc < cols && orr < rows) tile[cc][threadIdx.x] = o[static_cast<long long>(oc) * rows + orr];
      }
      __syncthreads();
    }
    const int c = c0 + threadIdx.x;
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) {
      const int rr = threadIdx.y + 8 * k, r = r0 + rr;
      if (r < rows && c < cols) {
        const long long i = static_cast<long long>(r) * cols + c;
        const float u = __bfloat162float(transposed ? tile[threadIdx.x][rr] : o[i]);
        const float v = p[i] * decay + alpha * u;
        p[i] = v;
        if (cache != nullptr) cache[static_cast<long long>(r) * cache_ld + c] = __float2bfloat16_rn(v);
      }
    }
    if (transposed) __syncthreads();
  }
}

int grid_for_tiles(int rows, int cols, int cap) {
  const long long tiles = static_cast<long long>((rows + kTile - 1) / kTile) * ((cols + kTile - 1) / kTile);
  return static_cast<int>(tiles < cap ? tiles : cap);
}

}  // namespace

void adamw_update(const AdamwTensor* tensors, int count, long long total_chunks, float lr, float beta1, float beta2,
                  float eps, float weight_decay, const float* grad_scale, cudaStream_t stream) {
  if (count <= 0 || total_chunks <= 0) return;
  adamw_count_kernel<<<1, 256, 0, stream>>>(tensors, count);
  TTB_CUDA_CHECK(cudaGetLastError());
  const long long cap = 8LL * num_sms();
  const int grid = static_cast<int>(total_chunks < cap ? total_chunks : cap);
  adamw_kernel<<<grid, 256, 0, stream>>>(tensors, count, total_chunks, AdamwScalars{lr, beta1, beta2, eps, weight_decay},
                                         grad_scale);
  TTB_CUDA_CHECK(cudaGetLastError());
}

int muon_prepare(const float* g, float* buf, __nv_bfloat16* x, float* partial, int rows, int cols, float w_buf,
                 float w_nesterov, bool nesterov, bool transpose, const float* grad_scale, cudaStream_t stream) {
  TTB_CHECK(rows > 0 && cols > 0, "muon_prepare: empty matrix");
  int cap = 4 * num_sms();
  if (cap > kMuonMaxPartials) cap = kMuonMaxPartials;
  const int grid = grid_for_tiles(rows, cols, cap);
  muon_prepare_kernel<<<grid, dim3(kTile, 8), 0, stream>>>(g, buf, x, partial, rows, cols, w_buf, w_nesterov,
                                                           nesterov ? 1 : 0, transpose ? 1 : 0, grad_scale);
  TTB_CUDA_CHECK(cudaGetLastError());
  return grid;
}

void muon_normalize(__nv_bfloat16* x, long long n, const float* partial, int n_partial, float eps,
                    cudaStream_t stream) {
  TTB_CHECK(n_partial > 0 && n_partial <= kMuonMaxPartials, "muon_normalize: bad partial count");
  TTB_CHECK((reinterpret_cast<uintptr_t>(x) & 3) == 0, "muon_normalize: x must be 4-byte aligned");
  const long long pairs = (n + 1) / 2;
  long long grid = (pairs + 255) / 256;
  if (grid > 8LL * num_sms()) grid = 8LL * num_sms();
  if (grid < 1) grid = 1;
  muon_normalize_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(x, n, partial, n_partial, eps);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void muon_apply(float* p, const __nv_bfloat16* o, int rows, int cols, bool transposed, float decay, float alpha,
                __nv_bfloat16* cache, long long cache_ld, cudaStream_t stream) {
  TTB_CHECK(rows > 0 && cols > 0, "muon_apply: empty matrix");
  const int grid = grid_for_tiles(rows, cols, 16 * num_sms());
  muon_apply_kernel<<<grid, dim3(kTile, 8), 0, stream>>>(p, o, rows, cols, transposed ? 1 : 0, decay, alpha, cache,
                                                         cache_ld);
  TTB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ttb
