// Chunked linear + cross-entropy on the tcgen05 GEMM: logits never reach HBM in the forward.
//
// Forward (per chunk of rows): logits tile = alpha * x W^T; the epilogue keeps an online
// (max, sum exp) over the tile's columns and picks the target logit, writing one partial per
// (row, column tile).  ce_combine reduces the partials in a fixed order to lse and per-row loss.
// Backward: the same GEMM recomputes the logits and its epilogue writes
//   dlogits = g * alpha * valid * (softmax - onehot)     (bf16, padded columns = 0)
// which two more GEMMs turn into dx = dlogits W and dW += dlogits^T x.
#include <math_constants.h>

#include "../common/host.h"
#include "api.h"
#include "ce_api.h"
#include "epilogues.cuh"
#include "gemm_launch.cuh"

namespace ttb {
namespace gemm {

template <int NB>
struct EpiCEFwd {
  float* pmax;
  float* psum;
  long long ldp;
  float* tlogit;
  const long long* targets;
  float alpha;
  int M, V;
  float* zout;     // optional: the scaled logits [M, Npad] (fp32, -inf past V), kept for the backward
  long long ldz;
  int Npad;
  static constexpr int kSmemPerThread = 256;  // per warp: one 4 KB chunk buffer for the logit stores

  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int, int tn, uint8_t* sm) const {
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;
    const long long tgt = row < M ? targets[row] : -1;
    float m = -CUDART_INF_F, s = 0.f, tz = 0.f;
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      float z[32];
      float cmax = -CUDART_INF_F;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        z[j] = (col0 + j < V) ? alpha * __uint_as_float(r[j]) : -CUDART_INF_F;
        cmax = fmaxf(cmax, z[j]);
        if (col0 + j == tgt) tz = z[j];
      }
      if (zout != nullptr && col0 < Npad) gemm::warp_store_f32(area, z, lane, zout, ldz, row - lane, col0, M, Npad);
      const float nm = fmaxf(m, cmax);
      if (nm == -CUDART_INF_F) continue;
      float cs = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) cs += expf(z[j] - nm);
      s = s * expf(m - nm) + cs;
      m = nm;
    }
    if (row < M) {
      pmax[row * ldp + tn] = m;
      psum[row * ldp + tn] = s;
      if (tgt >= n0 && tgt < n0 + NB) tlogit[row] = tz;
    }
  }
};

template <int NB>
struct EpiCEBwd {
  __nv_bfloat16* dlogits;
  long long ldd;
  const float* lse;
  const long long* targets;
  const float* grad;  // device scalar: upstream gradient of the summed loss
  float alpha;
  int M, N, V;
  static constexpr int kSmemPerThread = 256;  // per warp: one 2 KB chunk buffer (warp-coalesced stores)

  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int tm, int tn, uint8_t* sm) const {
    if (!(ldd % 8 == 0 && N % 8 == 0 && (reinterpret_cast<uintptr_t>(dlogits) & 15) == 0))
      return rowwise(taddr, row, n0);
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;
    const int row0 = row - lane;
    long long tgt = -1;
    float l = 0.f, coef = 0.f;
    if (row < M) {
      tgt = targets[row];
      l = lse[row];
      coef = tgt >= 0 && tgt < V ? grad[0] * alpha : 0.f;  // out-of-range targets: no loss, no gradient
    }
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      if (col0 >= N) continue;  // the same for the whole warp
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = col0 + j;
        float p = col < V ? expf(alpha * __uint_as_float(r[j]) - l) : 0.f;
        if (col == tgt) p -= 1.f;
        v[j] = p * coef;
      }
      gemm::warp_store_bf16(area, v, lane, dlogits, ldd, row0, col0, M, N);
    }
  }

  __device__ __forceinline__ void rowwise(uint32_t taddr, int row, int n0) const {
    long long tgt = -1;
    float l = 0.f, coef = 0.f;
    if (row < M) {
      tgt = targets[row];
      l = lse[row];
      coef = tgt >= 0 && tgt < V ? grad[0] * alpha : 0.f;  // out-of-range targets: no loss, no gradient
    }
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      if (row >= M || col0 >= N) continue;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = col0 + j;
        float p = col < V ? expf(alpha * __uint_as_float(r[j]) - l) : 0.f;
        if (col == tgt) p -= 1.f;
        v[j] = p * coef;
      }
      const int nv = min(32, N - col0);
      store_row32_bf16(dlogits + row * ldd + col0, nv == 32 && (ldd % 8 == 0), nv, v);
    }
  }
};

// dlogits from the logits the forward kept: one block per row, float4 in, four bf16 out.
__global__ void __launch_bounds__(256) ce_grad_from_logits_kernel(const float* __restrict__ z, long long ldz,
                                                                  const float* __restrict__ lse,
                                                                  const long long* __restrict__ targets,
                                                                  const float* __restrict__ grad, float alpha, int M,
                                                                  int Npad, __nv_bfloat16* __restrict__ dlog,
                                                                  long long ldd) {
  const int row = blockIdx.x;
  if (row >= M) return;
  const float l = lse[row];
  const long long t = targets[row];
  const float coef = t >= 0 && t < Npad ? grad[0] * alpha : 0.f;
  const float4* zr = reinterpret_cast<const float4*>(z + static_cast<long long>(row) * ldz);
  uint2* dr = reinterpret_cast<uint2*>(dlog + static_cast<long long>(row) * ldd);
  for (int i = threadIdx.x; i < Npad / 4; i += blockDim.x) {
    const float4 v = __ldcs(zr + i);  // read once: stream past L2
    float p[4] = {expf(v.x - l), expf(v.y - l), expf(v.z - l), expf(v.w - l)};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (4LL * i + k == t) p[k] -= 1.f;
      p[k] *= coef;
    }
    dr[i] = make_uint2(pack_bf16(p[0], p[1]), pack_bf16(p[2], p[3]));
  }
}

// A target outside [0, V) (other than the negative ignore ids) is recorded in the status word and
// its row contributes no loss.
__global__ void ce_combine_kernel(const float* __restrict__ pmax, const float* __restrict__ psum, long long ldp,
                                  int tiles, const float* __restrict__ tlogit, const long long* __restrict__ targets,
                                  float* __restrict__ lse, float* __restrict__ loss_row, int M, int V,
                                  uint32_t* status) {
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < M; row += gridDim.x * warps) {
    float mx = -CUDART_INF_F;
    for (int t = lane; t < tiles; t += 32) mx = fmaxf(mx, pmax[row * ldp + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = 0.f;
    for (int t = lane; t < tiles; t += 32) {
      const float pm = pmax[row * ldp + t];
      if (pm != -CUDART_INF_F) s += psum[row * ldp + t] * expf(pm - mx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      const float l = mx + logf(s);
      lse[row] = l;
      const long long t = targets[row];
      if (t >= V) record_error(status, kErrBadIndex);
      loss_row[row] = t >= 0 && t < V ? l - tlogit[row] : 0.f;
    }
  }
}

}  // namespace gemm

int ce_num_tiles(int V) { return (V + 255) / 256; }

void ce_forward(const Operand& x, const Operand& w, int M, int V, int K, float alpha, const long long* targets,
                float* pmax, float* psum, float* tlogit, float* lse, float* loss_row, cudaStream_t stream, float* zout,
                long long ldz, int Npad) {
  TTB_CHECK(M > 0 && V > 0 && K > 0, "empty CE");
  TTB_CHECK(zout == nullptr || (Npad >= V && Npad % 4 == 0 && ldz % 4 == 0 && (reinterpret_cast<uintptr_t>(zout) & 15) == 0),
            "CE logits buffer: width and stride multiples of 4, 16-byte aligned");
  const int tiles = ce_num_tiles(V);
  gemm::EpiCEFwd<256> epi{pmax, psum, tiles, tlogit, targets, alpha, M, V, zout, ldz, Npad};
  gemm::dispatch<256, 4, false>(x, w, nullptr, gemm::Shape{M, V, K, status_ptr()}, epi, stream);
  const int grid = (M + 7) / 8 < 4 * num_sms() ? (M + 7) / 8 : 4 * num_sms();
  gemm::ce_combine_kernel<<<grid, 256, 0, stream>>>(pmax, psum, tiles, tiles, tlogit, targets, lse, loss_row, M, V,
                                                    status_ptr());
  TTB_CUDA_CHECK(cudaGetLastError());
}

void ce_backward_from_logits(const float* z, long long ldz, int M, int Npad, float alpha, const long long* targets,
                             const float* lse, const float* grad, void* dlogits, long long ldd, cudaStream_t stream) {
  TTB_CHECK(M > 0 && Npad % 4 == 0 && ldz % 4 == 0 && ldd % 4 == 0, "CE backward from logits: widths and strides");
  gemm::ce_grad_from_logits_kernel<<<M, 256, 0, stream>>>(z, ldz, lse, targets, grad, alpha, M, Npad,
                                                          static_cast<__nv_bfloat16*>(dlogits), ldd);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void ce_backward_logits(const Operand& x, const Operand& w, int M, int Npad, int V, int K, float alpha,
                        const long long* targets, const float* lse, const float* grad, void* dlogits,
                        long long ldd, cudaStream_t stream) {
  TTB_CHECK(M > 0 && Npad >= V && K > 0, "empty CE");
  gemm::EpiCEBwd<256> epi{static_cast<__nv_bfloat16*>(dlogits), ldd, lse, targets, grad, alpha, M, Npad, V};
  gemm::dispatch<256, 4, false>(x, w, nullptr, gemm::Shape{M, Npad, K, status_ptr()}, epi, stream);
}

}  // namespace ttb
