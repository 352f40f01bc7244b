// Host launchers for the sm_100a GEMM family: plain/accumulating linear, bilinear (dual-B) and
// bilinear backward.  Operand "majorness" is chosen from strides by the caller.
#include "../common/host.h"
#include "api.h"
#include "epilogues.cuh"
#include "gemm_launch.cuh"

namespace ttb {

namespace gemm {
// Every warp of the launch copies gather chunks (the fused GEMM's copy without the GEMM).
__global__ void __launch_bounds__(256) gather_rows_kernel(const __grid_constant__ Gather g) {
  gather_warp<8>(g, threadIdx.x % 32);
  __syncthreads();
  if (threadIdx.x == 0) gather_finish(g);
}
}  // namespace gemm

uint32_t* gather_claim_counter() {
  static uint32_t* ptrs[64] = {nullptr};
  int dev = 0;
  TTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (ptrs[dev] == nullptr) {
    TTB_CUDA_CHECK(cudaMalloc(&ptrs[dev], 2 * sizeof(uint32_t)));
    TTB_CUDA_CHECK(cudaMemset(ptrs[dev], 0, 2 * sizeof(uint32_t)));
  }
  return ptrs[dev];
}

void gather_rows(const gemm::Gather& g, cudaStream_t stream) {
  TTB_CHECK(g.nops >= 1 && g.nops <= 2 && g.claim != nullptr, "gather: one or two operands and a chunk counter");
  const long long chunks = static_cast<long long>(g.nops) * (g.op[0].rows / gemm::kGatherSlabRows) *
                           gemm::gather_chunks_per_slab(g.op[0].cols);
  const int blocks = (chunks + 7) / 8 < num_sms() ? static_cast<int>((chunks + 7) / 8) : num_sms();
  gemm::gather_rows_kernel<<<blocks > 0 ? blocks : 1, 256, 0, stream>>>(g);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void gemm_linear(const Operand& a, const Operand& b, int M, int N, int K, void* D, long long ldd, bool d_f32,
                 const void* C, long long ldc, bool c_f32, float alpha, float beta, const float* bias,
                 cudaStream_t stream, const Operand* b2, int k_split, int tile_n, const gemm::Gather* gather) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  TTB_CHECK(tile_n == 0 || tile_n == 128 || tile_n == 256, "GEMM tile width must be 0 (automatic), 128 or 256");
  const gemm::Shape shape{M, N, K, status_ptr(), b2 != nullptr ? k_split : 0};
  if (tile_n == 128 || (tile_n == 0 && N <= 128)) {
    if (gather != nullptr) gather_rows(*gather, stream);  // the 128-wide tiles run without the fused copy
    gemm::EpiLinear<128> epi{D, ldd, d_f32, C, ldc, c_f32, alpha, beta, bias, M, N};
    gemm::dispatch<128, 6, false>(a, b, b2, shape, epi, stream);
  } else {
    gemm::EpiLinear<256> epi{D, ldd, d_f32, C, ldc, c_f32, alpha, beta, bias, M, N};
    gemm::dispatch<256, 4, false, true>(a, b, b2, shape, epi, stream, gather);
  }
}

void gemm_bilinear(const Operand& x, const Operand& wl, const Operand& wr, int M, int N, int K, void* H, void* Lo,
                   void* Ro, long long ld, const float* bias_l, const float* bias_r, int mode, cudaStream_t stream,
                   const gemm::Gather* gather) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  gemm::EpiBilinear<128> epi{static_cast<__nv_bfloat16*>(H), static_cast<__nv_bfloat16*>(Lo),
                             static_cast<__nv_bfloat16*>(Ro), ld, bias_l, bias_r, mode, M, N};
  gemm::dispatch<256, 4, true, true>(x, wl, &wr, gemm::Shape{M, N, K, status_ptr()}, epi, stream, gather);
}

void gemm_bilinear_grad(const Operand& dy, const Operand& wd, int M, int N, int K, const void* Lin, const void* Rin,
                        void* dL, void* dR, long long ld, long long ldo, int mode, cudaStream_t stream) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  TTB_CHECK(N % 8 == 0 && ld % 8 == 0 && ldo % 8 == 0,
            "bilinear backward: width and row strides must be multiples of 8 elements");
  gemm::EpiBilinearGrad<256> epi{static_cast<const __nv_bfloat16*>(Lin), static_cast<const __nv_bfloat16*>(Rin),
                                 static_cast<__nv_bfloat16*>(dL), static_cast<__nv_bfloat16*>(dR), ld, ldo, mode,
                                 M, N};
  gemm::dispatch<256, 4, false>(dy, wd, nullptr, gemm::Shape{M, N, K, status_ptr()}, epi, stream);
}

void gemm_qkv_rope(const Operand& x, const Operand& w, int M, int N, int K, void* D, long long ldd, int rope_cols,
                   int dk, const int* pos, const float* cos_t, const float* sin_t, cudaStream_t stream,
                   unsigned int* norm_max, const gemm::Gather* gather) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  TTB_CHECK(dk % 64 == 0 && 256 % dk == 0 && rope_cols % dk == 0 && rope_cols <= N,
            "qkv rope epilogue: dk in {64,128,256}, rope columns a multiple of dk");
  gemm::EpiRope<256> epi{static_cast<__nv_bfloat16*>(D), ldd, rope_cols, dk, pos, cos_t, sin_t, M, N, norm_max};
  gemm::dispatch<256, 4, false, true>(x, w, nullptr, gemm::Shape{M, N, K, status_ptr()}, epi, stream, gather);
}

}  // namespace ttb
