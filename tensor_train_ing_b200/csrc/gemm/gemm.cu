// Host launchers for the sm_100a GEMM family: plain/accumulating linear, bilinear (dual-B) and
// bilinear backward.  Operand "majorness" is chosen from strides by the caller.
#include "../common/host.h"
#include "api.h"
#include "epilogues.cuh"

namespace ttb {

namespace gemm {

template <int BN, int STAGES, bool DUAL, class Epi, bool A_MN, bool B_MN>
static void launch_impl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, Shape s, const Epi& epi,
                        cudaStream_t stream) {
  using L = Layout<BN, STAGES, DUAL>;
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, DUAL, Epi>;
  static bool configured = false;
  if (!configured) {
    TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes));
    configured = true;
  }
  constexpr int NB = L::kBNMma;
  const int tiles = ((s.M + BM - 1) / BM) * ((s.N + NB - 1) / NB);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kThreads, L::kSmemBytes, stream>>>(ta, tb, tb2, s, epi);
  TTB_CUDA_CHECK(cudaGetLastError());
}

template <int BN, int STAGES, bool DUAL, class Epi>
static void dispatch(const Operand& a, const Operand& b, const Operand* b2, Shape s, const Epi& epi,
                     cudaStream_t stream) {
  constexpr int NB = DUAL ? BN / 2 : BN;
  // A: rows = M, contraction = K.  K-major -> [M, K] rows; MN-major -> [K, M] rows.
  const CUtensorMap ta = a.mn_major
                             ? make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.M, s.K, a.ld, 64, BK)
                             : make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.K, s.M, a.ld, BK, BM);
  auto bmap = [&](const Operand& o) {
    return o.mn_major ? make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.N, s.K, o.ld, 64, BK)
                      : make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.K, s.N, o.ld, BK, NB);
  };
  const CUtensorMap tb = bmap(b);
  const CUtensorMap tb2 = b2 != nullptr ? bmap(*b2) : tb;
  TTB_CHECK(b2 == nullptr || b2->mn_major == b.mn_major, "dual GEMM operands must share a layout");
  if (a.mn_major) {
    if (b.mn_major)
      launch_impl<BN, STAGES, DUAL, Epi, true, true>(ta, tb, tb2, s, epi, stream);
    else
      launch_impl<BN, STAGES, DUAL, Epi, true, false>(ta, tb, tb2, s, epi, stream);
  } else {
    if (b.mn_major)
      launch_impl<BN, STAGES, DUAL, Epi, false, true>(ta, tb, tb2, s, epi, stream);
    else
      launch_impl<BN, STAGES, DUAL, Epi, false, false>(ta, tb, tb2, s, epi, stream);
  }
}

}  // namespace gemm

void gemm_linear(const Operand& a, const Operand& b, int M, int N, int K, void* D, long long ldd, bool d_f32,
                 const void* C, long long ldc, bool c_f32, float alpha, float beta, const float* bias,
                 cudaStream_t stream) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  if (N <= 128) {
    gemm::EpiLinear<128> epi{D, ldd, d_f32, C, ldc, c_f32, alpha, beta, bias, M, N};
    gemm::dispatch<128, 6, false>(a, b, nullptr, gemm::Shape{M, N, K, status_ptr()}, epi, stream);
  } else {
    gemm::EpiLinear<256> epi{D, ldd, d_f32, C, ldc, c_f32, alpha, beta, bias, M, N};
    gemm::dispatch<256, 4, false>(a, b, nullptr, gemm::Shape{M, N, K, status_ptr()}, epi, stream);
  }
}

void gemm_bilinear(const Operand& x, const Operand& wl, const Operand& wr, int M, int N, int K, void* H, void* Lo,
                   void* Ro, long long ld, const float* bias_l, const float* bias_r, int mode, cudaStream_t stream) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  gemm::EpiBilinear<128> epi{static_cast<__nv_bfloat16*>(H), static_cast<__nv_bfloat16*>(Lo),
                             static_cast<__nv_bfloat16*>(Ro), ld, bias_l, bias_r, mode, M, N};
  gemm::dispatch<256, 4, true>(x, wl, &wr, gemm::Shape{M, N, K, status_ptr()}, epi, stream);
}

void gemm_bilinear_grad(const Operand& dy, const Operand& wd, int M, int N, int K, const void* Lin, const void* Rin,
                        void* dL, void* dR, long long ld, int mode, cudaStream_t stream) {
  TTB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  gemm::EpiBilinearGrad<256> epi{static_cast<const __nv_bfloat16*>(Lin), static_cast<const __nv_bfloat16*>(Rin),
                                 static_cast<__nv_bfloat16*>(dL), static_cast<__nv_bfloat16*>(dR), ld, mode, M, N};
  gemm::dispatch<256, 4, false>(dy, wd, nullptr, gemm::Shape{M, N, K, status_ptr()}, epi, stream);
}

}  // namespace ttb
