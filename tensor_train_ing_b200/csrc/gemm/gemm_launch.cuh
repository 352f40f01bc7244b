// Host-side launch helpers for the GEMM kernel template (shared by every translation unit that
// instantiates a GEMM with its own epilogue).
#pragma once

#include "../common/host.h"
#include "api.h"
#include "gemm_sm100.cuh"

namespace ttb {
namespace gemm {

template <int BN, int STAGES, bool DUAL, class Epi, bool A_MN, bool B_MN>
inline void launch_impl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, Shape s, const Epi& epi,
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
inline void dispatch(const Operand& a, const Operand& b, const Operand* b2, Shape s, const Epi& epi,
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

}  // namespace ttb
