// Host-side launch helpers for the GEMM kernel template (shared by every translation unit that
// instantiates a GEMM with its own epilogue).
#pragma once

#include "../common/host.h"
#include "api.h"
#include "gemm_sm100.cuh"

#include <cstdlib>

namespace ttb {
namespace gemm {

template <int BN, int STAGES, bool DUAL, class Epi, bool A_MN, bool B_MN>
inline void launch_impl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, Shape s, const Epi& epi,
                        cudaStream_t stream) {
  using L = Layout<BN, STAGES, DUAL>;
  constexpr int kSmem = with_epi_smem<Epi>(L::kSmemBytes, L::kBarOffset, STAGES);
  static_assert(kSmem <= 232448, "GEMM shared memory exceeds 227 KB");
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, DUAL, Epi>;
  static bool configured = false;
  if (!configured) {
    TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured = true;
  }
  constexpr int NB = L::kBNMma;
  const int tiles = ((s.M + BM - 1) / BM) * ((s.N + NB - 1) / NB);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kThreads, kSmem, stream>>>(ta, tb, tb2, s, epi);
  TTB_CUDA_CHECK(cudaGetLastError());
}

constexpr int kPairStages = 6;

// CTA-pair GEMM for plain (single-B) problems with 256-column tiles; off when TTB_GEMM_PAIR=0.
inline bool pair_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TTB_GEMM_PAIR");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

template <class Epi, bool A_MN, bool B_MN, bool DUAL, bool GATHER>
inline void launch_pair_impl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, Shape s,
                             const Epi& epi, const Gather& g, cudaStream_t stream) {
  using L = PairLayout<kPairStages, DUAL>;
  constexpr int kSmem = with_epi_smem<Epi>(L::kSmemBytes, L::kBarOffset, kPairStages);
  static_assert(kSmem <= 232448, "GEMM shared memory exceeds 227 KB");
  auto kern = gemm_pair_kernel<kPairStages, A_MN, B_MN, DUAL, Epi, GATHER>;
  static bool configured = false;
  if (!configured) {
    TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured = true;
  }
  const int tiles = ((s.M + kPairBM - 1) / kPairBM) * ((s.N + L::kTileN - 1) / L::kTileN);
  const int pairs = num_sms() / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  kern<<<grid, GATHER ? kPairGatherThreads : kThreads, kSmem, stream>>>(ta, tb, tb2, s, epi, g);
  TTB_CUDA_CHECK(cudaGetLastError());
}

template <class Epi, bool A_MN, bool B_MN, bool DUAL, bool CAN_GATHER>
inline void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, Shape s, const Epi& epi,
                        const Gather* gather, cudaStream_t stream) {
  if constexpr (CAN_GATHER && !A_MN && !B_MN) {
    if (gather != nullptr) return launch_pair_impl<Epi, A_MN, B_MN, DUAL, true>(ta, tb, tb2, s, epi, *gather, stream);
  }
  TTB_CHECK(gather == nullptr, "the fused gather needs K-major A and B operands");
  launch_pair_impl<Epi, A_MN, B_MN, DUAL, false>(ta, tb, tb2, s, epi, Gather{}, stream);
}

// gather (nullable): B (and b2 for DUAL) are staging buffers filled from row shards by the GEMM
// itself (CTA-pair path) or, where the pair path does not apply, by a gather launch before it.
// CAN_GATHER instantiates the gathering kernels (only for the epilogues of weight-consuming GEMMs).
template <int BN, int STAGES, bool DUAL, bool CAN_GATHER = false, class Epi>
inline void dispatch(const Operand& a, const Operand& b, const Operand* b2, Shape s, const Epi& epi,
                     cudaStream_t stream, const Gather* gather = nullptr) {
  TTB_CHECK(gather == nullptr || (s.k_split == 0 && !b.mn_major && gather->nops == (DUAL ? 2 : 1)),
            "the fused gather takes K-major B operands without K concatenation, one per B");
  // contraction extents of the B operands: all of K, or the two parts of a K concatenation
  TTB_CHECK(s.k_split == 0 || (!DUAL && b2 != nullptr && s.k_split % BK == 0 && s.k_split < s.K),
            "K concatenation needs a second B operand and a split on a k-block boundary");
  const int k1 = s.k_split > 0 ? s.k_split : s.K;
  const int k2 = s.k_split > 0 ? s.K - s.k_split : s.K;
  if constexpr (BN == 256) {
    if (pair_enabled() && s.M >= kPairBM) {
      using L = PairLayout<kPairStages, DUAL>;
      // per CTA: 128-row A boxes and kBCols-column B boxes (MN-major operands use 64-wide boxes)
      const CUtensorMap ta = a.mn_major
                                 ? make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.M, s.K, a.ld, 64, BK)
                                 : make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.K, s.M, a.ld, BK, kPairHalf);
      auto bmap = [&](const Operand& o, int kx) {
        return o.mn_major ? make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.N, kx, o.ld, 64, BK)
                          : make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kx, s.N, o.ld, BK, L::kBCols);
      };
      const CUtensorMap tb = bmap(b, k1);
      const CUtensorMap tb2 = b2 != nullptr ? bmap(*b2, k2) : tb;
      TTB_CHECK(b2 == nullptr || b2->mn_major == b.mn_major, "dual GEMM operands must share a layout");
      if (a.mn_major) {
        if (b.mn_major) return launch_pair<Epi, true, true, DUAL, CAN_GATHER>(ta, tb, tb2, s, epi, gather, stream);
        return launch_pair<Epi, true, false, DUAL, CAN_GATHER>(ta, tb, tb2, s, epi, gather, stream);
      }
      if (b.mn_major) return launch_pair<Epi, false, true, DUAL, CAN_GATHER>(ta, tb, tb2, s, epi, gather, stream);
      return launch_pair<Epi, false, false, DUAL, CAN_GATHER>(ta, tb, tb2, s, epi, gather, stream);
    }
  }
  if (gather != nullptr) gather_rows(*gather, stream);
  constexpr int NB = DUAL ? BN / 2 : BN;
  // A: rows = M, contraction = K.  K-major -> [M, K] rows; MN-major -> [K, M] rows.
  const CUtensorMap ta = a.mn_major
                             ? make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.M, s.K, a.ld, 64, BK)
                             : make_tmap_2d(a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.K, s.M, a.ld, BK, BM);
  auto bmap = [&](const Operand& o, int kx) {
    return o.mn_major ? make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.N, kx, o.ld, 64, BK)
                      : make_tmap_2d(o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kx, s.N, o.ld, BK, NB);
  };
  const CUtensorMap tb = bmap(b, k1);
  const CUtensorMap tb2 = b2 != nullptr ? bmap(*b2, k2) : tb;
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
