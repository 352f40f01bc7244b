// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M, N] = epilogue( sum_k A[m, k] * B[n, k] )
//
// Roles (192 threads = 6 warps, one CTA per SM, grid = #SMs):
//   warp 0     : TMA producer (one elected lane) filling a STAGES-deep shared-memory ring
//   warp 1     : tcgen05.mma issuer (one elected lane); also owns the TMEM allocation
//   warps 2..5 : epilogue; drain an fp32 accumulator from TMEM (tcgen05.ld) and apply the functor
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap the mainloop of
// tile i+1.  Operands may be K-major or MN-major in global memory; both are staged with TMA
// into 128-byte-swizzled shared memory and described to the tensor core with UMMA descriptors.
// DUAL=true runs two B operands against the same A tile (two accumulators of BN/2 columns),
// which the bilinear MLP uses to form (x L^T) and (x R^T) from one read of x.
//
// The epilogue is a functor with
//   __device__ void operator()(uint32_t taddr, int row, int n0, int tile_m, int tile_n) const
// where taddr addresses this thread's TMEM lane at column 0 of the tile's accumulator.  A functor
// that declares ``static constexpr int kSmemPerThread`` gets that many bytes of shared memory per
// epilogue thread (after the pipeline's barriers) as a sixth argument, a uint8_t* of its own.
#pragma once

#include <type_traits>

#include "../common/sm100.cuh"
#include "gather.cuh"

namespace ttb {
namespace gemm {

template <class E, class = void>
struct EpiSmem {
  static constexpr int kPerThread = 0;
};
template <class E>
struct EpiSmem<E, std::void_t<decltype(E::kSmemPerThread)>> {
  static constexpr int kPerThread = E::kSmemPerThread;
};

constexpr int kEpiThreads = 128;  // four epilogue warps per CTA

// Shared-memory offset of the epilogue's private area (after the barriers; 128-byte aligned) and
// the dynamic shared memory a launch needs with it.
__host__ __device__ constexpr int epi_smem_offset(int bar_offset, int stages) { return (bar_offset + (2 * stages + 5) * 8 + 16 + 127) / 128 * 128; }
template <class Epi>
__host__ __device__ constexpr int with_epi_smem(int smem_bytes, int bar_offset, int stages) {
  return EpiSmem<Epi>::kPerThread == 0 ? smem_bytes
                                       : epi_smem_offset(bar_offset, stages) + kEpiThreads * EpiSmem<Epi>::kPerThread + 1024;
}

template <class Epi>
__device__ __forceinline__ void run_epilogue(const Epi& epi, uint32_t taddr, int row, int n0, int tm, int tn,
                                             uint8_t* epi_smem) {
  if constexpr (EpiSmem<Epi>::kPerThread > 0)
    epi(taddr, row, n0, tm, tn, epi_smem);
  else
    epi(taddr, row, n0, tm, tn);
}

constexpr int BM = 128;
constexpr int BK = 64;            // one 128-byte swizzle row of bf16
constexpr int kThreads = 192;
constexpr int kGroupM = 8;        // tile raster: groups of kGroupM row-tiles sweep all column-tiles

struct Shape {
  int M, N, K;
  uint32_t* status;  // device error word (bounded-wait timeouts)
  // K concatenation (non-DUAL only): when k_split > 0 the contraction runs over two B operands,
  // B rows [0, k_split) from tmB and [k_split, K) from tmB2 (a multiple of BK, so every k-block
  // lies in one of them); A is one [M, K] operand.
  int k_split;
};

// Tensor map and k coordinate of B for the k-block starting at k0.
__device__ __forceinline__ const CUtensorMap* b_source(const CUtensorMap* b1, const CUtensorMap* b2, int k_split,
                                                       int k0, int& kb) {
  if (k_split > 0 && k0 >= k_split) {
    kb = k0 - k_split;
    return b2;
  }
  kb = k0;
  return b1;
}

template <int BN, int STAGES, bool DUAL>
struct Layout {
  static constexpr int kBNMma = DUAL ? BN / 2 : BN;            // N of each UMMA
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = kBNMma * BK * 2;              // per B operand
  static constexpr int kStageBytes = kABytes + (DUAL ? 2 : 1) * kBBytes;
  static constexpr int kAccCols = BN;                          // per accumulator buffer
  static constexpr int kTmemCols = 2 * BN;                     // double buffered
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[STAGES], empty[STAGES], tfull[2], tempty[2], mma_done, tmem holder
  static constexpr int kSmemBytes = kBarOffset + (2 * STAGES + 5) * 8 + 16 + 1024;  // +1024 alignment slack
};

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& tm, int& tn) {
  const int per_group = kGroupM * n_tiles;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(m_tiles - first_m, kGroupM);
  const int in_group = tile - group * per_group;
  tm = first_m + in_group % gsize;
  tn = in_group / gsize;
}

// Tile raster of a GEMM that gathers its B operand while it runs: groups of kGroupN column panels
// sweep every row tile, so the first wave needs only kGroupN panels of the weight and the copy of
// later panels overlaps the MMAs of earlier ones (the default raster sweeps every column panel for
// its first rows, which would wait for the whole weight before the first group of rows finished).
constexpr int kGroupN = 4;
__device__ __forceinline__ void tile_coords_gather(int tile, int m_tiles, int n_tiles, int& tm, int& tn) {
  const int per_group = kGroupN * m_tiles;
  const int group = tile / per_group;
  const int first_n = group * kGroupN;
  const int gsize = min(n_tiles - first_n, kGroupN);
  const int in_group = tile - group * per_group;
  tn = first_n + in_group % gsize;
  tm = in_group / gsize;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool DUAL, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmB2, Shape s, Epi epi) {
  using L = Layout<BN, STAGES, DUAL>;
  constexpr int NB = L::kBNMma;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int m_tiles = (s.M + BM - 1) / BM;
  const int n_tiles = (s.N + NB - 1) / NB;  // output columns per tile: NB (BN/2 when DUAL)
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (s.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (DUAL || s.k_split > 0) prefetch_tmap(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;  // per stage: a load was issued / parity of its phase
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, m_tiles, n_tiles, tm, tn);
        const int m0 = tm * BM;
        const int n0 = tn * NB;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i) tma_load_2d(sa + i * 64 * BK * 2, &tmA, &full[stage], m0 + 64 * i, k0);
          } else {
            tma_load_2d(sa, &tmA, &full[stage], k0, m0);
          }
          int kB;
          const CUtensorMap* mB = b_source(&tmB, &tmB2, DUAL ? 0 : s.k_split, k0, kB);
          if (B_MN) {
#pragma unroll
            for (int i = 0; i < NB / 64; ++i) tma_load_2d(sb + i * 64 * BK * 2, mB, &full[stage], n0 + 64 * i, kB);
            if (DUAL) {
#pragma unroll
              for (int i = 0; i < NB / 64; ++i)
                tma_load_2d(sb + L::kBBytes + i * 64 * BK * 2, &tmB2, &full[stage], n0 + 64 * i, k0);
            }
          } else {
            if (DUAL) {
              tma_load_2d(sb, &tmB, &full[stage], k0, n0);
              tma_load_2d(sb + L::kBBytes, &tmB2, &full[stage], k0, n0);
            } else {
              tma_load_2d(sb, mB, &full[stage], kB, n0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let copies that may still be in flight land before the CTA exits (bounded waits).
        for (int i = 0; i < STAGES; ++i)
          if (issued & (1u << i)) mbar_wait(&full[i], (issued_parity >> i) & 1u, s.status, kErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, NB, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, s.status, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * L::kAccCols;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, s.status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 16 elements = 32 bytes inside the swizzled row.
            // MN-major: advance 16 K-rows = 2048 bytes; MN atoms are 64*BK*2 bytes apart.
            const uint64_t adesc = A_MN ? smem_desc(sa + k * 2048, 64 * BK * 2, 1024) : smem_desc(sa + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc(sb + k * 2048, 64 * BK * 2, 1024) : smem_desc(sb + k * 32, 16, 1024);
            const uint32_t accumulate = (kb > 0 || k > 0) ? 1u : 0u;
            umma_ss(d_tmem, adesc, bdesc, idesc, accumulate);
            if (DUAL) {
              const uint32_t sb2 = sb + L::kBBytes;
              const uint64_t bdesc2 =
                  B_MN ? smem_desc(sb2 + k * 2048, 64 * BK * 2, 1024) : smem_desc(sb2 + k * 32, 16, 1024);
              umma_ss(d_tmem + NB, adesc, bdesc2, idesc, accumulate);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // No tcgen05.mma may still be writing TMEM when it is released.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, s.status, kErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int sub = warp & 3;  // TMEM sub-partition this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, m_tiles, n_tiles, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, s.status, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + acc * L::kAccCols;
      const int row = tm * BM + sub * 32 + lane;
      run_epilogue(epi, taddr, row, tn * NB, tm, tn,
                   smem + epi_smem_offset(L::kBarOffset, STAGES) + (threadIdx.x - 64) * EpiSmem<Epi>::kPerThread);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  __syncwarp();  // reconverge the producer / issuer warps (only one lane of each looped)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ============================================================================ CTA-pair GEMM
// The same persistent, warp-specialised structure on a cluster of two CTAs (two SMs) that
// computes 256 x 256 output tiles with M=256 tcgen05.mma (cta_group::2): CTA r of the pair stages
// rows [128 r, 128 r + 128) of the A tile and columns [128 r, 128 r + 128) of the B tile, so each SM
// streams half of the B tile instead of all of it, and the even CTA issues the MMAs for both.
// Its full barriers count the TMA bytes of both CTAs; its commits arrive on the stage / accumulator
// barriers of both CTAs (multicast commit); the epilogue warps of both CTAs release an accumulator
// buffer by arriving on the even CTA's barrier.  Loads are never multicast.
constexpr int kPairBM = 256;   // rows per pair tile (128 per CTA)
constexpr int kPairBN = 256;   // columns per pair tile (128 of B staged per CTA)
constexpr int kPairHalf = 128;

// DUAL: two B operands of 128 columns each per pair tile (64 staged per CTA), as in the bilinear
// MLP; the two accumulators sit side by side in tensor memory.
template <int STAGES, bool DUAL>
struct PairLayout {
  static constexpr int kBCols = DUAL ? kPairHalf / 2 : kPairHalf;  // B columns staged per CTA, per operand
  static constexpr int kTileN = DUAL ? kPairBN / 2 : kPairBN;       // output columns per pair tile
  static constexpr int kABytes = kPairHalf * BK * 2;   // this CTA's 128 rows of A
  static constexpr int kBBytes = kBCols * BK * 2;      // this CTA's columns of one B operand
  static constexpr int kStageBytes = kABytes + (DUAL ? 2 : 1) * kBBytes;
  static constexpr int kAccCols = kPairBN;
  static constexpr int kTmemCols = 2 * kPairBN;        // double-buffered 256-column accumulators
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + (2 * STAGES + 5) * 8 + 16 + 1024;
};

// GATHER: B (and B2) are staging buffers that two extra warps per CTA (warps 6 and 7) fill from the
// ranks' row shards while the GEMM runs (gather.cuh); the producer waits for a tile's rows first.
constexpr int kPairGatherThreads = kThreads + 64;

template <int STAGES, bool A_MN, bool B_MN, bool DUAL, class Epi, bool GATHER = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GATHER ? kPairGatherThreads : kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmB2, Shape s, Epi epi, const __grid_constant__ Gather g) {
  static_assert(!GATHER || !B_MN, "the fused gather stages K-major B operands (weights [N, K])");
  using L = PairLayout<STAGES, DUAL>;
  constexpr int TN = L::kTileN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int m_tiles = (s.M + kPairBM - 1) / kPairBM;
  const int n_tiles = (s.N + TN - 1) / TN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (s.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);   // the even CTA's producer arrival (+ both CTAs' bytes)
      mbar_init(&empty[i], 1);  // the even CTA's multicast commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * 128);  // epilogue threads of both CTAs
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (DUAL || s.k_split > 0) prefetch_tmap(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int loaded = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int tm, tn;
        if constexpr (GATHER)
          tile_coords_gather(tile, m_tiles, n_tiles, tm, tn);
        else
          tile_coords(tile, m_tiles, n_tiles, tm, tn);
        const int m0 = tm * kPairBM + static_cast<int>(rank) * kPairHalf;
        const int n0 = tn * TN + static_cast<int>(rank) * L::kBCols;
        if constexpr (GATHER) {
          if (!gather_wait_rows(g, 0, n0, n0 + L::kBCols, s.status) ||
              (DUAL && !gather_wait_rows(g, 1, n0, n0 + L::kBCols, s.status))) {
            ok = false;
            break;
          }
        }
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int i = 0; i < kPairHalf / 64; ++i) tma_load_2d_pair(sa + i * 64 * BK * 2, &tmA, bar, m0 + 64 * i, k0);
          } else {
            tma_load_2d_pair(sa, &tmA, bar, k0, m0);
          }
          int kB;
          const CUtensorMap* mB = b_source(&tmB, &tmB2, DUAL ? 0 : s.k_split, k0, kB);
          if (B_MN) {
#pragma unroll
            for (int i = 0; i < L::kBCols / 64; ++i) {
              tma_load_2d_pair(sb + i * 64 * BK * 2, mB, bar, n0 + 64 * i, kB);
              if (DUAL) tma_load_2d_pair(sb + L::kBBytes + i * 64 * BK * 2, &tmB2, bar, n0 + 64 * i, k0);
            }
          } else {
            tma_load_2d_pair(sb, mB, bar, kB, n0);
            if (DUAL) tma_load_2d_pair(sb + L::kBBytes, &tmB2, bar, k0, n0);
          }
          ++loaded;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every stage this CTA filled must have been consumed before the pair tears down (the MMAs
      // read this CTA's shared memory); bounded waits.
      for (int i = 0; i < STAGES && i < loaded; ++i) {
        const int idx = loaded - 1 - i;
        mbar_wait(&empty[idx % STAGES], (idx / STAGES) & 1, s.status, kErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(kPairBM, TN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, s.status, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * L::kAccCols;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, s.status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? smem_desc(sa + k * 2048, 64 * BK * 2, 1024) : smem_desc(sa + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? smem_desc(sb + k * 2048, 64 * BK * 2, 1024) : smem_desc(sb + k * 32, 16, 1024);
            umma_ss_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            if (DUAL) {
              const uint32_t sb2 = sb + L::kBBytes;
              const uint64_t bdesc2 =
                  B_MN ? smem_desc(sb2 + k * 2048, 64 * BK * 2, 1024) : smem_desc(sb2 + k * 32, 16, 1024);
              umma_ss_pair(d_tmem + TN, adesc, bdesc2, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair(mma_done, 0x1);
      mbar_wait(mma_done, 0, s.status, kErrTimeoutMma);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int sub = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      int tm, tn;
      if constexpr (GATHER)
        tile_coords_gather(tile, m_tiles, n_tiles, tm, tn);
      else
        tile_coords(tile, m_tiles, n_tiles, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, s.status, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + acc * L::kAccCols;
      const int row = tm * kPairBM + static_cast<int>(rank) * kPairHalf + sub * 32 + lane;
      run_epilogue(epi, taddr, row, tn * TN, tm, tn,
                   smem + epi_smem_offset(L::kBarOffset, STAGES) + (threadIdx.x - 64) * EpiSmem<Epi>::kPerThread);
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------------ gather warps (6, 7)
    if constexpr (GATHER) gather_warp<16>(g, lane);  // 8 KB in flight per warp, 296 warps per GPU
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no MMA, commit or remote arrival of either CTA is still in flight
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
  if constexpr (GATHER) {
    if (threadIdx.x == 0) gather_finish(g);
  }
}

}  // namespace gemm
}  // namespace ttb
