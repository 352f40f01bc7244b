// Polynomial attention backward on the tcgen05 tensor cores: two deterministic kernels.
//
//   dP = dO V^T,  H = C * dP  (C = visible * row_scale)
//   signed_product:   dS1 = H * S2,             dS2 = H * S1
//   offset_square:    dS1 = 2 H (S1 + b)                          db  = sum dS1
//   lower_degree_mix: dS1 = H (c1 + c12 S2),    dS2 = H (c2 + c12 S1)
//                     dc0 = sum H, dc1 = sum H S1, dc2 = sum H S2, dc12 = sum H S1 S2
//   dQ = sm * dS K,   dK = sm * dS^T Q,   dV = P^T dO   with P = C * A(S1, S2)
//
// dq kernel  (one CTA per 128 queries): S1, S2, dP tiles of 64 keys in TMEM, dS written to
//            swizzled SMEM as the A operand of dQ1 += dS1 K1 and dQ2 += dS2 K2 (TMEM accumulators).
// dkv kernel (one CTA per 128 keys): the transposed scores S1^T, S2^T, dP^T of 32 queries in TMEM,
//            P^T and dS^T written to 64B-swizzled SMEM, accumulating dV, dK1, dK2 in TMEM (480 of
//            the 512 columns at head dim 128).  Learned kind parameters get per-key-block partial
//            sums reduced later in a fixed order.  Reference: tnlm/kernels/poly_attn.py:78-202.
#include "../common/host.h"
#include "attn_api.h"
#include "poly_common.cuh"

namespace ttb {
namespace attn {

constexpr int kBwdThreads = 320;  // 2 control warps + 8 poly warps (two per TMEM lane quadrant)
constexpr int kBwdPoly = 256;

// ============================================================================ dQ kernel
// Warps: 0 = TMA producer of Q1/Q2/dO (once) and the K1/K2 ring (3 stages), 1 = MMA issuer,
// 2 = TMA producer of the V ring (2 stages), 3..10 = poly warps.  dS1/dS2 go from the poly warps
// straight into tensor memory and are the A operands of dQ1 += dS1 K1, dQ2 += dS2 K2.
constexpr int DQ_BM = 128;  // queries per CTA
constexpr int DQ_BN = 64;   // keys per block
constexpr int kDqKStages = 3;
constexpr int kDqVStages = 2;
constexpr int kDqThreads = 352;
constexpr int kDqFirstPoly = 3;

template <int DK, int DV>
struct DqSmem {
  static constexpr int kQ = DK / 64 * DQ_BM * 128;
  static constexpr int kDO = DV / 64 * DQ_BM * 128;
  static constexpr int kK = DK / 64 * DQ_BN * 128;
  static constexpr int kV = DV / 64 * DQ_BN * 128;
  static constexpr int kKStage = 2 * kK;
  static constexpr int kOffQ1 = 0, kOffQ2 = kQ, kOffDO = 2 * kQ;
  static constexpr int kOffK = 2 * kQ + kDO;
  static constexpr int kOffV = kOffK + kDqKStages * kKStage;
  static constexpr int kOffBar = kOffV + kDqVStages * kV;
  static constexpr int kBytes = (kOffBar + 256 + 1024) > 120 * 1024 ? (kOffBar + 256 + 1024) : 120 * 1024;
};

template <int DK, int DV, int KIND>
__global__ void __launch_bounds__(kDqThreads, 1)
    poly_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                       const __grid_constant__ CUtensorMap tmDO, Params p) {
  using S = DqSmem<DK, DV>;
  constexpr bool kTwo = KIND != 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;    // [3]
  uint64_t* k_empty = bar + 4;   // [3]
  uint64_t* v_full = bar + 7;    // [2]
  uint64_t* v_empty = bar + 9;   // [2]
  uint64_t* sc_full = bar + 11;
  uint64_t* sc_empty = bar + 12;
  uint64_t* ds_full = bar + 13;
  uint64_t* ds_empty = bar + 14;
  uint64_t* acc_full = bar + 15;
  uint64_t* mma_done = bar + 16;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 18);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqb = (p.T + DQ_BM - 1) / DQ_BM;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qb * DQ_BM;
  const long long row0 = static_cast<long long>(b) * p.T;
  const int lo = q0 - p.pos[row0 + q0];
  const int kstart = (lo / DQ_BN) * DQ_BN;
  const int kend = min(q0 + DQ_BM, p.T);
  const int nkb = (kend - kstart + DQ_BN - 1) / DQ_BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kDqKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kDqVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(sc_full, 1);
    mbar_init(sc_empty, kBwdPoly);
    mbar_init(ds_full, kBwdPoly);
    mbar_init(ds_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // TMEM: S1 0, S2 64, dP 128, dS1 192 (bf16 pairs), dS2 224, dQ1 256, dQ2 256+DK
  const uint32_t tS1 = tmem, tS2 = tmem + 64, tDP = tmem + 128, tDS1 = tmem + 192, tDS2 = tmem + 224;
  const uint32_t tDQ1 = tmem + 256, tDQ2 = tmem + 256 + DK;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      prefetch_tmap(&tmDO);
      const int qrow = static_cast<int>(row0 + q0);
      mbar_arrive_expect_tx(q_full, (kTwo ? 2 : 1) * S::kQ + S::kDO);
      for (int i = 0; i < DK / 64; ++i) {
        tma_load_2d(smem + S::kOffQ1 + i * DQ_BM * 128, &tmQ, q_full, p.cq1 + h * DK + 64 * i, qrow);
        if (kTwo) tma_load_2d(smem + S::kOffQ2 + i * DQ_BM * 128, &tmQ, q_full, p.cq2 + h * DK + 64 * i, qrow);
      }
      for (int i = 0; i < DV / 64; ++i)
        tma_load_2d(smem + S::kOffDO + i * DQ_BM * 128, &tmDO, q_full, h * DV + 64 * i, qrow);
      int issued = 0;
      for (int j = 0; j < nkb; ++j) {
        const int st = j % kDqKStages;
        if (!mbar_wait(&k_empty[st], ((j / kDqKStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        uint8_t* sk = smem + S::kOffK + st * S::kKStage;
        const int krow = static_cast<int>(row0 + kstart + j * DQ_BN);
        mbar_arrive_expect_tx(&k_full[st], (kTwo ? 2 : 1) * S::kK);
        for (int i = 0; i < DK / 64; ++i) {
          tma_load_2d(sk + i * DQ_BN * 128, &tmKV, &k_full[st], p.ck1 + h * DK + 64 * i, krow);
          if (kTwo) tma_load_2d(sk + S::kK + i * DQ_BN * 128, &tmKV, &k_full[st], p.ck2 + h * DK + 64 * i, krow);
        }
        issued = j + 1;
      }
      mbar_wait(q_full, 0, p.status, kErrTimeoutProducer);
      for (int j = max(0, issued - kDqKStages); j < issued; ++j)
        mbar_wait(&k_full[j % kDqKStages], (j / kDqKStages) & 1, p.status, kErrTimeoutProducer);
    }
  } else if (warp == 2) {
    if (elect_one()) {
      int issued = 0;
      for (int j = 0; j < nkb; ++j) {
        const int st = j % kDqVStages;
        if (!mbar_wait(&v_empty[st], ((j / kDqVStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        uint8_t* sv = smem + S::kOffV + st * S::kV;
        const int krow = static_cast<int>(row0 + kstart + j * DQ_BN);
        mbar_arrive_expect_tx(&v_full[st], S::kV);
        for (int i = 0; i < DV / 64; ++i)
          tma_load_2d(sv + i * DQ_BN * 128, &tmKV, &v_full[st], p.cv + h * DV + 64 * i, krow);
        issued = j + 1;
      }
      for (int j = max(0, issued - kDqVStages); j < issued; ++j)
        mbar_wait(&v_full[j % kDqVStages], (j / kDqVStages) & 1, p.status, kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, DQ_BN, 0, 0);
      constexpr uint32_t idAcc = idesc_bf16_f32(128, DK, 0, 1);
      const uint32_t sQ1 = smem_u32(smem + S::kOffQ1), sQ2 = smem_u32(smem + S::kOffQ2);
      const uint32_t sDO = smem_u32(smem + S::kOffDO);
      bool ok = mbar_wait(q_full, 0, p.status, kErrTimeoutMma);
      auto accumulate = [&](int i) -> bool {
        const int ks = i % kDqKStages;
        if (!mbar_wait(ds_full, i & 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sK1 = smem_u32(smem + S::kOffK + ks * S::kKStage);
        const uint32_t sK2 = sK1 + S::kK;
#pragma unroll
        for (int k = 0; k < DQ_BN / 16; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          umma_ts(tDQ1, tDS1 + k * 8, mnmajor_desc(sK1, DQ_BN, k), idAcc, acc);
          if (kTwo) umma_ts(tDQ2, tDS2 + k * 8, mnmajor_desc(sK2, DQ_BN, k), idAcc, acc);
        }
        umma_commit(ds_empty);
        umma_commit(&k_empty[ks]);
        return true;
      };
      for (int j = 0; j < nkb && ok; ++j) {
        const int ks = j % kDqKStages, vs = j % kDqVStages;
        if (!mbar_wait(&k_full[ks], (j / kDqKStages) & 1, p.status, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(&v_full[vs], (j / kDqVStages) & 1, p.status, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(sc_empty, (j & 1) ^ 1, p.status, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sK1 = smem_u32(smem + S::kOffK + ks * S::kKStage);
        const uint32_t sK2 = sK1 + S::kK;
        const uint32_t sV = smem_u32(smem + S::kOffV + vs * S::kV);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          umma_ss(tS1, kmajor_desc(sQ1, DQ_BM, k), kmajor_desc(sK1, DQ_BN, k), idS, k > 0 ? 1u : 0u);
          if (kTwo) umma_ss(tS2, kmajor_desc(sQ2, DQ_BM, k), kmajor_desc(sK2, DQ_BN, k), idS, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < DV / 16; ++k)
          umma_ss(tDP, kmajor_desc(sDO, DQ_BM, k), kmajor_desc(sV, DQ_BN, k), idS, k > 0 ? 1u : 0u);
        umma_commit(sc_full);
        umma_commit(&v_empty[vs]);
        if (j > 0 && !accumulate(j - 1)) { ok = false; break; }
      }
      if (ok && accumulate(nkb - 1)) umma_commit(acc_full);
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kErrTimeoutMma);
    }
  } else {
    const int sub = warp & 3;
    const int half = (warp - kDqFirstPoly) >> 2;  // which 32 keys of the 64-key block
    const int r = sub * 32 + lane;
    const int t = q0 + r;
    const bool valid = t < p.T;
    const long long grow = row0 + (valid ? t : q0);
    const int dq = valid ? p.doc[grow] : -1;
    const int dstart = valid ? t - p.pos[grow] : 0;
    const float rs = (valid && dq >= 0) ? p.row_scale[grow] : 0.f;
    float c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = p.par[h * 4 + i];
    const float k0scale = p.sm * p.sm * rs;  // signed_product: dS1 = dP rs (s2 sm) etc., sm folded
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      if (!mbar_wait(sc_full, j & 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      uint32_t a[32], bb[32], g[32];
      tmem_ld32(tS1 + lane_off + half * 32, a);
      if (kTwo) tmem_ld32(tS2 + lane_off + half * 32, bb);
      tmem_ld32(tDP + lane_off + half * 32, g);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(sc_empty);
      const int kb0 = kstart + j * DQ_BN + half * 32;
      const bool full_vis = rs != 0.f && kb0 >= dstart && kb0 + 31 <= t;
      uint32_t d1[16], d2[16];
      if (KIND == 0 && full_vis) {
        // dS1 = H S2 = dP rs sm s2_raw ; the second sm of S2 is folded with the first: scale = sm^2 rs / sm
        const float sc = k0scale / p.sm;
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          const float h0 = __uint_as_float(g[jj]) * sc, h1 = __uint_as_float(g[jj + 1]) * sc;
          d1[jj / 2] = pack_bf16(h0 * __uint_as_float(bb[jj]), h1 * __uint_as_float(bb[jj + 1]));
          d2[jj / 2] = pack_bf16(h0 * __uint_as_float(a[jj]), h1 * __uint_as_float(a[jj + 1]));
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          float o1[2], o2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kt = kb0 + jj + e;
            const bool vis = full_vis || (rs != 0.f && kt <= t && kt >= dstart);
            const float s1 = __uint_as_float(a[jj + e]) * p.sm;
            const float s2 = kTwo ? __uint_as_float(bb[jj + e]) * p.sm : s1;
            const float hh = vis ? __uint_as_float(g[jj + e]) * rs : 0.f;
            if (KIND == 0) {
              o1[e] = hh * s2;
              o2[e] = hh * s1;
            } else if (KIND == 1) {
              o1[e] = 2.f * hh * (s1 + c[0]);
              o2[e] = 0.f;
            } else {
              o1[e] = hh * (c[1] + c[3] * s2);
              o2[e] = hh * (c[2] + c[3] * s1);
            }
          }
          d1[jj / 2] = pack_bf16(o1[0], o1[1]);
          d2[jj / 2] = pack_bf16(o2[0], o2[1]);
        }
      }
      // the dS buffers are free once dQ of block j-1 has completed
      if (!mbar_wait(ds_empty, (j & 1) ^ 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
      tmem_st16(tDS1 + lane_off + half * 16, d1);
      if (kTwo) tmem_st16(tDS2 + lane_off + half * 16, d2);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    if (ok && mbar_wait(acc_full, 0, p.status, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const long long qp = valid ? p.pos[grow] : 0;
      const float* ct = p.rope_cos ? p.rope_cos + qp * (DK / 2) : nullptr;
      const float* st = p.rope_sin ? p.rope_sin + qp * (DK / 2) : nullptr;
      if (half == 0)
        store_row<DK>(tDQ1 + lane_off, p.dq + grow * p.ldd + p.cq1 + h * DK, valid, p.sm, ct, st);
      else if (kTwo)
        store_row<DK>(tDQ2 + lane_off, p.dq + grow * p.ldd + p.cq2 + h * DK, valid, p.sm, ct, st);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ dK/dV kernel
constexpr int KV_BN = 128;  // keys per CTA
constexpr int KV_BM = 32;   // queries per block
constexpr int KV_STAGES = 3;

template <int DK, int DV>
struct DkvSmem {
  static constexpr int kK = DK / 64 * KV_BN * 128;
  static constexpr int kV = DV / 64 * KV_BN * 128;
  static constexpr int kQ = DK / 64 * KV_BM * 128;
  static constexpr int kDO = DV / 64 * KV_BM * 128;
  static constexpr int kStage = 2 * kQ + kDO;
  static constexpr int kT = KV_BN * 64;  // 128 rows x 32 queries bf16 (64-byte rows)
  static constexpr int kTile = 3 * kT;   // P^T, dS1^T, dS2^T
  static constexpr int kOffK1 = 0, kOffK2 = kK, kOffV = 2 * kK;
  static constexpr int kOffStage = 2 * kK + kV;
  static constexpr int kOffT = kOffStage + KV_STAGES * kStage;
  static constexpr int kOffRed = kOffT + 2 * kTile;        // 8 poly warps x 4 floats
  static constexpr int kOffBar = kOffRed + 256;
  static constexpr int kBytes = (kOffBar + 256 + 1024) > 120 * 1024 ? (kOffBar + 256 + 1024) : 120 * 1024;
};

// 64-byte swizzle (Swizzle<2,4,3>): 16-byte chunk c of row r
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t chunk) {
  return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

template <int DK, int DV, int KIND>
__global__ void __launch_bounds__(kBwdThreads, 1)
    poly_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmDO, const int* __restrict__ doc_end, Params p) {
  using S = DkvSmem<DK, DV>;
  constexpr bool kTwo = KIND != 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* k_full = bar + 0;
  uint64_t* q_full = bar + 1;    // [3]
  uint64_t* q_empty = bar + 4;   // [3]
  uint64_t* sc_full = bar + 7;
  uint64_t* sc_empty = bar + 8;
  uint64_t* t_full = bar + 9;    // [2]
  uint64_t* t_empty = bar + 11;  // [2]
  uint64_t* acc_full = bar + 13;
  uint64_t* mma_done = bar + 14;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 16);
  float* red = reinterpret_cast<float*>(smem + S::kOffRed);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int k0 = kb * KV_BN;
  const long long row0 = static_cast<long long>(b) * p.T;
  const int klast = min(k0 + KV_BN, p.T) - 1;
  const int hi = doc_end[row0 + klast];  // exclusive end of the last key's document
  const int nqb = (hi - k0 + KV_BM - 1) / KV_BM;

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(sc_full, 1);
    mbar_init(sc_empty, kBwdPoly);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], kBwdPoly);
      mbar_init(&t_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // TMEM: S1^T 0, S2^T 32, dP^T 64, dV at 128, dK1 at 128+DV, dK2 at 128+DV+DK
  const uint32_t tS1 = tmem, tS2 = tmem + 32, tDP = tmem + 64;
  const uint32_t tDV = tmem + 128, tDK1 = tmem + 128 + DV, tDK2 = tmem + 128 + DV + DK;

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmDO);
      const int krow = static_cast<int>(row0 + k0);
      mbar_arrive_expect_tx(k_full, (kTwo ? 2 : 1) * S::kK + S::kV);
      for (int i = 0; i < DK / 64; ++i) {
        tma_load_2d(smem + S::kOffK1 + i * KV_BN * 128, &tmK, k_full, p.ck1 + h * DK + 64 * i, krow);
        if (kTwo) tma_load_2d(smem + S::kOffK2 + i * KV_BN * 128, &tmK, k_full, p.ck2 + h * DK + 64 * i, krow);
      }
      for (int i = 0; i < DV / 64; ++i)
        tma_load_2d(smem + S::kOffV + i * KV_BN * 128, &tmK, k_full, p.cv + h * DV + 64 * i, krow);
      bool ok = true;
      for (int i = 0; i < nqb && ok; ++i) {
        const int st = i % KV_STAGES;
        if (!mbar_wait(&q_empty[st], ((i / KV_STAGES) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sq = smem + S::kOffStage + st * S::kStage;
        const int qrow = static_cast<int>(row0 + k0 + i * KV_BM);
        mbar_arrive_expect_tx(&q_full[st], (kTwo ? 2 : 1) * S::kQ + S::kDO);
        for (int c = 0; c < DK / 64; ++c) {
          tma_load_2d(sq + c * KV_BM * 128, &tmQ, &q_full[st], p.cq1 + h * DK + 64 * c, qrow);
          if (kTwo) tma_load_2d(sq + S::kQ + c * KV_BM * 128, &tmQ, &q_full[st], p.cq2 + h * DK + 64 * c, qrow);
        }
        for (int c = 0; c < DV / 64; ++c)
          tma_load_2d(sq + 2 * S::kQ + c * KV_BM * 128, &tmDO, &q_full[st], h * DV + 64 * c, qrow);
      }
      mbar_wait(k_full, 0, p.status, kErrTimeoutProducer);
      if (!ok)
        for (int i = max(0, nqb - KV_STAGES); i < nqb; ++i)
          mbar_wait(&q_full[i % KV_STAGES], (i / KV_STAGES) & 1, p.status, kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, KV_BM, 0, 0);
      constexpr uint32_t idDV = idesc_bf16_f32(128, DV, 0, 1);
      constexpr uint32_t idDK = idesc_bf16_f32(128, DK, 0, 1);
      const uint32_t sK1 = smem_u32(smem + S::kOffK1), sK2 = smem_u32(smem + S::kOffK2);
      const uint32_t sV = smem_u32(smem + S::kOffV);
      bool ok = mbar_wait(k_full, 0, p.status, kErrTimeoutMma);
      auto accumulate = [&](int i) -> bool {
        const int tb = i & 1;
        if (!mbar_wait(&t_full[tb], (i >> 1) & 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + S::kOffStage + (i % KV_STAGES) * S::kStage);
        const uint32_t sT = smem_u32(smem + S::kOffT + tb * S::kTile);
#pragma unroll
        for (int k = 0; k < KV_BM / 16; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          // A tiles (128 keys x 32 queries, 64-byte swizzle): P^T, dS1^T, dS2^T
          const uint64_t aP = smem_desc(sT + k * 32, 16, 512, 4);
          const uint64_t a1 = smem_desc(sT + S::kT + k * 32, 16, 512, 4);
          const uint64_t a2 = smem_desc(sT + 2 * S::kT + k * 32, 16, 512, 4);
          umma_ss(tDV, aP, mnmajor_desc(sq + 2 * S::kQ, KV_BM, k), idDV, acc);
          umma_ss(tDK1, a1, mnmajor_desc(sq, KV_BM, k), idDK, acc);
          if (kTwo) umma_ss(tDK2, a2, mnmajor_desc(sq + S::kQ, KV_BM, k), idDK, acc);
        }
        umma_commit(&t_empty[tb]);
        umma_commit(&q_empty[i % KV_STAGES]);
        return true;
      };
      for (int i = 0; i < nqb && ok; ++i) {
        const int st = i % KV_STAGES;
        if (!mbar_wait(&q_full[st], (i / KV_STAGES) & 1, p.status, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(sc_empty, (i & 1) ^ 1, p.status, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + S::kOffStage + st * S::kStage);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          umma_ss(tS1, kmajor_desc(sK1, KV_BN, k), kmajor_desc(sq, KV_BM, k), idS, k > 0 ? 1u : 0u);
          if (kTwo) umma_ss(tS2, kmajor_desc(sK2, KV_BN, k), kmajor_desc(sq + S::kQ, KV_BM, k), idS, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < DV / 16; ++k)
          umma_ss(tDP, kmajor_desc(sV, KV_BN, k), kmajor_desc(sq + 2 * S::kQ, KV_BM, k), idS, k > 0 ? 1u : 0u);
        umma_commit(sc_full);
        if (i > 0 && !accumulate(i - 1)) { ok = false; break; }
      }
      if (ok && nqb > 0 && accumulate(nqb - 1)) umma_commit(acc_full);
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kErrTimeoutMma);
    }
  } else {
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;  // which 16 queries of the 32-query block
    const int pw = warp - 2;           // poly warp index 0..7
    const int r = sub * 32 + lane;     // key row
    const int kt = k0 + r;
    const bool kvalid = kt < p.T;
    const long long krow = row0 + (kvalid ? kt : k0);
    const bool kreal = kvalid && p.doc[krow] >= 0;
    const int kend = kreal ? doc_end[krow] : kt;  // queries of the same document: [kt, kend)
    float c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = p.par[h * 4 + i];
    float g0 = 0.f, g1 = 0.f, g2 = 0.f, g12 = 0.f;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    bool ok = true;
    // row scales of this thread's 16 queries, loaded for block i+1 while block i is processed
    auto load_rs = [&](int i, float (&dst)[16]) {
      const int q = k0 + i * KV_BM + half * 16;
      const float* src = p.row_scale + row0 + q;
      if (q + 15 < p.T && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(src) + v);
          dst[v * 4 + 0] = f.x; dst[v * 4 + 1] = f.y; dst[v * 4 + 2] = f.z; dst[v * 4 + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) dst[e] = (q + e < p.T) ? __ldg(src + e) : 0.f;
      }
    };
    float rs_next[16];
    if (nqb > 0) load_rs(0, rs_next);
    for (int i = 0; i < nqb && ok; ++i) {
      float rsv[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) rsv[e] = rs_next[e];
      if (i + 1 < nqb) load_rs(i + 1, rs_next);
      if (!mbar_wait(sc_full, i & 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      uint32_t a[16], bb[16], g[16];
      tmem_ld16(tS1 + lane_off + half * 16, a);
      if (kTwo) tmem_ld16(tS2 + lane_off + half * 16, bb);
      tmem_ld16(tDP + lane_off + half * 16, g);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(sc_empty);
      const int qb0 = k0 + i * KV_BM + half * 16;
      const bool full_vis = kreal && qb0 >= kt && qb0 + 15 < kend;
      uint32_t pp[8], d1[8], d2[8];
#pragma unroll
      for (int jj = 0; jj < 16; jj += 2) {
        float vp[2], o1[2], o2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int qt = qb0 + jj + e;
          const bool vis = full_vis || (kreal && qt >= kt && qt < kend);
          const float rs = vis ? rsv[jj + e] : 0.f;
          const float s1 = __uint_as_float(a[jj + e]) * p.sm;
          const float s2 = kTwo ? __uint_as_float(bb[jj + e]) * p.sm : s1;
          const float hh = __uint_as_float(g[jj + e]) * rs;
          vp[e] = rs * poly<KIND>(s1, s2, c);
          if (KIND == 0) {
            o1[e] = hh * s2;
            o2[e] = hh * s1;
          } else if (KIND == 1) {
            o1[e] = 2.f * hh * (s1 + c[0]);
            o2[e] = 0.f;
            g0 += o1[e];
          } else {
            o1[e] = hh * (c[1] + c[3] * s2);
            o2[e] = hh * (c[2] + c[3] * s1);
            g0 += hh;
            g1 += hh * s1;
            g2 += hh * s2;
            g12 += hh * s1 * s2;
          }
        }
        pp[jj / 2] = pack_bf16(vp[0], vp[1]);
        d1[jj / 2] = pack_bf16(o1[0], o1[1]);
        d2[jj / 2] = pack_bf16(o2[0], o2[1]);
      }
      const int tb = i & 1;
      if (!mbar_wait(&t_empty[tb], ((i >> 1) & 1) ^ 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
      uint8_t* tp = smem + S::kOffT + tb * S::kTile;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        const uint32_t off = sw64_offset(r, half * 2 + ch);
        *reinterpret_cast<uint4*>(tp + off) = make_uint4(pp[ch * 4], pp[ch * 4 + 1], pp[ch * 4 + 2], pp[ch * 4 + 3]);
        *reinterpret_cast<uint4*>(tp + S::kT + off) =
            make_uint4(d1[ch * 4], d1[ch * 4 + 1], d1[ch * 4 + 2], d1[ch * 4 + 3]);
        if (kTwo)
          *reinterpret_cast<uint4*>(tp + 2 * S::kT + off) =
              make_uint4(d2[ch * 4], d2[ch * 4 + 1], d2[ch * 4 + 2], d2[ch * 4 + 3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&t_full[tb]);
    }
    // kind-parameter partials: fixed-order reduction over the 256 poly threads of this key block
    if (KIND != 0 && p.dpar != nullptr) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        g0 += __shfl_xor_sync(0xffffffffu, g0, o);
        g1 += __shfl_xor_sync(0xffffffffu, g1, o);
        g2 += __shfl_xor_sync(0xffffffffu, g2, o);
        g12 += __shfl_xor_sync(0xffffffffu, g12, o);
      }
      if (lane == 0) {
        red[pw * 4 + 0] = g0;
        red[pw * 4 + 1] = g1;
        red[pw * 4 + 2] = g2;
        red[pw * 4 + 3] = g12;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (pw == 0 && lane < 4) {
        float sum = 0.f;
        for (int w8 = 0; w8 < 8; ++w8) sum += red[w8 * 4 + lane];
        p.dpar[(static_cast<long long>(bh) * p.dpar_blocks + kb) * 4 + lane] = sum;
      }
    }
    if (ok && nqb > 0 && mbar_wait(acc_full, 0, p.status, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const long long kp = kvalid ? p.pos[krow] : 0;
      const float* ct = p.rope_cos ? p.rope_cos + kp * (DK / 2) : nullptr;
      const float* st = p.rope_sin ? p.rope_sin + kp * (DK / 2) : nullptr;
      if (half == 0) {
        store_row<DV>(tDV + lane_off, p.dq + krow * p.ldd + p.cv + h * DV, kvalid, 1.f, nullptr, nullptr);
        if (kTwo) store_row<DK>(tDK2 + lane_off, p.dq + krow * p.ldd + p.ck2 + h * DK, kvalid, p.sm, ct, st);
      } else {
        store_row<DK>(tDK1 + lane_off, p.dq + krow * p.ldd + p.ck1 + h * DK, kvalid, p.sm, ct, st);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int DK, int DV, int KIND>
void launch_bwd(const void* qkv, long long ld, const void* dout, long long ldo, const int* doc_end, long long rows,
                const Params& p, cudaStream_t stream) {
  {
    using S = DqSmem<DK, DV>;
    const CUtensorMap tq = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, DQ_BM);
    const CUtensorMap tkv = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, DQ_BN);
    const CUtensorMap tdo = make_tmap_2d(dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ldo, rows, ldo, 64, DQ_BM);
    auto kern = poly_bwd_dq_kernel<DK, DV, KIND>;
    static bool configured = false;
    if (!configured) {
      TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
      configured = true;
    }
    dim3 grid((p.T + DQ_BM - 1) / DQ_BM, p.B * p.H);
    kern<<<grid, kDqThreads, S::kBytes, stream>>>(tq, tkv, tdo, p);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
  {
    using S = DkvSmem<DK, DV>;
    const CUtensorMap tk = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, KV_BN);
    const CUtensorMap tq = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, KV_BM);
    const CUtensorMap tdo = make_tmap_2d(dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ldo, rows, ldo, 64, KV_BM);
    auto kern = poly_bwd_dkv_kernel<DK, DV, KIND>;
    static bool configured = false;
    if (!configured) {
      TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
      configured = true;
    }
    dim3 grid((p.T + KV_BN - 1) / KV_BN, p.B * p.H);
    kern<<<grid, kBwdThreads, S::kBytes, stream>>>(tk, tq, tdo, doc_end, p);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace attn

int poly_attention_dpar_blocks(int T) { return (T + attn::KV_BN - 1) / attn::KV_BN; }

void poly_attention_bwd(int kind, int dk, int dv, const void* qkv, long long ld, const void* dout, long long ldo,
                        const int* doc_end, attn::Params p, cudaStream_t stream) {
  TTB_CHECK((dk == 64 || dk == 128) && (dv == 64 || dv == 128), "poly attention: head dims must be 64 or 128");
  const long long rows = static_cast<long long>(p.B) * p.T;
  p.status = status_ptr();
  p.dpar_blocks = poly_attention_dpar_blocks(p.T);
#define TTB_BWD(DK_, DV_, K_)                                                                         \
  if (dk == DK_ && dv == DV_ && kind == K_)                                                          \
    return attn::launch_bwd<DK_, DV_, K_>(qkv, ld, dout, ldo, doc_end, rows, p, stream);
  TTB_BWD(64, 64, 0) TTB_BWD(64, 64, 1) TTB_BWD(64, 64, 2)
  TTB_BWD(128, 128, 0) TTB_BWD(128, 128, 1) TTB_BWD(128, 128, 2)
  TTB_BWD(64, 128, 0) TTB_BWD(64, 128, 1) TTB_BWD(64, 128, 2)
  TTB_BWD(128, 64, 0) TTB_BWD(128, 64, 1) TTB_BWD(128, 64, 2)
#undef TTB_BWD
  TTB_CHECK(false, "poly attention backward: unsupported configuration");
}

}  // namespace ttb
