// Polynomial attention backward on the tcgen05 tensor cores: two deterministic kernels.
//
//   dP = dO V^T,  H = C * dP  (C = visible * row_scale)
//   signed_product:   dS1 = H * S2,             dS2 = H * S1
//   offset_square:    dS1 = 2 H (S1 + b)                          db  = sum dS1
//   lower_degree_mix: dS1 = H (c1 + c12 S2),    dS2 = H (c2 + c12 S1)
//                     dc0 = sum H, dc1 = sum H S1, dc2 = sum H S2, dc12 = sum H S1 S2
//   dQ = sm * dS K,   dK = sm * dS^T Q,   dV = P^T dO   with P = C * A(S1, S2)
//
// Both kernels are persistent (one CTA per SM working through tiles of 128 queries or 128 keys
// taken from a device counter) with a dedicated epilogue warpgroup, so one tile's accumulator drain
// and the next tile's operand loads overlap the tensor-core work.
// dq kernel:  S1, S2, dP tiles of 64 keys in TMEM, dS written back into TMEM as the A operand of
//             dQ1 += dS1 K1 and dQ2 += dS2 K2 (TMEM accumulators).
// dkv kernel: the transposed scores S1^T, S2^T, dP^T of 32 queries in TMEM, P^T and dS^T written
//             to 64B-swizzled SMEM, accumulating dV, dK1, dK2 in TMEM (384 columns; 480 of the 512 with the scores, at
//             head dim 128).  Learned kind parameters get per-key-block partial sums reduced later
//             in a fixed order.  Reference: tnlm/kernels/poly_attn.py:78-202.
#include "../common/host.h"
#include "attn_api.h"
#include "poly_common.cuh"

namespace ttb {
namespace attn {

constexpr int kBwdPoly = 256;

// ============================================================================ dQ kernel
// Persistent: one CTA per SM takes (batch, head, 128-query) tiles from the dynamic scheduler in
// grid order (the query tiles of one head in a row, so that head's K and V stay in L2).
// Warpgroup 0: warp 0 = tile fetch + TMA producer of Q1/Q2/dO (once per tile) and the K1/K2 ring
// (3 stages), warp 1 = MMA issuer, warp 2 = TMA producer of the V ring (2 stages).  Warpgroups 1-2
// = poly warps: dS1/dS2 go from them straight into tensor memory and are the A operands of
// dQ1 += dS1 K1, dQ2 += dS2 K2.  Warpgroup 3 = epilogue: drains dQ of tile n (inverse RoPE,
// bf16) while tile n+1's Q load, score MMAs and first poly pass run; tile n+1's first dQ MMA
// waits for the drain.  The Q/dO buffer is reloaded as soon as tile n's last score MMAs finish.
constexpr int DQ_BM = 128;  // queries per tile
constexpr int DQ_BN = 64;   // keys per block
constexpr int kDqKStages = 3;
constexpr int kDqVStages = 2;
constexpr int kDqThreads = 512;
constexpr int kDqFirstPoly = 4;
constexpr int kDqFirstEpi = 12;
constexpr int kDqTileReaders = 1 + 1 + 8 + 4;  // V producer, MMA issuer, poly warps, epilogue warps
// Register split: 512 threads launch with 128 each (65536).  The control warpgroup keeps 80 (below
// that the MMA issuer and the producers spill), the poly warpgroups get 152 (their fp32 score
// slices are the largest live state), the epilogue keeps 128.
constexpr int kDqLaunchRegs = 128, kDqCtrlRegs = 80, kDqPolyRegs = 152, kDqEpiRegs = 128;
static_assert(128 * kDqCtrlRegs + 256 * kDqPolyRegs + 128 * kDqEpiRegs <= kDqThreads * kDqLaunchRegs,
              "dq register split exceeds the launch allocation");

// Scheduler counters of the dq kernel (next tile, finished CTAs); zero between launches.
__device__ unsigned int g_dq_sched[2];

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

struct DqTile {
  int q0, h, kstart, nkb;
  long long row0;
};

// Tile t of the grid-ordered sequence: head-major, heaviest (last) query block of a head first.
__device__ __forceinline__ DqTile dq_tile(int t, int nqb, const Params& p) {
  DqTile d;
  const int bh = t / nqb;
  const int qb = nqb - 1 - (t - bh * nqb);
  const int b = bh / p.H;
  d.h = bh - b * p.H;
  d.q0 = qb * DQ_BM;
  d.row0 = static_cast<long long>(b) * p.T;
  const int lo = d.q0 - p.pos[d.row0 + d.q0];  // start of the first query's document
  d.kstart = (lo / DQ_BN) * DQ_BN;
  const int kend = min(d.q0 + DQ_BM, p.T);
  d.nkb = (kend - d.kstart + DQ_BN - 1) / DQ_BN;
  return d;
}

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
  uint64_t* k_full = bar + 1;      // [3]
  uint64_t* k_empty = bar + 4;     // [3]
  uint64_t* v_full = bar + 7;      // [2]
  uint64_t* v_empty = bar + 9;     // [2]
  uint64_t* sc_full = bar + 11;
  uint64_t* sc_empty = bar + 12;
  uint64_t* ds_full = bar + 13;
  uint64_t* ds_empty = bar + 14;
  uint64_t* acc_full = bar + 15;   // dQ of the tile is complete in TMEM
  uint64_t* acc_empty = bar + 16;  // the epilogue has read dQ out of TMEM
  uint64_t* q_empty = bar + 17;    // the tile's score MMAs no longer read Q/dO
  uint64_t* tile_full = bar + 18;  // [2] tile id published
  uint64_t* tile_empty = bar + 20; // [2] tile id read by every role
  uint64_t* mma_done = bar + 22;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 23);
  int* tile_ids = reinterpret_cast<int*>(bar + 24);  // [2]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqb = (p.T + DQ_BM - 1) / DQ_BM;
  const int ntiles = nqb * p.B * p.H;

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
    mbar_init(acc_empty, 128);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tile_full[i], 1);
      mbar_init(&tile_empty[i], kDqTileReaders);
    }
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

  // Tile n of this CTA (bounded wait); -1 when the wait gave up.
  auto read_tile = [&](int n, uint32_t code) -> int {
    if (!mbar_wait(&tile_full[n & 1], (n >> 1) & 1, p.status, code)) return -1;
    return *reinterpret_cast<volatile int*>(&tile_ids[n & 1]);
  };

  if (warp < kDqFirstPoly) {
    reg_dealloc<kDqCtrlRegs>();
    if (warp == 0 && elect_one()) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      prefetch_tmap(&tmDO);
      uint32_t gj = 0;  // key blocks issued over all tiles
      int nq = 0;       // Q/dO loads issued
      for (int n = 0;; ++n) {
        if (!mbar_wait(&tile_empty[n & 1], ((n >> 1) & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int t = static_cast<int>(atomicAdd(&g_dq_sched[0], 1u));
        tile_ids[n & 1] = t;
        mbar_arrive(&tile_full[n & 1]);
        if (t >= ntiles) break;
        const DqTile d = dq_tile(t, nqb, p);
        if (!mbar_wait(q_empty, (n & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int qrow = static_cast<int>(d.row0 + d.q0);
        mbar_arrive_expect_tx(q_full, (kTwo ? 2 : 1) * S::kQ + S::kDO);
        for (int i = 0; i < DK / 64; ++i) {
          tma_load_2d(smem + S::kOffQ1 + i * DQ_BM * 128, &tmQ, q_full, p.cq1 + d.h * DK + 64 * i, qrow);
          if (kTwo) tma_load_2d(smem + S::kOffQ2 + i * DQ_BM * 128, &tmQ, q_full, p.cq2 + d.h * DK + 64 * i, qrow);
        }
        for (int i = 0; i < DV / 64; ++i)
          tma_load_2d(smem + S::kOffDO + i * DQ_BM * 128, &tmDO, q_full, d.h * DV + 64 * i, qrow);
        ++nq;
        bool ok = true;
        for (int j = 0; j < d.nkb; ++j, ++gj) {
          const int st = gj % kDqKStages;
          if (!mbar_wait(&k_empty[st], ((gj / kDqKStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sk = smem + S::kOffK + st * S::kKStage;
          const int krow = static_cast<int>(d.row0 + d.kstart + j * DQ_BN);
          mbar_arrive_expect_tx(&k_full[st], (kTwo ? 2 : 1) * S::kK);
          for (int i = 0; i < DK / 64; ++i) {
            tma_load_2d(sk + i * DQ_BN * 128, &tmKV, &k_full[st], p.ck1 + d.h * DK + 64 * i, krow);
            if (kTwo) tma_load_2d(sk + S::kK + i * DQ_BN * 128, &tmKV, &k_full[st], p.ck2 + d.h * DK + 64 * i, krow);
          }
        }
        if (!ok) break;
      }
      // every issued copy has landed before the CTA may exit
      if (nq > 0) mbar_wait(q_full, (nq - 1) & 1, p.status, kErrTimeoutProducer);
      for (uint32_t g = gj > kDqKStages ? gj - kDqKStages : 0; g < gj; ++g)
        mbar_wait(&k_full[g % kDqKStages], (g / kDqKStages) & 1, p.status, kErrTimeoutProducer);
    } else if (warp == 2 && elect_one()) {
      uint32_t gj = 0;
      for (int n = 0;; ++n) {
        const int t = read_tile(n, kErrTimeoutProducer);
        if (t < 0) break;
        mbar_arrive(&tile_empty[n & 1]);
        if (t >= ntiles) break;
        const DqTile d = dq_tile(t, nqb, p);
        bool ok = true;
        for (int j = 0; j < d.nkb; ++j, ++gj) {
          const int st = gj % kDqVStages;
          if (!mbar_wait(&v_empty[st], ((gj / kDqVStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sv = smem + S::kOffV + st * S::kV;
          const int krow = static_cast<int>(d.row0 + d.kstart + j * DQ_BN);
          mbar_arrive_expect_tx(&v_full[st], S::kV);
          for (int i = 0; i < DV / 64; ++i)
            tma_load_2d(sv + i * DQ_BN * 128, &tmKV, &v_full[st], p.cv + d.h * DV + 64 * i, krow);
        }
        if (!ok) break;
      }
      for (uint32_t g = gj > kDqVStages ? gj - kDqVStages : 0; g < gj; ++g)
        mbar_wait(&v_full[g % kDqVStages], (g / kDqVStages) & 1, p.status, kErrTimeoutProducer);
    } else if (warp == 1 && elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, DQ_BN, 0, 0);
      constexpr uint32_t idAcc = idesc_bf16_f32(128, DK, 0, 1);
      const uint32_t sQ1 = smem_u32(smem + S::kOffQ1), sQ2 = smem_u32(smem + S::kOffQ2);
      const uint32_t sDO = smem_u32(smem + S::kOffDO);
      // dQ += dS K of global key block g; the first block of tile n overwrites the accumulators once
      // the epilogue has read tile n-1's out
      auto accumulate = [&](uint32_t g, bool first, int n) -> bool {
        const int ks = g % kDqKStages;
        if (!mbar_wait(ds_full, g & 1, p.status, kErrTimeoutMma)) return false;
        if (first && !mbar_wait(acc_empty, (n & 1) ^ 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sK1 = smem_u32(smem + S::kOffK + ks * S::kKStage);
        const uint32_t sK2 = sK1 + S::kK;
#pragma unroll
        for (int k = 0; k < DQ_BN / 16; ++k) {
          const uint32_t acc = (!first || k > 0) ? 1u : 0u;
          umma_ts(tDQ1, tDS1 + k * 8, mnmajor_desc(sK1, DQ_BN, k), idAcc, acc);
          if (kTwo) umma_ts(tDQ2, tDS2 + k * 8, mnmajor_desc(sK2, DQ_BN, k), idAcc, acc);
        }
        umma_commit(ds_empty);
        umma_commit(&k_empty[ks]);
        return true;
      };
      uint32_t gj = 0;
      for (int n = 0;; ++n) {
        const int t = read_tile(n, kErrTimeoutMma);
        if (t < 0) break;
        mbar_arrive(&tile_empty[n & 1]);
        if (t >= ntiles) break;
        const DqTile d = dq_tile(t, nqb, p);
        if (!mbar_wait(q_full, n & 1, p.status, kErrTimeoutMma)) break;
        bool ok = true;
        for (int j = 0; j < d.nkb; ++j, ++gj) {
          const int ks = gj % kDqKStages, vs = gj % kDqVStages;
          if (!mbar_wait(&k_full[ks], (gj / kDqKStages) & 1, p.status, kErrTimeoutMma) ||
              !mbar_wait(&v_full[vs], (gj / kDqVStages) & 1, p.status, kErrTimeoutMma) ||
              !mbar_wait(sc_empty, (gj & 1) ^ 1, p.status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
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
          if (j == d.nkb - 1) umma_commit(q_empty);
          if (j > 0 && !accumulate(gj - 1, j == 1, n)) {
            ok = false;
            break;
          }
        }
        if (!ok || !accumulate(gj - 1, d.nkb == 1, n)) break;
        umma_commit(acc_full);
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kErrTimeoutMma);
    }
  } else if (warp < kDqFirstEpi) {
    reg_alloc<kDqPolyRegs>();
    const int sub = warp & 3;
    const int half = (warp - kDqFirstPoly) >> 2;  // which 32 keys of the 64-key block
    const int r = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    uint32_t gj = 0;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      const int t = read_tile(n, kErrTimeoutEpilogue);
      __syncwarp();
      if (t < 0) break;
      if (lane == 0) mbar_arrive(&tile_empty[n & 1]);
      if (t >= ntiles) break;
      const DqTile d = dq_tile(t, nqb, p);
      const int tq = d.q0 + r;
      const bool valid = tq < p.T;
      const long long grow = d.row0 + (valid ? tq : d.q0);
      const int dq = valid ? p.doc[grow] : -1;
      const int dstart = valid ? tq - p.pos[grow] : 0;
      const float rs = (valid && dq >= 0) ? p.row_scale[grow] : 0.f;
      float c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] = p.par[d.h * 4 + i];
      const float k0scale = p.sm * rs;  // signed_product: dS1 = dP rs s2 = dP (rs sm) s2_raw
      for (int j = 0; j < d.nkb; ++j, ++gj) {
        if (!mbar_wait(sc_full, gj & 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
        uint32_t a[32], bb[32], g[32];
        tmem_ld32(tS1 + lane_off + half * 32, a);
        if (kTwo) tmem_ld32(tS2 + lane_off + half * 32, bb);
        tmem_ld32(tDP + lane_off + half * 32, g);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(sc_empty);
        const int kb0 = d.kstart + j * DQ_BN + half * 32;
        const bool full_vis = rs != 0.f && kb0 >= dstart && kb0 + 31 <= tq;
        uint32_t d1[16], d2[16];
        if (KIND == 0 && full_vis) {
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            const float h0 = __uint_as_float(g[jj]) * k0scale, h1 = __uint_as_float(g[jj + 1]) * k0scale;
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
              const bool vis = full_vis || (rs != 0.f && kt <= tq && kt >= dstart);
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
        // the dS buffers are free once dQ of the previous block has completed
        if (!mbar_wait(ds_empty, (gj & 1) ^ 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
        tmem_st16(tDS1 + lane_off + half * 16, d1);
        if (kTwo) tmem_st16(tDS2 + lane_off + half * 16, d2);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(ds_full);
      }
    }
  } else {
    if constexpr (kDqEpiRegs < kDqLaunchRegs) reg_dealloc<kDqEpiRegs>();
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    for (int n = 0;; ++n) {
      const int t = read_tile(n, kErrTimeoutEpilogue);
      __syncwarp();
      if (t < 0) break;
      if (lane == 0) mbar_arrive(&tile_empty[n & 1]);
      if (t >= ntiles) break;
      const DqTile d = dq_tile(t, nqb, p);
      const int tq = d.q0 + r;
      const bool valid = tq < p.T;
      const long long grow = d.row0 + (valid ? tq : d.q0);
      const long long qp = valid ? p.pos[grow] : 0;
      const float* ct = p.rope_cos ? p.rope_cos + qp * (DK / 2) : nullptr;
      const float* st = p.rope_sin ? p.rope_sin + qp * (DK / 2) : nullptr;
      float cs[16], sn[16];
      if (ct != nullptr) rope_fetch16(ct, st, 0, cs, sn);  // in flight while dQ completes
      if (!mbar_wait(acc_full, n & 1, p.status, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      __nv_bfloat16* dst1 = p.dq + grow * p.ldd + p.cq1 + d.h * DK;
      __nv_bfloat16* dst2 = p.dq + grow * p.ldd + p.cq2 + d.h * DK;
      if (ct != nullptr && kTwo) {
        const uint32_t acc[2] = {tDQ1 + lane_off, tDQ2 + lane_off};
        __nv_bfloat16* const out[2] = {dst1, dst2};
        store_rows_rope<DK, 2>(acc, out, valid, p.sm, ct, st, cs, sn);
      } else if (ct != nullptr) {
        const uint32_t acc[1] = {tDQ1 + lane_off};
        __nv_bfloat16* const out[1] = {dst1};
        store_rows_rope<DK, 1>(acc, out, valid, p.sm, ct, st, cs, sn);
      } else {
        store_row_lean<DK>(tDQ1 + lane_off, dst1, valid, p.sm);
        if (kTwo) store_row_lean<DK>(tDQ2 + lane_off, dst2, valid, p.sm);
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) sched_finish(g_dq_sched);
}

// ============================================================================ dK/dV kernel
// Persistent like the dq kernel, over (batch, head, 128-key) tiles.  Warpgroup 0: warp 0 = tile
// fetch + TMA producer of K1/K2/V (once per tile) and the Q1/Q2/dO ring, warp 1 = MMA issuer.
// Warpgroups 1-2 = poly warps (P^T, dS1^T, dS2^T into swizzled SMEM); warpgroup 3 = epilogue
// (dV, dK1, dK2 out of TMEM while the next tile's scores run).
constexpr int KV_BN = 128;  // keys per tile
constexpr int KV_BM = 32;   // queries per block
constexpr int KV_STAGES = 3;
constexpr int kKvThreads = 512;
constexpr int kKvFirstPoly = 4;
constexpr int kKvFirstEpi = 12;
constexpr int kKvTileReaders = 1 + 8 + 4;  // MMA issuer, poly warps, epilogue warps
constexpr int kKvLaunchRegs = 128, kKvCtrlRegs = 80, kKvPolyRegs = 152, kKvEpiRegs = 128;
static_assert(128 * kKvCtrlRegs + 256 * kKvPolyRegs + 128 * kKvEpiRegs <= kKvThreads * kKvLaunchRegs,
              "dkv register split exceeds the launch allocation");

// Scheduler counters of the dkv kernel (next tile, finished CTAs); zero between launches.
__device__ unsigned int g_dkv_sched[2];

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
  static constexpr int kOffRed = kOffT + 2 * kTile;        // 2 x (8 poly warps x 4 floats)
  static constexpr int kOffBar = kOffRed + 256;
  static constexpr int kBytes = (kOffBar + 256 + 1024) > 120 * 1024 ? (kOffBar + 256 + 1024) : 120 * 1024;
};

// 64-byte swizzle (Swizzle<2,4,3>): 16-byte chunk c of row r
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t chunk) {
  return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

struct KvTile {
  int k0, h, kb, bh, nqb;
  long long row0;
};

// Tile t in grid order: head-major, the key block with the most queries (the first) first.
__device__ __forceinline__ KvTile kv_tile(int t, int nkt, const int* __restrict__ doc_end, const Params& p) {
  KvTile d;
  d.bh = t / nkt;
  d.kb = t - d.bh * nkt;
  const int b = d.bh / p.H;
  d.h = d.bh - b * p.H;
  d.k0 = d.kb * KV_BN;
  d.row0 = static_cast<long long>(b) * p.T;
  const int klast = min(d.k0 + KV_BN, p.T) - 1;
  const int hi = doc_end[d.row0 + klast];  // exclusive end of the last key's document (> klast)
  d.nqb = max(1, (hi - d.k0 + KV_BM - 1) / KV_BM);
  return d;
}

template <int DK, int DV, int KIND>
__global__ void __launch_bounds__(kKvThreads, 1)
    poly_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmDO, const int* __restrict__ doc_end, Params p) {
  using S = DkvSmem<DK, DV>;
  constexpr bool kTwo = KIND != 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* kv_full = bar + 0;
  uint64_t* q_full = bar + 1;      // [3]
  uint64_t* q_empty = bar + 4;     // [3]
  uint64_t* sc_full = bar + 7;
  uint64_t* sc_empty = bar + 8;
  uint64_t* t_full = bar + 9;      // [2]
  uint64_t* t_empty = bar + 11;    // [2]
  uint64_t* acc_full = bar + 13;
  uint64_t* mma_done = bar + 14;
  uint64_t* acc_empty = bar + 15;
  uint64_t* kv_empty = bar + 16;   // the tile's score MMAs no longer read K/V
  uint64_t* tile_full = bar + 17;  // [2]
  uint64_t* tile_empty = bar + 19; // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 21);
  int* tile_ids = reinterpret_cast<int*>(bar + 22);  // [2]
  uint64_t* red_full = bar + 23;   // [2] the poly warps' kind-parameter partials of a tile are in SMEM

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkt = (p.T + KV_BN - 1) / KV_BN;
  const int ntiles = nkt * p.B * p.H;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(sc_full, 1);
    mbar_init(sc_empty, kBwdPoly);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], kBwdPoly);
      mbar_init(&t_empty[i], 1);
      mbar_init(&tile_full[i], 1);
      mbar_init(&tile_empty[i], kKvTileReaders);
      mbar_init(&red_full[i], 8);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(acc_empty, 128);
    mbar_init(kv_empty, 1);
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

  auto read_tile = [&](int n, uint32_t code) -> int {
    if (!mbar_wait(&tile_full[n & 1], (n >> 1) & 1, p.status, code)) return -1;
    return *reinterpret_cast<volatile int*>(&tile_ids[n & 1]);
  };

  if (warp < kKvFirstPoly) {
    reg_dealloc<kKvCtrlRegs>();
    if (warp == 0 && elect_one()) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmDO);
      uint32_t gi = 0;  // query blocks issued over all tiles
      int nkv = 0;      // K/V loads issued
      for (int n = 0;; ++n) {
        if (!mbar_wait(&tile_empty[n & 1], ((n >> 1) & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int t = static_cast<int>(atomicAdd(&g_dkv_sched[0], 1u));
        tile_ids[n & 1] = t;
        mbar_arrive(&tile_full[n & 1]);
        if (t >= ntiles) break;
        const KvTile d = kv_tile(t, nkt, doc_end, p);
        if (!mbar_wait(kv_empty, (n & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int krow = static_cast<int>(d.row0 + d.k0);
        mbar_arrive_expect_tx(kv_full, (kTwo ? 2 : 1) * S::kK + S::kV);
        for (int i = 0; i < DK / 64; ++i) {
          tma_load_2d(smem + S::kOffK1 + i * KV_BN * 128, &tmK, kv_full, p.ck1 + d.h * DK + 64 * i, krow);
          if (kTwo) tma_load_2d(smem + S::kOffK2 + i * KV_BN * 128, &tmK, kv_full, p.ck2 + d.h * DK + 64 * i, krow);
        }
        for (int i = 0; i < DV / 64; ++i)
          tma_load_2d(smem + S::kOffV + i * KV_BN * 128, &tmK, kv_full, p.cv + d.h * DV + 64 * i, krow);
        ++nkv;
        bool ok = true;
        for (int i = 0; i < d.nqb; ++i, ++gi) {
          const int st = gi % KV_STAGES;
          if (!mbar_wait(&q_empty[st], ((gi / KV_STAGES) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sq = smem + S::kOffStage + st * S::kStage;
          const int qrow = static_cast<int>(d.row0 + d.k0 + i * KV_BM);
          mbar_arrive_expect_tx(&q_full[st], (kTwo ? 2 : 1) * S::kQ + S::kDO);
          for (int c = 0; c < DK / 64; ++c) {
            tma_load_2d(sq + c * KV_BM * 128, &tmQ, &q_full[st], p.cq1 + d.h * DK + 64 * c, qrow);
            if (kTwo) tma_load_2d(sq + S::kQ + c * KV_BM * 128, &tmQ, &q_full[st], p.cq2 + d.h * DK + 64 * c, qrow);
          }
          for (int c = 0; c < DV / 64; ++c)
            tma_load_2d(sq + 2 * S::kQ + c * KV_BM * 128, &tmDO, &q_full[st], d.h * DV + 64 * c, qrow);
        }
        if (!ok) break;
      }
      // every issued copy has landed before the CTA may exit
      if (nkv > 0) mbar_wait(kv_full, (nkv - 1) & 1, p.status, kErrTimeoutProducer);
      for (uint32_t g = gi > KV_STAGES ? gi - KV_STAGES : 0; g < gi; ++g)
        mbar_wait(&q_full[g % KV_STAGES], (g / KV_STAGES) & 1, p.status, kErrTimeoutProducer);
    } else if (warp == 1 && elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, KV_BM, 0, 0);
      constexpr uint32_t idDV = idesc_bf16_f32(128, DV, 0, 1);
      constexpr uint32_t idDK = idesc_bf16_f32(128, DK, 0, 1);
      const uint32_t sK1 = smem_u32(smem + S::kOffK1), sK2 = smem_u32(smem + S::kOffK2);
      const uint32_t sV = smem_u32(smem + S::kOffV);
      // dV, dK += (P^T, dS^T) (dO, Q) of global query block g; the first block of tile n overwrites
      // the accumulators once the epilogue has read tile n-1's out
      auto accumulate = [&](uint32_t g, bool first, int n) -> bool {
        const int tb = g & 1;
        if (!mbar_wait(&t_full[tb], (g >> 1) & 1, p.status, kErrTimeoutMma)) return false;
        if (first && !mbar_wait(acc_empty, (n & 1) ^ 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + S::kOffStage + (g % KV_STAGES) * S::kStage);
        const uint32_t sT = smem_u32(smem + S::kOffT + tb * S::kTile);
#pragma unroll
        for (int k = 0; k < KV_BM / 16; ++k) {
          const uint32_t acc = (!first || k > 0) ? 1u : 0u;
          // A tiles (128 keys x 32 queries, 64-byte swizzle): P^T, dS1^T, dS2^T
          const uint64_t aP = smem_desc(sT + k * 32, 16, 512, 4);
          const uint64_t a1 = smem_desc(sT + S::kT + k * 32, 16, 512, 4);
          const uint64_t a2 = smem_desc(sT + 2 * S::kT + k * 32, 16, 512, 4);
          umma_ss(tDV, aP, mnmajor_desc(sq + 2 * S::kQ, KV_BM, k), idDV, acc);
          umma_ss(tDK1, a1, mnmajor_desc(sq, KV_BM, k), idDK, acc);
          if (kTwo) umma_ss(tDK2, a2, mnmajor_desc(sq + S::kQ, KV_BM, k), idDK, acc);
        }
        umma_commit(&t_empty[tb]);
        umma_commit(&q_empty[g % KV_STAGES]);
        return true;
      };
      uint32_t gi = 0;
      for (int n = 0;; ++n) {
        const int t = read_tile(n, kErrTimeoutMma);
        if (t < 0) break;
        mbar_arrive(&tile_empty[n & 1]);
        if (t >= ntiles) break;
        const KvTile d = kv_tile(t, nkt, doc_end, p);
        if (!mbar_wait(kv_full, n & 1, p.status, kErrTimeoutMma)) break;
        bool ok = true;
        for (int i = 0; i < d.nqb; ++i, ++gi) {
          const int st = gi % KV_STAGES;
          if (!mbar_wait(&q_full[st], (gi / KV_STAGES) & 1, p.status, kErrTimeoutMma) ||
              !mbar_wait(sc_empty, (gi & 1) ^ 1, p.status, kErrTimeoutMma)) {
            ok = false;
            break;
          }
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
          if (i == d.nqb - 1) umma_commit(kv_empty);
          if (i > 0 && !accumulate(gi - 1, i == 1, n)) {
            ok = false;
            break;
          }
        }
        if (!ok || !accumulate(gi - 1, d.nqb == 1, n)) break;
        umma_commit(acc_full);
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kErrTimeoutMma);
    }
  } else if (warp < kKvFirstEpi) {
    reg_alloc<kKvPolyRegs>();
    const int sub = warp & 3;
    const int pw = warp - kKvFirstPoly;  // poly warp index 0..7
    const int half = pw >> 2;            // which 16 queries of the 32-query block
    const int r = sub * 32 + lane;       // key row
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    uint32_t gi = 0;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      const int t = read_tile(n, kErrTimeoutEpilogue);
      __syncwarp();
      if (t < 0) break;
      if (lane == 0) mbar_arrive(&tile_empty[n & 1]);
      if (t >= ntiles) break;
      const KvTile d = kv_tile(t, nkt, doc_end, p);
      const int kt = d.k0 + r;
      const bool kvalid = kt < p.T;
      const long long krow = d.row0 + (kvalid ? kt : d.k0);
      const bool kreal = kvalid && p.doc[krow] >= 0;
      const int kend = kreal ? doc_end[krow] : kt;  // queries of the same document: [kt, kend)
      float c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] = p.par[d.h * 4 + i];
      float g0 = 0.f, g1 = 0.f, g2 = 0.f, g12 = 0.f;
      // row scales of this thread's 16 queries, loaded for block i+1 while block i is processed
      auto load_rs = [&](int i, float (&dst)[16]) {
        const int q = d.k0 + i * KV_BM + half * 16;
        const float* src = p.row_scale + d.row0 + q;
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
      load_rs(0, rs_next);
      for (int i = 0; i < d.nqb; ++i, ++gi) {
        float rsv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) rsv[e] = rs_next[e];
        if (i + 1 < d.nqb) load_rs(i + 1, rs_next);
        if (!mbar_wait(sc_full, gi & 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
        uint32_t a[16], bb[16], g[16];
        tmem_ld16(tS1 + lane_off + half * 16, a);
        if (kTwo) tmem_ld16(tS2 + lane_off + half * 16, bb);
        tmem_ld16(tDP + lane_off + half * 16, g);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(sc_empty);
        const int qb0 = d.k0 + i * KV_BM + half * 16;
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
        const int tb = gi & 1;
        if (!mbar_wait(&t_empty[tb], ((gi >> 1) & 1) ^ 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
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
      // kind-parameter partials: fixed-order reduction over the 256 poly threads of this key block,
      // through one of two SMEM buffers handed to poly warp 0 by an mbarrier (bounded wait).  A buffer
      // is rewritten two tiles later, after warp 0 has passed the next tile's score blocks.
      if (ok && KIND != 0 && p.dpar != nullptr) {
        float* red = reinterpret_cast<float*>(smem + S::kOffRed) + (n & 1) * 32;
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
          mbar_arrive(&red_full[n & 1]);
        }
        if (pw == 0 && lane < 4 && mbar_wait(&red_full[n & 1], (n >> 1) & 1, p.status, kErrTimeoutEpilogue)) {
          float sum = 0.f;
          for (int w8 = 0; w8 < 8; ++w8) sum += red[w8 * 4 + lane];
          p.dpar[(static_cast<long long>(d.bh) * p.dpar_blocks + d.kb) * 4 + lane] = sum;
        }
      }
    }
  } else {
    if constexpr (kKvEpiRegs < kKvLaunchRegs) reg_dealloc<kKvEpiRegs>();
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    for (int n = 0;; ++n) {
      const int t = read_tile(n, kErrTimeoutEpilogue);
      __syncwarp();
      if (t < 0) break;
      if (lane == 0) mbar_arrive(&tile_empty[n & 1]);
      if (t >= ntiles) break;
      const KvTile d = kv_tile(t, nkt, doc_end, p);
      const int kt = d.k0 + r;
      const bool kvalid = kt < p.T;
      const long long krow = d.row0 + (kvalid ? kt : d.k0);
      const long long kp = kvalid ? p.pos[krow] : 0;
      const float* ct = p.rope_cos ? p.rope_cos + kp * (DK / 2) : nullptr;
      const float* st = p.rope_sin ? p.rope_sin + kp * (DK / 2) : nullptr;
      float cs[16], sn[16];
      if (ct != nullptr) rope_fetch16(ct, st, 0, cs, sn);  // in flight while the accumulators complete
      if (!mbar_wait(acc_full, n & 1, p.status, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      __nv_bfloat16* row = p.dq + krow * p.ldd;
      store_row_lean<DV>(tDV + lane_off, row + p.cv + d.h * DV, kvalid, 1.f);
      if (ct != nullptr && kTwo) {
        const uint32_t acc[2] = {tDK1 + lane_off, tDK2 + lane_off};
        __nv_bfloat16* const out[2] = {row + p.ck1 + d.h * DK, row + p.ck2 + d.h * DK};
        store_rows_rope<DK, 2>(acc, out, kvalid, p.sm, ct, st, cs, sn);
      } else if (ct != nullptr) {
        const uint32_t acc[1] = {tDK1 + lane_off};
        __nv_bfloat16* const out[1] = {row + p.ck1 + d.h * DK};
        store_rows_rope<DK, 1>(acc, out, kvalid, p.sm, ct, st, cs, sn);
      } else {
        store_row_lean<DK>(tDK1 + lane_off, row + p.ck1 + d.h * DK, kvalid, p.sm);
        if (kTwo) store_row_lean<DK>(tDK2 + lane_off, row + p.ck2 + d.h * DK, kvalid, p.sm);
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) sched_finish(g_dkv_sched);
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
      cudaFuncAttributes fa;
      TTB_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
      TTB_CHECK(fa.numRegs == kDqLaunchRegs, "poly attention dq: register split needs 128 registers at launch");
      configured = true;
    }
    const int tiles = (p.T + DQ_BM - 1) / DQ_BM * p.B * p.H;
    kern<<<persistent_grid(tiles), kDqThreads, S::kBytes, stream>>>(tq, tkv, tdo, p);
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
      cudaFuncAttributes fa;
      TTB_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
      TTB_CHECK(fa.numRegs == kKvLaunchRegs, "poly attention dkv: register split needs 128 registers at launch");
      configured = true;
    }
    const int tiles = (p.T + KV_BN - 1) / KV_BN * p.B * p.H;
    kern<<<persistent_grid(tiles), kKvThreads, S::kBytes, stream>>>(tk, tq, tdo, doc_end, p);
    TTB_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace attn

namespace {
int g_grid_limit = 0;
}
void poly_attention_set_grid_limit(int limit) { g_grid_limit = limit; }
int attn::persistent_grid(int tiles) {
  int g = tiles < num_sms() ? tiles : num_sms();
  if (g_grid_limit > 0 && g > g_grid_limit) g = g_grid_limit;
  return g > 0 ? g : 1;
}

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
