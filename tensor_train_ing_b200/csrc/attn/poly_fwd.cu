// Polynomial attention forward on the 5th-generation tensor cores (sm_100a).
//
// Persistent: one CTA per SM takes (batch, head, block of 128 queries) tiles from a dynamic
// scheduler in grid order (a head's query tiles in a row, so its K and V stay in L2).  Warp roles:
//   warp 0     tile fetch; TMA producer for Q1/Q2 (once per tile, as soon as the previous tile's
//              last score MMAs are done) and the K1/K2 ring (3 stages of 64 keys)
//   warp 1     tcgen05.mma issuer: S1 = Q1 K1^T, S2 = Q2 K2^T into a 3-deep ring of TMEM score
//              buffers, issued two key blocks ahead, then O += P V with P read straight from TMEM
//              (A operand in tensor memory)
//   warp 2     TMA producer for the V ring (3 stages)
//   warps 3-18 two groups of eight "poly" warps that take alternate key blocks.  Warp w owns TMEM
//              lane quadrant w%4 (32 query rows) and one half (32 keys) of its block; it tcgen05.ld's
//              its S1/S2 slice, forms P = visible * row_scale * A(S1, S2) in fp32 (no per-element mask
//              when the slice is fully visible), rounds to bf16 and tcgen05.st's it over the S1
//              columns it has just read; at the end of a tile all sixteen warps drain O to global
//              memory while the tensor pipe already runs the next tile's first score blocks.
// The elementwise step is the latency the MMAs must hide: with two groups, two key blocks are in
// the poly stage at once while the tensor pipe runs the next scores and the previous P V.  A score
// buffer is free again once the P V that read its P has completed.  K and V have separate rings,
// and key blocks before the start of the first query's document are skipped (documents are
// contiguous).
// Reference: tnlm/kernels/poly_attn.py:38-74.
#include "../common/host.h"
#include "attn_api.h"
#include "poly_common.cuh"

namespace ttb {
namespace attn {

constexpr int BMQ = 128;  // queries per CTA
constexpr int BNK = 64;   // keys per block
constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr int kSBufs = 3;       // TMEM score buffers (S1 and S2 each), P written over S1
constexpr int kThreads = 608;   // 3 control warps + 2 groups of 8 poly warps
constexpr int kGroupThreads = 256;
constexpr int kFirstPoly = 3;

template <int DK, int DV>
struct FwdSmem {
  static constexpr int kQ = DK / 64 * BMQ * 128;          // one of Q1/Q2
  static constexpr int kK = DK / 64 * BNK * 128;          // one of K1/K2
  static constexpr int kV = DV / 64 * BNK * 128;
  static constexpr int kKStage = 2 * kK;
  static constexpr int kOffQ1 = 0;
  static constexpr int kOffQ2 = kQ;
  static constexpr int kOffK = 2 * kQ;
  static constexpr int kOffV = kOffK + kKStages * kKStage;
  static constexpr int kOffBar = kOffV + kVStages * kV;
  // >= 120 KB keeps one CTA per SM, so the 512-column TMEM allocation never waits on a neighbour
  static constexpr int kBytes = (kOffBar + 256 + 1024) > 120 * 1024 ? (kOffBar + 256 + 1024) : 120 * 1024;
};

// Scheduler counters of the forward kernel (next tile, finished CTAs); zero between launches.
__device__ unsigned int g_fwd_sched[2];

struct FwdTile {
  int q0, h, kstart, nkb;
  long long row0;
};

// Tile t in grid order: head-major, heaviest (last) query block of a head first.
__device__ __forceinline__ FwdTile fwd_tile(int t, int nqb, const Params& p) {
  FwdTile d;
  const int bh = t / nqb;
  const int qb = nqb - 1 - (t - bh * nqb);
  const int b = bh / p.H;
  d.h = bh - b * p.H;
  d.q0 = qb * BMQ;
  d.row0 = static_cast<long long>(b) * p.T;
  const int lo = d.q0 - p.pos[d.row0 + d.q0];  // start of the first query's document
  d.kstart = (lo / BNK) * BNK;
  const int kend = min(d.q0 + BMQ, p.T);
  d.nkb = (kend - d.kstart + BNK - 1) / BNK;
  return d;
}

template <int DK, int DV, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    poly_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV, Params p) {
  using S = FwdSmem<DK, DV>;
  constexpr bool kTwo = KIND != 1;  // kinds with a second score S2
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;     // [3]
  uint64_t* k_empty = bar + 4;    // [3]
  uint64_t* v_full = bar + 7;     // [3]
  uint64_t* v_empty = bar + 10;   // [3]
  uint64_t* s_full = bar + 13;    // [3] scores of the buffer's block are in TMEM
  uint64_t* s_free = bar + 16;    // [3] the P V that read the buffer's P has completed
  uint64_t* p_full = bar + 19;    // [3] P of the buffer's block is in TMEM
  uint64_t* o_full = bar + 22;    // O of the tile is complete in TMEM
  uint64_t* mma_done = bar + 23;
  uint64_t* acc_empty = bar + 24; // the poly warps have read O out of TMEM
  uint64_t* q_empty = bar + 25;   // the tile's score MMAs no longer read Q
  uint64_t* tile_full = bar + 26; // [2]
  uint64_t* tile_empty = bar + 28;// [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 30);
  int* tile_ids = reinterpret_cast<int*>(bar + 31);  // [2]
  constexpr int kPolyThreads = 2 * kGroupThreads;
  constexpr int kTileReaders = 1 + 1 + kPolyThreads / 32;  // V producer, MMA issuer, poly warps

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqb = (p.T + BMQ - 1) / BMQ;
  const int ntiles = nqb * p.B * p.H;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 1);
      mbar_init(&p_full[i], kGroupThreads);
    }
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(acc_empty, kPolyThreads);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tile_full[i], 1);
      mbar_init(&tile_empty[i], kTileReaders);
    }
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
  // TMEM columns: S1[3] at 0/64/128, S2[3] at 192/256/320, O at 384.  P of a block (bf16 pairs)
  // overwrites the first 16 columns of each 32-key half of that block's S1.
  const uint32_t tS1 = tmem, tS2 = tmem + kSBufs * BNK, tO = tmem + 2 * kSBufs * BNK;
  static_assert(2 * kSBufs * BNK + DV <= 512, "TMEM budget");

  auto read_tile = [&](int n, uint32_t code) -> int {
    if (!mbar_wait(&tile_full[n & 1], (n >> 1) & 1, p.status, code)) return -1;
    return *reinterpret_cast<volatile int*>(&tile_ids[n & 1]);
  };

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      uint32_t gj = 0;  // key blocks issued over all tiles
      int nq = 0;       // Q loads issued
      for (int n = 0;; ++n) {
        if (!mbar_wait(&tile_empty[n & 1], ((n >> 1) & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int t = static_cast<int>(atomicAdd(&g_fwd_sched[0], 1u));
        tile_ids[n & 1] = t;
        mbar_arrive(&tile_full[n & 1]);
        if (t >= ntiles) break;
        const FwdTile d = fwd_tile(t, nqb, p);
        if (!mbar_wait(q_empty, (n & 1) ^ 1, p.status, kErrTimeoutProducer)) break;
        const int qrow = static_cast<int>(d.row0 + d.q0);
        mbar_arrive_expect_tx(q_full, (kTwo ? 2 : 1) * S::kQ);
        for (int i = 0; i < DK / 64; ++i) {
          tma_load_2d(smem + S::kOffQ1 + i * BMQ * 128, &tmQ, q_full, p.cq1 + d.h * DK + 64 * i, qrow);
          if (kTwo) tma_load_2d(smem + S::kOffQ2 + i * BMQ * 128, &tmQ, q_full, p.cq2 + d.h * DK + 64 * i, qrow);
        }
        ++nq;
        bool ok = true;
        for (int j = 0; j < d.nkb; ++j, ++gj) {
          const int st = gj % kKStages;
          if (!mbar_wait(&k_empty[st], ((gj / kKStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sk = smem + S::kOffK + st * S::kKStage;
          const int krow = static_cast<int>(d.row0 + d.kstart + j * BNK);
          mbar_arrive_expect_tx(&k_full[st], (kTwo ? 2 : 1) * S::kK);
          for (int i = 0; i < DK / 64; ++i) {
            tma_load_2d(sk + i * BNK * 128, &tmKV, &k_full[st], p.ck1 + d.h * DK + 64 * i, krow);
            if (kTwo) tma_load_2d(sk + S::kK + i * BNK * 128, &tmKV, &k_full[st], p.ck2 + d.h * DK + 64 * i, krow);
          }
        }
        if (!ok) break;
      }
      // let in-flight copies land before exit (bounded)
      if (nq > 0) mbar_wait(q_full, (nq - 1) & 1, p.status, kErrTimeoutProducer);
      for (uint32_t g = gj > kKStages ? gj - kKStages : 0; g < gj; ++g)
        mbar_wait(&k_full[g % kKStages], (g / kKStages) & 1, p.status, kErrTimeoutProducer);
    }
  } else if (warp == 2) {
    if (elect_one()) {
      uint32_t gj = 0;
      for (int n = 0;; ++n) {
        const int t = read_tile(n, kErrTimeoutProducer);
        if (t < 0) break;
        mbar_arrive(&tile_empty[n & 1]);
        if (t >= ntiles) break;
        const FwdTile d = fwd_tile(t, nqb, p);
        bool ok = true;
        for (int j = 0; j < d.nkb; ++j, ++gj) {
          const int st = gj % kVStages;
          if (!mbar_wait(&v_empty[st], ((gj / kVStages) & 1) ^ 1, p.status, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sv = smem + S::kOffV + st * S::kV;
          const int krow = static_cast<int>(d.row0 + d.kstart + j * BNK);
          mbar_arrive_expect_tx(&v_full[st], S::kV);
          for (int i = 0; i < DV / 64; ++i)
            tma_load_2d(sv + i * BNK * 128, &tmKV, &v_full[st], p.cv + d.h * DV + 64 * i, krow);
        }
        if (!ok) break;
      }
      for (uint32_t g = gj > kVStages ? gj - kVStages : 0; g < gj; ++g)
        mbar_wait(&v_full[g % kVStages], (g / kVStages) & 1, p.status, kErrTimeoutProducer);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, BNK, 0, 0);
      constexpr uint32_t idPV = idesc_bf16_f32(128, DV, 0, 1);
      const uint32_t sQ1 = smem_u32(smem + S::kOffQ1), sQ2 = smem_u32(smem + S::kOffQ2);
      // S1, S2 of global key block g into score buffer g % 3
      auto issue_s = [&](uint32_t g) -> bool {
        const int b = g % kSBufs, ks = g % kKStages;
        if (!mbar_wait(&k_full[ks], (g / kKStages) & 1, p.status, kErrTimeoutMma)) return false;
        // the buffer's previous block (g - 3) must have finished its P V
        if (!mbar_wait(&s_free[b], ((g / kSBufs) & 1) ^ 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sK1 = smem_u32(smem + S::kOffK + ks * S::kKStage);
        const uint32_t sK2 = sK1 + S::kK;
#pragma unroll
        for (int k = 0; k < DK / 16; ++k)
          umma_ss(tS1 + b * BNK, kmajor_desc(sQ1, BMQ, k), kmajor_desc(sK1, BNK, k), idS, k > 0 ? 1u : 0u);
        if (kTwo) {
#pragma unroll
          for (int k = 0; k < DK / 16; ++k)
            umma_ss(tS2 + b * BNK, kmajor_desc(sQ2, BMQ, k), kmajor_desc(sK2, BNK, k), idS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[b]);
        umma_commit(&k_empty[ks]);
        return true;
      };
      // O += P V of global key block g; the first block of tile n overwrites O once the poly warps
      // have drained tile n-1's
      auto issue_pv = [&](uint32_t g, bool first, int n) -> bool {
        const int b = g % kSBufs, vs = g % kVStages;
        if (!mbar_wait(&p_full[b], (g / kSBufs) & 1, p.status, kErrTimeoutMma)) return false;
        if (!mbar_wait(&v_full[vs], (g / kVStages) & 1, p.status, kErrTimeoutMma)) return false;
        if (first && !mbar_wait(acc_empty, (n & 1) ^ 1, p.status, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + S::kOffV + vs * S::kV);
        // P columns: keys 0..31 at +0..15, keys 32..63 at +32..47 of the block's S1 buffer
#pragma unroll
        for (int k = 0; k < BNK / 16; ++k)
          umma_ts(tO, tS1 + b * BNK + (k >> 1) * 32 + (k & 1) * 8, mnmajor_desc(sV, BNK, k), idPV,
                  (!first || k > 0) ? 1u : 0u);
        umma_commit(&s_free[b]);
        umma_commit(&v_empty[vs]);
        return true;
      };
      uint32_t gj = 0;
      for (int n = 0;; ++n) {
        const int t = read_tile(n, kErrTimeoutMma);
        if (t < 0) break;
        mbar_arrive(&tile_empty[n & 1]);
        if (t >= ntiles) break;
        const FwdTile d = fwd_tile(t, nqb, p);
        if (!mbar_wait(q_full, n & 1, p.status, kErrTimeoutMma)) break;
        bool ok = true;
        // scores run two blocks ahead of P V; Q is free once the tile's last scores are done
        for (int j = 0; j < 2 && j < d.nkb && ok; ++j) {
          ok = issue_s(gj + j);
          if (ok && j == d.nkb - 1) umma_commit(q_empty);
        }
        for (int j = 0; j < d.nkb && ok; ++j) {
          if (j + 2 < d.nkb) {
            if (!issue_s(gj + j + 2)) { ok = false; break; }
            if (j + 2 == d.nkb - 1) umma_commit(q_empty);
          }
          if (!issue_pv(gj + j, j == 0, n)) { ok = false; break; }
        }
        if (!ok) break;
        gj += d.nkb;
        umma_commit(o_full);
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, kErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------- poly warps (3..18)
    const int pw = warp - kFirstPoly;
    const int group = pw >> 3;                  // which alternate key blocks (by global block index)
    const int half = (pw >> 2) & 1;             // which 32 keys of the 64-key block
    const int sub = warp & 3;                   // TMEM lane quadrant this warp may access
    const int r = sub * 32 + lane;              // query row inside the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    uint32_t gj = 0;
    bool ok = true;
    for (int n = 0; ok; ++n) {
      const int tile = read_tile(n, kErrTimeoutEpilogue);
      __syncwarp();
      if (tile < 0) break;
      if (lane == 0) mbar_arrive(&tile_empty[n & 1]);
      if (tile >= ntiles) break;
      const FwdTile d = fwd_tile(tile, nqb, p);
      const int t = d.q0 + r;
      const bool valid = t < p.T;
      const long long grow = d.row0 + (valid ? t : d.q0);
      const int dq = valid ? p.doc[grow] : -1;
      const int dstart = valid ? t - p.pos[grow] : 0;  // documents are contiguous: keys [dstart, t]
      const float rs = (valid && dq >= 0) ? p.row_scale[grow] : 0.f;
      float c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] = p.par[d.h * 4 + i];
      // signed_product fast path: P = (s1 sm)(s2 sm) rs = s1 s2 (sm^2 rs)
      const float k0scale = p.sm * p.sm * rs;
      for (int j = static_cast<int>((gj & 1u) ^ static_cast<uint32_t>(group)); j < d.nkb; j += 2) {
        const uint32_t g = gj + j;
        const int b = g % kSBufs;
        if (!mbar_wait(&s_full[b], (g / kSBufs) & 1, p.status, kErrTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
        uint32_t a[32], bb[32];
        const uint32_t col = b * BNK + half * 32;
        tmem_ld32(tS1 + lane_off + col, a);
        if (kTwo) tmem_ld32(tS2 + lane_off + col, bb);
        tmem_ld_wait();
        const int kb0 = d.kstart + j * BNK + half * 32;
        const bool full_vis = rs != 0.f && kb0 >= dstart && kb0 + 31 <= t;
        uint32_t pk[16];
        if (full_vis && KIND == 0) {
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2)
            pk[jj / 2] = pack_bf16(__uint_as_float(a[jj]) * __uint_as_float(bb[jj]) * k0scale,
                                   __uint_as_float(a[jj + 1]) * __uint_as_float(bb[jj + 1]) * k0scale);
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            float v[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int kt = kb0 + jj + e;
              const float s1 = __uint_as_float(a[jj + e]) * p.sm;
              const float s2 = kTwo ? __uint_as_float(bb[jj + e]) * p.sm : s1;
              const bool vis = full_vis || (kt <= t && kt >= dstart);
              v[e] = vis ? poly<KIND>(s1, s2, c) * rs : 0.f;
            }
            pk[jj / 2] = pack_bf16(v[0], v[1]);
          }
        }
        // P over the first 16 columns of the S1 slice this warp has just read (nobody else reads them)
        tmem_st16(tS1 + lane_off + col, pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      gj += d.nkb;
      // drain O (the tensor pipe meanwhile runs the next tile's first score blocks)
      if (!mbar_wait(o_full, n & 1, p.status, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int part = group * 2 + half;  // four warps per lane quadrant share O's columns
#pragma unroll 1
      for (int cc = part; cc < DV / 32; cc += 4) {
        uint32_t a[32];
        tmem_ld32(tO + lane_off + cc * 32, a);
        tmem_ld_wait();
        if (valid) {
          float v[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(a[q]);
          store32_scaled(p.y + grow * p.ldy + d.h * DV + cc * 32, v);
        }
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
  if (threadIdx.x == 0) sched_finish(g_fwd_sched);
}

template <int DK, int DV, int KIND>
void launch_fwd(const void* qkv, long long ld, long long rows, const Params& p, cudaStream_t stream) {
  using S = FwdSmem<DK, DV>;
  const CUtensorMap tq = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, BMQ);
  const CUtensorMap tkv = make_tmap_2d(qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ld, rows, ld, 64, BNK);
  auto kern = poly_fwd_kernel<DK, DV, KIND>;
  static bool configured = false;
  if (!configured) {
    TTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
    configured = true;
  }
  const int tiles = (p.T + BMQ - 1) / BMQ * p.B * p.H;
  kern<<<persistent_grid(tiles), kThreads, S::kBytes, stream>>>(tq, tkv, p);
  TTB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace attn

void poly_attention_fwd(int kind, int dk, int dv, const void* qkv, long long ld, attn::Params p, cudaStream_t stream) {
  TTB_CHECK((dk == 64 || dk == 128) && (dv == 64 || dv == 128), "poly attention: head dims must be 64 or 128");
  TTB_CHECK(kind >= 0 && kind <= 2, "poly attention: bad kind");
  const long long rows = static_cast<long long>(p.B) * p.T;
  p.status = status_ptr();
#define TTB_FWD(DK_, DV_, K_) \
  if (dk == DK_ && dv == DV_ && kind == K_) return attn::launch_fwd<DK_, DV_, K_>(qkv, ld, rows, p, stream);
  TTB_FWD(64, 64, 0) TTB_FWD(64, 64, 1) TTB_FWD(64, 64, 2)
  TTB_FWD(128, 128, 0) TTB_FWD(128, 128, 1) TTB_FWD(128, 128, 2)
  TTB_FWD(64, 128, 0) TTB_FWD(64, 128, 1) TTB_FWD(64, 128, 2)
  TTB_FWD(128, 64, 0) TTB_FWD(128, 64, 1) TTB_FWD(128, 64, 2)
#undef TTB_FWD
}

}  // namespace ttb
