// Epilogue functors for the sm_100a GEMM.  Each thread owns one accumulator row (TMEM lane)
// and walks the tile's columns 32 at a time with tcgen05.ld.
#pragma once

#include "gemm_sm100.cuh"

namespace ttb {
namespace gemm {

__device__ __forceinline__ void load_row32_bf16(const __nv_bfloat16* p, bool full, int n_valid, float (&v)[32]) {
  if (full) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = *reinterpret_cast<const uint4*>(p + q * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[q * 8 + 2 * j] = bf16_lo(w[j]);
        v[q * 8 + 2 * j + 1] = bf16_hi(w[j]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < n_valid ? __bfloat162float(p[j]) : 0.f;
  }
}

__device__ __forceinline__ void load_row32_f32(const float* p, bool full, int n_valid, float (&v)[32]) {
  if (full) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 u = *reinterpret_cast<const float4*>(p + q * 4);
      v[q * 4 + 0] = u.x;
      v[q * 4 + 1] = u.y;
      v[q * 4 + 2] = u.z;
      v[q * 4 + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < n_valid ? p[j] : 0.f;
  }
}

__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* p, bool full, int n_valid, const float (&v)[32]) {
  if (full) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
      u.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
      u.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
      u.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
      *reinterpret_cast<uint4*>(p + q * 8) = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n_valid) p[j] = __float2bfloat16_rn(v[j]);
  }
}

__device__ __forceinline__ void store_row32_f32(float* p, bool full, int n_valid, const float (&v)[32]) {
  if (full) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4*>(p + q * 4) = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n_valid) p[j] = v[j];
  }
}

// ---------------------------------------------------------------- warp-coalesced chunk I/O
// An epilogue thread owns one accumulator row, so row-per-thread global accesses touch 32
// different 128-byte lines per warp instruction and keep L1 busy on the short-K GEMMs.  These
// helpers move a warp's 32 x 32 chunk through the warp's shared area instead: every thread writes
// (or reads) its own row there, and global memory is written / read 8 bf16 rows (64 bytes each) or
// 4 fp32 rows (128 bytes each) per instruction.  Rows are XOR-swizzled in 16-byte pieces, so
// both the row-wise and the coalesced accesses are free of bank conflicts.  Pieces outside the
// matrix (rows >= M, columns >= N) are skipped; N and the row strides must be multiples of 8
// (bf16) or 4 (fp32) elements and the base pointers 16-byte aligned.
__device__ __forceinline__ uint32_t sw_at16(int R, int q) {  // bf16: 4 pieces per 64-byte row
  return static_cast<uint32_t>(R * 64 + ((q ^ ((R >> 1) & 3)) << 4));
}
__device__ __forceinline__ uint32_t sw_at32(int R, int q) {  // fp32: 8 pieces per 128-byte row
  return static_cast<uint32_t>(R * 128 + ((q ^ (R & 7)) << 4));
}

__device__ __forceinline__ void warp_store_bf16(uint8_t* buf, const float (&v)[32], int lane, __nv_bfloat16* D,
                                                long long ldd, int row0, int col0, int M, int N) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(buf + sw_at16(lane, q)) =
        make_uint4(pack_bf16(v[q * 8 + 0], v[q * 8 + 1]), pack_bf16(v[q * 8 + 2], v[q * 8 + 3]),
                   pack_bf16(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16(v[q * 8 + 6], v[q * 8 + 7]));
  __syncwarp();
  const int q = lane & 3;
  const int col = col0 + q * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int R = i * 8 + (lane >> 2);
    if (row0 + R < M && col < N)
      *reinterpret_cast<uint4*>(D + static_cast<long long>(row0 + R) * ldd + col) =
          *reinterpret_cast<const uint4*>(buf + sw_at16(R, q));
  }
  __syncwarp();
}

__device__ __forceinline__ void warp_store_f32(uint8_t* buf, const float (&v)[32], int lane, float* D, long long ldd,
                                               int row0, int col0, int M, int N) {
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(buf + sw_at32(lane, q)) = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
  __syncwarp();
  const int q = lane & 7;
  const int col = col0 + q * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int R = i * 4 + (lane >> 3);
    if (row0 + R < M && col < N)
      *reinterpret_cast<float4*>(D + static_cast<long long>(row0 + R) * ldd + col) =
          *reinterpret_cast<const float4*>(buf + sw_at32(R, q));
  }
  __syncwarp();
}

// Queue the fp32 chunk C[row0 .., col0 ..] into buf with cp.async, 4 rows per instruction; closes
// one cp.async group.
__device__ __forceinline__ void warp_load_f32_async(uint8_t* buf, const float* C, long long ldc, int row0, int col0,
                                                    int M, int N, int lane) {
  const uint32_t base = smem_u32(buf);
  const int q = lane & 7;
  const int col = col0 + q * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int R = i * 4 + (lane >> 3);
    if (row0 + R < M && col < N) cp_async16(base + sw_at32(R, q), C + static_cast<long long>(row0 + R) * ldc + col);
  }
  cp_async_commit();
}

__device__ __forceinline__ void read_row_f32(const uint8_t* buf, int lane, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 u = *reinterpret_cast<const float4*>(buf + sw_at32(lane, q));
    v[q * 4] = u.x; v[q * 4 + 1] = u.y; v[q * 4 + 2] = u.z; v[q * 4 + 3] = u.w;
  }
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// D = alpha * acc + beta * C   (C optional, may alias D; D and C bf16 or fp32).
// Optionally also adds a per-column bias (fp32) before scaling by alpha.
template <int NB>
struct EpiLinear {
  void* D;
  long long ldd;
  int d_f32;
  const void* C;
  long long ldc;
  int c_f32;
  float alpha, beta;
  const float* bias;
  int M, N;

  static constexpr int kSmemPerThread = 256;  // per warp: two 4 KB chunk buffers

  // Warp-coalesced path: D fp32 or bf16, C absent or fp32 (prefetched two chunks ahead).
  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int tm, int tn, uint8_t* sm) const {
    constexpr int kChunks = NB / 32;
    const bool has_c = C != nullptr && beta != 0.f;
    const bool fast = aligned16(D) && (d_f32 ? (ldd % 4 == 0 && N % 4 == 0) : (ldd % 8 == 0 && N % 8 == 0)) &&
                      (!has_c || (c_f32 && aligned16(C) && ldc % 4 == 0));
    if (!fast) return rowwise(taddr, row, n0);
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;
    const int row0 = row - lane;
    const float* Cf = static_cast<const float*>(C);
    if (has_c) {
      warp_load_f32_async(area, Cf, ldc, row0, n0, M, N, lane);
      warp_load_f32_async(area + 4096, Cf, ldc, row0, n0 + 32, M, N, lane);
    }
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
      uint8_t* buf = area + (c & 1) * 4096;
      const int col0 = n0 + c * 32;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      if (has_c) {
        cp_async_wait<1>();  // this lane's part of chunk c has landed ...
        __syncwarp();        // ... and every other lane's
      }
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += (col0 + j < N) ? bias[col0 + j] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= alpha;
      if (has_c) {
        float cv[32];
        read_row_f32(buf, lane, cv);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += beta * cv[j];
        __syncwarp();  // every lane has read its C row before the buffer takes the outputs
      }
      if (col0 < N) {
        if (d_f32)
          warp_store_f32(buf, v, lane, static_cast<float*>(D), ldd, row0, col0, M, N);
        else
          warp_store_bf16(buf, v, lane, static_cast<__nv_bfloat16*>(D), ldd, row0, col0, M, N);
      }
      if (has_c) {
        if (c + 2 < kChunks)
          warp_load_f32_async(buf, Cf, ldc, row0, n0 + (c + 2) * 32, M, N, lane);
        else
          cp_async_commit();  // one group per chunk
      }
    }
    if (has_c) cp_async_wait<0>();
  }

  // Row-per-thread path for strides or widths the 16-byte pieces cannot cover.
  __device__ __forceinline__ void rowwise(uint32_t taddr, int row, int n0) const {
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      if (row >= M || col0 >= N) continue;
      const int nv = min(32, N - col0);
      const bool full = nv == 32;
      const bool d_vec = full && (d_f32 ? (ldd % 4 == 0) : (ldd % 8 == 0)) &&
                         (reinterpret_cast<uintptr_t>(D) & 15) == 0;
      const bool c_vec = full && (c_f32 ? (ldc % 4 == 0) : (ldc % 8 == 0)) &&
                         (reinterpret_cast<uintptr_t>(C) & 15) == 0;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += (j < nv) ? bias[col0 + j] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= alpha;
      if (C != nullptr && beta != 0.f) {
        float cv[32];
        if (c_f32)
          load_row32_f32(static_cast<const float*>(C) + row * ldc + col0, c_vec, nv, cv);
        else
          load_row32_bf16(static_cast<const __nv_bfloat16*>(C) + row * ldc + col0, c_vec, nv, cv);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += beta * cv[j];
      }
      if (d_f32)
        store_row32_f32(static_cast<float*>(D) + row * ldd + col0, d_vec, nv, v);
      else
        store_row32_bf16(static_cast<__nv_bfloat16*>(D) + row * ldd + col0, d_vec, nv, v);
    }
  }
};

// Bilinear / gated MLP hidden layer from a DUAL GEMM:
//   l = acc1 (+bl), r = acc2 (+br);  H = l * r  (mode 0)  or  silu(l) * r  (mode 1)
// H is written in bf16; l and r are also written (bf16) when pointers are given, for backward.
template <int NB>
struct EpiBilinear {
  __nv_bfloat16* H;
  __nv_bfloat16* Lo;
  __nv_bfloat16* Ro;
  long long ld;
  const float* bias_l;
  const float* bias_r;
  int mode;
  int M, N;
  static constexpr int kSmemPerThread = 256;  // per warp: three 2 KB chunk buffers (H, l, r)

  // l, r and h of one row chunk from the two accumulators (bias, bf16 rounding of the factors)
  __device__ __forceinline__ void factors(const uint32_t (&a)[32], const uint32_t (&b)[32], int col0, float (&l)[32],
                                          float (&r)[32], float (&h)[32]) const {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      l[j] = __uint_as_float(a[j]);
      r[j] = __uint_as_float(b[j]);
    }
    if (bias_l != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        l[j] += (col0 + j < N) ? bias_l[col0 + j] : 0.f;
        r[j] += (col0 + j < N) ? bias_r[col0 + j] : 0.f;
      }
    }
    // The reference rounds l and r to bf16 before multiplying; do the same so that the
    // saved factors and the product agree exactly with what backward sees.
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      l[j] = __bfloat162float(__float2bfloat16_rn(l[j]));
      r[j] = __bfloat162float(__float2bfloat16_rn(r[j]));
      const float g = mode == 1 ? l[j] / (1.f + __expf(-l[j])) : l[j];
      h[j] = g * r[j];
    }
  }

  // Warp-coalesced path (see warp_store_bf16).
  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int, int, uint8_t* sm) const {
    const bool fast = ld % 8 == 0 && N % 8 == 0 && aligned16(H) && (Lo == nullptr || aligned16(Lo)) &&
                      (Ro == nullptr || aligned16(Ro));
    if (!fast) return rowwise(taddr, row, n0);
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;
    const int row0 = row - lane;
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t a[32], b[32];
      tmem_ld32(taddr + c * 32, a);
      tmem_ld32(taddr + NB + c * 32, b);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      if (col0 >= N) continue;  // the same for the whole warp
      float l[32], r[32], h[32];
      factors(a, b, col0, l, r, h);
      warp_store_bf16(area, h, lane, H, ld, row0, col0, M, N);
      if (Lo != nullptr) warp_store_bf16(area + 2048, l, lane, Lo, ld, row0, col0, M, N);
      if (Ro != nullptr) warp_store_bf16(area + 4096, r, lane, Ro, ld, row0, col0, M, N);
    }
  }

  __device__ __forceinline__ void rowwise(uint32_t taddr, int row, int n0) const {
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t a[32], b[32];
      tmem_ld32(taddr + c * 32, a);
      tmem_ld32(taddr + NB + c * 32, b);
      tmem_ld_wait();
      const int col0 = n0 + c * 32;
      if (row >= M || col0 >= N) continue;
      const int nv = min(32, N - col0);
      const bool full = nv == 32 && (ld % 8 == 0);
      float l[32], r[32], h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        l[j] = __uint_as_float(a[j]);
        r[j] = __uint_as_float(b[j]);
      }
      if (bias_l != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          l[j] += (j < nv) ? bias_l[col0 + j] : 0.f;
          r[j] += (j < nv) ? bias_r[col0 + j] : 0.f;
        }
      }
      // The reference rounds l and r to bf16 before multiplying; do the same so that the
      // saved factors and the product agree exactly with what backward sees.
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        l[j] = __bfloat162float(__float2bfloat16_rn(l[j]));
        r[j] = __bfloat162float(__float2bfloat16_rn(r[j]));
        const float g = mode == 1 ? l[j] / (1.f + __expf(-l[j])) : l[j];
        h[j] = g * r[j];
      }
      const long long off = row * ld + col0;
      store_row32_bf16(H + off, full, nv, h);
      if (Lo != nullptr) store_row32_bf16(Lo + off, full, nv, l);
      if (Ro != nullptr) store_row32_bf16(Ro + off, full, nv, r);
    }
  }
};

// Backward of the bilinear hidden layer, fused into dH = dY @ D:
//   dl = dH * r            dr = dH * l          (mode 0)
//   dl = dH * r * silu'(l) dr = dH * silu(l)    (mode 1)
// l, r are the bf16 factors saved by the forward; dl/dr written bf16.
//
// With K = d_model the main loop of a tile is short and this epilogue moves 8 bytes per output
// element (l, r in; dl, dr out).  A thread owns one row of the accumulator, but global memory is
// accessed warp-cooperatively through shared memory: each warp stages the 32 x 32 chunks of l and r
// for its 32 rows with cp.async, 8 rows of 64 bytes per instruction (coalesced), two chunks ahead;
// every thread then reads its own row, writes its dl / dr row back into the same buffer, and the
// warp stores the chunk to global memory 8 rows per instruction.  Rows are 64-byte swizzled
// (16-byte piece q of row R at q ^ ((R >> 1) & 3)) so both access patterns are bank-conflict free.
// Requires N, ld and ldo to be multiples of 8 (16-byte pieces), which the launcher checks.
template <int NB>
struct EpiBilinearGrad {
  static constexpr int kSmemPerThread = 256;  // per warp: 2 buffers x (l 2 KB | r 2 KB)
  const __nv_bfloat16* Lin;
  const __nv_bfloat16* Rin;
  __nv_bfloat16* dL;
  __nv_bfloat16* dR;
  long long ld;   // row stride of Lin / Rin
  long long ldo;  // row stride of dL / dR
  int mode;
  int M, N;

  // byte offset of 16-byte piece q of row R in one 2 KB (32 rows x 64 bytes) area
  __device__ __forceinline__ static uint32_t at(int R, int q) {
    return static_cast<uint32_t>(R * 64 + ((q ^ ((R >> 1) & 3)) << 4));
  }

  // Queue chunk c of the warp's 32 rows (first row row0) into buffer area buf (l at +0, r at +2 KB).
  // Lane l copies pieces (row 8i + l/4, piece l%4), i = 0..3, of both factors; pieces outside the
  // matrix are skipped (their rows / columns are never stored).  One cp.async group per call.
  __device__ __forceinline__ void stage(uint8_t* buf, int row0, int col0, int lane) const {
    const uint32_t base = smem_u32(buf);
    const int q = lane & 3;
    const int col = col0 + q * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int R = i * 8 + (lane >> 2);
      const int row = row0 + R;
      if (row < M && col < N) {
        const long long off = static_cast<long long>(row) * ld + col;
        cp_async16(base + at(R, q), Lin + off);
        cp_async16(base + 2048 + at(R, q), Rin + off);
      }
    }
    cp_async_commit();
  }

  // smem: this warp's 8 KB area (the kernel hands each thread a 256-byte slice, 32 consecutive
  // slices per warp)
  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int, int, uint8_t* sm) const {
    constexpr int kChunks = NB / 32;
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;  // the warp's first slice
    const int row0 = row - lane;                 // this warp's first row
    const int R = lane;                          // this thread's row inside the chunk
    const bool row_ok = row < M;
    stage(area, row0, n0, lane);
    stage(area + 4096, row0, n0 + 32, lane);
#pragma unroll 1
    for (int c = 0; c < kChunks; ++c) {
      uint8_t* buf = area + (c & 1) * 4096;
      const int col0 = n0 + c * 32;
      uint32_t a[32];
      tmem_ld32(taddr + c * 32, a);
      cp_async_wait<1>();  // this lane's copies of chunk c have landed ...
      __syncwarp();        // ... and so have the other lanes'
      tmem_ld_wait();
      const int nv = max(0, min(32, N - col0));
      if (row_ok && nv > 0) {
        uint32_t lp[16], rp[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = *reinterpret_cast<const uint4*>(buf + at(R, q));
          const uint4 v = *reinterpret_cast<const uint4*>(buf + 2048 + at(R, q));
          lp[q * 4 + 0] = u.x; lp[q * 4 + 1] = u.y; lp[q * 4 + 2] = u.z; lp[q * 4 + 3] = u.w;
          rp[q * 4 + 0] = v.x; rp[q * 4 + 1] = v.y; rp[q * 4 + 2] = v.z; rp[q * 4 + 3] = v.w;
        }
        uint32_t ol[16], orr[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float dl[2], dr[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = j + e;
            const float l = (jj & 1) ? bf16_hi(lp[jj / 2]) : bf16_lo(lp[jj / 2]);
            const float r = (jj & 1) ? bf16_hi(rp[jj / 2]) : bf16_lo(rp[jj / 2]);
            // the reference's autograd sees dH rounded to bf16 (output grad of a bf16 product)
            const float dh = __bfloat162float(__float2bfloat16_rn(__uint_as_float(a[jj])));
            if (mode == 1) {
              const float sg = 1.f / (1.f + __expf(-l));
              dr[e] = dh * (l * sg);
              dl[e] = dh * r * (sg * (1.f + l * (1.f - sg)));
            } else {
              dl[e] = dh * r;
              dr[e] = dh * l;
            }
          }
          ol[j / 2] = pack_bf16(dl[0], dl[1]);
          orr[j / 2] = pack_bf16(dr[0], dr[1]);
        }
        // this thread's row of the buffer now holds its outputs (only this thread reads that row)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          *reinterpret_cast<uint4*>(buf + at(R, q)) = make_uint4(ol[q * 4], ol[q * 4 + 1], ol[q * 4 + 2], ol[q * 4 + 3]);
          *reinterpret_cast<uint4*>(buf + 2048 + at(R, q)) =
              make_uint4(orr[q * 4], orr[q * 4 + 1], orr[q * 4 + 2], orr[q * 4 + 3]);
        }
      }
      __syncwarp();
      {  // the warp stores the chunk, 8 rows of 64 bytes per instruction
        const int q = lane & 3;
        const int col = col0 + q * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int Rs = i * 8 + (lane >> 2);
          const int rw = row0 + Rs;
          if (rw < M && col < N) {
            const long long off = static_cast<long long>(rw) * ldo + col;
            *reinterpret_cast<uint4*>(dL + off) = *reinterpret_cast<const uint4*>(buf + at(Rs, q));
            *reinterpret_cast<uint4*>(dR + off) = *reinterpret_cast<const uint4*>(buf + 2048 + at(Rs, q));
          }
        }
      }
      __syncwarp();  // every lane is done with the buffer before it is refilled
      if (c + 2 < kChunks)
        stage(buf, row0, n0 + (c + 2) * 32, lane);
      else
        cp_async_commit();  // keep one group per chunk
    }
    cp_async_wait<0>();
  }
};

// Projection GEMM for the fused QKV buffer with the rotary embedding in the epilogue:
// columns < rope_cols hold heads of width dk whose pairs (i, i + dk/2) are rotated by the angle of
// the row's position, using cos/sin tables [positions, dk/2] (fp32) built once per forward.
// The tile width NB is a multiple of dk, so a thread sees both halves of every head it stores.
template <int NB>
struct EpiRope {
  __nv_bfloat16* D;
  long long ldd;
  int rope_cols, dk;
  const int* pos;
  const float* cos_t;
  const float* sin_t;
  int M, N;
  // optional side output: per rotated head (rope_cols / dk of them, in column order) the largest
  // row norm of the stored bf16 values, as float bits in an unsigned word (atomicMax on the bits
  // orders non-negative floats); the caller zeroes it.  Rows past M hold zeros and add nothing.
  unsigned int* norm_max;
  static constexpr int kSmemPerThread = 256;  // per warp: two 2 KB chunk buffers

  // squares of the bf16-rounded values: the norms of exactly what the attention kernels read
  __device__ __forceinline__ static float rounded_sq(const float* a, const float* b) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float x = __bfloat162float(__float2bfloat16_rn(a[j]));
      const float y = __bfloat162float(__float2bfloat16_rn(b[j]));
      s = fmaf(x, x, fmaf(y, y, s));
    }
    return s;
  }
  // after the last first-half chunk of a head: warp max of the 32 rows' norms, one atomic per warp
  __device__ __forceinline__ void publish_norm(float ss, int col0) const {
    float n = sqrtf(ss);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) n = fmaxf(n, __shfl_xor_sync(0xffffffffu, n, off));
    if ((threadIdx.x & 31) == 0) atomicMax(norm_max + col0 / dk, __float_as_uint(n));
  }

  // Warp-coalesced path (see warp_store_bf16).
  __device__ __forceinline__ void operator()(uint32_t taddr, int row, int n0, int, int, uint8_t* sm) const {
    if (!(ldd % 8 == 0 && N % 8 == 0 && aligned16(D))) return rowwise(taddr, row, n0);
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t* area = sm - lane * kSmemPerThread;
    const int row0 = row - lane;
    const int half = dk / 2;
    const int p = row < M ? pos[row] : 0;
    float ss = 0.f;  // running squared norm of this row's current head
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      const int col0 = n0 + c * 32;
      if (col0 < rope_cols) {
        const int o = col0 % dk;  // offset inside the head
        if (o >= half) continue;  // second half: stored together with its first-half partner
        const int cb = c + half / 32;
        uint32_t ra[32], rb[32];
        tmem_ld32(taddr + c * 32, ra);
        tmem_ld32(taddr + cb * 32, rb);
        tmem_ld_wait();
        if (col0 >= N) continue;
        float cs[32], sn[32], a[32], b[32];
        load_row32_f32(cos_t + static_cast<long long>(p) * half + o, (half % 4 == 0), 32, cs);
        load_row32_f32(sin_t + static_cast<long long>(p) * half + o, (half % 4 == 0), 32, sn);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x1 = __uint_as_float(ra[j]), x2 = __uint_as_float(rb[j]);
          a[j] = x1 * cs[j] - x2 * sn[j];
          b[j] = x1 * sn[j] + x2 * cs[j];
        }
        warp_store_bf16(area, a, lane, D, ldd, row0, col0, M, N);
        warp_store_bf16(area + 2048, b, lane, D, ldd, row0, col0 + half, M, N);
        if (norm_max != nullptr) {
          ss = (o == 0 ? 0.f : ss) + rounded_sq(a, b);
          if (o + 32 == half) publish_norm(ss, col0);
        }
      } else {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait();
        if (col0 >= N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        warp_store_bf16(area, v, lane, D, ldd, row0, col0, M, N);
      }
    }
  }

  __device__ __forceinline__ void rowwise(uint32_t taddr, int row, int n0) const {
    const bool vec = (ldd % 8 == 0);
    const int half = dk / 2;
    const int p = row < M ? pos[row] : 0;
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      const int col0 = n0 + c * 32;
      if (col0 < rope_cols) {
        const int o = col0 % dk;  // offset inside the head
        if (o >= half) continue;  // second half: stored together with its first-half partner
        const int cb = c + half / 32;
        uint32_t ra[32], rb[32];
        tmem_ld32(taddr + c * 32, ra);
        tmem_ld32(taddr + cb * 32, rb);
        tmem_ld_wait();
        if (col0 >= N) continue;
        float cs[32], sn[32], a[32], b[32];
        load_row32_f32(cos_t + static_cast<long long>(p) * half + o, (half % 4 == 0), 32, cs);
        load_row32_f32(sin_t + static_cast<long long>(p) * half + o, (half % 4 == 0), 32, sn);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x1 = __uint_as_float(ra[j]), x2 = __uint_as_float(rb[j]);
          a[j] = row < M ? x1 * cs[j] - x2 * sn[j] : 0.f;
          b[j] = row < M ? x1 * sn[j] + x2 * cs[j] : 0.f;
        }
        if (norm_max != nullptr) {  // every lane reaches the warp reduction
          ss = (o == 0 ? 0.f : ss) + rounded_sq(a, b);
          if (o + 32 == half) publish_norm(ss, col0);
        }
        if (row >= M) continue;
        store_row32_bf16(D + row * ldd + col0, vec, 32, a);
        store_row32_bf16(D + row * ldd + col0 + half, vec, 32, b);
      } else {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait();
        if (row >= M || col0 >= N) continue;
        const int nv = min(32, N - col0);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        store_row32_bf16(D + row * ldd + col0, vec && nv == 32, nv, v);
      }
    }
  }
};

}  // namespace gemm
}  // namespace ttb
