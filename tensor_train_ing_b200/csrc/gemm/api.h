// C++ entry points of the GEMM family (no torch types; the bindings translate tensors).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "gather.h"

namespace ttb {

// One bf16 matrix operand in global memory.
//  A operand (M x K):  mn_major=false -> stored [M][K] with row stride ld;  true -> stored [K][M].
//  B operand (N x K):  mn_major=false -> stored [N][K];                     true -> stored [K][N].
struct Operand {
  const void* ptr;
  long long ld;
  bool mn_major;
};

// D[M,N] = alpha * (A B^T + bias) + beta * C.  With b2 the contraction is concatenated: B rows
// [0, k_split) come from b and [k_split, K) from b2 (k_split a multiple of 64), so
// A[:, :k_split] b^T + A[:, k_split:] b2^T accumulates in one pass.  tile_n picks the output tile
// width (128: six K stages; 256: four); 0 takes 128 for N <= 128 and 256 otherwise.  Each output
// element accumulates its K blocks in the same order either way.
void gemm_linear(const Operand& a, const Operand& b, int M, int N, int K, void* D, long long ldd, bool d_f32,
                 const void* C, long long ldc, bool c_f32, float alpha, float beta, const float* bias,
                 cudaStream_t stream, const Operand* b2 = nullptr, int k_split = 0, int tile_n = 0,
                 const gemm::Gather* gather = nullptr);

// l = x Wl^T (+bl), r = x Wr^T (+br), H = l*r (mode 0) or silu(l)*r (mode 1); all [M, N] bf16 with row stride ld.
void gemm_bilinear(const Operand& x, const Operand& wl, const Operand& wr, int M, int N, int K, void* H, void* Lo,
                   void* Ro, long long ld, const float* bias_l, const float* bias_r, int mode, cudaStream_t stream,
                   const gemm::Gather* gather = nullptr);

// dH = dY Wd (B operand = Wd^T view), fused with the bilinear backward: writes dl, dr [M, N] bf16
// (row stride ldo; the saved factors Lin / Rin have row stride ld).
void gemm_bilinear_grad(const Operand& dy, const Operand& wd, int M, int N, int K, const void* Lin, const void* Rin,
                        void* dL, void* dR, long long ld, long long ldo, int mode, cudaStream_t stream);

// qkv[M, N] = x W^T (bf16) with the rotary embedding applied to the first rope_cols columns
// (heads of width dk; cos/sin tables [positions, dk/2] fp32; pos [M] int32).  With norm_max
// (rope_cols / dk zeroed words) the epilogue also records, per rotated head, the largest row norm
// of the stored values (float bits), from which score bounds follow.
void gemm_qkv_rope(const Operand& x, const Operand& w, int M, int N, int K, void* D, long long ldd, int rope_cols,
                   int dk, const int* pos, const float* cos_t, const float* sin_t, cudaStream_t stream,
                   unsigned int* norm_max = nullptr, const gemm::Gather* gather = nullptr);

// Fused all-gather of row-sharded weights (gemm/gather.cuh).  The gemm_* calls above take an
// optional Gather whose operands' staging buffers are their B operands (wl and wr for the bilinear
// form): the CTA-pair GEMM copies the rows from the ranks' shards while it runs.  gather_rows runs
// the copy alone (the same chunks and done words), for consumers that are not CTA-pair GEMMs.
// gather_claim_counter() is this device's chunk counter pair (zeroed once, returned to zero by
// every launch).
void gather_rows(const gemm::Gather& g, cudaStream_t stream);
uint32_t* gather_claim_counter();

}  // namespace ttb
