// Launch parameters of the polynomial-attention kernels (host and device visible, no device code).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace ttb {
namespace attn {

struct Params {
  int B, T, H;
  int cq1, ck1, cq2, ck2, cv;  // column offsets of head 0 of each projection inside qkv
  const int* pos;              // [B*T] position inside the document
  const int* doc;              // [B*T] document id (<0 = padding)
  const float* row_scale;      // [B*T] n_visible^-p, 0 for padding
  const float* par;            // [H*4] kind parameters (b or c0,c1,c2,c12)
  float sm;                    // 1/sqrt(dk)
  __nv_bfloat16* y;            // forward output [B*T, H*dv]
  long long ldy;
  // backward
  __nv_bfloat16* dq;           // [B*T, ld] gradient buffer in the qkv layout (dq1, dk1, dq2, dk2, dv)
  long long ldd;
  float* dpar;                 // [B*H, nblocks, 4] per-key-block partials of the kind-parameter grads
  int dpar_blocks;
  uint32_t* status;
  // rotary tables [positions, dk/2] fp32: when set, the backward writes dq/dk with the rotary
  // embedding undone (gradients w.r.t. the pre-rotation projections)
  const float* rope_cos;
  const float* rope_sin;
};

}  // namespace attn
}  // namespace ttb
