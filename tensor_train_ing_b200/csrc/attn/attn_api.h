// Polynomial attention entry points (see poly_fwd.cu / poly_bwd.cu).
#pragma once

#include <cuda_runtime.h>

#include "params.h"

namespace ttb {

// y[B*T, H*dv] from the fused qkv buffer (bf16, row stride ld).  kind: 0 signed_product,
// 1 offset_square, 2 lower_degree_mix.  Head dims 64 or 128.
void poly_attention_fwd(int kind, int dk, int dv, const void* qkv, long long ld, attn::Params p, cudaStream_t stream);
// Writes dq1, dk1, (dq2, dk2), dv into p.dq (qkv layout, row stride p.ldd) and, for kinds 1/2,
// per-key-block kind-parameter partials into p.dpar [B*H, poly_attention_dpar_blocks(T), 4].
void poly_attention_bwd(int kind, int dk, int dv, const void* qkv, long long ld, const void* dout, long long ldo,
                        const int* doc_end, attn::Params p, cudaStream_t stream);
int poly_attention_dpar_blocks(int T);
// The persistent attention kernels launch min(tiles, SMs, limit) CTAs; limit 0 means no limit.
// Tests set a small limit so that every CTA works through many tiles.
void poly_attention_set_grid_limit(int limit);
namespace attn {
int persistent_grid(int tiles);
}

}  // namespace ttb
