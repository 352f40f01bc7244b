// Fused linear + cross-entropy entry points (see ce.cu).
#pragma once

#include <cuda_runtime.h>

#include "api.h"

namespace ttb {

// Number of 256-wide vocabulary tiles: the second dimension of the pmax/psum partial buffers.
int ce_num_tiles(int V);
// Forward over M rows: lse[M], loss_row[M] (0 where target < 0).  pmax/psum: [M, ce_num_tiles(V)].
// With zout, the scaled logits are also written there ([M, Npad] fp32, row stride ldz, -inf past V).
void ce_forward(const Operand& x, const Operand& w, int M, int V, int K, float alpha, const long long* targets,
                float* pmax, float* psum, float* tlogit, float* lse, float* loss_row, cudaStream_t stream,
                float* zout = nullptr, long long ldz = 0, int Npad = 0);
// dlogits as ce_backward_logits, from the logits the forward kept (an elementwise pass, no GEMM).
void ce_backward_from_logits(const float* z, long long ldz, int M, int Npad, float alpha, const long long* targets,
                             const float* lse, const float* grad, void* dlogits, long long ldd, cudaStream_t stream);
// dlogits [M, Npad] bf16 (row stride ldd) = grad * alpha * valid * (softmax(alpha x W^T) - onehot(target)).
void ce_backward_logits(const Operand& x, const Operand& w, int M, int Npad, int V, int K, float alpha,
                        const long long* targets, const float* lse, const float* grad, void* dlogits,
                        long long ldd, cudaStream_t stream);

}  // namespace ttb
