// Optimizer update kernels: AdamW over a list of tensors and the element-wise stages of Muon
// around its Newton-Schulz GEMMs. The gradient-clip coefficient is read from device memory, so a
// step needs no host synchronisation and no separate pass that scales the gradients first.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ttb {

// One tensor of a multi-tensor AdamW launch (fp32, contiguous, n elements). Eight 8-byte fields,
// so a [count, 8] int64 device tensor built on the host can be passed as the descriptor array.
struct AdamwTensor {
  float* p;
  const float* g;
  float* exp_avg;
  float* exp_avg_sq;
  float* step;             // this tensor's step counter (a float, like torch's AdamW state)
  __nv_bfloat16* cache;    // optional bf16 copy of p written after the update (nullptr: none)
  long long n;
  long long first_chunk;   // chunks (of kAdamwChunk elements) of the tensors before this one
};
static_assert(sizeof(AdamwTensor) == 64, "descriptor layout is shared with the host");

constexpr long long kAdamwChunk = 16384;

// Increments every step counter, then applies one AdamW update (decoupled decay) to every tensor:
// g' = g * grad_scale (if given); p -= lr*wd*p; m = b1 m + (1-b1) g'; v = b2 v + (1-b2) g'^2;
// p -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps).
void adamw_update(const AdamwTensor* tensors, int count, long long total_chunks, float lr, float beta1, float beta2,
                  float eps, float weight_decay, const float* grad_scale, cudaStream_t stream);

// Muon, first stage, for a [rows, cols] matrix: g' = g * grad_scale; buf = lerp(buf, g', w_buf);
// u = nesterov ? lerp(g', buf, w_nesterov) : buf; x = bf16(u), stored [rows, cols] or, with
// transpose, [cols, rows]; partial[b] = sum of x^2 over the tiles block b handled. Returns the
// number of partials written (at most kMuonMaxPartials).
int muon_prepare(const float* g, float* buf, __nv_bfloat16* x, float* partial, int rows, int cols, float w_buf,
                 float w_nesterov, bool nesterov, bool transpose, const float* grad_scale, cudaStream_t stream);

constexpr int kMuonMaxPartials = 1024;

// Muon, second stage: x = bf16(x / d) with d = max(bf16(sqrt(sum(partial))), eps), the rounding
// of a bf16 matrix divided by its bf16 Frobenius norm.
void muon_normalize(__nv_bfloat16* x, long long n, const float* partial, int n_partial, float eps,
                    cudaStream_t stream);

// Muon, last stage, for p [rows, cols]: p = p * decay + alpha * o, where o is the orthogonalised
// update stored [rows, cols] or (transposed) [cols, rows]; optionally writes bf16(p) into cache
// (row-major, leading dimension cache_ld).
void muon_apply(float* p, const __nv_bfloat16* o, int rows, int cols, bool transposed, float decay, float alpha,
                __nv_bfloat16* cache, long long cache_ld, cudaStream_t stream);

}  // namespace ttb
