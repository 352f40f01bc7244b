// Kernels of the spectral (sigma-reparameterised) linear map; see spectral.cu for the formulas.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ttb {

constexpr int kSpectralMaxPartials = 1024;

// fp32 scratch floats the three entry points need for a [rows, cols] weight.
long long spectral_scratch_floats(int rows, int cols);

// sigma_out[0] = u^T W v; out (bf16, row stride ld) = W * gamma / max(|sigma|, floor).
void spectral_cast(const float* W, int rows, int cols, const float* gamma, const float* u, const float* v, float floor_,
                   float* sigma_out, float* partials, __nv_bfloat16* out, long long ld, cudaStream_t stream);

// dW (contiguous) and dgamma[0] from dW_eff (row stride ld) and the forward's sigma.
void spectral_grad(const float* dWe, long long ld, const float* W, int rows, int cols, const float* gamma,
                   const float* u, const float* v, const float* sigma, float floor_, float* partials, float* dW,
                   float* dgamma, cudaStream_t stream);

// One power-iteration step on u [rows] and v [cols].
void spectral_power_step(const float* W, int rows, int cols, float* u, float* v, float floor_, float* scratch,
                         cudaStream_t stream);

}  // namespace ttb
