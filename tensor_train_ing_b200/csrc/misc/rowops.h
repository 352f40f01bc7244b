// Row-wise / elementwise kernels (see rowops.cu).
#pragma once

#include <cuda_runtime.h>

namespace ttb {

// (group) RMSNorm: y = bf16(x * rstd * w); rstd [N, G]
void rmsnorm_fwd(const float* x, const float* w, void* y, float* rstd, int N, int d, int G, float eps,
                 cudaStream_t stream);
// Number of per-CTA weight-grad partial rows rmsnorm_bwd needs in dw_part ([P, d] fp32).
int rmsnorm_bwd_partials(int N);
void rmsnorm_bwd(const void* dy, bool dy_f32, const float* x, const float* w, const float* rstd, float* dres,
                 bool accumulate, float* dw_part, float* dw, bool dw_accumulate, int N, int d, int G,
                 cudaStream_t stream);
// As rmsnorm_bwd; when out16 is not null it also writes bf16(dres_new * scale16) to out16 [N, d]
// (the bf16 operand the next backward GEMM needs, produced without a separate conversion pass).
void rmsnorm_bwd_ex(const void* dy, bool dy_f32, const float* x, const float* w, const float* rstd, float* dres,
                    bool accumulate, float* dw_part, float* dw, bool dw_accumulate, int N, int d, int G,
                    void* out16, float scale16, cudaStream_t stream);
// In-place rotary embedding of the first rope_cols columns (heads of width dk) of a bf16 [N, ld] buffer.
void rope_apply(void* buf, long long ld, int N, int rope_cols, int dk, const int* pos, const float* inv_freq,
                bool inverse, cudaStream_t stream);
// Embedding rows of a V-row table; ids outside [0, V) set kErrBadIndex in the status word and are
// skipped (zero rows forward, no gradient backward).
void embed_fwd(const long long* idx, const float* W, float* x, int N, int d, long long V, cudaStream_t stream);
void embed_bwd(const long long* sorted_ids, const long long* order, const float* dx, float* dW, int N, int d,
               long long V, cudaStream_t stream);

}  // namespace ttb
