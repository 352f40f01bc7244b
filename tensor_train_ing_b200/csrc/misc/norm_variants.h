// Row-normalisation variants beyond plain (group) RMSNorm, on one kernel family:
//
//   y[n, j] = x[n, j] * (a_n * w[j] + b * w2[j])
//
//   kNormLagged  a_n = *a_dev (1 / sqrt(lagged mean square + eps), a detached device scalar), b = 0
//   kNormTaper   a_n = g / r_n, b = (1 - g) c   (TaperNorm; r_n = sqrt(mean_j x^2 + eps))
//   kNormRms     a_n = 1 / r_n, b = 0           (RMSNorm with an fp32 result, for branch-output norms)
//
// The forward writes a bf16 result (a GEMM operand) and/or an fp32 result (optionally
// resid + alpha * y), and on request the per-row r_n and mean squares. The backward adds (or
// writes) dx, including the gradient through r_n (taper, rms) and an optional incoming gradient
// with respect to r_n (TaperNorm's anchor term), and reduces dw / dw2 in a fixed order.
#pragma once

#include <cuda_runtime.h>

namespace ttb {

enum NormVariant { kNormLagged = 0, kNormTaper = 1, kNormRms = 2 };

struct NormVariantArgs {
  int mode;
  int N, d;
  float eps;
  float g;            // taper gate
  float b;            // coefficient of w2
  const float* a_dev; // lagged scale (device scalar)
  const float* w;
  const float* w2;    // taper weight_tilde (nullptr when b == 0)
};

// resid (optional, fp32 [N, d]): y32 = resid + alpha * y. Any output pointer may be null.
void norm_variant_fwd(const NormVariantArgs& a, const float* x, const float* resid, float alpha, void* y16,
                      float* y32, float* r_out, float* msq_out, cudaStream_t stream);

// Rows of weight-gradient partials the backward uses for N rows.
int norm_variant_partials(int N);

// dy: bf16 or fp32 [N, d], scaled by dy_scale; r_row: the forward's r_out (needed for taper and rms);
// dr_row (optional): incoming gradient with respect to r_n. dx is written or added (dx_accumulate).
// dw / dw2 (optional) receive sum_n dy * dL/dw; partials: fp32 scratch of norm_variant_partials(N) * d
// (two such blocks when dw2 is given).
void norm_variant_bwd(const NormVariantArgs& a, const void* dy, bool dy_f32, float dy_scale, const float* x,
                      const float* r_row, const float* dr_row, float* dx, bool dx_accumulate, float* dw, float* dw2,
                      float* partials, cudaStream_t stream);

}  // namespace ttb
