// RMSNorm backward callable from C with no device-memory allocation.
//
// This entry point has no counterpart in the reference framework. It exists for callers that
// must not allocate device memory on the call path: an allocator that is itself being
// instrumented or rebuilt, a host runtime that reserves all device memory up front, or a
// program that links the kernel library from C without PyTorch's caching allocator. The
// PyTorch binding `rmsnorm_bwd` allocates its weight-gradient partials through torch on every
// call; this entry point instead uses a fixed scratch array that lives in the library's own
// device image (a file-scope `__device__` array), so the library allocates nothing on any call.
//
// Contract:
//  * Same math and the same kernels as the PyTorch binding: dx is written into (or added to,
//    accumulate != 0) the fp32 residual gradient `dres` [N, d]; the weight gradient `dw` [d] is
//    written (or added to, dw_accumulate != 0). dy is fp32 (dy_f32 != 0) or bf16 [N, d]; x [N, d]
//    fp32; w [d] fp32; rstd [N, G] fp32 from the forward pass.
//  * Scratch limit: the call needs rmsnorm_bwd_noalloc_scratch_floats(N, d) floats of scratch
//    and the array holds TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS (8 MiB of fp32). A call that
//    needs more is rejected with TTB_NOALLOC_TOO_LARGE before anything is launched.
//    The need is min(ceil(N / 8), 4 * SMs) * d floats (one partial row per CTA). On a 148-SM
//    B200 that is at most 592 * d, so every N fits for d <= 3540; at d = 4096 calls fit up to
//    N = 4096 rows, at d = 8192 up to N = 2048 rows.
//  * Nothing has to start at zero: every launch writes each scratch element it later reads.
//  * The first call on each device (with that device current) looks up the scratch address
//    with cudaGetSymbolAddress. Make that first call before any CUDA stream capture begins.
//    The address is then cached per device index for the life of the process: it belongs to
//    the CUDA runtime's primary context of that device. Callers that make another context
//    current through the driver API, or that call cudaDeviceReset, must not use this entry
//    point afterwards in the same process.
//  * All calls on one device share the one scratch array. Calls that may overlap in time (two
//    streams without ordering between them, or two host threads) race on it; order them on one
//    stream or synchronise between them.
//  * Return value: 0 on success, else one of the codes below; rmsnorm_bwd_noalloc_last_error()
//    then gives a message for the calling thread.
#pragma once

#include <cuda_runtime.h>

#define TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS (2 * 1024 * 1024)

enum {
  TTB_NOALLOC_OK = 0,
  TTB_NOALLOC_BAD_ARGUMENT = 1,  // null pointer, non-positive size, d % 4 != 0, d > 8192, bad G
  TTB_NOALLOC_TOO_LARGE = 2,     // the call needs more scratch than the fixed array holds
  TTB_NOALLOC_SETUP_FAILED = 3,  // device query or scratch address lookup failed
  TTB_NOALLOC_LAUNCH_FAILED = 4  // a kernel launch reported a CUDA error
};

#ifdef __cplusplus
extern "C" {
#endif

int rmsnorm_bwd_noalloc(const void* dy, int dy_f32, const float* x, const float* w, const float* rstd, float* dres,
                        int accumulate, float* dw, int dw_accumulate, int N, int d, int G, cudaStream_t stream);

// Scratch floats a call with these sizes needs (the launch's partial rows times d).
long long rmsnorm_bwd_noalloc_scratch_floats(int N, int d);

// Capacity of the fixed scratch array, in floats.
long long rmsnorm_bwd_noalloc_max_scratch_floats(void);

// Message describing the calling thread's last failed call ("" if none failed).
const char* rmsnorm_bwd_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
