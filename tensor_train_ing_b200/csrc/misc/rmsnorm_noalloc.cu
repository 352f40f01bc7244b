// RMSNorm backward with its weight-gradient scratch in a fixed `__device__` array, callable from C.
// No counterpart in the reference framework; the contract (scratch limit, first-call setup,
// no overlapping calls) is documented in rmsnorm_noalloc.h.
//
// The launches are the ones the PyTorch binding makes (ttb::rmsnorm_bwd: the per-CTA partial
// kernel, then the fixed-order column sum), so results match that binding exactly; only the
// home of the [partials, d] fp32 scratch differs.
#include <cstdint>
#include <cstdio>
#include <exception>
#include <mutex>

#include "../common/host.h"
#include "rmsnorm_noalloc.h"
#include "rowops.h"

namespace {

constexpr int kMaxDevices = 64;

// The scratch: partial weight-gradient rows, one per CTA of the partial kernel.
static __device__ __align__(256) float g_rmsnorm_dw_scratch[TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS];

float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_setup_mutex;
thread_local char g_last_error[256] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "rmsnorm_bwd_noalloc: %s", msg);
  return code;
}

bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// Device address of the scratch array for the current device (looked up once per device).
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TTB_NOALLOC_SETUP_FAILED, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(TTB_NOALLOC_SETUP_FAILED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rmsnorm_dw_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(TTB_NOALLOC_SETUP_FAILED, e != cudaSuccess ? cudaGetErrorString(e) : "null scratch address");
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return TTB_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) long long rmsnorm_bwd_noalloc_scratch_floats(int N, int d) {
  if (N <= 0 || d <= 0) return 0;
  try {
    return static_cast<long long>(ttb::rmsnorm_bwd_partials(N)) * d;
  } catch (const std::exception&) {
    return -1;
  }
}

extern "C" __attribute__((visibility("default"))) long long rmsnorm_bwd_noalloc_max_scratch_floats(void) {
  return TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS;
}

extern "C" __attribute__((visibility("default"))) const char* rmsnorm_bwd_noalloc_last_error(void) {
  return g_last_error;
}

extern "C" __attribute__((visibility("default"))) int rmsnorm_bwd_noalloc(
    const void* dy, int dy_f32, const float* x, const float* w, const float* rstd, float* dres, int accumulate,
    float* dw, int dw_accumulate, int N, int d, int G, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (!dy || !x || !w || !rstd || !dres || !dw) return fail(TTB_NOALLOC_BAD_ARGUMENT, "null pointer");
  if (N <= 0 || d <= 0 || d % 4 != 0 || d > 8192)
    return fail(TTB_NOALLOC_BAD_ARGUMENT, "need N > 0 and d a positive multiple of 4, at most 8192");
  if (G < 1 || G > 8 || d % G != 0 || (d / G) % 4 != 0)
    return fail(TTB_NOALLOC_BAD_ARGUMENT, "need 1 <= G <= 8 with d / G a multiple of 4");
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(dres, 16) || !aligned(dy, dy_f32 ? 16 : 8))
    return fail(TTB_NOALLOC_BAD_ARGUMENT, "x, w, dres (and fp32 dy) need 16-byte alignment, bf16 dy 8-byte");
  const long long need = rmsnorm_bwd_noalloc_scratch_floats(N, d);
  if (need < 0) return fail(TTB_NOALLOC_SETUP_FAILED, "device query failed");
  if (need > TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "N=%d, d=%d needs %lld scratch floats; the fixed array holds %d", N, d, need,
                  TTB_RMSNORM_NOALLOC_MAX_SCRATCH_FLOATS);
    return fail(TTB_NOALLOC_TOO_LARGE, msg);
  }
  float* scratch = nullptr;
  if (const int rc = scratch_for_current_device(&scratch)) return rc;
  try {
    ttb::rmsnorm_bwd(dy, dy_f32 != 0, x, w, rstd, dres, accumulate != 0, scratch, dw, dw_accumulate != 0, N, d, G,
                     stream);
  } catch (const std::exception& ex) {
    return fail(TTB_NOALLOC_LAUNCH_FAILED, ex.what());
  }
  return TTB_NOALLOC_OK;
}
