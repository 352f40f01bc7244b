// Host-side helpers shared by the launchers: TMA descriptor encoding through the driver entry
// point (no link-time dependency on libcuda), device properties and error checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace ttb {

#define TTB_CUDA_CHECK(expr)                                                                           \
  do {                                                                                                 \
    cudaError_t _e = (expr);                                                                           \
    if (_e != cudaSuccess)                                                                             \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " __FILE__ \
                               ":" + std::to_string(__LINE__));                                        \
  } while (0)

#define TTB_CHECK(cond, msg)                                                             \
  do {                                                                                   \
    if (!(cond)) throw std::invalid_argument(std::string("tensor_train_ing_b200: ") + msg); \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Driver-API calls need a current context on the calling thread (autograd runs backward on its
// own worker threads): touch the runtime once per thread so the primary context is bound.
inline void ensure_context() {
  thread_local bool bound = false;
  if (!bound) {
    TTB_CUDA_CHECK(cudaFree(nullptr));
    bound = true;
  }
}

inline EncodeTiledFn encode_tiled_fn() {
  ensure_context();
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    TTB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Row-major 2-D map: `inner` contiguous elements per row, `outer` rows, `ld` elements between rows.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                                uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  TTB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TTB_CHECK((ld * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TTB_CHECK((box_inner * elem_bytes) % 16 == 0, "TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

// 3-D map (inner, mid, outer) with explicit byte strides for mid and outer.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                                uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                                uint32_t b0, uint32_t b1, uint32_t b2,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  TTB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TTB_CHECK(stride1_bytes % 16 == 0 && stride2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed: " + std::to_string(int(r)));
  return m;
}

// One error word per device, allocated on first use; kernels record bounded-wait timeouts here.
inline uint32_t* status_ptr() {
  static uint32_t* ptrs[64] = {nullptr};
  int dev = 0;
  TTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (ptrs[dev] == nullptr) {
    TTB_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(uint32_t)));
    TTB_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(uint32_t)));
  }
  return ptrs[dev];
}

// Reads the device error word of the current device and clears it (synchronous).
inline uint32_t status_read_and_reset() {
  uint32_t v = 0;
  uint32_t* p = status_ptr();
  TTB_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost));
  TTB_CUDA_CHECK(cudaMemset(p, 0, sizeof(uint32_t)));
  return v;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    TTB_CUDA_CHECK(cudaGetDevice(&dev));
    TTB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

}  // namespace ttb
