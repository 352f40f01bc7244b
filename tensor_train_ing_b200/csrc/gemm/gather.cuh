// All-gather of a row-sharded bf16 weight fused into the GEMM that consumes it.
//
// Under parameter sharding each rank of a data-parallel group holds a slice of rows of every
// weight matrix (rank r: rows [cut[r], cut[r+1])) in symmetric memory, mapped into every rank's
// address space over NVLink.  A GEMM whose B operand is such a matrix takes a local staging buffer
// [rows, cols] as B and a Gather description: besides the producer / MMA / epilogue warps, two
// gather warps per CTA claim chunks of the matrix from a device counter (slab order, the
// order in which the tiles consume them), copy each from the owning rank's memory into the staging
// buffer with plain 16-byte loads and stores, and count the chunk into its 64-row slab's done word.
// (A chunk is a 32 KB piece of a 64-row slab, so matrices of any width split into many claims.)
// Before the TMA producer loads a B tile it waits, bounded, until the tile's slabs are complete.
// So every weight row crosses NVLink exactly once per call, the copy of later slabs overlaps the
// MMAs of earlier tiles, and TMA only ever reads this GPU's memory (never a peer's, never
// multicast).
//
// Ordering: the writer of a chunk (all lanes' stores, then __syncwarp, then lane 0) issues
// fence.proxy.async.global and a gpu-scope fence before its relaxed atomic increment; the producer
// reads the done word with ld.acquire.gpu and issues fence.proxy.async.global before its TMA loads,
// so the async-proxy reads observe the generic-proxy writes.
//
// Done words only grow: the e-th gather into a done array passes target = e * chunks per slab, so
// no reset is needed between calls (zero them once when the array is created).  The chunk counter is
// a {next, finished CTAs} pair that the last CTA to finish returns to zero, so launches that share
// one counter must be ordered on a stream.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "../common/sm100.cuh"
#include "gather.h"

namespace ttb {
namespace gemm {

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t gather_chunks(const Gather& g) {
  return static_cast<uint32_t>(g.nops) * static_cast<uint32_t>(g.op[0].rows / kGatherSlabRows) *
         static_cast<uint32_t>(gather_chunks_per_slab(g.op[0].cols));
}

// One warp copies chunks until every chunk of the call has been claimed.  Chunks are claimed in slab
// order (the two operands of a dual-B GEMM alternate slab by slab), each a 32 KB piece of a 64-row
// slab, so a wide matrix still splits into many claims.
template <int kUnroll>
__device__ __forceinline__ void gather_warp(const Gather& g, int lane) {
  const uint32_t total = gather_chunks(g);
  const uint32_t cps = static_cast<uint32_t>(gather_chunks_per_slab(g.op[0].cols));
  for (;;) {
    uint32_t c = 0;
    if (lane == 0) c = atomicAdd(g.claim, 1u);
    c = __shfl_sync(0xffffffffu, c, 0);
    if (c >= total) break;
    const uint32_t j = c / cps;  // position in slab order
    const int o = g.nops == 2 ? static_cast<int>(j & 1u) : 0;
    const int slab = static_cast<int>(g.nops == 2 ? (j >> 1) : j);
    const GatherOp& op = g.op[o];
    const int row = slab * kGatherSlabRows;
    int r = 0;
    while (r + 1 < op.world && row >= op.cut[r + 1]) ++r;
    const long long slab_vecs = static_cast<long long>(kGatherSlabRows) * op.cols / 8;
    const long long v0 = static_cast<long long>(c % cps) * kGatherChunkVecs;
    const int nvec = static_cast<int>(min(static_cast<long long>(kGatherChunkVecs), slab_vecs - v0));
    const uint4* s =
        reinterpret_cast<const uint4*>(op.src[r] + static_cast<long long>(row - op.cut[r]) * op.cols) + v0;
    uint4* d = reinterpret_cast<uint4*>(op.dst + static_cast<long long>(row) * op.cols) + v0;
    int i = lane;
    // peer memory through L2 only (__ldcg).  NVLink reads take microseconds, so the link is kept busy
    // only with many bytes in flight: kUnroll 16-byte loads per lane before the stores.
    for (; i + (kUnroll - 1) * 32 < nvec; i += kUnroll * 32) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = __ldcg(s + i + u * 32);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) d[i + u * 32] = v[u];
    }
    for (; i < nvec; i += 32) d[i] = __ldcg(s + i);
    __syncwarp();
    if (lane == 0) {
      fence_proxy_async_global();
      __threadfence();
      atomicAdd(op.done + slab, 1u);
    }
  }
}

// Bounded wait until staging rows [r0, r1) of operand o are complete; false (status recorded) when
// a wait ran out.
__device__ __forceinline__ bool gather_wait_rows(const Gather& g, int o, int r0, int r1, uint32_t* status) {
  const GatherOp& op = g.op[o];
  if (r1 > op.rows) r1 = op.rows;
  for (int slab = r0 / kGatherSlabRows; slab * kGatherSlabRows < r1; ++slab) {
    const uint32_t* w = op.done + slab;
    if (static_cast<int32_t>(ld_acquire_gpu(w) - op.target) >= 0) continue;
    const long long t0 = clock64();
    while (static_cast<int32_t>(ld_acquire_gpu(w) - op.target) < 0) {
      if (clock64() - t0 > kWaitLimitCycles) {
        record_error(status, kErrTimeoutProducer);
        return false;
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// Called by thread 0 of every CTA after its last barrier: the last CTA of the launch returns the
// chunk counter to zero for the next launch.
__device__ __forceinline__ void gather_finish(const Gather& g) {
  __threadfence();
  if (atomicAdd(g.claim + 1, 1u) == gridDim.x - 1) {
    atomicExch(g.claim, 0u);
    atomicExch(g.claim + 1, 0u);
  }
}

}  // namespace gemm
}  // namespace ttb
