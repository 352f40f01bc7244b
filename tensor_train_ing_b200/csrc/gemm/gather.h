// Host- and device-visible description of a row gather fused into a GEMM (see gather.cuh).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace ttb {
namespace gemm {

constexpr int kGatherMaxRanks = 8;
constexpr int kGatherSlabRows = 64;    // readiness granularity (rows of one done word)
constexpr int kGatherChunkVecs = 2048; // 16-byte vectors one warp copies per claim (32 KB)

// Chunks of one 64-row slab of a matrix with `cols` bf16 columns (a slab is 8 * cols vectors).
__host__ __device__ constexpr int gather_chunks_per_slab(int cols) {
  return (kGatherSlabRows * cols / 8 + kGatherChunkVecs - 1) / kGatherChunkVecs;
}

// One row-sharded operand.  dst is the local staging buffer [rows, cols] (row stride cols); rank r's
// rows start at src[r] (row stride cols).  rows % 64 == 0, cut[r] % 64 == 0 (a slab lies in one
// shard), cols % 8 == 0, every pointer 16-byte aligned.  A call that is the e-th gather into a done
// array passes target = e * gather_chunks_per_slab(cols).
struct GatherOp {
  const __nv_bfloat16* src[kGatherMaxRanks];
  int cut[kGatherMaxRanks + 1];
  int world;
  int rows, cols;
  __nv_bfloat16* dst;
  uint32_t* done;    // [rows / 64]
  uint32_t target;   // value every done word reaches when this call's copy of its slab is complete
};

struct Gather {
  GatherOp op[2];
  int nops;         // 0: no gather; 2: two operands of equal rows, slabs interleaved (dual-B GEMM)
  uint32_t* claim;  // {next chunk, finished CTAs}
};

}  // namespace gemm
}  // namespace ttb
