// Peer-memory collectives for data parallelism (see peer.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ttb {

constexpr int kMaxPeers = 8;

// Device addresses of the same symmetric buffer on every rank (index = rank).
struct PeerPtrs {
  void* p[kMaxPeers];
};

// One copy segment of the all-gather: n fp32 values from src (any rank's memory) to dst32 (local,
// optional) and as bf16 to dst16 (local, optional).  n is a multiple of 4; all pointers 16-byte aligned.
struct CopySeg {
  const float* src;
  float* dst32;
  __nv_bfloat16* dst16;
  long long n;
};

// Every rank's wait gives up after limit_cycles SM clock cycles and sets the timeout status word.
void peer_barrier(const PeerPtrs& pads, int world, int rank, uint32_t epoch, long long limit_cycles,
                  cudaStream_t stream);
int rs_reduce_blocks();
// out[i] (+)= sum over ranks of peers[q][off + i]; partial (nullable) gets per-block sums of squares
// (one per block of the default grid, rs_reduce_blocks()).  blocks > 0 caps the grid (a pull that
// runs beside compute kernels on another stream should leave them most of the SMs).
void rs_reduce_sq(const PeerPtrs& peers, int world, long long off, long long n, float* out, double* partial,
                  bool accumulate, int blocks, cudaStream_t stream);
void ag_pull_cast(const CopySeg* segs_device, int nseg, long long max_n, cudaStream_t stream);

}  // namespace ttb
