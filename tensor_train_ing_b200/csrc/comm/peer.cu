// Data-parallel collectives fused with their neighbouring work, reading peer GPUs' memory directly
// over NVLink / NVSwitch (symmetric buffers mapped into every rank's address space).
//
//   peer_barrier     every rank stores an epoch into each peer's signal slot (system-scope release)
//                    and waits, bounded, until all peers' epochs reached it (acquire).
//   rs_reduce_sq     reduce-scatter of the flat fp32 gradient buffer by pulling: rank r sums its own
//                    region of every rank's buffer in rank order (deterministic) into its own buffer
//                    and, in the same pass, emits per-CTA partial sums of squares for the global
//                    gradient-norm clip.  With ``accumulate`` the sum is added to the output instead
//                    (the per-layer gradient reduction of parameter-sharded training, which adds
//                    every micro-batch's summed layer gradient into the owner's accumulator).
//   ag_pull_cast     all-gather of the flat fp32 parameter buffer by pulling each owner's region, fused
//                    with the bf16 operand caches of the GEMM weights (one pass writes both).
//
// No TMA is used here (plain vector loads and stores), so nothing multicasts.
#include <cuda_bf16.h>

#include "../common/host.h"
#include "../common/sm100.cuh"
#include "peer.h"

namespace ttb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One block; thread q signals peer q and then waits for peer q's signal (epochs only grow).
__global__ void peer_barrier_kernel(PeerPtrs pads, int world, int rank, uint32_t epoch, long long limit,
                                    uint32_t* status) {
  const int q = threadIdx.x;
  if (q < world) {
    __threadfence_system();  // this GPU's earlier writes (previous kernels) before the signal
    uint32_t* remote = reinterpret_cast<uint32_t*>(pads.p[q]) + rank;  // my slot in peer q's pad
    st_release_sys(remote, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(pads.p[rank]) + q;
    const long long t0 = clock64();
    while (static_cast<int32_t>(ld_acquire_sys(mine) - epoch) < 0) {
      if (clock64() - t0 > limit) {
        atomicCAS(status, 0u, static_cast<uint32_t>(kErrTimeoutPeer));
        break;
      }
    }
    __threadfence_system();
  }
  __syncthreads();
}

// out[i] = sum_q peers[q][off + i] (+ out[i] when accumulating) for i < n (float4 granularity; n and
// off multiples of 4), partial[blockIdx.x] = sum of out[i]^2 over this block's elements (fp32 tree
// inside the block; skipped when partial is null).
__global__ void __launch_bounds__(kThreads) rs_reduce_sq_kernel(PeerPtrs peers, int world, long long off, long long n,
                                                               float* out, double* partial, int accumulate) {
  __shared__ float red[kThreads / 32];
  float acc = 0.f;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // peer memory is read through L2 only (__ldcg): no stale L1 lines across steps
    float4 s = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers.p[0]) + off) + i);
    for (int q = 1; q < world; ++q) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers.p[q]) + off) + i);
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    if (accumulate) {
      const float4 o = reinterpret_cast<const float4*>(out)[i];
      s.x += o.x; s.y += o.y; s.z += o.z; s.w += o.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0 && partial != nullptr) {
    double t = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

// Segment j: copy n fp32 values from src to dst32 (if not null) and write bf16 copies to dst16 (if
// not null).  Blocks are spread over the segments in proportion to their sizes by the host.
__global__ void __launch_bounds__(kThreads) ag_pull_cast_kernel(const CopySeg* __restrict__ segs, int nseg) {
  const int j = blockIdx.y;
  if (j >= nseg) return;
  const CopySeg sg = segs[j];
  const long long n4 = sg.n / 4;
  const float4* src = reinterpret_cast<const float4*>(sg.src);
  // four 16-byte loads in flight per thread before the stores: a peer read takes microseconds, so
  // the link stays busy only with several MB outstanding across the grid
  constexpr int kUnroll = 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = __ldcg(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (sg.dst32 != nullptr) reinterpret_cast<float4*>(sg.dst32)[i + u * stride] = v[u];
      if (sg.dst16 != nullptr)
        reinterpret_cast<uint2*>(sg.dst16)[i + u * stride] =
            make_uint2(pack_bf16(v[u].x, v[u].y), pack_bf16(v[u].z, v[u].w));
    }
  }
  for (; i < n4; i += stride) {
    const float4 v = __ldcg(src + i);
    if (sg.dst32 != nullptr) reinterpret_cast<float4*>(sg.dst32)[i] = v;
    if (sg.dst16 != nullptr)
      reinterpret_cast<uint2*>(sg.dst16)[i] = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
  }
}

}  // namespace

void peer_barrier(const PeerPtrs& pads, int world, int rank, uint32_t epoch, long long limit_cycles,
                  cudaStream_t stream) {
  TTB_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "peer_barrier: bad world/rank");
  TTB_CHECK(limit_cycles > 0, "peer_barrier: the wait needs a limit");
  peer_barrier_kernel<<<1, 32, 0, stream>>>(pads, world, rank, epoch, limit_cycles, status_ptr());
  TTB_CUDA_CHECK(cudaGetLastError());
}

int rs_reduce_blocks() { return 4 * num_sms(); }

void rs_reduce_sq(const PeerPtrs& peers, int world, long long off, long long n, float* out, double* partial,
                  bool accumulate, int blocks, cudaStream_t stream) {
  TTB_CHECK(world >= 1 && world <= kMaxPeers, "rs_reduce_sq: bad world");
  TTB_CHECK(n % 4 == 0 && off % 4 == 0, "rs_reduce_sq: region must be float4 aligned");
  TTB_CHECK(partial == nullptr || blocks == 0, "rs_reduce_sq: partial sums need the default grid");
  if (n == 0) return;
  const int grid = blocks > 0 && blocks < rs_reduce_blocks() ? blocks : rs_reduce_blocks();
  rs_reduce_sq_kernel<<<grid, kThreads, 0, stream>>>(peers, world, off, n, out, partial, accumulate ? 1 : 0);
  TTB_CUDA_CHECK(cudaGetLastError());
}

void ag_pull_cast(const CopySeg* segs_device, int nseg, long long max_n, cudaStream_t stream) {
  if (nseg == 0) return;
  const long long per_block = static_cast<long long>(kThreads) * 4 * 8;
  long long bx = (max_n + per_block - 1) / per_block;
  if (bx < 1) bx = 1;
  if (bx > 256) bx = 256;
  TTB_CHECK(nseg <= 65535, "ag_pull_cast: too many segments");
  ag_pull_cast_kernel<<<dim3(static_cast<unsigned>(bx), nseg), kThreads, 0, stream>>>(segs_device, nseg);
  TTB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ttb
