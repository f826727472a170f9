// Expert-parallel token exchange over NVLink peer memory (one symmetric allocation per EP group, mapped by every
// rank; no NCCL on this path).
//
// Dispatch: each rank pushes its quantized token rows straight into the receive slots of the ranks that own at
// least one of the token's top-k experts, and into its own slot (the local shared expert reads it there); 16-byte
// peer stores issued by the SMs, a token goes to each owner once, not once per expert.  Routing ids go to every rank
// (tiny).  Slot (src, t) of every receiver is fixed, so no
// counts have to be exchanged before the data: a rank with fewer than T_max tokens marks the remaining slots' ids
// -1.  The grouped expert GEMM then gathers its rows from the local receive buffer, and its epilogue stores each
// expert output row directly into the owning rank's combine buffer over NVLink (see `out_peers` in moe_gemm.cu):
// the GEMM -> combine transfer is fused into the GEMM.  The owner sums its tokens' rows in slot order with the
// routing weights (deterministic, fp32).
//
// The reference's fused DP-MoE does the same push / pull with Triton kernels over torch symmetric memory
// (`moe-gemm/dp-moe-symmetric-memory/symm_collectives.py:30-90`, `numinous_dp_moe.py:131-140`); idle ranks still
// join both barriers (`numinous_dp_moe.py:539-545`), as here (a rank with T = 0 runs the same launches).
//
// Barrier: one monotonically increasing epoch per group; every call signals epoch e to every peer (release, system
// scope, after a system fence) and waits -- bounded, ~2 s -- until every peer's flag reached e.  Two barriers per
// MoE layer (after dispatch, after the expert GEMMs) make buffer reuse across layers safe: a rank can overwrite a
// peer's receive buffer only after that peer passed the previous layer's second barrier.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One CTA per token slot t in [0, T_max).
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpDispatchArgs a) {
  const int t = blockIdx.x;
  const int row = a.rank * a.T_max + t;                       // receive slot on every peer
  __shared__ uint32_t dest_mask;
  if (threadIdx.x == 0) {
    uint32_t m = 0;
    if (t < a.T) {
      m = 1u << a.rank;               // own slot always: the shared expert reads every local token from it
      for (int k = 0; k < a.topk; ++k) {
        const int e = a.ids[t * a.topk + k];
        if (e >= 0 && e < a.world * a.E_loc) m |= 1u << (e / a.E_loc);
      }
    }
    dest_mask = m;
  }
  __syncthreads();
  // routing ids to every rank (-1 for empty slots)
  for (int i = threadIdx.x; i < a.world * a.topk; i += blockDim.x) {
    const int r = i / a.topk, k = i % a.topk;
    int* dst = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[r]) + a.off_ids) + row * a.topk + k;
    *dst = t < a.T ? a.ids[t * a.topk + k] : -1;
  }
  if (t >= a.T) {
    __threadfence_system();
    return;
  }
  const uint32_t m = dest_mask;
  const int n16 = a.row_bytes / 16, s4 = a.scale_bytes / 4;
  const uint4* xs = reinterpret_cast<const uint4*>(a.xq + static_cast<size_t>(t) * a.row_bytes);
  const uint32_t* ss = reinterpret_cast<const uint32_t*>(a.xs + static_cast<size_t>(t) * a.scale_bytes);
  for (int r = 0; r < a.world; ++r) {
    if (!(m & (1u << r))) continue;
    uint4* dx = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.peers[r]) + a.off_x +
                                         static_cast<size_t>(row) * a.row_bytes);
    uint32_t* ds = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a.peers[r]) + a.off_s +
                                               static_cast<size_t>(row) * a.scale_bytes);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dx[i] = xs[i];
    for (int i = threadIdx.x; i < s4; i += blockDim.x) ds[i] = ss[i];
  }
  // the peer stores (and the id stores above) are visible system-wide before the barrier kernel that follows
  // releases its flag
  __threadfence_system();
}

__global__ void ep_barrier_kernel(const long long* peers, long long off_flags, int rank, int world, int* epoch,
                                  int* status) {
  const int e = epoch[0] + 1;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    int* f = reinterpret_cast<int*>(reinterpret_cast<char*>(peers[threadIdx.x]) + off_flags) + rank;
    st_release_sys(f, e);
  }
  if (threadIdx.x < world) {
    const int* mine = reinterpret_cast<const int*>(reinterpret_cast<const char*>(peers[rank]) + off_flags) +
                      threadIdx.x;
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 0; ld_acquire_sys(mine) < e; ++it) {
      if ((it & 255) == 255 && global_ns() - t0 > kWaitLimitNs) {
        record_status(status, kTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) epoch[0] = e;
}

}  // namespace

cudaError_t ep_dispatch(const EpDispatchArgs& a, cudaStream_t s) {
  if (a.T_max <= 0 || a.T < 0 || a.T > a.T_max || a.world <= 0 || a.world > 32 || a.row_bytes % 16 ||
      a.scale_bytes % 4 || a.off_x % 16 || a.off_s % 4 || a.off_ids % 4)
    return cudaErrorInvalidValue;
  ep_dispatch_kernel<<<a.T_max, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t ep_barrier(const long long* peers, long long off_flags, int rank, int world, int* epoch, int* status,
                       cudaStream_t s) {
  if (world <= 0 || world > 32 || rank < 0 || rank >= world || off_flags % 4) return cudaErrorInvalidValue;
  ep_barrier_kernel<<<1, 32, 0, s>>>(peers, off_flags, rank, world, epoch, status);
  return cudaGetLastError();
}

}  // namespace iob
