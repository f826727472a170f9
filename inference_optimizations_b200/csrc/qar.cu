// Quantized two-shot all-reduce over peer memory: FP8 E4M3 payload with one fp32 scale per 128 values, so about
// half the bytes of a bf16 all-reduce cross the links (the reference's PCIe all-reduce,
// `parallelism/fp8-pcie-allreduce/fp8_pcie_allreduce.py:1-30`; here over NVLink peer stores).
//   1. push:    every rank quantizes its tensor per 128-value group and stores group g into the receive buffer of
//               the rank owning g (contiguous group ranges, one per rank), slot [src];
//   2. reduce:  (after a barrier) the owner dequantizes its groups from every source in rank order, sums in fp32,
//               quantizes the sum once and stores it into every rank's gather buffer;
//   3. gather:  (after a barrier) every rank dequantizes all reduced groups.
// Every rank reads the same reduced bytes, so the results are bitwise identical on all ranks.  Each barrier is
// folded into the start of the kernel that needs it (every CTA signals the call's epoch to every peer, then waits
// for all peers' flags, bounded; flags only grow).  The push kernel bumps the epoch, so the two later kernels of the
// call read it after it changed (stream order).  A rank overwrites a peer's receive buffer (next call's push) only
// after passing this call's gather barrier, i.e. after every peer finished reading it in its reduce.
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

// Group record: 128 E4M3 bytes + fp32 scale (132 bytes, stored as 128 + 4 in two arrays for alignment).
struct QarView {
  char* base;
  __device__ uint8_t* q(const QarArgs& a, int region, int src, int t, int g) const {
    return reinterpret_cast<uint8_t*>(base + (region ? a.off_gather_q : a.off_recv_q)) +
           ((static_cast<size_t>(src) * a.T_max + t) * a.G + g) * 128;
  }
  __device__ float* s(const QarArgs& a, int region, int src, int t, int g) const {
    return reinterpret_cast<float*>(base + (region ? a.off_gather_s : a.off_recv_s)) +
           (static_cast<size_t>(src) * a.T_max + t) * a.G + g;
  }
};

__device__ __forceinline__ bool qar_barrier(const QarArgs& a, int phase) {
  __shared__ int ok_s;
  const int e = a.epoch[0];                     // bumped by this call's push kernel
  if (threadIdx.x < a.nranks) {
    int* pf = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[threadIdx.x]) + a.off_flags) +
              phase * a.nranks + a.rank;
    __threadfence_system();
    st_release_sys(pf, e);
  }
  if (threadIdx.x == 0) {
    const int* mine = reinterpret_cast<const int*>(reinterpret_cast<const char*>(a.peers[a.rank]) + a.off_flags) +
                      phase * a.nranks;
    int good = 1;
    const unsigned long long t0 = global_ns();
    for (int r = 0; r < a.nranks && good; ++r) {
      for (uint32_t it = 0; ld_acquire_sys(mine + r) < e; ++it) {
        if ((it & 255) == 255 && global_ns() - t0 > kWaitLimitNs) {
          good = 0;
          record_status(a.status, kTimeoutPeer);
          break;
        }
      }
    }
    ok_s = good;
  }
  __syncthreads();
  return ok_s != 0;
}

// Quantize 128 values held 4 per lane: returns the packed E4M3 word of this lane and the group scale.
__device__ __forceinline__ uint32_t quant128(const float v[4], float& scale) {
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  m = warp_max(m);
  scale = m > 0.f ? m / 448.f : 1.f;
  const float inv = 1.f / scale;
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) w |= static_cast<uint32_t>(float_to_e4m3(v[j] * inv)) << (8 * j);
  return w;
}

// grid (T, ceil(G / 8)), 256 threads: warp = one 128-value group.
__global__ void __launch_bounds__(256) qar_push_kernel(const QarArgs a) {
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) a.epoch[0] = a.epoch[0] + 1;   // this call's epoch
  const int t = blockIdx.x, g = blockIdx.y * 8 + warp_id(), lane = lane_id();
  if (g >= a.G) return;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x) + static_cast<size_t>(t) * a.H + g * 128;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(x[lane * 4 + j]);
  float sc;
  const uint32_t w = quant128(v, sc);
  const int owner = g / a.per;
  const QarView peer{reinterpret_cast<char*>(a.peers[owner])};
  reinterpret_cast<uint32_t*>(peer.q(a, 0, a.rank, t, g))[lane] = w;
  if (lane == 0) *peer.s(a, 0, a.rank, t, g) = sc;
  __threadfence_system();   // peer stores visible before the next kernel's barrier releases its flag
}

__global__ void __launch_bounds__(256) qar_reduce_kernel(const QarArgs a) {
  if (!qar_barrier(a, 0)) return;
  const int t = blockIdx.x, lane = lane_id();
  const int g = a.rank * a.per + blockIdx.y * 8 + warp_id();
  if (g >= min(a.G, (a.rank + 1) * a.per)) return;
  const QarView me{reinterpret_cast<char*>(a.peers[a.rank])};
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  for (int src = 0; src < a.nranks; ++src) {               // fixed order: identical sums everywhere
    const uint32_t w = reinterpret_cast<const volatile uint32_t*>(me.q(a, 0, src, t, g))[lane];
    const float sc = *reinterpret_cast<const volatile float*>(me.s(a, 0, src, t, g));
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] += e4m3_to_float(static_cast<uint8_t>(w >> (8 * j))) * sc;
  }
  float sc;
  const uint32_t w = quant128(v, sc);
  for (int r = 0; r < a.nranks; ++r) {
    const QarView peer{reinterpret_cast<char*>(a.peers[r])};
    reinterpret_cast<uint32_t*>(peer.q(a, 1, 0, t, g))[lane] = w;
    if (lane == 0) *peer.s(a, 1, 0, t, g) = sc;
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) qar_gather_kernel(const QarArgs a) {
  if (!qar_barrier(a, 1)) return;
  const int t = blockIdx.x, g = blockIdx.y * 8 + warp_id(), lane = lane_id();
  if (g >= a.G) return;
  const QarView me{reinterpret_cast<char*>(a.peers[a.rank])};
  const uint32_t w = reinterpret_cast<const volatile uint32_t*>(me.q(a, 1, 0, t, g))[lane];
  const float sc = *reinterpret_cast<const volatile float*>(me.s(a, 1, 0, t, g));
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(a.y) + static_cast<size_t>(t) * a.H + g * 128 + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) y[j] = __float2bfloat16(e4m3_to_float(static_cast<uint8_t>(w >> (8 * j))) * sc);
}

}  // namespace

cudaError_t qar_allreduce(const QarArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.H % 128 || a.T > a.T_max || a.nranks < 1 || a.nranks > 32 || a.G != a.H / 128 ||
      a.per != (a.G + a.nranks - 1) / a.nranks)
    return cudaErrorInvalidValue;
  const dim3 grid(a.T, (a.G + 7) / 8), grid_r(a.T, (a.per + 7) / 8);
  qar_push_kernel<<<grid, 256, 0, s>>>(a);
  qar_reduce_kernel<<<grid_r, 256, 0, s>>>(a);
  qar_gather_kernel<<<grid, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace iob
