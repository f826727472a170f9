// Prefill -> decode KV page transfer inside one node (prefill and decode engines on different GPUs): the prefill
// side pushes finished pages straight into the decode engine's pool over NVLink with 16-byte peer stores -- one launch
// for every (page pair x layer) -- then publishes a sequence number in the decode GPU's memory; the decode side waits
// for it on its own stream (bounded) before the step that reads the pages.  The reference does the same with a
// Triton copy over CUDA-IPC-mapped pools (`parallelism/in-node-pd-disaggregation/pd_nvlink_copy.py:1-30`).
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

// grid (pairs, layers): CTA copies page src_pages[i] of layer l into page dst_pages[i] of the peer's layer l.
__global__ void __launch_bounds__(256) pd_copy_kernel(const PdCopyArgs a) {
  const int i = blockIdx.x, l = blockIdx.y;
  const int sp = a.src_pages[i], dp = a.dst_pages[i];
  if (sp < 0 || dp < 0) return;
  const uint4* src = reinterpret_cast<const uint4*>(a.src + l * a.src_layer_stride + static_cast<long long>(sp) *
                                                                                          a.page_bytes);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.dst) + l * a.dst_layer_stride +
                                        static_cast<long long>(dp) * a.page_bytes);
  const int n16 = static_cast<int>(a.page_bytes / 16);
  for (int k = threadIdx.x; k < n16; k += blockDim.x) dst[k] = src[k];
  __threadfence_system();   // the peer stores are visible before pd_signal's release (a separate kernel)
}

__global__ void pd_signal_kernel(int* peer_flag, int value) {
  __threadfence_system();
  st_release_sys(peer_flag, value);
}

__global__ void pd_wait_kernel(const int* flag, int value, int* status) {
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0; ld_acquire_sys(flag) < value; ++it) {
    if ((it & 255) == 255 && global_ns() - t0 > kWaitLimitNs) {
      record_status(status, kTimeoutPeer);
      return;
    }
  }
}

}  // namespace

cudaError_t pd_copy(const PdCopyArgs& a, cudaStream_t s) {
  if (a.n_pairs == 0) return cudaSuccess;
  if (a.page_bytes % 16 || a.src_layer_stride % 16 || a.dst_layer_stride % 16 || a.layers <= 0 ||
      reinterpret_cast<uintptr_t>(a.src) % 16 || reinterpret_cast<uintptr_t>(a.dst) % 16)
    return cudaErrorInvalidValue;
  pd_copy_kernel<<<dim3(a.n_pairs, a.layers), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t pd_signal(int* peer_flag, int value, cudaStream_t s) {
  pd_signal_kernel<<<1, 1, 0, s>>>(peer_flag, value);
  return cudaGetLastError();
}

cudaError_t pd_wait(const int* flag, int value, int* status, cudaStream_t s) {
  pd_wait_kernel<<<1, 1, 0, s>>>(flag, value, status);
  return cudaGetLastError();
}

}  // namespace iob
