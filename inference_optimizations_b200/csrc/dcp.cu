// Decode context parallelism (DCP): the partial-softmax merge of sparse-MLA decode over NVLink peer memory.
//
// Every rank of a DCP group holds the latent rows of the positions it owns (owner rule p -> rank p % S, local slot
// p / S; `parallelism/dsa-decode-context-parallel/dcp_topk.py:3-9`) and runs the sparse-MLA decode kernel over its
// owned share of each token's top-k selection, writing (o_r bf16 [T, H, 512], lse_r fp32 [T, H], natural log) straight
// into its half of a symmetric buffer.  This kernel then merges the S partials for the heads this rank keeps
// (head group r: heads [r H / S, (r + 1) H / S), the input of a row-parallel o_proj):
//     m = max_s lse_s,  w_s = exp(lse_s - m),  o = sum_s w_s o_s / sum_s w_s,  lse = m + log(sum_s w_s)
// reading the peers' partials with 16-byte loads over NVLink; a rank that owns none of a token's rows contributes
// (0, -inf).  The reference merges with SGLang's all-gather + LSE combine (`0002-*.patch`, `_forward_flashmla_kv_dcp`);
// here the merge is a head-sharded pull, so each rank moves only 1/S of every partial.
//
// Synchronisation is folded into the kernel (as in comm.cu): call k uses buffer half b = k % 2 and flag value
// epoch[b]; every CTA signals every peer (system-scope release, idempotent) and waits -- bounded -- for every peer's
// flag, and CTA 0 bumps epoch[1 - b] for call k + 1.  Peers rewrite half b only after passing call k + 1's barrier.
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
__device__ __forceinline__ uint4 ld_peer16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// grid (T, ceil(Hg / 4)), 256 threads: 4 heads per CTA, 64 threads per head (8 latent dims each).
template <int NR>
__global__ void __launch_bounds__(256) dcp_merge_kernel(const DcpMergeArgs a) {
  __shared__ int ok_s;
  const int b = a.half;
  const int e = a.epoch[b];
  if (threadIdx.x < NR) {            // every CTA signals (idempotent): no CTA's progress depends on another's
    int* pf = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[threadIdx.x]) + a.off_flags);
    __threadfence_system();
    st_release_sys(pf + b * NR + a.rank, e);
  }
  if (threadIdx.x == 0) {
    const int* mine = reinterpret_cast<const int*>(reinterpret_cast<const char*>(a.peers[a.rank]) + a.off_flags);
    int good = 1;
    const unsigned long long t0 = global_ns();     // bounded: kWaitLimitNs for all peers together
    for (int r = 0; r < NR && good; ++r) {
      for (uint32_t it = 0; ld_acquire_sys(mine + b * NR + r) < e; ++it) {
        if ((it & 255) == 255 && global_ns() - t0 > kWaitLimitNs) {
          good = 0;
          record_status(a.status, kTimeoutPeer);
          break;
        }
      }
    }
    ok_s = good;
    if (blockIdx.x == 0 && blockIdx.y == 0) a.epoch[1 - b] = a.epoch[1 - b] + 1;
  }
  __syncthreads();
  if (!ok_s) return;
  const int t = blockIdx.x;
  const int hl = blockIdx.y * 4 + threadIdx.x / 64;             // head within this rank's group
  if (hl >= a.Hg) return;
  const int h = a.rank * a.Hg + hl;
  const int c = threadIdx.x % 64;                                 // 8-dim chunk
  // half b of every rank's buffer: o [T_max, H, 512] bf16, then lse [T_max, H] fp32
  const size_t half_bytes = static_cast<size_t>(a.T_max) * a.H * (512 * 2 + 4);
  const size_t o_off = a.off_data + b * half_bytes + (static_cast<size_t>(t) * a.H + h) * 1024 + c * 16;
  const size_t l_off = a.off_data + b * half_bytes + static_cast<size_t>(a.T_max) * a.H * 1024 +
                       (static_cast<size_t>(t) * a.H + h) * 4;
  float lse[NR];
  float m = -INFINITY;
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    lse[r] = *reinterpret_cast<const volatile float*>(reinterpret_cast<const char*>(a.peers[r]) + l_off);
    m = fmaxf(m, lse[r]);
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float den = 0.f;
  if (m != -INFINITY) {
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      if (lse[r] == -INFINITY) continue;
      const float w = __expf(lse[r] - m);
      den += w;
      const uint4 u = ld_peer16(reinterpret_cast<const char*>(a.peers[r]) + o_off);
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(hv[i]);
        acc[2 * i] += w * f.x;
        acc[2 * i + 1] += w * f.y;
      }
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    ow[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (static_cast<size_t>(t) * a.Hg + hl) * 512 +
                            c * 8) = o;
  if (c == 0 && a.lse_out) a.lse_out[static_cast<size_t>(t) * a.Hg + hl] = den > 0.f ? m + __logf(den) : -INFINITY;
}

}  // namespace

cudaError_t dcp_merge(const DcpMergeArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.T > a.T_max || a.H % a.nranks || a.Hg != a.H / a.nranks || (a.half != 0 && a.half != 1) || a.rank < 0 ||
      a.rank >= a.nranks || a.off_data % 16 || a.off_flags % 4)
    return cudaErrorInvalidValue;
  const dim3 grid(a.T, (a.Hg + 3) / 4);
  switch (a.nranks) {
    case 1: dcp_merge_kernel<1><<<grid, 256, 0, s>>>(a); break;
    case 2: dcp_merge_kernel<2><<<grid, 256, 0, s>>>(a); break;
    case 4: dcp_merge_kernel<4><<<grid, 256, 0, s>>>(a); break;
    case 8: dcp_merge_kernel<8><<<grid, 256, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace iob
