// Tensor-parallel all-reduce fused with the normalisation that follows it, over NVLink peer memory.
//
// Every rank's row-parallel GEMM (o_proj / down_proj) writes its partial [T, H] into its own half of a symmetric
// buffer (same offset on every rank, mapped into every peer's address space) -- or, in the push form, the GEMM's own
// epilogue stores each finished tile into this rank's slot of EVERY rank's buffer, so the NVLink transfer overlaps the
// remaining tiles' math and the sum below reads local memory only.  One kernel then, per row:
//   1. signals "my partial of call k is ready" to every peer (one flag store per peer, release at system scope) and
//      waits, bounded, until every peer's flag for call k has arrived (acquire);
//   2. reads the N partials over NVLink (16-byte peer loads) and sums them in fp32 in rank order 0..N-1, so every
//      rank computes bit-identical results;
//   3. applies, fused: o = rmsnorm(sum, w1); resid += o; x = rmsnorm(resid, w2) (the Gemma post-norm / residual /
//      pre-norm chain; w1 = null skips the first norm, w2 = null returns resid itself).
// Semantics of the reference's symmetric-memory pull-reduce (`moe-gemm/dp-moe-symmetric-memory/symm_collectives.py:
// 57-90`, fixed peer order, fp32 accumulation) applied to the TP all-reduce, with the norm chain of
// `attention/gemma-fused-glue/rtx_glue.py:68-195` folded in.
//
// NVLS form (NVLink SHARP through a multicast mapping of the same buffer, `multimem` instructions): after the
// partials-ready barrier, rank r reduces column shard r of each row in the switch (one multimem.ld_reduce per 16
// bytes: the switch reads and adds every rank's copy, fp32 accumulation) and writes it to every rank's reduced-rows
// area with one multimem.st; a per-row flag, itself multicast, says the shard arrived everywhere.  A rank's NVLink
// traffic is one partial row out of the switch's reduction and the reduced row in, instead of (nranks - 1) partial
// rows; all ranks read the same reduced bytes.  The reference measures these instructions for its decode push /
// pull (`moe-gemm/dp-moe-symmetric-memory/symm_collectives.py:240-271`).
//
// Call k uses buffer half b = k % 2 and flag value e = epoch[b]; CTA 0 bumps epoch[1 - b] for call k + 1 (no CTA of
// call k + 1 can run before call k ends, stream order).  Rank r rewrites half b only at call k + 2, after passing call
// k + 1's barrier, which every peer entered only after finishing call k: two halves need one barrier per call.  The
// kernel arguments are the same for every call of a given parity, so a CUDA graph of a step replays correctly.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kArThreads = 256;

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

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = warp_id(), l = lane_id();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[32] = s;
  }
  __syncthreads();
  s = red[32];
  __syncthreads();
  return s;
}

// NVLink SHARP (NVLS) accesses through a multicast address: the switch reduces the loads of every rank's copy
// (fp32 accumulation of bf16 pairs) and replicates the stores into every rank's copy.
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(const void* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void mc_st16(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void mc_st_release_u32(int* p, int v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

template <int NR, int VPT, bool NVLS>
__global__ void __launch_bounds__(kArThreads) ar_norm2_kernel(const ArNormArgs a) {
  __shared__ float red[33];
  __shared__ int ok_s;
  const int b = a.half;
  const int e = a.epoch[b];
  // 1. signal every peer (flags of half b live after the data: [2][NR] ints at a.flag_offset bytes)
  if (blockIdx.x == 0 && threadIdx.x < NR) {
    int* peer_flags = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[threadIdx.x]) + a.flag_offset);
    st_release_sys(peer_flags + b * NR + a.rank, e);
  }
  if (threadIdx.x == 0) {
    const int* mine = reinterpret_cast<const int*>(reinterpret_cast<const char*>(a.peers[a.rank]) + a.flag_offset);
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
    if (blockIdx.x == 0) a.epoch[1 - b] = a.epoch[1 - b] + 1;   // call k + 1's flag value
  }
  __syncthreads();
  if (!ok_s) return;
  const int row = blockIdx.x;
  if constexpr (NVLS) {
    // 2'. this rank's column shard of the row: reduced in the switch, multicast into every rank's reduced rows
    const int chunks = a.H / 8, c0 = a.rank * chunks / NR, c1 = (a.rank + 1) * chunks / NR;
    const size_t poff = (static_cast<size_t>(b) * a.rows_cap + row) * a.H * 2;        // bytes
    char* mc = reinterpret_cast<char*>(a.mc);
    for (int c = c0 + threadIdx.x; c < c1; c += kArThreads)
      mc_st16(mc + a.res_offset + poff + c * 16, mc_ld_reduce_bf16x8(mc + poff + c * 16));
    __syncthreads();
    int* rflags = reinterpret_cast<int*>(mc + a.rowflag_offset) + (static_cast<size_t>(b) * a.rows_cap + row) * NR;
    if (threadIdx.x == 0) {
      __threadfence_system();
      mc_st_release_u32(rflags + a.rank, e);                    // "my shard of this row is in every copy"
      const int* mine = reinterpret_cast<const int*>(reinterpret_cast<const char*>(a.peers[a.rank]) +
                                                     a.rowflag_offset) + (static_cast<size_t>(b) * a.rows_cap + row) * NR;
      int good = 1;
      const unsigned long long t0 = global_ns();
      for (int r = 0; r < NR && good; ++r) {
        for (uint32_t it = 0; ld_acquire_sys(mine + r) < e; ++it) {
          if ((it & 255) == 255 && global_ns() - t0 > kWaitLimitNs) {
            good = 0;
            record_status(a.status, kTimeoutPeer);
            break;
          }
        }
      }
      asm volatile("fence.proxy.alias;" ::: "memory");         // the rows arrived through the multicast alias
      ok_s = good;
    }
    __syncthreads();
    if (!ok_s) return;
  }
  // 2. sum the partials of this row in rank order (pull: rank r's own buffer; push: slot r of this rank's buffer;
  // NVLS: the switch-reduced row, read once from this rank's buffer)

  const size_t off = (static_cast<size_t>(b) * (a.slots ? NR : 1) * a.rows_cap + row) * a.H;
  const size_t slot_elems = a.slots ? static_cast<size_t>(a.rows_cap) * a.H : 0;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * kArThreads;          // 8-element chunk
#pragma unroll
    for (int i = 0; i < 8; ++i) v[k][i] = 0.f;
    if (c * 8 >= a.H) continue;
#pragma unroll
    for (int r = 0; r < (NVLS ? 1 : NR); ++r) {
      const uint4 u = NVLS ? ld_peer16(reinterpret_cast<const char*>(a.peers[a.rank]) + a.res_offset +
                                       (static_cast<size_t>(b) * a.rows_cap + row) * a.H * 2 + c * 16)
                           : ld_peer16(reinterpret_cast<const __nv_bfloat16*>(a.peers[a.slots ? a.rank : r]) + off +
                                       r * slot_elems + c * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[k][2 * i] += f.x;
        v[k][2 * i + 1] += f.y;
      }
    }
    // the unfused path rounds the all-reduced tensor to bf16 before the norm
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[k][i] = __bfloat162float(__float2bfloat16(v[k][i]));
      ss += v[k][i] * v[k][i];
    }
  }
  __nv_bfloat16* resid = reinterpret_cast<__nv_bfloat16*>(a.resid) + static_cast<size_t>(row) * a.H;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out) + static_cast<size_t>(row) * a.H;
  const __nv_bfloat16* w1 = reinterpret_cast<const __nv_bfloat16*>(a.w1);
  const __nv_bfloat16* w2 = reinterpret_cast<const __nv_bfloat16*>(a.w2);
  // 3. o = norm1(sum); resid += o; x = norm2(resid)
  float inv1 = 1.f;
  if (w1) inv1 = rsqrtf(block_sum(ss, red) / a.H + a.eps);
  float ss2 = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * kArThreads;
    if (c * 8 >= a.H) continue;
    const uint4 ru = *reinterpret_cast<const uint4*>(resid + c * 8);
    const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&ru);
    uint4 wu = make_uint4(0, 0, 0, 0);
    if (w1) wu = *reinterpret_cast<const uint4*>(w1 + c * 8);
    const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wu);
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 rf = __bfloat1622float2(rh[i]);
      float o0 = v[k][2 * i], o1 = v[k][2 * i + 1];
      if (w1) {
        const float2 wf = __bfloat1622float2(wh[i]);
        o0 = __bfloat162float(__float2bfloat16(o0 * inv1 * (wf.x + a.plus_one)));
        o1 = __bfloat162float(__float2bfloat16(o1 * inv1 * (wf.y + a.plus_one)));
      }
      const __nv_bfloat162 nr = __floats2bfloat162_rn(rf.x + o0, rf.y + o1);
      packed[i] = *reinterpret_cast<const uint32_t*>(&nr);
      const float2 nf = __bfloat1622float2(nr);
      v[k][2 * i] = nf.x;
      v[k][2 * i + 1] = nf.y;
      ss2 += nf.x * nf.x + nf.y * nf.y;
    }
    *reinterpret_cast<uint4*>(resid + c * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  if (!w2) return;
  const float inv2 = rsqrtf(block_sum(ss2, red) / a.H + a.eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * kArThreads;
    if (c * 8 >= a.H) continue;
    const uint4 wu = *reinterpret_cast<const uint4*>(w2 + c * 8);
    const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wu);
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 wf = __bfloat1622float2(wh[i]);
      const __nv_bfloat162 o = __floats2bfloat162_rn(v[k][2 * i] * inv2 * (wf.x + a.plus_one),
                                                     v[k][2 * i + 1] * inv2 * (wf.y + a.plus_one));
      packed[i] = *reinterpret_cast<const uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(out + c * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

template <int NR, bool NVLS>
cudaError_t launch_nr(const ArNormArgs& a, cudaStream_t s) {
  const int chunks = a.H / 8;
  const int vpt = (chunks + kArThreads - 1) / kArThreads;
  switch (vpt) {
    case 1: ar_norm2_kernel<NR, 1, NVLS><<<a.T, kArThreads, 0, s>>>(a); break;
    case 2: ar_norm2_kernel<NR, 2, NVLS><<<a.T, kArThreads, 0, s>>>(a); break;
    case 3: ar_norm2_kernel<NR, 3, NVLS><<<a.T, kArThreads, 0, s>>>(a); break;
    case 4: ar_norm2_kernel<NR, 4, NVLS><<<a.T, kArThreads, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <int NR>
cudaError_t launch_mode(const ArNormArgs& a, cudaStream_t s) {
  return a.mc ? launch_nr<NR, true>(a, s) : launch_nr<NR, false>(a, s);
}

}  // namespace

cudaError_t ar_norm2(const ArNormArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.H % 8 || a.T > a.rows_cap || (a.half != 0 && a.half != 1) || a.rank < 0 || a.rank >= a.nranks)
    return cudaErrorInvalidValue;
  if (a.mc && (a.slots || a.nranks < 2 || a.res_offset % 16 || a.rowflag_offset % 16 ||
               reinterpret_cast<uintptr_t>(a.mc) % 16))
    return cudaErrorInvalidValue;
  switch (a.nranks) {
    case 1: return launch_mode<1>(a, s);
    case 2: return launch_mode<2>(a, s);
    case 4: return launch_mode<4>(a, s);
    case 8: return launch_mode<8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace iob
