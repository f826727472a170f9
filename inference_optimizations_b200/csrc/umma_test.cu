// Minimal tcgen05 GEMM used by the GPU tests to validate the primitives every tensor-core kernel here is built on:
// SW128 K-major shared-memory descriptors, the kind::f16 instruction descriptor, single-thread UMMA issue with
// commit-to-mbarrier, and the TMEM accumulator layout read back with tcgen05.ld (lane = row, column = n).
// C[M, N] fp32 = A[M, K] * B[N, K]^T; A, B bf16 row-major; M % 128 == 0, N % 16 == 0, N <= 256, K % 64 == 0.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

__global__ void __launch_bounds__(128) umma_gemm_kernel(const __nv_bfloat16* __restrict__ A,
                                                        const __nv_bfloat16* __restrict__ B, float* __restrict__ C,
                                                        int N, int K, int sw64) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                 // 128 x 128 B
  uint8_t* sB = smem + 128 * 128;     // N x 128 B
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int m0 = blockIdx.x * 128;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)N) ncols <<= 1;
  if (warp_id() == 0) {
    tmem_alloc(&tmem_base, ncols);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  const uint32_t idesc = idesc_dense(1, 1, 128, N);
  uint32_t phase = 0;
  if (sw64) {  // 64-byte swizzle variant: K slabs of 32 bf16
    for (int k0 = 0; k0 < K; k0 += 32) {
      for (int c = threadIdx.x; c < 128 * 4; c += blockDim.x) {
        const int r = c >> 2, ch = c & 3;
        *reinterpret_cast<uint4*>(sA + sw64_chunk(r, ch)) =
            *reinterpret_cast<const uint4*>(A + (size_t)(m0 + r) * K + k0 + ch * 8);
      }
      for (int c = threadIdx.x; c < N * 4; c += blockDim.x) {
        const int r = c >> 2, ch = c & 3;
        *reinterpret_cast<uint4*>(sB + sw64_chunk(r, ch)) =
            *reinterpret_cast<const uint4*>(B + (size_t)r * K + k0 + ch * 8);
      }
      fence_proxy_async_smem();
      __syncthreads();
      if (threadIdx.x == 0) {
        tc_fence_after();
        for (int kk = 0; kk < 2; ++kk)
          umma_f16_ss(tbase, desc_sw64(smem_u32(sA) + kk * 32), desc_sw64(smem_u32(sB) + kk * 32), idesc,
                      (k0 > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bar);
      }
      mbar_wait(&bar, phase, nullptr, nullptr, 0);
      phase ^= 1;
      tc_fence_after();
    }
  }
  for (int k0 = 0; k0 < K && !sw64; k0 += 64) {
    for (int c = threadIdx.x; c < 128 * 8; c += blockDim.x) {
      const int r = c >> 3, ch = c & 7;
      *reinterpret_cast<uint4*>(sA + sw128_chunk(r, ch)) =
          *reinterpret_cast<const uint4*>(A + (size_t)(m0 + r) * K + k0 + ch * 8);
    }
    for (int c = threadIdx.x; c < N * 8; c += blockDim.x) {
      const int r = c >> 3, ch = c & 7;
      *reinterpret_cast<uint4*>(sB + sw128_chunk(r, ch)) =
          *reinterpret_cast<const uint4*>(B + (size_t)r * K + k0 + ch * 8);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        umma_f16_ss(tbase, desc_sw128(smem_u32(sA) + kk * 32), desc_sw128(smem_u32(sB) + kk * 32), idesc,
                    (k0 > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&bar);
    }
    mbar_wait(&bar, phase, nullptr, nullptr, 0);
    phase ^= 1;
    tc_fence_after();
  }
  const int w = warp_id();
  for (int col = 0; col < N; col += 16) {
    uint32_t r[16];
    tmem_ld16(tbase + (static_cast<uint32_t>(32 * w) << 16) + col, r);
    tmem_ld_wait();
    float* dst = C + (size_t)(m0 + 32 * w + lane_id()) * N + col;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[j] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) tmem_dealloc(tbase, ncols);
}

}  // namespace

cudaError_t umma_gemm_test(const void* A, const void* B, float* C, int M, int N, int K, int sw64, cudaStream_t s) {
  if (M % 128 || N % 16 || N > 256 || K % 64) return cudaErrorInvalidValue;
  const int smem = 1024 + 128 * 128 + N * 128;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(umma_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  umma_gemm_kernel<<<M / 128, 128, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(A),
                                             reinterpret_cast<const __nv_bfloat16*>(B), C, N, K, sw64);
  return cudaGetLastError();
}

}  // namespace iob

// ---------------------------------------------------------------------------------------------------------------
// Issue-rate probe (diagnostic): one thread per issuing warp issues `count` UMMAs back to back.
// variant: 0 kind::f16 SS M128; 1 kind::f16 TS M128; 2 SS without a memory clobber; 3 kind::f8f6f4 SS M128 (K=32);
//          4 kind::f16 .ws SS M128 (N >= 64); 5 kind::f16 SS M64; 6 as 0 with two issuing warps (own accumulators).
// out[0] = cycles issuing, out[1] = cycles to completion of all.  Operands are zero-filled.
namespace iob {
namespace {
__device__ __forceinline__ void umma_f16_ss_nc(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_f16_ws_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.ws.cta_group::1.kind::f16 [%0], %1, %2, %3, p, 0;\n\t}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__global__ void __launch_bounds__(128) umma_rate_kernel(int n, int count, int nacc, int variant, long long* out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar[2];
  __shared__ uint32_t tmem_base;
  for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (warp_id() == 0) { tmem_alloc(&tmem_base, 512); tmem_relinquish(); }
  if (threadIdx.x == 0) { mbar_init(&bar[0], 1); mbar_init(&bar[1], 1); fence_mbar_init(); }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t t = tmem_base;
  const int issuers = variant == 6 ? 2 : 1;
  if (variant == 10 && warp_id() == 0) {
    // whole warp converged in the loop; one elected lane issues each MMA (E4M3, both operands K-major)
    const uint32_t idesc = idesc_dense(0, 0, 128, n);
    const uint64_t a = desc_sw128(smem_u32(smem)), b = desc_sw128(smem_u32(smem + 16384));
    const long long c0 = clock64();
    for (int i = 0; i < count; ++i) {
      const uint32_t d = t + (i % nacc) * n;
      if (elect_one()) umma_f8_ss(d, a, b, idesc, 1u);
      __syncwarp();
    }
    const long long c1 = clock64();
    if (elect_one()) umma_commit(&bar[0]);
    __syncwarp();
    mbar_wait(&bar[0], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    if (threadIdx.x == 0) {
      out[0] = c1 - c0;
      out[1] = c2 - c0;
    }
  } else if ((variant == 11 || variant == 12) && threadIdx.x == 0) {
    // E4M3 K-major, descriptors and predicate hoisted; 11: one MMA per asm statement without a memory clobber,
    // 12: four MMAs per asm statement
    const uint32_t idesc = idesc_dense(0, 0, 128, n);
    const uint64_t a = desc_sw128(smem_u32(smem)), b = desc_sw128(smem_u32(smem + 16384));
    const long long c0 = clock64();
    if (variant == 11) {
      for (int i = 0; i < count; ++i) {
        const uint32_t d = t + (i % nacc) * n;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
            "l"(a), "l"(b), "r"(idesc), "r"(1u));
      }
    } else {
      for (int i = 0; i < count; i += 4) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(t),
            "l"(a), "l"(b), "r"(idesc), "r"(1u));
      }
    }
    const long long c1 = clock64();
    umma_commit(&bar[0]);
    mbar_wait(&bar[0], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    out[0] = c1 - c0;
    out[1] = c2 - c0;
  } else if ((variant == 13 || variant == 14) && threadIdx.x == 0) {
    // batched helpers with distinct operands per MMA (K steps of a 128 B slab), 13: A in smem, 14: A in TMEM
    const uint32_t idesc = idesc_dense(0, 0, 128, n);
    const long long c0 = clock64();
    for (int i = 0; i < count; i += 4) {
      uint32_t d[4];
      uint64_t a[4], b[4];
      uint32_t at[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        d[k] = t + ((i / 4) % nacc) * n;
        a[k] = desc_sw128(smem_u32(smem) + 32 * k);
        b[k] = desc_sw128(smem_u32(smem + 16384) + 32 * k);
        at[k] = t + 256 + 8 * k;
      }
      if (variant == 13) umma_f8_ss_x4(d, a, b, idesc, 0xFu);
      else umma_f8_ts_x4(d, at, b, idesc, 0xFu);
    }
    const long long c1 = clock64();
    umma_commit(&bar[0]);
    mbar_wait(&bar[0], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    out[0] = c1 - c0;
    out[1] = c2 - c0;
  } else if (variant >= 17 && variant <= 19 && warp_id() == 0) {
    // K-step batches: descriptors advanced inside the statement (17: one lane issues; 18: converged warp + elect;
    // 19: converged warp + elect, A in TMEM)
    const uint32_t idesc = idesc_dense(0, 0, 128, n);
    const uint64_t a = desc_sw128(smem_u32(smem)), b = desc_sw128(smem_u32(smem + 16384));
    const long long c0 = clock64();
    for (int i = 0; i < count; i += 4) {
      const uint32_t d = t + ((i / 4) % nacc) * n;
      if (variant == 17) {
        if (lane_id() == 0) umma_f8_ss_k4<2, 2>(d, a, b, idesc, 1u);
      } else if (elect_one()) {
        if (variant == 18) umma_f8_ss_k4<2, 2>(d, a, b, idesc, 1u);
        else umma_f8_ts_k4<8, 2>(d, t + 256, b, idesc, 1u);
      }
      __syncwarp();
    }
    const long long c1 = clock64();
    if (elect_one()) umma_commit(&bar[0]);
    __syncwarp();
    mbar_wait(&bar[0], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    if (threadIdx.x == 0) {
      out[0] = c1 - c0;
      out[1] = c2 - c0;
    }
  } else if ((variant == 15 || variant == 16) && warp_id() == 0) {
    // whole warp converged, operands computed by every lane, one elected lane issues batched MMAs
    // (15: four per statement, distinct K-step descriptors; 16: the same with A in TMEM)
    const uint32_t idesc = idesc_dense(0, 0, 128, n);
    const uint32_t sa = smem_u32(smem), sb = smem_u32(smem + 16384);
    const long long c0 = clock64();
    for (int i = 0; i < count; i += 4) {
      uint32_t d[4], at[4];
      uint64_t a[4], b[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        d[k] = t + ((i / 4) % nacc) * n;
        a[k] = desc_sw128(sa + 32 * k);
        b[k] = desc_sw128(sb + 32 * k);
        at[k] = t + 256 + 8 * k;
      }
      if (elect_one()) {
        if (variant == 15) umma_f8_ss_x4(d, a, b, idesc, 0xFu);
        else umma_f8_ts_x4(d, at, b, idesc, 0xFu);
      }
      __syncwarp();
    }
    const long long c1 = clock64();
    if (elect_one()) umma_commit(&bar[0]);
    __syncwarp();
    mbar_wait(&bar[0], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    if (threadIdx.x == 0) {
      out[0] = c1 - c0;
      out[1] = c2 - c0;
    }
  } else if (variant != 10 && variant < 11 && lane_id() == 0 && warp_id() < issuers) {
    const int m = (variant == 5 || variant == 9) ? 64 : 128;
    const bool f8 = variant == 3 || variant >= 7;
    uint32_t idesc = f8 ? idesc_dense(0, 0, m, n) : idesc_dense(1, 1, m, n);
    if (variant == 8) idesc |= 1u << 15;                              // A MN-major
    const uint64_t a = desc_sw128(smem_u32(smem)), b = desc_sw128(smem_u32(smem + 16384));
    const uint32_t dbase = t + warp_id() * 128;
    const long long c0 = clock64();
    for (int i = 0; i < count; ++i) {
      const uint32_t d = dbase + (i % nacc) * n;
      switch (variant) {
        case 1: umma_f16_ts(d, t + 256, b, idesc, 1u); break;
        case 2: umma_f16_ss_nc(d, a, b, idesc, 1u); break;
        case 3: umma_f8_ss(d, a, b, idesc, 1u); break;
        case 4: umma_f16_ws_ss(d, a, b, idesc, 1u); break;
        case 7: umma_f8_ts(d, t + 256, b, idesc, 1u); break;                       // E4M3, A from TMEM
        case 8: umma_f8_ss(d, desc_mn128(smem_u32(smem), 16384), b, idesc, 1u); break;  // E4M3, A MN-major
        case 9: umma_f8_ss(d, a, b, idesc, 1u); break;                             // E4M3, M = 64
        default: umma_f16_ss(d, a, b, idesc, 1u); break;
      }
    }
    const long long c1 = clock64();
    umma_commit(&bar[warp_id()]);
    mbar_wait(&bar[warp_id()], 0, nullptr, nullptr, 0);
    const long long c2 = clock64();
    if (threadIdx.x == 0) {
      out[0] = c1 - c0;
      out[1] = c2 - c0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) { tc_fence_after(); tmem_dealloc(t, 512); }
}
}  // namespace

cudaError_t umma_rate_test(int n, int count, int nacc, int variant, long long* out, cudaStream_t s) {
  const int smem = 1024 + 16384 + 256 * 128;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(umma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  umma_rate_kernel<<<1, 128, smem, s>>>(n, count, nacc, variant, out);
  return cudaGetLastError();
}
}  // namespace iob

// ---------------------------------------------------------------------------------------------------------------
// kind::f8f6f4 with an MN-major B operand: C[128, N] fp32 = A[128, K] (E4M3, row-major) * B[K, N] (E4M3, row-major:
// N contiguous).  A is staged K-major SW128 in [128 x 128 B] slabs; B is staged as N-atoms of 128 columns, each a
// [K x 128 B] block with chunk c of K-row r at c ^ (r & 7) -- the same bytes a K-major SW128 tile of K rows holds,
// which is what lets an attention kernel reuse one dequantized K tile as the V operand.  N in {128, 256}, K <= 256.
namespace iob {
namespace {
__global__ void __launch_bounds__(128) umma_f8_mn_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                                                         float* __restrict__ C, int N, int K) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                   // (K / 128) slabs of 128 x 128 B
  uint8_t* sB = smem + 128 * K;         // (N / 128) atoms of K x 128 B
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  if (warp_id() == 0) { tmem_alloc(&tmem_base, 256); tmem_relinquish(); }
  if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_mbar_init(); }
  for (int c = threadIdx.x; c < 128 * (K / 16); c += blockDim.x) {
    const int r = c / (K / 16), ch = c % (K / 16);
    *reinterpret_cast<uint4*>(sA + (ch >> 3) * 16384 + sw128_chunk(r, ch & 7)) =
        *reinterpret_cast<const uint4*>(A + (size_t)r * K + ch * 16);
  }
  for (int c = threadIdx.x; c < K * (N / 16); c += blockDim.x) {
    const int r = c / (N / 16), ch = c % (N / 16);
    *reinterpret_cast<uint4*>(sB + (ch >> 3) * (K * 128) + sw128_chunk(r, ch & 7)) =
        *reinterpret_cast<const uint4*>(B + (size_t)r * N + ch * 16);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t t = tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_dense(0, 0, 128, N) | (1u << 16);  // B MN-major
    for (int kk = 0; kk < K / 32; ++kk) {
      const uint64_t a = desc_sw128(smem_u32(sA) + (kk >> 2) * 16384 + (kk & 3) * 32);
      const uint64_t b = desc_mn128(smem_u32(sB) + kk * 32 * 128, K * 128);
      umma_f8_ss(t, a, b, idesc, kk > 0 ? 1u : 0u);
    }
    umma_commit(&bar);
  }
  mbar_wait(&bar, 0, nullptr, nullptr, 0);
  tc_fence_after();
  const int w = warp_id();
  for (int col = 0; col < N; col += 16) {
    uint32_t r[16];
    tmem_ld16(t + (static_cast<uint32_t>(32 * w) << 16) + col, r);
    tmem_ld_wait();
    float* dst = C + (size_t)(32 * w + lane_id()) * N + col;
#pragma unroll
    for (int j = 0; j < 16; ++j) dst[j] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp_id() == 0) { tc_fence_after(); tmem_dealloc(t, 256); }
}
}  // namespace

cudaError_t umma_f8_mn_test(const void* A, const void* B, float* C, int N, int K, cudaStream_t s) {
  if ((N != 128 && N != 256) || K % 128 || K > 256) return cudaErrorInvalidValue;
  const int smem = 1024 + 128 * K + K * N;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(umma_f8_mn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  umma_f8_mn_kernel<<<1, 128, smem, s>>>(reinterpret_cast<const uint8_t*>(A), reinterpret_cast<const uint8_t*>(B),
                                         C, N, K);
  return cudaGetLastError();
}
}  // namespace iob

// ---------------------------------------------------------------------------------------------------------------
// NVFP4 -> E4M3 lookup-table decode (f4_scale_table + f4_decode8) against per-value conversion (f4_word_to_e4m3):
// every non-negative finite E4M3 scale (block scales are amax / 6 >= 0 by construction) x `nwords` code words.
// out[0] = mismatching words.
namespace iob {
namespace {
__global__ void nvfp4_lut_kernel(const uint32_t* __restrict__ words, int nwords, int* out) {
  const int scale = blockIdx.x;                              // 0..126
  if (scale >= 0x7F) return;
  const uint2 tab = f4_scale_table(static_cast<uint32_t>(scale));
  const uint32_t s2 = e4m3x2_to_f16x2(static_cast<uint16_t>(scale | (scale << 8)));
  int bad = 0;
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) {
    const uint2 a = f4_decode8(words[i], tab);
    const uint2 b = f4_word_to_e4m3(words[i], s2);
    bad += (a.x != b.x) || (a.y != b.y);
  }
  if (bad) atomicAdd(out, bad);
}
}  // namespace

cudaError_t nvfp4_lut_test(const uint32_t* words, int nwords, int* out, cudaStream_t s) {
  nvfp4_lut_kernel<<<127, 256, 0, s>>>(words, nwords, out);
  return cudaGetLastError();
}
}  // namespace iob

// ---------------------------------------------------------------------------------------------------------------
// Conversion / exp2 throughput probe: 4 warps (one per SM sub-partition), each thread runs `iters` rounds of 8
// independent chains of one instruction kind.  out[variant] = cycles per round (one warp instruction per chain).
namespace iob {
namespace {
template <int variant>
__global__ void __launch_bounds__(128) cvt_rate_kernel(int iters, long long* out, uint32_t* sink) {
  uint32_t x[8];
  float f[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[i] = 0x3C003C00u + threadIdx.x + i;
    f[i] = 0.5f + 0.01f * (threadIdx.x + i);
  }
  __syncthreads();
  const long long c0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      switch (variant) {   // compile-time
        case 0: asm volatile("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(x[i]) : "f"(f[i]), "f"(__uint_as_float(x[i]))); break;
        case 1: asm volatile("ex2.approx.f16x2 %0, %0;" : "+r"(x[i])); break;
        case 2: asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(f[i])); break;
        case 3: {
          uint16_t h;
          asm volatile("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(h) : "r"(x[i]));
          x[i] = x[i] ^ h;
          break;
        }
        case 4: {
          uint16_t h;
          asm volatile("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(h) : "f"(f[i]), "f"(f[(i + 1) & 7]));
          x[i] = x[i] ^ h;
          break;
        }
        case 5: asm volatile("add.rn.f16x2 %0, %0, %1;" : "+r"(x[i]) : "r"(x[(i + 3) & 7])); break;
        default: asm volatile("fma.rn.f32 %0, %0, %1, %1;" : "+f"(f[i]) : "f"(f[(i + 1) & 7])); break;
      }
    }
  }
  const long long c1 = clock64();
  uint32_t acc = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc ^= x[i] ^ __float_as_uint(f[i]);
  sink[threadIdx.x] = acc;
  if (threadIdx.x == 0) out[0] = (c1 - c0) / iters;
}
}  // namespace

cudaError_t cvt_rate_test(int iters, int variant, long long* out, uint32_t* sink, cudaStream_t s) {
  switch (variant) {
    case 0: cvt_rate_kernel<0><<<1, 128, 0, s>>>(iters, out, sink); break;
    case 1: cvt_rate_kernel<1><<<1, 128, 0, s>>>(iters, out, sink); break;
    case 2: cvt_rate_kernel<2><<<1, 128, 0, s>>>(iters, out, sink); break;
    case 3: cvt_rate_kernel<3><<<1, 128, 0, s>>>(iters, out, sink); break;
    case 4: cvt_rate_kernel<4><<<1, 128, 0, s>>>(iters, out, sink); break;
    case 5: cvt_rate_kernel<5><<<1, 128, 0, s>>>(iters, out, sink); break;
    default: cvt_rate_kernel<6><<<1, 128, 0, s>>>(iters, out, sink); break;
  }
  return cudaGetLastError();
}
}  // namespace iob
