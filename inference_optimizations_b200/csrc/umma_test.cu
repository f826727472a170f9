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
