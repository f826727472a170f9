// Writers for two more 4-bit latent-row formats (byte layouts in ops/formats.py):
//   * the 288-byte rope-free NVFP4 row (GLM-Flash DSA layers): 512 E2M1 values + 32 E4M3 scales, the MLA row's
//     encoding without the rope tail (`kv-cache-4bit/glmflash-kv4/glmflash_kv4.py:1-20`);
//   * the DeepSeek V4 Pro cell, 320 bytes (E4M3 rope) or 384 bytes (bf16 rope): 448 E2M1 values with 28 E4M3
//     scales chosen per block by a 4-way scale search on squared error, E2M1 ties to even, 4 zero bytes, rope
//     (`kv-cache-4bit/kv4pro-deepseek/kv4pro_fp4.py:1-30`).
// One warp per token; lane l owns 16-value block l.  Slot < 0 skips the token.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

__device__ __forceinline__ float bfv(__nv_bfloat16 v) { return __bfloat162float(v); }

__global__ void glmflash_write_kernel(const __nv_bfloat16* __restrict__ nope, int stride, const int* __restrict__ slot,
                                      uint8_t* __restrict__ pool, int T) {
  const int t = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (t >= T) return;
  const int s = slot[t];
  if (s < 0) return;
  const int lane = lane_id();
  float v[16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = bfv(nope[static_cast<size_t>(t) * stride + lane * 16 + j]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  const uint8_t s8 = nvfp4_block_scale(amax);
  const float sf = e4m3_to_float(s8);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) lo |= e2m1_code(v[j] / sf) << (4 * j);
#pragma unroll
  for (int j = 0; j < 8; ++j) hi |= e2m1_code(v[8 + j] / sf) << (4 * j);
  uint8_t* row = pool + static_cast<size_t>(s) * 288;
  *reinterpret_cast<uint2*>(row + lane * 8) = make_uint2(lo, hi);
  row[256 + lane] = s8;
}

// E2M1 magnitude code, round to nearest, ties to even, saturating at 6.
__device__ __forceinline__ uint32_t e2m1_mag_even(float a) {
  a = fminf(a, 6.f);
  return (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
}
__device__ __forceinline__ float e2m1_val(uint32_t mag) {
  return mag < 4 ? 0.5f * mag : (mag == 4 ? 2.f : (mag == 5 ? 3.f : (mag == 6 ? 4.f : 6.f)));
}

__global__ void v4pro_write_kernel(const __nv_bfloat16* __restrict__ x, int stride, const int* __restrict__ slot,
                                   uint8_t* __restrict__ pool, int T, int cell, int rope_bf16) {
  const int t = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (t >= T) return;
  const int s = slot[t];
  if (s < 0) return;
  const int lane = lane_id();
  uint8_t* c = pool + static_cast<size_t>(s) * cell;
  const __nv_bfloat16* xr = x + static_cast<size_t>(t) * stride;
  if (lane < 28) {
    float v[16];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = bfv(xr[lane * 16 + j]);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    const float f[4] = {1.0f, 0.93f, 0.86f, 0.8f};
    uint32_t best_lo = 0, best_hi = 0;
    uint8_t best_s8 = 0;
    float best_err = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint8_t s8 = float_to_e4m3(fminf((amax / 6.0f) * f[k], 448.f));
      const float sf = e4m3_to_float(s8);
      const float inv = sf > 0.f ? 1.0f / sf : 0.f;
      uint32_t lo = 0, hi = 0;
      float err = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float q = v[j] * inv;
        const uint32_t mag = e2m1_mag_even(fabsf(q));
        const uint32_t code = mag | ((q < 0.f && mag > 0) ? 8u : 0u);
        const float d = (q < 0.f ? -e2m1_val(mag) : e2m1_val(mag)) * sf - v[j];
        err += d * d;
        if (j < 8) lo |= code << (4 * j); else hi |= code << (4 * (j - 8));
      }
      if (k == 0 || err < best_err) {
        best_err = err;
        best_lo = lo;
        best_hi = hi;
        best_s8 = s8;
      }
    }
    *reinterpret_cast<uint2*>(c + lane * 8) = make_uint2(best_lo, best_hi);
    c[224 + lane] = best_s8;
  } else {
    c[224 + lane] = 0;                                  // bytes 252..255: zero pad
  }
  // rope: 64 values, two per lane
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * lane + j;
    const __nv_bfloat16 r = xr[448 + i];
    if (rope_bf16) reinterpret_cast<__nv_bfloat16*>(c + 256)[i] = r;
    else c[256 + i] = float_to_e4m3(fminf(fmaxf(bfv(r), -448.f), 448.f));
  }
}

}  // namespace

cudaError_t glmflash_write(const void* nope, int stride, const int* slot, uint8_t* pool, int T, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  glmflash_write_kernel<<<(T + 3) / 4, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(nope), stride, slot, pool, T);
  return cudaGetLastError();
}

cudaError_t v4pro_write(const void* x, int stride, const int* slot, uint8_t* pool, int T, int rope_bf16,
                        cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  v4pro_write_kernel<<<(T + 3) / 4, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(x), stride, slot, pool, T,
                                                 rope_bf16 ? 384 : 320, rope_bf16);
  return cudaGetLastError();
}

}  // namespace iob
