// Fused per-layer glue of the MLA + DSA attention block: two launches replace the ~50 small elementwise kernels
// (norms, RoPE, concatenations, pool writes, indexer query quantization) that sit between the projection GEMMs.
//
// mla_prep_kv (after x -> [q_a | kv_a | k_pe | k_i | w_i], one CTA per token, 8 warps):
//   warps 0-3  q_a RMSNorm -> bf16 (the input of the q_a -> (q_nope | q_pe | q_i) projection)
//   warp 4     latent RMSNorm + NeoX RoPE of k_pe -> the token's latent pool row (NVFP4 352 B or E4M3 576 B)
//   warp 5     indexer key LayerNorm + RoPE of its first 64 dims -> the index pool (E4M3 + fp32 scale, page layout)
//   warp 6     indexer head weights w_i * Hi^-1/2 * 128^-1/2 -> fp32
// mla_prep_q (after q_a -> (q_nope | q_pe | q_i) and the head-batched q_nope W_UK product that wrote columns 0..511
//   of the attention query in place, one CTA per token):
//   RoPE of every head's q_pe -> columns 512..575 of the attention query; indexer query RoPE + per-(token, head)
//   E4M3 quantization with the scale folded into the head weight.
//
// Arithmetic follows the framework's torch reference path (models/mla.py) step by step: fp32 math, bf16 rounding at
// the same points (normed latent, roped k_pe / q_pe, roped and plain index key / query values), the pool writers' own
// quantization rules (kv_formats / elementwise.cu).
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

__device__ __forceinline__ float bfv(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16(v)); }

// NeoX rotate-half on a 64-wide vector held as 4 values per lane in lanes 0..15 (dims 4 l .. 4 l + 3): dim i < 32
// pairs with i + 32, held by lane l ^ 8.  Lanes 16..31 hold dims 64.. and pass through.
__device__ __forceinline__ void rope4(float (&v)[4], int lane, const float* cs) {
  float p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = __shfl_xor_sync(0xffffffffu, v[j], 8);
  if (lane < 16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * (lane & 7) + j;                 // index into the 32 (cos, sin) pairs
      const float c = cs[i], s = cs[32 + i];
      v[j] = lane < 8 ? v[j] * c - p[j] * s : v[j] * c + p[j] * s;
    }
  }
}

constexpr int kQaMax = 16;          // q_lora <= 16 x 128 (DeepSeek-V3 1536, GLM-5 2048)

__global__ void __launch_bounds__(256) mla_prep_kv_kernel(const MlaPrepArgs a) {
  const int t = blockIdx.x;
  const int warp = warp_id(), lane = lane_id();
  const __nv_bfloat16* y = static_cast<const __nv_bfloat16*>(a.ya) + static_cast<size_t>(t) * a.ya_stride;
  const int pos = a.pos[t];
  const float* cs = a.rope + static_cast<size_t>(pos) * 64;
  const int slot = a.slot[t];
  const int lat_slot = a.lat_slot ? a.lat_slot[t] : slot;
  __shared__ float red[4];
  if (warp < 4) {
    // ---------------------------------------------------------------- q_a RMSNorm (128 threads)
    // Thread tid holds element tid of every 128-wide block (kQaMax blocks at most), loaded up front: one round of
    // independent loads instead of a dependent load per block, and one barrier for every block's FP8 amax.
    const int tid = threadIdx.x;
    float v[kQaMax], wv[kQaMax];
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(a.q_norm);
#pragma unroll
    for (int j = 0; j < kQaMax; ++j) {
      const int c = tid + 128 * j;
      v[j] = c < a.q_lora ? bfv(y, c) : 0.f;
      wv[j] = c < a.q_lora ? bfv(w, c) : 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kQaMax; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    asm volatile("bar.sync 1, 128;");
    const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / a.q_lora + a.eps);
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.qa_out) + static_cast<size_t>(t) * a.q_lora;
    __shared__ float bmax[4][kQaMax];
#pragma unroll
    for (int j = 0; j < kQaMax; ++j) {
      const int c = tid + 128 * j;
      const __nv_bfloat16 b = __float2bfloat16(v[j] * inv * wv[j]);
      if (c < a.q_lora) o[c] = b;
      v[j] = __bfloat162float(b);
    }
    if (a.qa_q) {
#pragma unroll
      for (int j = 0; j < kQaMax; ++j) {
        const float m = warp_max(fabsf(v[j]));
        if (lane == 0) bmax[warp][j] = m;
      }
      asm volatile("bar.sync 1, 128;");
#pragma unroll
      for (int j = 0; j < kQaMax; ++j) {
        const int c = tid + 128 * j;
        if (c < a.q_lora) {
          const uint32_t eb = ue8m0_for(fmaxf(fmaxf(bmax[0][j], bmax[1][j]), fmaxf(bmax[2][j], bmax[3][j])));
          a.qa_q[static_cast<size_t>(t) * a.q_lora + c] = float_to_e4m3(v[j] * __uint_as_float((254u - eb) << 23));
          if (tid == 0) a.qa_s[static_cast<size_t>(t) * (a.q_lora / 128) + j] = eb * 0x01010101u;
        }
      }
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- latent row
    const __nv_bfloat16* kv = y + a.q_lora;
    float v[16];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = bfv(kv, 16 * lane + j);
      ss += v[j] * v[j];
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / 512.f + a.eps);
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(a.kv_norm);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = rbf(v[j] * inv * bfv(w, 16 * lane + j));
    const float x1 = bfv(kv, 512 + lane), x2 = bfv(kv, 512 + 32 + lane);
    const float c = cs[lane], s = cs[32 + lane];
    const float r1 = rbf(x1 * c - x2 * s), r2 = rbf(x2 * c + x1 * s);
    // mixed-format page space: slots from split_slot on live in the second pool, in its format
    const bool second = a.latent_pool2 != nullptr && lat_slot >= a.split_slot;
    const int fmt = second ? a.latent_fmt2 : a.latent_fmt;
    uint8_t* const pool = second ? a.latent_pool2 : a.latent_pool;
    const int lrow = second ? lat_slot - a.split_slot : lat_slot;
    if (lat_slot >= 0) {
      if (fmt == kKvNvfp4) {
        uint8_t* row = pool + static_cast<size_t>(lrow) * 352;
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const uint8_t s8 = nvfp4_block_scale(amax);
        const float sf = e4m3_to_float(s8);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) lo |= e2m1_code(v[j] / sf) << (4 * j);
#pragma unroll
        for (int j = 0; j < 8; ++j) hi |= e2m1_code(v[8 + j] / sf) << (4 * j);
        *reinterpret_cast<uint2*>(row + lane * 8) = make_uint2(lo, hi);
        row[256 + lane] = s8;
        row[288 + lane] = float_to_e4m3(r1);
        row[288 + 32 + lane] = float_to_e4m3(r2);
      } else {
        uint8_t* row = pool + static_cast<size_t>(lrow) * 576;
        uint32_t wq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          wq[q] = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) wq[q] |= static_cast<uint32_t>(float_to_e4m3(v[q * 4 + j])) << (8 * j);
        }
        *reinterpret_cast<uint4*>(row + lane * 16) = make_uint4(wq[0], wq[1], wq[2], wq[3]);
        row[512 + lane] = float_to_e4m3(r1);
        row[512 + 32 + lane] = float_to_e4m3(r2);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- indexer key
    const __nv_bfloat16* k = y + a.q_lora + 576;
    float v[4];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = bfv(k, 4 * lane + j);
      sum += v[j];
    }
    const float mean = warp_sum(sum) / 128.f;
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) var += (v[j] - mean) * (v[j] - mean);
    const float rstd = rsqrtf(warp_sum(var) / 128.f + a.eps);
    const __nv_bfloat16* lw = static_cast<const __nv_bfloat16*>(a.ik_w);
    const __nv_bfloat16* lb = static_cast<const __nv_bfloat16*>(a.ik_b);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = (v[j] - mean) * rstd * bfv(lw, 4 * lane + j) + bfv(lb, 4 * lane + j);
    rope4(v, lane, cs);
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = rbf(v[j]);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    amax = fmaxf(warp_max(amax), 1e-10f);
    if (slot >= 0) {
      const float sc = amax / 448.f;
      uint8_t* page = a.index_pool + static_cast<size_t>(slot >> 6) * (64 * 132);
      const int r = slot & 63;
      uint32_t wq = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) wq |= static_cast<uint32_t>(float_to_e4m3(v[j] / sc)) << (8 * j);
      const int byte = lane * 4;
      *reinterpret_cast<uint32_t*>(page + r * 128 + (((byte >> 4) ^ (r & 7)) << 4) + (byte & 15)) = wq;
      if (lane == 0) *reinterpret_cast<float*>(page + 64 * 128 + 4 * r) = sc;
    }
  } else if (warp == 6) {
    // ---------------------------------------------------------------- indexer head weights
    const __nv_bfloat16* w = y + a.q_lora + 576 + 128;
    for (int h = lane; h < a.Hi; h += 32) a.iw_out[static_cast<size_t>(t) * a.Hi + h] = bfv(w, h) * a.iw_scale;
  }
}

__global__ void __launch_bounds__(256) mla_prep_q_kernel(const MlaPrepArgs a) {
  const int t = blockIdx.x;
  const int warp = warp_id(), lane = lane_id();
  const __nv_bfloat16* y = static_cast<const __nv_bfloat16*>(a.yb) + static_cast<size_t>(t) * a.yb_stride;
  const float* cs = a.rope + static_cast<size_t>(a.pos[t]) * 64;
  const float c = cs[lane], s = cs[32 + lane];
  __nv_bfloat16* qf = static_cast<__nv_bfloat16*>(a.qf) + static_cast<size_t>(t) * a.H * 576;
  const __nv_bfloat16* qpe = y + a.H * a.dn;
  const int hw = blockIdx.y * 8 + warp, hstep = gridDim.y * 8;     // heads over the CTAs of this token
  for (int h = hw; h < a.H; h += hstep) {
    const float x1 = bfv(qpe, h * 64 + lane), x2 = bfv(qpe, h * 64 + 32 + lane);
    qf[h * 576 + 512 + lane] = __float2bfloat16(x1 * c - x2 * s);
    qf[h * 576 + 512 + 32 + lane] = __float2bfloat16(x2 * c + x1 * s);
  }
  const __nv_bfloat16* iq = y + a.H * (a.dn + 64);
  for (int h = hw; h < a.Hi; h += hstep) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = bfv(iq, h * 128 + 4 * lane + j);
    rope4(v, lane, cs);
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = rbf(v[j]);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    amax = warp_max(amax);
    const float sc = amax > 0.f ? amax / 448.f : 1.f;
    uint32_t wq = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) wq |= static_cast<uint32_t>(float_to_e4m3(v[j] / sc)) << (8 * j);
    const size_t row = static_cast<size_t>(t) * a.Hi + h;
    *reinterpret_cast<uint32_t*>(a.q8 + row * 128 + 4 * lane) = wq;
    if (lane == 0) a.w_eff[row] = a.iw_out[row] * sc;
  }
}

}  // namespace

cudaError_t mla_prep_kv(const MlaPrepArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.latent_pool2 && ((a.latent_fmt2 != kKvNvfp4 && a.latent_fmt2 != kKvFp8) || a.split_slot < 0))
    return cudaErrorInvalidValue;
  if (a.q_lora <= 0 || a.q_lora > 128 * kQaMax || a.Hi <= 0 || (a.latent_fmt != kKvNvfp4 && a.latent_fmt != kKvFp8) || !a.ya || !a.rope ||
      !a.pos || !a.slot || !a.qa_out || !a.latent_pool || !a.index_pool || !a.iw_out ||
      (a.qa_q && (!a.qa_s || a.q_lora % 128)))
    return cudaErrorInvalidValue;
  mla_prep_kv_kernel<<<a.T, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t mla_prep_q(const MlaPrepArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.H <= 0 || a.Hi <= 0 || a.dn <= 0 || !a.yb || !a.qf || !a.q8 || !a.w_eff || !a.iw_out ||
      (reinterpret_cast<uintptr_t>(a.q8) & 3))
    return cudaErrorInvalidValue;
  const int per_token = max(1, min(16, (max(a.H, a.Hi) + 15) / 16));   // ~2 heads per warp
  mla_prep_q_kernel<<<dim3(a.T, per_token), 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace iob
