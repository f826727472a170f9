// Memory-bound glue kernels: RMSNorm (+residual), activations, embedding, row argmax, the fused GQA QKV epilogue
// (qk-norm + RoPE + KV quant-write, the reference's K36/K37 fusion: `attention/gemma-fused-glue/rtx_kv_store.py`,
// `rtx_qkv_norm_rope.py`) and the MLA / indexer row writers (K25: `kv-cache-4bit/glm-kv4/glm_kv4.py:170-203`).
// All vectorised with 16-byte accesses; one CTA (or warp) per row so any row count is one launch.
#include "common.cuh"
#include "kernels.h"

namespace iob {

namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

template <int VPT>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                               __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ w, int hidden,
                               int x_stride, float eps, bool plus_one, bool add_residual, uint8_t* __restrict__ q8,
                               uint32_t* __restrict__ qs) {
  griddep_launch();                   // a GEMM launched after this may set up and stream weights meanwhile
  const int row = blockIdx.x;
  const int nvec = hidden / 8;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      uint4 raw = reinterpret_cast<const uint4*>(x + (size_t)row * x_stride)[c];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      uint4 rr;
      if (add_residual) rr = reinterpret_cast<const uint4*>(residual + (size_t)row * hidden)[c];
      const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float f = bf(e[j]);
        if (add_residual) f = bf(__float2bfloat16(f + bf(re[j])));  // residual stream is stored in bf16
        v[i][j] = f;
        ss += f * f;
      }
      if (add_residual) {
        uint4 o;
        __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) oe[j] = __float2bfloat16(v[i][j]);
        reinterpret_cast<uint4*>(residual + (size_t)row * hidden)[c] = o;
      }
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if (lane_id() == 0) red[warp_id()] = ss;
  __syncthreads();
  if (warp_id() == 0) {
    float t = lane_id() < (int)(blockDim.x / 32) ? red[lane_id()] : 0.f;
    t = warp_sum(t);
    if (lane_id() == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / hidden + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    float y[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c < nvec) {
      uint4 wr = reinterpret_cast<const uint4*>(w)[c];
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wr);
      uint4 o;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = plus_one ? 1.f + bf(we[j]) : bf(we[j]);
        oe[j] = __float2bfloat16(v[i][j] * inv * g);
        y[j] = bf(oe[j]);
      }
      reinterpret_cast<uint4*>(out + (size_t)row * hidden)[c] = o;
    }
    if (q8) {
      // FP8 copy for a block-scaled GEMM (E4M3 + one UE8M0 scale per 128 values = 16 consecutive threads' groups):
      // the same bytes as quantizing the bf16 output afterwards, without the extra launch
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(y[j]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (c < nvec) {
        const uint32_t eb = ue8m0_for(m);
        const float sc = __uint_as_float((254u - eb) << 23);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) lo |= static_cast<uint32_t>(float_to_e4m3(y[j] * sc)) << (8 * j);
#pragma unroll
        for (int j = 0; j < 4; ++j) hi |= static_cast<uint32_t>(float_to_e4m3(y[4 + j] * sc)) << (8 * j);
        *reinterpret_cast<uint2*>(q8 + (size_t)row * hidden + 8 * c) = make_uint2(lo, hi);
        if ((c & 15) == 0) qs[(size_t)row * (hidden / 128) + c / 16] = eb * 0x01010101u;
      }
    }
  }
}

__device__ __forceinline__ float gelu_tanh(float g) { return gelu_tanh_f(g); }

template <bool GELU>
__global__ void act_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int ffn) {
  const int row = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= ffn / 8) return;
  uint4 g = reinterpret_cast<const uint4*>(gu + (size_t)row * 2 * ffn)[c];
  uint4 u = reinterpret_cast<const uint4*>(gu + (size_t)row * 2 * ffn + ffn)[c];
  const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&g);
  const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&u);
  uint4 o;
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float gv = bf(ge[j]);
    const float a = GELU ? gelu_tanh(gv) : gv / (1.f + __expf(-gv));
    oe[j] = __float2bfloat16(a * bf(ue[j]));
  }
  reinterpret_cast<uint4*>(out + (size_t)row * ffn)[c] = o;
}

__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int hidden, float scale) {
  const int row = blockIdx.x;
  const int id = ids[row];
  for (int c = threadIdx.x; c < hidden / 8; c += blockDim.x) {
    uint4 v = reinterpret_cast<const uint4*>(table + (size_t)id * hidden)[c];
    if (scale != 1.f) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = __float2bfloat16(bf(e[j]) * scale);
    }
    reinterpret_cast<uint4*>(out + (size_t)row * hidden)[c] = v;
  }
}

// Row argmax, smallest index on ties (the greedy-sampling rule of `attention/gemma-fused-glue/rtx_draft_top1.py`).
template <bool F32>
__global__ void argmax_kernel(const void* __restrict__ logits, int* __restrict__ out_idx,
                              float* __restrict__ out_val, int vocab, int stride) {
  const int row = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if (F32) {
    const float* p = reinterpret_cast<const float*>(logits) + (size_t)row * stride;
    for (int c = threadIdx.x; c < vocab / 4; c += blockDim.x) {
      float4 v = reinterpret_cast<const float4*>(p)[c];
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (e[j] > best) { best = e[j]; bi = c * 4 + j; }
    }
  } else {
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(logits) + (size_t)row * stride;
    for (int c = threadIdx.x; c < vocab / 8; c += blockDim.x) {
      uint4 v = reinterpret_cast<const uint4*>(p)[c];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float f = bf(e[j]);
        if (f > best) { best = f; bi = c * 8 + j; }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  if (lane_id() == 0) { sb[warp_id()] = best; si[warp_id()] = bi; }
  __syncthreads();
  if (warp_id() == 0) {
    const int nw = blockDim.x / 32;
    best = lane_id() < nw ? sb[lane_id()] : -INFINITY;
    bi = lane_id() < nw ? si[lane_id()] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane_id() == 0) {
      out_idx[row] = bi;
      if (out_val) out_val[row] = best;
    }
  }
}

// ------------------------------------------------------------------------------------------ GQA QKV epilogue
// One warp per (token, head) vector.  Lane l owns E/2 consecutive elements of each half of the head vector
// (E = D / 32), so both members of every NeoX RoPE pair (i, i + D/2) live in the same thread.
template <int D>
__global__ void gqa_prep_kernel(GqaPrepArgs a) {
  constexpr int E = D / 32;
  constexpr int H2 = E / 2;          // elements per lane per half
  constexpr int LPB = 16 / H2;       // lanes per 16-element FP4 block
  const int t = blockIdx.x;
  const int head = blockIdx.y * (blockDim.x / 32) + warp_id();
  const int nheads = a.Hq + 2 * a.Hk;
  if (head >= nheads) return;
  const int lane = lane_id();
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + (size_t)t * a.qkv_stride + head * D;
  float x[E];
#pragma unroll
  for (int j = 0; j < H2; ++j) {
    x[j] = bf(src[lane * H2 + j]);
    x[H2 + j] = bf(src[D / 2 + lane * H2 + j]);
  }
  const bool is_q = head < a.Hq;
  const bool is_k = !is_q && head < a.Hq + a.Hk;
  if (is_q || is_k) {
    const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(is_q ? a.q_norm : a.k_norm);
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss += x[j] * x[j];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + a.eps);
#pragma unroll
      for (int j = 0; j < H2; ++j) {
        const float w0 = bf(nw[lane * H2 + j]), w1 = bf(nw[D / 2 + lane * H2 + j]);
        // round through bf16 like the unfused sequence (norm output is a bf16 tensor there)
        x[j] = bf(__float2bfloat16(x[j] * inv * (a.plus_one ? 1.f + w0 : w0)));
        x[H2 + j] = bf(__float2bfloat16(x[H2 + j] * inv * (a.plus_one ? 1.f + w1 : w1)));
      }
    }
    const float* cs = a.cos_sin + (size_t)a.pos[t] * D;
#pragma unroll
    for (int j = 0; j < H2; ++j) {
      const int i = lane * H2 + j;
      const float c = cs[i], s = cs[D / 2 + i];
      const float x1 = x[j], x2 = x[H2 + j];
      x[j] = x1 * c - x2 * s;
      x[H2 + j] = x2 * c + x1 * s;
    }
  }
  if (is_q) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.q_out) + ((size_t)t * a.Hq + head) * D;
#pragma unroll
    for (int j = 0; j < H2; ++j) {
      dst[lane * H2 + j] = __float2bfloat16(x[j]);
      dst[D / 2 + lane * H2 + j] = __float2bfloat16(x[H2 + j]);
    }
    return;
  }
  const int slot = a.slot[t];
  if (slot < 0) return;
  const int kvh = is_k ? head - a.Hq : head - a.Hq - a.Hk;
  const int page = slot / a.page, off = slot % a.page;
  const int blk = gqa_block_bytes(a.fmt, D, a.page);
  uint8_t* base = a.pool + ((size_t)page * a.Hk + kvh) * blk;
  // K/V values are rounded to bf16 first (the unfused path stores bf16 k/v before quantizing)
#pragma unroll
  for (int j = 0; j < E; ++j) x[j] = bf(__float2bfloat16(x[j]));
  if (a.fmt == kKvBf16) {
    uint8_t* d = base + (is_k ? 0 : a.page * D * 2) + off * D * 2;
#pragma unroll
    for (int j = 0; j < H2; ++j) {
      const int e0 = lane * H2 + j, e1 = D / 2 + lane * H2 + j;
      *reinterpret_cast<__nv_bfloat16*>(d + kv_swizzle_byte(e0 * 2, off, D * 2)) = __float2bfloat16(x[j]);
      *reinterpret_cast<__nv_bfloat16*>(d + kv_swizzle_byte(e1 * 2, off, D * 2)) = __float2bfloat16(x[H2 + j]);
    }
  } else if (a.fmt == kKvFp8) {
    const float sc = is_k ? a.k_scale : a.v_scale;
    uint8_t* d = base + (is_k ? 0 : a.page * D) + off * D;
#pragma unroll
    for (int j = 0; j < H2; ++j) {
      const int e0 = lane * H2 + j, e1 = D / 2 + lane * H2 + j;
      d[kv_swizzle_byte(e0, off, D)] = float_to_e4m3(x[j] / sc);
      d[kv_swizzle_byte(e1, off, D)] = float_to_e4m3(x[H2 + j] / sc);
    }
  } else {
    const float g = is_k ? a.k_scale : a.v_scale;
    const int half_bytes = a.page * (D / 2 + D / 16);
    uint8_t* codes = base + (is_k ? 0 : half_bytes) + off * (D / 2);  // row start; bytes swizzled below
    uint8_t* scales = base + (is_k ? 0 : half_bytes) + a.page * (D / 2) + off * (D / 16);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < H2; ++j) amax = fmaxf(amax, fabsf(x[hh * H2 + j] / g));
#pragma unroll
      for (int o = 1; o < LPB; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint8_t s8 = nvfp4_block_scale(amax);
      const float sf = e4m3_to_float(s8);
      const int e0 = hh * (D / 2) + lane * H2;  // first element index of this lane's run
      if ((lane % LPB) == 0) scales[e0 / 16] = s8;
#pragma unroll
      for (int j = 0; j < H2; j += 2) {
        const uint32_t c0 = e2m1_code((x[hh * H2 + j] / g) / sf);
        const uint32_t c1 = e2m1_code((x[hh * H2 + j + 1] / g) / sf);
        codes[kv_swizzle_byte((e0 + j) / 2, off, D / 2)] = static_cast<uint8_t>(c0 | (c1 << 4));
      }
    }
  }
}

// ------------------------------------------------------------------------------------------ MLA rows
// One warp per token.  NVFP4: lane l quantizes latent block l (16 values -> 8 code bytes + 1 scale), and rope values
// 2l, 2l+1.  FP8: lane l writes 16 latent bytes + 2 rope bytes.
__global__ void mla_write_kernel(const __nv_bfloat16* __restrict__ nope, int nope_stride,
                                 const __nv_bfloat16* __restrict__ rope, int rope_stride, const int* __restrict__ slot,
                                 uint8_t* __restrict__ pool, int T, int fmt) {
  const int t = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (t >= T) return;
  const int s = slot[t];
  if (s < 0) return;
  const int lane = lane_id();
  float v[16];
  const uint4* src = reinterpret_cast<const uint4*>(nope + (size_t)t * nope_stride + lane * 16);
  uint4 r0 = src[0], r1 = src[1];
  const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&r0);
  const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&r1);
#pragma unroll
  for (int j = 0; j < 8; ++j) { v[j] = bf(e0[j]); v[8 + j] = bf(e1[j]); }
  const float r_0 = bf(rope[(size_t)t * rope_stride + 2 * lane]);
  const float r_1 = bf(rope[(size_t)t * rope_stride + 2 * lane + 1]);
  if (fmt == kKvNvfp4) {
    uint8_t* row = pool + (size_t)s * 352;
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
    row[288 + 2 * lane] = float_to_e4m3(r_0);
    row[288 + 2 * lane + 1] = float_to_e4m3(r_1);
  } else {
    uint8_t* row = pool + (size_t)s * 576;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      w[q] = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) w[q] |= static_cast<uint32_t>(float_to_e4m3(v[q * 4 + j])) << (8 * j);
    }
    *reinterpret_cast<uint4*>(row + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    row[512 + 2 * lane] = float_to_e4m3(r_0);
    row[512 + 2 * lane + 1] = float_to_e4m3(r_1);
  }
}

__global__ void index_key_kernel(const __nv_bfloat16* __restrict__ k, int k_stride, const int* __restrict__ slot,
                                 uint8_t* __restrict__ pool, int T) {
  const int t = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (t >= T) return;
  const int s = slot[t];
  if (s < 0) return;
  const int lane = lane_id();
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = bf(k[(size_t)t * k_stride + lane * 4 + j]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = fmaxf(warp_max(amax), 1e-10f);
  const float sc = amax / 448.f;
  // page-blocked layout: [64 x 128 B values, 16-byte chunk c of row r at c ^ (r & 7)][64 x fp32 scales]
  uint8_t* page = pool + (size_t)(s >> 6) * (64 * 132);
  const int r = s & 63;
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) w |= static_cast<uint32_t>(float_to_e4m3(v[j] / sc)) << (8 * j);
  const int byte = lane * 4;
  *reinterpret_cast<uint32_t*>(page + r * 128 + (((byte >> 4) ^ (r & 7)) << 4) + (byte & 15)) = w;
  if (lane == 0) *reinterpret_cast<float*>(page + 64 * 128 + 4 * r) = sc;
}

}  // namespace

cudaError_t rmsnorm(const void* x, void* residual, void* out, const void* weight, int rows, int hidden, int x_stride,
                    float eps, bool plus_one, bool add_residual, cudaStream_t s, uint8_t* q8, uint32_t* qs) {
  if (hidden % 8 != 0 || rows == 0) return rows == 0 ? cudaSuccess : cudaErrorInvalidValue;
  if (q8 && (hidden % 128 || !qs)) return cudaErrorInvalidValue;
  const int nvec = hidden / 8;
  const int threads = nvec >= 1024 ? 1024 : ((nvec + 31) / 32) * 32;
  const int vpt = (nvec + threads - 1) / threads;
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto R = reinterpret_cast<__nv_bfloat16*>(residual);
  auto O = reinterpret_cast<__nv_bfloat16*>(out);
  auto W = reinterpret_cast<const __nv_bfloat16*>(weight);
  if (vpt == 1)
    rmsnorm_kernel<1><<<rows, threads, 0, s>>>(X, R, O, W, hidden, x_stride, eps, plus_one, add_residual, q8, qs);
  else if (vpt == 2)
    rmsnorm_kernel<2><<<rows, threads, 0, s>>>(X, R, O, W, hidden, x_stride, eps, plus_one, add_residual, q8, qs);
  else if (vpt <= 4)
    rmsnorm_kernel<4><<<rows, threads, 0, s>>>(X, R, O, W, hidden, x_stride, eps, plus_one, add_residual, q8, qs);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t gelu_tanh_mul(const void* gate_up, void* out, int rows, int ffn, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  dim3 grid((ffn / 8 + 127) / 128, rows);
  act_mul_kernel<true><<<grid, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(gate_up),
                                            reinterpret_cast<__nv_bfloat16*>(out), ffn);
  return cudaGetLastError();
}

cudaError_t silu_mul(const void* gate_up, void* out, int rows, int ffn, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  dim3 grid((ffn / 8 + 127) / 128, rows);
  act_mul_kernel<false><<<grid, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(gate_up),
                                             reinterpret_cast<__nv_bfloat16*>(out), ffn);
  return cudaGetLastError();
}

cudaError_t embed(const int* ids, const void* table, void* out, int rows, int hidden, float scale, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  embed_kernel<<<rows, 256, 0, s>>>(ids, reinterpret_cast<const __nv_bfloat16*>(table),
                                    reinterpret_cast<__nv_bfloat16*>(out), hidden, scale);
  return cudaGetLastError();
}

cudaError_t argmax_rows(const void* logits, int* out_idx, float* out_val, int rows, int vocab, int stride,
                        bool logits_fp32, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (logits_fp32) argmax_kernel<true><<<rows, 1024, 0, s>>>(logits, out_idx, out_val, vocab, stride);
  else argmax_kernel<false><<<rows, 1024, 0, s>>>(logits, out_idx, out_val, vocab, stride);
  return cudaGetLastError();
}

cudaError_t gqa_prep(const GqaPrepArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  const int warps = 4;
  dim3 grid(a.T, (a.Hq + 2 * a.Hk + warps - 1) / warps);
  switch (a.D) {
    case 128: gqa_prep_kernel<128><<<grid, warps * 32, 0, s>>>(a); break;
    case 256: gqa_prep_kernel<256><<<grid, warps * 32, 0, s>>>(a); break;
    case 512: gqa_prep_kernel<512><<<grid, warps * 32, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t mla_quant_write(const void* nope, int nope_stride, const void* rope, int rope_stride, const int* slot,
                            uint8_t* pool, int T, int fmt, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  mla_write_kernel<<<(T + 3) / 4, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(nope), nope_stride,
                                               reinterpret_cast<const __nv_bfloat16*>(rope), rope_stride, slot, pool,
                                               T, fmt);
  return cudaGetLastError();
}

cudaError_t index_key_write(const void* k, int k_stride, const int* slot, uint8_t* pool, int T, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  index_key_kernel<<<(T + 3) / 4, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(k), k_stride, slot, pool, T);
  return cudaGetLastError();
}

}  // namespace iob
