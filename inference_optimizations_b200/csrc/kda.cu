// Kimi Delta Attention (KDA, gated delta-rule linear attention) decode step, fused into one launch per layer:
//   short causal conv (q, k, v; SiLU) -> decay gate -> L2-normalised q/k -> delta-rule state update -> output ->
//   sigmoid-gated RMSNorm.
// The reference fuses the same span (six upstream launches) into one Triton program
// (`linear-attention-kda/kda-fused-decode/kda.py:1-60`); the math contract it states is followed here:
//   * state h [Dv, Dk] value-major, fp32, updated in place
//   * conv: out = sum_j state[j] w[j] + x w[W-1] (oldest first), SiLU; the state shifts and appends the raw input
//   * g = -exp(A_log) * softplus(g_proj + dt_bias) (softplus linear above 20), decay exp(g) per key channel
//   * q, k divided by sqrt(sum x^2 + 1e-6); q scaled by Dk^-1/2
//   * h *= exp(g); u = beta (v - h k); h += u k^T; o = h q
//   * o *= sigmoid(g2); o = o / sqrt(mean(o^2) + 1e-5) * norm_w
// q/k heads equal value heads here (each CTA owns its q/k conv state: no cross-CTA read/shift race).
// One CTA per (batch row, value head), 256 threads: threads 0..Dk-1 run the q/k conv, threads Dk.. the v conv;
// warp w then owns value rows w, w + 8, ... of the state, each lane 4 key channels (float4 row access).
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kKdaThreads = 256;

__device__ __forceinline__ float bfr(const __nv_bfloat16* p, int i) { return __bfloat162float(p[i]); }

__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kKdaThreads / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

template <int DK, int DV, int W>
__global__ void __launch_bounds__(kKdaThreads) kda_decode_kernel(const KdaDecodeArgs a) {
  static_assert(DK == 128 && DV == 128, "head dims 128");
  const int b = blockIdx.x, hv = blockIdx.y;
  const int h = hv / (a.HV / a.H);
  const int tid = threadIdx.x;
  __shared__ float sq[DK], sk[DK], sg[DK], sv[DV], so[DV];
  __shared__ float red[kKdaThreads / 32];
  // ---- 1. short causal conv, state shift
  const bool is_qk = tid < DK;
  const int c = is_qk ? tid : tid - DK;                   // channel within the head
  {
    float xq = 0.f, xk = 0.f, xv = 0.f, aq = 0.f, ak = 0.f, av = 0.f;
    if (is_qk) {
      const size_t ch = static_cast<size_t>(h) * DK + c;
      float* csq = a.conv_q + (static_cast<size_t>(b) * a.H * DK + ch) * (W - 1);
      float* csk = a.conv_k + (static_cast<size_t>(b) * a.H * DK + ch) * (W - 1);
      xq = bfr(a.q, (b * a.H + h) * DK + c);
      xk = bfr(a.k, (b * a.H + h) * DK + c);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) {
        aq += csq[j] * a.conv_wq[ch * W + j];
        ak += csk[j] * a.conv_wk[ch * W + j];
      }
      aq += xq * a.conv_wq[ch * W + W - 1];
      ak += xk * a.conv_wk[ch * W + W - 1];
#pragma unroll
      for (int j = 0; j < W - 2; ++j) {
        csq[j] = csq[j + 1];
        csk[j] = csk[j + 1];
      }
      csq[W - 2] = xq;
      csk[W - 2] = xk;
      sq[c] = aq / (1.f + __expf(-aq));
      sk[c] = ak / (1.f + __expf(-ak));
      // gate for key channel c
      float gp = bfr(a.g_proj, (b * a.HV + hv) * DK + c) + a.dt_bias[hv * DK + c];
      const float sp = gp > 20.f ? gp : log1pf(__expf(gp));
      sg[c] = __expf(-__expf(a.A_log[hv]) * sp);       // decay factor exp(g)
    } else if (c < DV) {
      const size_t ch = static_cast<size_t>(hv) * DV + c;
      float* csv = a.conv_v + (static_cast<size_t>(b) * a.HV * DV + ch) * (W - 1);
      xv = bfr(a.v, (b * a.HV + hv) * DV + c);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) av += csv[j] * a.conv_wv[ch * W + j];
      av += xv * a.conv_wv[ch * W + W - 1];
#pragma unroll
      for (int j = 0; j < W - 2; ++j) csv[j] = csv[j + 1];
      csv[W - 2] = xv;
      sv[c] = av / (1.f + __expf(-av));
    }
  }
  __syncthreads();
  // ---- 2. L2-normalise q and k (eps inside the root), scale q
  const float qq = block_sum256(tid < DK ? sq[tid] * sq[tid] : 0.f, red);
  const float kk = block_sum256(tid < DK ? sk[tid] * sk[tid] : 0.f, red);
  const float rq = rsqrtf(qq + 1e-6f) * a.scale, rk = rsqrtf(kk + 1e-6f);
  __syncthreads();
  // ---- 3. delta-rule update: warp w owns value rows w, w + 8, ...; lane owns key channels 4 l .. 4 l + 3
  const int warp = warp_id(), lane = lane_id();
  float4 qv = *reinterpret_cast<const float4*>(&sq[4 * lane]);
  float4 kv = *reinterpret_cast<const float4*>(&sk[4 * lane]);
  const float4 gv = *reinterpret_cast<const float4*>(&sg[4 * lane]);
  qv.x *= rq; qv.y *= rq; qv.z *= rq; qv.w *= rq;
  kv.x *= rk; kv.y *= rk; kv.z *= rk; kv.w *= rk;
  float* hbase = a.state + (static_cast<size_t>(b) * a.HV + hv) * DV * DK;
  for (int r = warp; r < DV; r += kKdaThreads / 32) {
    float4* hp = reinterpret_cast<float4*>(hbase + static_cast<size_t>(r) * DK) + lane;
    float4 hr = *hp;
    hr.x *= gv.x; hr.y *= gv.y; hr.z *= gv.z; hr.w *= gv.w;
    const float hk = warp_sum(hr.x * kv.x + hr.y * kv.y + hr.z * kv.z + hr.w * kv.w);
    const float beta = a.beta_headwise ? a.beta[(b * a.HV + hv) * DV + r] : a.beta[b * a.HV + hv];
    const float u = (sv[r] - hk) * beta;
    hr.x += u * kv.x; hr.y += u * kv.y; hr.z += u * kv.z; hr.w += u * kv.w;
    const float o = warp_sum(hr.x * qv.x + hr.y * qv.y + hr.z * qv.z + hr.w * qv.w);
    *hp = hr;
    if (lane == 0) so[r] = o;
  }
  __syncthreads();
  // ---- 4. sigmoid-gated RMSNorm over the value head
  float o = 0.f;
  if (tid < DV) {
    const float g2 = bfr(a.g2, (b * a.HV + hv) * DV + tid);
    o = so[tid] / (1.f + __expf(-g2));
  }
  const float ss = block_sum256(tid < DV ? o * o : 0.f, red);
  if (tid < DV) {
    const float y = o * rsqrtf(ss / DV + 1e-5f) * a.norm_w[tid];
    a.out[(static_cast<size_t>(b) * a.HV + hv) * DV + tid] = __float2bfloat16(y);
  }
}

}  // namespace

cudaError_t kda_decode(const KdaDecodeArgs& a, cudaStream_t s) {
  if (a.B == 0) return cudaSuccess;
  if (a.DK != 128 || a.DV != 128 || a.H <= 0 || a.HV != a.H || (a.W != 4 && a.W != 3 && a.W != 2))
    return cudaErrorInvalidValue;
  const dim3 grid(a.B, a.HV);
  switch (a.W) {
    case 2: kda_decode_kernel<128, 128, 2><<<grid, kKdaThreads, 0, s>>>(a); break;
    case 3: kda_decode_kernel<128, 128, 3><<<grid, kKdaThreads, 0, s>>>(a); break;
    default: kda_decode_kernel<128, 128, 4><<<grid, kKdaThreads, 0, s>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace iob
