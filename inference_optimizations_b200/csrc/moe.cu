// MoE router: sigmoid scores, bias-corrected group-limited top-k, renormalised weights (ops/moe.py route_ref is the
// oracle; semantics of the DeepSeek `noaux_tc` router).  One warp per token; the E <= 256 biased scores are staged
// in shared memory, groups and experts are picked by repeated warp arg-max (ties: lower index).
//
// Register form (E a multiple of 32, groups of a multiple of 32 experts: DeepSeek-V3 256 / 8, GLM-5 160 / 1): lane l
// holds experts l + 32 j in registers, so a group is a set of whole registers; group scores come from one top-2
// butterfly per group, the K picks from register arg-max + one warp arg-max each -- no shared-memory passes.  It
// also reads the router GEMM's split-K fp32 partials directly (summed in split order, as the reduction kernel
// would), so the reduction launch disappears.  Same picks and weights as the shared-memory form, bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kRouteWarps = 4;

// (value, index) arg-max across the warp, ties to the lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
}

__global__ void __launch_bounds__(32 * kRouteWarps) moe_route_kernel(const float* __restrict__ logits,
                                                                     const float* __restrict__ bias, int* ids,
                                                                     float* wts, int T, int E, int K, int G, int KG,
                                                                     float scale) {
  __shared__ float sel[kRouteWarps][256];
  __shared__ float prob[kRouteWarps][256];
  const int w = warp_id(), lane = lane_id();
  const int t = blockIdx.x * kRouteWarps + w;
  if (t >= T) return;
  const float* lg = logits + static_cast<size_t>(t) * E;
  for (int e = lane; e < E; e += 32) {
    const float p = 1.f / (1.f + __expf(-lg[e]));
    prob[w][e] = p;
    sel[w][e] = p + bias[e];
  }
  __syncwarp();
  if (G > 1) {
    // group score = sum of the group's two best biased scores; keep the KG best groups
    const int gs = E / G;
    float gscore = -INFINITY;
    if (lane < G) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = lane * gs; e < (lane + 1) * gs; ++e) {
        const float v = sel[w][e];
        if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
      }
      gscore = b1 + b2;
    }
    unsigned keep = 0;
    for (int r = 0; r < KG; ++r) {
      float v = (lane < G && !((keep >> lane) & 1u)) ? gscore : -INFINITY;
      int i = lane;
      warp_argmax(v, i);
      keep |= 1u << i;
    }
    __syncwarp();
    for (int e = lane; e < E; e += 32)
      if (!((keep >> (e / gs)) & 1u)) sel[w][e] = -INFINITY;
    __syncwarp();
  }
  float sum = 0.f;
  int myid = -1;
  float myw = 0.f;
  for (int r = 0; r < K; ++r) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float x = sel[w][e];
      if (x > v || (x == v && e < i)) { v = x; i = e; }
    }
    warp_argmax(v, i);
    if (i >= E) i = 0;                        // fewer eligible experts than K (never with valid configs)
    if (lane == 0) sel[w][i] = -INFINITY;     // taken
    __syncwarp();
    const float p = prob[w][i];
    sum += p;
    if (lane == r) { myid = i; myw = p; }
  }
  if (lane < K) {
    ids[static_cast<size_t>(t) * K + lane] = myid;
    wts[static_cast<size_t>(t) * K + lane] = myw / fmaxf(sum, 1e-20f) * scale;
  }
}

// (b1, b2) = the two largest of a warp's (b1, b2) pairs (duplicates counted), on every lane.
__device__ __forceinline__ void warp_top2(float& b1, float& b2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, b1, o), o2 = __shfl_xor_sync(0xffffffffu, b2, o);
    const float hi = fmaxf(b1, o1), lo = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
    b1 = hi;
    b2 = lo;
  }
}

// One CTA (8 warps) per token: the warps stage the token's ksplit x E partials in shared memory with coalesced
// loads (one round of independent loads however many splits), then warp 0 sums them in split order and routes.
constexpr int kRegThreads = 256;

template <int NJ>
__global__ void __launch_bounds__(kRegThreads) moe_route_reg_kernel(const float* __restrict__ part, int ksplit,
                                                                    const float* __restrict__ bias, int* ids,
                                                                    float* wts, int T, int K, int G, int KG,
                                                                    float scale) {
  constexpr int E = 32 * NJ;
  extern __shared__ float stage[];                          // [ksplit][E]
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < ksplit * E; i += kRegThreads) {
    const int k = i / E, e = i - k * E;
    stage[i] = part[(static_cast<size_t>(k) * T + t) * E + e];
  }
  __syncthreads();
  if (warp_id() != 0) return;
  const int lane = lane_id();
  float acc[NJ], p[NJ], v[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) acc[j] = 0.f;
  for (int k = 0; k < ksplit; ++k)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j] += stage[k * E + lane + 32 * j];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    p[j] = 1.f / (1.f + __expf(-acc[j]));
    v[j] = p[j] + bias[lane + 32 * j];
  }
  if (G > 1) {
    const int jpg = NJ / G;                  // registers per group
    float gscore[NJ];
#pragma unroll
    for (int g = 0; g < NJ; ++g) {
      gscore[g] = -INFINITY;
      if (g < G) {
        float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          if (j / jpg == g) {
            const float x = v[j];
            if (x > b1) { b2 = b1; b1 = x; } else if (x > b2) { b2 = x; }
          }
        }
        warp_top2(b1, b2);
        gscore[g] = b1 + b2;
      }
    }
    unsigned keep = 0;
    for (int r = 0; r < KG; ++r) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int g = 0; g < NJ; ++g)
        if (g < G && !((keep >> g) & 1u) && (gscore[g] > best || (gscore[g] == best && g < bi))) {
          best = gscore[g];
          bi = g;
        }
      if (bi < G) keep |= 1u << bi;
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      if (!((keep >> (j / jpg)) & 1u)) v[j] = -INFINITY;
  }
  float sum = 0.f;
  int myid = -1;
  float myw = 0.f;
  for (int r = 0; r < K; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      if (v[j] > bv || (v[j] == bv && e < bi)) { bv = v[j]; bi = e; }
    }
    warp_argmax(bv, bi);
    if (bi >= E) bi = 0;
    float pw = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      if (j == bi / 32) {
        pw = p[j];
        if (lane == (bi & 31)) v[j] = -INFINITY;     // taken
      }
    pw = __shfl_sync(0xffffffffu, pw, bi & 31);
    sum += pw;
    if (lane == r) { myid = bi; myw = pw; }
  }
  if (lane < K) {
    ids[static_cast<size_t>(t) * K + lane] = myid;
    wts[static_cast<size_t>(t) * K + lane] = myw / fmaxf(sum, 1e-20f) * scale;
  }
}

}  // namespace

cudaError_t moe_route(const float* logits, const float* bias, int* ids, float* wts, int T, int E, int K, int G,
                      int KG, float scale, cudaStream_t s, int ksplit) {
  if (T == 0) return cudaSuccess;
  if (E > 256 || K > 32 || K > E || G < 1 || G > 32 || E % G || KG < 1 || KG > G || ksplit < 1)
    return cudaErrorInvalidValue;
  const int grid = (T + kRouteWarps - 1) / kRouteWarps;
  const int stage_bytes = ksplit * E * static_cast<int>(sizeof(float));
  if (E % 32 == 0 && (E / G) % 32 == 0 && stage_bytes <= 200 * 1024) {
    switch (E / 32) {
#define IOB_ROUTE(nj)                                                                                              \
  case nj:                                                                                                         \
    if (stage_bytes > 48 * 1024)                                                                                   \
      IOB_CUDA_CHECK(cudaFuncSetAttribute(moe_route_reg_kernel<nj>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                          stage_bytes));                                                           \
    moe_route_reg_kernel<nj><<<T, kRegThreads, stage_bytes, s>>>(logits, ksplit, bias, ids, wts, T, K, G, KG,      \
                                                                 scale);                                           \
    return cudaGetLastError();
      IOB_ROUTE(1) IOB_ROUTE(2) IOB_ROUTE(3) IOB_ROUTE(4) IOB_ROUTE(5) IOB_ROUTE(6) IOB_ROUTE(7) IOB_ROUTE(8)
#undef IOB_ROUTE
      default: break;
    }
  }
  if (ksplit != 1) return cudaErrorInvalidValue;     // the shared-memory form reads summed logits
  moe_route_kernel<<<grid, 32 * kRouteWarps, 0, s>>>(logits, bias, ids, wts, T, E, K, G, KG, scale);
  return cudaGetLastError();
}

}  // namespace iob
