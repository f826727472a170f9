// MoE router: sigmoid scores, bias-corrected group-limited top-k, renormalised weights (ops/moe.py route_ref is the
// oracle; semantics of the DeepSeek `noaux_tc` router).  One warp per token; the E <= 256 biased scores are staged
// in shared memory, groups and experts are picked by repeated warp arg-max (ties: lower index).
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

}  // namespace

cudaError_t moe_route(const float* logits, const float* bias, int* ids, float* wts, int T, int E, int K, int G,
                      int KG, float scale, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (E > 256 || K > 32 || K > E || G < 1 || G > 32 || E % G || KG < 1 || KG > G) return cudaErrorInvalidValue;
  moe_route_kernel<<<(T + kRouteWarps - 1) / kRouteWarps, 32 * kRouteWarps, 0, s>>>(logits, bias, ids, wts, T, E, K, G,
                                                                                     KG, scale);
  return cudaGetLastError();
}

}  // namespace iob
