// DSA lightning indexer: per-token relevance scores over the cached positions, then the top-k positions as pool slots.
//
// Semantics (the reference's indexer, `negative-results/code/idx_epilogue/triton_mla_logits.py:1-12` and the
// DeepGEMM paged MQA-logits interface it patches): for query token t with Hi <= 64 indexer heads,
//     score[t, j] = k_scale[j] * sum_h w[t, h] * relu(q[t, h] . k[j])          for positions j < limit[t]
// with E4M3 queries (the per-(token, head) query scale folded into w by the caller) and the 132-byte E4M3 keys
// (128 values + fp32 scale) of the index pool.  Then the `topk` highest-scoring positions per token (ties: lower
// position first; fewer positions than topk -> all of them, padded with -1), emitted as pool slots through the page
// table, in ascending position order.
//
// indexer_logits_kernel: the index pool stores each 64-token page as [64 x 128 B values in the 128-byte-swizzle
// order][64 x fp32 scales] (ops/kvcache.py), so one plain bulk copy per page lands a ready K-major UMMA operand.
// Swap-AB kind::f8f6f4 UMMA: D[128 positions x 64 heads] = K[128 x 128] Q^T (4 MMAs of K = 32), double-buffered
// in TMEM; four epilogue warps (thread = position = TMEM lane) apply relu, the head weights and the key scale.
// One producer thread streams pages through a 4-stage ring.  Memory-bound by design: 132 B per position.
//
// indexer_topk_kernel: one CTA per token, radix select on the order-preserving integer image of the fp32 scores
// (12 + 12 + 8 bits, shared-memory histograms), then a position-ordered compaction.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kITile = 128;                 // positions per tile (two pages)
constexpr int kIStages = 4;
constexpr int kIStageBytes = 2 * 64 * 128;  // values of two pages
constexpr int kIThreads = 192;              // warp 0 producer, warp 1 MMA, warps 2..5 epilogue
constexpr int kIPageBytes = 64 * 132;

struct IdxSmem {
  uint64_t full[kIStages], empty[kIStages];
  uint64_t d_full[2], d_empty[2];
  uint64_t q_ready, fin;
  float scales[kIStages][kITile];
  uint32_t tmem_base;
  int abort;
};

template <int DUMMY = 0>
__global__ void __launch_bounds__(kIThreads, 1) indexer_logits_kernel(const IndexerArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                   // kIStages x 16 KB
  uint8_t* sq = ring + kIStages * kIStageBytes;           // Q: 64 heads x 128 B, SW128
  IdxSmem& sm = *reinterpret_cast<IdxSmem*>(sq + 64 * 128);

  const int t = blockIdx.y;
  const int limit = a.limit[t];
  const int ntile_all = (limit + kITile - 1) / kITile;
  const int tile0 = blockIdx.x * a.tiles_per_cta;
  const int ntiles = min(ntile_all, tile0 + a.tiles_per_cta) - tile0;
  if (ntiles <= 0) return;
  const int warp = warp_id(), lane = lane_id();
  const int* pt = a.page_table + static_cast<size_t>(a.req_idx ? a.req_idx[t] : t) * a.pt_stride;
  const int n_pages = (limit + 63) / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kIStages; ++i) { mbar_init(&sm.full[i], 1); mbar_init(&sm.empty[i], 1 + 4); }
    for (int i = 0; i < 2; ++i) { mbar_init(&sm.d_full[i], 1); mbar_init(&sm.d_empty[i], 4); }
    mbar_init(&sm.q_ready, 4);
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&sm.tmem_base, 128); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer: two pages per tile
    if (lane == 0) {
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kIStages;
        if (j >= kIStages && !mbar_wait(&sm.empty[st], ((j / kIStages) - 1) & 1, abort, a.status, kTimeoutProducer))
          break;
        uint32_t bytes = 0;
        int phys[2];
        for (int pg = 0; pg < 2; ++pg) {
          const int lp = 2 * (tile0 + j) + pg;
          phys[pg] = lp < n_pages ? pt[lp] : -1;
          if (phys[pg] >= 0) bytes += 64 * 128 + 64 * 4;
        }
        if (bytes) mbar_expect_tx(&sm.full[st], bytes);
        for (int pg = 0; pg < 2; ++pg) {
          if (phys[pg] < 0) continue;
          const uint8_t* page = a.pool + static_cast<size_t>(phys[pg]) * kIPageBytes;
          bulk_g2s(ring + st * kIStageBytes + pg * 64 * 128, page, 64 * 128, &sm.full[st]);
          bulk_g2s(&sm.scales[st][64 * pg], page + 64 * 128, 64 * 4, &sm.full[st]);
        }
        if (!bytes) mbar_arrive(&sm.full[st]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc = idesc_dense(0, 0, 128, 64);
      const uint32_t ring_a = smem_u32(ring), q_a = smem_u32(sq);
      bool ok = mbar_wait(&sm.q_ready, 0, abort, a.status, kTimeoutMma);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j % kIStages, db = j & 1;
        if (!(ok = mbar_wait(&sm.full[st], (j / kIStages) & 1, abort, a.status, kTimeoutMma))) break;
        if (j >= 2 && !(ok = mbar_wait(&sm.d_empty[db], ((j >> 1) - 1) & 1, abort, a.status, kTimeoutMma))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f8_ss(tmem + 64 * db, desc_sw128(ring_a + st * kIStageBytes + 32 * kk), desc_sw128(q_a + 32 * kk), idesc,
                     kk > 0 ? 1u : 0u);
        umma_commit(&sm.d_full[db]);
        umma_commit(&sm.empty[st]);
      }
      umma_commit(&sm.fin);            // every issued MMA has completed before TMEM is released
      mbar_wait(&sm.fin, 0, nullptr, a.status, kTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------------ epilogue: thread = position in tile
    const int quad = warp & 3;                    // TMEM lane quadrant this warp may access
    const int row = 32 * quad + lane;             // position within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    // Q [64 heads x 128 B] (head h = row of the B operand) -> SW128 shared memory, zero beyond Hi
    for (int i = threadIdx.x - 64; i < 64 * 8; i += 128) {
      const int h = i >> 3, c = i & 7;
      const uint4 v = h < a.Hi ? *reinterpret_cast<const uint4*>(a.q8 + (static_cast<size_t>(t) * a.Hi + h) * 128 + 16 * c)
                               : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sq + sw128_chunk(h, c)) = v;
    }
    float w[64];
#pragma unroll
    for (int h = 0; h < 64; ++h) w[h] = h < a.Hi ? a.w[static_cast<size_t>(t) * a.Hi + h] : 0.f;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.q_ready);
    float* out = a.scores + static_cast<size_t>(t) * a.score_stride;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % kIStages, db = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.d_full[db], (j >> 1) & 1, abort, a.status, kTimeoutConsumer))) break;
      tc_fence_after();
      uint32_t d[64];
      tmem_ld32(tmem + lane_base + 64 * db, d);
      tmem_ld32(tmem + lane_base + 64 * db + 32, d + 32);
      tmem_ld_wait();
      // the key scales came in with the stage's bulk copies: acquire that phase here too before reading them
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.full[st], (j / kIStages) & 1, abort, a.status, kTimeoutConsumer))) break;
      const float ks = sm.scales[st][row];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) { mbar_arrive(&sm.d_empty[db]); mbar_arrive(&sm.empty[st]); }
      float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
      for (int h = 0; h < 64; h += 4) {
        acc0 = fmaf(w[h], fmaxf(__uint_as_float(d[h]), 0.f), acc0);
        acc1 = fmaf(w[h + 1], fmaxf(__uint_as_float(d[h + 1]), 0.f), acc1);
        acc2 = fmaf(w[h + 2], fmaxf(__uint_as_float(d[h + 2]), 0.f), acc2);
        acc3 = fmaf(w[h + 3], fmaxf(__uint_as_float(d[h + 3]), 0.f), acc3);
      }
      const int pos = (tile0 + j) * kITile + row;
      if (pos < a.score_stride) out[pos] = pos < limit ? ks * ((acc0 + acc1) + (acc2 + acc3)) : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kKThreads = 1024;

// Block-wide exclusive prefix sum of one int per thread (1024 threads); returns the total through `total`.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = lane_id(), warp = warp_id();
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = warp_sums[lane];
    int wincl = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wincl, o);
      if (lane >= o) wincl += n;
    }
    warp_sums[lane] = wincl - ws;
    if (lane == 31) warp_sums[32] = wincl;
  }
  __syncthreads();
  const int res = warp_sums[warp] + incl - v;
  total = warp_sums[32];
  __syncthreads();
  return res;
}

// Keys a thread holds in registers in the register form (score rows up to kRegKeys x kKThreads = 16384 positions).
constexpr int kRegKeys = 16;

// REG: the row's order keys are loaded once into registers (each thread a contiguous range of up to kRegKeys
// positions, 16-byte loads) and every radix pass and the compaction run from them -- one round of global loads
// instead of five passes over the row.  Otherwise every pass re-reads the scores (rows longer than 16384).
template <bool REG>
__global__ void __launch_bounds__(kKThreads) indexer_topk_kernel(const IndexerArgs a) {
  __shared__ int hist[4096];
  __shared__ int warp_sums[33];
  __shared__ int sel_bin, sel_above;
  const int t = blockIdx.x;
  const int L = min(a.limit[t], a.score_stride);
  const int K = a.topk;
  const float* sc = a.scores + static_cast<size_t>(t) * a.score_stride;
  const int* pt = a.page_table + static_cast<size_t>(a.req_idx ? a.req_idx[t] : t) * a.pt_stride;
  int* out = a.out_slots + static_cast<size_t>(t) * K;
  int* out_pos = a.out_pos ? a.out_pos + static_cast<size_t>(t) * K : nullptr;
  auto emit = [&](int i, int p) {
    out[i] = p >= 0 ? pt[p >> 6] * 64 + (p & 63) : -1;
    if (out_pos) out_pos[i] = p;
  };
  if (L <= K) {
    for (int i = threadIdx.x; i < K; i += kKThreads) emit(i, i < L ? i : -1);
    return;
  }
  // this thread's contiguous range [i0, i1) (position order is thread order: the compaction emits in it)
  const int chunk = REG ? (((L + kKThreads - 1) / kKThreads + 3) & ~3) : (L + kKThreads - 1) / kKThreads;
  const int i0 = threadIdx.x * chunk, i1 = min(L, i0 + chunk);
  uint32_t keys[REG ? kRegKeys : 1];
  if constexpr (REG) {
#pragma unroll
    for (int j = 0; j < kRegKeys; j += 4) {
      if (i0 + j + 3 < i1) {
        const float4 v = *reinterpret_cast<const float4*>(sc + i0 + j);
        keys[j] = order_key(v.x);
        keys[j + 1] = order_key(v.y);
        keys[j + 2] = order_key(v.z);
        keys[j + 3] = order_key(v.w);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) keys[j + q] = i0 + j + q < i1 ? order_key(sc[i0 + j + q]) : 0u;
      }
    }
  }
  // ---- radix select of the K-th largest order key: 12 + 12 + 8 bits
  uint32_t prefix = 0, mask = 0;
  int remaining = K;
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], nb = 1 << widths[pass];
    for (int b = threadIdx.x; b < 4096; b += kKThreads) hist[b] = 0;
    __syncthreads();
    if constexpr (REG) {
      // (warp-aggregated counts through __match_any_sync measured slower here: 12.6 -> 19.4 us per call at 8 tokens)
#pragma unroll
      for (int j = 0; j < kRegKeys; ++j)
        if (i0 + j < i1 && (keys[j] & mask) == prefix) atomicAdd(&hist[(keys[j] >> sh) & (nb - 1)], 1);
    } else {
      for (int i = threadIdx.x; i < L; i += kKThreads) {
        const uint32_t u = order_key(sc[i]);
        if ((u & mask) == prefix) atomicAdd(&hist[(u >> sh) & (nb - 1)], 1);
      }
    }
    __syncthreads();
    // suffix sums from the top bin: each thread owns 4 consecutive bins (nb / 1024 <= 4)
    const int per = nb / kKThreads > 0 ? nb / kKThreads : 1;
    const int b0 = nb - (threadIdx.x + 1) * per;       // thread 0 owns the highest bins
    int mine = 0;
    if (b0 >= 0)
      for (int k = 0; k < per; ++k) mine += hist[b0 + k];
    int total;
    const int above = block_exclusive_scan(mine, warp_sums, total);   // count in bins higher than this thread's
    if (b0 >= 0 && above < remaining && above + mine >= remaining) {
      int acc = above;
      for (int k = per - 1; k >= 0; --k) {
        const int c = hist[b0 + k];
        if (acc + c >= remaining) { sel_bin = b0 + k; sel_above = acc; break; }
        acc += c;
      }
    }
    __syncthreads();
    remaining -= sel_above;
    prefix |= static_cast<uint32_t>(sel_bin) << sh;
    mask |= static_cast<uint32_t>(nb - 1) << sh;
    __syncthreads();
  }
  // ---- compaction in position order: keys above the threshold, then the first `remaining` equal ones
  int gt = 0, eq = 0;
  if constexpr (REG) {
#pragma unroll
    for (int j = 0; j < kRegKeys; ++j)
      if (i0 + j < i1) {
        gt += keys[j] > prefix;
        eq += keys[j] == prefix;
      }
  } else {
    for (int i = i0; i < i1; ++i) {
      const uint32_t u = order_key(sc[i]);
      gt += u > prefix;
      eq += u == prefix;
    }
  }
  int tot;
  const int eq_before = block_exclusive_scan(eq, warp_sums, tot);
  const int take_eq = max(0, min(eq, remaining - eq_before));
  const int off = block_exclusive_scan(gt + take_eq, warp_sums, tot);
  int w = off, eq_seen = 0;
  if constexpr (REG) {
#pragma unroll
    for (int j = 0; j < kRegKeys; ++j)
      if (i0 + j < i1 && (keys[j] > prefix || (keys[j] == prefix && eq_seen++ < take_eq))) emit(w++, i0 + j);
  } else {
    for (int i = i0; i < i1; ++i) {
      const uint32_t u = order_key(sc[i]);
      if (u > prefix || (u == prefix && eq_seen++ < take_eq)) emit(w++, i);
    }
  }
}

// Cluster form for long rows (16,384 < positions <= kClMax x kClKeys x kKThreads = 262,144): the row is split into
// CL contiguous spans, one per CTA of a thread-block cluster, each span's order keys held in registers (up to
// kClKeys per thread).  Each radix pass builds one histogram per CTA; every CTA then sums the CL histograms of its
// bins over distributed shared memory and takes the same threshold decision, so the select costs one round of
// global loads spread over CL SMs instead of one SM re-reading the row five times.  The compaction keeps position
// order across the cluster: a CTA's outputs start after the keys above the threshold, and the equal keys taken, of
// the spans before it.  All waits are the cluster's hardware barriers, which every CTA of the cluster reaches (the
// branch on the row length is the same for the whole cluster).
constexpr int kClKeys = 32;
constexpr int kClMax = 8;

__global__ void __launch_bounds__(kKThreads, 1) indexer_topk_cluster_kernel(const IndexerArgs a) {
  __shared__ int hist[4096];
  __shared__ int warp_sums[33];
  __shared__ int sel_bin, sel_above;
  __shared__ int sums[4096];                 // the cluster-wide counts of the bins this CTA's threads own
  __shared__ int counts[2];                  // this span's keys above the threshold / equal to it
  const int t = blockIdx.y;
  const int cr = static_cast<int>(cluster_ctarank()), cn = static_cast<int>(cluster_nctarank());
  const int L = min(a.limit[t], a.score_stride);
  const int K = a.topk;
  const float* sc = a.scores + static_cast<size_t>(t) * a.score_stride;
  const int* pt = a.page_table + static_cast<size_t>(a.req_idx ? a.req_idx[t] : t) * a.pt_stride;
  int* out = a.out_slots + static_cast<size_t>(t) * K;
  int* out_pos = a.out_pos ? a.out_pos + static_cast<size_t>(t) * K : nullptr;
  auto emit = [&](int i, int p) {
    out[i] = p >= 0 ? pt[p >> 6] * 64 + (p & 63) : -1;
    if (out_pos) out_pos[i] = p;
  };
  if (L <= K) {
    if (cr == 0)
      for (int i = threadIdx.x; i < K; i += kKThreads) emit(i, i < L ? i : -1);
    return;
  }
  // this CTA's span [c0, c1) and this thread's n positions from i0 in it (multiples of 4: 16-byte loads)
  const int span = ((L + cn - 1) / cn + 3) & ~3;               // <= kClKeys x kKThreads (host-side bound)
  const int c0 = min(L, cr * span), c1 = min(L, c0 + span);
  const int chunk = ((span + kKThreads - 1) / kKThreads + 3) & ~3;
  const int i0 = c0 + threadIdx.x * chunk, n = max(0, min(c1, i0 + chunk) - i0);
  uint32_t keys[kClKeys];
#pragma unroll
  for (int j = 0; j < kClKeys; j += 4) {
    if (j + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(sc + i0 + j);
      keys[j] = order_key(v.x);
      keys[j + 1] = order_key(v.y);
      keys[j + 2] = order_key(v.z);
      keys[j + 3] = order_key(v.w);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) keys[j + q] = j + q < n ? order_key(sc[i0 + j + q]) : 0u;
    }
  }
  const uint32_t hist_addr = smem_u32(hist);
  uint32_t prefix = 0, mask = 0;
  int remaining = K;
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], nb = 1 << widths[pass];
    for (int b = threadIdx.x; b < 4096; b += kKThreads) hist[b] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kClKeys; ++j)
      if (j < n && (keys[j] & mask) == prefix) atomicAdd(&hist[(keys[j] >> sh) & (nb - 1)], 1);
    cluster_sync_all();                      // every span's histogram complete and visible to the cluster
    // this thread's `per` bins (thread 0 the highest), summed over the cluster's histograms in CTA order
    const int per = nb / kKThreads > 0 ? nb / kKThreads : 1;
    const int b0 = nb - (threadIdx.x + 1) * per;
    int mine = 0;
    if (b0 >= 0)
      for (int k = 0; k < per; ++k) {
        int c = 0;
        for (int r = 0; r < cn; ++r) c += static_cast<int>(ld_cluster_u32(mapa_shared(hist_addr + 4u * (b0 + k), r)));
        sums[b0 + k] = c;
        mine += c;
      }
    int total;
    const int above = block_exclusive_scan(mine, warp_sums, total);
    if (b0 >= 0 && above < remaining && above + mine >= remaining) {
      int acc = above;
      for (int k = per - 1; k >= 0; --k) {
        const int c = sums[b0 + k];
        if (acc + c >= remaining) { sel_bin = b0 + k; sel_above = acc; break; }
        acc += c;
      }
    }
    __syncthreads();
    remaining -= sel_above;
    prefix |= static_cast<uint32_t>(sel_bin) << sh;
    mask |= static_cast<uint32_t>(nb - 1) << sh;
    cluster_sync_all();                      // no CTA clears its histogram while another still reads it
  }
  // ---- compaction in position order across the cluster
  int gt = 0, eq = 0;
#pragma unroll
  for (int j = 0; j < kClKeys; ++j)
    if (j < n) {
      gt += keys[j] > prefix;
      eq += keys[j] == prefix;
    }
  int gt_span, eq_span;
  const int eq_before = block_exclusive_scan(eq, warp_sums, eq_span);
  block_exclusive_scan(gt, warp_sums, gt_span);
  if (threadIdx.x == 0) { counts[0] = gt_span; counts[1] = eq_span; }
  cluster_sync_all();
  int gt_prev = 0, eq_prev = 0;               // the spans before this one
  const uint32_t counts_addr = smem_u32(counts);
  for (int r = 0; r < cr; ++r) {
    gt_prev += static_cast<int>(ld_cluster_u32(mapa_shared(counts_addr, r)));
    eq_prev += static_cast<int>(ld_cluster_u32(mapa_shared(counts_addr + 4u, r)));
  }
  cluster_sync_all();                        // last remote read: a CTA may exit after this barrier
  const int take_eq = max(0, min(eq, remaining - eq_prev - eq_before));
  int tot;
  const int off = gt_prev + min(eq_prev, remaining) + block_exclusive_scan(gt + take_eq, warp_sums, tot);
  int w = off, eq_seen = 0;
#pragma unroll
  for (int j = 0; j < kClKeys; ++j)
    if (j < n && (keys[j] > prefix || (keys[j] == prefix && eq_seen++ < take_eq))) emit(w++, i0 + j);
}

}  // namespace

cudaError_t indexer_logits(const IndexerArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.Hi < 1 || a.Hi > 64 || a.tiles_per_cta < 1 || a.max_tiles < 1 || a.T > 65535) return cudaErrorInvalidValue;
  const int smem = 1024 + kIStages * kIStageBytes + 64 * 128 + static_cast<int>(sizeof(IdxSmem));
  auto kern = indexer_logits_kernel<0>;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kern<<<dim3((a.max_tiles + a.tiles_per_cta - 1) / a.tiles_per_cta, a.T), kIThreads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t indexer_topk(const IndexerArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.topk < 1) return cudaErrorInvalidValue;
  constexpr int kClSpan = kClKeys * kKThreads;
  if (a.score_stride <= kRegKeys * kKThreads) {
    indexer_topk_kernel<true><<<a.T, kKThreads, 0, s>>>(a);
  } else if (a.score_stride <= kClMax * kClSpan && a.T <= 65535) {
    const unsigned cl = static_cast<unsigned>((a.score_stride + kClSpan - 1) / kClSpan);   // 1 .. 8 CTAs per row
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, a.T);
    cfg.blockDim = dim3(kKThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // a cluster of full-SM CTAs needs cl SMs of one GPC free to it (an SM partition of the device may hold fewer):
    // the re-reading form serves the row when no such cluster fits
    int fits = 0;
    if (cudaOccupancyMaxActiveClusters(&fits, indexer_topk_cluster_kernel, &cfg) == cudaSuccess && fits > 0)
      return cudaLaunchKernelEx(&cfg, indexer_topk_cluster_kernel, a);
    (void)cudaGetLastError();
  }
  if (a.score_stride > kRegKeys * kKThreads) indexer_topk_kernel<false><<<a.T, kKThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace iob
