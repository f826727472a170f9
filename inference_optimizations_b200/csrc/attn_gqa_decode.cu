// GQA-packed split-K decode / speculative-verify attention over a paged NVFP4 / FP8 / bf16 KV pool, sm_100a.
//
// Capability of the reference's split-K verify and NVFP4 decode kernels (`attention/verify-splitk/gemma31_verify.py`
// K29, `kv-cache-4bit/kv4tri-triton-backend/kv4tri_nvfp4_attention.py:257` nvfp4_decode_fwd): one CTA per
// (request, kv head, split); its rows are the request's n_q query tokens x the G query heads sharing the kv head, so
// every KV byte is read once per kv head.  Designed for tcgen05 rather than transliterated:
//
//  * swap-AB: tokens are the MMA M dimension (128 per tile), query rows the N dimension (16), so a decode step with
//    2..16 rows still issues full-height UMMAs.  S^T = K Q^T lands in TMEM with lane = token, column = row.
//  * K never touches shared memory after its raw bytes: the dequant warp that owns a token (TMEM lane) expands it
//    to f16 and writes it straight into TMEM with tcgen05.st; QK is the A-from-TMEM UMMA form.  One handoff per tile.
//  * O^T = V^T P^T with V (MN-major) read from f16 128-byte-swizzled slabs in a shared-memory ring.
//  * the pool is read by one bulk async copy per (page, kv head, K|V) into a raw ring; pool rows are stored with a
//    16-byte chunk XOR swizzle so the dequant reads and slab writes are bank-conflict free.
//  * skewed schedule: iteration j handles K of tile j, then V of tile j-1, so the softmax of tile j-1 overlaps the
//    next tile's loads, dequant and QK instead of sitting between QK and PV.
//  * warp roles: 0-3 softmax + O accumulation (registers), 4-11 dequant, 12 bulk-copy producer, 13 UMMA issuer.
//  * split-K partials (o normalised, lse in log2 units) are merged by a second kernel.
//  * every mbarrier wait is bounded; a timeout records a status code and the CTA unwinds.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kTileTok = 128;
constexpr int kN = 16;           // UMMA N (query rows, padded)
constexpr int kSlabBytes = kTileTok * 128;
constexpr int kThreads = 448;
constexpr int kSoftmaxWarps = 4;
constexpr int kDequantWarps = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemK = 256;  // K tile: D/2 columns (two f16 per column)
constexpr int kSParts = 4;        // independent partial S accumulators (QK k-steps interleaved across them)

struct Smem {
  uint64_t raw_full[8], raw_empty[8];
  uint64_t ring_full[8], ring_empty[8];
  uint64_t k_full, k_empty;
  uint64_t s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2];
  uint64_t kf[2], ke[2];  // E4M3 path: double-buffered K tile in TMEM
  uint64_t pe[2], od;     // E4M3 path, <= 2 query rows: P buffer released by the PV warps; final O in smem
  uint32_t tmem_base;
  int abort;
  int raw_valid[8];       // stage holds a real page (else the dequant writes zeros); published by the producer
  float red[kSoftmaxWarps][kN];
  float row_m[kN];
  float q_scale[kN];      // E4M3 path: per-row Q scale (q = e4m3 * q_scale)
};
constexpr int kF4TabBytes = 256 * 8;   // E4M3 path, NVFP4 pools: scale byte -> E4M3 products, after Smem

// must match kv_swizzle_byte() (kernels.h), which the pool writers use
__device__ __forceinline__ int pool_chunk_pos(int j, int r, int nch) {
  return (j & ~(nch - 1)) | ((j ^ r) & (nch - 1));
}

__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(lbo_bytes >> 4) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  float2 f = __bfloat1622float2(b);
  __half2 h = __float22half2_rn(f);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int FMT, int D>
__device__ __forceinline__ constexpr int part_bytes() {
  return FMT == kKvNvfp4 ? 64 * (D / 2 + D / 16) : (FMT == kKvFp8 ? 64 * D : 64 * D * 2);
}
// Shared memory split: V slab ring (4 x 16 KB) + Q + P, the rest is raw staging (bytes in flight are what bounds
// a latency-limited stream; the L2 prefetch below covers the remaining distance).
template <int FMT, int D>
__device__ __host__ __forceinline__ constexpr int ring_slabs() { return part_bytes<FMT, D>() <= 20 * 1024 ? 6 : 4; }

// Diagnostic timeline (CTA 0 only, when a.trace is set): event e of tile j at trace[e * 512 + j].
enum TraceEv { kEvKDeqStart, kEvKDeqEnd, kEvVDeqStart, kEvVDeqEnd, kEvQkStart, kEvQkEnd, kEvPvStart, kEvPvEnd,
               kEvSReady, kEvPReady, kEvODone, kEvProdK, kEvProdV, kEvKRaw, kEvStart, kEvEnd };
__device__ __forceinline__ void trace_ev(long long* tr, int ev, int j) {
  if (tr != nullptr && blockIdx.x == 0 && j < 512) tr[ev * 512 + j] = clock64();
}
template <int FMT, int D>
__device__ __host__ __forceinline__ constexpr int raw_stages() {
  // 224 KB minus ring, Q and P, in whole parts; at least 2 (a part is two pages resident together), at most 8
  return (229376 - ring_slabs<FMT, D>() * 16384 - (D / 64) * 2048 - 8192) / part_bytes<FMT, D>() > 8   ? 8
         : (229376 - ring_slabs<FMT, D>() * 16384 - (D / 64) * 2048 - 8192) / part_bytes<FMT, D>() < 2 ? 2
         : (229376 - ring_slabs<FMT, D>() * 16384 - (D / 64) * 2048 - 8192) / part_bytes<FMT, D>();
}
constexpr int kPrefetchParts = 4;   // L2 prefetch distance, in parts (2 tiles)

// 16 code bytes (32 values) of an NVFP4 row at 16-byte chunk j -> 16 f16x2, scaled by the two block scales.
__device__ __forceinline__ void nvfp4_chunk(const uint8_t* row, int pos, uint32_t s0, uint32_t s1, uint32_t* ow) {
  const uint4 in = *reinterpret_cast<const uint4*>(row + pos * 16);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&in);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t f[4];
    e2m1x8_to_f16x2x4(w[i], f);
#pragma unroll
    for (int k = 0; k < 4; ++k) ow[4 * i + k] = hmul2_u32(f[k], i < 2 ? s0 : s1);
  }
}
__device__ __forceinline__ uint32_t scale_h2(uint16_t two, int which) {
  const uint32_t f = e4m3x2_to_f16x2(two);
  return half2_bcast(__ushort_as_half(static_cast<unsigned short>(which ? (f >> 16) : (f & 0xFFFF))));
}

// Expand 32 values (one token row, dims [64c + 32 half, +32)) to 16 f16x2 words.
template <int FMT, int D>
__device__ __forceinline__ void dequant_32(const uint8_t* part, int r, int c, int half, uint32_t* ow) {
  if constexpr (FMT == kKvNvfp4) {
    constexpr int RB = D / 2, NCH = (RB / 16) < 8 ? (RB / 16) : 8;
    const uint16_t sc = *reinterpret_cast<const uint16_t*>(part + 64 * RB + r * (D / 16) + c * 4 + half * 2);
    nvfp4_chunk(part + r * RB, pool_chunk_pos(2 * c + half, r, NCH), scale_h2(sc, 0), scale_h2(sc, 1), ow);
  } else if constexpr (FMT == kKvFp8) {
    constexpr int RB = D, NCH = 8;
    const uint8_t* row = part + r * RB;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint4 in = *reinterpret_cast<const uint4*>(row + pool_chunk_pos(4 * c + 2 * half + k, r, NCH) * 16);
      const uint16_t* h = reinterpret_cast<const uint16_t*>(&in);
#pragma unroll
      for (int i = 0; i < 8; ++i) ow[8 * k + i] = e4m3x2_to_f16x2(h[i]);
    }
  } else {
    constexpr int RB = 2 * D, NCH = 8;
    const uint8_t* row = part + r * RB;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 in = *reinterpret_cast<const uint4*>(row + pool_chunk_pos(8 * c + 4 * half + k, r, NCH) * 16);
      const uint32_t* iw = reinterpret_cast<const uint32_t*>(&in);
#pragma unroll
      for (int i = 0; i < 4; ++i) ow[4 * k + i] = bf16x2_to_f16x2(iw[i]);
    }
  }
}

template <int FMT, int D, int RMAX>
__global__ void __launch_bounds__(kThreads, 1) gqa_decode_kernel(const GqaDecodeArgs a) {
  constexpr int NS = D / 64;                       // 64-dim slabs per head vector
  constexpr int PB = part_bytes<FMT, D>();         // bytes of K (or V) of one (page, head)
  constexpr int NST = raw_stages<FMT, D>();
  constexpr int RING = ring_slabs<FMT, D>();
  constexpr int MB = D / 128;                      // 128-dim M blocks of O^T
  constexpr int kOCols = MB * kN;
  static_assert(RMAX <= kN, "rows");
  static_assert(RING % 2 == 0, "V slab pairs need an even ring");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                   // RING x 16 KB (V slabs)
  uint8_t* sq = ring + RING * kSlabBytes;                 // NS x 2 KB
  uint8_t* sp = sq + NS * kN * 128;                       // 2 x (2 x 2 KB)
  uint8_t* raw = sp + 2 * 2 * kN * 128;                   // NST x PB
  Smem& sm = *reinterpret_cast<Smem*>(raw + NST * PB);

  const int G = a.Hq / a.Hk;
  const int R = a.n_q * G;
  const int work = blockIdx.x;
  const int split = work % a.num_splits;
  const int bh = work / a.num_splits;
  const int h = bh % a.Hk;
  const int b = bh / a.Hk;
  const int kv_len = a.kv_len[b];
  const int q_first = kv_len - a.n_q;                     // position of query token 0
  const int kv_begin = a.window > 0 ? max(0, q_first - a.window + 1) : 0;
  const int tile0 = kv_begin / kTileTok + split * a.tiles_per_split;
  const int tile_end = min((kv_len + kTileTok - 1) / kTileTok, kv_begin / kTileTok + (split + 1) * a.tiles_per_split);
  const int ntiles = tile_end - tile0;
  const size_t part_out = (static_cast<size_t>(bh) * a.num_splits + split);
  if (ntiles <= 0) {  // empty split: publish an empty partial
    if (a.num_splits > 1 && threadIdx.x < RMAX) a.lse_part[part_out * RMAX + threadIdx.x] = -INFINITY;
    return;
  }
  const int first_page = kv_begin / a.page;
  const int n_pages = (kv_len + a.page - 1) / a.page;
  const int* pt = a.page_table + static_cast<size_t>(a.req_idx ? a.req_idx[b] : b) * a.pt_stride;
  const int warp = warp_id(), lane = lane_id();

  // ---- Q -> f16 slabs (rows >= R zero), barriers, TMEM
  {
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
    for (int idx = threadIdx.x; idx < kN * NS * 8; idx += kThreads) {
      const int row = idx / (NS * 8), rem = idx % (NS * 8), c = rem / 8, ch = rem % 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row < R) {
        const int t = row / G, g = row % G;
        const uint4 in = *reinterpret_cast<const uint4*>(
            q + ((static_cast<size_t>(b) * a.n_q + t) * a.Hq + h * G + g) * D + c * 64 + ch * 8);
        const uint32_t* iw = reinterpret_cast<const uint32_t*>(&in);
        uint32_t* ow = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) ow[i] = bf16x2_to_f16x2(iw[i]);
      }
      *reinterpret_cast<uint4*>(sq + c * (kN * 128) + sw128_chunk(row, ch)) = v;
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) { mbar_init(&sm.raw_full[i], 1); mbar_init(&sm.raw_empty[i], kDequantWarps); }
    for (int i = 0; i < RING; ++i) { mbar_init(&sm.ring_full[i], kDequantWarps); mbar_init(&sm.ring_empty[i], 1); }
    mbar_init(&sm.k_full, kDequantWarps);
    mbar_init(&sm.k_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1); mbar_init(&sm.s_empty[i], kSoftmaxWarps);
      mbar_init(&sm.p_full[i], kSoftmaxWarps); mbar_init(&sm.o_full[i], 1); mbar_init(&sm.o_empty[i], kSoftmaxWarps);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) { tmem_alloc(&sm.tmem_base, kTmemCols); tmem_relinquish(); }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tS = tmem;            // 2 buffers x kSParts partial S accumulators x 16 columns
  const uint32_t tO = tmem + 128;      // 2 x kOCols columns
  const uint32_t tK = tmem + kTmemK;   // D/2 columns
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) trace_ev(a.trace, kEvStart, 0);

  // Work order (every role walks it identically): iteration j = 0..ntiles handles the K part of tile j (when
  // j < ntiles), then the V part of tile j - 1 (when j >= 1).  A "part" is one (K | V, tile): 2 raw pages
  // (raw seq 2p, 2p+1).  V parts also own NS ring slabs (ring seq NS v .. NS v + NS - 1, v = tile index).
  auto parts_before = [&](int j) { return min(j, ntiles) + max(0, j - 1); };
  auto part_index = [&](int j, int which) { return parts_before(j) + ((which == 1 && j < ntiles) ? 1 : 0); };

  if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint8_t* pool = a.pool;
      // part index -> (tile, which): 0 = K0; 2j-1 = K(j) (j < ntiles) or V(ntiles-1) (last); 2j = V(j-1)
      auto prefetch_part = [&](int p) {
        if (p >= 2 * ntiles) return;
        int tile, which;
        if (p == 0) { tile = 0; which = 0; }
        else if (p & 1) { const int j = (p + 1) / 2; if (j < ntiles) { tile = j; which = 0; } else { tile = ntiles - 1; which = 1; } }
        else { tile = p / 2 - 1; which = 1; }
        for (int pg = 0; pg < 2; ++pg) {
          const int pidx = (tile0 + tile) * 2 + pg;
          const int phys = (pidx >= first_page && pidx < n_pages) ? pt[pidx] : -1;
          if (phys >= 0) prefetch_l2(pool + (static_cast<size_t>(phys) * a.Hk + h) * (2 * PB) + which * PB, PB);
        }
      };
      for (int p = 0; p < kPrefetchParts; ++p) prefetch_part(p);
      int issued = 0;
      for (int j = 0; j <= ntiles && !*abort; ++j) {
        for (int which = 0; which < 2; ++which) {
          const int tile = which == 0 ? j : j - 1;
          if (tile < 0 || tile >= ntiles) continue;
          const int pidx0 = part_index(j, which);
          prefetch_part(pidx0 + kPrefetchParts);
          for (int pg = 0; pg < 2; ++pg) {
            const int seq = 2 * pidx0 + pg, st = seq % NST;
            if (*abort) break;
            if (!mbar_wait(&sm.raw_empty[st], ((seq / NST) & 1) ^ 1, abort, a.status, kTimeoutProducer)) break;
            issued = seq + 1;
            if (pg == 0) trace_ev(a.trace, which == 0 ? kEvProdK : kEvProdV, tile);
            const int pidx = (tile0 + tile) * 2 + pg;
            const int phys = (pidx >= first_page && pidx < n_pages) ? pt[pidx] : -1;
            if (phys >= 0) {
              const uint8_t* src = pool + (static_cast<size_t>(phys) * a.Hk + h) * (2 * PB) + which * PB;
              sm.raw_valid[st] = 1;
              mbar_expect_tx(&sm.raw_full[st], PB);
              bulk_g2s(raw + st * PB, src, PB, &sm.raw_full[st]);
            } else {
              sm.raw_valid[st] = 0;
              mbar_arrive(&sm.raw_full[st]);
            }
          }
        }
      }
      // drain: the last copies must land before the CTA may exit
      for (int seq = max(0, issued - NST); seq < issued; ++seq)
        mbar_wait(&sm.raw_full[seq % NST], (seq / NST) & 1, nullptr, a.status, kTimeoutProducer);
    }
  } else if (warp >= kSoftmaxWarps && warp < kSoftmaxWarps + kDequantWarps) {
    // ---------------------------------------------------------------- dequant warps
    const int dw = warp - kSoftmaxWarps;
    // K role: thread = TMEM lane = token; warps dw and dw + 4 split the head dims in halves
    const int kq = warp & 3, ktok = 32 * kq + lane, kpg = ktok / 64, kr = ktok % 64;
    const int kdim0 = (dw >> 2) * (D / 2);
    const uint32_t k_lane = static_cast<uint32_t>(32 * kq) << 16;
    // V role: warp dw covers tokens 16 dw .. 16 dw + 15 x two 32-dim halves of a slab
    const int vtok = 16 * dw + (lane & 7) + 8 * (lane >> 4);
    const int vhalf = (lane >> 3) & 1;
    const int vpg = vtok / 64, vr = vtok % 64;
    for (int j = 0; j <= ntiles; ++j) {
      if (j < ntiles) {  // ---- K(j) -> TMEM
        const int p = part_index(j, 0);
        const int seq0 = 2 * p, st0 = seq0 % NST, st1 = (seq0 + 1) % NST;
        if (!mbar_wait(&sm.raw_full[st0], (seq0 / NST) & 1, abort, a.status, kTimeoutConsumer)) break;
        if (!mbar_wait(&sm.raw_full[st1], ((seq0 + 1) / NST) & 1, abort, a.status, kTimeoutConsumer)) break;
        if (dw == 0 && lane == 0) trace_ev(a.trace, kEvKRaw, j);
        if (!mbar_wait(&sm.k_empty, (j & 1) ^ 1, abort, a.status, kTimeoutConsumer)) break;
        tc_fence_after();
        if (dw == 0 && lane == 0) trace_ev(a.trace, kEvKDeqStart, j);
        const int st = kpg ? st1 : st0;
        const bool valid = sm.raw_valid[st] != 0;
        const uint8_t* part = raw + st * PB;
#pragma unroll 1
        for (int d0 = kdim0; d0 < kdim0 + D / 2; d0 += 64) {
          uint32_t v[32];
          if (valid) {
            dequant_32<FMT, D>(part, kr, d0 / 64, 0, v);
            dequant_32<FMT, D>(part, kr, d0 / 64, 1, v + 16);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0;
          }
          tmem_st32(tK + k_lane + d0 / 2, v);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.k_full);
          mbar_arrive(&sm.raw_empty[st0]);
          mbar_arrive(&sm.raw_empty[st1]);
          if (dw == 0) trace_ev(a.trace, kEvKDeqEnd, j);
        }
      }
      if (j == 0) continue;
      {  // ---- V(j-1) -> shared-memory ring
        const int i = j - 1;
        const int p = part_index(j, 1);
        const int seq0 = 2 * p, st0 = seq0 % NST, st1 = (seq0 + 1) % NST;
        if (!mbar_wait(&sm.raw_full[st0], (seq0 / NST) & 1, abort, a.status, kTimeoutConsumer)) break;
        if (!mbar_wait(&sm.raw_full[st1], ((seq0 + 1) / NST) & 1, abort, a.status, kTimeoutConsumer)) break;
        const int st = vpg ? st1 : st0;
        const bool valid = sm.raw_valid[st] != 0;
        if (dw == 0 && lane == 0) trace_ev(a.trace, kEvVDeqStart, i);
        bool ok = true;
        for (int c = 0; c < NS; ++c) {
          const int seq = NS * i + c, buf = seq % RING;
          if (!(ok = mbar_wait(&sm.ring_empty[buf], ((seq / RING) & 1) ^ 1, abort, a.status, kTimeoutConsumer)))
            break;
          uint32_t o[16];
          if (valid) dequant_32<FMT, D>(raw + st * PB, vr, c, vhalf, o);
          else {
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = 0;
          }
          uint8_t* slab = ring + buf * kSlabBytes;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(slab + sw128_chunk(vtok, vhalf * 4 + q)) =
                make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.ring_full[buf]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) { mbar_arrive(&sm.raw_empty[st0]); mbar_arrive(&sm.raw_empty[st1]); }
        if (dw == 0 && lane == 0) trace_ev(a.trace, kEvVDeqEnd, i);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- UMMA issuer (one thread)
    if (lane == 0) {
      const uint32_t id_qk = idesc_dense(0, 0, 128, kN);
      const uint32_t id_pv = idesc_dense(0, 0, 128, kN) | (1u << 15);   // A (V^T) MN-major
      const uint32_t ring_addr = smem_u32(ring), q_addr = smem_u32(sq), p_addr = smem_u32(sp);
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {  // QK(j): A = K tile in TMEM, B = Q slabs
          const int sb = j & 1;
          if (!mbar_wait(&sm.s_empty[sb], ((j >> 1) & 1) ^ 1, abort, a.status, kTimeoutMma)) break;
          if (!mbar_wait(&sm.k_full, j & 1, abort, a.status, kTimeoutMma)) break;
          tc_fence_after();
          trace_ev(a.trace, kEvQkStart, j);
          // k-step s accumulates into partial s % kSParts: consecutive MMAs are independent (no accumulator chain)
#pragma unroll 4
          for (int s = 0; s < D / 16; ++s)
            umma_f16_ts(tS + sb * (kSParts * kN) + (s % kSParts) * kN, tK + 8 * s,
                        desc_sw128(q_addr + (s >> 2) * (kN * 128) + (s & 3) * 32), id_qk, s >= kSParts ? 1u : 0u);
          umma_commit(&sm.s_full[sb]);
          umma_commit(&sm.k_empty);
          trace_ev(a.trace, kEvQkEnd, j);
        }
        if (j == 0) continue;
        // PV(j - 1)
        const int i = j - 1, sb = i & 1;
        if (!mbar_wait(&sm.p_full[sb], (i >> 1) & 1, abort, a.status, kTimeoutMma)) break;
        if (!mbar_wait(&sm.o_empty[sb], ((i >> 1) & 1) ^ 1, abort, a.status, kTimeoutMma)) break;
        trace_ev(a.trace, kEvPvStart, i);
        bool ok = true;
        // M blocks in groups of two (4 ring slabs), their MMAs interleaved so consecutive MMAs are independent
        constexpr int GS = MB < 2 ? MB : 2;
        for (int mg = 0; mg < MB; mg += GS) {
          for (int q = 0; q < 2 * GS && ok; ++q) {
            const int seq = NS * i + 2 * mg + q;
            ok = mbar_wait(&sm.ring_full[seq % RING], (seq / RING) & 1, abort, a.status, kTimeoutMma);
          }
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int g = 0; g < GS; ++g) {
              const int buf0 = (NS * i + 2 * (mg + g)) % RING;
              umma_f16_ss(tO + sb * kOCols + (mg + g) * kN,
                          desc_mn_sw128(ring_addr + buf0 * kSlabBytes + kk * 2048, kSlabBytes),
                          desc_sw128(p_addr + sb * (2 * kN * 128) + (kk >> 2) * (kN * 128) + (kk & 3) * 32), id_pv,
                          kk > 0 ? 1u : 0u);
            }
          }
          for (int q = 0; q < 2 * GS; ++q) umma_commit(&sm.ring_empty[(NS * i + 2 * mg + q) % RING]);
        }
        if (!ok) break;
        umma_commit(&sm.o_full[sb]);
        trace_ev(a.trace, kEvPvEnd, i);
      }
    }
  } else if (warp < kSoftmaxWarps) {
    // ---------------------------------------------------------------- softmax + O accumulation
    const float scale_log2 = a.sm_scale * a.k_scale * 1.4426950408889634f;
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    float acc[MB][RMAX];
    float lpart[RMAX];
    float alpha_prev[RMAX];
#pragma unroll
    for (int n = 0; n < RMAX; ++n) {
      lpart[n] = 0.f;
      alpha_prev[n] = 1.f;
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) acc[mb][n] = 0.f;
    }
    if (threadIdx.x < kN) sm.row_m[threadIdx.x] = -INFINITY;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    bool ok = true;
    auto consume_o = [&](int i) -> bool {
      const int sb = i & 1;
      if (!mbar_wait(&sm.o_full[sb], (i >> 1) & 1, abort, a.status, kTimeoutConsumer)) return false;
      tc_fence_after();
      uint32_t r[MB][RMAX];
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) {
        if constexpr (RMAX == 8) tmem_ld8(tO + lane_base + sb * kOCols + mb * kN, r[mb]);
        else tmem_ld16(tO + lane_base + sb * kOCols + mb * kN, r[mb]);
      }
      tmem_ld_wait();
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) {
#pragma unroll
        for (int n = 0; n < RMAX; ++n) acc[mb][n] = acc[mb][n] * alpha_prev[n] + __uint_as_float(r[mb][n]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_empty[sb]);
      if (threadIdx.x == 0) trace_ev(a.trace, kEvODone, i);
      return true;
    };
    for (int j = 0; j < ntiles && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&sm.s_full[sb], (j >> 1) & 1, abort, a.status, kTimeoutConsumer)) { ok = false; break; }
      tc_fence_after();
      if (threadIdx.x == 0) trace_ev(a.trace, kEvSReady, j);
      float sacc[RMAX];
      {
        uint32_t sr[kSParts][RMAX];
#pragma unroll
        for (int q = 0; q < kSParts; ++q) {
          if constexpr (RMAX == 8) tmem_ld8(tS + lane_base + sb * (kSParts * kN) + q * kN, sr[q]);
          else tmem_ld16(tS + lane_base + sb * (kSParts * kN) + q * kN, sr[q]);
        }
        tmem_ld_wait();
#pragma unroll
        for (int n = 0; n < RMAX; ++n) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < kSParts; ++q) v += __uint_as_float(sr[q][n]);
          sacc[n] = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_empty[sb]);
      const int tokpos = (tile0 + j) * kTileTok + 32 * warp + lane;
      float s[RMAX];
      float tmax[RMAX];
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        const int t = n / G;
        const int qpos = q_first + t;
        const bool vis = n < R && tokpos <= qpos && tokpos >= kv_begin &&
                         (a.window <= 0 || qpos - tokpos < a.window);
        s[n] = vis ? sacc[n] * scale_log2 : -INFINITY;
        tmax[n] = warp_max(s[n]);
      }
      if (lane == 0) {
#pragma unroll
        for (int n = 0; n < RMAX; ++n) sm.red[warp][n] = tmax[n];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      float mnew[RMAX], alpha[RMAX];
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        const float mt = fmaxf(fmaxf(sm.red[0][n], sm.red[1][n]), fmaxf(sm.red[2][n], sm.red[3][n]));
        const float mo = sm.row_m[n];
        mnew[n] = fmaxf(mo, mt);
        alpha[n] = (mnew[n] == -INFINITY) ? 1.f : exp2f(mo - mnew[n]);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
      for (int n = 0; n < RMAX; ++n)
        if (threadIdx.x == n) sm.row_m[n] = mnew[n];
      // P (f16) into the B operand: row n, token k -> slab k / 64, SW128 K-major
      uint8_t* pbuf = sp + sb * (2 * kN * 128);
      const int k = 32 * warp + lane;
#pragma unroll
      for (int n = 0; n < kN; ++n) {
        float p = 0.f;
        if (n < RMAX) {
          p = (s[n] == -INFINITY) ? 0.f : exp2f(s[n] - mnew[n]);
          lpart[n] = lpart[n] * alpha[n] + p;
        }
        *reinterpret_cast<__half*>(pbuf + (k >> 6) * (kN * 128) + sw128_off16(n, k & 63)) = __float2half_rn(p);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[sb]);
      if (threadIdx.x == 0) trace_ev(a.trace, kEvPReady, j);
      if (j > 0) ok = consume_o(j - 1);
#pragma unroll
      for (int n = 0; n < RMAX; ++n) alpha_prev[n] = alpha[n];
    }
    if (ok) ok = consume_o(ntiles - 1);
    // ---- epilogue: row sums, normalise, store
    float l[RMAX];
#pragma unroll
    for (int n = 0; n < RMAX; ++n) l[n] = warp_sum(lpart[n]);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (lane == 0) {
#pragma unroll
      for (int n = 0; n < RMAX; ++n) sm.red[warp][n] = l[n];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
    for (int n = 0; n < RMAX; ++n) l[n] = sm.red[0][n] + sm.red[1][n] + sm.red[2][n] + sm.red[3][n];
    if (ok) {
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        if (n >= R) break;
        const int t = n / G, g = n % G;
        const float inv = l[n] > 0.f ? a.v_scale / l[n] : 0.f;
        if (a.num_splits == 1) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) +
                             ((static_cast<size_t>(b) * a.n_q + t) * a.Hq + h * G + g) * D;
#pragma unroll
          for (int mb = 0; mb < MB; ++mb) o[mb * 128 + 32 * warp + lane] = __float2bfloat16(acc[mb][n] * inv);
        } else {
          float* o = a.o_part + (part_out * RMAX + n) * D;
#pragma unroll
          for (int mb = 0; mb < MB; ++mb) o[mb * 128 + 32 * warp + lane] = acc[mb][n] * inv;
          if (warp == 0 && lane == 0)
            a.lse_part[part_out * RMAX + n] = l[n] > 0.f ? sm.row_m[n] + log2f(l[n]) : -INFINITY;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_ev(a.trace, kEvEnd, 0);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}


// =====================================================================================================================
// E4M3-operand variant (kind::f8f6f4, K = 32 per UMMA).  A UMMA instruction costs about the same whatever its N, so a
// decode tile with 2..16 query rows is bound by the instruction count: K = 32 halves it for both QK and PV.  K/V are
// dequantized to E4M3 (E2M1 x block scale rounded once, the kv4mla "fp8" mode), Q gets a per-row scale, P is stored
// as E4M3 x 256.  V slabs are one full 128-dim M block (128 B of E4M3 per token row).
template <int FMT, int D>
__device__ __host__ __forceinline__ constexpr int ring_f8() { return part_bytes<FMT, D>() <= 20 * 1024 ? 6 : 4; }
// Optional decode variant: with <= 2 query rows P V runs on the CUDA cores (CC = true): the V slab ring is replaced
// by a 24 KB area (P in fp32, the cross-thread O reduction, the final O) and the freed shared memory goes to raw
// staging.  Measured on B200 (32 x 32k tokens, head_dim 512, NVFP4): 3.36 ms against 3.18 ms for the tensor-core
// P V (the FFMA + conversion stream of the 8 PV warps is issue-limited), so it is off.
constexpr bool kCudaCorePv = false;
constexpr int kCcBytes = 24576;
template <int FMT, int D, bool CC>
__device__ __host__ __forceinline__ constexpr int ring_bytes_f8() { return CC ? kCcBytes : ring_f8<FMT, D>() * 16384; }
template <int FMT, int D, bool CC>
__device__ __host__ __forceinline__ constexpr int raw_stages_f8() {
  return (229376 - ring_bytes_f8<FMT, D, CC>() - (D / 128) * 2048 - 4096 - kF4TabBytes) / part_bytes<FMT, D>() > 8
             ? 8
         : (229376 - ring_bytes_f8<FMT, D, CC>() - (D / 128) * 2048 - 4096 - kF4TabBytes) / part_bytes<FMT, D>() < 4
             ? 4
             : (229376 - ring_bytes_f8<FMT, D, CC>() - (D / 128) * 2048 - 4096 - kF4TabBytes) / part_bytes<FMT, D>();
}

__device__ __forceinline__ uint32_t pack_e4m3x4(uint32_t h01, uint32_t h23) {
  return static_cast<uint32_t>(f16x2_to_e4m3x2(h01)) | (static_cast<uint32_t>(f16x2_to_e4m3x2(h23)) << 16);
}

// 64 values of one token row (dims [d0, d0 + 64)) as E4M3 bytes packed four per word: 16 words.
template <int FMT, int D>
__device__ __forceinline__ void dequant_e4m3_64(const uint8_t* part, int r, int d0, uint32_t* out,
                                                const uint2* f4tab) {
  if constexpr (FMT == kKvNvfp4) {
    // one 8-byte shared-memory table per 16-value block (scale byte -> the eight E4M3 products), then byte permutes
    constexpr int RB = D / 2, NCH = (RB / 16) < 8 ? (RB / 16) : 8;
    const int c = d0 / 64;
    const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(part + 64 * RB + r * (D / 16) + c * 4);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint4 in = *reinterpret_cast<const uint4*>(part + r * RB + pool_chunk_pos(2 * c + half, r, NCH) * 16);
      const uint32_t w[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint2 tab = f4tab[(sc4 >> (8 * (2 * half + (q >> 1)))) & 0xFFu];
        const uint2 e = f4_decode8(w[q], tab);
        out[8 * half + 2 * q] = e.x;
        out[8 * half + 2 * q + 1] = e.y;
      }
    }
  } else if constexpr (FMT == kKvFp8) {
    constexpr int RB = D, NCH = 8;
    const uint8_t* row = part + r * RB;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 in = *reinterpret_cast<const uint4*>(row + pool_chunk_pos(d0 / 16 + k, r, NCH) * 16);
      out[4 * k] = in.x; out[4 * k + 1] = in.y; out[4 * k + 2] = in.z; out[4 * k + 3] = in.w;
    }
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t h[16];
      dequant_32<FMT, D>(part, r, d0 / 64, half, h);
#pragma unroll
      for (int i = 0; i < 8; ++i) out[8 * half + i] = pack_e4m3x4(h[2 * i], h[2 * i + 1]);
    }
  }
}

// E4M3 kernel roles: warps 0-3 softmax, 4-11 K dequant, 12-19 V dequant, 20 producer, 21 QK issuer, 22 PV issuer,
// 23 idle
// (six full warpgroups so setmaxnreg can move registers: softmax 160, dequant 72, producer/issuer 32 per thread;
// 128 x 160 + 512 x 72 + 128 x 32 = 61440 = 768 threads x 80 at launch).
constexpr int kThreadsF8 = 768;
constexpr int kProducerWarpF8 = 20;
constexpr int kMmaWarpF8 = 21;
constexpr int kPvWarpF8 = 22;

// TMEM rows (columns) [0, RMAX) of this thread's lane.
template <int RMAX>
__device__ __forceinline__ void tmem_ld_rows(uint32_t taddr, uint32_t* r) {
  if constexpr (RMAX == 2) tmem_ld2(taddr, r);
  else if constexpr (RMAX == 4) tmem_ld4(taddr, r);
  else if constexpr (RMAX == 8) tmem_ld8(taddr, r);
  else tmem_ld16(taddr, r);
}

template <int FMT, int D, int RMAX>
__global__ void __launch_bounds__(kThreadsF8, 1) gqa_decode_f8_kernel(const GqaDecodeArgs a) {
  constexpr int NQS = D / 128;                     // 128-dim slabs (Q rows, V M blocks)
  constexpr int PB = part_bytes<FMT, D>();
  constexpr bool kCc = kCudaCorePv && RMAX <= 2;   // P V on the CUDA cores (decode)
  constexpr int NST = raw_stages_f8<FMT, D, kCc>();
  // K and V parts go through separate raw rings (page slots [0, NSTK) and [NSTK, NST)): each ring is consumed in
  // order by one warp group, so no mbarrier is ever waited on more than one phase ahead.
  constexpr int NSTK = NST / 2, NSTV = NST - NSTK;
  static_assert(NSTK >= 2 && NSTV >= 2, "each raw ring holds at least one part (two pages)");
  constexpr int RING = kCc ? D / 128 : ring_f8<FMT, D>();
  constexpr int MB = D / 128;
  constexpr int kOCols = MB * kN;
  constexpr float kPScale = 256.f;
  static_assert(RMAX <= kN, "rows");
  static_assert(RING >= MB, "all V blocks of a tile are multiplied together");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                   // RING x 16 KB (V slabs, E4M3) or the CC area
  uint8_t* sq = ring + ring_bytes_f8<FMT, D, kCc>();      // NQS x 2 KB (Q, E4M3)
  // CC area: P fp32 [2 bufs][2 rows][128] + alpha [2][2] | O partials [TG][2][D] | final O [2][D]
  float* cc_p = reinterpret_cast<float*>(ring);
  float* cc_alpha = cc_p + 2 * 2 * 128;
  float* cc_red = cc_p + 1024;
  float* cc_o = cc_red + 2 * 2048;
  uint8_t* sp = sq + NQS * kN * 128;                      // 2 x 2 KB (P, E4M3)
  uint8_t* raw = sp + 2 * kN * 128;                       // NST x PB
  Smem& sm = *reinterpret_cast<Smem*>(raw + NST * PB);

  const int G = a.Hq / a.Hk;
  const int R = a.n_q * G;
  const int work = blockIdx.x;
  const int split = work % a.num_splits;
  const int bh = work / a.num_splits;
  const int h = bh % a.Hk;
  const int b = bh / a.Hk;
  const int kv_len = a.kv_len[b];
  const int q_first = kv_len - a.n_q;
  const int kv_begin = a.window > 0 ? max(0, q_first - a.window + 1) : 0;
  const int tile0 = kv_begin / kTileTok + split * a.tiles_per_split;
  const int tile_end = min((kv_len + kTileTok - 1) / kTileTok, kv_begin / kTileTok + (split + 1) * a.tiles_per_split);
  const int ntiles = tile_end - tile0;
  const size_t part_out = (static_cast<size_t>(bh) * a.num_splits + split);
  if (ntiles <= 0) {
    if (a.num_splits > 1 && threadIdx.x < RMAX) a.lse_part[part_out * RMAX + threadIdx.x] = -INFINITY;
    return;
  }
  const int first_page = kv_begin / a.page;
  const int n_pages = (kv_len + a.page - 1) / a.page;
  const int* pt = a.page_table + static_cast<size_t>(a.req_idx ? a.req_idx[b] : b) * a.pt_stride;
  const int warp = warp_id(), lane = lane_id();
  const __nv_bfloat16* qg = reinterpret_cast<const __nv_bfloat16*>(a.q);
  auto qrow = [&](int row) {
    const int t = row / G, g = row % G;
    return qg + ((static_cast<size_t>(b) * a.n_q + t) * a.Hq + h * G + g) * D;
  };

  // ---- Q -> per-row scale, E4M3 slabs (rows >= R zero)
  for (int row = warp; row < kN; row += kThreadsF8 / 32) {
    float amax = 0.f;
    if (row < R) {
      const __nv_bfloat16* qr = qrow(row);
      for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(__bfloat162float(qr[d])));
    }
    amax = warp_max(amax);
    if (lane == 0) sm.q_scale[row] = fmaxf(amax, 1e-20f) / 448.f;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) { mbar_init(&sm.raw_full[i], 1); mbar_init(&sm.raw_empty[i], kDequantWarps); }
    for (int i = 0; i < RING; ++i) { mbar_init(&sm.ring_full[i], kDequantWarps); mbar_init(&sm.ring_empty[i], 1); }
    mbar_init(&sm.k_full, kDequantWarps);
    mbar_init(&sm.k_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kf[i], kDequantWarps); mbar_init(&sm.ke[i], 1); mbar_init(&sm.pe[i], kDequantWarps);
    }
    mbar_init(&sm.od, kDequantWarps);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1); mbar_init(&sm.s_empty[i], kSoftmaxWarps);
      mbar_init(&sm.p_full[i], kSoftmaxWarps); mbar_init(&sm.o_full[i], 1); mbar_init(&sm.o_empty[i], kSoftmaxWarps);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  uint2* f4tab = reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(&sm) + ((sizeof(Smem) + 15) & ~size_t(15)));
  if constexpr (FMT == kKvNvfp4) f4_table_fill(f4tab);
  if (warp == kMmaWarpF8) { tmem_alloc(&sm.tmem_base, kTmemCols); tmem_relinquish(); }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kN * NQS * 8; idx += kThreadsF8) {
    const int row = idx / (NQS * 8), rem = idx % (NQS * 8), c = rem / 8, ch = rem % 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < R) {
      const float inv = 1.f / sm.q_scale[row];
      const uint4* src = reinterpret_cast<const uint4*>(qrow(row) + c * 128 + ch * 16);
      const uint4 i0 = src[0], i1 = src[1];
      const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&i0);
      const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&i1);
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat16* e = k < 2 ? e0 : e1;
        const int o = (k & 1) * 4;
        w[k] = static_cast<uint32_t>(f32x2_to_e4m3x2(__bfloat162float(e[o]) * inv, __bfloat162float(e[o + 1]) * inv)) |
               (static_cast<uint32_t>(f32x2_to_e4m3x2(__bfloat162float(e[o + 2]) * inv,
                                                       __bfloat162float(e[o + 3]) * inv)) << 16);
      }
      v = make_uint4(w[0], w[1], w[2], w[3]);
    }
    *reinterpret_cast<uint4*>(sq + c * (kN * 128) + sw128_chunk(row, ch)) = v;
  }
  for (int idx = threadIdx.x; idx < 2 * kN * 128 / 16; idx += kThreadsF8)
    reinterpret_cast<uint4*>(sp)[idx] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 128;
  const uint32_t tK = tmem + kTmemK;   // two buffers of D/4 columns (four E4M3 per column)
  static_assert(kTmemK + 2 * (D / 4) <= kTmemCols, "TMEM: double-buffered K");
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) trace_ev(a.trace, kEvStart, 0);

  auto parts_before = [&](int j) { return min(j, ntiles) + max(0, j - 1); };
  auto part_index = [&](int j, int which) { return parts_before(j) + ((which == 1 && j < ntiles) ? 1 : 0); };

  // register split (per thread): softmax kSmRegs, dequant 72, producer / issuers kIssRegs; 128 kSmRegs + 512 x 72 +
  // 128 kIssRegs = 61440 = the 768 x 80 the block is launched with.  The batched MMA issue needs more than 32.
  constexpr uint32_t kSmRegs = RMAX > 8 ? 160 : 136, kIssRegs = RMAX > 8 ? 32 : 56;
  static_assert(128 * kSmRegs + 512 * 72 + 128 * kIssRegs == kThreadsF8 * 80, "register split");
  if (warp < kSoftmaxWarps) {
    regs_inc<kSmRegs>();
    const float base_scale = a.sm_scale * a.k_scale * 1.4426950408889634f;
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    float acc[MB][RMAX];
    float lpart[RMAX];
    float alpha_prev[RMAX];
    float rs[RMAX];
#pragma unroll
    for (int n = 0; n < RMAX; ++n) {
      lpart[n] = 0.f;
      alpha_prev[n] = 1.f;
      rs[n] = base_scale * sm.q_scale[n];
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) acc[mb][n] = 0.f;
    }
    if (threadIdx.x < kN) sm.row_m[threadIdx.x] = -INFINITY;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    bool ok = true;
    auto consume_o = [&](int i) -> bool {
      const int sb = i & 1;
      if (!mbar_wait(&sm.o_full[sb], (i >> 1) & 1, abort, a.status, kTimeoutConsumer)) return false;
      tc_fence_after();
      uint32_t r[MB][RMAX];
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) tmem_ld_rows<RMAX>(tO + lane_base + sb * kOCols + mb * kN, r[mb]);
      tmem_ld_wait();
#pragma unroll
      for (int mb = 0; mb < MB; ++mb) {
#pragma unroll
        for (int n = 0; n < RMAX; ++n) acc[mb][n] = acc[mb][n] * alpha_prev[n] + __uint_as_float(r[mb][n]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_empty[sb]);
      if (threadIdx.x == 0) trace_ev(a.trace, kEvODone, i);
      return true;
    };
    for (int j = 0; j < ntiles && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&sm.s_full[sb], (j >> 1) & 1, abort, a.status, kTimeoutConsumer)) { ok = false; break; }
      tc_fence_after();
      if (threadIdx.x == 0) trace_ev(a.trace, kEvSReady, j);
      float sacc[RMAX];
      {
        uint32_t sr[kSParts][RMAX];
#pragma unroll
        for (int q = 0; q < kSParts; ++q) tmem_ld_rows<RMAX>(tS + lane_base + sb * (kSParts * kN) + q * kN, sr[q]);
        tmem_ld_wait();
#pragma unroll
        for (int n = 0; n < RMAX; ++n) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < kSParts; ++q) v += __uint_as_float(sr[q][n]);
          sacc[n] = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_empty[sb]);
      const int tokpos = (tile0 + j) * kTileTok + 32 * warp + lane;
      float s[RMAX];
      float tmax[RMAX];
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        const int t = n / G;
        const int qpos = q_first + t;
        const bool vis = n < R && tokpos <= qpos && tokpos >= kv_begin && (a.window <= 0 || qpos - tokpos < a.window);
        s[n] = vis ? sacc[n] * rs[n] : -INFINITY;
        tmax[n] = warp_max(s[n]);
      }
      if (lane == 0) {
#pragma unroll
        for (int n = 0; n < RMAX; ++n) sm.red[warp][n] = tmax[n];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      float mnew[RMAX], alpha[RMAX];
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        const float mt = fmaxf(fmaxf(sm.red[0][n], sm.red[1][n]), fmaxf(sm.red[2][n], sm.red[3][n]));
        const float mo = sm.row_m[n];
        mnew[n] = fmaxf(mo, mt);
        alpha[n] = (mnew[n] == -INFINITY) ? 1.f : exp2f(mo - mnew[n]);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
      for (int n = 0; n < RMAX; ++n)
        if (threadIdx.x == n) sm.row_m[n] = mnew[n];
      if constexpr (kCc) {
        // P (fp32) and the rescale factor of the running O for the PV warps; buffer sb last held tile j - 2
        if (j >= 2 && !mbar_wait(&sm.pe[sb], ((j >> 1) - 1) & 1, abort, a.status, kTimeoutConsumer)) {
          ok = false;
          break;
        }
        float* pp = cc_p + sb * 256;
        const int k = 32 * warp + lane;
#pragma unroll
        for (int n = 0; n < RMAX; ++n) {
          const float p = (s[n] == -INFINITY) ? 0.f : exp2f(s[n] - mnew[n]);
          lpart[n] = lpart[n] * alpha[n] + p;
          pp[n * 128 + k] = p;
        }
        if (threadIdx.x < RMAX) cc_alpha[sb * 2 + threadIdx.x] = threadIdx.x == 0 ? alpha[0] : alpha[RMAX - 1];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[sb]);
        if (threadIdx.x == 0) trace_ev(a.trace, kEvPReady, j);
        continue;
      }
      // P (E4M3 x 256) into the B operand: row n, token k, SW128 K-major (one 128-token slab)
      uint8_t* pbuf = sp + sb * (kN * 128);
      const int k = 32 * warp + lane;
#pragma unroll
      for (int n = 0; n < RMAX; n += 2) {
        float p0 = 0.f, p1 = 0.f;
        p0 = (s[n] == -INFINITY) ? 0.f : exp2f(s[n] - mnew[n]);
        lpart[n] = lpart[n] * alpha[n] + p0;
        if (n + 1 < RMAX) {
          p1 = (s[n + 1] == -INFINITY) ? 0.f : exp2f(s[n + 1] - mnew[n + 1]);
          lpart[n + 1] = lpart[n + 1] * alpha[n + 1] + p1;
        }
        const uint16_t e = f32x2_to_e4m3x2(p0 * kPScale, p1 * kPScale);
        pbuf[n * 128 + (((k >> 4) ^ (n & 7)) << 4) + (k & 15)] = static_cast<uint8_t>(e & 0xFF);
        pbuf[(n + 1) * 128 + (((k >> 4) ^ ((n + 1) & 7)) << 4) + (k & 15)] = static_cast<uint8_t>(e >> 8);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[sb]);
      if (threadIdx.x == 0) trace_ev(a.trace, kEvPReady, j);
      if (j > 0) ok = consume_o(j - 1);
#pragma unroll
      for (int n = 0; n < RMAX; ++n) alpha_prev[n] = alpha[n];
    }
    if constexpr (!kCc) {
      if (ok) ok = consume_o(ntiles - 1);
    } else {
      if (ok) ok = mbar_wait(&sm.od, 0, abort, a.status, kTimeoutConsumer);   // final O of the PV warps
    }
    float l[RMAX];
#pragma unroll
    for (int n = 0; n < RMAX; ++n) l[n] = warp_sum(lpart[n]);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (lane == 0) {
#pragma unroll
      for (int n = 0; n < RMAX; ++n) sm.red[warp][n] = l[n];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
    for (int n = 0; n < RMAX; ++n) l[n] = sm.red[0][n] + sm.red[1][n] + sm.red[2][n] + sm.red[3][n];
    if (ok) {
#pragma unroll
      for (int n = 0; n < RMAX; ++n) {
        if (n >= R) break;
        const int t = n / G, g = n % G;
        const float inv = l[n] > 0.f ? a.v_scale / (l[n] * (kCc ? 1.f : kPScale)) : 0.f;
        auto oval = [&](int mb) {
          if constexpr (kCc) return cc_o[n * D + mb * 128 + 32 * warp + lane];
          else return acc[mb][n];
        };
        if (a.num_splits == 1) {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) +
                             ((static_cast<size_t>(b) * a.n_q + t) * a.Hq + h * G + g) * D;
#pragma unroll
          for (int mb = 0; mb < MB; ++mb) o[mb * 128 + 32 * warp + lane] = __float2bfloat16(oval(mb) * inv);
        } else {
          float* o = a.o_part + (part_out * RMAX + n) * D;
#pragma unroll
          for (int mb = 0; mb < MB; ++mb) o[mb * 128 + 32 * warp + lane] = oval(mb) * inv;
          if (warp == 0 && lane == 0)
            a.lse_part[part_out * RMAX + n] = l[n] > 0.f ? sm.row_m[n] + log2f(l[n]) : -INFINITY;
        }
      }
    }
    } else if (warp < kSoftmaxWarps + kDequantWarps) {
    regs_dec<72>();
    // ---- K warps: K(j) -> TMEM (E4M3); thread = TMEM lane = token, warps dw and dw + 4 split the dims
    const int dw = warp - kSoftmaxWarps;
    const int kq = warp & 3, ktok = 32 * kq + lane, kpg = ktok / 64, kr = ktok % 64;
    const int kdim0 = (dw >> 2) * (D / 2);
    const uint32_t k_lane = static_cast<uint32_t>(32 * kq) << 16;
    for (int j = 0; j < ntiles; ++j) {
      const int seq0 = 2 * j, st0 = seq0 % NSTK, st1 = (seq0 + 1) % NSTK;
      if (!mbar_wait(&sm.raw_full[st0], (seq0 / NSTK) & 1, abort, a.status, kTimeoutConsumer)) break;
      if (!mbar_wait(&sm.raw_full[st1], ((seq0 + 1) / NSTK) & 1, abort, a.status, kTimeoutConsumer)) break;
      const int kb = j & 1;
      if (!mbar_wait(&sm.ke[kb], ((j >> 1) & 1) ^ 1, abort, a.status, kTimeoutConsumer)) break;
      tc_fence_after();
      if (dw == 0 && lane == 0) trace_ev(a.trace, kEvKDeqStart, j);
      const int st = kpg ? st1 : st0;
      const bool valid = sm.raw_valid[st] != 0;
      const uint8_t* part = raw + st * PB;
#pragma unroll 1
      for (int d0 = kdim0; d0 < kdim0 + D / 2; d0 += 64) {
        uint32_t v[16];
        if (valid) dequant_e4m3_64<FMT, D>(part, kr, d0, v, f4tab);
        else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0;
        }
        tmem_st16(tK + kb * (D / 4) + k_lane + d0 / 4, v);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.kf[kb]);
        mbar_arrive(&sm.raw_empty[st0]);
        mbar_arrive(&sm.raw_empty[st1]);
        if (dw == 0) trace_ev(a.trace, kEvKDeqEnd, j);
      }
    }
  } else if (kCc && warp < kSoftmaxWarps + 2 * kDequantWarps) {
    regs_dec<72>();
    // ---- PV warps (<= 2 query rows): O += P V on the CUDA cores straight from the raw pages (no E4M3 slabs, no
    // PV MMAs).  Thread = (8-dim group dg, token group tg): it accumulates 2 rows x 8 dims over its tokens.
    constexpr int DG = D / 8, TG = 256 / DG, TPT = 128 / TG;
    const int tv = (warp - kSoftmaxWarps - kDequantWarps) * 32 + lane;
    const int dg = tv % DG, tg = tv / DG;
    float acc0[8], acc1[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc0[e] = acc1[e] = 0.f;
    bool okv = true;
    for (int i = 0; i < ntiles; ++i) {
      const int seq0 = 2 * i, st0 = NSTK + seq0 % NSTV, st1 = NSTK + (seq0 + 1) % NSTV;
      const int sb = i & 1;
      if (!(okv = mbar_wait(&sm.raw_full[st0], (seq0 / NSTV) & 1, abort, a.status, kTimeoutConsumer))) break;
      if (!(okv = mbar_wait(&sm.raw_full[st1], ((seq0 + 1) / NSTV) & 1, abort, a.status, kTimeoutConsumer))) break;
      if (!(okv = mbar_wait(&sm.p_full[sb], (i >> 1) & 1, abort, a.status, kTimeoutConsumer))) break;
      if (tv == 0) trace_ev(a.trace, kEvVDeqStart, i);
      const float al0 = cc_alpha[sb * 2], al1 = cc_alpha[sb * 2 + 1];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc0[e] *= al0;
        acc1[e] *= al1;
      }
      // this thread's TPT consecutive tokens lie in one page; masked tokens carry P = 0 (finite data, no branch)
      const int tfirst = tg * TPT;
      const int st = (tfirst >> 6) ? st1 : st0;
      if (sm.raw_valid[st]) {
        const float* pp0 = cc_p + sb * 256 + tfirst;
        const float* pp1 = pp0 + 128;
        const uint8_t* part = raw + st * PB;
#pragma unroll 1
        for (int u0 = 0; u0 < TPT; u0 += 4) {
          const float4 P0 = *reinterpret_cast<const float4*>(pp0 + u0);
          const float4 P1 = *reinterpret_cast<const float4*>(pp1 + u0);
          const float p0s[4] = {P0.x, P0.y, P0.z, P0.w}, p1s[4] = {P1.x, P1.y, P1.z, P1.w};
          if constexpr (FMT == kKvNvfp4) {
            constexpr int RB = D / 2, NCH = (RB / 16) < 8 ? (RB / 16) : 8;
            uint32_t w[4];
            uint32_t sbyte[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {                       // all loads first: latency overlaps
              const int r = (tfirst + u0 + q) & 63;
              w[q] = *reinterpret_cast<const uint32_t*>(part + r * RB + pool_chunk_pos(dg >> 2, r, NCH) * 16 +
                                                        (dg & 3) * 4);
              sbyte[q] = part[64 * RB + r * (D / 16) + (dg >> 1)];
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float sc = e4m3_to_float(static_cast<uint8_t>(sbyte[q]));
              const float c0 = p0s[q] * sc, c1 = p1s[q] * sc;
              uint32_t hh[4];
              e2m1x8_to_f16x2x4(w[q], hh);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hh[e]));
                acc0[2 * e] = fmaf(c0, f.x, acc0[2 * e]);
                acc0[2 * e + 1] = fmaf(c0, f.y, acc0[2 * e + 1]);
                acc1[2 * e] = fmaf(c1, f.x, acc1[2 * e]);
                acc1[2 * e + 1] = fmaf(c1, f.y, acc1[2 * e + 1]);
              }
            }
          } else {
            uint2 w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int r = (tfirst + u0 + q) & 63;
              w[q] = *reinterpret_cast<const uint2*>(part + r * D + pool_chunk_pos(dg >> 1, r, 8) * 16 + (dg & 1) * 8);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t ww[2] = {w[q].x, w[q].y};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint32_t hq = e4m3x2_to_f16x2(static_cast<uint16_t>(ww[e >> 1] >> (16 * (e & 1))));
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hq));
                acc0[2 * e] = fmaf(p0s[q], f.x, acc0[2 * e]);
                acc0[2 * e + 1] = fmaf(p0s[q], f.y, acc0[2 * e + 1]);
                acc1[2 * e] = fmaf(p1s[q], f.x, acc1[2 * e]);
                acc1[2 * e + 1] = fmaf(p1s[q], f.y, acc1[2 * e + 1]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.raw_empty[st0]);
        mbar_arrive(&sm.raw_empty[st1]);
        mbar_arrive(&sm.pe[sb]);
      }
      if (tv == 0) trace_ev(a.trace, kEvVDeqEnd, i);
    }
    // reduce the token groups: partials to smem, then each thread sums a slice of the 2 x D outputs
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      cc_red[(tg * 2 + 0) * D + 8 * dg + e] = acc0[e];
      cc_red[(tg * 2 + 1) * D + 8 * dg + e] = acc1[e];
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    for (int idx = tv; idx < 2 * D; idx += 256) {
      const int rr = idx / D, d = idx % D;
      float sum = 0.f;
#pragma unroll
      for (int g2 = 0; g2 < TG; ++g2) sum += cc_red[(g2 * 2 + rr) * D + d];
      cc_o[idx] = sum;
    }
    __syncwarp();
    if (okv && lane == 0) mbar_arrive(&sm.od);
  } else if (warp < kSoftmaxWarps + 2 * kDequantWarps) {
    regs_dec<72>();
    // ---- V warps: V(i) -> ring, one 128-dim E4M3 slab per M block; warp covers 16 tokens x two 64-dim halves
    const int dw = warp - kSoftmaxWarps - kDequantWarps;
    const int vtok = 16 * dw + (lane & 7) + 8 * (lane >> 4);
    const int vhalf = (lane >> 3) & 1;
    const int vpg = vtok / 64, vr = vtok % 64;
    for (int i = 0; i < ntiles; ++i) {
      const int seq0 = 2 * i, st0 = NSTK + seq0 % NSTV, st1 = NSTK + (seq0 + 1) % NSTV;
      if (!mbar_wait(&sm.raw_full[st0], (seq0 / NSTV) & 1, abort, a.status, kTimeoutConsumer)) break;
      if (!mbar_wait(&sm.raw_full[st1], ((seq0 + 1) / NSTV) & 1, abort, a.status, kTimeoutConsumer)) break;
      const int st = vpg ? st1 : st0;
      const bool valid = sm.raw_valid[st] != 0;
      if (dw == 0 && lane == 0) trace_ev(a.trace, kEvVDeqStart, i);
      bool ok = true;
      // every slab of the tile is written, then one proxy fence publishes them all (PV waits for the whole tile)
      for (int mb = 0; mb < MB; ++mb) {
        const int seq = MB * i + mb, buf = seq % RING;
        if (!(ok = mbar_wait(&sm.ring_empty[buf], ((seq / RING) & 1) ^ 1, abort, a.status, kTimeoutConsumer)))
          break;
        if (dw == 0 && lane == 0 && (mb == 1 || mb == 2))   // slab timings (diagnostic timeline)
          trace_ev(a.trace, mb == 1 ? kEvProdK : kEvProdV, i);
        uint32_t o[16];
        if (valid) dequant_e4m3_64<FMT, D>(raw + st * PB, vr, 128 * mb + 64 * vhalf, o, f4tab);
        else {
#pragma unroll
          for (int k = 0; k < 16; ++k) o[k] = 0;
        }
        uint8_t* slab = ring + buf * kSlabBytes;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(slab + sw128_chunk(vtok, vhalf * 4 + q)) =
              make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
      if (!ok) break;
      if (dw == 0 && lane == 0) trace_ev(a.trace, kEvKRaw, i);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0)
        for (int mb = 0; mb < MB; ++mb) mbar_arrive(&sm.ring_full[(MB * i + mb) % RING]);
      __syncwarp();
      if (lane == 0) { mbar_arrive(&sm.raw_empty[st0]); mbar_arrive(&sm.raw_empty[st1]); }
      if (dw == 0 && lane == 0) trace_ev(a.trace, kEvVDeqEnd, i);
    }
  } else {
    regs_dec<kIssRegs>();
    if (warp == kProducerWarpF8) {
    if (lane == 0) {
      const uint8_t* pool = a.pool;
      auto prefetch_part = [&](int p) {
        if (p >= 2 * ntiles) return;
        int tile, which;
        if (p == 0) { tile = 0; which = 0; }
        else if (p & 1) { const int j = (p + 1) / 2; if (j < ntiles) { tile = j; which = 0; } else { tile = ntiles - 1; which = 1; } }
        else { tile = p / 2 - 1; which = 1; }
        for (int pg = 0; pg < 2; ++pg) {
          const int pidx = (tile0 + tile) * 2 + pg;
          const int phys = (pidx >= first_page && pidx < n_pages) ? pt[pidx] : -1;
          if (phys >= 0) prefetch_l2(pool + (static_cast<size_t>(phys) * a.Hk + h) * (2 * PB) + which * PB, PB);
        }
      };
      for (int p = 0; p < kPrefetchParts; ++p) prefetch_part(p);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j <= ntiles && !*abort; ++j) {
        for (int which = 0; which < 2; ++which) {
          const int tile = which == 0 ? j : j - 1;
          if (tile < 0 || tile >= ntiles) continue;
          const int pidx0 = part_index(j, which);
          prefetch_part(pidx0 + kPrefetchParts);
          for (int pg = 0; pg < 2; ++pg) {
            const int rs = 2 * tile + pg;                       // sequence within this part's ring
            const int nst = which == 0 ? NSTK : NSTV;
            const int st = (which == 0 ? 0 : NSTK) + rs % nst;
            if (*abort) break;
            if (!mbar_wait(&sm.raw_empty[st], ((rs / nst) & 1) ^ 1, abort, a.status, kTimeoutProducer)) break;
            (which == 0 ? issued_k : issued_v) = rs + 1;
            const int pidx = (tile0 + tile) * 2 + pg;
            const int phys = (pidx >= first_page && pidx < n_pages) ? pt[pidx] : -1;
            if (phys >= 0) {
              sm.raw_valid[st] = 1;
              mbar_expect_tx(&sm.raw_full[st], PB);
              bulk_g2s(raw + st * PB, pool + (static_cast<size_t>(phys) * a.Hk + h) * (2 * PB) + which * PB, PB,
                       &sm.raw_full[st]);
            } else {
              sm.raw_valid[st] = 0;
              mbar_arrive(&sm.raw_full[st]);
            }
          }
        }
      }
      for (int rs = max(0, issued_k - NSTK); rs < issued_k; ++rs)
        mbar_wait(&sm.raw_full[rs % NSTK], (rs / NSTK) & 1, nullptr, a.status, kTimeoutProducer);
      for (int rs = max(0, issued_v - NSTV); rs < issued_v; ++rs)
        mbar_wait(&sm.raw_full[NSTK + rs % NSTV], (rs / NSTV) & 1, nullptr, a.status, kTimeoutProducer);
    }
    } else if (warp == kMmaWarpF8) {
    // QK issuer: the whole warp runs the loop (descriptor arithmetic stays warp-uniform), one elected lane issues
    // the MMAs four per asm statement.  P V is issued by a second warp (kPvWarpF8).  (Issued one per statement by a
    // lone lane, consecutive tcgen05.mma measured ~250 cycles apart whatever their shape; batched from a converged
    // warp, ~65-80 cycles for these N = 16 MMAs.)
    const bool el = elect_one();
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.status, kTimeoutMma));
    };
    const uint32_t id_qk = idesc_dense(0, 0, 128, kN);                 // E4M3 x E4M3, K-major both
    const uint32_t q_addr = smem_u32(sq);
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      if (!wwait(&sm.s_empty[sb], ((j >> 1) & 1) ^ 1)) break;
      if (!wwait(&sm.kf[sb], (j >> 1) & 1)) break;
      tc_fence_after();
      if (el) trace_ev(a.trace, kEvQkStart, j);
      static_assert(kSParts == 4, "one batch of four MMAs = one K step into each partial accumulator");
#pragma unroll
      for (int s0 = 0; s0 < D / 32; s0 += 4) {
        uint32_t d4[4], a4[4];
        uint64_t b4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int s = s0 + k;
          d4[k] = tS + sb * (kSParts * kN) + k * kN;
          a4[k] = tK + sb * (D / 4) + 8 * s;
          b4[k] = desc_sw128(q_addr + (s >> 2) * (kN * 128) + (s & 3) * 32);
        }
        if (el) umma_f8_ts_x4(d4, a4, b4, id_qk, s0 > 0 ? 0xFu : 0u);
      }
      if (el) {
        umma_commit(&sm.s_full[sb]);
        umma_commit(&sm.ke[sb]);
        trace_ev(a.trace, kEvQkEnd, j);
      }
      __syncwarp();
    }
    } else if (warp == kPvWarpF8 && !kCc) {
    const bool el = elect_one();
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.status, kTimeoutMma));
    };
    const uint32_t id_pv = idesc_dense(0, 0, 128, kN) | (1u << 15);   // A (V^T) MN-major
    const uint32_t ring_addr = smem_u32(ring), p_addr = smem_u32(sp);
    for (int i = 0; i < ntiles; ++i) {
      const int sb = i & 1;
      if (!wwait(&sm.p_full[sb], (i >> 1) & 1)) break;
      if (!wwait(&sm.o_empty[sb], ((i >> 1) & 1) ^ 1)) break;
      if (el) trace_ev(a.trace, kEvPvStart, i);
      bool ok = true;
      for (int mb = 0; mb < MB && ok; ++mb) {
        const int seq = MB * i + mb;
        ok = wwait(&sm.ring_full[seq % RING], (seq / RING) & 1);
      }
      if (!ok) break;
      tc_fence_after();
      static_assert((4 * MB) % 4 == 0, "PV MMAs come in batches of four");
      uint32_t d4[4];
      uint64_t a4[4], b4[4];
      uint32_t mask = 0;
      int n4 = 0;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int mb = 0; mb < MB; ++mb) {
          const int buf = (MB * i + mb) % RING;
          d4[n4] = tO + sb * kOCols + mb * kN;
          a4[n4] = desc_mn_sw128(ring_addr + buf * kSlabBytes + kk * 4096, kSlabBytes);
          b4[n4] = desc_sw128(p_addr + sb * (kN * 128) + kk * 32);
          if (kk > 0) mask |= 1u << n4;
          if (++n4 == 4) {
            if (el) umma_f8_ss_x4(d4, a4, b4, id_pv, mask);
            n4 = 0;
            mask = 0;
          }
        }
      }
      if (el) {
        for (int mb = 0; mb < MB; ++mb) umma_commit(&sm.ring_empty[(MB * i + mb) % RING]);
        umma_commit(&sm.o_full[sb]);
        trace_ev(a.trace, kEvPvEnd, i);
      }
      __syncwarp();
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_ev(a.trace, kEvEnd, 0);
  if (warp == kMmaWarpF8) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge split partials: out = sum_s 2^(lse_s - lse_max) o_s / sum_s 2^(lse_s - lse_max).  One CTA per (b, kvh, row).
template <int RMAX>
__global__ void gqa_combine_kernel(const GqaDecodeArgs a) {
  const int G = a.Hq / a.Hk;
  const int n = blockIdx.x % RMAX;
  const int bh = blockIdx.x / RMAX;
  if (n >= a.n_q * G) return;
  const int h = bh % a.Hk, b = bh / a.Hk;
  const int t = n / G, g = n % G;
  const float* lse = a.lse_part + static_cast<size_t>(bh) * a.num_splits * RMAX;
  float m = -INFINITY;
  for (int s = 0; s < a.num_splits; ++s) m = fmaxf(m, lse[s * RMAX + n]);
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + ((static_cast<size_t>(b) * a.n_q + t) * a.Hq + h * G + g) * a.D;
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < a.num_splits; ++s) {
      const float ls = lse[s * RMAX + n];
      if (ls == -INFINITY) continue;
      const float w = exp2f(ls - m);
      num += w * a.o_part[((static_cast<size_t>(bh) * a.num_splits + s) * RMAX + n) * a.D + d];
      den += w;
    }
    o[d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

template <int FMT, int D, int RMAX>
cudaError_t launch_t(const GqaDecodeArgs& a, cudaStream_t s) {
  constexpr int PB = part_bytes<FMT, D>();
  constexpr int NST = raw_stages<FMT, D>();
  constexpr int RING = ring_slabs<FMT, D>();
  const int smem = 1024 + RING * kSlabBytes + (D / 64) * kN * 128 + 4 * kN * 128 + NST * PB + sizeof(Smem);
  static_assert(1024 + RING * kSlabBytes + (D / 64) * kN * 128 + 4 * kN * 128 + NST * PB + sizeof(Smem) <= 232448,
                "shared memory budget");
  bool launched = false;
  if constexpr (FMT != kKvBf16) {
    if (!a.exact) {
    constexpr bool CC = kCudaCorePv && RMAX <= 2;
    constexpr int NST8 = raw_stages_f8<FMT, D, CC>();
    constexpr int smem8 = 1024 + ring_bytes_f8<FMT, D, CC>() + (D / 128) * kN * 128 + 2 * kN * 128 + NST8 * PB +
                          ((sizeof(Smem) + 15) & ~size_t(15)) + kF4TabBytes;
    static_assert(smem8 <= 232448, "shared memory budget (E4M3 path)");
    auto kern8 = gqa_decode_f8_kernel<FMT, D, RMAX>;
    IOB_CUDA_CHECK(cudaFuncSetAttribute(kern8, cudaFuncAttributeMaxDynamicSharedMemorySize, smem8));
    kern8<<<a.B * a.Hk * a.num_splits, kThreadsF8, smem8, s>>>(a);
    launched = true;
    }
  }
  if (!launched) {
    auto kern = gqa_decode_kernel<FMT, D, RMAX>;
    IOB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<a.B * a.Hk * a.num_splits, kThreads, smem, s>>>(a);
  }
  IOB_CUDA_CHECK(cudaGetLastError());
  if (a.num_splits > 1) {
    gqa_combine_kernel<RMAX><<<a.B * a.Hk * RMAX, 128, 0, s>>>(a);
    IOB_CUDA_CHECK(cudaGetLastError());
  }
  return cudaSuccess;
}

template <int FMT, int D>
cudaError_t launch_r(const GqaDecodeArgs& a, cudaStream_t s) {
  const int R = a.n_q * (a.Hq / a.Hk);
  if (R <= 2 && FMT != kKvBf16 && !a.exact) return launch_t<FMT, D, 2>(a, s);
  if (R <= 8) return launch_t<FMT, D, 8>(a, s);
  if (R <= 16) return launch_t<FMT, D, 16>(a, s);
  return cudaErrorInvalidValue;
}

template <int FMT>
cudaError_t launch_d(const GqaDecodeArgs& a, cudaStream_t s) {
  switch (a.D) {
    case 128: return launch_r<FMT, 128>(a, s);
    case 256: return launch_r<FMT, 256>(a, s);
    case 512: return launch_r<FMT, 512>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t gqa_decode(const GqaDecodeArgs& a, cudaStream_t s) {
  if (a.B == 0) return cudaSuccess;
  if (a.page != 64 || a.Hq % a.Hk != 0 || a.num_splits < 1 || a.tiles_per_split < 1) return cudaErrorInvalidValue;
  switch (a.fmt) {
    case kKvNvfp4: return launch_d<kKvNvfp4>(a, s);
    case kKvFp8: return launch_d<kKvFp8>(a, s);
    case kKvBf16: return launch_d<kKvBf16>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace iob
