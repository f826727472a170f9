// GQA-packed extend (prefill) attention over a paged NVFP4 / FP8 KV pool, sm_100a.
//
// Capability of the reference's hd512 extend kernel (`attention/extend-gqa/extend_attention_gqa.py:38-184`: one
// program per (request, kv head, BLOCK_T query tokens), rows = G query heads x tokens, prefix from the paged pool,
// window rule q - kv < W).  Built for tcgen05 rather than transliterated:
//
//  * one CTA per (block of BT = 128 / G consecutive query tokens of one request, kv head, V half): its 128 rows
//    (token-major, row = t G + g) are the M of full-height UMMAs, so each K/V byte the block reads serves 128 query
//    rows.  (Prefill through the decode kernel serves 16 rows per read.)
//  * the KV range [kv_lo, kv_hi) of the block is walked in 128-token tiles (two 64-token pages) through a 2-deep
//    ring.  Eight dequant warps expand K (all D dims) and this CTA's V half (256 dims) from global memory -- NVFP4
//    raw bytes are held a tile ahead in registers, E4M3 rows go by cp.async -- into E4M3 128-byte-swizzled slabs.
//    The pool already stores each row's 16-byte chunks XOR-swizzled by the row index, so a pool chunk lands at the
//    same chunk position in the slab.  QK reads K as its K-major B operand; PV reads V as its MN-major B operand.
//  * TMEM: O half [128 x 256] fp32 at column 0, S [128 x 128] at 256, Q (E4M3 with a per-row scale; the A operand
//    of QK) at 384.  head_dim 512 runs as two CTAs per block, one per V half (O [128 x 512] does not fit next to S);
//    head_dim 256 as one.
//  * softmax: thread = row = TMEM lane.  Causal and window masks come from the row's position; base-2 running max
//    with a lazy rescale (O in TMEM is rescaled only when the max grows by more than 2^8); P = 2^(s - m) <= 256 in
//    E4M3 is the A operand of PV.
//  * one thread issues QK and PV in whichever order their inputs become ready.
//  * every wait is bounded (2 s): a wait past its limit records a status code and the CTA unwinds.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kXThreads = 512;
constexpr int kXTile = 128;                      // kv tokens per tile: N of QK, K extent of one PV
constexpr int kXBlk = kXTile * 128;              // one 128-dim E4M3 slab of a tile (16 KB)
constexpr int kXVBytes = 2 * kXBlk;              // the CTA's V tile: 256 dims
constexpr int kXPBytes = 128 * kXTile;           // P: 128 rows x 128 kv tokens, E4M3, SW128 K-major
constexpr uint32_t kXColO = 0, kXColS = 256, kXColQ = 384;
constexpr float kXTau = 8.f;                     // lazy-rescale threshold, log2 units
constexpr int kXSoftmaxWarps = 4, kXDequantWarps = 8, kXMmaWarp = 12;

struct ExtSmem {
  uint64_t tile_full[2];   // K and V tiles stored           (8 dequant-warp arrivals)
  uint64_t p_full[2];      // P written                      (4 softmax-warp arrivals)
  uint64_t pv_done[2];     // PV committed: frees the tile stage and its P buffer
  uint64_t s_full;         // QK committed
  uint64_t s_free;         // S loaded into registers        (4 softmax-warp arrivals)
  uint64_t q_ready, fin;
  uint32_t tmem_base;
  int abort;
};

template <int D>
__host__ __device__ constexpr int x_kbytes() { return (D / 128) * kXBlk; }
template <int D>
__host__ __device__ constexpr int x_np() { return D == 512 ? 1 : 2; }   // P buffers (shared-memory budget)
template <int D>
__host__ __device__ constexpr int x_smem_bytes() {
  return 1024 + 2 * (x_kbytes<D>() + kXVBytes) + x_np<D>() * kXPBytes + 256 * 8 + static_cast<int>(sizeof(ExtSmem));
}
static_assert(x_smem_bytes<512>() <= 232448, "shared memory budget (hd 512)");
static_assert(x_smem_bytes<256>() <= 232448, "shared memory budget (hd 256)");

__device__ __forceinline__ uint4 ldg16x(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void cp_async16x(void* smem, const void* g, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(g), "r"(src_bytes)
               : "memory");
}

// physical 16-byte chunk of logical chunk j of pool row r (the pool writers' swizzle, kv_swizzle_byte in kernels.h)
__device__ __forceinline__ int x_chunk_pos(int j, int r, int nch) { return (j & ~(nch - 1)) | ((j ^ r) & (nch - 1)); }

__device__ __forceinline__ float ex2x(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 8 bf16 (one 16-byte load) * inv -> 8 E4M3 bytes (two words, value 0 in the low byte)
__device__ __forceinline__ uint2 bf16x8_to_e4m3(const uint4& v, float inv) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float f[4];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t x = w[2 * h + k];
      f[2 * k] = __uint_as_float(x << 16) * inv;
      f[2 * k + 1] = __uint_as_float(x & 0xFFFF0000u) * inv;
    }
    o[h] = static_cast<uint32_t>(f32x2_to_e4m3x2(f[0], f[1])) | (static_cast<uint32_t>(f32x2_to_e4m3x2(f[2], f[3])) << 16);
  }
  return make_uint2(o[0], o[1]);
}

// f16x2 helpers for the softmax (value `lo` in the low half)
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint16_t h2_to_e4m3x2(uint32_t h2) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
  return r;
}

__device__ __forceinline__ float bf16x8_amax(const uint4& v, float m) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[k] << 16)), fabsf(__uint_as_float(w[k] & 0xFFFF0000u))));
  return m;
}

// Diagnostic timeline of CTA (0, 0, 0): clock64 per event and tile, [kXEvCount][64] for the first 64 tiles.
enum ExtTraceEv { kXEvQk, kXEvPv, kXEvSSeen, kXEvPReady, kXEvDeqStart, kXEvDeqEnd, kXEvStart, kXEvEnd, kXEvMax,
                  kXEvPFree, kXEvSLoaded, kXEvPWritten, kXEvCount };
__device__ __forceinline__ void x_trace(long long* tr, int ev, int j) {
  if (tr != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && j < 64) tr[ev * 64 + j] = clock64();
}

// NVFP4 raw bytes of one 64-value unit of a row: two 16-byte code chunks and four block-scale bytes.
struct F4Unit {
  uint4 c0, c1;
  uint32_t sc;
};

template <int FMT, int D>
__global__ void __launch_bounds__(kXThreads, 1) gqa_extend_kernel(const GqaExtendArgs a) {
  constexpr int KB = x_kbytes<D>(), NP = x_np<D>();
  constexpr int RB = FMT == kKvNvfp4 ? D / 2 : D;              // code (NVFP4) or value (E4M3) bytes per row
  constexpr int NCH = (RB / 16) < 8 ? (RB / 16) : 8;
  constexpr int PB = FMT == kKvNvfp4 ? 64 * (D / 2 + D / 16) : 64 * D;   // one (page, head, K|V) part
  constexpr int NKU = D / 128, NVU = 2;                        // 64-value units per dequant thread: K, V
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ktile = base;                                       // 2 x KB
  uint8_t* vtile = ktile + 2 * KB;                             // 2 x 32 KB
  uint8_t* sp = vtile + 2 * kXVBytes;                          // NP x 16 KB
  uint2* f4tab = reinterpret_cast<uint2*>(sp + NP * kXPBytes);
  ExtSmem& sm = *reinterpret_cast<ExtSmem*>(f4tab + 256);

  const int half = blockIdx.x;                                 // V half (head_dim 512), else 0
  const int blk = a.nblocks - 1 - static_cast<int>(blockIdx.y);   // later blocks (longer KV ranges) first
  const int kvh = blockIdx.z;
  const int G = a.Hq / a.Hk, BT = kXTile / G;
  const int q_row0 = a.blocks[4 * blk], n_tok = a.blocks[4 * blk + 1], pos0 = a.blocks[4 * blk + 2];
  const int preq = a.blocks[4 * blk + 3];
  if (n_tok <= 0 || n_tok > BT) {
    if (threadIdx.x == 0 && n_tok > BT) record_status(a.status, kBadIndex);
    return;
  }
  const int kv_hi = pos0 + n_tok;
  const int kv_lo = a.window > 0 ? max(0, pos0 - a.window + 1) : 0;
  const int t0 = kv_lo & ~(kXTile - 1);
  const int ntiles = (kv_hi - t0 + kXTile - 1) / kXTile;
  const int* pt = a.page_table + static_cast<size_t>(preq) * a.pt_stride;
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tile_full[i], kXDequantWarps);
      mbar_init(&sm.pv_done[i], 1);
      mbar_init(&sm.p_full[i], kXSoftmaxWarps);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, kXSoftmaxWarps);
    mbar_init(&sm.q_ready, kXSoftmaxWarps);
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if constexpr (FMT == kKvNvfp4) f4_table_fill(f4tab);
  if (warp == kXMmaWarp) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) x_trace(a.trace, kXEvStart, 0);

  if (warp < kXSoftmaxWarps) {
    regs_inc<200>();   // 128 x 200 (softmax) + 256 x 128 (dequant, unchanged) + 128 x 56 = 512 x 128 launched
    // ------------------------------------------------------------------ softmax: thread = row = TMEM lane
    const int qd = warp & 3;
    const int r = 32 * qd + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * qd) << 16;
    const int tq = r / G, g = r - (r / G) * G;
    const bool live = tq < n_tok;
    const int pos = pos0 + tq;
    // Q row -> E4M3 (scale amax / 448) -> TMEM columns [384, 384 + D / 4)
    const __nv_bfloat16* qr = reinterpret_cast<const __nv_bfloat16*>(a.q) +
                              (static_cast<size_t>(q_row0 + tq) * a.Hq + kvh * G + g) * D;
    float amax = 0.f;
    if (live) {
#pragma unroll 4
      for (int c = 0; c < D / 8; ++c) amax = bf16x8_amax(ldg16x(qr + 8 * c), amax);
    }
    const float qsc = fmaxf(amax, 1e-20f) / 448.f;
    const float qinv = 1.f / qsc;
#pragma unroll 1
    for (int b = 0; b < D / 128; ++b) {
      uint32_t w[32];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint2 e = bf16x8_to_e4m3(live ? ldg16x(qr + 128 * b + 8 * k) : make_uint4(0, 0, 0, 0), qinv);
        w[2 * k] = e.x;
        w[2 * k + 1] = e.y;
      }
      tmem_st32(tmem + lane_base + kXColQ + 32 * b, w);
    }
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.q_ready);

    // waits are warp-uniform: the warp-collective tcgen05.ld/st below need every lane
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.status, kTimeoutConsumer));
    };
    const float sc2 = qsc * a.sm_scale * a.k_scale * 1.4426950408889634f;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!wwait(&sm.s_full, j & 1)) { ok = false; break; }
      if (r == 0) x_trace(a.trace, kXEvSSeen, j);
      tc_fence_after();
      uint32_t sr[kXTile];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(tmem + lane_base + kXColS + 32 * q4, sr + 32 * q4);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free);
      if (r == 0) x_trace(a.trace, kXEvSLoaded, j);
      // columns inside [lo, hi] are visible (causal: kv <= pos; window: kv > pos - W).  Interior tiles (every row
      // sees every column) skip the mask; masked scores become -inf.  The max is taken on the raw scores (the
      // scale sc2 > 0 is applied to the max, and folded into one FFMA per score below).
      const int kv0 = t0 + j * kXTile;
      const int hi = live ? pos - kv0 : -1;
      const int lo = a.window > 0 ? pos - a.window + 1 - kv0 : -(1 << 30);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (__all_sync(0xffffffffu, hi >= kXTile - 1 && lo <= 0)) {
#pragma unroll
        for (int c = 0; c < kXTile; ++c) mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sr[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kXTile; ++c) {
          if (!(c <= hi && c >= lo)) sr[c] = __float_as_uint(-INFINITY);
          mx[c & 3] = fmaxf(mx[c & 3], __uint_as_float(sr[c]));
        }
      }
      const float mraw = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float mt = mraw * sc2;
      const bool first = (m_ref == -INFINITY) && (mt > -INFINITY);
      const bool grow = (m_ref > -INFINITY) && (mt > m_ref + kXTau);
      const float alpha = grow ? ex2x(m_ref - mt) : 1.f;
      if (first || grow) m_ref = mt;
      l *= alpha;
      if (r == 0) x_trace(a.trace, kXEvMax, j);
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        // O must hold PV(j - 1) before it is rescaled
        if (!wwait(&sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kXColO + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st32(tmem + lane_base + kXColO + 32 * c, o);
        }
        tmem_st_wait();
      }
      // the P buffer is free once the PV that read it (tile j - NP) completed
      if (j >= NP) {
        const int jj = j - NP;
        if (!wwait(&sm.pv_done[jj & 1], (jj >> 1) & 1)) { ok = false; break; }
      }
      const int pb = NP == 1 ? 0 : (j & 1);
      if (r == 0) x_trace(a.trace, kXEvPFree, j);
      uint8_t* prow = sp + pb * kXPBytes + r * 128;   // SW128 row of 128 P columns
      // P = 2^(S sc2 - m) <= 2^tau: two values per f16x2 exp2 (P is E4M3 anyway), row sums in f16x2 per 16-column
      // chunk, then fp32
      float lsum[4] = {0.f, 0.f, 0.f, 0.f};
      const bool any = m_ref > -INFINITY;
      const float nm = any ? -m_ref : 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
        uint32_t hs = 0;                                   // f16x2 partial sums of this chunk
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int b0 = 16 * c + 4 * k;
          uint32_t e01 = 0, e23 = 0;
          if (any) {
            e01 = ex2_h2(pack_h2(fmaf(__uint_as_float(sr[b0]), sc2, nm), fmaf(__uint_as_float(sr[b0 + 1]), sc2, nm)));
            e23 = ex2_h2(pack_h2(fmaf(__uint_as_float(sr[b0 + 2]), sc2, nm), fmaf(__uint_as_float(sr[b0 + 3]), sc2, nm)));
          }
          hs = k == 0 ? hadd2_u32(e01, e23) : hadd2_u32(hs, hadd2_u32(e01, e23));
          w[k] = static_cast<uint32_t>(h2_to_e4m3x2(e01)) | (static_cast<uint32_t>(h2_to_e4m3x2(e23)) << 16);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hs));
        lsum[c & 3] += f.x + f.y;
      }
      l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
      if (r == 0) x_trace(a.trace, kXEvPWritten, j);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[pb]);
      if (r == 0) x_trace(a.trace, kXEvPReady, j);
    }
    if (ok) ok = wwait(&sm.pv_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1);
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? a.v_scale / l : 0.f;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out) +
                            (static_cast<size_t>(q_row0 + tq) * a.Hq + kvh * G + g) * D + 256 * half;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kXColO + 32 * c, o);
        tmem_ld_wait();
        if (!live) continue;
        uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(o[8 * q + 2 * k]) * inv,
                                                           __uint_as_float(o[8 * q + 2 * k + 1]) * inv);
            w[k] = *reinterpret_cast<const uint32_t*>(&v);
          }
          dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  } else if (warp < kXSoftmaxWarps + kXDequantWarps) {
    // ------------------------------------------------------------------ dequant: two threads per tile row
    const int dt = threadIdx.x - 32 * kXSoftmaxWarps;
    const int row = dt & (kXTile - 1), sub = dt >> 7;
    const int vc0 = D == 512 ? 4 * half : 0;                    // first 64-value unit of this CTA's V half
    // pool part (K or V) holding tile j's row, or null when the row is outside [kv_lo, kv_hi)
    auto part_of = [&](int j, int which, int& rr) -> const uint8_t* {
      const int kv = t0 + j * kXTile + row;
      rr = kv & 63;
      if (j >= ntiles || kv < kv_lo || kv >= kv_hi) return nullptr;
      const int phys = (kv >> 6) < a.pt_stride ? pt[kv >> 6] : -1;
      if (phys < 0 || phys >= a.pool_pages) {
        record_status(a.status, kBadIndex);
        return nullptr;
      }
      return a.pool + (static_cast<size_t>(phys) * a.Hk + kvh) * (2 * PB) + which * PB;
    };
    // unit u of this thread: K units c = sub + 2 u (u < NKU), then V units c = vc0 + sub + 2 (u - NKU)
    auto unit_c = [&](int u) { return u < NKU ? sub + 2 * u : vc0 + sub + 2 * (u - NKU); };
    auto unit_dst = [&](int stage, int u, int k) -> uint8_t* {   // 16-byte chunk k (0..3) of unit u
      const int c = unit_c(u);
      const int lc = c - (u < NKU ? 0 : vc0);                    // unit index within its tile
      uint8_t* t = u < NKU ? ktile + stage * KB : vtile + stage * kXVBytes;
      return t + (lc >> 1) * kXBlk + sw128_chunk(row, (lc & 1) * 4 + k);
    };
    if constexpr (FMT == kKvNvfp4) {
      F4Unit cur[NKU + NVU];
      bool cur_ok[2];
      auto load = [&](int j) {
        int rr;
        const uint8_t* pk = part_of(j, 0, rr);
        const uint8_t* pv = pk ? pk + PB : nullptr;
        cur_ok[0] = pk != nullptr;
        cur_ok[1] = pv != nullptr;
#pragma unroll
        for (int u = 0; u < NKU + NVU; ++u) {
          const uint8_t* p = u < NKU ? pk : pv;
          const int c = unit_c(u);
          if (p) {
            cur[u].c0 = ldg16x(p + rr * RB + x_chunk_pos(2 * c, rr, NCH) * 16);
            cur[u].c1 = ldg16x(p + rr * RB + x_chunk_pos(2 * c + 1, rr, NCH) * 16);
            cur[u].sc = __ldg(reinterpret_cast<const uint32_t*>(p + 64 * RB + rr * (D / 16) + 4 * c));
          }
        }
      };
      load(0);
      for (int j = 0; j < ntiles; ++j) {
        const int stage = j & 1;
        if (j >= 2 && !mbar_wait(&sm.pv_done[stage], ((j - 2) >> 1) & 1, abort, a.status, kTimeoutProducer)) break;
        if (dt == 0) x_trace(a.trace, kXEvDeqStart, j);
#pragma unroll
        for (int u = 0; u < NKU + NVU; ++u) {
          const bool okv = cur_ok[u < NKU ? 0 : 1];
          const uint32_t w[8] = {cur[u].c0.x, cur[u].c0.y, cur[u].c0.z, cur[u].c0.w,
                                 cur[u].c1.x, cur[u].c1.y, cur[u].c1.z, cur[u].c1.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {          // 16 values = one block scale
            uint4 o = make_uint4(0, 0, 0, 0);
            if (okv) {
              const uint2 tab = f4tab[(cur[u].sc >> (8 * k)) & 0xFFu];
              const uint2 e0 = f4_decode8(w[2 * k], tab), e1 = f4_decode8(w[2 * k + 1], tab);
              o = make_uint4(e0.x, e0.y, e1.x, e1.y);
            }
            *reinterpret_cast<uint4*>(unit_dst(stage, u, k)) = o;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tile_full[stage]);
        if (dt == 0) x_trace(a.trace, kXEvDeqEnd, j);
        load(j + 1);
      }
    } else {
      // E4M3 rows need no conversion: asynchronous 16-byte copies into the slab (zero-filled outside the range)
      for (int j = 0; j < ntiles; ++j) {
        const int stage = j & 1;
        if (j >= 2 && !mbar_wait(&sm.pv_done[stage], ((j - 2) >> 1) & 1, abort, a.status, kTimeoutProducer)) break;
        int rr;
        const uint8_t* pk = part_of(j, 0, rr);
#pragma unroll
        for (int u = 0; u < NKU + NVU; ++u) {
          const uint8_t* p = pk ? (u < NKU ? pk : pk + PB) : nullptr;
          const int c = unit_c(u);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint8_t* src = p ? p + rr * RB + x_chunk_pos(4 * c + k, rr, NCH) * 16 : a.pool;
            cp_async16x(unit_dst(stage, u, k), src, p ? 16u : 0u);
          }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tile_full[stage]);
      }
    }
  } else {
    regs_dec<56>();
    if (warp == kXMmaWarp) {
      // ---------------------------------------------------------------- MMA issue: the whole warp runs the loop
      // (warp-uniform descriptor arithmetic), one elected lane issues four MMAs per asm statement
      const bool el = elect_one();
      const uint32_t id_qk = idesc_dense(0, 0, 128, kXTile);
      const uint32_t id_pv = idesc_dense(0, 0, 128, 256) | (1u << 16);   // B (V) MN-major
      const uint32_t k_a = smem_u32(ktile), v_a = smem_u32(vtile), p_a = smem_u32(sp);
      const uint32_t tO = tmem + kXColO, tS = tmem + kXColS, tQ = tmem + kXColQ;
      bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, abort, a.status, kTimeoutMma));
      int nq = 0, np = 0;
      unsigned long long tw = global_ns();
      uint32_t idle = 0;
      // barrier probes by lane 0, broadcast, so every lane takes the same branch
      auto test = [&](uint64_t* bar, uint32_t parity) {
        return __shfl_sync(0xffffffffu, lane == 0 ? static_cast<int>(mbar_test(bar, parity)) : 0, 0) != 0;
      };
      while (ok && np < ntiles) {
        bool progressed = false;
        // QK(nq) needs tile nq and S free (softmax loaded S(nq - 1))
        if (nq < ntiles && test(&sm.tile_full[nq & 1], (nq >> 1) & 1) &&
            (nq < 1 || test(&sm.s_free, (nq - 1) & 1))) {
          tc_fence_after();
          const uint32_t kt = k_a + (nq & 1) * KB;
#pragma unroll
          for (int k0 = 0; k0 < D / 32; k0 += 4) {
            uint32_t d4[4], a4[4];
            uint64_t b4[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int kk = k0 + k;
              d4[k] = tS;
              a4[k] = tQ + 8 * kk;
              b4[k] = desc_sw128(kt + (kk >> 2) * kXBlk + (kk & 3) * 32);
            }
            if (el) umma_f8_ts_x4(d4, a4, b4, id_qk, k0 > 0 ? 0xFu : 0xEu);
          }
          if (el) {
            umma_commit(&sm.s_full);
            x_trace(a.trace, kXEvQk, nq);
          }
          __syncwarp();
          ++nq;
          progressed = true;
        }
        // PV(np) needs P(np)
        if (np < nq) {
          const int pb = NP == 1 ? 0 : (np & 1);
          const uint32_t par = NP == 1 ? (np & 1) : ((np >> 1) & 1);
          if (test(&sm.p_full[pb], par)) {
            tc_fence_after();
            const uint32_t vt = v_a + (np & 1) * kXVBytes;
            uint32_t d4[4];
            uint64_t a4[4], b4[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              d4[kk] = tO;
              a4[kk] = desc_sw128(p_a + pb * kXPBytes + 32 * kk);
              b4[kk] = desc_mn128(vt + kk * 32 * 128, kXBlk);
            }
            if (el) {
              umma_f8_ss_x4(d4, a4, b4, id_pv, np > 0 ? 0xFu : 0xEu);
              umma_commit(&sm.pv_done[np & 1]);
              x_trace(a.trace, kXEvPv, np);
            }
            __syncwarp();
            ++np;
            progressed = true;
          }
        }
        if (progressed) {
          tw = global_ns();
          idle = 0;
        } else if ((++idle & 63) == 0) {
          const int ab = __shfl_sync(0xffffffffu, *abort, 0);
          if (ab) {
            ok = false;
          } else if (__shfl_sync(0xffffffffu, static_cast<int>(global_ns() - tw > kWaitLimitNs), 0)) {
            if (lane == 0) {
              *abort = 1;
              record_status(a.status, kTimeoutMma);
            }
            ok = false;
          }
        }
      }
      // every issued MMA has completed before TMEM is released
      if (el) umma_commit(&sm.fin);
      __syncwarp();
      mbar_wait(&sm.fin, 0, nullptr, a.status, kTimeoutMma);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) x_trace(a.trace, kXEvEnd, 0);
  if (warp == kXMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int FMT, int D>
cudaError_t launch_extend(const GqaExtendArgs& a, cudaStream_t s) {
  constexpr int smem = x_smem_bytes<D>();
  auto k = gqa_extend_kernel<FMT, D>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(D == 512 ? 2 : 1, a.nblocks, a.Hk);
  k<<<grid, kXThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t gqa_extend(const GqaExtendArgs& a, cudaStream_t s) {
  if (a.nblocks == 0) return cudaSuccess;
  if (a.Hk <= 0 || a.Hq % a.Hk || a.Hq / a.Hk > 128 || a.page != 64 || a.nblocks > 65535 || a.Hk > 65535)
    return cudaErrorInvalidValue;
  if (a.fmt == kKvNvfp4) {
    if (a.D == 512) return launch_extend<kKvNvfp4, 512>(a, s);
    if (a.D == 256) return launch_extend<kKvNvfp4, 256>(a, s);
  } else if (a.fmt == kKvFp8) {
    if (a.D == 512) return launch_extend<kKvFp8, 512>(a, s);
    if (a.D == 256) return launch_extend<kKvFp8, 256>(a, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace iob
