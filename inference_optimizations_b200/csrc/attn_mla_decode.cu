// Sparse MLA decode: the DSA attention of DeepSeek-V3.2 / GLM-5-class models over a pool of compressed latent rows.
//
// Semantics (fp32 oracle: ops/formats.py sparse_mla_reference).  Query token t has H <= 128 heads; q[t, h] holds
// 576 values (512 latent "nope" dims, then 64 rope dims) and attends to the pool rows idx[t, 0..topk) (-1 = masked);
// K = the 576-value row, V = its first 512 values.  out[t, h] = softmax(q K^T * sm_scale) V; lse[t, h] is the
// natural-log logsumexp (-inf and a zero output when every row is masked).
// Row formats: NVFP4 352-B rows (256 B of E2M1 pairs, element 2i in the low nibble; 32 E4M3 scales, one per 16
// values; 64 E4M3 rope values at byte 288 -- the 4-bit MLA KV row of kv-cache-4bit/glm-kv4/glm_kv4.py:1-36) or
// plain E4M3 576-B rows (the FP8 pool it is measured against).
//
// Design (replaces kv-cache-4bit/kv4mla/csrc/glm_fp4_decode_fp8.cu; built B200-first, not translated):
//   * M = 128 heads of one token fill a full-height UMMA (kind::f8f6f4, E4M3 operands, K = 32 per MMA).  The O
//     accumulator [128 x 512] fp32 does not fit TMEM next to S and Q, so a token runs as two CTAs, one per V half.
//     TMEM: O half [128 x 256] at cols 0..255, S [128 heads x 128 rows] at 256, Q (E4M3, the A operand of QK) at
//     384.  A tcgen05.mma costs about the same whatever its N, so tiles are as wide as TMEM allows (N = 128).
//   * the top-k list is walked in 128-row tiles through a 2-deep ring: four dequant warps gather each tile's rows
//     straight from global memory (the next tile's loads in flight while the current one is converted; one warp
//     warms L2 with the split's rows), convert E2M1 x E4M3 -> f16 -> E4M3 and store the tile once as
//     [128 rows x 576] E4M3: four 128-feature SW128 blocks plus an SW64 rope block.  QK reads it K-major; PV reads
//     the same bytes as its MN-major V operand (an SW128 atom is 8 rows x 128 bytes either way).
//   * one thread issues QK and PV in whichever order their inputs become ready, so the tensor pipe never waits
//     behind a tile that is still being gathered.
//   * softmax: one warpgroup, thread = head = TMEM lane holding its 128-column S row; running max with a lazy rescale (O in TMEM is rescaled
//     only when the max grows by more than 2^8); P = 2^(s - m) <= 256 in E4M3 is the A operand of PV.
//   * split-K over the top-k list when tokens are fewer than SMs; mla_combine_kernel merges the partials.
// Every wait is bounded: a wait past its limit records a status code and the CTA unwinds.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kMThreads = 512;
constexpr int kMTile = 128;                            // rows per tile: N of QK, K extent of one PV
constexpr int kMRing = 2;                              // tiles in flight
constexpr int kMBlk = kMTile * 128;                    // one 128-feature E4M3 block of a tile (16 KB)
constexpr int kMRopeOff = 4 * kMBlk;                   // SW64 rope block: 128 rows x 64 B
constexpr int kMTileBytes = kMRopeOff + kMTile * 64;   // 72 KB
constexpr int kMPBytes = 128 * kMTile;                 // P: 128 heads x 128 rows, E4M3, SW128 K-major
constexpr uint32_t kMColO = 0, kMColS = 256, kMColQ = 384;
constexpr float kMTau = 8.f;                           // lazy-rescale threshold, log2 units
constexpr int kMSoftmaxWarps = 4, kMDequantWarps = 8, kMMmaWarp = 12, kMPrefetchWarp = 13;
constexpr int kF4Row = 352, kF4FlashRow = 288, kV4ProRow = 320, kV4ProBf16Row = 384, kF8Row = 576;
constexpr bool is_v4pro(int fmt) { return fmt == kKvV4Pro || fmt == kKvV4ProBf16Rope; }

struct MlaSmem {
  uint64_t tile_full[kMRing];   // tile rows stored                       (4 dequant-warp arrivals)
  uint64_t p_full[kMRing];      // P written                              (8 softmax-warp arrivals)
  uint64_t pv_done[kMRing];     // PV committed                           (tcgen05.commit)
  uint64_t s_full;              // QK committed                           (tcgen05.commit)
  uint64_t s_free;              // S loaded into registers                (8 softmax-warp arrivals)
  uint64_t q_ready, fin;
  alignas(16) float bias[kMRing][kMTile];   // 0 live row, -inf masked (read as float4)
  uint2 f4tab[256];             // scale byte -> E4M3 products {0, .5, 1, 1.5, 2, 3, 4, 6} x scale
  uint32_t tmem_base;
  int abort;
};

constexpr int mla_smem_bytes() {
  return 1024 + kMRing * kMTileBytes + kMRing * kMPBytes + 128 * 64 + static_cast<int>(sizeof(MlaSmem));
}
static_assert(mla_smem_bytes() <= 232448, "shared memory budget");
static_assert(offsetof(MlaSmem, bias) % 16 == 0, "bias is read with 16-byte loads");

// Diagnostic timeline of CTA (0, 0, 0): clock64 at each event, [event][tile] with up to 64 tiles.
enum MlaTraceEv { kMlaEvStart, kMlaEvQReady, kMlaEvDeqStart, kMlaEvDeqEnd, kMlaEvQk, kMlaEvSSeen, kMlaEvPReady,
                  kMlaEvPv, kMlaEvEpi, kMlaEvEnd, kMlaEvLoad, kMlaEvSLoaded, kMlaEvMax, kMlaEvPWait, kMlaEvShip,
                  kMlaEvCount };
__device__ __forceinline__ void mla_trace(long long* tr, int ev, int j) {
  if (tr != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && j < 64) tr[ev * 64 + j] = clock64();
}

// 2^x on the SFU (ex2.approx.ftz: relative error ~2^-22, subnormal results flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Debug builds (-DIOB_MLA_CHECKS) check every computed global index against its allocation and record a status
// code (200 + site) instead of performing an out-of-range access.
#ifdef IOB_MLA_CHECKS
#define MLA_IN_RANGE(cond, site) ((cond) ? true : (record_status(a.status, 200 + (site)), false))
#else
#define MLA_IN_RANGE(cond, site) true
#endif

__device__ __forceinline__ void cp_async16(void* smem, const void* g, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(g), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint32_t u4_get(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// One dequant thread's share of a row: 128-feature blocks 2 q and 2 q + 1 of the latent (NVFP4: 128 code bytes +
// 16 scales; E4M3: 256 bytes) and rope values [32 q, 32 q + 32).
template <int FMT>
struct RawRow {
  uint4 v[FMT == kKvFp8 ? 16 : 8];
  uint4 sc;
  uint4 rope[FMT == kKvV4ProBf16Rope ? 4 : 2];   // 32 E4M3 values, or 32 bf16 values of the 384-byte cell
};

template <int FMT>
__device__ __forceinline__ void load_row(const uint8_t* row, int q, RawRow<FMT>& x) {
  constexpr int NV = FMT == kKvFp8 ? 16 : 8;
  if (row) {
    if constexpr (is_v4pro(FMT)) {
      // 320 / 384-byte cell: 448 latent values (codes at 0..223, scales at 224..251, zero pad to 256) + 64 rope
      // values at 256 (E4M3, or bf16 in the 384-byte cell); latent dims 448..511 read as zero codes (thread 1's last
      // two code chunks) under the zero pad scales
#pragma unroll
      for (int i = 0; i < NV; ++i) x.v[i] = (q == 0 || i < 6) ? ldg16(row + 128 * q + 16 * i) : make_uint4(0, 0, 0, 0);
      x.sc = ldg16(row + 224 + 16 * q);
      if constexpr (FMT == kKvV4ProBf16Rope) {
#pragma unroll
        for (int i = 0; i < 4; ++i) x.rope[i] = ldg16(row + 256 + 64 * q + 16 * i);
      } else {
        x.rope[0] = ldg16(row + 256 + 32 * q);
        x.rope[1] = ldg16(row + 256 + 32 * q + 16);
      }
    } else if constexpr (FMT != kKvFp8) {     // NVFP4 latent (352-B row; the 288-B row has no rope block)
#pragma unroll
      for (int i = 0; i < NV; ++i) x.v[i] = ldg16(row + 128 * q + 16 * i);
      x.sc = ldg16(row + 256 + 16 * q);
      if constexpr (FMT == kKvNvfp4) {
        x.rope[0] = ldg16(row + 288 + 32 * q);
        x.rope[1] = ldg16(row + 288 + 32 * q + 16);
      } else {
        x.rope[0] = x.rope[1] = make_uint4(0, 0, 0, 0);
      }
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) x.v[i] = ldg16(row + 256 * q + 16 * i);
      x.sc = make_uint4(0, 0, 0, 0);
      x.rope[0] = ldg16(row + 512 + 32 * q);
      x.rope[1] = ldg16(row + 512 + 32 * q + 16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) x.v[i] = make_uint4(0, 0, 0, 0);
    x.sc = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < (FMT == kKvV4ProBf16Rope ? 4 : 2); ++i) x.rope[i] = make_uint4(0, 0, 0, 0);
  }
}

// Rope chunk c (16 values) of a raw row share as E4M3: the stored bytes, or the 384-byte cell's bf16 values rounded
// to nearest-even E4M3 (saturating) for the FP8 tensor-core QK product.
template <int FMT>
__device__ __forceinline__ uint4 rope_chunk(const RawRow<FMT>& x, int c) {
  if constexpr (FMT == kKvV4ProBf16Rope) {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 b = x.rope[2 * c + h];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t p0 = u4_get(b, 2 * k), p1 = u4_get(b, 2 * k + 1);
        const uint32_t lo = f32x2_to_e4m3x2(__uint_as_float(p0 << 16), __uint_as_float(p0 & 0xFFFF0000u));
        const uint32_t hi = f32x2_to_e4m3x2(__uint_as_float(p1 << 16), __uint_as_float(p1 & 0xFFFF0000u));
        w[2 * h + k] = lo | (hi << 16);
      }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    return x.rope[c];
  }
}

// The 16-byte E4M3 chunk c (0..15: values 16 c .. 16 c + 15 of the thread's 256) of a raw row share; `tabs` is the
// CTA's scale-byte -> E4M3 product table (f4_table_fill).
template <int FMT>
__device__ __forceinline__ uint4 row_chunk(const RawRow<FMT>& x, int c, const uint2* tabs) {
  if constexpr (FMT != kKvFp8) {
    const uint4& cw = x.v[c >> 1];                    // 32 values per code chunk
    const uint32_t sb = (u4_get(x.sc, c >> 2) >> (8 * (c & 3))) & 0xFFu;   // scale of these 16 values
    const uint2 tab = tabs[sb];
    const uint2 lo = f4_decode8(u4_get(cw, 2 * (c & 1)), tab);
    const uint2 hi = f4_decode8(u4_get(cw, 2 * (c & 1) + 1), tab);
    return make_uint4(lo.x, lo.y, hi.x, hi.y);
  } else {
    return x.v[c];
  }
}

template <int FMT>
__global__ void __launch_bounds__(kMThreads, 1) mla_decode_kernel(const MlaDecodeArgs a) {
  constexpr int RB = FMT == kKvNvfp4 ? kF4Row : FMT == kKvNvfp4NoRope ? kF4FlashRow : FMT == kKvV4Pro ? kV4ProRow : FMT == kKvV4ProBf16Rope ? kV4ProBf16Row
                                                                                                    : kF8Row;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = base;                                  // 2 x 72 KB
  uint8_t* sp = tiles + kMRing * kMTileBytes;             // 2 x 16 KB P
  uint8_t* sqr = sp + kMRing * kMPBytes;                  // Q rope, SW64 128 x 64 B
  MlaSmem& sm = *reinterpret_cast<MlaSmem*>(sqr + 128 * 64);

  griddep_launch();                                       // the W_UV GEMM after this may set up meanwhile
  const int half = blockIdx.x;                            // V half
  const int t = blockIdx.y, split = blockIdx.z;
  const int ntiles_all = (a.topk + kMTile - 1) / kMTile;
  const int tile0 = split * a.tiles_per_split;
  const int ntiles = min(ntiles_all, tile0 + a.tiles_per_split) - tile0;
  const int warp = warp_id(), lane = lane_id();
  const int* idx_row = a.idx + static_cast<size_t>(t) * a.idx_stride;
  if (a.tok_sel && a.tok_sel[t] != a.sel) return;        // this token's rows live in the other pool's launch

  if (ntiles <= 0) {  // empty split: an empty partial
    if (a.num_splits > 1 && half == 0 && threadIdx.x < a.H)
      a.lse_part[(static_cast<size_t>(split) * a.T + t) * a.H + threadIdx.x] = -INFINITY;
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMRing; ++i) {
      mbar_init(&sm.tile_full[i], kMDequantWarps);
      mbar_init(&sm.p_full[i], kMSoftmaxWarps);
      mbar_init(&sm.pv_done[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, kMSoftmaxWarps);
    mbar_init(&sm.q_ready, kMSoftmaxWarps);
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if constexpr (FMT != kKvFp8) f4_table_fill(sm.f4tab);
  if (warp == kMMmaWarp) { tmem_alloc(&sm.tmem_base, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) mla_trace(a.trace, kMlaEvStart, 0);

  if (warp < kMSoftmaxWarps) {
    regs_inc<200>();   // 128 x 200 (softmax) + 256 x 128 (dequant, unchanged) + 128 x 56 = 512 x 128 launched
    // ---------------------------------------------------------------- softmax: thread = head = TMEM lane
    const int qd = warp & 3, ch = 0;             // lane quadrant; one warp covers all S columns
    const int h = 32 * qd + lane;
    const bool hv = h < a.H;
    const uint32_t lane_base = static_cast<uint32_t>(32 * qd) << 16;
    // Q (E4M3, quantized per head by mla_q_quant_kernel): the 512 latent values -> TMEM (A operand of QK), the 64
    // rope values -> shared memory (SW64), in two halves of 18 loads each issued before their first use.
#pragma unroll 1
    for (int hf = 0; hf < 2; ++hf) {
      const uint8_t* qh = a.q8 + (static_cast<size_t>(t) * a.H + h) * 576;
      const bool q_ok = hv && MLA_IN_RANGE(static_cast<size_t>(t) * a.H + h < static_cast<size_t>(a.T) * a.H, 1);
      uint4 qv[18];
#pragma unroll
      for (int c = 0; c < 16; ++c) qv[c] = q_ok ? ldg16(qh + 256 * hf + 16 * c) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < 2; ++c) qv[16 + c] = q_ok ? ldg16(qh + 512 + 32 * hf + 16 * c) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint32_t w[32];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          w[4 * k] = qv[8 * b + k].x; w[4 * k + 1] = qv[8 * b + k].y;
          w[4 * k + 2] = qv[8 * b + k].z; w[4 * k + 3] = qv[8 * b + k].w;
        }
        tmem_st32(tmem + lane_base + kMColQ + 64 * hf + 32 * b, w);
      }
#pragma unroll
      for (int c = 0; c < 2; ++c)     // rope-free rows: the rope MMAs add q_pe . 0 (query rope zeroed)
        *reinterpret_cast<uint4*>(sqr + sw64_chunk(h, 2 * hf + c)) =
            FMT == kKvNvfp4NoRope ? make_uint4(0, 0, 0, 0) : qv[16 + c];
    }
    const float qs = hv ? a.q_scale[static_cast<size_t>(t) * a.H + h] : 1.f;
    tmem_st_wait();
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.q_ready);

    // waits are made warp-uniform: the warp-collective tcgen05.ld/st and votes below need every lane
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.status, kTimeoutConsumer));
    };
    constexpr int NC = kMTile;                   // S columns per thread (128)
    const float sc2 = qs * a.sm_scale * 1.4426950408889634f;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1, rb = j % kMRing;
      if (!wwait(&sm.s_full, j & 1)) { ok = false; break; }
      if (h == 0) mla_trace(a.trace, kMlaEvSSeen, j);
      tc_fence_after();
      uint32_t sr[NC];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(tmem + lane_base + kMColS + 32 * q4, sr + 32 * q4);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free);
      if (lane == 0) mla_trace(a.trace, kMlaEvCount + 12 + warp, j);
      if (!wwait(&sm.tile_full[rb], (j / kMRing) & 1)) { ok = false; break; }   // row biases visible
      if (h == 0) mla_trace(a.trace, kMlaEvSLoaded, j);
      // s = S * scale + bias (bias = -inf on masked rows), max over four independent chains
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const float4* bp = reinterpret_cast<const float4*>(sm.bias[rb] + NC * ch);
#pragma unroll
      for (int q4 = 0; q4 < NC / 4; ++q4) {
        const float4 bb = bp[q4];
        const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float v = fmaf(__uint_as_float(sr[4 * q4 + k]), sc2, bv[k]);
          sr[4 * q4 + k] = __float_as_uint(v);
          mx[k] = fmaxf(mx[k], v);
        }
      }
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      // lazy rescale: keep the reference max unless this tile exceeds it by more than 2^tau
      const bool first = (m_ref == -INFINITY) && (mt > -INFINITY);
      const bool grow = (m_ref > -INFINITY) && (mt > m_ref + kMTau);
      const float alpha = grow ? ex2_approx(m_ref - mt) : 1.f;
      if (first || grow) m_ref = mt;
      l *= alpha;
      if (h == 0) mla_trace(a.trace, kMlaEvMax, j);
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        if (!wwait(&sm.pv_done[(j - 1) % kMRing], ((j - 1) / kMRing) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kMColO + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st32(tmem + lane_base + kMColO + 32 * c, o);
        }
        tmem_st_wait();
      }
      if (j >= kMRing && !wwait(&sm.pv_done[rb], ((j - kMRing) / kMRing) & 1)) { ok = false; break; }
      if (h == 0) mla_trace(a.trace, kMlaEvPWait, j);
      uint8_t* prow = sp + rb * kMPBytes + h * 128;  // SW128 row of 128 P columns
      float lsum[4] = {0.f, 0.f, 0.f, 0.f};
      const bool live = m_ref > -INFINITY;   // every row so far masked: P = 0
      const float nm = live ? -m_ref : 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {          // columns 16 c .. 16 c + 15 = 16-byte chunk c of the P row
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            p[e] = live ? ex2_approx(__uint_as_float(sr[16 * c + 4 * k + e]) + nm) : 0.f;
            lsum[e] += p[e];
          }
          w[k] = static_cast<uint32_t>(f32x2_to_e4m3x2(p[0], p[1])) |
                 (static_cast<uint32_t>(f32x2_to_e4m3x2(p[2], p[3])) << 16);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (h & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[rb]);
      if (h == 0) mla_trace(a.trace, kMlaEvPReady, j);
      if (lane == 0) mla_trace(a.trace, kMlaEvCount + warp, j);         // per softmax warp: P arrival

    }
    if (ok) ok = wwait(&sm.pv_done[(ntiles - 1) % kMRing], ((ntiles - 1) / kMRing) & 1);
    if (h == 0) mla_trace(a.trace, kMlaEvEpi, 0);
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const size_t row = static_cast<size_t>(t) * a.H + h;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kMColO + 32 * c, o);
        tmem_ld_wait();
        if (!hv) continue;
        const int d0 = 256 * half + 32 * c;
        if (!MLA_IN_RANGE(row < static_cast<size_t>(a.T) * a.H && split < a.num_splits && d0 + 32 <= 512, 2)) continue;
        if (a.num_splits == 1) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + row * 512 + d0);
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
        } else {
          float4* dst = reinterpret_cast<float4*>(a.o_part + (static_cast<size_t>(split) * a.T * a.H + row) * 512 + d0);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            dst[q] = make_float4(__uint_as_float(o[4 * q]) * inv, __uint_as_float(o[4 * q + 1]) * inv,
                                 __uint_as_float(o[4 * q + 2]) * inv, __uint_as_float(o[4 * q + 3]) * inv);
        }
      }
      if (hv && half == 0) {
        const float lse2 = l > 0.f ? m_ref + log2f(l) : -INFINITY;
        if (a.num_splits == 1) {
          if (a.lse) a.lse[row] = lse2 * 0.6931471805599453f;
        } else {
          a.lse_part[static_cast<size_t>(split) * a.T * a.H + row] = lse2;
        }
      }
    }
  } else if (warp < kMSoftmaxWarps + kMDequantWarps) {
    // ---------------------------------------------------------------- dequant: two threads per gathered row
    const int dt = threadIdx.x - 32 * kMSoftmaxWarps;
    const int trow = dt >> 1, q = dt & 1;        // tile row 0..127, blocks 2 q and 2 q + 1
    auto row_id = [&](int j) -> int {
      const int p = (tile0 + j) * kMTile + trow;
      if (!MLA_IN_RANGE(p >= 0, 4)) return -1;
      const int id0 = (j < ntiles && p < a.topk) ? idx_row[p] : -1;
      if (id0 < 0) return -1;
      const int id = id0 - a.row_lo;
      if (id < 0 || id >= a.pool_rows) {  // a row outside the pool: treated as masked, reported once
        record_status(a.status, kBadIndex);
        return -1;
      }
      return id;
    };
    auto row_ptr = [&](int id) -> const uint8_t* {
      return (id >= 0 && MLA_IN_RANGE(id < a.pool_rows, 3)) ? a.pool + static_cast<size_t>(id) * RB : nullptr;
    };
    if constexpr (FMT != kKvFp8) {
      // NVFP4: raw rows are loaded into registers a tile ahead.  The loads for tile j + 1 are issued right after
      // tile j is published: the proxy fence before the arrival would otherwise also wait for them.
      int id_cur = row_id(0), id_nxt = row_id(1);
      RawRow<FMT> cur;
      load_row<FMT>(row_ptr(id_cur), q, cur);
      for (int j = 0; j < ntiles; ++j) {
        const int rb = j % kMRing;
        if (j >= kMRing && !mbar_wait(&sm.pv_done[rb], ((j - kMRing) / kMRing) & 1, abort, a.status, kTimeoutProducer))
          break;
        if (dt == 0) mla_trace(a.trace, kMlaEvDeqStart, j);
        uint8_t* tb = tiles + rb * kMTileBytes;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(tb + (2 * q + (c >> 3)) * kMBlk + sw128_chunk(trow, c & 7)) = row_chunk<FMT>(cur, c, sm.f4tab);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4*>(tb + kMRopeOff + sw64_chunk(trow, 2 * q + c)) = rope_chunk<FMT>(cur, c);
        if (q == 0) sm.bias[rb][trow] = id_cur >= 0 ? 0.f : -INFINITY;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tile_full[rb]);
        if (dt == 0) mla_trace(a.trace, kMlaEvDeqEnd, j);
        id_cur = id_nxt;
        id_nxt = row_id(j + 2);
        load_row<FMT>(row_ptr(id_cur), q, cur);
      }
    } else {
      // E4M3 rows need no conversion: asynchronous 16-byte copies straight into the swizzled tile (zero-filled
      // for masked rows) once the buffer is free
      for (int j = 0; j < ntiles; ++j) {
        const int rb = j % kMRing;
        if (j >= kMRing && !mbar_wait(&sm.pv_done[rb], ((j - kMRing) / kMRing) & 1, abort, a.status, kTimeoutProducer))
          break;
        uint8_t* tb = tiles + rb * kMTileBytes;
        const int id = row_id(j);
        const uint8_t* src = row_ptr(id);
        const uint32_t n = src ? 16u : 0u;
        if (!src) src = a.pool;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          cp_async16(tb + (2 * q + (c >> 3)) * kMBlk + sw128_chunk(trow, c & 7), src + (n ? 256 * q + 16 * c : 0), n);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          cp_async16(tb + kMRopeOff + sw64_chunk(trow, 2 * q + c), src + (n ? 512 + 32 * q + 16 * c : 0), n);
        if (q == 0) sm.bias[rb][trow] = n ? 0.f : -INFINITY;
        cp_async_wait_all();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tile_full[rb]);
      }
    }
  } else {
    regs_dec<56>();
    if (warp == kMMmaWarp) {
      // ------------------------------------------------------------ MMA issue: the whole warp runs the loop
      // (warp-uniform descriptor arithmetic), one elected lane issues the MMAs, four per asm statement
      const bool el = elect_one();
      const uint32_t id_qk = idesc_dense(0, 0, 128, kMTile);
      const uint32_t id_pv = idesc_dense(0, 0, 128, 256) | (1u << 16);  // B (V) MN-major
      const uint32_t tiles_a = smem_u32(tiles), p_a = smem_u32(sp), qr_a = smem_u32(sqr);
      const uint32_t tO = tmem + kMColO, tQ = tmem + kMColQ;
      bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_ready, 0, abort, a.status, kTimeoutMma));
      if (el) mla_trace(a.trace, kMlaEvQReady, 0);
      auto test = [&](uint64_t* bar, uint32_t parity) {
        return __shfl_sync(0xffffffffu, lane == 0 ? static_cast<int>(mbar_test(bar, parity)) : 0, 0) != 0;
      };
      // Issue QK(nq) and PV(np) in whichever order their inputs become ready: QK(j) needs tile j and S free
      // (softmax(j - 1) loaded it); PV(j) needs P(j).  The tensor pipe runs them in issue order.
      int nq = 0, np = 0;
      unsigned long long t0 = global_ns();
      uint32_t idle = 0;
      while (ok && np < ntiles) {
        bool progressed = false;
        if (nq < ntiles) {
          const int rb = nq % kMRing;
          if (test(&sm.tile_full[rb], (nq / kMRing) & 1) && (nq < 1 || test(&sm.s_free, (nq - 1) & 1))) {
            tc_fence_after();
            const uint32_t tile = tiles_a + rb * kMTileBytes;
            const uint32_t tS = tmem + kMColS;
#pragma unroll
            for (int k0 = 0; k0 < 16; k0 += 4) {
              uint32_t d4[4], a4[4];
              uint64_t b4[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int kk = k0 + k;
                d4[k] = tS;
                a4[k] = tQ + 8 * kk;
                b4[k] = desc_sw128(tile + (kk >> 2) * kMBlk + (kk & 3) * 32);
              }
              if (el) umma_f8_ts_x4(d4, a4, b4, id_qk, k0 > 0 ? 0xFu : 0xEu);
            }
            if (el) {
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)
                umma_f8_ss(tS, desc_sw64(qr_a + 32 * kk), desc_sw64(tile + kMRopeOff + 32 * kk), id_qk, 1u);
              umma_commit(&sm.s_full);
              mla_trace(a.trace, kMlaEvQk, nq);
            }
            __syncwarp();
            ++nq;
            progressed = true;
          }
        }
        if (np < nq) {
          const int rb = np % kMRing;
          if (test(&sm.p_full[rb], (np / kMRing) & 1)) {
            tc_fence_after();
            const uint32_t vt = tiles_a + rb * kMTileBytes + half * 2 * kMBlk;
            uint32_t d4[4];
            uint64_t a4[4], b4[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              d4[kk] = tO;
              a4[kk] = desc_sw128(p_a + rb * kMPBytes + 32 * kk);
              b4[kk] = desc_mn128(vt + kk * 32 * 128, kMBlk);
            }
            if (el) {
              umma_f8_ss_x4(d4, a4, b4, id_pv, np > 0 ? 0xFu : 0xEu);
              umma_commit(&sm.pv_done[rb]);
              mla_trace(a.trace, kMlaEvPv, np);
            }
            __syncwarp();
            ++np;
            progressed = true;
          }
        }
        if (progressed) {
          t0 = global_ns();
          idle = 0;
        } else if ((++idle & 63) == 0) {
          if (__shfl_sync(0xffffffffu, *abort, 0)) {
            ok = false;
          } else if (__shfl_sync(0xffffffffu, static_cast<int>(global_ns() - t0 > kWaitLimitNs), 0)) {
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
    } else if (warp == kMPrefetchWarp) {
      // ------------------------------------------------------------ warm L2 with the split's rows, in order
      const int p0 = tile0 * kMTile, p1 = min(a.topk, (tile0 + ntiles) * kMTile);
      for (int p = p0 + lane; p < p1 && !*abort; p += 32) {
        const int id = idx_row[p] - a.row_lo;
        if (idx_row[p] >= 0 && id >= 0 && id < a.pool_rows) prefetch_l2(a.pool + static_cast<size_t>(id) * RB, RB);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) mla_trace(a.trace, kMlaEvEnd, 0);
  if (warp == kMMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per-(token, head) E4M3 quantization of the bf16 query: scale = amax / 448 over the 576 values, q8 = q / scale
// (round to nearest even).  One warp per (token, head).
__global__ void __launch_bounds__(128) mla_q_quant_kernel(const __nv_bfloat16* __restrict__ q, uint8_t* __restrict__ q8,
                                                         float* __restrict__ q_scale, int rows) {
  const int row = blockIdx.x * 4 + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  const uint4* src = reinterpret_cast<const uint4*>(q + static_cast<size_t>(row) * 576);
  uint4 v[3];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < 72 ? src[c] : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(e[k]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = warp_max(amax);
  const float qs = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / qs;
  if (lane == 0) q_scale[row] = qs;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int c = lane + 32 * i;
    if (c >= 72) break;
    const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float2 f0 = __bfloat1622float2(e[2 * k]), f1 = __bfloat1622float2(e[2 * k + 1]);
      w[k] = static_cast<uint32_t>(f32x2_to_e4m3x2(f0.x * inv, f0.y * inv)) |
             (static_cast<uint32_t>(f32x2_to_e4m3x2(f1.x * inv, f1.y * inv)) << 16);
    }
    reinterpret_cast<uint2*>(q8 + static_cast<size_t>(row) * 576)[c] = make_uint2(w[0], w[1]);
  }
}

// out[t, h] = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M); lse in natural log.  One CTA (128 threads) per (t, h).
__global__ void __launch_bounds__(128) mla_combine_kernel(const MlaDecodeArgs a) {
  griddep_launch();
  const int row = blockIdx.x;  // t * H + h
  if (a.tok_sel && a.tok_sel[row / a.H] != a.sel) return;
  const size_t plane = static_cast<size_t>(a.T) * a.H;
  float m = -INFINITY;
  for (int s = 0; s < a.num_splits; ++s) m = fmaxf(m, a.lse_part[s * plane + row]);
  float den = 0.f;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < a.num_splits; ++s) {
    const float ls = a.lse_part[s * plane + row];
    if (ls == -INFINITY) continue;
    const float w = exp2f(ls - m);
    den += w;
    const float4 v = reinterpret_cast<const float4*>(a.o_part + (s * plane + row) * 512)[threadIdx.x];
    num.x += w * v.x; num.y += w * v.y; num.z += w * v.z; num.w += w * v.w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const __nv_bfloat162 lo = __floats2bfloat162_rn(num.x * inv, num.y * inv);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(num.z * inv, num.w * inv);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&lo);
  w.y = *reinterpret_cast<const uint32_t*>(&hi);
  reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + static_cast<size_t>(row) * 512)[threadIdx.x] = w;
  if (threadIdx.x == 0 && a.lse) a.lse[row] = den > 0.f ? (m + log2f(den)) * 0.6931471805599453f : -INFINITY;
}

template <int FMT>
cudaError_t launch_mla(const MlaDecodeArgs& a, cudaStream_t s) {
  constexpr int smem = mla_smem_bytes();
  if (a.q && a.q8_out) {
    mla_q_quant_kernel<<<(a.T * a.H + 3) / 4, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(a.q), a.q8_out,
                                                          a.q_scale_out, a.T * a.H);
    IOB_CUDA_CHECK(cudaGetLastError());
  }
  auto kern = mla_decode_kernel<FMT>;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kern<<<dim3(2, a.T, a.num_splits), kMThreads, smem, s>>>(a);   // x = the CTA pair of one (token, split)
  IOB_CUDA_CHECK(cudaGetLastError());
  if (a.num_splits > 1) {
    mla_combine_kernel<<<a.T * a.H, 128, 0, s>>>(a);
    IOB_CUDA_CHECK(cudaGetLastError());
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t mla_decode(const MlaDecodeArgs& a, cudaStream_t s) {
  if (a.T == 0) return cudaSuccess;
  if (a.H < 1 || a.H > 128 || a.topk < 1 || a.T > 65535 || a.idx_stride < a.topk || a.tiles_per_split < 1 || a.num_splits < 1 ||
      a.num_splits > 65535 || (reinterpret_cast<uintptr_t>(a.pool) & 15) || (reinterpret_cast<uintptr_t>(a.q8) & 15) ||
      (reinterpret_cast<uintptr_t>(a.q) & 15) || !a.q_scale || (a.q && a.q8_out != a.q8))
    return cudaErrorInvalidValue;
  if (static_cast<long long>(a.tiles_per_split) * a.num_splits * kMTile < a.topk) return cudaErrorInvalidValue;
  if (a.num_splits > 1 && (!a.o_part || !a.lse_part)) return cudaErrorInvalidValue;
  switch (a.fmt) {
    case kKvNvfp4: return launch_mla<kKvNvfp4>(a, s);
    case kKvNvfp4NoRope: return launch_mla<kKvNvfp4NoRope>(a, s);
    case kKvV4Pro: return launch_mla<kKvV4Pro>(a, s);
    case kKvV4ProBf16Rope: return launch_mla<kKvV4ProBf16Rope>(a, s);
    case kKvFp8: return launch_mla<kKvFp8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace iob
