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
//   * M = 128 heads of one token fill a full-height UMMA.  A CTA owns (token, V half, split): TMEM's 512 columns
//     hold the O half [128 x 256] fp32 (cols 0..255), S [128 heads x 128 rows] (256..383) and the token's E4M3 Q
//     latent as the A operand of QK (384..511).  Both V halves compute the same S; nothing else is shared.
//   * rows are gathered 128 per tile by eight dequant warps directly from global memory (the next tile's loads are
//     in flight while the current tile is converted; one warp warms L2 with the split's rows at start), converted
//     E2M1 x E4M3 -> f16 -> E4M3 and stored once per tile as [128 rows x 576] E4M3 in shared memory: four
//     128-feature SW128 blocks plus an SW64 rope block.  QK reads that tile K-major (kind::f8f6f4, K = 32 per MMA)
//     and PV reads the same bytes as its MN-major V operand -- an SW128 atom is 8 rows x 128 bytes either way.
//   * softmax warpgroup: thread = head = TMEM lane, the S row (128 values) in registers, running max with a lazy
//     rescale (O in TMEM is rescaled only when the max grows by more than 2^8), P = 2^(s - m) <= 256 in E4M3
//     written as the A operand of PV.
//   * split-K over the top-k list when tokens are fewer than SMs; mla_combine_kernel merges the partials.
// Every wait is bounded: a wait past its limit records a status code and the CTA unwinds.
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kMThreads = 512;
constexpr int kMTile = 128;                            // gathered rows per tile: N of QK, K extent of PV
constexpr int kMBlk = kMTile * 128;                    // one 128-feature E4M3 block of a tile (16 KB)
constexpr int kMRopeOff = 4 * kMBlk;                   // SW64 rope block: 128 rows x 64 B
constexpr int kMTileBytes = kMRopeOff + kMTile * 64;   // 72 KB
constexpr int kMPBytes = 128 * kMTile;                 // P: 128 heads x 128 rows, E4M3
constexpr uint32_t kMColO = 0, kMColS = 256, kMColQ = 384;
constexpr float kMTau = 8.f;                           // lazy-rescale threshold, log2 units
constexpr int kMSoftmaxWarps = 4, kMDequantWarps = 8, kMMmaWarp = 12, kMPrefetchWarp = 13;
constexpr int kF4Row = 352, kF8Row = 576;

struct MlaSmem {
  uint64_t tile_full[2];
  uint64_t pv_done[2];
  uint64_t p_full[2];
  uint64_t s_full, s_free, q_ready, fin;
  int idx[2][kMTile];
  uint32_t tmem_base;
  int abort;
};

constexpr int mla_smem_bytes() {
  return 1024 + 2 * kMTileBytes + 2 * kMPBytes + 128 * 64 + static_cast<int>(sizeof(MlaSmem));
}
static_assert(mla_smem_bytes() <= 232448, "shared memory budget");

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void cp_async16(void* smem, const void* g, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(g), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// One dequant thread's share of an NVFP4 row: code bytes [128 s, 128 s + 128) (values 256 s .. 256 s + 255),
// their 16 scales, and rope bytes [32 s, 32 s + 32).
struct RawF4 {
  uint4 code[8];
  uint4 sc;
  uint4 rope[2];
};

__device__ __forceinline__ void load_f4(const uint8_t* row, int s, RawF4& x) {
  if (row) {
#pragma unroll
    for (int i = 0; i < 8; ++i) x.code[i] = ldg16(row + 128 * s + 16 * i);
    x.sc = ldg16(row + 256 + 16 * s);
    x.rope[0] = ldg16(row + 288 + 32 * s);
    x.rope[1] = ldg16(row + 288 + 32 * s + 16);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x.code[i] = make_uint4(0, 0, 0, 0);
    x.sc = make_uint4(0, 0, 0, 0);
    x.rope[0] = x.rope[1] = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ uint32_t u4_get(const uint4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// E2M1 x E4M3 -> f16 (exact) -> E4M3 (round to nearest even): 8 values of one code word, one scale.
__device__ __forceinline__ uint2 f4_word_to_e4m3(uint32_t w, uint32_t scale_h2) {
  uint32_t h[4];
  e2m1x8_to_f16x2x4(w, h);
  const uint32_t e0 = f16x2_to_e4m3x2(hmul2_u32(h[0], scale_h2));
  const uint32_t e1 = f16x2_to_e4m3x2(hmul2_u32(h[1], scale_h2));
  const uint32_t e2 = f16x2_to_e4m3x2(hmul2_u32(h[2], scale_h2));
  const uint32_t e3 = f16x2_to_e4m3x2(hmul2_u32(h[3], scale_h2));
  return make_uint2(e0 | (e1 << 16), e2 | (e3 << 16));
}

__device__ __forceinline__ void store_f4(const RawF4& x, uint8_t* tile, int r, int s) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // code chunk c = 8 s + i holds values 32 c .. 32 c + 31: block c / 4, 16-byte chunks 2 (c % 4) and + 1
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int sbyte = 2 * i + (k >> 1);  // scale of values 32 c + 8 k .. +7 (two scales per code chunk)
      const uint32_t sb = (u4_get(x.sc, sbyte >> 2) >> (8 * (sbyte & 3))) & 0xFFu;
      const uint2 e = f4_word_to_e4m3(u4_get(x.code[i], k), e4m3x2_to_f16x2(static_cast<uint16_t>(sb | (sb << 8))));
      o[2 * k] = e.x;
      o[2 * k + 1] = e.y;
    }
    uint8_t* blk = tile + (2 * s + (i >> 2)) * kMBlk;
    *reinterpret_cast<uint4*>(blk + sw128_chunk(r, 2 * (i & 3))) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(blk + sw128_chunk(r, 2 * (i & 3) + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
  *reinterpret_cast<uint4*>(tile + kMRopeOff + sw64_chunk(r, 2 * s)) = x.rope[0];
  *reinterpret_cast<uint4*>(tile + kMRopeOff + sw64_chunk(r, 2 * s + 1)) = x.rope[1];
}

// E4M3 576-B rows: asynchronous 16-byte copies straight into the swizzled tile (zero-filled for masked rows).
__device__ __forceinline__ void copy_f8(const uint8_t* row, const uint8_t* any, uint8_t* tile, int r, int s) {
  const uint32_t n = row ? 16u : 0u;
  const uint8_t* src = row ? row : any;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = 16 * s + i;  // nope chunk: values 16 c .. 16 c + 15
    cp_async16(tile + (c >> 3) * kMBlk + sw128_chunk(r, c & 7), src + (row ? 16 * c : 0), n);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
    cp_async16(tile + kMRopeOff + sw64_chunk(r, 2 * s + i), src + (row ? 512 + 32 * s + 16 * i : 0), n);
}

template <int FMT>
__global__ void __launch_bounds__(kMThreads, 1) mla_decode_kernel(const MlaDecodeArgs a) {
  constexpr int RB = FMT == kKvNvfp4 ? kF4Row : kF8Row;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = base;                                  // 2 x 72 KB
  uint8_t* sp = tiles + 2 * kMTileBytes;                  // 2 x 16 KB P
  uint8_t* sqr = sp + 2 * kMPBytes;                       // Q rope, SW64 128 x 64 B
  MlaSmem& sm = *reinterpret_cast<MlaSmem*>(sqr + 128 * 64);

  const int t = blockIdx.x, half = blockIdx.y, split = blockIdx.z;
  const int ntiles_all = (a.topk + kMTile - 1) / kMTile;
  const int tile0 = split * a.tiles_per_split;
  const int ntiles = min(ntiles_all, tile0 + a.tiles_per_split) - tile0;
  const int warp = warp_id(), lane = lane_id();
  const int* idx_row = a.idx + static_cast<size_t>(t) * a.idx_stride;

  if (ntiles <= 0) {  // empty split: an empty partial
    if (a.num_splits > 1 && half == 0 && threadIdx.x < a.H)
      a.lse_part[(static_cast<size_t>(split) * a.T + t) * a.H + threadIdx.x] = -INFINITY;
    return;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.tile_full[i], kMDequantWarps * 32);
      mbar_init(&sm.pv_done[i], 1);
      mbar_init(&sm.p_full[i], kMSoftmaxWarps * 32);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, kMSoftmaxWarps * 32);
    mbar_init(&sm.q_ready, kMSoftmaxWarps * 32);
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMMmaWarp) { tmem_alloc(&sm.tmem_base, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp < kMSoftmaxWarps) {
    regs_inc<208>();
    // ---------------------------------------------------------------- softmax: thread = head = TMEM lane
    const int h = threadIdx.x;
    const bool hv = h < a.H;
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    const __nv_bfloat16* qh = reinterpret_cast<const __nv_bfloat16*>(a.q) + (static_cast<size_t>(t) * a.H + h) * 576;
    float amax = 0.f;
    if (hv) {
      for (int c = 0; c < 72; ++c) {
        const uint4 v = ldg16(qh + 8 * c);
        const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(e[k]);
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
    const float qs = amax > 0.f ? amax / 448.f : 1.f;
    const float qinv = 1.f / qs;
    auto q_words = [&](int v0, uint32_t* w, int nw) {  // E4M3 words of values v0 .. v0 + 4 nw
      for (int k = 0; k < nw; k += 2) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (hv) v = ldg16(qh + v0 + 4 * k);
        const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&v);
        const float2 f0 = __bfloat1622float2(e[0]), f1 = __bfloat1622float2(e[1]);
        const float2 f2 = __bfloat1622float2(e[2]), f3 = __bfloat1622float2(e[3]);
        w[k] = static_cast<uint32_t>(f32x2_to_e4m3x2(f0.x * qinv, f0.y * qinv)) |
               (static_cast<uint32_t>(f32x2_to_e4m3x2(f1.x * qinv, f1.y * qinv)) << 16);
        w[k + 1] = static_cast<uint32_t>(f32x2_to_e4m3x2(f2.x * qinv, f2.y * qinv)) |
                   (static_cast<uint32_t>(f32x2_to_e4m3x2(f3.x * qinv, f3.y * qinv)) << 16);
      }
    };
#pragma unroll 1
    for (int b = 0; b < 4; ++b) {
      uint32_t w[32];
      q_words(128 * b, w, 32);
      tmem_st32(tmem + lane_base + kMColQ + 32 * b, w);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t w[4];
      q_words(512 + 16 * c, w, 4);
      *reinterpret_cast<uint4*>(sqr + sw64_chunk(h, c)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    tmem_st_wait();
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&sm.q_ready);

    // waits are made warp-uniform: the warp-collective tcgen05.ld/st and votes below need every lane
    auto wwait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.status, kTimeoutConsumer));
    };
    const float sc2 = qs * a.sm_scale * 1.4426950408889634f;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int buf = j & 1;
      if (!wwait(&sm.s_full, j & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[kMTile];
#pragma unroll
      for (int b = 0; b < 4; ++b) tmem_ld32(tmem + lane_base + kMColS + 32 * b, sr + 32 * b);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&sm.s_free);
      if (!wwait(&sm.tile_full[buf], (j >> 1) & 1)) { ok = false; break; }
      float mt = -INFINITY;
      const int4* ip = reinterpret_cast<const int4*>(sm.idx[buf]);
#pragma unroll
      for (int q4 = 0; q4 < kMTile / 4; ++q4) {
        const int4 iv = ip[q4];
        const int ids[4] = {iv.x, iv.y, iv.z, iv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float v = ids[k] >= 0 ? __uint_as_float(sr[4 * q4 + k]) * sc2 : -INFINITY;
          sr[4 * q4 + k] = __float_as_uint(v);
          mt = fmaxf(mt, v);
        }
      }
      // lazy rescale: keep the reference max unless this tile exceeds it by more than 2^tau
      const bool first = (m_ref == -INFINITY) && (mt > -INFINITY);
      const bool grow = (m_ref > -INFINITY) && (mt > m_ref + kMTau);
      const float alpha = grow ? exp2f(m_ref - mt) : 1.f;
      if (first || grow) m_ref = mt;
      l *= alpha;
      if (__any_sync(0xffffffffu, grow) && j > 0) {
        const int pb = (j - 1) & 1;
        if (!wwait(&sm.pv_done[pb], ((j - 1) >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int b = 0; b < 8; ++b) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kMColO + 32 * b, o);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st32(tmem + lane_base + kMColO + 32 * b, o);
        }
        tmem_st_wait();
      }
      if (j >= 2 && !wwait(&sm.pv_done[buf], ((j - 2) >> 1) & 1)) { ok = false; break; }
      uint8_t* prow = sp + buf * kMPBytes + h * 128;
      float ls = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float v = __uint_as_float(sr[16 * c + 4 * k + e]);
            p[e] = v == -INFINITY ? 0.f : exp2f(v - m_ref);
            ls += p[e];
          }
          w[k] = static_cast<uint32_t>(f32x2_to_e4m3x2(p[0], p[1])) |
                 (static_cast<uint32_t>(f32x2_to_e4m3x2(p[2], p[3])) << 16);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (h & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += ls;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full[buf]);
    }
    if (ok) ok = wwait(&sm.pv_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1);
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const size_t row = static_cast<size_t>(t) * a.H + h;
#pragma unroll 1
      for (int b = 0; b < 8; ++b) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kMColO + 32 * b, o);
        tmem_ld_wait();
        if (!hv) continue;
        const int d0 = 256 * half + 32 * b;
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
    const int r = dt >> 1, s = dt & 1;
    auto row_id = [&](int j) -> int {
      const int p = (tile0 + j) * kMTile + r;
      return (j < ntiles && p < a.topk) ? idx_row[p] : -1;
    };
    auto row_ptr = [&](int id) -> const uint8_t* {
      return id >= 0 ? a.pool + static_cast<size_t>(id) * RB : nullptr;
    };
    int id_cur = row_id(0), id_nxt = row_id(1);
    if constexpr (FMT == kKvNvfp4) {
      RawF4 cur, nxt;
      load_f4(row_ptr(id_cur), s, cur);
      for (int j = 0; j < ntiles; ++j) {
        const int buf = j & 1;
        const int id_n2 = row_id(j + 2);
        load_f4(row_ptr(id_nxt), s, nxt);
        if (j >= 2 && !mbar_wait(&sm.pv_done[buf], ((j - 2) >> 1) & 1, abort, a.status, kTimeoutProducer)) break;
        store_f4(cur, tiles + buf * kMTileBytes, r, s);
        if (s == 0) sm.idx[buf][r] = id_cur;
        fence_proxy_async_smem();
        mbar_arrive(&sm.tile_full[buf]);
        cur = nxt;
        id_cur = id_nxt;
        id_nxt = id_n2;
      }
    } else {
      for (int j = 0; j < ntiles; ++j) {
        const int buf = j & 1;
        if (j >= 2 && !mbar_wait(&sm.pv_done[buf], ((j - 2) >> 1) & 1, abort, a.status, kTimeoutProducer)) break;
        copy_f8(row_ptr(id_cur), a.pool, tiles + buf * kMTileBytes, r, s);
        if (s == 0) sm.idx[buf][r] = id_cur;
        id_cur = id_nxt;
        id_nxt = row_id(j + 2);
        cp_async_wait_all();
        fence_proxy_async_smem();
        mbar_arrive(&sm.tile_full[buf]);
      }
    }
  } else {
    regs_dec<48>();
    if (warp == kMMmaWarp) {
      if (lane == 0) {
        // ------------------------------------------------------------ MMA issue (one thread)
        const uint32_t id_qk = idesc_dense(0, 0, 128, kMTile);
        const uint32_t id_pv = idesc_dense(0, 0, 128, 256) | (1u << 16);  // B (V) MN-major
        const uint32_t tiles_a = smem_u32(tiles), p_a = smem_u32(sp), qr_a = smem_u32(sqr);
        const uint32_t tS = tmem + kMColS, tO = tmem + kMColO, tQ = tmem + kMColQ;
        bool ok = mbar_wait(&sm.q_ready, 0, abort, a.status, kTimeoutMma);
        for (int j = 0; j <= ntiles && ok; ++j) {
          if (j < ntiles) {
            const uint32_t tile = tiles_a + (j & 1) * kMTileBytes;
            if (!(ok = mbar_wait(&sm.tile_full[j & 1], (j >> 1) & 1, abort, a.status, kTimeoutMma))) break;
            if (j >= 1 && !(ok = mbar_wait(&sm.s_free, (j - 1) & 1, abort, a.status, kTimeoutMma))) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 16; ++kk)
              umma_f8_ts(tS, tQ + 8 * kk, desc_sw128(tile + (kk >> 2) * kMBlk + (kk & 3) * 32), id_qk,
                         kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              umma_f8_ss(tS, desc_sw64(qr_a + 32 * kk), desc_sw64(tile + kMRopeOff + 32 * kk), id_qk, 1u);
            umma_commit(&sm.s_full);
          }
          if (j == 0) continue;
          const int i = j - 1, b = i & 1;
          if (!(ok = mbar_wait(&sm.p_full[b], (i >> 1) & 1, abort, a.status, kTimeoutMma))) break;
          tc_fence_after();
          const uint32_t vt = tiles_a + b * kMTileBytes + half * 2 * kMBlk;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f8_ss(tO, desc_sw128(p_a + b * kMPBytes + 32 * kk), desc_mn128(vt + kk * 32 * 128, kMBlk), id_pv,
                       (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.pv_done[b]);
        }
        // every issued MMA has completed before TMEM is released
        umma_commit(&sm.fin);
        mbar_wait(&sm.fin, 0, nullptr, a.status, kTimeoutMma);
      }
    } else if (warp == kMPrefetchWarp) {
      // ------------------------------------------------------------ warm L2 with this split's rows, in order
      const int p0 = tile0 * kMTile, p1 = min(a.topk, (tile0 + ntiles) * kMTile);
      for (int p = p0 + lane; p < p1 && !*abort; p += 32) {
        const int id = idx_row[p];
        if (id >= 0) prefetch_l2(a.pool + static_cast<size_t>(id) * RB, RB);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// out[t, h] = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M); lse in natural log.  One CTA (128 threads) per (t, h).
__global__ void __launch_bounds__(128) mla_combine_kernel(const MlaDecodeArgs a) {
  const int row = blockIdx.x;  // t * H + h
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
  auto kern = mla_decode_kernel<FMT>;
  IOB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kern<<<dim3(a.T, 2, a.num_splits), kMThreads, smem, s>>>(a);
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
  if (a.H < 1 || a.H > 128 || a.topk < 1 || a.idx_stride < a.topk || a.tiles_per_split < 1 || a.num_splits < 1 ||
      a.num_splits > 65535 || (reinterpret_cast<uintptr_t>(a.pool) & 15) || (reinterpret_cast<uintptr_t>(a.q) & 15))
    return cudaErrorInvalidValue;
  if (static_cast<long long>(a.tiles_per_split) * a.num_splits * kMTile < a.topk) return cudaErrorInvalidValue;
  if (a.num_splits > 1 && (!a.o_part || !a.lse_part)) return cudaErrorInvalidValue;
  switch (a.fmt) {
    case kKvNvfp4: return launch_mla<kKvNvfp4>(a, s);
    case kKvFp8: return launch_mla<kKvFp8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace iob
