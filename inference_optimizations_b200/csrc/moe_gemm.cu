// Grouped, block-scaled expert GEMM on the 5th-generation tensor cores, plus the routing prep it reads.
//
//   out[p, n] = sum_k  x[src(p), k] * W_e[n, k]      for every (token, expert) pair p routed to expert e
//
// Weights are FP8 E4M3 with one UE8M0 scale per 128 x 128 block, activations FP8 E4M3 with one UE8M0 scale per
// 1 x 128 block (the DeepSeek-V3 FP8 recipe in its power-of-two-scale form, `moe-gemm/norm-quant-fused/
// pro_norm_quant.py:1-17`).  The scales are applied INSIDE the MMA: `tcgen05.mma ... kind::mxf8f6f4.block_scale`
// with one scale per 32 K-values, fed the 128-block scale replicated four times.
//
// Swap-AB: the weight tile is the 128-row M operand and the expert's tokens are the N operand (N = 16..128), so a
// decode step with a handful of tokens per expert streams every touched weight exactly once at full tensor-core
// width -- the weight-streaming regime the reference's grouped MoE decode GEMMs target
// (`moe-gemm/w4a4-moe-decode-gemm/moe_decode_gemm.py:1-25`, `moe-gemm/cutedsl-grouped-nvfp4/grouped_gemm.py`).
//
// Weights are pre-packed once at load time into UMMA-ready blocks: for (expert, 128-row tile, 128-wide K chunk)
// G tiles of 128 rows x 128 bytes in the SW128 K-major layout, then their G scale-factor atoms (512 bytes each:
// row r = r0 + 32 r1 at byte r0 * 16 + r1 * 4 + j, j = the four 32-wide K sub-blocks).  One plain bulk copy per
// pipeline stage fetches a whole block.  G = 2 packs the gate and up projections of the same 128 FFN columns, so
// one CTA holds both accumulators and the epilogue applies SwiGLU and re-quantizes to FP8 (per-128 UE8M0 scale)
// for the down projection without another pass over memory.
//
// Activation rows are gathered by pair id with cp.async (16-byte chunks, landing in SW128 order) -- the token
// permutation never materializes.  Persistent CTAs (one per SM) walk the list of non-empty (expert, token tile,
// weight tile) items; TMEM holds two accumulator sets when they fit, so the epilogue of one item overlaps the
// mainloop of the next.
//
// Roles (256 threads): warp 0 weight producer (bulk copies), warp 1 MMA issuer + TMEM owner, warps 2-3 activation
// gather (cp.async), warps 4-7 epilogue (TMEM lanes 32 (w - 4) ..).  Every wait is bounded (status + unwind).
#include "common.cuh"
#include "kernels.h"

namespace iob {
namespace {

constexpr int kMgThreads = 256;
constexpr uint32_t kTile = 16384;      // 128 rows x 128 bytes
constexpr uint32_t kSfAtom = 512;      // 128 rows x 4 scale bytes
constexpr int kMaxExperts = 1024;
constexpr int kMaxGemmExperts = 1023;  // buckets per GEMM launch (the work prefix lives in shared memory)
constexpr uint32_t kSmemBudget = 227 * 1024;

// KIND 0: E4M3 operands, UE8M0 scale per 32 K (one scale word per row per 128-byte chunk, 4 MMAs of K = 32 read
// its four bytes).  KIND 1: packed E2M1 operands (256 values per 128-byte chunk), E4M3 scale per 16 K (four words
// per row per chunk: MMA j of K = 64 reads word j's four bytes).
// KIND 2: bf16 operands without block scales (kind::f16, K = 16 per MMA; 64 values per 128-byte chunk): the same
// weight-streaming GEMM for dense bf16 linears (one "expert", every token).
template <int NT, int G, int KIND>
struct Cfg {
  static constexpr int kSfw = KIND == 0 ? 1 : (KIND == 1 ? 4 : 0);   // scale words (atoms) per row per chunk
  static constexpr uint32_t kX = NT * 128;
  static constexpr uint32_t kWBlk = G * (kTile + kSfw * kSfAtom);  // packed weight bytes per stage
  static constexpr uint32_t kRaw = kWBlk + kX + kSfw * kSfAtom;
  static constexpr uint32_t kStage = (kRaw + 1023) / 1024 * 1024;
  static constexpr uint32_t kCtrl = 5120;                         // barriers, work prefix, reduction scratch
  // pipeline stages first (keeping at least 4 KB back), then what is left (up to 16 KB) stages the epilogue's rows
  static constexpr int kStagesFit = (kSmemBudget - kCtrl - 1024 - 4096) / kStage;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr uint32_t kLeft = kSmemBudget - kCtrl - 1024 - kStages * kStage;
  static constexpr uint32_t kEpi = kLeft >= 16384 ? 16384 : (kLeft / 1024) * 1024;
  static constexpr int kAccCols = G * NT;
  static constexpr int kSfCols = KIND == 2 ? 0 : 4 * kSfw * (G + 1);
  static constexpr int kAccBufs = (2 * kAccCols + kSfCols <= 512) ? 2 : 1;
  static constexpr int kUsed = kAccBufs * kAccCols + kSfCols;
  static constexpr uint32_t kTmemCols = kUsed <= 32 ? 32 : kUsed <= 64 ? 64 : kUsed <= 128 ? 128 : kUsed <= 256 ? 256 : 512;
  static constexpr uint32_t kSmem = kCtrl + 1024 + kEpi + kStages * kStage;
  static_assert(kStages >= 2, "pipeline too shallow");
  static_assert(kUsed <= 512, "TMEM overflow");
  static_assert(kSmem <= kSmemBudget, "smem overflow");
};

struct MgCtrl {
  uint64_t w_full[8], x_full[8], empty[8];
  uint64_t acc_full[2], acc_empty[2], fin;
  uint32_t tmem_base;
  int abort;
  int n_items;
  int tile_last;                      // folded split-K: this CTA completed the tile
};

// Shared-memory matrix descriptor for a 32-row x 16-byte no-swizzle source (tcgen05.cp 32x128b): 8-row core
// matrices 128 bytes apart.
__device__ __forceinline__ uint64_t desc_sf(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(128 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
// smem (32 rows x 128 bits) -> TMEM lanes 0..31, broadcast to all four lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// Block-scaled MMAs: scale TMEM addresses carry the byte index in their top two bits, mirrored in the instruction
// descriptor's scale-factor id fields; kind::mxf8f6f4 takes UE8M0 scales per 32 K values (E4M3 operands, K = 32),
// kind::mxf4nvf4 E4M3 scales per 16 (packed E2M1 operands, K = 64).
// Four MMAs per asm statement (MMA i: d[i], a[i], b[i], idesc[i], scale TMEM addresses sfa[i] / sfb[i],
// accumulate iff bit i of acc_mask): issued one per statement, consecutive tcgen05.mma instructions were measured
// ~250 cycles apart from one lane whatever their shape; in batches of four they issue several times faster.
// KIND 0: kind::mxf8f6f4.block_scale (UE8M0 / 32), 1: kind::mxf4nvf4.block_scale.block16, 2: kind::f16 (no scales).
template <int KIND>
__device__ __forceinline__ void umma_bs_x4(const uint32_t (&d)[4], const uint64_t (&a)[4], const uint64_t (&b)[4],
                                           const uint32_t (&idesc)[4], const uint32_t (&sfa)[4],
                                           const uint32_t (&sfb)[4], uint32_t acc_mask) {
  if constexpr (KIND == 2) {
    asm volatile(
        "{\n\t.reg .pred p0, p1, p2, p3;\n\t"
        "setp.ne.b32 p0, %16, 0;\n\tsetp.ne.b32 p1, %17, 0;\n\tsetp.ne.b32 p2, %18, 0;\n\tsetp.ne.b32 p3, %19, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %12, p0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %5, %9, %13, p1;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%2], %6, %10, %14, p2;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], %7, %11, %15, p3;\n\t}\n" ::"r"(d[0]),
        "r"(d[1]), "r"(d[2]), "r"(d[3]), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
        "l"(b[2]), "l"(b[3]), "r"(idesc[0]), "r"(idesc[1]), "r"(idesc[2]), "r"(idesc[3]), "r"(acc_mask & 1u),
        "r"(acc_mask & 2u), "r"(acc_mask & 4u), "r"(acc_mask & 8u));
  } else {
    if constexpr (KIND == 0) {
      asm volatile(
          "{\n\t.reg .pred p0, p1, p2, p3;\n\t"
          "setp.ne.b32 p0, %24, 0;\n\tsetp.ne.b32 p1, %25, 0;\n\tsetp.ne.b32 p2, %26, 0;\n\tsetp.ne.b32 p3, %27, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %4, %8, %12, [%16], [%20], p0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%1], %5, %9, %13, [%17], [%21], p1;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%2], %6, %10, %14, [%18], [%22], p2;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%3], %7, %11, %15, [%19], [%23], p3;\n\t}\n" ::"r"(d[0]),
          "r"(d[1]), "r"(d[2]), "r"(d[3]), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
          "l"(b[2]), "l"(b[3]), "r"(idesc[0]), "r"(idesc[1]), "r"(idesc[2]), "r"(idesc[3]), "r"(sfa[0]), "r"(sfa[1]),
          "r"(sfa[2]), "r"(sfa[3]), "r"(sfb[0]), "r"(sfb[1]), "r"(sfb[2]), "r"(sfb[3]), "r"(acc_mask & 1u),
          "r"(acc_mask & 2u), "r"(acc_mask & 4u), "r"(acc_mask & 8u));
    } else {
      asm volatile(
          "{\n\t.reg .pred p0, p1, p2, p3;\n\t"
          "setp.ne.b32 p0, %24, 0;\n\tsetp.ne.b32 p1, %25, 0;\n\tsetp.ne.b32 p2, %26, 0;\n\tsetp.ne.b32 p3, %27, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %4, %8, %12, [%16], [%20], p0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%1], %5, %9, %13, [%17], [%21], p1;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%2], %6, %10, %14, [%18], [%22], p2;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%3], %7, %11, %15, [%19], [%23], p3;\n\t}\n" ::"r"(d[0]),
          "r"(d[1]), "r"(d[2]), "r"(d[3]), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]),
          "l"(b[2]), "l"(b[3]), "r"(idesc[0]), "r"(idesc[1]), "r"(idesc[2]), "r"(idesc[3]), "r"(sfa[0]), "r"(sfa[1]),
          "r"(sfa[2]), "r"(sfa[3]), "r"(sfb[0]), "r"(sfb[1]), "r"(sfb[2]), "r"(sfb[3]), "r"(acc_mask & 1u),
          "r"(acc_mask & 2u), "r"(acc_mask & 4u), "r"(acc_mask & 8u));
    }
  }
}
// kind::mxf4nvf4 descriptor: E2M1 x E2M1 (format code 1), both K-major, E4M3 scales, M = 128, K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t n) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (0u << 23) | ((128u >> 4) << 24);
}
// kind::mxf8f6f4 block-scaled descriptor: E4M3 x E4M3, both K-major, UE8M0 scales, M = 128.
__host__ __device__ constexpr uint32_t idesc_mxf8(uint32_t n, uint32_t sf_id) {
  return (sf_id << 4) | (0u << 7) | (0u << 10) | ((n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (sf_id << 29);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

__device__ __forceinline__ void mg_trace(const MoeGemmArgs& a, int ev) {
  if (a.trace && blockIdx.x == 0) {
    long long t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    a.trace[ev] = t;
  }
}

// Item i of this launch -> (expert, token tile, weight tile, K split), via the per-expert prefix of item counts.
__device__ __forceinline__ void item_coords(const int* prefix, int E, int n_tiles, int ksplit, int i, int& e, int& tt,
                                            int& nt, int& ks) {
  int lo = 0, hi = E;                 // find e with prefix[e] <= i < prefix[e + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= i) lo = mid; else hi = mid;
  }
  e = lo;
  int local = i - prefix[e];
  ks = local % ksplit;
  local /= ksplit;
  tt = local / n_tiles;
  nt = local - tt * n_tiles;
}
// K chunks [kc0, kc1) of split ks.
__device__ __forceinline__ void split_range(int KC, int ksplit, int ks, int& kc0, int& kc1) {
  const int per = (KC + ksplit - 1) / ksplit;
  kc0 = min(KC, ks * per);
  kc1 = min(KC, kc0 + per);
}

// Activation row of pair p: p / src_div for routed pairs, src_shared_base + p - src_limit for the shared-expert
// rows after them.
__device__ __forceinline__ int src_row(const MoeGemmArgs& a, int p) {
  if (p >= a.src_limit) return a.src_shared_base + p - a.src_limit;
  const int q = p / a.src_div;
  return a.src_group > 0 ? (q / a.src_group) * a.src_group_stride + q % a.src_group : q;
}


// Plain-output epilogue of one item (this thread = TMEM lane = output column n_local of each of the G column tiles):
// groups of kGrp tokens are loaded from TMEM, staged as token rows in shared memory (a warp writes 32 consecutive
// columns of one token: conflict-free), then each warp stores whole rows, one 16-byte store per lane, to the row's
// destination (bf16 out, fp32 split-K partial, or the owning peer's combine buffer).  The code is a short rolled loop
// on purpose: a small GEMM runs each CTA's epilogue once, from a cold instruction cache, and fully unrolled staging
// code cost more in instruction fetch than in execution.  Groups past the item's valid tokens are skipped.
// pid: the item's pair ids in shared memory.  ESZ: bytes per output element.
template <class C, int NT, int G, int ESZ>
__device__ __forceinline__ void store_rows(const MoeGemmArgs& a, uint8_t* epi, const int* pid, uint32_t acc,
                                           float emul, int rows, int nt, int ks, int q, int lane, int n_local) {
  constexpr int kRowB = G * 128 * ESZ;
  constexpr int kGrp = (static_cast<int>(C::kEpi) / kRowB) >= 8 ? 8 : 4;
  static_assert(static_cast<int>(C::kEpi) / kRowB >= 4, "epilogue staging too small");
#pragma unroll 1
  for (int c = 0; c < NT && c < rows; c += kGrp) {
    uint32_t v[G][kGrp];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if constexpr (kGrp == 8) tmem_ld8(acc + g * NT + c, v[g]); else tmem_ld4(acc + g * NT + c, v[g]);
    }
    tmem_ld_wait();
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int t = 0; t < kGrp; ++t) {
        float x = __uint_as_float(v[g][t]) * emul;
        if (a.mode == kMoeOutBf16Weighted) x *= c + t < rows ? a.pair_w[pid[c + t]] : 0.f;
        if constexpr (ESZ == 4)
          reinterpret_cast<float*>(epi)[t * (G * 128) + g * 128 + n_local] = x;
        else
          reinterpret_cast<__nv_bfloat16*>(epi)[t * (G * 128) + g * 128 + n_local] = __float2bfloat16(x);
      }
    }
    named_bar(2, 128);
#pragma unroll 1
    for (int t = q; t < kGrp; t += 4) {
      const int r = c + t;
      if (r >= rows) break;
      const int p = pid[r];
      const uint4* src = reinterpret_cast<const uint4*>(epi + t * kRowB);
      // tensor-parallel broadcast: the row goes to every rank (own first, then the next ranks in ring order)
      const int nd = (ESZ == 2 && a.out_peers && a.out_bcast > 0) ? a.out_bcast : 1;
#pragma unroll 1
      for (int d = 0; d < nd; ++d) {
        char* dst;
        if constexpr (ESZ == 4) {
          dst = reinterpret_cast<char*>(a.out) +
                ((static_cast<size_t>(ks) * a.split_rows + p) * a.out_stride + static_cast<size_t>(nt) * G * 128) * 4;
        } else if (a.out_peers) {               // expert parallelism: the row goes to its token's owner
          const bool bc = a.out_bcast > 0, sh = !bc && p >= a.pairs_total;
          const int rr = bc ? (a.out_rank + d) % a.out_bcast : (sh ? a.out_rank : p / a.out_div);
          const long long row = bc ? p : (sh ? a.out_shared_base + (p - a.pairs_total) : p % a.out_div);
          dst = reinterpret_cast<char*>(a.out_peers[rr]) + a.out_offset +
                (row * a.out_stride + static_cast<long long>(nt) * G * 128) * 2;
        } else {
          dst = reinterpret_cast<char*>(a.out) +
                (static_cast<size_t>(p) * a.out_stride + static_cast<size_t>(nt) * G * 128) * 2;
        }
#pragma unroll 1
        for (int k = lane; k < kRowB / 16; k += 32) reinterpret_cast<uint4*>(dst)[k] = src[k];
      }
    }
    named_bar(2, 128);
  }
}

// Folded split-K reduction (the epilogue's 128 threads, after this split's partial rows were stored): the split that
// brings the tile's counter to ksplit sums the ksplit partials of the tile's rows in split order (as splitk_reduce:
// deterministic, whichever split finishes last) and writes the final rows; it re-arms the counter.
template <int G>
__device__ __forceinline__ void split_reduce_tail(const MoeGemmArgs& a, MgCtrl& ctl, int tile, const int* pid,
                                                  int rows, int nt) {
  __threadfence();                    // this split's partial rows are visible device-wide before it is counted
  named_bar(2, 128);
  if (threadIdx.x == 128) {
    const int old = atomicAdd(a.tile_cnt + tile, 1);
    const int last = old == a.ksplit - 1;
    if (last) a.tile_cnt[tile] = 0;
    ctl.tile_last = last;
  }
  named_bar(2, 128);
  const bool last = ctl.tile_last;
  named_bar(2, 128);                  // every thread read the flag before the next item may overwrite it
  if (!last) return;
  __threadfence();
  const int tid = threadIdx.x - 128;
  const float* part = reinterpret_cast<const float*>(a.out);
  constexpr int kQuads = G * 128 / 4;                 // float4 columns of the tile
#pragma unroll 1
  for (int e = tid; e < rows * kQuads; e += 128) {    // (row, float4 column) over all 128 threads
    const int r = e / kQuads, c4 = e - r * kQuads;
    const int p = pid[r];
    const size_t col = static_cast<size_t>(nt) * G * 128 + 4 * c4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < a.ksplit; ++k) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(
          part + (static_cast<size_t>(k) * a.split_rows + p) * a.out_stride + col));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (a.red_f32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.red_out) + static_cast<size_t>(p) * a.red_stride + col) =
          acc;
    } else {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&lo);
      w.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.red_out) + static_cast<size_t>(p) * a.red_stride +
                                col) = w;
    }
  }
}

template <int NT, int G, int KIND>
__global__ void __launch_bounds__(kMgThreads, 1) moe_gemm_kernel(const MoeGemmArgs a) {
  using C = Cfg<NT, G, KIND>;
  constexpr int kSfw = C::kSfw;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  MgCtrl& ctl = *reinterpret_cast<MgCtrl*>(base);
  int* prefix = reinterpret_cast<int*>(base + 256);                // [E + 1], E <= kMaxGemmExperts
  float* red = reinterpret_cast<float*>(base + 4608);              // [4 warps][32 tokens]
  uint8_t* epi = base + C::kCtrl;                                  // epilogue row staging (kEpi bytes)
  uint8_t* stages = base + C::kCtrl + C::kEpi;
  const int warp = warp_id(), lane = lane_id();
  volatile int* abort = &ctl.abort;

  if (threadIdx.x == 0) {
    mg_trace(a, kMgEvStart);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&ctl.w_full[s], 1);
      mbar_init(&ctl.x_full[s], 64);
      mbar_init(&ctl.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl.acc_full[b], 1);
      mbar_init(&ctl.acc_empty[b], 128);
    }
    mbar_init(&ctl.fin, 1);
    ctl.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl.tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  if (!a.static_index) griddep_wait();  // expert offsets / pair ids come from the previous kernel
  if (warp == 2) {                    // per-expert prefix of item counts (warp scan over chunks of experts)
    const int per = (a.E + 31) / 32;
    int local = 0;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < a.E) {
        const int cnt = a.expert_off[e + 1] - a.expert_off[e];
        local += (cnt + NT - 1) / NT * a.n_tiles * a.ksplit;
      }
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < a.E) {
        prefix[e] = run;
        const int cnt = a.expert_off[e + 1] - a.expert_off[e];
        run += (cnt + NT - 1) / NT * a.n_tiles * a.ksplit;
      }
    }
    if (lane == 31) {
      prefix[a.E] = incl;
      ctl.n_items = incl;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int n_items = ctl.n_items;
  const uint32_t tmem = ctl.tmem_base;
  if (threadIdx.x == 0) mg_trace(a, kMgEvSetup);
  griddep_launch();                   // the next kernel may be scheduled as this grid's CTAs retire
  const uint32_t sfa_col = C::kAccBufs * C::kAccCols;
  const uint32_t sfb_col = sfa_col + 4 * G * kSfw;

  if (warp == 0) {
    // ---------------------------------------------------------------- weight producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        int e, tt, nt, ks, kc0, kc1;
        item_coords(prefix, a.E, a.n_tiles, a.ksplit, i, e, tt, nt, ks);
        split_range(a.KC, a.ksplit, ks, kc0, kc1);
        const uint8_t* src = a.wpack + ((static_cast<size_t>(e) * a.n_tiles + nt) * a.KC) * C::kWBlk;
        for (int kc = kc0; kc < kc1; ++kc, ++it) {
          const uint32_t s = it % C::kStages;
          if (it >= static_cast<uint32_t>(C::kStages) &&
              !mbar_wait(&ctl.empty[s], ((it / C::kStages) - 1) & 1, abort, a.status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + s * C::kStage;
          if (it == 0) mg_trace(a, kMgEvFirstCopy);
          mbar_expect_tx(&ctl.w_full[s], C::kWBlk);
          const uint8_t* blk = src + static_cast<size_t>(kc) * C::kWBlk;
          bulk_g2s(st, blk, G * kTile, &ctl.w_full[s]);
          bulk_g2s(st + G * kTile + C::kX, blk + G * kTile, G * kSfw * kSfAtom, &ctl.w_full[s]);
        }
      }
      // drain: every issued copy has landed before the CTA can exit (bounded, regardless of abort)
      const uint32_t first = it > static_cast<uint32_t>(C::kStages) ? it - C::kStages : 0;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&ctl.w_full[j % C::kStages], (j / C::kStages) & 1, nullptr,
                                                      a.status, kTimeoutProducer);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t it = 0;
      int li = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++li) {
        const int buf = li % C::kAccBufs, use = li / C::kAccBufs;
        if (use > 0 && !mbar_wait(&ctl.acc_empty[buf], (use - 1) & 1, abort, a.status, kTimeoutMma)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * C::kAccCols;
        int e_, tt_, nt_, ks, kc0, kc1;
        item_coords(prefix, a.E, a.n_tiles, a.ksplit, i, e_, tt_, nt_, ks);
        split_range(a.KC, a.ksplit, ks, kc0, kc1);
        for (int kc = kc0; kc < kc1; ++kc, ++it) {
          const uint32_t s = it % C::kStages, ph = (it / C::kStages) & 1;
          if (!mbar_wait(&ctl.w_full[s], ph, abort, a.status, kTimeoutMma) ||
              !mbar_wait(&ctl.x_full[s], ph, abort, a.status, kTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();
          if (it == 0) mg_trace(a, kMgEvFirstReady);
          const uint32_t st = smem_u32(stages + s * C::kStage);
          const uint32_t x_s = st + G * kTile;
          const uint32_t sfa_s = x_s + C::kX;
          const uint32_t sfb_s = sfa_s + G * kSfw * kSfAtom;
#pragma unroll
          for (int w = 0; w < G * kSfw; ++w) tmem_cp_sf(tmem + sfa_col + 4 * w, desc_sf(sfa_s + w * kSfAtom));
#pragma unroll
          for (int w = 0; w < kSfw; ++w) tmem_cp_sf(tmem + sfb_col + 4 * w, desc_sf(sfb_s + w * kSfAtom));
          (void)sfb_s;
          // the 4 G MMAs of this stage (K steps j outer, weight tiles g inner), four per asm statement
          static_assert((4 * G) % 4 == 0, "MMAs come in batches of four");
          uint32_t d4[4], i4[4], fa4[4], fb4[4], mask = 0;
          uint64_t a4[4], b4[4];
          int n4 = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
              d4[n4] = acc + g * NT;
              a4[n4] = desc_sw128(st + g * kTile + 32 * j);
              b4[n4] = desc_sw128(x_s + 32 * j);
              if constexpr (KIND == 2) {
                i4[n4] = idesc_dense(1, 1, 128, NT);
                fa4[n4] = fb4[n4] = 0;
              } else if constexpr (KIND == 0) {
                i4[n4] = idesc_mxf8(NT, j);
                fa4[n4] = (tmem + sfa_col + 4 * g) | (static_cast<uint32_t>(j) << 30);
                fb4[n4] = (tmem + sfb_col) | (static_cast<uint32_t>(j) << 30);
              } else {
                i4[n4] = idesc_nvf4(NT);
                fa4[n4] = tmem + sfa_col + 4 * (g * 4 + j);
                fb4[n4] = tmem + sfb_col + 4 * j;
              }
              if (kc != kc0 || j) mask |= 1u << n4;
              if (++n4 == 4) {
                umma_bs_x4<KIND>(d4, a4, b4, i4, fa4, fb4, mask);
                n4 = 0;
                mask = 0;
              }
            }
          }
          umma_commit(&ctl.empty[s]);
        }
        if (!ok) break;
        umma_commit(&ctl.acc_full[buf]);
        mg_trace(a, kMgEvLastMma);
      }
      umma_commit(&ctl.fin);          // every MMA issued above has completed before TMEM is freed
      mbar_wait(&ctl.fin, 0, nullptr, a.status, kTimeoutMma);
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------- activation gather (64 threads)
    griddep_wait();                   // activations (and their scales) are the previous kernel's output
    const int t64 = threadIdx.x - 64;
    uint32_t it = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
      int e, tt, nt, ks, kc0, kc1;
      item_coords(prefix, a.E, a.n_tiles, a.ksplit, i, e, tt, nt, ks);
      split_range(a.KC, a.ksplit, ks, kc0, kc1);
      const int row0 = a.expert_off[e] + tt * NT;
      const int rows = min(NT, a.expert_off[e + 1] - row0);
      // rows handled by this thread: r = t64 / 8 + 8 m (chunk t64 % 8); scale rows t64, t64 + 64
      constexpr int kRpt = NT / 8;
      const uint8_t* xrow[kRpt];
#pragma unroll
      for (int m = 0; m < kRpt; ++m) {
        const int r = t64 / 8 + 8 * m;
        xrow[m] = r < rows ? a.x + static_cast<size_t>(src_row(a, a.pairs[row0 + r])) * a.x_stride : nullptr;
      }
      const uint32_t* srow[2];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int r = t64 + 64 * m;
        srow[m] = (KIND != 2 && r < rows && r < NT)
                      ? a.x_scale + static_cast<size_t>(src_row(a, a.pairs[row0 + r])) * (a.KC * kSfw)
                      : nullptr;
      }
      for (int kc = kc0; kc < kc1; ++kc, ++it) {
        const uint32_t s = it % C::kStages;
        if (it >= static_cast<uint32_t>(C::kStages) &&
            !mbar_wait(&ctl.empty[s], ((it / C::kStages) - 1) & 1, abort, a.status, kTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t x_s = smem_u32(stages + s * C::kStage) + G * kTile;
        const uint32_t sfb_s = x_s + C::kX + G * kSfw * kSfAtom;
        const int c = t64 & 7;
#pragma unroll
        for (int m = 0; m < kRpt; ++m) {
          const int r = t64 / 8 + 8 * m;
          if (xrow[m]) cp_async16(x_s + sw128_chunk(r, c), xrow[m] + kc * 128 + c * 16);
        }
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const int r = t64 + 64 * m;
          if (srow[m]) {
#pragma unroll
            for (int w = 0; w < kSfw; ++w)
              cp_async4(sfb_s + w * kSfAtom + (r & 31) * 16 + (r >> 5) * 4, srow[m] + kc * kSfw + w);
          }
        }
        cp_async_arrive_noinc(&ctl.x_full[s]);
      }
    }
    cp_async_wait_all();
  } else {
    // ---------------------------------------------------------------- epilogue (128 threads)
    const int q = warp - 4;                       // TMEM lane quarter
    const int n_local = q * 32 + lane;            // weight row within the 128-row tile
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int li = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++li) {
      int e, tt, nt, ks;
      item_coords(prefix, a.E, a.n_tiles, a.ksplit, i, e, tt, nt, ks);
      const int row0 = a.expert_off[e] + tt * NT;
      const int rows = min(NT, a.expert_off[e + 1] - row0);
      const int buf = li % C::kAccBufs, use = li / C::kAccBufs;
      // plain modes: the item's pair ids go to shared memory with one load per thread, issued before the
      // accumulator wait so their latency hides under the mainloop (the previous item's row stores ended with a
      // barrier, so the array is free; the SwiGLU mode uses this scratch for its row maxima instead)
      int* pid = reinterpret_cast<int*>(red);
      if (a.mode != kMoeOutSwigluQuant) {
        const int tid = threadIdx.x - 128;
        if (tid < rows) pid[tid] = a.pairs[row0 + tid];
        named_bar(2, 128);
      }
      if (!mbar_wait(&ctl.acc_full[buf], use & 1, abort, a.status, kTimeoutConsumer)) break;
      tc_fence_after();
      if (li == 0 && threadIdx.x == 128) mg_trace(a, kMgEvAccSeen);
      const uint32_t acc = tmem + lane_addr + buf * C::kAccCols;
      const float emul = a.out_mul * (a.expert_mul ? a.expert_mul[e] : 1.f);
      constexpr int kChunk = NT < 32 ? NT : 32;
      if (a.mode == kMoeOutF32Split) {               // split-K partial, summed by splitk_reduce or folded in
        store_rows<C, NT, G, 4>(a, epi, pid, acc, emul, rows, nt, ks, q, lane, n_local);
        if (a.red_out) split_reduce_tail<G>(a, ctl, i / a.ksplit, pid, rows, nt);
      } else if (a.mode != kMoeOutSwigluQuant) {
        store_rows<C, NT, G, 2>(a, epi, pid, acc, emul, rows, nt, ks, q, lane, n_local);
      } else
      for (int c0 = 0; c0 < NT; c0 += kChunk) {
        uint32_t v0[kChunk], v1[kChunk];
        if constexpr (kChunk == 16) tmem_ld16(acc + c0, v0); else tmem_ld32(acc + c0, v0);
        if constexpr (G == 2) {
          if constexpr (kChunk == 16) tmem_ld16(acc + NT + c0, v1); else tmem_ld32(acc + NT + c0, v1);
        }
        tmem_ld_wait();
        if (a.mode == kMoeOutSwigluQuant && KIND == 0) {
          float h[kChunk];
#pragma unroll
          for (int t = 0; t < kChunk; ++t) {
            const float g = __uint_as_float(v0[t]) * emul;
            const float u = G == 2 ? __uint_as_float(v1[t]) * emul : 1.f;
            h[t] = g / (1.f + __expf(-g)) * u;
            const float m = warp_max(fabsf(h[t]));
            if (lane == 0) red[q * 32 + t] = m;
          }
          named_bar(1, 128);
#pragma unroll
          for (int t = 0; t < kChunk; ++t) {
            const int r = c0 + t;
            const float amax = fmaxf(fmaxf(red[t], red[32 + t]), fmaxf(red[64 + t], red[96 + t]));
            const uint32_t eb = ue8m0_for(amax);
            if (r < rows) {
              const int p = a.pairs[row0 + r];
              const float inv = __uint_as_float((254u - eb) << 23);          // 2^-(eb - 127)
              reinterpret_cast<uint8_t*>(a.out)[static_cast<size_t>(p) * a.out_stride + nt * 128 + n_local] =
                  float_to_e4m3(h[t] * inv);
              if (n_local == 0) a.out_scale[static_cast<size_t>(p) * a.out_scale_stride + nt] = eb * 0x01010101u;
            }
          }
          named_bar(1, 128);
        } else if (a.mode == kMoeOutSwigluQuant) {
          // NVFP4 output: 16 consecutive columns (16 lanes) share one E4M3 scale; element 2i in the low nibble
#pragma unroll
          for (int t = 0; t < kChunk; ++t) {
            const float g = __uint_as_float(v0[t]) * emul;
            const float u = G == 2 ? __uint_as_float(v1[t]) * emul : 1.f;
            const float h = g / (1.f + __expf(-g)) * u;
            float m = fabsf(h);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const uint8_t sb = nvfp4_block_scale(m);
            const uint32_t code = e2m1_code(h / e4m3_to_float(sb));
            const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
            const int r = c0 + t;
            if (r < rows) {
              const int p = a.pairs[row0 + r];
              const int col = nt * 128 + n_local;
              if ((lane & 1) == 0)
                reinterpret_cast<uint8_t*>(a.out)[static_cast<size_t>(p) * a.out_stride + col / 2] =
                    static_cast<uint8_t>(code | (hi << 4));
              if ((lane & 15) == 0)
                reinterpret_cast<uint8_t*>(a.out_scale)[static_cast<size_t>(p) * a.out_scale_stride * 4 + col / 16] =
                    sb;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctl.acc_empty[buf]);
      if (threadIdx.x == 128) mg_trace(a, kMgEvEpiDone);
    }
    // rows stored into peers' memory must be visible system-wide before the next kernel's barrier releases its
    // flag (that release orders only the releasing thread's own writes)
    if (a.out_peers) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0) mg_trace(a, kMgEvEnd);
}

template <int NT, int G, int KIND>
cudaError_t launch_mg(const MoeGemmArgs& a, cudaStream_t s) {
  using C = Cfg<NT, G, KIND>;
  static bool attr = false;
  if (!attr) {
    IOB_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<NT, G, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(C::kSmem)));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_ctas);
  cfg.blockDim = dim3(kMgThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute pdl_attr[1];
  pdl_attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl_attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl_attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_gemm_kernel<NT, G, KIND>, a);
}

// ------------------------------------------------------------------------------------------------ routing prep
// Pairs p (token p / topk, slot p % topk) whose expert lies in [e0, e0 + E) are bucketed by expert: off[nb + 1] and
// pairs sorted by expert (order inside an expert is irrelevant: each pair is its own MMA column).  With a shared
// bucket (nb = E + 1) the `extra` rows P .. P + extra - 1 all go to bucket E (a shared expert run as one more group
// of the same launch; extra may be 0).
__global__ void __launch_bounds__(1024) moe_align_kernel(const int* ids, int P, int e0, int E, int nb, int extra,
                                                         int* off, int* pairs) {
  griddep_launch();
  __shared__ int cnt[kMaxExperts + 2];
  __shared__ int pos[kMaxExperts + 2];
  for (int e = threadIdx.x; e < nb; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = ids[p] - e0;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  if (threadIdx.x == 0 && nb > E) cnt[E] = extra;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < nb; ++e) {
      off[e] = run;
      pos[e] = run;
      run += cnt[e];
    }
    off[nb] = run;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = ids[p] - e0;
    if (e >= 0 && e < E) pairs[atomicAdd(&pos[e], 1)] = p;
  }
  for (int t = threadIdx.x; t < extra; t += blockDim.x) pairs[pos[E] + t] = P + t;
}

// y[t] = sum_k w[t, k] * rows[t * topk + k] (+ rows[shared_base + t] when shared_base >= 0), fp32 in slot order,
// bf16 out.  w null: the rows already carry their routing weights.
__global__ void moe_combine_kernel(const __nv_bfloat16* rows, int T, int topk, int H, int shared_base,
                                   const float* w, __nv_bfloat16* y) {
  griddep_launch();
  const int t = blockIdx.x;           // grid (T, column blocks): a decode step's few tokens still spread over SMs
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < H / 8; c += gridDim.y * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k <= topk; ++k) {
      if (k == topk && shared_base < 0) break;
      const size_t r = k < topk ? static_cast<size_t>(t) * topk + k : static_cast<size_t>(shared_base) + t;
      const float wk = (k < topk && w) ? w[t * topk + k] : 1.f;
      if (wk == 0.f) continue;        // a pair this launch did not compute (experts of other ranks): row unwritten
      const uint4 u = *reinterpret_cast<const uint4*>(rows + r * H + c * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += wk * f.x;
        acc[2 * i + 1] += wk * f.y;
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(y + static_cast<size_t>(t) * H + c * 8) = o;
  }
}

// RMSNorm (optional) + quantization of a row for the block-scaled GEMM.  fmt 0: FP8 E4M3 with one UE8M0 scale per
// 128 columns (scale words replicate the exponent byte four times: the layout the GEMM gathers).  fmt 1: NVFP4 --
// E2M1 pairs (element 2i in the low nibble) with one E4M3 scale e4m3(clamp(amax / 6, 2^-9, 448)) per 16 columns.
// `w` null: quantize x as is.
// Quantize one row of H values given by val(c) (already rounded to bf16): fmt 0 = E4M3 + one UE8M0 scale per 128
// (stored as four identical bytes, the layout the block-scaled GEMM reads), fmt 1 = NVFP4 (E2M1 pairs + one E4M3 scale
// per 16).  Called by every thread of the block.
// part / parts: this CTA's share of the row's column groups (a row spread over several CTAs when there are few rows).
template <class Val>
__device__ __forceinline__ void quant_row(Val val, int row, int H, int fmt, uint8_t* q, uint32_t* sc, int part = 0,
                                          int parts = 1) {
  if (fmt == 0) {
    // one warp per 128-column group: 4 values per lane
    const int nw = blockDim.x / 32;
    for (int g = part * nw + warp_id(); g < H / 128; g += parts * nw) {
      float v[4];
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = val(g * 128 + lane_id() * 4 + j);
        m = fmaxf(m, fabsf(v[j]));
      }
      m = warp_max(m);
      const uint32_t eb = ue8m0_for(m);
      const float s = __uint_as_float((254u - eb) << 23);
      uint32_t packed = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) packed |= static_cast<uint32_t>(float_to_e4m3(v[j] * s)) << (8 * j);
      reinterpret_cast<uint32_t*>(q + static_cast<size_t>(row) * H + g * 128)[lane_id()] = packed;
      if (lane_id() == 0) sc[static_cast<size_t>(row) * (H / 128) + g] = eb * 0x01010101u;
    }
  } else {
    // one thread per 16-column block
    uint8_t* sb_row = reinterpret_cast<uint8_t*>(sc) + static_cast<size_t>(row) * (H / 16);
    for (int b = part * blockDim.x + threadIdx.x; b < H / 16; b += parts * blockDim.x) {
      float v[16];
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[j] = val(b * 16 + j);
        m = fmaxf(m, fabsf(v[j]));
      }
      const uint8_t sb = nvfp4_block_scale(m);
      const float sf = e4m3_to_float(sb);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) lo |= e2m1_code(v[j] / sf) << (4 * j);
#pragma unroll
      for (int j = 0; j < 8; ++j) hi |= e2m1_code(v[8 + j] / sf) << (4 * j);
      *reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * (H / 2) + b * 8) = make_uint2(lo, hi);
      sb_row[b] = sb;
    }
  }
}

__global__ void rmsnorm_quant_kernel(const __nv_bfloat16* x, const __nv_bfloat16* w, float eps, float plus_one,
                                     int H, int fmt, uint8_t* q, uint32_t* sc) {
  griddep_launch();                   // a GEMM launched after this may set up and stream weights meanwhile
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + static_cast<size_t>(row) * H;
  __shared__ float red[32];
  float inv = 1.f;
  if (w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float v = __bfloat162float(xr[i]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane_id() == 0) red[warp_id()] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    inv = rsqrtf(red[0] / H + eps);
  }
  quant_row([&](int c) {
    float f = __bfloat162float(xr[c]);
    if (w) f = __bfloat162float(__float2bfloat16(f * inv * (__bfloat162float(w[c]) + plus_one)));
    return f;
  }, row, H, fmt, q, sc, blockIdx.y, gridDim.y);
}

// act(gate) * up -> quantized, one pass over gate_up [T, 2F] (gate = first F columns): the GEMM1 -> GEMM2 glue of a
// block-scaled dense MLP.  The product is rounded to bf16 before quantization, so the output equals quantizing the
// bf16 act_mul result bit for bit (the reference's one-pass `attention/gemma-fused-glue/gelu_tanh_quant.cuh:1-25`).
template <bool GELU>
__global__ void act_quant_kernel(const __nv_bfloat16* gu, int F, int fmt, uint8_t* q, uint32_t* sc) {
  const int row = blockIdx.x;
  const __nv_bfloat16* g = gu + static_cast<size_t>(row) * 2 * F;
  quant_row([&](int c) {
    const float gv = __bfloat162float(g[c]);
    const float a = GELU ? gelu_tanh_f(gv) : gv / (1.f + __expf(-gv));
    return __bfloat162float(__float2bfloat16(a * __bfloat162float(g[F + c])));
  }, row, F, fmt, q, sc);
}

// One CTA per output row: the K splits' fp32 partials summed in split order, then rounded once to bf16 (OutT = bf16)
// or kept in fp32 (OutT = float: router logits).
template <class OutT>
__global__ void splitk_reduce_kernel(const float* part, int ksplit, int rows, int N, OutT* out,
                                     const long long* peers, long long peer_offset, int nbcast, int rank) {
  griddep_launch();
  const int r = blockIdx.x;
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < N / 4; c += gridDim.y * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < ksplit; ++k) {
      const float4 v = reinterpret_cast<const float4*>(part + (static_cast<size_t>(k) * rows + r) * N)[c];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if constexpr (sizeof(OutT) == 4) {
      reinterpret_cast<float4*>(out + static_cast<size_t>(r) * N)[c] = acc;
    } else {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&lo);
      w.y = *reinterpret_cast<const uint32_t*>(&hi);
      if (!peers) {
        reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * N)[c] = w;
      } else {
        // tensor-parallel push: the row into this rank's slot of every rank's buffer (own first)
        for (int d = 0; d < nbcast; ++d) {
          char* dst = reinterpret_cast<char*>(peers[(rank + d) % nbcast]) + peer_offset;
          reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(dst) + static_cast<size_t>(r) * N)[c] = w;
        }
      }
    }
  }
  // the rows stored into peers' memory are visible system-wide before the next kernel releases its ready flag
  if (peers) __threadfence_system();
}

}  // namespace

cudaError_t moe_gemm(const MoeGemmArgs& a, cudaStream_t s) {
  if (a.ksplit < 1 || a.ksplit > a.KC || (a.ksplit > 1 && a.mode != kMoeOutF32Split) ||
      (a.mode == kMoeOutF32Split && a.out_peers) || (a.red_out && (a.mode != kMoeOutF32Split || !a.tile_cnt)) ||
      (a.red_out && (a.red_stride % 4 || reinterpret_cast<uintptr_t>(a.red_out) % 16)))
    return cudaErrorInvalidValue;
  if (a.src_group < 0 || (a.src_group > 0 && a.src_group_stride < a.src_group)) return cudaErrorInvalidValue;
  if (a.out_bcast < 0 || (a.out_bcast > 0 && (!a.out_peers || a.out_rank < 0 || a.out_rank >= a.out_bcast ||
                                               (a.mode != kMoeOutBf16 && a.mode != kMoeOutBf16Weighted))))
    return cudaErrorInvalidValue;
  if (a.mode != kMoeOutSwigluQuant) {         // plain epilogues store 16-byte row segments
    const int esz = a.mode == kMoeOutF32Split ? 4 : 2;
    if ((static_cast<long long>(a.out_stride) * esz) % 16 || a.out_offset % 16 ||
        (!a.out_peers && reinterpret_cast<uintptr_t>(a.out) % 16))
      return cudaErrorInvalidValue;
  }
  if (a.E <= 0 || a.E > kMaxGemmExperts || a.KC <= 0 || a.n_tiles <= 0 || a.num_ctas <= 0 || a.src_div <= 0 ||
      (a.x_stride % 16) || (reinterpret_cast<uintptr_t>(a.x) % 16) || (reinterpret_cast<uintptr_t>(a.wpack) % 16) ||
      (a.mode == kMoeOutSwigluQuant && (a.G != 2 || a.kind == 2)) || a.kind < 0 || a.kind > 2)
    return cudaErrorInvalidValue;
#define IOB_MG(NT_, G_, K_) \
  if (a.NT == NT_ && a.G == G_ && a.kind == K_) return launch_mg<NT_, G_, K_>(a, s);
  IOB_MG(16, 1, 0) IOB_MG(32, 1, 0) IOB_MG(64, 1, 0) IOB_MG(128, 1, 0)
  IOB_MG(16, 2, 0) IOB_MG(32, 2, 0) IOB_MG(64, 2, 0) IOB_MG(128, 2, 0)
  IOB_MG(16, 1, 1) IOB_MG(32, 1, 1) IOB_MG(64, 1, 1) IOB_MG(128, 1, 1)
  IOB_MG(16, 2, 1) IOB_MG(32, 2, 1) IOB_MG(64, 2, 1) IOB_MG(128, 2, 1)
  IOB_MG(16, 1, 2) IOB_MG(32, 1, 2) IOB_MG(64, 1, 2) IOB_MG(128, 1, 2)
  IOB_MG(16, 2, 2) IOB_MG(32, 2, 2) IOB_MG(64, 2, 2) IOB_MG(128, 2, 2)
#undef IOB_MG
  return cudaErrorInvalidValue;
}

cudaError_t splitk_reduce(const float* part, int ksplit, int rows, int N, void* out, bool out_f32, cudaStream_t s,
                          const long long* peers, long long peer_offset, int nbcast, int rank) {
  if (rows == 0) return cudaSuccess;
  if (N % 4 || ksplit < 1) return cudaErrorInvalidValue;
  if (peers && (out_f32 || nbcast < 1 || rank < 0 || rank >= nbcast || peer_offset % 16)) return cudaErrorInvalidValue;
  // (row, column block of 256 float4s): a wide output is reduced by enough CTAs to stream the partials at full rate
  const dim3 grid(rows, (N / 4 + 255) / 256);
  if (out_f32)
    splitk_reduce_kernel<float><<<grid, 256, 0, s>>>(part, ksplit, rows, N, static_cast<float*>(out), nullptr, 0, 0, 0);
  else
    splitk_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(part, ksplit, rows, N, static_cast<__nv_bfloat16*>(out),
                                                             peers, peer_offset, nbcast, rank);
  return cudaGetLastError();
}

cudaError_t moe_align(const int* ids, int P, int e0, int E, int shared_bucket, int extra, int* off, int* pairs,
                      cudaStream_t s) {
  if (E <= 0 || E > kMaxExperts || (!shared_bucket && extra)) return cudaErrorInvalidValue;
  moe_align_kernel<<<1, 1024, 0, s>>>(ids, P, e0, E, E + (shared_bucket ? 1 : 0), extra, off, pairs);
  return cudaGetLastError();
}

cudaError_t moe_combine(const void* rows, int T, int topk, int H, int shared_base, const float* w, void* y,
                        cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (H % 8) return cudaErrorInvalidValue;
  moe_combine_kernel<<<dim3(T, (H / 8 + 127) / 128), 128, 0, s>>>(static_cast<const __nv_bfloat16*>(rows), T, topk,
                                                                  H, shared_base, w, static_cast<__nv_bfloat16*>(y));
  return cudaGetLastError();
}

cudaError_t rmsnorm_quant(const void* x, const void* w, float eps, float plus_one, int T, int H, int fmt, uint8_t* q,
                          uint32_t* sc, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if ((fmt == 0 && H % 128) || (fmt == 1 && H % 64) || fmt < 0 || fmt > 1) return cudaErrorInvalidValue;
  // without a norm (no row-wide sum) a row may spread over several CTAs: with few rows each warp then quantizes one
  // or two column groups instead of walking the row (a chain of dependent loads per warp at decode sizes)
  int parts = 1;
  if (!w) {
    const int per_cta = fmt == 0 ? 8 * 128 : 256 * 16;   // columns one pass of a 256-thread CTA covers
    parts = max(1, min((H + per_cta - 1) / per_cta, (2 * 148 + T - 1) / T));
  }
  rmsnorm_quant_kernel<<<dim3(T, parts), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                      static_cast<const __nv_bfloat16*>(w), eps, plus_one, H, fmt,
                                                      q, sc);
  return cudaGetLastError();
}

cudaError_t act_quant(const void* gate_up, int T, int F, bool gelu, int fmt, uint8_t* q, uint32_t* sc, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if ((fmt == 0 && F % 128) || (fmt == 1 && F % 64) || fmt < 0 || fmt > 1) return cudaErrorInvalidValue;
  const auto* gu = static_cast<const __nv_bfloat16*>(gate_up);
  if (gelu)
    act_quant_kernel<true><<<T, 256, 0, s>>>(gu, F, fmt, q, sc);
  else
    act_quant_kernel<false><<<T, 256, 0, s>>>(gu, F, fmt, q, sc);
  return cudaGetLastError();
}

}  // namespace iob
