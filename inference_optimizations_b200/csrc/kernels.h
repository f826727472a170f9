// Host-side launch API of the CUDA kernels.  Plain pointers and a stream: no torch types, so the .cu files compile
// without torch headers and the same launchers serve the torch bindings (bindings.cpp) and C callers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <cuda_bf16.h>

namespace iob {

enum KvFormat : int { kKvBf16 = 0, kKvFp8 = 1, kKvNvfp4 = 2,
                      kKvNvfp4NoRope = 3,     // MLA only: the rope-free 288-byte NVFP4 row (GLM-Flash latent)
                      kKvV4Pro = 4,           // MLA only: the 320-byte DeepSeek V4 Pro cell (448 NVFP4 + 64 E4M3 rope)
                      kKvV4ProBf16Rope = 5 }; // MLA only: the 384-byte V4 Pro cell (448 NVFP4 + 64 bf16 rope)

// Bytes of one (page, kv_head) block of a GQA pool page: K then V, each page_size tokens of head_dim values.
//   bf16 : [K 64 x D x 2][V 64 x D x 2]
//   fp8  : [K 64 x D][V 64 x D]                      (E4M3, per-layer k/v scale)
//   nvfp4: [Kcodes 64 x D/2][Kscales 64 x D/16][Vcodes 64 x D/2][Vscales 64 x D/16]   (+ per-layer global scale)
#if defined(__CUDACC__)
__host__ __device__
#endif
inline int gqa_block_bytes(int fmt, int head_dim, int page) {
  if (fmt == kKvBf16) return 2 * page * head_dim * 2;
  if (fmt == kKvFp8) return 2 * page * head_dim;
  return 2 * page * (head_dim / 2 + head_dim / 16);
}

// ---- elementwise / normalisation (elementwise.cu)
// q8 / qs (optional): also write the output as E4M3 + one UE8M0 scale word per 128 values (the FP8 GEMM input).
cudaError_t rmsnorm(const void* x, void* residual, void* out, const void* weight, int rows, int hidden,
                    int x_stride, float eps, bool plus_one, bool add_residual, cudaStream_t s,
                    uint8_t* q8 = nullptr, uint32_t* qs = nullptr);
cudaError_t gelu_tanh_mul(const void* gate_up, void* out, int rows, int ffn, cudaStream_t s);
cudaError_t silu_mul(const void* gate_up, void* out, int rows, int ffn, cudaStream_t s);
cudaError_t embed(const int* ids, const void* table, void* out, int rows, int hidden, float scale, cudaStream_t s);
cudaError_t argmax_rows(const void* logits, int* out_idx, float* out_val, int rows, int vocab, int stride,
                        bool logits_fp32, cudaStream_t s);

// Fused GQA QKV epilogue: per-head RMSNorm of q and k, NeoX RoPE (cos/sin table [max_pos, D]: D/2 cos then D/2
// sin), q written as bf16 [T, Hq, D], k/v quantized into the paged pool at slot[t] (page = slot / 64).
struct GqaPrepArgs {
  const void* qkv;      // bf16 [T, (Hq + 2 Hk) * D], row stride qkv_stride elements
  int qkv_stride;
  const void* q_norm;   // bf16 [D] or null (no norm)
  const void* k_norm;
  const float* cos_sin; // fp32 [max_pos, D]
  const int* pos;       // [T]
  const int* slot;      // [T], -1 = do not write
  void* q_out;          // bf16 [T, Hq, D]
  uint8_t* pool;        // layer pool base: [num_pages, Hk, block_bytes]
  int fmt;
  float k_scale, v_scale;  // fp8: e4m3(x / scale); nvfp4: global scale
  int T, Hq, Hk, D, page;
  float eps;
  bool plus_one;
};
cudaError_t gqa_prep(const GqaPrepArgs& a, cudaStream_t s);

// MLA latent rows: nope [T, 512] + rope [T, 64] (bf16) -> pool row slot[t]; fmt kKvNvfp4 (352 B) or kKvFp8 (576 B).
cudaError_t mla_quant_write(const void* nope, int nope_stride, const void* rope, int rope_stride, const int* slot,
                            uint8_t* pool, int T, int fmt, cudaStream_t s);
// Indexer keys [T, 128] bf16 -> 132-byte rows (E4M3 * per-token fp32 scale).
cudaError_t index_key_write(const void* k, int k_stride, const int* slot, uint8_t* pool, int T, cudaStream_t s);

// Pool rows (one token's K or V codes of one head) are stored with their 16-byte chunks XOR-swizzled by the token's
// row in the page: chunk j of row r lives at chunk (j & ~(n-1)) | ((j ^ r) & (n-1)), n = min(8, row_bytes / 16).
// Readers that fetch the same chunk of 8 consecutive rows then hit 8 different shared-memory bank groups.
#if defined(__CUDACC__)
__host__ __device__
#endif
inline int kv_swizzle_byte(int byte_in_row, int row, int row_bytes) {
  const int nch = (row_bytes / 16) < 8 ? (row_bytes / 16) : 8;
  const int j = byte_in_row >> 4;
  const int pos = (j & ~(nch - 1)) | ((j ^ row) & (nch - 1));
  return (pos << 4) | (byte_in_row & 15);
}

// ---- GQA split-K decode / verify attention (attn_gqa_decode.cu)
struct GqaDecodeArgs {
  const void* q;           // bf16 [B * n_q, Hq, D] (normed + roped)
  const uint8_t* pool;     // layer pool [num_pages, Hk, 2 parts (K, V), part_bytes]
  const int* page_table;   // [rows, pt_stride] physical page per logical page
  const int* req_idx;      // [B] page-table row of batch entry b (null: row b)
  const int* kv_len;       // [B] tokens in the pool (query tokens included, they are the last n_q)
  void* out;               // bf16 [B * n_q, Hq, D]
  float* o_part;           // [B * Hk * num_splits, RMAX, D]  (num_splits > 1)
  float* lse_part;         // [B * Hk * num_splits, RMAX]     (log2 units)
  int* status;             // device status word (bounded-wait timeouts)
  int B, n_q, Hq, Hk, D, pt_stride, page, window, fmt;
  int tiles_per_split, num_splits;
  float sm_scale, k_scale, v_scale;
  long long* trace;        // optional [16 events x 512 tiles] clock64 timeline of CTA 0 (diagnostics), else null
  int exact;               // 1: f16 operands (exact dequant); 0: E4M3 operands (K = 32 UMMAs) for NVFP4 / FP8 pools
};
cudaError_t gqa_decode(const GqaDecodeArgs& a, cudaStream_t s);

// ---- GQA-packed extend / prefill attention (attn_gqa_extend.cu): 128 query rows (BT = 128 / G tokens x G heads)
// of one kv head per CTA over an NVFP4 / FP8 pool, causal + sliding window.
struct GqaExtendArgs {
  const void* q;           // bf16 [rows, Hq, D] query tokens (normed + roped)
  const uint8_t* pool;     // layer pool [num_pages, Hk, 2 parts (K, V), part_bytes]
  const int* page_table;   // [requests, pt_stride]
  const int* blocks;       // [nblocks, 4]: first q row, tokens (1..128 / G), position of the first token, page-table row
  void* out;               // bf16 [rows, Hq, D]; rows outside every block are not written
  int* status;             // device status word (bounded-wait timeouts, bad page ids)
  int nblocks, Hq, Hk, D, pt_stride, page, window, fmt, pool_pages;
  float sm_scale, k_scale, v_scale;
  long long* trace;        // optional [12 events x 64 tiles] clock64 timeline of CTA (0, 0, 0) (diagnostics), else null
};
cudaError_t gqa_extend(const GqaExtendArgs& a, cudaStream_t s);

// ---- sparse MLA decode (attn_mla_decode.cu): DSA attention over gathered latent rows, H <= 128 heads.
struct MlaDecodeArgs {
  const void* q;           // bf16 [T, H, 576] (512 latent dims then 64 rope dims), quantized first into q8_out, or null
  uint8_t* q8_out;         // with q: E4M3 destination (== q8) and q_scale_out (== q_scale)
  float* q_scale_out;
  const uint8_t* q8;       // E4M3 [T, H, 576]: q / q_scale
  const float* q_scale;    // [T, H] per-head scale (amax / 448)
  const uint8_t* pool;     // [rows, 352] NVFP4 latent rows (fmt = kKvNvfp4) or [rows, 576] E4M3 rows (kKvFp8)
  const int* idx;          // [T, idx_stride] pool rows attended by each token; -1 = masked
  void* out;               // bf16 [T, H, 512]
  float* lse;              // [T, H] natural-log logsumexp, or null
  float* o_part;           // [num_splits, T, H, 512] (num_splits > 1)
  float* lse_part;         // [num_splits, T, H] log2 units (num_splits > 1)
  int* status;             // device status word (bounded-wait timeouts)
  int T, H, topk, idx_stride, fmt;
  int pool_rows;           // rows in the pool: an index outside [0, pool_rows) is treated as masked (status kBadIndex)
  int tiles_per_split, num_splits;  // 128-row tiles of the top-k list per split
  // Mixed-format pools (one launch per pool format over one page-id space): index i of a token addresses pool row
  // i - row_lo; tokens with tok_sel[t] != sel are skipped by this launch (their rows live in the other pool and
  // another launch writes their output).  tok_sel null: every token, row_lo 0.
  const int* tok_sel;
  int sel, row_lo;
  float sm_scale;
  long long* trace;        // optional [40 events x 64 tiles] clock64 timeline of CTA (0, 0, 0), else null
};
cudaError_t mla_decode(const MlaDecodeArgs& a, cudaStream_t s);

// ---- DSA lightning indexer (indexer.cu): scores over the cached positions, then top-k positions as pool slots.
struct IndexerArgs {
  const uint8_t* q8;       // E4M3 [T, Hi, 128] indexer queries
  const float* w;          // [T, Hi] head weights (the query scale folded in)
  const uint8_t* pool;     // index pool [pages, 64 x 132 B] (values swizzled per page, then scales)
  const int* page_table;   // [rows, pt_stride]
  const int* req_idx;      // [T] page-table row of each token (null: row t)
  const int* limit;        // [T] visible positions 0 .. limit - 1
  float* scores;           // [T, score_stride] fp32 (logits output / top-k input)
  int* out_slots;          // [T, topk] pool slots, -1 padded
  int* out_pos;            // [T, topk] positions (optional)
  int* status;
  int T, Hi, pt_stride, score_stride;
  int tiles_per_cta, max_tiles;   // 128-position tiles per CTA; tiles of the longest token
  int topk;
};
cudaError_t indexer_logits(const IndexerArgs& a, cudaStream_t s);
cudaError_t indexer_topk(const IndexerArgs& a, cudaStream_t s);

// ---- tensor-parallel all-reduce fused with the following norm chain (comm.cu), over symmetric peer memory.
struct ArNormArgs {
  void* const* peers;      // [nranks] device pointers to every rank's symmetric buffer (peers[rank] = own)
  long long flag_offset;   // byte offset of the [2][nranks] int flags inside each buffer
  int rows_cap, H, T, half, rank, nranks;
  int* epoch;              // [2] this rank's flag values for the two halves (initialised {1, 0})
  void* resid;             // bf16 [T, H], updated in place: resid += o
  void* out;               // bf16 [T, H]: rmsnorm(resid, w2)
  const void* w1;          // bf16 [H] norm applied to the reduced sum first (null: none)
  const void* w2;          // bf16 [H] norm of the new residual (null: out is not written)
  float eps, plus_one;
  int* status;
  // 0: pull -- each rank's partial sits in its own buffer, data [2][rows_cap][H], read over NVLink.  1: push -- the
  // row-parallel GEMM stored its partial into slot `rank` of every rank's buffer, data [2][nranks][rows_cap][H],
  // so the sum reads local memory only.
  int slots;
  // NVLS (mc != null; pull layout for the partials): the NVLink multicast address of the same buffer.  Rank r sums
  // column shard r of each row inside the switch (multimem.ld_reduce over every rank's partial) and multicasts the
  // reduced shard into the reduced-rows area [2][rows_cap][H] at res_offset of every rank; per-row arrival flags
  // [2][rows_cap][nranks] ints at rowflag_offset.
  void* mc;
  long long res_offset, rowflag_offset;
};
cudaError_t ar_norm2(const ArNormArgs& a, cudaStream_t s);

// ---- MoE router (moe.cu): sigmoid, bias-corrected group-limited top-k, renormalised * scale.
// ksplit > 1: `logits` holds ksplit fp32 partials [ksplit][T][E] of the router GEMM, summed here in split order
// (register form only: E and the group size multiples of 32).
cudaError_t moe_route(const float* logits, const float* bias, int* ids, float* wts, int T, int E, int K, int G,
                      int KG, float scale, cudaStream_t s, int ksplit = 1);

// ---- primitive check (umma_test.cu): C[M, N] fp32 = A[M, K] * B[N, K]^T, bf16 inputs, one CTA per 128 rows.
// ---- grouped block-scaled expert GEMM + routing prep (moe_gemm.cu)
enum MoeOutMode { kMoeOutBf16 = 0, kMoeOutSwigluQuant = 1, kMoeOutBf16Weighted = 2,
                  kMoeOutF32Split = 3 };   // split-K: fp32 partials [ksplit][split_rows][out_stride] into `out`
struct MoeGemmArgs {
  const uint8_t* wpack;       // [E][n_tiles][KC] blocks: G SW128 tiles (128 x 128 B) then G scale atoms (512 B);
                              // plain modes: the G tiles are output columns (nt G + g) 128 ..; SwiGLU: gate, up
  const uint8_t* x;           // FP8 E4M3 activation rows, row stride x_stride bytes
  const uint32_t* x_scale;    // kind 0: UE8M0 x4 words [rows][KC]; kind 1: E4M3 bytes [rows][K / 16]
  const int* expert_off;      // [E + 1]
  const int* pairs;           // pair ids bucketed by expert
  const float* pair_w;        // per-pair weight (kMoeOutBf16Weighted)
  void* out;                  // bf16 [pairs][out_stride] or FP8 [pairs][out_stride] (SwiGLU mode)
  uint32_t* out_scale;        // SwiGLU mode: UE8M0 x4 words [pairs][out_scale_stride]
  const float* expert_mul;    // optional per-expert output multiplier (NVFP4 weight global scales)
  // Optional peer-memory output (expert parallelism): row p < pairs_total goes to rank p / out_div, row p % out_div
  // of the region at byte offset out_offset of that rank's symmetric buffer; shared-expert rows p >= pairs_total
  // go to this rank (out_rank), row out_shared_base + p - pairs_total.  Plain bf16 modes only.
  // Broadcast form (tensor parallelism, out_bcast = ranks > 0): row p goes to EVERY rank rr < out_bcast, row p of
  // the region at out_offset of rank rr's buffer (this rank's slot there), starting with rank out_rank.
  const long long* out_peers;
  long long out_offset;
  int out_div, out_rank, out_shared_base, pairs_total, out_bcast;
  int* status;
  int E, n_tiles, KC, G, NT, mode, src_div, src_limit, src_shared_base, x_stride, out_stride, out_scale_stride;
  // Optional grouped source rows (0 = off): activation row of a pair p below src_limit is
  // (q / src_group) * src_group_stride + q % src_group with q = p / src_div -- e.g. head h of token t at row
  // t * src_group_stride + h when a projection's output holds every head's slice back to back.
  int src_group, src_group_stride;
  int ksplit;                 // split-K factor (>= 1): item = (expert, token tile, weight tile, K range)
  int split_rows;             // kMoeOutF32Split: rows between two splits' partials
  int num_ctas;
  int kind;                   // 0: FP8 E4M3 + UE8M0 per 32 (128-blocks replicated); 1: NVFP4 (E2M1 + E4M3 per 16)
  float out_mul;
  long long* trace;           // optional diagnostic timeline of CTA 0 (kMgEv* events, clock64), null = off
  // Programmatic dependent launch: the kernel may start while the previous kernel of the stream runs; it sets up and
  // (static_index) streams its first weight stages before waiting for that kernel's outputs.  static_index: the
  // expert offsets and pair ids were written before the previous kernel (cached index tensors), so the work list can
  // be built before the wait; else everything waits first.
  int pdl, static_index;
  // Split-K with the reduction folded in (kMoeOutF32Split): after writing its partial, a split bumps the tile's
  // counter; the split that completes the tile sums the partials in split order and writes red_out (bf16, or fp32
  // with red_f32; row stride red_stride), then re-arms the counter (zero before and after every launch).
  void* red_out;
  int* tile_cnt;
  int red_stride, red_f32;
};
// GEMM timeline events (trace[ev]): kernel start, setup done, first weight copy issued, first stage ready at the
// MMA warp, last MMA committed, first accumulator seen by the epilogue, epilogue done, kernel end.
// Slots 8 + 4 c + {0, 1, 2}: chunk c (32 tokens, c < 3) of the epilogue: accumulator loaded, first pass staged,
// first pass stored.
enum MgTraceEv { kMgEvStart, kMgEvSetup, kMgEvFirstCopy, kMgEvFirstReady, kMgEvLastMma, kMgEvAccSeen, kMgEvEpiDone,
                 kMgEvEnd, kMgEvCount = 20 };
cudaError_t moe_gemm(const MoeGemmArgs& a, cudaStream_t s);
cudaError_t moe_align(const int* ids, int P, int e0, int E, int shared_bucket, int extra, int* off, int* pairs,
                      cudaStream_t s);
// out [rows][N] (bf16, or fp32 with out_f32) = sum over splits of part fp32 [ksplit][rows][N] (fixed split order:
// deterministic).
// peers (optional, bf16 only): the rows also go, at byte offset peer_offset, to every rank's buffer in peers[nbcast]
// (this rank's slot there; tensor-parallel push of a row-parallel GEMM's result), starting with rank `rank`.
cudaError_t splitk_reduce(const float* part, int ksplit, int rows, int N, void* out, bool out_f32, cudaStream_t s,
                          const long long* peers = nullptr, long long peer_offset = 0, int nbcast = 0, int rank = 0);
cudaError_t moe_combine(const void* rows, int T, int topk, int H, int shared_base, const float* w, void* y,
                        cudaStream_t s);

// ---- fused MLA attention-block glue (mla_prep.cu)
struct MlaPrepArgs {
  const void* ya;             // bf16 [T, ya_stride]: q_a (q_lora) | kv latent (512) | k_pe (64) | k_i (128) | w_i (Hi)
  int ya_stride;
  const void* q_norm;         // bf16 [q_lora]
  const void* kv_norm;        // bf16 [512]
  const void* ik_w;           // bf16 [128] LayerNorm weight / bias of the indexer key
  const void* ik_b;
  const float* rope;          // fp32 [max_pos, 64]: cos (32) | sin (32)
  const int* pos;             // [T]
  const int* slot;            // [T] pool slot (-1: not written)
  const int* lat_slot;        // [T] latent pool row when it differs from `slot` (context parallelism: the owning
                              // rank's local row, -1 elsewhere); null = slot
  void* qa_out;               // bf16 [T, q_lora]
  uint8_t* qa_q;              // optional E4M3 [T, q_lora] + UE8M0 x4 words [T, q_lora / 128] of the normed q_a (the
  uint32_t* qa_s;             // FP8 block-scaled input of the next projection; null = not written)
  uint8_t* latent_pool;       // [slots, 352] NVFP4 or [slots, 576] E4M3
  int latent_fmt;
  uint8_t* latent_pool2;      // optional second pool (mixed-format page space): latent slots >= split_slot are row
  int latent_fmt2, split_slot;  // slot - split_slot of this pool, in its format; null = one pool
  uint8_t* index_pool;        // [pages, 64 * 132]
  float* iw_out;              // fp32 [T, Hi]: w_i * iw_scale
  float iw_scale;
  const void* yb;             // bf16 [T, yb_stride]: q_nope (H dn) | q_pe (H 64) | q_i (Hi 128)
  int yb_stride;
  void* qf;                   // bf16 [T, H, 576]; columns 512.. written
  uint8_t* q8;                // E4M3 [T, Hi, 128]
  float* w_eff;               // fp32 [T, Hi]
  int T, q_lora, H, dn, Hi;
  float eps;
};
cudaError_t mla_prep_kv(const MlaPrepArgs& a, cudaStream_t s);
cudaError_t mla_prep_q(const MlaPrepArgs& a, cudaStream_t s);

// ---- FP8-quantized two-shot all-reduce over peer memory (qar.cu)
struct QarArgs {
  const long long* peers;      // [nranks] symmetric buffer bases
  long long off_recv_q, off_recv_s, off_gather_q, off_gather_s, off_flags;
  const void* x;               // bf16 [T, H] this rank's addend
  void* y;                     // bf16 [T, H] sum (identical on every rank)
  int* epoch;                  // device [1]
  int* status;
  int T, T_max, H, G, per, rank, nranks;
};
cudaError_t qar_allreduce(const QarArgs& a, cudaStream_t s);

// ---- Kimi delta attention decode step (kda.cu)
struct KdaDecodeArgs {
  const __nv_bfloat16 *q, *k, *v;        // [B, H, DK], [B, H, DK], [B, HV, DV] (projections, pre-conv)
  const __nv_bfloat16* g_proj;           // [B, HV, DK]
  const float* dt_bias;                  // [HV * DK]
  const float* A_log;                    // [HV]
  const float* beta;                     // [B, HV] or [B, HV, DV]
  const __nv_bfloat16* g2;               // [B, HV, DV] output-gate input
  const float* norm_w;                   // [DV]
  const float *conv_wq, *conv_wk, *conv_wv;   // [H * DK, W], [H * DK, W], [HV * DV, W]
  float *conv_q, *conv_k, *conv_v;       // [B, H * DK, W - 1] ... (oldest first), updated in place
  float* state;                          // [B, HV, DV, DK] fp32, updated in place
  __nv_bfloat16* out;                    // [B, HV, DV]
  float scale;
  int B, H, HV, DK, DV, W, beta_headwise;
};
cudaError_t kda_decode(const KdaDecodeArgs& a, cudaStream_t s);

// ---- prefill -> decode KV page transfer over peer memory (pd.cu)
struct PdCopyArgs {
  const uint8_t* src;         // this GPU's pool (layer 0), layer l at src + l * src_layer_stride
  void* dst;                  // the decode GPU's pool (peer mapping), same layout with dst_layer_stride
  const int* src_pages;       // [n_pairs]
  const int* dst_pages;       // [n_pairs]
  long long page_bytes, src_layer_stride, dst_layer_stride;
  int n_pairs, layers;
};
cudaError_t pd_copy(const PdCopyArgs& a, cudaStream_t s);
cudaError_t pd_signal(int* peer_flag, int value, cudaStream_t s);
cudaError_t pd_wait(const int* flag, int value, int* status, cudaStream_t s);

// ---- more latent-row formats (kv_formats.cu)
cudaError_t glmflash_write(const void* nope, int stride, const int* slot, uint8_t* pool, int T, cudaStream_t s);
cudaError_t v4pro_write(const void* x, int stride, const int* slot, uint8_t* pool, int T, int rope_bf16,
                        cudaStream_t s);

// ---- decode context parallelism: partial-softmax merge over peer memory (dcp.cu)
struct DcpMergeArgs {
  const long long* peers;     // [nranks] symmetric buffer bases
  long long off_data, off_flags;
  void* out;                  // bf16 [T, Hg, 512]: this rank's head group, merged
  float* lse_out;             // optional fp32 [T, Hg]
  int* epoch;                 // device [2]
  int* status;
  int T, T_max, H, Hg, rank, nranks, half;
};
cudaError_t dcp_merge(const DcpMergeArgs& a, cudaStream_t s);

// ---- expert-parallel exchange over peer memory (ep.cu)
struct EpDispatchArgs {
  const long long* peers;     // [world] base address of every rank's symmetric buffer (device)
  const uint8_t* xq;          // this rank's quantized rows [T, row_bytes]
  const uint8_t* xs;          // their scale bytes [T, scale_bytes]
  const int* ids;             // [T, topk] global expert ids
  long long off_x, off_s, off_ids;   // byte offsets of the receive regions inside the symmetric buffer
  int T, T_max, topk, rank, world, E_loc, row_bytes, scale_bytes;
};
cudaError_t ep_dispatch(const EpDispatchArgs& a, cudaStream_t s);
cudaError_t ep_barrier(const long long* peers, long long off_flags, int rank, int world, int* epoch, int* status,
                       cudaStream_t s);
// act(gate) * up over gate_up [T, 2F] -> quantized (fmt 0 E4M3 + UE8M0 per 128, fmt 1 NVFP4 per 16).
cudaError_t act_quant(const void* gate_up, int T, int F, bool gelu, int fmt, uint8_t* q, uint32_t* sc, cudaStream_t s);
cudaError_t rmsnorm_quant(const void* x, const void* w, float eps, float plus_one, int T, int H, int fmt, uint8_t* q,
                          uint32_t* sc, cudaStream_t s);

cudaError_t umma_gemm_test(const void* A, const void* B, float* C, int M, int N, int K, int sw64, cudaStream_t s);
cudaError_t umma_f8_mn_test(const void* A, const void* B, float* C, int N, int K, cudaStream_t s);
cudaError_t nvfp4_lut_test(const uint32_t* words, int nwords, int* out, cudaStream_t s);

// Two green contexts over disjoint SM sets (first_sms rounded up by the driver, and the rest), one stream each:
// streams[0..1] (CUstream handles), sms[0..1].  Returns 0, or -1 with a message in err.
int sm_lanes_create(int device, int first_sms, unsigned long long* streams, int* sms, char* err, int errlen);

}  // namespace iob
