// Torch bindings for the sm_100a kernels.  Each binding validates shapes/dtypes, then calls the plain-pointer launcher
// on the current CUDA stream (so CUDA-graph capture and stream ordering follow torch's).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"

namespace {

#define CHECK_CUDA_OK(expr)                                                         \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    TORCH_CHECK(_e == cudaSuccess, #expr, " failed: ", cudaGetErrorString(_e));     \
  } while (0)

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void req(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}

void rmsnorm(const at::Tensor& x, c10::optional<at::Tensor> residual, at::Tensor out, const at::Tensor& w, double eps,
             bool plus_one, const c10::optional<at::Tensor>& q8, const c10::optional<at::Tensor>& qs) {
  req(x, at::kBFloat16, "x");
  req(out, at::kBFloat16, "out");
  req(w, at::kBFloat16, "weight");
  const int hidden = x.size(-1);
  const int rows = x.numel() / hidden;
  TORCH_CHECK(x.stride(-1) == 1 && out.is_contiguous() && w.is_contiguous(), "layout");
  const int stride = x.dim() > 1 ? x.stride(-2) : hidden;
  void* res = nullptr;
  if (residual.has_value()) {
    req(*residual, at::kBFloat16, "residual");
    TORCH_CHECK(residual->is_contiguous(), "residual layout");
    res = residual->data_ptr();
  }
  const at::cuda::CUDAGuard g(x.device());
  uint8_t* q8p = nullptr;
  uint32_t* qsp = nullptr;
  if (q8.has_value()) {
    TORCH_CHECK(qs.has_value() && q8->scalar_type() == at::kByte && qs->scalar_type() == at::kInt &&
                    q8->is_contiguous() && qs->is_contiguous() && q8->numel() == static_cast<int64_t>(rows) * hidden &&
                    qs->numel() == static_cast<int64_t>(rows) * (hidden / 128) && hidden % 128 == 0,
                "rmsnorm FP8 output: q8 uint8 [rows, hidden], qs int32 [rows, hidden / 128]");
    q8p = q8->data_ptr<uint8_t>();
    qsp = reinterpret_cast<uint32_t*>(qs->data_ptr<int>());
  }
  CHECK_CUDA_OK(iob::rmsnorm(x.data_ptr(), res, out.data_ptr(), w.data_ptr(), rows, hidden, stride, eps, plus_one,
                             res != nullptr, stream(), q8p, qsp));
}

void act_mul(const at::Tensor& gu, at::Tensor out, bool gelu) {
  req(gu, at::kBFloat16, "gate_up");
  req(out, at::kBFloat16, "out");
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous(), "layout");
  const int ffn = out.size(-1);
  const int rows = out.numel() / ffn;
  TORCH_CHECK(gu.size(-1) == 2 * ffn && ffn % 8 == 0, "shape");
  const at::cuda::CUDAGuard g(gu.device());
  if (gelu) CHECK_CUDA_OK(iob::gelu_tanh_mul(gu.data_ptr(), out.data_ptr(), rows, ffn, stream()));
  else CHECK_CUDA_OK(iob::silu_mul(gu.data_ptr(), out.data_ptr(), rows, ffn, stream()));
}

void embed(const at::Tensor& ids, const at::Tensor& table, at::Tensor out, double scale) {
  req(ids, at::kInt, "ids");
  req(table, at::kBFloat16, "table");
  req(out, at::kBFloat16, "out");
  const at::cuda::CUDAGuard g(ids.device());
  CHECK_CUDA_OK(iob::embed(ids.data_ptr<int>(), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1),
                           scale, stream()));
}

void argmax(const at::Tensor& logits, at::Tensor idx, c10::optional<at::Tensor> val) {
  TORCH_CHECK(logits.is_cuda() && logits.stride(-1) == 1, "logits");
  req(idx, at::kInt, "idx");
  const bool f32 = logits.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || logits.scalar_type() == at::kBFloat16, "logits dtype");
  const int vocab = logits.size(-1);
  TORCH_CHECK(vocab % 8 == 0, "vocab % 8");
  float* v = nullptr;
  if (val.has_value()) { req(*val, at::kFloat, "val"); v = val->data_ptr<float>(); }
  const at::cuda::CUDAGuard g(logits.device());
  CHECK_CUDA_OK(iob::argmax_rows(logits.data_ptr(), idx.data_ptr<int>(), v, logits.numel() / vocab, vocab,
                                 logits.dim() > 1 ? logits.stride(-2) : vocab, f32, stream()));
}

void gqa_prep(const at::Tensor& qkv, c10::optional<at::Tensor> q_norm, c10::optional<at::Tensor> k_norm,
              const at::Tensor& cos_sin, const at::Tensor& pos, const at::Tensor& slot, at::Tensor q_out,
              at::Tensor pool, int64_t fmt, double k_scale, double v_scale, int64_t Hq, int64_t Hk, int64_t D,
              int64_t page, double eps, bool plus_one) {
  req(qkv, at::kBFloat16, "qkv");
  req(cos_sin, at::kFloat, "cos_sin");
  req(pos, at::kInt, "pos");
  req(slot, at::kInt, "slot");
  req(q_out, at::kBFloat16, "q_out");
  req(pool, at::kByte, "pool");
  TORCH_CHECK(qkv.stride(-1) == 1 && qkv.size(-1) >= (Hq + 2 * Hk) * D, "qkv shape");
  TORCH_CHECK(cos_sin.size(-1) == D, "cos_sin width");
  iob::GqaPrepArgs a{};
  a.qkv = qkv.data_ptr();
  a.qkv_stride = qkv.stride(0);
  a.q_norm = q_norm.has_value() ? q_norm->data_ptr() : nullptr;
  a.k_norm = k_norm.has_value() ? k_norm->data_ptr() : nullptr;
  a.cos_sin = cos_sin.data_ptr<float>();
  a.pos = pos.data_ptr<int>();
  a.slot = slot.data_ptr<int>();
  a.q_out = q_out.data_ptr();
  a.pool = pool.data_ptr<uint8_t>();
  a.fmt = fmt;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.T = qkv.size(0);
  a.Hq = Hq; a.Hk = Hk; a.D = D; a.page = page;
  a.eps = eps;
  a.plus_one = plus_one;
  const at::cuda::CUDAGuard g(qkv.device());
  CHECK_CUDA_OK(iob::gqa_prep(a, stream()));
}

void mla_quant_write(const at::Tensor& nope, const at::Tensor& rope, const at::Tensor& slot, at::Tensor pool,
                     int64_t fmt) {
  req(nope, at::kBFloat16, "nope");
  req(rope, at::kBFloat16, "rope");
  req(slot, at::kInt, "slot");
  req(pool, at::kByte, "pool");
  TORCH_CHECK(nope.size(-1) == 512 && rope.size(-1) == 64 && nope.stride(-1) == 1 && rope.stride(-1) == 1, "shape");
  TORCH_CHECK(pool.size(-1) == (fmt == iob::kKvNvfp4 ? 352 : 576), "pool row bytes");
  const at::cuda::CUDAGuard g(nope.device());
  CHECK_CUDA_OK(iob::mla_quant_write(nope.data_ptr(), nope.stride(0), rope.data_ptr(), rope.stride(0),
                                     slot.data_ptr<int>(), pool.data_ptr<uint8_t>(), nope.size(0), fmt, stream()));
}

void index_key_write(const at::Tensor& k, const at::Tensor& slot, at::Tensor pool) {
  req(k, at::kBFloat16, "k");
  req(slot, at::kInt, "slot");
  req(pool, at::kByte, "pool");
  TORCH_CHECK(k.size(-1) == 128 && k.stride(-1) == 1 && pool.size(-1) == 64 * 132 && pool.is_contiguous(),
              "k [T, 128], pool [pages, 64 x 132]");
  const at::cuda::CUDAGuard g(k.device());
  CHECK_CUDA_OK(iob::index_key_write(k.data_ptr(), k.stride(0), slot.data_ptr<int>(), pool.data_ptr<uint8_t>(),
                                     k.size(0), stream()));
}

void gqa_extend(const at::Tensor& q, const at::Tensor& pool, const at::Tensor& page_table, const at::Tensor& blocks,
                at::Tensor out, at::Tensor status, int64_t Hk, int64_t window, int64_t fmt, double sm_scale,
                double k_scale, double v_scale, c10::optional<at::Tensor> trace) {
  req(q, at::kBFloat16, "q");
  req(pool, at::kByte, "pool");
  req(page_table, at::kInt, "page_table");
  req(blocks, at::kInt, "blocks");
  req(out, at::kBFloat16, "out");
  req(status, at::kInt, "status");
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && out.is_contiguous() && out.sizes() == q.sizes(), "q / out [rows, Hq, D]");
  TORCH_CHECK(page_table.dim() == 2 && page_table.is_contiguous(), "page_table");
  TORCH_CHECK(blocks.dim() == 2 && blocks.size(1) == 4 && blocks.is_contiguous(), "blocks [n, 4]");
  TORCH_CHECK(pool.dim() == 4 && pool.size(1) == Hk && pool.size(2) == 2, "pool [pages, Hk, 2, part]");
  iob::GqaExtendArgs a{};
  a.q = q.data_ptr();
  a.pool = pool.data_ptr<uint8_t>();
  a.page_table = page_table.data_ptr<int>();
  a.blocks = blocks.data_ptr<int>();
  a.out = out.data_ptr();
  a.status = status.data_ptr<int>();
  a.nblocks = static_cast<int>(blocks.size(0));
  a.Hq = static_cast<int>(q.size(1));
  a.Hk = static_cast<int>(Hk);
  a.D = static_cast<int>(q.size(2));
  a.pt_stride = static_cast<int>(page_table.size(1));
  a.page = 64;
  a.window = static_cast<int>(window);
  a.fmt = static_cast<int>(fmt);
  a.pool_pages = static_cast<int>(pool.size(0));
  a.sm_scale = static_cast<float>(sm_scale);
  a.k_scale = static_cast<float>(k_scale);
  a.v_scale = static_cast<float>(v_scale);
  if (trace.has_value()) {
    req(*trace, at::kLong, "trace");
    TORCH_CHECK(trace->numel() >= 12 * 64, "trace [12 x 64]");
    a.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  TORCH_CHECK(2 * pool.size(3) == iob::gqa_block_bytes(a.fmt, a.D, 64), "pool part bytes");
  const at::cuda::CUDAGuard g(q.device());
  CHECK_CUDA_OK(iob::gqa_extend(a, stream()));
}

void gqa_decode(const at::Tensor& q, const at::Tensor& pool, const at::Tensor& page_table,
                c10::optional<at::Tensor> req_idx, const at::Tensor& kv_len, at::Tensor out, at::Tensor o_part, at::Tensor lse_part, at::Tensor status, int64_t n_q, int64_t Hk,
                int64_t page, int64_t window, int64_t fmt, int64_t tiles_per_split, int64_t num_splits,
                double sm_scale, double k_scale, double v_scale, c10::optional<at::Tensor> trace,
                int64_t exact) {
  req(q, at::kBFloat16, "q");
  req(pool, at::kByte, "pool");
  req(page_table, at::kInt, "page_table");
  req(kv_len, at::kInt, "kv_len");
  req(out, at::kBFloat16, "out");
  req(o_part, at::kFloat, "o_part");
  req(lse_part, at::kFloat, "lse_part");
  req(status, at::kInt, "status");
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous() && page_table.is_contiguous(), "layout");
  TORCH_CHECK(q.dim() == 3, "q [B*n_q, Hq, D]");
  iob::GqaDecodeArgs a{};
  a.q = q.data_ptr();
  a.pool = pool.data_ptr<uint8_t>();
  a.page_table = page_table.data_ptr<int>();
  if (req_idx.has_value()) { req(*req_idx, at::kInt, "req_idx"); a.req_idx = req_idx->data_ptr<int>(); }
  a.kv_len = kv_len.data_ptr<int>();
  a.out = out.data_ptr();
  a.o_part = o_part.data_ptr<float>();
  a.lse_part = lse_part.data_ptr<float>();
  a.status = status.data_ptr<int>();
  a.B = kv_len.size(0);
  a.n_q = n_q;
  a.Hq = q.size(1);
  a.Hk = Hk;
  a.D = q.size(2);
  a.pt_stride = page_table.size(1);
  a.page = page;
  a.window = window;
  a.fmt = fmt;
  a.tiles_per_split = tiles_per_split;
  a.num_splits = num_splits;
  a.sm_scale = sm_scale;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  if (trace.has_value()) { req(*trace, at::kLong, "trace"); a.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>()); }
  a.exact = static_cast<int>(exact);
  TORCH_CHECK(q.size(0) == a.B * n_q, "q rows");
  const int rmax = a.n_q * (a.Hq / a.Hk) <= 8 ? 8 : 16;
  if (num_splits > 1)
    TORCH_CHECK(o_part.numel() >= (int64_t)a.B * Hk * num_splits * rmax * a.D &&
                    lse_part.numel() >= (int64_t)a.B * Hk * num_splits * rmax,
                "split workspace too small");
  const at::cuda::CUDAGuard g(q.device());
  CHECK_CUDA_OK(iob::gqa_decode(a, stream()));
}

void mla_decode(c10::optional<at::Tensor> q, at::Tensor q8, at::Tensor q_scale, const at::Tensor& pool,
                const at::Tensor& idx, at::Tensor out, c10::optional<at::Tensor> lse, at::Tensor o_part,
                at::Tensor lse_part, at::Tensor status, int64_t fmt, int64_t tiles_per_split, int64_t num_splits,
                double sm_scale, c10::optional<at::Tensor> trace, c10::optional<at::Tensor> tok_sel, int64_t sel,
                int64_t row_lo) {
  req(q8, at::kByte, "q8");
  req(q_scale, at::kFloat, "q_scale");
  req(pool, at::kByte, "pool");
  req(idx, at::kInt, "idx");
  req(out, at::kBFloat16, "out");
  req(o_part, at::kFloat, "o_part");
  req(lse_part, at::kFloat, "lse_part");
  req(status, at::kInt, "status");
  TORCH_CHECK(q8.is_contiguous() && out.is_contiguous() && pool.is_contiguous() && q_scale.is_contiguous(), "layout");
  TORCH_CHECK(q8.dim() == 3 && q8.size(2) == 576, "q8 [T, H, 576]");
  const int64_t T = q8.size(0), H = q8.size(1);
  TORCH_CHECK(q_scale.numel() >= T * H, "q_scale [T, H]");
  TORCH_CHECK(idx.dim() == 2 && idx.stride(1) == 1 && idx.size(0) == T, "idx [T, topk]");
  TORCH_CHECK(out.size(0) == T && out.size(1) == H && out.size(2) == 512, "out [T, H, 512]");
  const int64_t rb = fmt == iob::kKvNvfp4 ? 352 : fmt == iob::kKvNvfp4NoRope ? 288 : fmt == iob::kKvV4Pro ? 320 :
                     fmt == iob::kKvV4ProBf16Rope ? 384 : 576;
  TORCH_CHECK(pool.dim() == 2 && pool.size(1) == rb, "pool row bytes");
  iob::MlaDecodeArgs a{};
  if (q.has_value()) {
    req(*q, at::kBFloat16, "q");
    TORCH_CHECK(q->is_contiguous() && q->sizes() == q8.sizes(), "q [T, H, 576] bf16");
    a.q = q->data_ptr();
    a.q8_out = q8.data_ptr<uint8_t>();
    a.q_scale_out = q_scale.data_ptr<float>();
  }
  a.q8 = q8.data_ptr<uint8_t>();
  a.q_scale = q_scale.data_ptr<float>();
  a.pool = pool.data_ptr<uint8_t>();
  a.idx = idx.data_ptr<int>();
  a.out = out.data_ptr();
  if (lse.has_value()) {
    req(*lse, at::kFloat, "lse");
    TORCH_CHECK(lse->numel() >= T * H, "lse size");
    a.lse = lse->data_ptr<float>();
  }
  a.o_part = o_part.data_ptr<float>();
  a.lse_part = lse_part.data_ptr<float>();
  a.status = status.data_ptr<int>();
  a.T = T;
  a.H = H;
  a.topk = idx.size(1);
  a.idx_stride = idx.stride(0);
  a.fmt = fmt;
  a.pool_rows = static_cast<int>(std::min<int64_t>(pool.size(0), INT32_MAX));
  if (tok_sel.has_value()) {
    req(*tok_sel, at::kInt, "tok_sel");
    TORCH_CHECK(tok_sel->numel() >= T && row_lo >= 0, "tok_sel [T], row_lo >= 0");
    a.tok_sel = tok_sel->data_ptr<int>();
    a.sel = static_cast<int>(sel);
    a.row_lo = static_cast<int>(row_lo);
  }
  a.tiles_per_split = tiles_per_split;
  a.num_splits = num_splits;
  a.sm_scale = sm_scale;
  if (trace.has_value()) {
    req(*trace, at::kLong, "trace");
    TORCH_CHECK(trace->numel() >= 40 * 64, "trace size");
    a.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  if (num_splits > 1)
    TORCH_CHECK(o_part.numel() >= num_splits * T * H * 512 && lse_part.numel() >= num_splits * T * H,
                "split workspace too small");
  const at::cuda::CUDAGuard g(q8.device());
  CHECK_CUDA_OK(iob::mla_decode(a, stream()));
}

void indexer(const at::Tensor& q8, const at::Tensor& w, const at::Tensor& pool, const at::Tensor& page_table,
             c10::optional<at::Tensor> req_idx, const at::Tensor& limit, at::Tensor scores, at::Tensor out_slots,
             c10::optional<at::Tensor> out_pos, at::Tensor status, int64_t tiles_per_cta, int64_t max_tiles,
             int64_t do_logits, int64_t do_topk) {
  req(q8, at::kByte, "q8");
  req(w, at::kFloat, "w");
  req(pool, at::kByte, "pool");
  req(page_table, at::kInt, "page_table");
  req(limit, at::kInt, "limit");
  req(scores, at::kFloat, "scores");
  req(out_slots, at::kInt, "out_slots");
  req(status, at::kInt, "status");
  TORCH_CHECK(q8.dim() == 3 && q8.size(2) == 128 && q8.is_contiguous(), "q8 [T, Hi, 128]");
  TORCH_CHECK(pool.size(-1) == 64 * 132 || (pool.dim() == 1 && pool.numel() % (64 * 132) == 0), "index pool pages");
  iob::IndexerArgs a{};
  a.q8 = q8.data_ptr<uint8_t>();
  a.w = w.data_ptr<float>();
  a.pool = pool.data_ptr<uint8_t>();
  a.page_table = page_table.data_ptr<int>();
  if (req_idx.has_value()) { req(*req_idx, at::kInt, "req_idx"); a.req_idx = req_idx->data_ptr<int>(); }
  a.limit = limit.data_ptr<int>();
  a.scores = scores.data_ptr<float>();
  a.out_slots = out_slots.data_ptr<int>();
  if (out_pos.has_value()) { req(*out_pos, at::kInt, "out_pos"); a.out_pos = out_pos->data_ptr<int>(); }
  a.status = status.data_ptr<int>();
  a.T = q8.size(0);
  a.Hi = q8.size(1);
  a.pt_stride = page_table.size(1);
  a.score_stride = scores.size(1);
  a.tiles_per_cta = tiles_per_cta;
  a.max_tiles = max_tiles;
  a.topk = out_slots.size(1);
  TORCH_CHECK(scores.size(0) >= a.T && out_slots.size(0) >= a.T && w.numel() >= a.T * a.Hi, "shapes");
  const at::cuda::CUDAGuard g(q8.device());
  if (do_logits) CHECK_CUDA_OK(iob::indexer_logits(a, stream()));
  if (do_topk) CHECK_CUDA_OK(iob::indexer_topk(a, stream()));
}

void ar_norm2(const at::Tensor& peers, int64_t flag_offset, int64_t rows_cap, int64_t half, int64_t rank,
              at::Tensor epoch, at::Tensor resid, at::Tensor out, c10::optional<at::Tensor> w1,
              c10::optional<at::Tensor> w2, double eps, double plus_one, at::Tensor status, bool slots,
              int64_t mc, int64_t res_offset, int64_t rowflag_offset) {
  req(peers, at::kLong, "peers");
  req(epoch, at::kInt, "epoch");
  req(resid, at::kBFloat16, "resid");
  req(out, at::kBFloat16, "out");
  req(status, at::kInt, "status");
  TORCH_CHECK(resid.is_contiguous() && out.is_contiguous() && resid.dim() == 2, "resid [T, H]");
  iob::ArNormArgs a{};
  a.peers = reinterpret_cast<void* const*>(peers.data_ptr<int64_t>());
  a.flag_offset = flag_offset;
  a.rows_cap = rows_cap;
  a.H = resid.size(1);
  a.T = resid.size(0);
  a.half = half;
  a.rank = rank;
  a.nranks = peers.numel();
  a.epoch = epoch.data_ptr<int>();
  a.resid = resid.data_ptr();
  a.out = out.data_ptr();
  if (w1.has_value()) { req(*w1, at::kBFloat16, "w1"); a.w1 = w1->data_ptr(); }
  if (w2.has_value()) { req(*w2, at::kBFloat16, "w2"); a.w2 = w2->data_ptr(); }
  a.eps = eps;
  a.plus_one = plus_one;
  a.status = status.data_ptr<int>();
  a.slots = slots ? 1 : 0;
  a.mc = reinterpret_cast<void*>(static_cast<uintptr_t>(mc));
  a.res_offset = res_offset;
  a.rowflag_offset = rowflag_offset;
  const at::cuda::CUDAGuard g(resid.device());
  CHECK_CUDA_OK(iob::ar_norm2(a, stream()));
}

void moe_route(const at::Tensor& logits, const at::Tensor& bias, at::Tensor ids, at::Tensor wts, int64_t n_group,
               int64_t topk_group, double scale, int64_t ksplit) {
  req(logits, at::kFloat, "logits");
  req(bias, at::kFloat, "bias");
  req(ids, at::kInt, "ids");
  req(wts, at::kFloat, "wts");
  // logits [T, E], or the router GEMM's split-K partials [ksplit * T, E] (split-major)
  TORCH_CHECK(ksplit >= 1 && logits.dim() == 2 && logits.is_contiguous() && bias.numel() == logits.size(1) &&
              logits.size(0) == ksplit * ids.size(0), "logits [ksplit * T, E]");
  const at::cuda::CUDAGuard g(logits.device());
  CHECK_CUDA_OK(iob::moe_route(logits.data_ptr<float>(), bias.data_ptr<float>(), ids.data_ptr<int>(),
                               wts.data_ptr<float>(), ids.size(0), logits.size(1), ids.size(1), n_group, topk_group,
                               scale, stream(), ksplit));
}

void moe_gemm(const at::Tensor& wpack, const at::Tensor& x, const at::Tensor& x_scale, const at::Tensor& off,
              const at::Tensor& pairs, const c10::optional<at::Tensor>& pair_w, at::Tensor out,
              const c10::optional<at::Tensor>& out_scale, at::Tensor status, int64_t n_tiles, int64_t kc, int64_t G,
              int64_t NT, int64_t mode, int64_t src_div, int64_t src_limit, int64_t src_shared_base, double out_mul,
              int64_t num_ctas,
              int64_t kind, const c10::optional<at::Tensor>& expert_mul,
              const c10::optional<at::Tensor>& out_peers, int64_t out_offset, int64_t out_div, int64_t out_rank,
              int64_t out_shared_base, int64_t pairs_total, int64_t ksplit, int64_t split_rows, int64_t src_group,
              int64_t src_group_stride, const c10::optional<at::Tensor>& trace, bool pdl, bool static_index,
              const c10::optional<at::Tensor>& red_out, const c10::optional<at::Tensor>& tile_cnt,
              int64_t out_bcast) {
  req(wpack, at::kByte, "wpack");
  req(x, at::kByte, "x");
  req(off, at::kInt, "off");
  req(pairs, at::kInt, "pairs");
  req(status, at::kInt, "status");
  TORCH_CHECK(kind == 0 || kind == 1 || kind == 2, "kind");
  const int64_t sfw = kind == 0 ? 1 : (kind == 1 ? 4 : 0);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) == kc * 128, "x [rows, KC*128 bytes]");
  if (sfw)
    TORCH_CHECK(x_scale.scalar_type() == at::kInt && x_scale.dim() == 2 && x_scale.is_contiguous() &&
                    x_scale.size(1) == kc * sfw && x_scale.size(0) == x.size(0),
                "x_scale [rows, KC * words]");
  const int64_t E = off.numel() - 1;
  TORCH_CHECK(wpack.numel() == E * n_tiles * kc * G * (16384 + 512 * sfw), "wpack size");
  if (expert_mul.has_value())
    TORCH_CHECK(expert_mul->scalar_type() == at::kFloat && expert_mul->numel() >= E, "expert_mul fp32 [E]");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "out [pairs, N]");
  if (mode == iob::kMoeOutSwigluQuant) {
    req(out, at::kByte, "out");
    TORCH_CHECK(out_scale.has_value() && out_scale->scalar_type() == at::kInt && out_scale->dim() == 2 &&
                    out_scale->is_contiguous() && out_scale->size(1) >= n_tiles * (kind == 0 ? 1 : 2) &&
                    out.size(1) >= n_tiles * (kind == 0 ? 128 : 64),
                "out_scale [pairs, n_tiles words] / out [pairs, F bytes]");
  } else if (mode == iob::kMoeOutF32Split) {
    req(out, at::kFloat, "out");
    TORCH_CHECK(ksplit >= 1 && ksplit <= kc && out.size(1) >= n_tiles * G * 128 && out.size(0) >= ksplit * split_rows,
                "split-K partials [ksplit * split_rows, N] fp32");
  } else {
    req(out, at::kBFloat16, "out");
    TORCH_CHECK(out.size(1) >= n_tiles * G * 128, "out width");
    TORCH_CHECK(ksplit == 1, "split-K needs the fp32 partials mode");
  }
  if (mode == iob::kMoeOutBf16Weighted)
    TORCH_CHECK(pair_w.has_value() && pair_w->scalar_type() == at::kFloat, "pair_w fp32");
  iob::MoeGemmArgs a{};
  a.wpack = wpack.data_ptr<uint8_t>();
  a.x = x.data_ptr<uint8_t>();
  a.x_scale = sfw ? reinterpret_cast<const uint32_t*>(x_scale.data_ptr<int>()) : nullptr;
  a.expert_off = off.data_ptr<int>();
  a.pairs = pairs.data_ptr<int>();
  a.pair_w = pair_w.has_value() ? pair_w->data_ptr<float>() : nullptr;
  a.out = out.data_ptr();
  a.out_scale = out_scale.has_value() ? reinterpret_cast<uint32_t*>(out_scale->data_ptr<int>()) : nullptr;
  a.status = status.data_ptr<int>();
  a.E = static_cast<int>(E);
  a.n_tiles = static_cast<int>(n_tiles);
  a.KC = static_cast<int>(kc);
  a.G = static_cast<int>(G);
  a.NT = static_cast<int>(NT);
  a.mode = static_cast<int>(mode);
  a.src_div = static_cast<int>(src_div);
  a.src_limit = static_cast<int>(src_limit);
  a.src_shared_base = static_cast<int>(src_shared_base);
  a.x_stride = static_cast<int>(x.stride(0));
  a.out_stride = static_cast<int>(out.stride(0));
  a.out_scale_stride = out_scale.has_value() ? static_cast<int>(out_scale->stride(0)) : 0;
  a.ksplit = static_cast<int>(ksplit);
  a.split_rows = static_cast<int>(split_rows);
  a.src_group = static_cast<int>(src_group);
  a.src_group_stride = static_cast<int>(src_group_stride);
  a.pdl = pdl ? 1 : 0;
  a.static_index = static_index ? 1 : 0;
  if (red_out.has_value()) {
    TORCH_CHECK(mode == iob::kMoeOutF32Split && tile_cnt.has_value() && tile_cnt->scalar_type() == at::kInt &&
                    tile_cnt->is_contiguous() && red_out->dim() == 2 && red_out->stride(1) == 1 &&
                    (red_out->scalar_type() == at::kBFloat16 || red_out->scalar_type() == at::kFloat) &&
                    red_out->size(1) >= n_tiles * G * 128 && red_out->size(0) >= split_rows,
                "folded split-K: red_out [rows, N] bf16 / fp32 and an int32 tile counter array");
    a.red_out = red_out->data_ptr();
    a.tile_cnt = tile_cnt->data_ptr<int>();
    a.red_stride = static_cast<int>(red_out->stride(0));
    a.red_f32 = red_out->scalar_type() == at::kFloat ? 1 : 0;
  }
  if (trace.has_value()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->numel() >= iob::kMgEvCount && trace->is_cuda(),
                "trace int64 [>= kMgEvCount]");
    a.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  a.num_ctas = static_cast<int>(num_ctas);
  a.out_mul = static_cast<float>(out_mul);
  a.kind = static_cast<int>(kind);
  a.expert_mul = expert_mul.has_value() ? expert_mul->data_ptr<float>() : nullptr;
  if (out_peers.has_value()) {
    TORCH_CHECK(out_peers->scalar_type() == at::kLong && mode != iob::kMoeOutSwigluQuant && out_div > 0,
                "out_peers: int64 table, plain bf16 mode");
    a.out_peers = reinterpret_cast<const long long*>(out_peers->data_ptr<int64_t>());
  }
  a.out_offset = out_offset;
  a.out_div = static_cast<int>(out_div);
  a.out_rank = static_cast<int>(out_rank);
  a.out_shared_base = static_cast<int>(out_shared_base);
  a.pairs_total = static_cast<int>(pairs_total);
  a.out_bcast = static_cast<int>(out_bcast);
  TORCH_CHECK(out_bcast == 0 || (out_peers.has_value() && out_peers->numel() >= out_bcast &&
                                 out_rank < out_bcast && out_peers->is_cuda()),
              "out_bcast: a peer table of out_bcast entries, out_rank below it");
  const at::cuda::CUDAGuard g(x.device());
  CHECK_CUDA_OK(iob::moe_gemm(a, stream()));
}

void splitk_reduce(const at::Tensor& part, int64_t ksplit, at::Tensor out, const c10::optional<at::Tensor>& peers,
                   int64_t peer_offset, int64_t nbcast, int64_t rank) {
  req(part, at::kFloat, "part");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "splitk_reduce: bf16 or fp32 out");
  TORCH_CHECK(out.is_cuda(), "splitk_reduce: CUDA tensors");
  TORCH_CHECK(part.is_contiguous() && out.is_contiguous() && out.dim() == 2 &&
                  part.numel() >= ksplit * out.size(0) * out.size(1),
              "splitk_reduce shapes");
  if (peers.has_value())
    TORCH_CHECK(peers->scalar_type() == at::kLong && peers->is_cuda() && peers->numel() >= nbcast && nbcast >= 1 &&
                    rank >= 0 && rank < nbcast && out.scalar_type() == at::kBFloat16,
                "splitk_reduce push: int64 peer table of nbcast entries, bf16 rows");
  const at::cuda::CUDAGuard g(out.device());
  CHECK_CUDA_OK(iob::splitk_reduce(part.data_ptr<float>(), static_cast<int>(ksplit), static_cast<int>(out.size(0)),
                                   static_cast<int>(out.size(1)), out.data_ptr(), out.scalar_type() == at::kFloat,
                                   stream(),
                                   peers.has_value() ? reinterpret_cast<const long long*>(peers->data_ptr<int64_t>())
                                                     : nullptr,
                                   peer_offset, static_cast<int>(nbcast), static_cast<int>(rank)));
}

void moe_align(const at::Tensor& ids, int64_t e0, int64_t E, int64_t extra, at::Tensor off, at::Tensor pairs) {
  req(ids, at::kInt, "ids");
  req(off, at::kInt, "off");
  req(pairs, at::kInt, "pairs");
  // off has E + 1 entries (routed only) or E + 2 (one shared bucket after the routed ones, `extra` rows)
  const bool shared = off.numel() == E + 2;
  TORCH_CHECK(ids.is_contiguous() && (shared || (off.numel() == E + 1 && extra == 0)) &&
                  pairs.numel() >= ids.numel() + extra,
              "moe_align shapes");
  const at::cuda::CUDAGuard g(ids.device());
  CHECK_CUDA_OK(iob::moe_align(ids.data_ptr<int>(), static_cast<int>(ids.numel()), static_cast<int>(e0),
                               static_cast<int>(E), shared ? 1 : 0, static_cast<int>(extra), off.data_ptr<int>(),
                               pairs.data_ptr<int>(), stream()));
}

void moe_combine(const at::Tensor& rows, int64_t T, int64_t topk, int64_t shared_base,
                 const c10::optional<at::Tensor>& w, at::Tensor y) {
  req(rows, at::kBFloat16, "rows");
  req(y, at::kBFloat16, "y");
  TORCH_CHECK(rows.is_contiguous() && y.is_contiguous() && rows.size(1) == y.size(1) &&
                  rows.size(0) >= T * topk && (shared_base < 0 || rows.size(0) >= shared_base + T) && y.size(0) >= T,
              "moe_combine shapes");
  if (w.has_value()) TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() >= T * topk, "w");
  const at::cuda::CUDAGuard g(y.device());
  CHECK_CUDA_OK(iob::moe_combine(rows.data_ptr(), static_cast<int>(T), static_cast<int>(topk),
                                 static_cast<int>(y.size(1)), static_cast<int>(shared_base),
                                 w.has_value() ? w->data_ptr<float>() : nullptr, y.data_ptr(), stream()));
}

void ep_dispatch(const at::Tensor& peers, const at::Tensor& xq, const at::Tensor& xs, const at::Tensor& ids,
                 int64_t off_x, int64_t off_s, int64_t off_ids, int64_t T_max, int64_t rank, int64_t world,
                 int64_t E_loc) {
  req(peers, at::kLong, "peers");
  req(xq, at::kByte, "xq");
  req(xs, at::kInt, "xs");
  req(ids, at::kInt, "ids");
  TORCH_CHECK(xq.is_contiguous() && xs.is_contiguous() && ids.is_contiguous() && ids.dim() == 2 &&
                  xq.size(0) >= ids.size(0) && xs.size(0) >= ids.size(0) && peers.numel() == world,
              "ep_dispatch shapes");
  iob::EpDispatchArgs a{};
  a.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  a.xq = xq.data_ptr<uint8_t>();
  a.xs = reinterpret_cast<const uint8_t*>(xs.data_ptr<int>());
  a.ids = ids.data_ptr<int>();
  a.off_x = off_x;
  a.off_s = off_s;
  a.off_ids = off_ids;
  a.T = static_cast<int>(ids.size(0));
  a.T_max = static_cast<int>(T_max);
  a.topk = static_cast<int>(ids.size(1));
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.E_loc = static_cast<int>(E_loc);
  a.row_bytes = static_cast<int>(xq.size(1));
  a.scale_bytes = static_cast<int>(xs.size(1) * 4);
  const at::cuda::CUDAGuard g(xq.device());
  CHECK_CUDA_OK(iob::ep_dispatch(a, stream()));
}

void dcp_merge(const at::Tensor& peers, int64_t off_data, int64_t off_flags, int64_t T, int64_t T_max, int64_t H,
               int64_t rank, int64_t nranks, int64_t half, at::Tensor epoch, at::Tensor out,
               const c10::optional<at::Tensor>& lse_out, at::Tensor status) {
  req(peers, at::kLong, "peers");
  req(epoch, at::kInt, "epoch");
  req(out, at::kBFloat16, "out");
  req(status, at::kInt, "status");
  TORCH_CHECK(out.is_contiguous() && out.size(0) >= T && out.size(1) == H / nranks && out.size(2) == 512, "out");
  if (lse_out.has_value()) TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->numel() >= T * H / nranks, "lse");
  iob::DcpMergeArgs a{};
  a.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  a.off_data = off_data;
  a.off_flags = off_flags;
  a.out = out.data_ptr();
  a.lse_out = lse_out.has_value() ? lse_out->data_ptr<float>() : nullptr;
  a.epoch = epoch.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.T = static_cast<int>(T);
  a.T_max = static_cast<int>(T_max);
  a.H = static_cast<int>(H);
  a.Hg = static_cast<int>(H / nranks);
  a.rank = static_cast<int>(rank);
  a.nranks = static_cast<int>(nranks);
  a.half = static_cast<int>(half);
  const at::cuda::CUDAGuard g(out.device());
  CHECK_CUDA_OK(iob::dcp_merge(a, stream()));
}

void glmflash_write(const at::Tensor& nope, const at::Tensor& slot, at::Tensor pool) {
  req(nope, at::kBFloat16, "nope");
  req(slot, at::kInt, "slot");
  req(pool, at::kByte, "pool");
  TORCH_CHECK(nope.dim() == 2 && nope.size(1) == 512 && nope.stride(1) == 1 && pool.size(1) == 288 &&
                  slot.numel() == nope.size(0),
              "glmflash_write shapes");
  const at::cuda::CUDAGuard g(nope.device());
  CHECK_CUDA_OK(iob::glmflash_write(nope.data_ptr(), static_cast<int>(nope.stride(0)), slot.data_ptr<int>(),
                                    pool.data_ptr<uint8_t>(), static_cast<int>(nope.size(0)), stream()));
}

void v4pro_write(const at::Tensor& x, const at::Tensor& slot, at::Tensor pool, int64_t rope_bf16) {
  req(x, at::kBFloat16, "x");
  req(slot, at::kInt, "slot");
  req(pool, at::kByte, "pool");
  TORCH_CHECK(x.dim() == 2 && x.size(1) == 512 && x.stride(1) == 1 && pool.size(1) == (rope_bf16 ? 384 : 320) &&
                  slot.numel() == x.size(0),
              "v4pro_write shapes");
  const at::cuda::CUDAGuard g(x.device());
  CHECK_CUDA_OK(iob::v4pro_write(x.data_ptr(), static_cast<int>(x.stride(0)), slot.data_ptr<int>(),
                                 pool.data_ptr<uint8_t>(), static_cast<int>(x.size(0)), static_cast<int>(rope_bf16),
                                 stream()));
}

void pd_copy(const at::Tensor& src, int64_t dst_ptr, const at::Tensor& src_pages, const at::Tensor& dst_pages,
             int64_t page_bytes, int64_t layers, int64_t src_layer_stride, int64_t dst_layer_stride) {
  req(src, at::kByte, "src");
  req(src_pages, at::kInt, "src_pages");
  req(dst_pages, at::kInt, "dst_pages");
  TORCH_CHECK(src_pages.numel() == dst_pages.numel() && src.is_contiguous(), "pd_copy shapes");
  iob::PdCopyArgs a{};
  a.src = src.data_ptr<uint8_t>();
  a.dst = reinterpret_cast<void*>(dst_ptr);
  a.src_pages = src_pages.data_ptr<int>();
  a.dst_pages = dst_pages.data_ptr<int>();
  a.page_bytes = page_bytes;
  a.src_layer_stride = src_layer_stride;
  a.dst_layer_stride = dst_layer_stride;
  a.n_pairs = static_cast<int>(src_pages.numel());
  a.layers = static_cast<int>(layers);
  const at::cuda::CUDAGuard g(src.device());
  CHECK_CUDA_OK(iob::pd_copy(a, stream()));
}

void pd_signal(int64_t peer_flag_ptr, int64_t value, const at::Tensor& like) {
  const at::cuda::CUDAGuard g(like.device());
  CHECK_CUDA_OK(iob::pd_signal(reinterpret_cast<int*>(peer_flag_ptr), static_cast<int>(value), stream()));
}

void pd_wait(const at::Tensor& flag, int64_t value, at::Tensor status) {
  req(flag, at::kInt, "flag");
  req(status, at::kInt, "status");
  const at::cuda::CUDAGuard g(flag.device());
  CHECK_CUDA_OK(iob::pd_wait(flag.data_ptr<int>(), static_cast<int>(value), status.data_ptr<int>(), stream()));
}

void kda_decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g_proj,
                const at::Tensor& dt_bias, const at::Tensor& A_log, const at::Tensor& beta, const at::Tensor& g2,
                const at::Tensor& norm_w, const at::Tensor& cwq, const at::Tensor& cwk, const at::Tensor& cwv,
                at::Tensor csq, at::Tensor csk, at::Tensor csv, at::Tensor state, at::Tensor out, double scale) {
  const std::vector<const at::Tensor*> bf = {&q, &k, &v, &g_proj, &g2};
  for (const at::Tensor* t : bf) req(*t, at::kBFloat16, "kda bf16 input");
  const std::vector<const at::Tensor*> f32 = {&dt_bias, &A_log, &beta, &norm_w, &cwq, &cwk, &cwv, &csq, &csk, &csv,
                                              &state};
  for (const at::Tensor* t : f32) req(*t, at::kFloat, "kda fp32 input");
  req(out, at::kBFloat16, "out");
  const int64_t B = q.size(0), H = q.size(1), DK = q.size(2), HV = v.size(1), DV = v.size(2), W = cwq.size(1);
  TORCH_CHECK(k.sizes() == q.sizes() && g_proj.size(2) == DK && g2.size(1) == HV && g2.size(2) == DV &&
                  state.numel() == B * HV * DV * DK && csq.numel() == B * H * DK * (W - 1) &&
                  csv.numel() == B * HV * DV * (W - 1) && out.numel() == B * HV * DV,
              "kda shapes");
  const std::vector<const at::Tensor*> all = {&q, &k, &v, &g_proj, &g2, &csq, &csk, &csv, &state, &out, &beta};
  for (const at::Tensor* t : all) TORCH_CHECK(t->is_contiguous(), "kda: contiguous tensors");
  iob::KdaDecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.g_proj = reinterpret_cast<const __nv_bfloat16*>(g_proj.data_ptr());
  a.dt_bias = dt_bias.data_ptr<float>();
  a.A_log = A_log.data_ptr<float>();
  a.beta = beta.data_ptr<float>();
  a.g2 = reinterpret_cast<const __nv_bfloat16*>(g2.data_ptr());
  a.norm_w = norm_w.data_ptr<float>();
  a.conv_wq = cwq.data_ptr<float>();
  a.conv_wk = cwk.data_ptr<float>();
  a.conv_wv = cwv.data_ptr<float>();
  a.conv_q = csq.data_ptr<float>();
  a.conv_k = csk.data_ptr<float>();
  a.conv_v = csv.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.scale = static_cast<float>(scale);
  a.B = static_cast<int>(B);
  a.H = static_cast<int>(H);
  a.HV = static_cast<int>(HV);
  a.DK = static_cast<int>(DK);
  a.DV = static_cast<int>(DV);
  a.W = static_cast<int>(W);
  a.beta_headwise = beta.dim() == 3 ? 1 : 0;
  const at::cuda::CUDAGuard g(q.device());
  CHECK_CUDA_OK(iob::kda_decode(a, stream()));
}

void qar_allreduce(const at::Tensor& peers, const std::vector<int64_t>& offs, const at::Tensor& x, at::Tensor y,
                   int64_t T_max, int64_t rank, int64_t nranks, at::Tensor epoch, at::Tensor status) {
  req(peers, at::kLong, "peers");
  req(x, at::kBFloat16, "x");
  req(y, at::kBFloat16, "y");
  req(epoch, at::kInt, "epoch");
  req(status, at::kInt, "status");
  TORCH_CHECK(offs.size() == 5 && x.dim() == 2 && x.is_contiguous() && y.sizes() == x.sizes() && y.is_contiguous(),
              "qar shapes");
  iob::QarArgs a{};
  a.peers = reinterpret_cast<const long long*>(peers.data_ptr<int64_t>());
  a.off_recv_q = offs[0];
  a.off_recv_s = offs[1];
  a.off_gather_q = offs[2];
  a.off_gather_s = offs[3];
  a.off_flags = offs[4];
  a.x = x.data_ptr();
  a.y = y.data_ptr();
  a.epoch = epoch.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.T = static_cast<int>(x.size(0));
  a.T_max = static_cast<int>(T_max);
  a.H = static_cast<int>(x.size(1));
  a.G = a.H / 128;
  a.nranks = static_cast<int>(nranks);
  a.per = (a.G + a.nranks - 1) / a.nranks;
  a.rank = static_cast<int>(rank);
  const at::cuda::CUDAGuard g(x.device());
  CHECK_CUDA_OK(iob::qar_allreduce(a, stream()));
}

void ep_barrier(const at::Tensor& peers, int64_t off_flags, int64_t rank, int64_t world, at::Tensor epoch,
                at::Tensor status) {
  req(peers, at::kLong, "peers");
  req(epoch, at::kInt, "epoch");
  req(status, at::kInt, "status");
  const at::cuda::CUDAGuard g(epoch.device());
  CHECK_CUDA_OK(iob::ep_barrier(reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), off_flags,
                                static_cast<int>(rank), static_cast<int>(world), epoch.data_ptr<int>(),
                                status.data_ptr<int>(), stream()));
}

void rmsnorm_quant(const at::Tensor& x, const c10::optional<at::Tensor>& w, double eps, double plus_one, at::Tensor q,
                   at::Tensor sc, int64_t fmt) {
  req(x, at::kBFloat16, "x");
  req(q, at::kByte, "q");
  req(sc, at::kInt, "sc");
  TORCH_CHECK(fmt == 0 || fmt == 1, "fmt");
  TORCH_CHECK(x.is_contiguous() && q.is_contiguous() && sc.is_contiguous() && q.size(0) == x.size(0) &&
                  q.size(1) * (fmt == 0 ? 1 : 2) == x.size(1) && sc.size(0) == x.size(0) &&
                  sc.size(1) * (fmt == 0 ? 128 : 64) == x.size(1),
              "rmsnorm_quant shapes");
  if (w.has_value()) TORCH_CHECK(w->scalar_type() == at::kBFloat16 && w->numel() == x.size(1), "w");
  const at::cuda::CUDAGuard g(x.device());
  CHECK_CUDA_OK(iob::rmsnorm_quant(x.data_ptr(), w.has_value() ? w->data_ptr() : nullptr, static_cast<float>(eps),
                                   static_cast<float>(plus_one), static_cast<int>(x.size(0)),
                                   static_cast<int>(x.size(1)), static_cast<int>(fmt), q.data_ptr<uint8_t>(),
                                   reinterpret_cast<uint32_t*>(sc.data_ptr<int>()), stream()));
}

void act_quant(const at::Tensor& gu, bool gelu, at::Tensor q, at::Tensor sc, int64_t fmt) {
  req(gu, at::kBFloat16, "gate_up");
  req(q, at::kByte, "q");
  req(sc, at::kInt, "sc");
  TORCH_CHECK(fmt == 0 || fmt == 1, "fmt");
  const int64_t F = gu.size(1) / 2;
  TORCH_CHECK(gu.dim() == 2 && gu.size(1) % 2 == 0 && gu.is_contiguous() && q.is_contiguous() && sc.is_contiguous() &&
                  q.size(0) == gu.size(0) && q.size(1) * (fmt == 0 ? 1 : 2) == F && sc.size(0) == gu.size(0) &&
                  sc.size(1) * (fmt == 0 ? 128 : 64) == F,
              "act_quant shapes");
  const at::cuda::CUDAGuard g(gu.device());
  CHECK_CUDA_OK(iob::act_quant(gu.data_ptr(), static_cast<int>(gu.size(0)), static_cast<int>(F), gelu,
                               static_cast<int>(fmt), q.data_ptr<uint8_t>(),
                               reinterpret_cast<uint32_t*>(sc.data_ptr<int>()), stream()));
}

void umma_gemm_test(const at::Tensor& A, const at::Tensor& B, at::Tensor C, int64_t sw64) {
  req(A, at::kBFloat16, "A");
  req(B, at::kBFloat16, "B");
  req(C, at::kFloat, "C");
  const at::cuda::CUDAGuard g(A.device());
  CHECK_CUDA_OK(iob::umma_gemm_test(A.data_ptr(), B.data_ptr(), C.data_ptr<float>(), A.size(0), B.size(0),
                                    A.size(1), static_cast<int>(sw64), stream()));
}

void umma_f8_mn_test(const at::Tensor& A, const at::Tensor& B, at::Tensor C) {
  req(A, at::kByte, "A");
  req(B, at::kByte, "B");
  req(C, at::kFloat, "C");
  TORCH_CHECK(A.size(0) == 128 && B.size(0) == A.size(1) && C.size(0) == 128 && C.size(1) == B.size(1), "shapes");
  const at::cuda::CUDAGuard g(A.device());
  CHECK_CUDA_OK(iob::umma_f8_mn_test(A.data_ptr(), B.data_ptr(), C.data_ptr<float>(), B.size(1), A.size(1), stream()));
}

void nvfp4_lut_test(const at::Tensor& words, at::Tensor out) {
  req(words, at::kInt, "words");
  req(out, at::kInt, "out");
  const at::cuda::CUDAGuard g(words.device());
  CHECK_CUDA_OK(iob::nvfp4_lut_test(reinterpret_cast<const uint32_t*>(words.data_ptr<int>()), words.numel(),
                                    out.data_ptr<int>(), stream()));
}

void mla_prep_kv(const at::Tensor& ya, const at::Tensor& q_norm, const at::Tensor& kv_norm, const at::Tensor& ik_w,
                 const at::Tensor& ik_b, const at::Tensor& rope, const at::Tensor& pos, const at::Tensor& slot,
                 at::Tensor qa_out, at::Tensor latent_pool, at::Tensor index_pool, at::Tensor iw_out, double iw_scale,
                 int64_t q_lora, int64_t Hi, double eps, const c10::optional<at::Tensor>& lat_slot,
                 const c10::optional<at::Tensor>& qa_q, const c10::optional<at::Tensor>& qa_s,
                 const c10::optional<at::Tensor>& latent_pool2, int64_t split_slot) {
  req(ya, at::kBFloat16, "ya");
  req(rope, at::kFloat, "rope");
  req(pos, at::kInt, "pos");
  req(slot, at::kInt, "slot");
  req(qa_out, at::kBFloat16, "qa_out");
  req(latent_pool, at::kByte, "latent_pool");
  req(index_pool, at::kByte, "index_pool");
  req(iw_out, at::kFloat, "iw_out");
  const int64_t T = pos.numel();
  TORCH_CHECK(ya.dim() == 2 && ya.stride(1) == 1 && ya.size(0) == T && ya.size(1) >= q_lora + 576 + 128 + Hi,
              "ya [T, >= q_lora + 704 + Hi]");
  TORCH_CHECK(rope.dim() == 2 && rope.size(1) == 64 && rope.is_contiguous(), "rope [max_pos, 64]");
  TORCH_CHECK(qa_out.is_contiguous() && qa_out.numel() == T * q_lora && iw_out.is_contiguous() &&
                  iw_out.numel() == T * Hi && slot.numel() == T,
              "qa_out [T, q_lora], iw_out [T, Hi]");
  TORCH_CHECK(latent_pool.dim() == 2 && (latent_pool.size(1) == 352 || latent_pool.size(1) == 576) &&
                  latent_pool.is_contiguous() && index_pool.is_contiguous() && index_pool.size(-1) == 64 * 132,
              "pools");
  iob::MlaPrepArgs a{};
  a.ya = ya.data_ptr();
  a.ya_stride = static_cast<int>(ya.stride(0));
  a.q_norm = q_norm.data_ptr();
  a.kv_norm = kv_norm.data_ptr();
  a.ik_w = ik_w.data_ptr();
  a.ik_b = ik_b.data_ptr();
  a.rope = rope.data_ptr<float>();
  a.pos = pos.data_ptr<int>();
  a.slot = slot.data_ptr<int>();
  if (lat_slot.has_value()) {
    req(*lat_slot, at::kInt, "lat_slot");
    TORCH_CHECK(lat_slot->numel() == T, "lat_slot [T]");
    a.lat_slot = lat_slot->data_ptr<int>();
  }
  if (qa_q.has_value()) {
    TORCH_CHECK(qa_s.has_value() && qa_q->scalar_type() == at::kByte && qa_s->scalar_type() == at::kInt &&
                    qa_q->is_contiguous() && qa_s->is_contiguous() && qa_q->numel() == T * q_lora &&
                    qa_s->numel() == T * (q_lora / 128) && q_lora % 128 == 0,
                "qa_q uint8 [T, q_lora], qa_s int32 [T, q_lora / 128]");
    a.qa_q = qa_q->data_ptr<uint8_t>();
    a.qa_s = reinterpret_cast<uint32_t*>(qa_s->data_ptr<int>());
  }
  a.qa_out = qa_out.data_ptr();
  a.latent_pool = latent_pool.data_ptr<uint8_t>();
  a.latent_fmt = latent_pool.size(1) == 352 ? iob::kKvNvfp4 : iob::kKvFp8;
  if (latent_pool2.has_value()) {
    req(*latent_pool2, at::kByte, "latent_pool2");
    TORCH_CHECK(latent_pool2->dim() == 2 && (latent_pool2->size(1) == 352 || latent_pool2->size(1) == 576) &&
                    latent_pool2->is_contiguous() && split_slot >= 0,
                "latent_pool2 [slots, 352 | 576]");
    a.latent_pool2 = latent_pool2->data_ptr<uint8_t>();
    a.latent_fmt2 = latent_pool2->size(1) == 352 ? iob::kKvNvfp4 : iob::kKvFp8;
    a.split_slot = static_cast<int>(split_slot);
  }
  a.index_pool = index_pool.data_ptr<uint8_t>();
  a.iw_out = iw_out.data_ptr<float>();
  a.iw_scale = static_cast<float>(iw_scale);
  a.T = static_cast<int>(T);
  a.q_lora = static_cast<int>(q_lora);
  a.Hi = static_cast<int>(Hi);
  a.eps = static_cast<float>(eps);
  const at::cuda::CUDAGuard g(ya.device());
  CHECK_CUDA_OK(iob::mla_prep_kv(a, stream()));
}

void mla_prep_q(const at::Tensor& yb, const at::Tensor& rope, const at::Tensor& pos, at::Tensor qf, at::Tensor q8,
                at::Tensor w_eff, const at::Tensor& iw, int64_t H, int64_t dn, int64_t Hi) {
  req(yb, at::kBFloat16, "yb");
  req(rope, at::kFloat, "rope");
  req(pos, at::kInt, "pos");
  req(qf, at::kBFloat16, "qf");
  req(q8, at::kByte, "q8");
  req(w_eff, at::kFloat, "w_eff");
  req(iw, at::kFloat, "iw");
  const int64_t T = pos.numel();
  TORCH_CHECK(yb.dim() == 2 && yb.stride(1) == 1 && yb.size(0) == T && yb.size(1) >= H * (dn + 64) + Hi * 128,
              "yb [T, >= H (dn + 64) + Hi 128]");
  TORCH_CHECK(qf.is_contiguous() && qf.numel() == T * H * 576 && q8.is_contiguous() && q8.numel() == T * Hi * 128 &&
                  w_eff.numel() == T * Hi && iw.numel() == T * Hi && rope.size(1) == 64,
              "qf [T, H, 576], q8 [T, Hi, 128], w_eff / iw [T, Hi]");
  iob::MlaPrepArgs a{};
  a.yb = yb.data_ptr();
  a.yb_stride = static_cast<int>(yb.stride(0));
  a.rope = rope.data_ptr<float>();
  a.pos = pos.data_ptr<int>();
  a.qf = qf.data_ptr();
  a.q8 = q8.data_ptr<uint8_t>();
  a.w_eff = w_eff.data_ptr<float>();
  a.iw_out = const_cast<float*>(iw.data_ptr<float>());
  a.T = static_cast<int>(T);
  a.H = static_cast<int>(H);
  a.dn = static_cast<int>(dn);
  a.Hi = static_cast<int>(Hi);
  const at::cuda::CUDAGuard g(yb.device());
  CHECK_CUDA_OK(iob::mla_prep_q(a, stream()));
}

std::vector<int64_t> sm_lanes(int64_t device, int64_t first_sms) {
  unsigned long long streams[2] = {0, 0};
  int sms[2] = {0, 0};
  char err[256] = {0};
  TORCH_CHECK(iob::sm_lanes_create(static_cast<int>(device), static_cast<int>(first_sms), streams, sms, err,
                                   sizeof(err)) == 0, "sm_lanes: ", err);
  return {static_cast<int64_t>(streams[0]), static_cast<int64_t>(streams[1]), sms[0], sms[1]};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("rmsnorm", &rmsnorm);
  m.def("act_mul", &act_mul);
  m.def("embed", &embed);
  m.def("argmax", &argmax);
  m.def("gqa_prep", &gqa_prep);
  m.def("mla_quant_write", &mla_quant_write);
  m.def("index_key_write", &index_key_write);
  m.def("gqa_decode", &gqa_decode);
  m.def("mla_decode", &mla_decode);
  m.def("indexer", &indexer);
  m.def("ar_norm2", &ar_norm2);
  m.def("moe_route", &moe_route);
  m.def("moe_gemm", &moe_gemm);
  m.def("moe_align", &moe_align);
  m.def("moe_combine", &moe_combine);
  m.def("rmsnorm_quant", &rmsnorm_quant);
  m.def("gqa_extend", &gqa_extend);
  m.def("act_quant", &act_quant);
  m.def("splitk_reduce", &splitk_reduce);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_barrier", &ep_barrier);
  m.def("dcp_merge", &dcp_merge);
  m.def("glmflash_write", &glmflash_write);
  m.def("pd_copy", &pd_copy);
  m.def("kda_decode", &kda_decode);
  m.def("qar_allreduce", &qar_allreduce);
  m.def("pd_signal", &pd_signal);
  m.def("pd_wait", &pd_wait);
  m.def("v4pro_write", &v4pro_write);
  m.def("umma_gemm_test", &umma_gemm_test);
  m.def("umma_f8_mn_test", &umma_f8_mn_test);
  m.def("nvfp4_lut_test", &nvfp4_lut_test);
  m.def("sm_lanes", &sm_lanes);
  m.def("mla_prep_kv", &mla_prep_kv);
  m.def("mla_prep_q", &mla_prep_q);
}
