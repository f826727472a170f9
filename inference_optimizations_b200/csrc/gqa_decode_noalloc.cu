// Allocation-free entry point of the GQA split-K decode kernel (declared in gqa_decode_noalloc.h, which explains
// who needs it).  The split-K scratch lives in a file-scope device array; host code never passes the array's name to
// a kernel (on the host it is only a stand-in symbol) but the device address cudaGetSymbolAddress returns for it.
#include <mutex>

#include "gqa_decode_noalloc.h"
#include "kernels.h"

namespace {

struct NoAllocScratch {
  float o_part[IOB_NOALLOC_MAX_PARTIAL_FLOATS];
  float lse_part[IOB_NOALLOC_MAX_PARTIAL_ROWS];
  int status[64];
};

// One instance per GPU that loads the library; kept until process exit.
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

std::mutex g_setup_mu;

// Device address of the scratch on the current device.  Resolved on every call with that device current (the
// lookup allocates nothing and is cheap), so an address is never reused after the device's context was torn down
// and the module reloaded.
int scratch_for_current_device(NoAllocScratch** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return IOB_NOALLOC_ESETUP;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) return IOB_NOALLOC_ESETUP;
  *out = static_cast<NoAllocScratch*>(p);
  return IOB_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int iob_gqa_decode_noalloc(
    const void* q, const void* pool, const int* page_table, int pt_stride, const int* req_idx, const int* kv_len,
    void* out, int B, int n_q, int Hq, int Hk, int D, int window, int fmt, int tiles_per_split, int num_splits,
    float sm_scale, float k_scale, float v_scale, int exact, cudaStream_t stream) {
  if (B == 0) return IOB_NOALLOC_OK;
  if (!q || !pool || !page_table || !kv_len || !out || B < 0 || n_q < 1 || Hk < 1 || Hq % Hk != 0 ||
      num_splits < 1 || tiles_per_split < 1 || (fmt != iob::kKvBf16 && fmt != iob::kKvFp8 && fmt != iob::kKvNvfp4))
    return IOB_NOALLOC_EINVAL;
  // rows per partial: the same rule the kernel launcher uses to pick its row tile
  const int R = n_q * (Hq / Hk);
  const int rmax = (R <= 2 && fmt != iob::kKvBf16 && !exact) ? 2 : (R <= 8 ? 8 : 16);
  if (R > 16) return IOB_NOALLOC_EINVAL;
  const long long rows = static_cast<long long>(B) * Hk * num_splits * rmax;
  if (num_splits > 1 && (rows > IOB_NOALLOC_MAX_PARTIAL_ROWS || rows * D > IOB_NOALLOC_MAX_PARTIAL_FLOATS))
    return IOB_NOALLOC_ETOOBIG;
  NoAllocScratch* s = nullptr;
  const int rc = scratch_for_current_device(&s);
  if (rc != IOB_NOALLOC_OK) return rc;
  // the bounded waits of the kernel report into the status word: clear it for this call (not an allocation)
  cudaError_t e = cudaMemsetAsync(s->status, 0, sizeof(int), stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  iob::GqaDecodeArgs a{};
  a.q = q;
  a.pool = static_cast<const uint8_t*>(pool);
  a.page_table = page_table;
  a.req_idx = req_idx;
  a.kv_len = kv_len;
  a.out = out;
  a.o_part = s->o_part;
  a.lse_part = s->lse_part;
  a.status = s->status;
  a.B = B;
  a.n_q = n_q;
  a.Hq = Hq;
  a.Hk = Hk;
  a.D = D;
  a.pt_stride = pt_stride;
  a.page = 64;
  a.window = window;
  a.fmt = fmt;
  a.tiles_per_split = tiles_per_split;
  a.num_splits = num_splits;
  a.sm_scale = sm_scale;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.trace = nullptr;
  a.exact = exact;
  e = iob::gqa_decode(a, stream);
  return static_cast<int>(e);
}

extern "C" __attribute__((visibility("default"))) int iob_gqa_decode_noalloc_status(int* host_out,
                                                                                   cudaStream_t stream) {
  if (!host_out) return IOB_NOALLOC_EINVAL;
  NoAllocScratch* s = nullptr;
  const int rc = scratch_for_current_device(&s);
  if (rc != IOB_NOALLOC_OK) return rc;
  cudaError_t e = cudaMemcpyAsync(host_out, s->status, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  return static_cast<int>(e);
}

extern "C" __attribute__((visibility("default"))) const char* iob_gqa_decode_noalloc_strerror(int code) {
  switch (code) {
    case IOB_NOALLOC_OK: return "ok";
    case IOB_NOALLOC_ETOOBIG:
      return "split-K workspace exceeds the built-in scratch (max 1M partial floats / 64K partial rows): use fewer "
             "splits or the allocating entry point";
    case IOB_NOALLOC_EINVAL: return "invalid argument";
    case IOB_NOALLOC_ESETUP: return "could not resolve the scratch address on the current device";
    default: return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}
