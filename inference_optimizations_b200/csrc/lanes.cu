// SM partitions for the prefill / decode lanes: two green contexts over disjoint SM sets of one GPU, one stream each.
//
// Driver green-context API (CUDA 12.4+): the device's SM resource is split into a group of `first_sms` SMs and the
// remaining SMs; each set becomes a green context, and a stream created in it runs its kernels on that set only
// (launches from the runtime API on that stream included).  Partitions on sm_90 and later are multiples of 8 SMs, and
// the driver rounds the requested count up to that granule.  The contexts and streams are never destroyed: they live
// as long as the process (destroying a green context while a stream or graph of it is referenced ends the CUDA
// context).  Host code only; no kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>

#include "kernels.h"

namespace iob {
namespace {
// Driver entry points are looked up through the runtime (cudaGetDriverEntryPoint), so the extension does not link
// libcuda and still imports on a machine without a GPU driver.
typedef CUresult (*PfnDeviceGet)(CUdevice*, int);
typedef CUresult (*PfnGetDevResource)(CUdevice, CUdevResource*, CUdevResourceType);
typedef CUresult (*PfnSplitByCount)(CUdevResource*, unsigned int*, const CUdevResource*, CUdevResource*, unsigned int,
                                    unsigned int);
typedef CUresult (*PfnGenerateDesc)(CUdevResourceDesc*, CUdevResource*, unsigned int);
typedef CUresult (*PfnGreenCtxCreate)(CUgreenCtx*, CUdevResourceDesc, CUdevice, unsigned int);
typedef CUresult (*PfnGreenCtxStreamCreate)(CUstream*, CUgreenCtx, unsigned int, int);
typedef CUresult (*PfnGreenCtxDestroy)(CUgreenCtx);
typedef CUresult (*PfnStreamDestroy)(CUstream);
typedef CUresult (*PfnGetErrorString)(CUresult, const char**);

template <typename T>
bool entry(const char* name, T& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      p == nullptr)
    return false;
  fn = reinterpret_cast<T>(p);
  return true;
}

int fail(char* err, int errlen, const char* what, CUresult r, PfnGetErrorString es) {
  const char* s = nullptr;
  if (es) es(r, &s);
  snprintf(err, errlen, "%s: %s", what, s ? s : "driver error");
  return -1;
}
}  // namespace

// Restores the caller's current device on every return path (the lanes belong to `device`, the calling thread's
// torch work stays where it was).
struct DeviceRestore {
  int prev = -1;
  DeviceRestore() { cudaGetDevice(&prev); }
  ~DeviceRestore() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int sm_lanes_create(int device, int first_sms, unsigned long long* streams, int* sms, char* err, int errlen) {
  DeviceRestore restore;
  if (cudaSetDevice(device) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
    snprintf(err, errlen, "cudaSetDevice(%d) failed", device);
    return -1;
  }
  PfnDeviceGet device_get;
  PfnGetDevResource get_res;
  PfnSplitByCount split;
  PfnGenerateDesc gen_desc;
  PfnGreenCtxCreate gctx_create;
  PfnGreenCtxStreamCreate gstream_create;
  PfnGreenCtxDestroy gctx_destroy = nullptr;
  PfnStreamDestroy stream_destroy = nullptr;
  PfnGetErrorString es = nullptr;
  entry("cuGetErrorString", es);
  entry("cuGreenCtxDestroy", gctx_destroy);
  entry("cuStreamDestroy", stream_destroy);
  if (!entry("cuDeviceGet", device_get) || !entry("cuDeviceGetDevResource", get_res) ||
      !entry("cuDevSmResourceSplitByCount", split) || !entry("cuDevResourceGenerateDesc", gen_desc) ||
      !entry("cuGreenCtxCreate", gctx_create) || !entry("cuGreenCtxStreamCreate", gstream_create)) {
    snprintf(err, errlen, "the driver has no green-context entry points");
    return -1;
  }
  CUdevice dev;
  CUresult r = device_get(&dev, device);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDeviceGet", r, es);
  CUdevResource full, part, rest;
  r = get_res(dev, &full, CU_DEV_RESOURCE_TYPE_SM);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDeviceGetDevResource", r, es);
  unsigned int n = 1;
  r = split(&part, &n, &full, &rest, 0, (unsigned)first_sms);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDevSmResourceSplitByCount", r, es);
  if (n != 1 || rest.sm.smCount == 0) {
    snprintf(err, errlen, "SM split of %d gave %u group(s), %u SMs left", first_sms, n, rest.sm.smCount);
    return -1;
  }
  // Everything made before a failing step is released again: nothing of a failed call has been handed out yet, so
  // no stream or graph can reference these contexts.
  CUgreenCtx made_ctx[2] = {nullptr, nullptr};
  CUstream made_stream[2] = {nullptr, nullptr};
  auto unwind = [&]() {
    for (int i = 0; i < 2; ++i) {
      if (made_stream[i] && stream_destroy) stream_destroy(made_stream[i]);
      if (made_ctx[i] && gctx_destroy) gctx_destroy(made_ctx[i]);
    }
  };
  CUdevResource* sets[2] = {&part, &rest};
  for (int i = 0; i < 2; ++i) {
    CUdevResourceDesc desc;
    r = gen_desc(&desc, sets[i], 1);
    if (r != CUDA_SUCCESS) {
      unwind();
      return fail(err, errlen, "cuDevResourceGenerateDesc", r, es);
    }
    r = gctx_create(&made_ctx[i], desc, dev, CU_GREEN_CTX_DEFAULT_STREAM);
    if (r != CUDA_SUCCESS) {
      made_ctx[i] = nullptr;
      unwind();
      return fail(err, errlen, "cuGreenCtxCreate", r, es);
    }
    r = gstream_create(&made_stream[i], made_ctx[i], CU_STREAM_NON_BLOCKING, 0);
    if (r != CUDA_SUCCESS) {
      made_stream[i] = nullptr;
      unwind();
      return fail(err, errlen, "cuGreenCtxStreamCreate", r, es);
    }
  }
  for (int i = 0; i < 2; ++i) {
    streams[i] = reinterpret_cast<unsigned long long>(made_stream[i]);
    sms[i] = (int)sets[i]->sm.smCount;
  }
  return 0;
}

}  // namespace iob
