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
int fail(char* err, int errlen, const char* what, CUresult r) {
  const char* s = nullptr;
  cuGetErrorString(r, &s);
  snprintf(err, errlen, "%s: %s", what, s ? s : "unknown driver error");
  return -1;
}
}  // namespace

int sm_lanes_create(int device, int first_sms, unsigned long long* streams, int* sms, char* err, int errlen) {
  if (cudaSetDevice(device) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
    snprintf(err, errlen, "cudaSetDevice(%d) failed", device);
    return -1;
  }
  CUdevice dev;
  CUresult r = cuDeviceGet(&dev, device);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDeviceGet", r);
  CUdevResource full, part, rest;
  r = cuDeviceGetDevResource(dev, &full, CU_DEV_RESOURCE_TYPE_SM);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDeviceGetDevResource", r);
  unsigned int n = 1;
  r = cuDevSmResourceSplitByCount(&part, &n, &full, &rest, 0, (unsigned)first_sms);
  if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDevSmResourceSplitByCount", r);
  if (n != 1 || rest.sm.smCount == 0) {
    snprintf(err, errlen, "SM split of %d gave %u group(s), %u SMs left", first_sms, n, rest.sm.smCount);
    return -1;
  }
  CUdevResource* sets[2] = {&part, &rest};
  for (int i = 0; i < 2; ++i) {
    CUdevResourceDesc desc;
    r = cuDevResourceGenerateDesc(&desc, sets[i], 1);
    if (r != CUDA_SUCCESS) return fail(err, errlen, "cuDevResourceGenerateDesc", r);
    CUgreenCtx g;
    r = cuGreenCtxCreate(&g, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM);
    if (r != CUDA_SUCCESS) return fail(err, errlen, "cuGreenCtxCreate", r);
    CUstream s;
    r = cuGreenCtxStreamCreate(&s, g, CU_STREAM_NON_BLOCKING, 0);
    if (r != CUDA_SUCCESS) return fail(err, errlen, "cuGreenCtxStreamCreate", r);
    streams[i] = reinterpret_cast<unsigned long long>(s);
    sms[i] = (int)sets[i]->sm.smCount;
  }
  return 0;
}

}  // namespace iob
