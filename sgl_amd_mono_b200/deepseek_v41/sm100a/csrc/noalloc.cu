// dsv41_gemv_fp8_noalloc: the FP8 weight-streaming GEMV for callers that cannot allocate
// device memory -- e.g. a serving process that handed all spare HBM to its KV-cache pool at
// start-up, or a foreign runtime binding the C ABI without a device allocator of its own.
// The GEMV's K-slice partials (its only scratch) live in a library-owned device array below
// instead of caller scratch; inputs and outputs are still the caller's. The argument check,
// plan and slice-ordered sum are dsv41_gemv_fp8's own (gemv_entry.cuh), so both entries give
// the same bits.
#include <cuda.h>

#include <cstdio>
#include <mutex>
#include <utility>
#include <vector>

#include "../../../../include/dsv41_b200.h"
#include "gemv_entry.cuh"

using namespace dsv41;

namespace {

// The partials array. Every GPU that loads the library holds these bytes until the process
// exits; all calls share them, so calls whose work overlaps on the GPU (another stream, or
// another host thread's stream) race on the contents. Nothing in it needs clearing: each call
// writes every partial it later sums.
__device__ __align__(256) uint8_t g_noalloc_scratch[DSV41_NOALLOC_SCRATCH_BYTES];

struct Resolved {
  unsigned long long ctx_id;  // cuCtxGetId of the context the address belongs to
  void* addr;
  int sms;
};
std::mutex g_mu;
std::vector<Resolved> g_resolved;

// The two driver calls, through the runtime's driver entry point (the library does not link
// libcuda, so it loads on a machine without a driver).
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
template <class Fn>
Fn driver_fn(const char* name) {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(f);
}

// Set-up on first use in each CUDA context, with that context current: the array's device
// address there. The module (and so the array) has its own address in every context -- the
// primary context of each device, a driver-API caller's own context, the new primary context
// after a cudaDeviceReset -- so the cache is keyed by the context's unique id, which is never
// reused within the process. In host code the array's name is only a host-side stand-in,
// never a device pointer.
cudaError_t device_scratch(void** addr, int* sms) {
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (!get_current || !get_id) return cudaErrorDeviceUninitialized;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
  cudaError_t e = cudaSuccess;
  if (!ctx) {
    // no context bound to this thread yet: bind the current device's primary context, as the
    // runtime would at its first call
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess) return e;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return cudaErrorDeviceUninitialized;
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
  std::lock_guard<std::mutex> lock(g_mu);
  for (const Resolved& r : g_resolved)
    if (r.ctx_id == id) {
      *addr = r.addr;
      *sms = r.sms;
      return cudaSuccess;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  int dev = 0, n = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  g_resolved.push_back({id, p, n});
  *addr = p;
  *sms = n;
  return cudaSuccess;
}

}  // namespace

extern "C" int dsv41_gemv_fp8_noalloc(const Dsv41GemvArgs* a, void* stream) {
  if (!gemv_entry_args_ok(a)) return DSV41_EINVAL;
  void* scratch = nullptr;
  int sms = 0;
  cudaError_t e = device_scratch(&scratch, &sms);
  if (e != cudaSuccess) {
    fprintf(stderr, "dsv41_gemv_fp8_noalloc: device set-up failed: %s\n", cudaGetErrorString(e));
    return DSV41_ELAUNCH;
  }
  const GemvArgs g = gemv_entry_plan(a, sms);
  const int64_t need = gemv_entry_partials_bytes(g);
  if (need > DSV41_NOALLOC_SCRATCH_BYTES) {
    fprintf(stderr,
            "dsv41_gemv_fp8_noalloc: M=%lld N=%lld K=%lld needs %lld bytes of partials, over the "
            "%d-byte library array; use dsv41_gemv_fp8 with caller scratch\n",
            (long long)a->M, (long long)a->N, (long long)a->K, (long long)need, DSV41_NOALLOC_SCRATCH_BYTES);
    return DSV41_ESCRATCH;
  }
  e = gemv_entry_launch(g, reinterpret_cast<float*>(a->y), reinterpret_cast<float*>(scratch),
                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    fprintf(stderr, "dsv41_gemv_fp8_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return DSV41_ELAUNCH;
  }
  return DSV41_OK;
}
