// dsv41_gemv_fp8_noalloc: the FP8 weight-streaming GEMV for callers that cannot allocate
// device memory -- e.g. a serving process that handed all spare HBM to its KV-cache pool at
// start-up, or a foreign runtime binding the C ABI without a device allocator of its own.
// The GEMV's K-slice partials (its only scratch) live in a library-owned device array below
// instead of caller scratch; inputs and outputs are still the caller's.
#include <cstdio>
#include <mutex>

#include "../../../../include/dsv41_b200.h"
#include "gemv.cuh"

using namespace dsv41;

namespace {

// The partials array. Every GPU that loads the library holds these bytes until the process
// exits; all calls share them, so calls whose work overlaps on the GPU (another stream, or
// another host thread's stream) race on the contents. Nothing in it needs clearing: each call
// writes every partial it later sums.
__device__ __align__(256) uint8_t g_noalloc_scratch[DSV41_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

// Set-up on first use per device, with that device current: the array's device address.
// In host code the array's name is only a host-side stand-in, never a device pointer.
cudaError_t device_scratch(void** addr, int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    g_sms[dev] = n;
    g_addr[dev] = p;
  }
  *addr = g_addr[dev];
  *sms = g_sms[dev];
  return cudaSuccess;
}

__global__ void noalloc_sum_kernel(const float* __restrict__ p, float* __restrict__ y, int slices,
                                   int total) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    float v = p[i];
    for (int s = 1; s < slices; ++s) v += p[(size_t)s * total + i];
    y[i] = v;
  }
}

}  // namespace

extern "C" int dsv41_gemv_fp8_noalloc(const Dsv41GemvArgs* a, void* stream) {
  if (!a || !a->w || !a->codes || !a->x || !a->y || a->M < 1 || a->M > 48 || a->N < 1 ||
      a->K < 128 || a->K % 128 || a->x_ld < a->K || a->x_ld % 4 || a->w % 16 || a->x % 8 ||
      (a->x_group_rows && (a->x_group_rows % 16 || a->N % a->x_group_rows)))
    return DSV41_EINVAL;
  void* scratch = nullptr;
  int sms = 0;
  cudaError_t e = device_scratch(&scratch, &sms);
  if (e != cudaSuccess) {
    fprintf(stderr, "dsv41_gemv_fp8_noalloc: device set-up failed: %s\n", cudaGetErrorString(e));
    return DSV41_ELAUNCH;
  }
  GemvArgs g = gemv_plan(reinterpret_cast<const uint8_t*>(a->w), reinterpret_cast<const uint8_t*>(a->codes),
                         reinterpret_cast<const __nv_bfloat16*>(a->x), reinterpret_cast<float*>(a->y),
                         (int)a->M, (int)a->N, (int)a->K, (int)a->x_ld, (int)a->x_group_rows, sms);
  if (g.kslices > 1) {
    const int64_t need = (int64_t)g.kslices * a->M * a->N * 4;
    if (need > DSV41_NOALLOC_SCRATCH_BYTES) {
      fprintf(stderr,
              "dsv41_gemv_fp8_noalloc: M=%lld N=%lld K=%lld needs %lld bytes of partials, over the "
              "%d-byte library array; use dsv41_gemv_fp8 with caller scratch\n",
              (long long)a->M, (long long)a->N, (long long)a->K, (long long)need,
              DSV41_NOALLOC_SCRATCH_BYTES);
      return DSV41_ESCRATCH;
    }
    g.out = reinterpret_cast<float*>(scratch);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (gemv_launch(g, st, false) != cudaSuccess) {
    fprintf(stderr, "dsv41_gemv_fp8_noalloc: launch failed: %s\n", cudaGetErrorString(cudaGetLastError()));
    return DSV41_ELAUNCH;
  }
  if (g.kslices > 1) {
    const int total = (int)(a->M * a->N);
    int grid = (total + 255) / 256;
    if (grid > 4096) grid = 4096;
    noalloc_sum_kernel<<<grid, 256, 0, st>>>(g.out, reinterpret_cast<float*>(a->y), g.kslices, total);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "dsv41_gemv_fp8_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return DSV41_ELAUNCH;
  }
  return DSV41_OK;
}
