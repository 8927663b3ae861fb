// The host side shared by the two C-ABI GEMV entries (dsv41_gemv_fp8 with caller scratch, and
// dsv41_gemv_fp8_noalloc with the library's own array): the argument check, the plan, the
// partials' size, and the launch of the GEMV followed by the in-order K-slice sum. Both entries
// call these, so their limits, plans and slice order cannot drift apart.
#pragma once

#include "../../../../include/dsv41_b200.h"
#include "gemv.cuh"

namespace dsv41 {

inline bool gemv_entry_args_ok(const Dsv41GemvArgs* a) {
  return a && a->w && a->codes && a->x && a->y && a->M >= 1 && a->M <= 48 && a->N >= 1 &&
         a->K >= 128 && a->K % 128 == 0 && a->x_ld >= a->K && a->x_ld % 4 == 0 &&
         (a->x_group_rows == 0 || (a->x_group_rows % 16 == 0 && a->N % a->x_group_rows == 0)) &&
         a->w % 16 == 0 && a->x % 8 == 0;
}

inline GemvArgs gemv_entry_plan(const Dsv41GemvArgs* a, int sms) {
  return gemv_plan(reinterpret_cast<const uint8_t*>(a->w), reinterpret_cast<const uint8_t*>(a->codes),
                   reinterpret_cast<const __nv_bfloat16*>(a->x), reinterpret_cast<float*>(a->y), (int)a->M,
                   (int)a->N, (int)a->K, (int)a->x_ld, (int)a->x_group_rows, sms);
}

// Bytes of fp32 K-slice partials the plan writes before its sum (0: one slice, written to y).
inline int64_t gemv_entry_partials_bytes(const GemvArgs& g) {
  return g.kslices > 1 ? (int64_t)g.kslices * g.M * g.N * 4 : 0;
}

namespace {
// y[i] = sum over K slices of p[s][i], in slice order.
__global__ void gemv_entry_sum_kernel(const float* __restrict__ p, float* __restrict__ y, int slices, int total) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    float v = p[i];
    for (int s = 1; s < slices; ++s) v += p[(size_t)s * total + i];
    y[i] = v;
  }
}
}  // namespace

// The GEMV into y, through `partials` (gemv_entry_partials_bytes of them) when K is sliced.
inline cudaError_t gemv_entry_launch(GemvArgs g, float* y, float* partials, cudaStream_t st) {
  if (g.kslices > 1) g.out = partials;
  else g.out = y;
  cudaError_t e = gemv_launch(g, st, false);
  if (e != cudaSuccess || g.kslices == 1) return e;
  const int total = g.M * g.N;
  const int grid = std::min((total + 255) / 256, 4096);
  gemv_entry_sum_kernel<<<grid, 256, 0, st>>>(partials, y, g.kslices, total);
  return cudaGetLastError();
}

}  // namespace dsv41
