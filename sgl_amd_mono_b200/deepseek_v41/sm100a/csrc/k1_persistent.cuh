// K1 as one persistent launch, for the rows whose projections run on the CUDA-core GEMV (M below
// the tcgen05 dense kernel's threshold): the reference's K1 (gfx950/layer.py:189-468) is one
// launch a layer, and at small M the layer's time goes to the fixed cost of each dependent
// launch rather than to bytes.
//
// A grid of CTAs that are all resident (the launch sizes it from the occupancy: two an SM) runs
// K1's stages in order, each as a loop over that stage's work items (the launch sequence's
// blocks, by the same device functions, so both paths give the same bits), with a grid-wide
// barrier between dependent stages:
//   1  the seam's 32-column slices, and K2's key table (independent of the rest)
//   2  the seam's gates and norm, a row an item
//   3  the wqkv_a GEMV (K slice x row group items)
//   4  q_norm -> MXFP8 q, kv_norm + RoPE -> the FP8 KV record, a row an item
//   5  the wq_b GEMV
//   6  wq_b's epilogue: bf16 + RoPE -> q
// Before its inputs are ready (programmatic dependent launch), every CTA asks L2 to prefetch its
// share of both GEMVs' weights, so they stream while the latency-bound seam stages run.
// The barrier is one word, zeroed by the host before the launch, by sense reversal (CTA 0 adds
// 2^31 - (n - 1), the others 1: the top bit flips when the last CTA arrives, and the low bits
// return to their start); its wait is bounded (2 s of %globaltimer), after which it raises the
// device error word (dsv41_device_error) and lets the CTA continue, so a stuck launch ends.
#pragma once

#include "attn_tc.cuh"
#include "front.cuh"
#include "gemv.cuh"
#include "seam.cuh"

namespace dsv41 {

struct K1PArgs {
  SeamArgs s;
  KeyTableArgs k;
  int kt_rows, kt_y;    // key-table items: rows x blocks a row (0 rows: no table)
  GemvArgs g1;          // wqkv_a
  FrontArgs f;
  GemvArgs g2;          // wq_b
  QRopeArgs qr;
  int qr_x;             // q_rope blocks a row
  unsigned* bar;        // the barrier word (zero at launch)
  const uint8_t* pf[2]; // weights to prefetch into L2 (null: none), and their bytes
  int64_t pf_bytes[2];
};

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ inline void k1p_grid_sync(unsigned* bar) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned nb = gridDim.x;
    const unsigned add = blockIdx.x == 0 ? 0x80000000u - (nb - 1) : 1u;
    __threadfence();
    const unsigned old = atomicAdd(bar, add);
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
      if (((old ^ ld_acquire_gpu_u32(bar)) & 0x80000000u) != 0) break;
      if ((it & 255) != 0) continue;
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > 2000000000ull) {
        atomicExch(&g_tc_error, 2);
        break;
      }
    }
    __threadfence();
  }
  __syncthreads();
}

template <int NT>
__global__ void __launch_bounds__(256, 2) k1_persistent_kernel(const K1PArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = gridDim.x;
  // this CTA's share of both GEMVs' weights into L2: they wait on nothing
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (!a.pf[i]) continue;
      const int64_t share = ((a.pf_bytes[i] + nb - 1) / nb + 15) / 16 * 16;
      const int64_t b0 = share * blockIdx.x;
      const int64_t n = min(share, a.pf_bytes[i] - b0);
      for (int64_t o = 0; o < n; o += (1 << 20)) {
        const uint32_t sz = (uint32_t)min((int64_t)(1 << 20), n - o);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf[i] + b0 + o), "r"(sz) : "memory");
      }
    }
  }
  pdl_wait();
  // 1: seam slices, then the key table
  const int slices = a.s.H / kSliceCols;
  for (int vb = blockIdx.x; vb < slices + a.kt_rows * a.kt_y; vb += nb) {
    if (vb < slices) {
      seam_slice_body(a.s, vb, reinterpret_cast<float*>(smem), false);
    } else {
      const int r = vb - slices;
      key_table_body(a.k, r / a.kt_y, r % a.kt_y, a.kt_y);
    }
    __syncthreads();
  }
  k1p_grid_sync(a.bar);
  // 2: gates and norm
  for (int vb = blockIdx.x; vb < a.s.M; vb += nb) {
    seam_gate_norm_body(a.s, vb);
    __syncthreads();
  }
  k1p_grid_sync(a.bar);
  // 3: wqkv_a
  for (int vb = blockIdx.x; vb < a.g1.kslices * a.g1.row_groups; vb += nb) {
    gemv_body<NT>(a.g1, vb, smem, false);
    __syncthreads();
  }
  k1p_grid_sync(a.bar);
  // 4: q and kv
  for (int vb = blockIdx.x; vb < a.f.M; vb += nb) {
    front_qkv_body(a.f, vb);
    __syncthreads();
  }
  k1p_grid_sync(a.bar);
  // 5: wq_b
  for (int vb = blockIdx.x; vb < a.g2.kslices * a.g2.row_groups; vb += nb) {
    gemv_body<NT>(a.g2, vb, smem, false);
    __syncthreads();
  }
  k1p_grid_sync(a.bar);
  // 6: q = bf16 + RoPE
  for (int vb = blockIdx.x; vb < a.qr_x * a.qr.M; vb += nb) q_rope_body(a.qr, vb % a.qr_x, a.qr_x, vb / a.qr_x);
  pdl_launch();
}

}  // namespace dsv41
