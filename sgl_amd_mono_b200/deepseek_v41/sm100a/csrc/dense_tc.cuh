// Dense FP8 projections with MXFP8 inputs on the 5th-generation tensor cores: y = x W^T for
// wqkv_a, wq_b, wo_b and the shared expert's gate/up and down (attention/gemv.py:141-194,
// stages/gemv.py:182-214), as tcgen05.mma.kind::mxf8f6f4.block_scale -- the tokens' MXFP8
// activations (e4m3 + E8M0 a 32 K) times the weight's e4m3 with its E8M0 code a 128 x 128 block,
// both scales applied inside the MMA, fp32 accumulation in TMEM.
//
// W is read in place (row-major [N, K] e4m3) by TMA: one request = 256 rows x 128 K (32 KB, the
// 128-byte swizzle, rows past N read as zeros), the MMA's B operand (N = 256). A = the M <= 48
// token rows (M = 128 of the MMA; its real 8-row groups staged as K-major core matrices, the rest
// reading the shared memory that follows, as in moe_tc.cuh). A weight block's code is the same
// for its 128 rows and 128 K, so the producer warp writes each stage's two TMEM scale atoms (rows
// 0..127, 128..255) as that code byte repeated; tcgen05.cp.32x128b.warpx4 replicates them.
//
// Work item = (K slice, group of 256-row tiles); CTAs loop over items (persistent, one an SM).
// Roles and pipelines as the routed experts' kernel: warp 0 copies (lane 0 issues, the warp
// writes the scale atoms), warp 1 issues the MMAs, warps 2-5 stage the item's activations. The
// M <= 48 tokens sit in accumulator lanes 0..47, readable by warps 0 and 1 mod 4: warps 4 and 5
// drain columns 0..127 of lanes 0..31 and 32..63, warps 8 and 9 columns 128..255, and each
// releases the accumulator once its columns are in registers, before its (uncoalesced, a token
// row a lane) stores of the partials. Output: fp32 partials out[kslice][m][n], summed over K slices in order by
// the consumer -- the contract of gemv_fp8_kernel, which it replaces for MXFP8 inputs.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "moe_tc.cuh"

namespace dsv41 {

constexpr int kDnStages = 4;
constexpr int kDnThreads = 320;  // 10 warps: copies, MMA, 4 stagers, 2 idle, 2 more drainers
constexpr int kDnMaxRows = 48;
constexpr int kDnKsMax = 512;  // K slice bound
constexpr int kDnGroups = kDnMaxRows / 8;

struct DenseTcArgs {
  int M, N, K;          // y[m][n] = sum_k x[m][k] W[n][k]
  int ks_len, kslices;  // K slices (ks_len a multiple of 128, <= kDnKsMax)
  int rtiles;           // ceil(N / 256)
  int row_groups;       // groups of 256-row tiles an item covers
  const uint8_t* codes; // E8M0 [ceil(N / 128), K / 128]
  const uint8_t* x;     // e4m3 [M, x_ld]
  const uint8_t* xs;    // E8M0 [M, x_ld / 32]
  int x_ld;             // bytes between x rows (a multiple of 16)
  float* out;           // [kslices][M][N]
};

struct DnSmem {
  static constexpr int kABytes = (kDnKsMax / 128) * kDnGroups * 1024;  // [K step][group][8 chunks][8 x 16 B]
  static constexpr int kA = 0;                                         // 2 buffers, in front of the ring
  static constexpr int kStage = 256 * 128;
  static constexpr int kW = 2 * kABytes;                               // stages (1024-aligned)
  static constexpr int kSfw = kW + kDnStages * kStage;                 // stages x 2 atoms x 512
  static constexpr int kSfxBytes = (kDnKsMax / 128) * 512;
  static constexpr int kSfx = kSfw + kDnStages * 1024;                 // 2 x [K step][32 lanes][16 B]
  static constexpr int kBar = kSfx + 2 * kSfxBytes;
  // bars: full[S], empty[S], b_ready[2], b_free[2], d_full, d_empty, drain
  static constexpr int kNumBars = 2 * kDnStages + 7;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16 + 1024;
};

// kind::mxf8f6f4: A e4m3, B e4m3, K-major both, E8M0 scales, M = 128, N = 256, sf ids = K block b.
__device__ __forceinline__ uint32_t dn_idesc(int b) {
  return ((uint32_t)b << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(256 >> 3) << 17) | (1u << 23) |
         ((uint32_t)(128 >> 4) << 24) | ((uint32_t)b << 29);
}
__device__ __forceinline__ void dn_tma_tile(uint32_t dst, const CUtensorMap* map, int k, int row, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(k), "r"(row), "r"(bar)
      : "memory");
}

// The CTA's items in order (every role walks the same sequence).
struct DnWalk {
  int items, grid, item, ks, tile_lo, tile_hi, tiles_per;
  __device__ bool load(const DenseTcArgs& a) {
    for (; item < items; item += grid) {
      const int rg = item / a.kslices;
      ks = item % a.kslices;
      tile_lo = rg * tiles_per;
      tile_hi = min(a.rtiles, tile_lo + tiles_per);
      if (tile_lo < tile_hi) return true;
    }
    return false;
  }
  __device__ bool start(const DenseTcArgs& a, int grid_, int cta) {
    grid = grid_;
    tiles_per = cdiv(a.rtiles, a.row_groups);
    items = a.kslices * a.row_groups;
    item = cta;
    return load(a);
  }
  __device__ bool next(const DenseTcArgs& a) {
    item += grid;
    return load(a);
  }
};

__global__ void __launch_bounds__(kDnThreads, 1)
    dense_tc_kernel(const __grid_constant__ CUtensorMap wmap, const DenseTcArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  using L = DnSmem;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  auto full = [&](int s) { return smem_u32(bars + s); };
  auto empty = [&](int s) { return smem_u32(bars + kDnStages + s); };
  auto b_ready = [&](int i) { return smem_u32(bars + 2 * kDnStages + i); };
  auto b_free = [&](int i) { return smem_u32(bars + 2 * kDnStages + 2 + i); };
  const uint32_t d_full = smem_u32(bars + 2 * kDnStages + 4);
  const uint32_t d_empty = smem_u32(bars + 2 * kDnStages + 5);
  const uint32_t drain = smem_u32(bars + 2 * kDnStages + 6);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  if (tid == 0) {
    for (int s = 0; s < kDnStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(b_ready(i), 1);
      mbar_init(b_free(i), 1);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 4);
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  // TMEM columns: the accumulator 0 .. 255 (lane = token, column = weight row); activation scales
  // 256 + 16 buffer + 4 K step; weight scales 320 + 8 stage (rows 0..127, then 128..255)
  const uint32_t t_d = tmem, t_sfx = tmem + 256, t_sfw = tmem + 320;
  const int ksteps = a.ks_len / 128;
  const int G = (a.M + 7) / 8;
  const int nrb = (a.N + 127) / 128, nkb = a.K / 128;
  DnWalk w;

  if (warp == 0) {
    // ================= copies: weights need nothing from the previous kernel, so they stream
    // before the dependency wait. Lane 0 issues; the warp writes each stage's scale atoms.
    int c = 0;
    bool ok = true;
    for (bool live = w.start(a, gridDim.x, blockIdx.x); ok && live; live = w.next(a))
      for (int t = w.tile_lo; ok && t < w.tile_hi; ++t)
        for (int s = 0; s < ksteps; ++s, ++c) {
          const int st = c % kDnStages;
          bool waited = true;
          if (lane == 0 && c >= kDnStages) waited = mbar_wait(empty(st), ((c / kDnStages) - 1) & 1, abort);
          if (!(ok = __shfl_sync(0xffffffffu, waited, 0))) break;
          const int kb = w.ks * ksteps + s;
          const int rb0 = 2 * t, rb1 = 2 * t + 1;
          const uint32_t c0 = rb0 < nrb ? a.codes[(size_t)rb0 * nkb + kb] : 0u;
          const uint32_t c1 = rb1 < nrb ? a.codes[(size_t)rb1 * nkb + kb] : 0u;
          const uint32_t r0 = c0 * 0x01010101u, r1 = c1 * 0x01010101u;
          uint8_t* atoms = smem + L::kSfw + st * 1024;
          *reinterpret_cast<uint4*>(atoms + 16 * lane) = make_uint4(r0, r0, r0, r0);
          *reinterpret_cast<uint4*>(atoms + 512 + 16 * lane) = make_uint4(r1, r1, r1, r1);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            mx_expect_tx(full(st), 256 * 128);
            dn_tma_tile(smem_u32(smem + L::kW + st * L::kStage), &wmap, kb * 128, 256 * t, full(st));
          }
        }
    // copies still in flight land before the CTA can exit (bounded, also after an abort)
    if (lane == 0)
      for (int k = max(0, c - kDnStages); k < c; ++k)
        for (uint32_t it = 0; it < kTcWaitPolls && !mbar_try(full(k % kDnStages), (k / kDnStages) & 1); ++it) {
        }
  } else if (warp == 1) {
    // ================= MMA issue (one thread)
    if (lane == 0) {
      int c = 0, bi = 0, ti = 0;
      bool ok = true;
      for (bool live = w.start(a, gridDim.x, blockIdx.x); ok && live; live = w.next(a), ++bi) {
        const int bb = bi & 1;
        if (!(ok = mbar_wait(b_ready(bb), (bi >> 1) & 1, abort))) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + L::kA + bb * L::kABytes);
        for (int s = 0; s < ksteps; ++s)
          mx_cp_sf(t_sfx + 16 * bb + 4 * s, smem_u32(smem + L::kSfx + bb * L::kSfxBytes + s * 512));
        for (int t = w.tile_lo; ok && t < w.tile_hi; ++t, ++ti) {
          if (ti >= 1 && !(ok = mbar_wait(d_empty, (ti - 1) & 1, abort))) break;
          tc_fence_after();
          for (int s = 0; s < ksteps; ++s, ++c) {
            const int st = c % kDnStages;
            if (!(ok = mbar_wait(full(st), (c / kDnStages) & 1, abort))) break;
            tc_fence_after();
            mx_cp_sf(t_sfw + 8 * st, smem_u32(smem + L::kSfw + st * 1024));
            mx_cp_sf(t_sfw + 8 * st + 4, smem_u32(smem + L::kSfw + st * 1024 + 512));
            const uint32_t sw = smem_u32(smem + L::kW + st * L::kStage);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint64_t da = umma_sdesc(sa + (s * G * 8 + 2 * b) * 128, 128, 1024);
              mx_mma(t_d, da, mx_sdesc_sw128(sw + 32 * b), dn_idesc(b), s > 0 || b > 0,
                     (t_sfx + 16 * bb + 4 * s) | ((uint32_t)b << 30), (t_sfw + 8 * st) | ((uint32_t)b << 30));
            }
            umma_commit(empty(st));
          }
          if (!ok) break;
          umma_commit(d_full);
        }
        umma_commit(b_free(bb));
      }
      umma_commit(drain);
      mbar_wait(drain, 0, abort);
    }
  } else {
    pdl_wait();
    // One drain warp's columns col0 .. col0 + 127 of its 32 lanes (tokens 32 q + lane) for every
    // tile of the current item: into registers, the accumulator released (d_empty counts the
    // four drain warps), then the stores.
    const int q = warp & 3;
    const int m = 32 * q + lane;  // this thread's token
    auto drain = [&](const DnWalk& dw, int& ti, int col0) -> bool {
      float* orow = a.out + ((size_t)dw.ks * a.M + (m < a.M ? m : 0)) * a.N;
      for (int t = dw.tile_lo; t < dw.tile_hi; ++t, ++ti) {
        if (!__all_sync(0xffffffffu, mbar_wait(d_full, ti & 1, abort))) return false;
        tc_fence_after();
        uint32_t v[128];
        if (32 * q < a.M) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tmem_ld32(t_d + ((uint32_t)(32 * q) << 16) + col0 + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty);
        const int row0 = 256 * t + col0;
        if (m < a.M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int r = row0 + 4 * j;
            if (r + 3 < a.N)
              *reinterpret_cast<float4*>(orow + r) = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (r + e < a.N) orow[r + e] = __uint_as_float(v[4 * j + e]);
            }
          }
        }
      }
      return true;
    };
    if (warp < 6) {
      // ================= activation staging (warps 2-5, 128 threads, deciding together through
      // softmax_all: the AND over named barrier 1); warps 4 and 5 also drain columns 0..127
      const int et = tid - 64;
      auto stage = [&](const DnWalk& sw, int bi) -> bool {
        const int bb = bi & 1;
        if (bi >= 2 && !softmax_all(mbar_wait(b_free(bb), ((bi >> 1) - 1) & 1, abort))) return false;
        const int k0 = sw.ks * a.ks_len;
        uint8_t* sa = smem + L::kA + bb * L::kABytes;
        uint8_t* sf = smem + L::kSfx + bb * L::kSfxBytes;
        const int kc_n = a.ks_len / 16;
        for (int i = et; i < 8 * G * kc_n; i += 128) {
          const int mm = i / kc_n, kc = i % kc_n;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (mm < a.M) v = ldg16(a.x + (size_t)mm * a.x_ld + k0 + 16 * kc);
          *reinterpret_cast<uint4*>(sa + ((kc >> 3) * G + (mm >> 3)) * 1024 + (kc & 7) * 128 + (mm & 7) * 16) = v;
        }
        // scale atoms, one a K step: token m at lane m % 32, word m / 32, bytes = blocks 0..3
        for (int i = et; i < ksteps * 32; i += 128) {
          const int s = i / 32, l = i % 32;
          uint32_t v[4] = {0, 0, 0, 0};
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int mm = l + 32 * j;
            if (mm < a.M) v[j] = *reinterpret_cast<const uint32_t*>(a.xs + (size_t)mm * (a.x_ld / 32) + k0 / 32 + 4 * s);
          }
          *reinterpret_cast<uint4*>(sf + s * 512 + l * 16) = make_uint4(v[0], v[1], v[2], v[3]);
        }
        fence_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (et == 0) mbar_arrive(b_ready(bb));
        return true;
      };
      DnWalk sw = w;
      bool s_live = sw.start(a, gridDim.x, blockIdx.x), ok = true;
      int si = 0;
      for (; ok && s_live && si < 2; ++si, s_live = sw.next(a)) ok = stage(sw, si);
      int ti = 0;
      bool live = ok && w.start(a, gridDim.x, blockIdx.x);
      for (int bi = 0; ok && live; live = w.next(a), ++bi) {
        if (warp >= 4) ok = drain(w, ti, 0);
        // the item two ahead reuses this item's activation buffers (b_free)
        ok = softmax_all(ok);
        if (ok && s_live) {
          ok = stage(sw, si);
          ++si;
          s_live = sw.next(a);
        }
      }
    } else if (warp >= 8) {
      // ================= the drain's other half (columns 128..255)
      int ti = 0;
      bool ok = true;
      for (bool live = w.start(a, gridDim.x, blockIdx.x); ok && live; live = w.next(a)) ok = drain(w, ti, 128);
    }
  }
  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  pdl_launch();
}

}  // namespace dsv41
