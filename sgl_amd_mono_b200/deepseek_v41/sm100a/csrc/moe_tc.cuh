// Routed experts on the 5th-generation tensor cores: the grouped MXFP4 x MXFP8 GEMM of
// stages/moe.py (gate/up over the expert union's token rows, down over the picks' MXFP8
// activations) as tcgen05.mma.kind::mxf8f6f4.block_scale -- e2m1 weights times e4m3
// activations with their E8M0 block scales (one per 32 K) applied inside the MMA, fp32
// accumulation in TMEM.
//
// Weights (one-time relayout, relayout_mxfp4_kernel): 128-row x 128-K tiles of packed e2m1,
// [E][ceil(N / 128)][K / 128][128 rows][64 B] (even K in the low nibble; rows past N zero),
// each tile 8 KB contiguous; their codes in the TMEM scale-atom order, [E][rtiles][K / 128]
// [512 B] with row m's code of K block b at (m % 32) * 16 + (m / 32) * 4 + b. A TMA tensor
// copy (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 128-byte swizzle) lands a tile in shared memory
// as the MMA's unpacked FP4 operand (each 8 bytes of 16 values followed by an 8-byte gap),
// K-major with the 128-byte swizzle; a bulk copy brings the 512 code bytes, and
// tcgen05.cp.32x128b.warpx4 replicates them into the four TMEM sub-partitions.
//
// CTA (persistent): warp 0 issues the copies (one thread), warp 1 allocates TMEM and issues
// the MMAs (one thread), warps 2-5 stage each pick batch's activations (e4m3, K-major core
// matrices) and scale codes, and drain the accumulators. Work item = (expert of the union,
// K slice, group of row tiles); a batch = up to 32 of the expert's picks; N of the MMA = the
// batch's picks rounded up to 8, 16 or 32. Pipelines: a 4-stage weight ring of two K steps a
// stage (one 16 KB TMA request: 8 KB requests stream at ~4.1 TB/s over 148 SMs, 16 KB ones at
// ~6.1; full: TMA transaction bytes; empty: MMA commit), two activation buffers (ready: the stagers; free:
// MMA commit), two accumulators (full: MMA commit; empty: the drainers). Every wait is
// bounded; a timeout sets the device error word and unwinds every role.
#pragma once

#include <cuda.h>

#include "attn_tc.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int kMxStages = 4;
constexpr int kMxDepth = 2;    // K steps (128-K tiles) a stage: one 16 KB TMA request
constexpr int kMxThreads = 192;
constexpr int kMxMaxPicks = 32;
constexpr int kMxKsMax = 1024;  // K slice bound (activation staging bytes a pick)

struct ExpertTcArgs {
  int M, topk, N, K;       // expert matrix rows N (2 I gate/up, H down), K
  int kslices, ks_len;     // K slices (ks_len a multiple of 128, <= kMxKsMax)
  int rtiles;              // ceil(N / 128)
  const uint8_t* ws;       // codes [E][rtiles][K / 128][512] (scale-atom order)
  const uint8_t* x;        // e4m3 [rows, K]: token rows (gate/up) or pick rows (down)
  const uint8_t* xs;       // codes [rows, K / 32]
  int x_by_pick;           // 1: x rows are pick indices; 0: token rows (pick / topk)
  const int32_t* n_u;
  const int32_t* u_expert;
  const int32_t* u_off;
  const int32_t* picks;
  float* out;              // [kslices][M topk][N] fp32 partials, by natural pick index
};

struct MxSmem {
  static constexpr int kStage = kMxDepth * 16384;
  static constexpr int kA = 0;                                 // stages x depth x 16 KB (1024-aligned)
  static constexpr int kSfa = kMxStages * kStage;              // stages x depth x 512
  static constexpr int kB = kSfa + kMxStages * kMxDepth * 512; // 2 x [32 picks][kMxKsMax]
  static constexpr int kBBytes = kMxMaxPicks * kMxKsMax;
  static constexpr int kSfb = kB + 2 * kBBytes;                // 2 x [K step][32 lanes][16 B]
  static constexpr int kSfbBytes = (kMxKsMax / 128) * 512;
  static constexpr int kPicks = kSfb + 2 * kSfbBytes;          // 2 x int [32]
  static constexpr int kBar = kPicks + 2 * kMxMaxPicks * 4;
  // bars: full[S], empty[S], b_ready[2], b_free[2], d_full[2], d_empty[2], drain
  static constexpr int kNumBars = 2 * kMxStages + 9;
  static constexpr int kMisc = kBar + kNumBars * 8;            // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16 + 1024;             // + slack to align the base to 1 KB
};

__device__ __forceinline__ uint64_t mx_sdesc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 B apart (leading offset unused)
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::mxf8f6f4 instruction descriptor: A e2m1, B e4m3, K-major both, E8M0 scales, M = 128,
// scale-factor ids (the byte of each TMEM scale word) = K block b.
__device__ __forceinline__ uint32_t mx_idesc(int N, int b) {
  return ((uint32_t)b << 4) | (5u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(128 >> 4) << 24) | ((uint32_t)b << 29);
}
__device__ __forceinline__ void mx_mma(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc,
                                       uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}
// 32 lanes x 16 B of shared memory (core matrices of 8 rows, 128 B apart) -> 4 TMEM columns of
// every sub-partition
__device__ __forceinline__ void mx_cp_sf(uint32_t tmem_col, uint32_t saddr) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_col), "l"(umma_sdesc(saddr, 128, 128)));
}
__device__ __forceinline__ void mx_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// kMxDepth consecutive tiles (K steps) from `tile` on; tiles past the map read as zeros
__device__ __forceinline__ void mx_tma_tile(uint32_t dst, const CUtensorMap* map, int tile, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(map), "r"(0), "r"(0), "r"(tile), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mx_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// The CTA's work in order: items (expert unit, K slice, row-tile group), each in pick batches;
// every role walks the same sequence.
struct MxWalk {
  int items, RG, tiles_per, grid, item;
  int u, ks, tile_lo, tile_hi, e, p0, np_all, pb;
  __device__ bool load(const ExpertTcArgs& a) {
    for (; item < items; item += grid) {
      const int rg = item % RG, pair = item / RG;
      ks = pair % a.kslices;
      u = pair / a.kslices;
      tile_lo = rg * tiles_per;
      tile_hi = min(a.rtiles, tile_lo + tiles_per);
      if (tile_lo >= tile_hi) continue;
      e = a.u_expert[u];
      p0 = a.u_off[u];
      np_all = a.u_off[u + 1] - p0;
      pb = 0;
      if (np_all > 0) return true;
    }
    return false;
  }
  __device__ bool start(const ExpertTcArgs& a, int nu, int grid_, int cta) {
    grid = grid_;
    const int pairs = nu * a.kslices;
    RG = max(1, min(cdiv(8 * grid, max(pairs, 1)), a.rtiles));
    tiles_per = cdiv(a.rtiles, RG);
    items = pairs * RG;
    item = cta;
    return load(a);
  }
  __device__ bool next(const ExpertTcArgs& a) {  // the next batch
    pb += kMxMaxPicks;
    if (pb < np_all) return true;
    item += grid;
    return load(a);
  }
  __device__ int np() const { return min(kMxMaxPicks, np_all - pb); }
};

__device__ __forceinline__ int mx_ncols(int np) { return np <= 8 ? 8 : np <= 16 ? 16 : 32; }

__global__ void __launch_bounds__(kMxThreads, 1)
    expert_tc_kernel(const __grid_constant__ CUtensorMap wmap, const ExpertTcArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  using L = MxSmem;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  auto full = [&](int s) { return smem_u32(bars + s); };
  auto empty = [&](int s) { return smem_u32(bars + kMxStages + s); };
  auto b_ready = [&](int i) { return smem_u32(bars + 2 * kMxStages + i); };
  auto b_free = [&](int i) { return smem_u32(bars + 2 * kMxStages + 2 + i); };
  auto d_full = [&](int i) { return smem_u32(bars + 2 * kMxStages + 4 + i); };
  auto d_empty = [&](int i) { return smem_u32(bars + 2 * kMxStages + 6 + i); };
  const uint32_t drain = smem_u32(bars + 2 * kMxStages + 8);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  int* s_picks = reinterpret_cast<int*>(smem + L::kPicks);

  if (tid == 0) {
    for (int s = 0; s < kMxStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(b_ready(i), 1);
      mbar_init(b_free(i), 1);
      mbar_init(d_full(i), 1);
      mbar_init(d_empty(i), 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  // TMEM columns: accumulators 0, 32 (up to 32 picks); weight scales 64 + 4 (stage, K step); activation
  // scales 128 + 32 buffer + 4 K step (a scale operand starts on a 4-column boundary: the
  // 32-lane x 4-column atom of tcgen05.cp.32x128b)
  const uint32_t t_d = tmem, t_sfa = tmem + 64, t_sfb = tmem + 128;
  const int ksteps = a.ks_len / 128;

  pdl_wait();
  const int nu = *a.n_u;
  MxWalk w;

  if (warp == 0) {
    // ================= copies (one thread)
    if (lane == 0) {
      int c = 0;
      for (bool live = w.start(a, nu, gridDim.x, blockIdx.x); live; live = w.next(a)) {
        bool ok = true;
        for (int t = w.tile_lo; ok && t < w.tile_hi; ++t)
          for (int s = 0; s < ksteps; s += kMxDepth, ++c) {
            const int st = c % kMxStages;
            if (c >= kMxStages && !mbar_wait(empty(st), ((c / kMxStages) - 1) & 1, abort)) {
              ok = false;
              break;
            }
            const int nk = min(kMxDepth, ksteps - s);  // K steps of this slice in the stage
            const int tile = ((w.e * a.rtiles + t) * (a.K / 128)) + w.ks * ksteps + s;
            mx_expect_tx(full(st), kMxDepth * 8192 + nk * 512);
            mx_tma_tile(smem_u32(smem + L::kA + st * L::kStage), &wmap, tile, full(st));
            mx_bulk(smem_u32(smem + L::kSfa + st * kMxDepth * 512), a.ws + (size_t)tile * 512, nk * 512, full(st));
          }
        if (!ok) break;
      }
      // copies still in flight land before the CTA can exit (bounded, also after an abort)
      for (int k = max(0, c - kMxStages); k < c; ++k)
        for (uint32_t it = 0; it < kTcWaitPolls && !mbar_try(full(k % kMxStages), (k / kMxStages) & 1); ++it) {
        }
    }
  } else if (warp == 1) {
    // ================= MMA issue (one thread)
    if (lane == 0) {
      int c = 0, bi = 0, ti = 0;
      bool ok = true;
      for (bool live = w.start(a, nu, gridDim.x, blockIdx.x); ok && live; live = w.next(a), ++bi) {
        const int bb = bi & 1;
        const int N = mx_ncols(w.np());
        if (!(ok = mbar_wait(b_ready(bb), (bi >> 1) & 1, abort))) break;
        tc_fence_after();
        const uint32_t sb = smem_u32(smem + L::kB + bb * L::kBBytes);
        for (int s = 0; s < ksteps; ++s)
          mx_cp_sf(t_sfb + 32 * bb + 4 * s, smem_u32(smem + L::kSfb + bb * L::kSfbBytes + s * 512));
        for (int t = w.tile_lo; ok && t < w.tile_hi; ++t, ++ti) {
          const int dd = ti & 1;
          if (ti >= 2 && !(ok = mbar_wait(d_empty(dd), ((ti >> 1) - 1) & 1, abort))) break;
          tc_fence_after();
          for (int s0 = 0; s0 < ksteps; s0 += kMxDepth, ++c) {
            const int st = c % kMxStages;
            if (!(ok = mbar_wait(full(st), (c / kMxStages) & 1, abort))) break;
            tc_fence_after();
            const int nk = min(kMxDepth, ksteps - s0);
            for (int j = 0; j < nk; ++j) {
              const int s = s0 + j, slot = st * kMxDepth + j;
              mx_cp_sf(t_sfa + 4 * slot, smem_u32(smem + L::kSfa + slot * 512));
              const uint32_t sa = smem_u32(smem + L::kA + st * L::kStage + j * 16384);
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const uint64_t db = umma_sdesc(sb + (8 * s + 2 * b) * 128, 128, (a.ks_len / 16) * 128);
                mx_mma(t_d + 32 * dd, mx_sdesc_sw128(sa + 32 * b), db, mx_idesc(N, b), s > 0 || b > 0,
                       (t_sfa + 4 * slot) | ((uint32_t)b << 30), (t_sfb + 32 * bb + 4 * s) | ((uint32_t)b << 30));
              }
            }
            umma_commit(empty(st));
          }
          if (!ok) break;
          umma_commit(d_full(dd));
        }
        umma_commit(b_free(bb));
      }
      // every issued MMA (and scale copy) complete before the TMEM is freed
      umma_commit(drain);
      mbar_wait(drain, 0, abort);
    }
  } else {
    // ================= activation staging + accumulator drain (warps 2-5, 128 threads)
    const int et = tid - 64;
    const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
    const int P = a.M * a.topk;
    // (the 128 threads decide together -- softmax_all is the AND over named barrier 1 -- so none
    // leaves while the others wait at a barrier)
    auto stage = [&](const MxWalk& sw, int bi) -> bool {
      const int bb = bi & 1;
      if (bi >= 2 && !softmax_all(mbar_wait(b_free(bb), ((bi >> 1) - 1) & 1, abort))) return false;
      const int np = sw.np(), N = mx_ncols(np);
      const int k0 = sw.ks * a.ks_len;
      int* pk = s_picks + bb * kMxMaxPicks;
      uint8_t* sb = smem + L::kB + bb * L::kBBytes;
      uint8_t* sf = smem + L::kSfb + bb * L::kSfbBytes;
      if (et < kMxMaxPicks) pk[et] = et < np ? a.picks[sw.p0 + sw.pb + et] : 0;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int kc_n = a.ks_len / 16;
      for (int i = et; i < N * kc_n; i += 128) {
        const int n = i / kc_n, kc = i % kc_n;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < np) {
          const int row = a.x_by_pick ? pk[n] : pk[n] / a.topk;
          v = ldg16(a.x + (size_t)row * a.K + k0 + 16 * kc);
        }
        *reinterpret_cast<uint4*>(sb + ((n >> 3) * kc_n + kc) * 128 + (n & 7) * 16) = v;
      }
      // scale atoms, one a K step: [lane n][16 B], bytes 0..3 = the codes of blocks 0..3
      for (int i = et; i < ksteps * 32; i += 128) {
        const int s = i / 32, n = i % 32;
        uint32_t v = 0;
        if (n < np) {
          const int row = a.x_by_pick ? pk[n] : pk[n] / a.topk;
          v = *reinterpret_cast<const uint32_t*>(a.xs + (size_t)row * (a.K / 32) + k0 / 32 + 4 * s);
        }
        *reinterpret_cast<uint4*>(sf + s * 512 + n * 16) = make_uint4(v, 0, 0, 0);
      }
      fence_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) mbar_arrive(b_ready(bb));
      return true;
    };
    MxWalk sw = w;  // the staging walk runs up to two batches ahead of the drain walk
    bool s_live = sw.start(a, nu, gridDim.x, blockIdx.x), ok = true;
    int si = 0;
    for (; ok && s_live && si < 2; ++si, s_live = sw.next(a)) ok = stage(sw, si);
    int ti = 0;
    bool live = ok && w.start(a, nu, gridDim.x, blockIdx.x);
    for (int bi = 0; ok && live; live = w.next(a), ++bi) {
      const int np = w.np(), N = mx_ncols(np);
      const int* pk = s_picks + (bi & 1) * kMxMaxPicks;
      float* out = a.out + (size_t)w.ks * P * a.N;
      for (int t = w.tile_lo; t < w.tile_hi; ++t, ++ti) {
        const int dd = ti & 1;
        if (!(ok = softmax_all(mbar_wait(d_full(dd), (ti >> 1) & 1, abort)))) break;
        tc_fence_after();
        uint32_t v[32];
        const uint32_t src = t_d + 32 * dd + lane_addr;
        tmem_ld16(src, *reinterpret_cast<uint32_t(*)[16]>(v));
        if (N > 16) tmem_ld16(src + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(dd));
        const int row = 128 * t + 32 * (warp & 3) + lane;
        if (row < a.N) {
#pragma unroll
          for (int n = 0; n < 32; ++n)
            if (n < np) out[(size_t)pk[n] * a.N + row] = __uint_as_float(v[n]);
        }
      }
      // the batch two ahead reuses this batch's buffers (its MMAs are done: its last
      // accumulator was drained)
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (ok && s_live) {
        ok = stage(sw, si);
        ++si;
        s_live = sw.next(a);
      }
    }
  }
  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
  pdl_launch();
}

}  // namespace dsv41
