// Routed experts on the 5th-generation tensor cores: the grouped MXFP4 x MXFP8 GEMM of
// stages/moe.py (gate/up over the expert union's token rows, down over the picks' MXFP8
// activations) as tcgen05.mma.kind::mxf8f6f4.block_scale -- e4m3 activations times e2m1 weights
// with their E8M0 block scales (one per 32 K) applied inside the MMA, fp32 accumulation in TMEM.
//
// Operands: A = the batch's picks' activations (M = 128 rows, of which the first np are real),
// B = 256 rows of the expert's weights (N = 256): one MMA covers 256 weight rows x 32 K in ~135
// cycles, against ~119 cycles for 128 rows with the weights as A (the instruction's floor), so
// the MMA keeps ahead of HBM. A is staged in shared memory as K-major core matrices of only the
// real 8-row groups; the MMA reads all 16 groups, and the rows past np read whatever shared
// memory follows (the activation buffers sit in front of the weight ring, so every such read
// stays inside the CTA's allocation); those accumulator rows are never stored.
//
// Weights (one-time relayout, relayout_mxfp4_kernel): 256-row x 128-K tiles of packed e2m1,
// [E][ceil(N / 256)][K / 128][256 rows][64 B] (even K in the low nibble; rows past N zero), 16 KB
// contiguous a tile -- one TMA request (CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 128-byte swizzle:
// the MMA's unpacked FP4 operand, each 8 bytes of 16 values followed by an 8-byte gap, 32 KB in
// shared memory). Their codes: 1 KB a tile, two 512-byte TMEM scale atoms (rows 0..127, then
// 128..255), row m's code of K block b at (m % 32) * 16 + (m / 32) * 4 + b within its atom; a bulk
// copy brings them and tcgen05.cp.32x128b.warpx4 replicates each atom into the four TMEM
// sub-partitions (weight row n -> lane n % 32, column n / 32, byte = the K block).
//
// CTA (persistent, one an SM): warp 0 issues the copies (one thread), warp 1 allocates TMEM and
// issues the MMAs (one thread), warps 2-5 stage each pick batch's activations and scale atoms.
// A batch's picks sit in accumulator lanes 0..31, which only warps whose index is 0 mod 4 can
// read: warp 4 drains columns 0..127 and warp 8 columns 128..255, side by side, and each frees
// the accumulator once its columns are in registers -- the stores to the partials (one pick row a
// lane, so uncoalesced) come after. Work item = (expert of the
// union, K slice, group of 256-row tiles); a batch = up to 32 of the expert's picks. Pipelines: a
// 4-stage weight ring (full: TMA transaction bytes; empty: MMA commit), two activation buffers
// (ready: the stagers; free: MMA commit), one accumulator (256 columns; full: MMA commit; empty:
// the drainers -- TMEM has no room for a second one beside the scale columns). Every wait is
// bounded; a timeout sets the device error word and unwinds every role.
#pragma once

#include <cuda.h>

#include "attn_tc.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int kMxStages = 4;
constexpr int kMxRows = 256;     // weight rows a tile (N of the MMA)
constexpr int kMxThreads = 288;  // 9 warps: copies, MMA, 4 stagers, 2 idle, the second drainer
constexpr int kMxMaxPicks = 32;
constexpr int kMxKsMax = 1024;   // K slice bound (activation staging bytes a pick)

struct ExpertTcArgs {
  int M, topk, N, K;       // expert matrix rows N (2 I gate/up, H down), K
  int kslices, ks_len;     // K slices (ks_len a multiple of 128, <= kMxKsMax)
  int rtiles;              // ceil(N / 256)
  const uint8_t* ws;       // codes [E][rtiles][K / 128][1024] (two scale atoms)
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
  // activation buffers first: the MMA's reads past a batch's real rows land in what follows
  static constexpr int kABytes = kMxMaxPicks * kMxKsMax;       // [K step][group][8 chunks][8 x 16 B]
  static constexpr int kA = 0;                                 // 2 buffers
  static constexpr int kStage = kMxRows * 128;                 // 32 KB: 256 rows x 128 B, swizzled
  static constexpr int kW = kA + 2 * kABytes;                  // stages (1024-aligned)
  static constexpr int kSfw = kW + kMxStages * kStage;         // stages x 1 KB weight scale atoms
  static constexpr int kSfxBytes = (kMxKsMax / 128) * 512;
  static constexpr int kSfx = kSfw + kMxStages * 1024;         // 2 x [K step][32 lanes][16 B]
  static constexpr int kPicks = kSfx + 2 * kSfxBytes;          // 2 x int [32]
  static constexpr int kBar = kPicks + 2 * kMxMaxPicks * 4;
  // bars: full[S], empty[S], b_ready[2], b_free[2], d_full, d_empty, drain
  static constexpr int kNumBars = 2 * kMxStages + 7;
  static constexpr int kMisc = kBar + kNumBars * 8;            // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16 + 1024;             // + slack to align the base to 1 KB
};

__device__ __forceinline__ uint64_t mx_sdesc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 B apart (leading offset unused)
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::mxf8f6f4 instruction descriptor: A e4m3, B e2m1, K-major both, E8M0 scales, M = 128,
// N = 256; scale-factor ids (the byte of each TMEM scale word) = K block b.
__device__ __forceinline__ uint32_t mx_idesc(int b) {
  return ((uint32_t)b << 4) | (0u << 7) | (5u << 10) | ((uint32_t)(kMxRows >> 3) << 17) | (1u << 23) |
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
// one 256-row x 128-K weight tile (16 KB of global memory)
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
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(v));
  tmem_ld16(taddr + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
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

__device__ __forceinline__ int mx_groups(int np) { return (np + 7) / 8; }  // real 8-row groups of A

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
  const uint32_t d_full = smem_u32(bars + 2 * kMxStages + 4);
  const uint32_t d_empty = smem_u32(bars + 2 * kMxStages + 5);
  const uint32_t drain = smem_u32(bars + 2 * kMxStages + 6);
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
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 2);  // the two drain warps
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
  // TMEM columns: the accumulator 0 .. 255 (lane = pick, column = weight row); activation scales
  // 256 + 32 buffer + 4 K step; weight scales 320 + 8 stage (rows 0..127, then 128..255). Every
  // scale operand starts on a 4-column boundary.
  const uint32_t t_d = tmem, t_sfx = tmem + 256, t_sfw = tmem + 320;
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
          for (int s = 0; s < ksteps; ++s, ++c) {
            const int st = c % kMxStages;
            if (c >= kMxStages && !mbar_wait(empty(st), ((c / kMxStages) - 1) & 1, abort)) {
              ok = false;
              break;
            }
            const int tile = ((w.e * a.rtiles + t) * (a.K / 128)) + w.ks * ksteps + s;
            mx_expect_tx(full(st), 16384 + 1024);
            mx_tma_tile(smem_u32(smem + L::kW + st * L::kStage), &wmap, tile, full(st));
            mx_bulk(smem_u32(smem + L::kSfw + st * 1024), a.ws + (size_t)tile * 1024, 1024, full(st));
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
        const int G = mx_groups(w.np());
        if (!(ok = mbar_wait(b_ready(bb), (bi >> 1) & 1, abort))) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + L::kA + bb * L::kABytes);
        for (int s = 0; s < ksteps; ++s)
          mx_cp_sf(t_sfx + 32 * bb + 4 * s, smem_u32(smem + L::kSfx + bb * L::kSfxBytes + s * 512));
        for (int t = w.tile_lo; ok && t < w.tile_hi; ++t, ++ti) {
          // the accumulator's previous tile has been drained
          if (ti >= 1 && !(ok = mbar_wait(d_empty, (ti - 1) & 1, abort))) break;
          tc_fence_after();
          for (int s = 0; s < ksteps; ++s, ++c) {
            const int st = c % kMxStages;
            if (!(ok = mbar_wait(full(st), (c / kMxStages) & 1, abort))) break;
            tc_fence_after();
            mx_cp_sf(t_sfw + 8 * st, smem_u32(smem + L::kSfw + st * 1024));
            mx_cp_sf(t_sfw + 8 * st + 4, smem_u32(smem + L::kSfw + st * 1024 + 512));
            const uint32_t sw = smem_u32(smem + L::kW + st * L::kStage);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              // A: K step s of the batch's activations, G real 8-row groups 1 KB apart
              const uint64_t da = umma_sdesc(sa + (s * G * 8 + 2 * b) * 128, 128, 1024);
              mx_mma(t_d, da, mx_sdesc_sw128(sw + 32 * b), mx_idesc(b), s > 0 || b > 0,
                     (t_sfx + 32 * bb + 4 * s) | ((uint32_t)b << 30), (t_sfw + 8 * st) | ((uint32_t)b << 30));
            }
            umma_commit(empty(st));
          }
          if (!ok) break;
          umma_commit(d_full);
        }
        umma_commit(b_free(bb));
      }
      // every issued MMA (and scale copy) complete before the TMEM is freed
      umma_commit(drain);
      mbar_wait(drain, 0, abort);
    }
  } else {
    const int P = a.M * a.topk;
    // One drain warp's columns col0 .. col0 + 127 of every tile of the walk's current batch (picks
    // in lanes 0..31, lane = pick slot): into registers, the accumulator released (d_empty counts
    // both drain warps), then the uncoalesced stores of each pick's row of partials. The pick
    // index comes from the routing plan in global memory (the stagers' shared copy may not be
    // written yet when warp 8 starts a batch).
    auto drain = [&](const MxWalk& dw, int& ti, int col0) -> bool {
      const int np = dw.np();
      const bool mine = lane < np;
      float* orow = a.out + ((size_t)dw.ks * P + (mine ? a.picks[dw.p0 + dw.pb + lane] : 0)) * a.N;
      for (int t = dw.tile_lo; t < dw.tile_hi; ++t, ++ti) {
        if (!__all_sync(0xffffffffu, mbar_wait(d_full, ti & 1, abort))) return false;
        tc_fence_after();
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_d + col0 + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty);
        const int row0 = kMxRows * t + col0;
        if (mine) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int r = row0 + 4 * j;
            if (r + 3 < a.N)
              *reinterpret_cast<float4*>(orow + r) = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
          }
        }
      }
      return true;
    };
    if (warp < 6) {
      // ================= activation staging (warps 2-5, 128 threads) and warp 4's half of the drain
      // (the 128 threads decide together -- softmax_all is the AND over named barrier 1 -- so none
      // leaves while the others wait at a barrier)
      const int et = tid - 64;
      auto stage = [&](const MxWalk& sw, int bi) -> bool {
        const int bb = bi & 1;
        if (bi >= 2 && !softmax_all(mbar_wait(b_free(bb), ((bi >> 1) - 1) & 1, abort))) return false;
        const int np = sw.np(), G = mx_groups(np);
        const int k0 = sw.ks * a.ks_len;
        int* pk = s_picks + bb * kMxMaxPicks;
        uint8_t* sa = smem + L::kA + bb * L::kABytes;
        uint8_t* sf = smem + L::kSfx + bb * L::kSfxBytes;
        if (et < kMxMaxPicks) pk[et] = et < np ? a.picks[sw.p0 + sw.pb + et] : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        // A: [K step][group][8 chunks of 16 K][8 rows x 16 B]
        const int kc_n = a.ks_len / 16;
        for (int i = et; i < 8 * G * kc_n; i += 128) {
          const int n = i / kc_n, kc = i % kc_n;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (n < np) {
            const int row = a.x_by_pick ? pk[n] : pk[n] / a.topk;
            v = ldg16(a.x + (size_t)row * a.K + k0 + 16 * kc);
          }
          *reinterpret_cast<uint4*>(sa + ((kc >> 3) * G + (n >> 3)) * 1024 + (kc & 7) * 128 + (n & 7) * 16) = v;
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
        if (warp == 4) ok = drain(w, ti, 0);
        // the batch two ahead reuses this batch's activation and pick buffers (b_free)
        ok = softmax_all(ok);
        if (ok && s_live) {
          ok = stage(sw, si);
          ++si;
          s_live = sw.next(a);
        }
      }
    } else if (warp == 8) {
      // ================= the drain's other half (columns 128..255)
      int ti = 0;
      bool ok = true;
      for (bool live = w.start(a, nu, gridDim.x, blockIdx.x); ok && live; live = w.next(a)) ok = drain(w, ti, 128);
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
