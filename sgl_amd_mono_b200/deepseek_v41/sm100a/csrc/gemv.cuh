// Weight-streaming GEMV for decode widths (M <= 48): y[m][n] = sum_k x[m][k] W[n][k].
//
// W is an SGLang-loaded FP8 e4m3 weight read in place, row-major [N, K], with one E8M0 code
// per 128 x 128 block (a power-of-two fp32 block scale, as V4 checkpoints store them).
// x is bf16 [M, K] holding the exactly dequantized MXFP8 (or bf16) activations.
//
// Tensor cores: mma.sync m16n8k16 bf16 -> fp32, weights as the A operand (16 rows), tokens
// as B (8 a tile). A lane streams 16 contiguous bytes of row g and of row g + 8 per 64-K
// step (ld.global.nc, no L1 allocation): a warp reads 8 rows x 64 B, two full sectors a
// row. The 4 bytes a lane holds for mma j become two bf16x2 registers by a shift (values
// times 2^-120, exact) -- the K order inside the mma is therefore a fixed permutation of the
// physical order within each 64-K step; x is staged in shared memory in that same order
// (scaled by 2^64 so no product underflows), and read with ldmatrix. Partial sums of each
// 128-K block are scaled by the block's code times 2^56 into the fp32 accumulator.
//
// Work split (host-chosen, GemvPlan): CTA = (K slice, row group); x's K slice is staged once
// per CTA and reused by every row tile of the group; 8 warps = (8 / wk) tile lanes x wk K
// lanes, K lanes reduced through shared memory in fixed order. Output: fp32 partials
// out[kslice][m][n], summed over K slices in order by the consumer.
#pragma once

#include "common.cuh"

namespace dsv41 {

struct GemvArgs {
  const uint8_t* w;        // e4m3 [N, K], row stride K bytes
  const uint8_t* codes;    // E8M0 [ceil(N / 128), K / 128]
  const __nv_bfloat16* x;  // [M, x_ld]
  float* out;              // [kslices][M][N]
  int M, N, K;
  int x_ld;          // elements between x rows
  int x_group_rows;  // rows n use x columns (n / x_group_rows) * K .. + K (grouped wo_a)
  int kslices;       // K slices (grid.x = kslices * row_groups)
  int ks_blocks;     // 128-K blocks a slice
  int row_groups;
  int tiles_per_group;  // 16-row tiles a row group
  int wk;               // K lanes a tile (1, 2, 4 or 8)
};

// Shared-memory bytes of a launch.
__host__ __device__ inline int gemv_smem_bytes(int M, int ks_blocks) {
  int mpad = (M + 7) / 8 * 8;
  int xs = mpad * (ks_blocks * 128 + 8) * 2;
  int red = 8 * 16 * mpad * 4;
  return xs + red;
}

// Host planning: K slices bounded by shared memory, then enough CTAs and warps in flight.
inline GemvArgs gemv_plan(const uint8_t* w, const uint8_t* codes, const __nv_bfloat16* x,
                          float* out, int M, int N, int K, int x_ld, int x_group_rows,
                          int sms) {
  GemvArgs a;
  a.w = w;
  a.codes = codes;
  a.x = x;
  a.out = out;
  a.M = M;
  a.N = N;
  a.K = K;
  a.x_ld = x_ld;
  a.x_group_rows = x_group_rows > 0 ? x_group_rows : N;
  const int mpad = (M + 7) / 8 * 8;
  const int nb = K / 128;
  const int budget = 100 * 1024 - 8 * 16 * mpad * 4;
  int cap_blocks = (budget / (2 * mpad) - 8) / 128;
  if (cap_blocks < 1) cap_blocks = 1;
  int kslices = cdiv(nb, cap_blocks);
  const int tiles = cdiv(N, 16);
  const int want_warps = sms * 16;  // two 8-warp CTAs an SM
  // K lanes inside a CTA when there are few row tiles
  int wk = 1;
  while (wk < 8 && tiles * wk * kslices < want_warps && nb / kslices >= 2 * wk) wk *= 2;
  // more K slices (shorter K a CTA) while still short of warps and the partials stay small
  while (tiles * wk * kslices < want_warps && nb / (kslices * 2) >= wk &&
         (long)kslices * 2 * M * 4 <= (long)K / 4)
    kslices *= 2;
  a.kslices = kslices;
  a.ks_blocks = cdiv(nb, kslices);
  a.kslices = cdiv(nb, a.ks_blocks);
  a.wk = wk;
  const int lanes = 8 / wk;
  // row groups: tiles a group a multiple of the tile lanes, inside one x group
  const int xg_tiles = a.x_group_rows / 16;
  int want_ctas = cdiv(want_warps, 8);
  int groups = cdiv(want_ctas, a.kslices);
  int tpg = cdiv(tiles, groups);
  tpg = cdiv(tpg, lanes) * lanes;
  if (x_group_rows > 0 && x_group_rows < N) {
    // a divisor of the group's tiles
    if (tpg >= xg_tiles) tpg = xg_tiles;
    while (xg_tiles % tpg != 0) ++tpg;
  }
  a.tiles_per_group = tpg;
  a.row_groups = cdiv(tiles, tpg);
  return a;
}

// Work item blk (K slice, row group) of a planned GEMV, by a CTA of 256 threads with
// gemv_smem_bytes of shared memory. The launch (gemv_fp8_kernel) waits for its inputs after the
// first weight loads (wait = true); the persistent K1 has waited already.
template <int NT>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, int blk, uint8_t* smem, bool wait) {
  constexpr int MP = 8 * NT;
  const int ks = blk % a.kslices;
  const int rg = blk / a.kslices;
  const int nblocks = a.K / 128;
  const int kb0 = ks * a.ks_blocks;
  const int kb1 = min(kb0 + a.ks_blocks, nblocks);
  const int tiles = (a.N + 15) / 16;
  const int tile0 = rg * a.tiles_per_group;
  const int tile1 = min(tile0 + a.tiles_per_group, tiles);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  if (kb0 >= kb1 || tile0 >= tiles) return;
  const int KS = (kb1 - kb0) * 128;
  const int xs_ld = a.ks_blocks * 128 + 8;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);
  float* red = reinterpret_cast<float*>(smem + MP * xs_ld * 2);

  const int wk = a.wk;
  const int lanes = 8 / wk;
  const int wt = warp / wk, wkk = warp - wt * wk;
  const int nb = kb1 - kb0;
  const int kw0 = wkk * nb / wk, kw1 = (wkk + 1) * nb / wk;
  const int nsteps = 2 * (kw1 - kw0);
  const int ntiles_local = cdiv(tile1 - tile0 - wt, lanes);
  constexpr int PF = 4;
  uint4 wa[PF], wb[PF];
  auto tile_ptrs = [&](int it, const uint8_t*& p0, const uint8_t*& p1) {
    const int row0 = (tile0 + wt + it * lanes) * 16;
    const int r0 = min(row0 + g, a.N - 1), r1 = min(row0 + g + 8, a.N - 1);
    p0 = a.w + (size_t)r0 * a.K + (size_t)(kb0 + kw0) * 128 + 16 * t;
    p1 = a.w + (size_t)r1 * a.K + (size_t)(kb0 + kw0) * 128 + 16 * t;
  };
  // the weights wait on nothing: stream the first tile's first steps before the dependency
  // wait, overlapping the previous kernel's tail (programmatic dependent launch)
  if (ntiles_local > 0) {
    const uint8_t *p0, *p1;
    tile_ptrs(0, p0, p1);
#pragma unroll
    for (int i = 0; i < PF; ++i)
      if (i < nsteps) {
        wa[i] = ldg_stream(p0 + 64 * i);
        wb[i] = ldg_stream(p1 + 64 * i);
      }
  }

  if (wait) pdl_wait();
  // ---- stage x's K slice, permuted into mma slot order and scaled by 2^64
  {
    const int xg = (tile0 * 16) / a.x_group_rows;
    const int col0 = xg * a.K + kb0 * 128;
    const int quads = KS / 4;
    auto stage = [&](int i) {
      const int m = i / quads, q = i - m * quads;
      const uint2 v = *reinterpret_cast<const uint2*>(a.x + (size_t)m * a.x_ld + col0 + 4 * q);
      const float s = 18446744073709551616.0f;  // 2^64
      float x0 = __uint_as_float(v.x << 16) * s, x1 = __uint_as_float(v.x & 0xffff0000u) * s;
      float x2 = __uint_as_float(v.y << 16) * s, x3 = __uint_as_float(v.y & 0xffff0000u) * s;
      const int o = 4 * q, c = o >> 6, r = o & 63;
      const int tp = r >> 4, j = (r >> 2) & 3;
      __nv_bfloat16* row = xs + m * xs_ld + c * 64 + 16 * j + 2 * tp;
      *reinterpret_cast<uint32_t*>(row) = pack_bf16x2(x0, x2);
      *reinterpret_cast<uint32_t*>(row + 8) = pack_bf16x2(x1, x3);
    };
    // only the M real rows: the token tile's rows past M feed only the MMA output columns of
    // tokens past M (each output column reads its own B column), which are never stored. (A
    // full tile keeps the compile-time trip count, which the compiler schedules better.)
    if (a.M == MP) {
      for (int i = threadIdx.x; i < MP * quads; i += blockDim.x) stage(i);
    } else {
      for (int i = threadIdx.x; i < a.M * quads; i += blockDim.x) stage(i);
    }
  }
  __syncthreads();

  const uint32_t xs_base = smem_u32(xs);
  // ldmatrix row address of this lane: token (lane & 7) of the n-tile, 8 slots at 8 * (lane >> 3)
  const uint32_t lm_off = ((lane & 7) * xs_ld + 8 * (lane >> 3)) * 2;

  // The next row tile's first PF steps are loaded during this tile's last PF steps (when the
  // steps divide evenly into load slots), so a warp's loads do not drain at tile boundaries. The
  // warp's E8M0 codes of a tile (one a 128-K block, at most 64) are loaded one a lane with the
  // tile's first weights (the next tile's with its first cross-tile loads) and read by shuffles.
  // Token tiles past 2 (M > 16) keep the per-tile loads: their accumulators need the registers.
  constexpr bool kX = NT <= 2;
  const bool xt = kX && nsteps % PF == 0;
  const int ncodes = kX ? kw1 - kw0 : 65;
  auto codes_of = [&](int it, uint32_t& c0, uint32_t& c1) {
    const uint8_t* cp = a.codes + (size_t)(((tile0 + wt + it * lanes) * 16) >> 7) * nblocks + kb0 + kw0;
    c0 = lane < ncodes ? __ldg(cp + lane) : 0u;
    c1 = 32 + lane < ncodes ? __ldg(cp + 32 + lane) : 0u;
  };
  uint32_t cc0 = 0, cc1 = 0, cn0 = 0, cn1 = 0;
  if (ntiles_local > 0 && ncodes <= 64) codes_of(0, cc0, cc1);
  for (int it = 0; it < ntiles_local; ++it) {
    const int tile = tile0 + wt + it * lanes;
    const int row0 = tile * 16;
    const uint8_t *p0, *p1, *q0 = nullptr, *q1 = nullptr;
    tile_ptrs(it, p0, p1);
    const bool pf_next = xt && it + 1 < ntiles_local;
    if (pf_next) tile_ptrs(it + 1, q0, q1);
    const uint8_t* cp = a.codes + (size_t)(row0 >> 7) * nblocks + kb0 + kw0;
    float acc[NT][4];
    float blk[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[n][i] = blk[n][i] = 0.f;

    if (it > 0 && !xt) {
#pragma unroll
      for (int i = 0; i < PF; ++i)
        if (i < nsteps) {
          wa[i] = ldg_stream(p0 + 64 * i);
          wb[i] = ldg_stream(p1 + 64 * i);
        }
    }
    for (int s0 = 0; s0 < nsteps; s0 += PF) {
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const int st = s0 + i;
        if (st < nsteps) {
          const uint4 A = wa[i], B = wb[i];
          if (st + PF < nsteps) {
            wa[i] = ldg_stream(p0 + 64 * (st + PF));
            wb[i] = ldg_stream(p1 + 64 * (st + PF));
          } else if (pf_next) {
            // (st + PF - nsteps) % PF == i: the next tile's step lands in this slot
            wa[i] = ldg_stream(q0 + 64 * (st + PF - nsteps));
            wb[i] = ldg_stream(q1 + 64 * (st + PF - nsteps));
            if (st + PF == nsteps && ncodes <= 64) codes_of(it + 1, cn0, cn1);
          }
          const uint32_t aw[4] = {A.x, A.y, A.z, A.w};
          const uint32_t bw[4] = {B.x, B.y, B.z, B.w};
          const uint32_t col = (uint32_t)((kw0 * 128 + st * 64) * 2);
#pragma unroll
          for (int jp = 0; jp < 2; ++jp) {
            uint32_t a0[2], a1[2], a2[2], a3[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              e4m3x4_bf16(aw[2 * jp + h], a0[h], a2[h]);
              e4m3x4_bf16(bw[2 * jp + h], a1[h], a3[h]);
            }
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              uint32_t b[4];
              ldmatrix_x4(b, xs_base + lm_off + (uint32_t)(n * 8 * xs_ld * 2) + col + jp * 64);
              mma_bf16(blk[n], a0[0], a1[0], a2[0], a3[0], b[0], b[1]);
              mma_bf16(blk[n], a0[1], a1[1], a2[1], a3[1], b[2], b[3]);
            }
          }
          if (st & 1) {
            const int b = st >> 1;
            const uint32_t code = ncodes > 64 ? (uint32_t)__ldg(cp + b)
                                  : __shfl_sync(0xffffffffu, b < 32 ? cc0 : cc1, b & 31);
            const float sc = pow2c((int)code) * 72057594037927936.0f;  // * 2^56
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                acc[n][i] = fmaf(blk[n][i], sc, acc[n][i]);
                blk[n][i] = 0.f;
              }
          }
        }
      }
    }
    if (ncodes <= 64) {
      if (pf_next) {
        cc0 = cn0;
        cc1 = cn1;
      } else if (it + 1 < ntiles_local) {
        codes_of(it + 1, cc0, cc1);
      }
    }
    // ---- K lanes: reduce in lane order through shared memory, then store
    float* out = a.out + (size_t)ks * a.M * a.N;
    if (wk == 1) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = row0 + g + 8 * (i >> 1), m = n * 8 + 2 * t + (i & 1);
          if (row < a.N && m < a.M) out[(size_t)m * a.N + row] = acc[n][i];
        }
    } else {
      float* mine = red + (size_t)warp * 16 * MP;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = g + 8 * (i >> 1), m = n * 8 + 2 * t + (i & 1);
          mine[r * MP + m] = acc[n][i];
        }
      __syncwarp();
      // all K lanes of this tile lane must have written: a named barrier per tile lane
      asm volatile("bar.sync %0, %1;" ::"r"(1 + wt), "r"(wk * 32));
      if (wkk == 0) {
        const float* base = red + (size_t)(wt * wk) * 16 * MP;
        for (int e = lane; e < 16 * MP; e += 32) {
          float v = base[e];
          for (int q = 1; q < wk; ++q) v += base[q * 16 * MP + e];
          const int r = e / MP, m = e - r * MP, row = row0 + r;
          if (row < a.N && m < a.M) out[(size_t)m * a.N + row] = v;
        }
      }
      asm volatile("bar.sync %0, %1;" ::"r"(1 + wt), "r"(wk * 32));
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(256, 2) gemv_fp8_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  gemv_body<NT>(a, blockIdx.x, smem, true);
  pdl_launch();
}

// Launch with the NT (token tiles) the width needs.
inline cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const int nt = (a.M + 7) / 8;
  const int smem = gemv_smem_bytes(a.M, a.ks_blocks);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.kslices * a.row_groups);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define DSV41_GEMV_CASE(NT)                                                                 \
  case NT: {                                                                                \
    auto k = gemv_fp8_kernel<NT>;                                                           \
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(k), smem);                    \
    if (e != cudaSuccess) return e;                                                         \
    return cudaLaunchKernelEx(&cfg, k, a);                                                  \
  }
  switch (nt) {
    DSV41_GEMV_CASE(1)
    DSV41_GEMV_CASE(2)
    DSV41_GEMV_CASE(3)
    DSV41_GEMV_CASE(4)
    DSV41_GEMV_CASE(5)
    DSV41_GEMV_CASE(6)
    default:
      return cudaErrorInvalidValue;
  }
#undef DSV41_GEMV_CASE
}

}  // namespace dsv41
