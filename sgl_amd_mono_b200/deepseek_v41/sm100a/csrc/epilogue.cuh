// GEMV epilogues that need no stage-specific math: K-slice sums rounded to bf16, optionally
// requantized to vLLM-rule MXFP8; the rank-order all-reduce sum; the MXFP4 fragment relayout.
#pragma once

#include "common.cuh"

namespace dsv41 {

struct FinalizeArgs {
  int M, N, kslices;
  const float* part;      // [kslices][M][N]
  __nv_bfloat16* out;     // [M, N] bf16(sum) (or the dequantized MXFP8 when q8 is set)
  uint8_t* q8;            // optional [M, N] e4m3 (vLLM rule)
  uint8_t* q8s;           // [M, N / 32]
};

// A thread = 8 consecutive columns (4 threads a 32-group when requantizing).
__global__ void finalize_kernel(const FinalizeArgs a) {
  pdl_wait();
  const int g8 = a.N / 8;
  const int total = a.M * g8, padded = (total + 31) / 32 * 32;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < padded; i += gridDim.x * blockDim.x) {
    const bool live = i < total;
    const int t = live ? i / g8 : 0, c = live ? (i % g8) * 8 : 0;
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float s = 0.f;
      for (int k = 0; live && k < a.kslices; ++k) s += a.part[((size_t)k * a.M + t) * a.N + c + q];
      v[q] = bf16r(s);
    }
    uint32_t o[4];
    if (a.q8) {
      float amax = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(v[q]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const int code = mx_code_vllm(amax);
      const float mul = mx_mul(code), sc = pow2c(code);
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint8_t b = e4m3_byte(v[q] * mul);
        if (q < 4) w0 |= (uint32_t)b << (8 * q);
        else w1 |= (uint32_t)b << (8 * (q - 4));
        v[q] = e4m3_float(b) * sc;
      }
      if (live) {
        *reinterpret_cast<uint2*>(a.q8 + (size_t)t * a.N + c) = make_uint2(w0, w1);
        if ((c & 31) == 0) a.q8s[(size_t)t * (a.N / 32) + c / 32] = (uint8_t)code;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
    if (live) *reinterpret_cast<uint4*>(a.out + (size_t)t * a.N + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  pdl_launch();
}

// MXFP4 weight [E][N][K/2] (even K in the low nibble) + E8M0 [E][N][K/32] -> fragment order:
// tile (e, rt, kc) of 16 rows x 128 K is 1024 bytes; byte 16 L + q of half h (h = 0, 1) of
// lane L = 4 g + t holds, for jj = q / 4 (block b = 2 h + jj / 2, half j = jj % 2) and
// e = q % 4, the source byte of row 16 rt + g + 8 (e & 1) at K index
// 128 kc + 32 b + 16 j + 8 (e >> 1) + 2 t. Codes: 64 bytes a tile, 8 a row pair g:
// (g, b0), (g + 8, b0), (g, b1), (g + 8, b1), ... (g + 8, b3).
__global__ void relayout_mxfp4_kernel(const uint8_t* __restrict__ src, const uint8_t* __restrict__ src_codes,
                                      uint8_t* __restrict__ dst, uint8_t* __restrict__ dst_codes,
                                      int64_t E, int N, int K) {
  const int64_t tiles = (int64_t)E * (N / 16) * (K / 128);
  const int64_t total = tiles * 1024;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = i / 1024;
    const int r = (int)(i % 1024);
    const int h = r / 512, L = (r % 512) / 16, q = r % 16;
    const int g = L / 4, t = L % 4, jj = q / 4, e = q % 4;
    const int b = 2 * h + jj / 2, j = jj % 2;
    const int kc = (int)(tile % (K / 128));
    const int64_t rt_all = tile / (K / 128);  // e * (N / 16) + rt
    const int64_t ex = rt_all / (N / 16);
    const int rt = (int)(rt_all % (N / 16));
    const int row = 16 * rt + g + 8 * (e & 1);
    const int k = 128 * kc + 32 * b + 16 * j + 8 * (e >> 1) + 2 * t;
    dst[i] = src[(ex * N + row) * (int64_t)(K / 2) + k / 2];
    if (i % 16 == 0 && L < 8 && h == 0) {
      // codes of row pair g = L (one writer a row pair)
      const int gg = L;
      for (int bb = 0; bb < 4; ++bb)
        for (int ee = 0; ee < 2; ++ee)
          dst_codes[tile * 64 + 8 * gg + 2 * bb + ee] =
              src_codes[(ex * N + 16 * rt + gg + 8 * ee) * (int64_t)(K / 32) + 4 * kc + bb];
    }
  }
}

}  // namespace dsv41
