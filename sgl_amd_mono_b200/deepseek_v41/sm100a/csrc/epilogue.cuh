// GEMV epilogues that need no stage-specific math: K-slice sums rounded to bf16, optionally
// requantized to vLLM-rule MXFP8; the rank-order all-reduce sum; the MXFP4 tensor-core tile relayout.
#pragma once

#include "common.cuh"
#include "peer.cuh"

namespace dsv41 {

struct FinalizeArgs {
  int M, N, kslices;
  const float* part;      // [kslices][M][N]
  __nv_bfloat16* out;     // [M, N] bf16(sum) (or the dequantized MXFP8 when q8 is set)
  uint8_t* q8;            // optional [M, N] e4m3 (vLLM rule)
  uint8_t* q8s;           // [M, N / 32]
  PeerLL x;               // x.peers set: out is this rank's partial of a TP all-reduce into x.reduced
};

// A thread = 8 consecutive columns (4 threads a 32-group when requantizing). With an exchange
// (wo_b's epilogue at tp > 1: the attention all-reduce), each thread pushes its groups to every
// rank, then reduces the same groups from every rank (peer.cuh's fused exchange).
__global__ void finalize_kernel(const FinalizeArgs a) {
  pdl_wait();
  int xfail = 1;
  const uint32_t e = a.x.peers ? ll_begin(a.x, &xfail) : 0u;
  const int g8 = a.N / 8;
  const int total = a.M * g8, padded = (total + 31) / 32 * 32;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < padded; i += gridDim.x * blockDim.x) {
    const bool live = i < total;
    const int t = live ? i / g8 : 0, c = live ? (i % g8) * 8 : 0;
    float v[8];
    sum_slices8(a.part + (size_t)t * a.N + c, (size_t)a.M * a.N, live ? a.kslices : 0, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = bf16r(v[q]);
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
    if (live && !xfail) ll_push(a.x, e, i, o);
  }
  if (a.x.peers) {
    if (!xfail)
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        uint32_t o[4];
        if (!ll_reduce(a.x, e, i, o)) break;
        reinterpret_cast<uint4*>(a.x.reduced)[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    ll_end(a.x, e);
  }
  pdl_launch();
}

// MXFP4 weight [E][N][K/2] (even K in the low nibble) + E8M0 [E][N][K/32] -> the tensor-core
// tiles of expert_tc_kernel: tile (e, rt, kt) = 256 rows x 128 K at ((e RT + rt) KT + kt) 16384,
// RT = ceil(N / 256), KT = K / 128; its row r holds source row 256 rt + r, bytes 64 kt ..
// 64 kt + 63 (zero past N). Codes: 1024 bytes a tile, two TMEM scale atoms (rows 0..127, then
// 128..255); row r's code of K block 4 kt + b at (r / 128) * 512 + (r % 32) * 16 +
// ((r % 128) / 32) * 4 + b. 16 bytes (4 code bytes) a step.
__global__ void relayout_mxfp4_kernel(const uint8_t* __restrict__ src, const uint8_t* __restrict__ src_codes,
                                      uint8_t* __restrict__ dst, uint8_t* __restrict__ dst_codes,
                                      int64_t E, int N, int K) {
  const int RT = (N + 255) / 256, KT = K / 128;
  const int64_t tiles = E * RT * KT;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tiles * 1024; i += stride) {
    const int64_t tile = i / 1024;
    const int within = (int)(i % 1024) * 16;
    const int r = within / 64, cb = within % 64;
    const int kt = (int)(tile % KT);
    const int rt = (int)((tile / KT) % RT);
    const int64_t ex = tile / ((int64_t)KT * RT);
    const int row = 256 * rt + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < N) v = *reinterpret_cast<const uint4*>(src + (ex * N + row) * (int64_t)(K / 2) + 64 * kt + cb);
    *reinterpret_cast<uint4*>(dst + i * 16) = v;
  }
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < tiles * 256; j += stride) {
    const int64_t tile = j / 256;
    const int q = (int)(j % 256);  // (r / 128) * 128 + (r % 32) * 4 + (r % 128) / 32
    const int r = 128 * (q / 128) + (q % 128) / 4 + 32 * (q % 4);
    const int kt = (int)(tile % KT);
    const int rt = (int)((tile / KT) % RT);
    const int64_t ex = tile / ((int64_t)KT * RT);
    const int row = 256 * rt + r;
    uint32_t v = 0;
    if (row < N) v = *reinterpret_cast<const uint32_t*>(src_codes + (ex * N + row) * (int64_t)(K / 32) + 4 * kt);
    *reinterpret_cast<uint32_t*>(dst_codes + tile * 1024 + 4 * q) = v;
  }
}

}  // namespace dsv41
