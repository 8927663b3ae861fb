// The indexer's FP4 query of decode rows, K2i's input: SGLang's index_q_rope_pack_weights (called
// with the split-K head-weight GEMV at spec.py:744-763 of the reference), restated on the device.
//
// Contract (oracle/indexer.py:index_query), per row t:
//   head weights  w[h] = bf16(fp32(x . Wp[h]) * s): the dot of the normed row with the head's
//                 weight-projection row as router_kernel sums it (exact bf16 products, fp64 in a
//                 fixed lane order, one rounding to fp32), times the fp32 scale s, rounded once;
//   RoPE          on the last `rope` of the head's dims, GPT-J pairs (2j, 2j + 1) with the
//                 layer's cos / sin: e0 = k0 c - k1 s, e1 = k0 s + k1 c, each product and sum
//                 rounded in fp32 (no fused multiply-add);
//   MXFP4         per 32 dims: code = the E8M0 ceiling of fp32(max(amax, 2^-126) / 6) (exponent
//                 field, plus one when the mantissa is not zero), values times 2^(127 - code) to
//                 E2M1 by round to nearest even with saturation (cvt.rn.satfinite.e2m1x2.f32),
//                 sign kept (a negative value that rounds to zero is E2M1 -0); even dims in the
//                 low nibble.
// Layout: q_out [M, heads, dim / 2] bytes; qscale [M, 1, 4, 16, 4] with head h's chunk c at
// [c, h % 16, h / 16] (K2i's); w_out [M, heads] bf16.
#pragma once

#include "common.cuh"

namespace dsv41 {

struct IndexQueryArgs {
  int M, heads, dim, rope;
  const __nv_bfloat16* q;      // [M, heads, dim] (wq_b's output)
  const float* cos_sin;        // [rope_rows, rope]: rope / 2 cos, then rope / 2 sin
  int64_t rope_rows;
  const int64_t* pos;          // [M]
  const float* hw;             // [M, heads] fp32 head-weight dots (router_kernel)
  float scale;                 // head_weight_scale
  uint8_t* q_out;              // [M, heads, dim / 2]
  uint8_t* qscale;             // [M, 256]
  __nv_bfloat16* w_out;        // [M, heads]
};

__device__ __forceinline__ uint32_t e2m1x2(float even, float odd) {
  uint16_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.u16.u8 %0, t; }" : "=h"(r) : "f"(odd), "f"(even));
  return r;
}

// grid M, 256 threads: thread i = (head i / 4, 32-dim chunk i % 4) of the row; the first heads
// threads also write the head weights.
__global__ void __launch_bounds__(256) index_query_kernel(const IndexQueryArgs a) {
  pdl_wait();
  const int t = blockIdx.x;
  const int chunks = a.dim / 32;
  const int64_t p = min(max(a.pos[t], (int64_t)0), a.rope_rows - 1);
  const float* cs = a.cos_sin + p * a.rope;
  const int rope0 = a.dim - a.rope;
  for (int i = threadIdx.x; i < a.heads * chunks; i += blockDim.x) {
    const int h = i / chunks, c = i % chunks;
    const __nv_bfloat16* src = a.q + ((size_t)t * a.heads + h) * a.dim + 32 * c;
    float v[32];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + 8 * u);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[8 * u + 2 * q] = __uint_as_float(ws[q] << 16);
        v[8 * u + 2 * q + 1] = __uint_as_float(ws[q] & 0xffff0000u);
      }
    }
    if (32 * c + 32 > rope0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int d = 32 * c + 2 * j;
        if (d < rope0) continue;
        const int pr = (d - rope0) / 2;
        const float co = cs[pr], si = cs[a.rope / 2 + pr];
        const float k0 = v[2 * j], k1 = v[2 * j + 1];
        v[2 * j] = __fsub_rn(__fmul_rn(k0, co), __fmul_rn(k1, si));
        v[2 * j + 1] = __fadd_rn(__fmul_rn(k0, si), __fmul_rn(k1, co));
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float q6 = __fdiv_rn(fmaxf(amax, 1.17549435082228750797e-38f), 6.0f);
    const uint32_t bits = __float_as_uint(q6);
    const int code = min((int)((bits >> 23) & 0xff) + ((bits & 0x7fffff) != 0), 253);
    const float mul = __uint_as_float((uint32_t)(254 - code) << 23);  // 2^(127 - code)
    uint32_t out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t wd = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int j = 8 * q + 2 * b;
        wd |= e2m1x2(v[j] * mul, v[j + 1] * mul) << (8 * b);
      }
      out[q] = wd;
    }
    *reinterpret_cast<uint4*>(a.q_out + ((size_t)t * a.heads + h) * (a.dim / 2) + 16 * c) =
        make_uint4(out[0], out[1], out[2], out[3]);
    a.qscale[(size_t)t * 256 + c * 64 + (h % 16) * 4 + h / 16] = (uint8_t)code;
  }
  for (int h = threadIdx.x; h < a.heads; h += blockDim.x)
    a.w_out[(size_t)t * a.heads + h] = __float2bfloat16_rn(__fmul_rn(a.hw[(size_t)t * a.heads + h], a.scale));
  pdl_launch();
}

}  // namespace dsv41
