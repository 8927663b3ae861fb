// mHC seam (hc_mult 4): the boundary before each sublayer (K1's attention seam, K2's FFN
// seam). Restates seam.py:137-378 of the reference:
//   R_new[o] = bf16(fma(c3 r3, ((post_o x + r0 c0o) + c1o r1) + c2o r2))   (a post owed)
//   LIN      = bf16(sum_h pre_prev[h] R_new[h])  (copy 0 of R on the first layer)
//   mixes    = hc_fn . R_new (24), sumsq = |R_new|^2  -> gate: pre / post / comb (Sinkhorn)
//   normed   = bf16((LIN rstd) w)  -> MXFP8 (vLLM rule; K2 also the aiter rule)
// Two launches: seam_slice (32-column slices, partial mixes per slice) and seam_gate_norm (a
// CTA per row: slices summed in slice order, gate, RMSNorm and quantization).
#pragma once

#include "common.cuh"

namespace dsv41 {

constexpr int kHC = 4;
constexpr int kMix = 24;
constexpr int kPart = kMix + 1;  // a slice's partials a row: 24 mixes, then the sum of squares
constexpr int kSliceCols = 32;
constexpr float kHcEps = 1e-6f;

struct SeamArgs {
  int M, H;
  int fold;   // a post is owed: fold x into the residual
  int first;  // the first layer: the collapse is copy 0
  int aiter;  // also write the aiter-rule MXFP8 (routed experts' input)
  const __nv_bfloat16* res_in;  // [M, 4, H]
  const __nv_bfloat16* x;       // [M, H] pending sublayer output (fold)
  const float* post_in;         // [M, 4]
  const float* comb_in;         // [M, 4(src), 4(dst)]
  const float* pre_in;          // [M, 4] previous pre (collapse)
  const float* hc_fn;           // [24, 4 H]
  const float* hc_scale;        // [3]
  const float* hc_base;         // [24]
  const __nv_bfloat16* norm_w;  // [H]
  // outputs
  __nv_bfloat16* res_out;   // [M, 4, H]
  float* pre_out;           // [M, 4]
  float* post_out;          // [M, 4]
  float* comb_out;          // [M, 4, 4]
  __nv_bfloat16* normed;    // [M, H]
  uint8_t* x8;              // [M, H] e4m3 (vLLM rule)
  uint8_t* x8s;             // [M, H / 32] codes
  __nv_bfloat16* xq;        // [M, H] x8 dequantized (the GEMVs' input)
  uint8_t* x8r;             // [M, H] e4m3 (aiter rule), when aiter
  uint8_t* x8rs;            // [M, H / 32]
  // scratch
  __nv_bfloat16* lin;       // [M, H]
  float* part;              // [M, H / 32, 25]
};

constexpr int kSeamSliceSmem = (kMix + 48) * kHC * kSliceCols * 4;  // a slice's mix weights, R_new of every row

// One 32-column slice s of every row (a CTA of 256 threads; smem: kSeamSliceSmem bytes). The
// launch (seam_slice_kernel) waits for its inputs between the mix-weight loads and the rest
// (wait = true); the persistent K1 has waited already.
__device__ __forceinline__ void seam_slice_body(const SeamArgs& a, int s, float* smem, bool wait) {
  float* fn = smem;                               // this slice's mix weights
  float* rs = smem + kMix * kHC * kSliceCols;     // R_new of every row (bf16-valued)
  const int c0 = s * kSliceCols, H = a.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // mix weights first: they wait on nothing
  for (int e = tid; e < kMix * kHC * kSliceCols; e += blockDim.x) {
    const int j = e / (kHC * kSliceCols), r = e % (kHC * kSliceCols), o = r / kSliceCols,
              c = r % kSliceCols;
    fn[e] = __ldg(a.hc_fn + (size_t)j * kHC * H + (size_t)o * H + c0 + c);
  }
  if (wait) pdl_wait();
  // R_new of (row t, column c) and the collapsed layer input: one thread an element, its loads
  // before any store
#pragma unroll 2
  for (int e = tid; e < a.M * kSliceCols; e += blockDim.x) {
    const int t = e / kSliceCols, c = e % kSliceCols;
    const size_t col = (size_t)t * kHC * H + c0 + c;  // copy o at + o * H
    float rv[kHC];
    if (a.fold) {
      float r[kHC];
#pragma unroll
      for (int h = 0; h < kHC; ++h) r[h] = bf2f(a.res_in[col + (size_t)h * H]);
      const float xv = bf2f(a.x[(size_t)t * H + c0 + c]);
      const float* cm = a.comb_in + t * 16;
#pragma unroll
      for (int o = 0; o < kHC; ++o) {
        float v = __fadd_rn(__fmul_rn(a.post_in[t * kHC + o], xv), __fmul_rn(r[0], cm[0 * 4 + o]));
        v = __fadd_rn(v, __fmul_rn(cm[1 * 4 + o], r[1]));
        v = __fadd_rn(v, __fmul_rn(cm[2 * 4 + o], r[2]));
        rv[o] = bf16r(__fmaf_rn(cm[3 * 4 + o], r[3], v));
      }
    } else {
#pragma unroll
      for (int o = 0; o < kHC; ++o) rv[o] = bf2f(a.res_in[col + (size_t)o * H]);
    }
    float acc;  // the layer input: R_new collapsed with the previous pre, h in order
    if (a.first) {
      acc = rv[0];
    } else {
      acc = 0.f;
#pragma unroll
      for (int h = 0; h < kHC; ++h) acc = __fadd_rn(acc, __fmul_rn(a.pre_in[t * kHC + h], rv[h]));
    }
#pragma unroll
    for (int o = 0; o < kHC; ++o) {
      a.res_out[col + (size_t)o * H] = __float2bfloat16_rn(rv[o]);
      rs[t * kHC * kSliceCols + o * kSliceCols + c] = rv[o];
    }
    a.lin[(size_t)t * H + c0 + c] = __float2bfloat16_rn(acc);
  }
  __syncthreads();
  // partial mixes and the sum of squares: a warp a row, its 25 dot products of 4 terms a lane
  // reduced over the warp together (lane j takes product j)
  const int nslices = H / kSliceCols;
  for (int t = warp; t < a.M; t += 8) {
    const float* r = rs + t * kHC * kSliceCols;
    float rr[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) rr[q] = r[lane + 32 * q];
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float acc = 0.f;
      if (j < kPart) {
#pragma unroll
        for (int q = 0; q < 4; ++q) acc = fmaf(j < kMix ? fn[j * kHC * kSliceCols + lane + 32 * q] : rr[q], rr[q], acc);
      }
      v[j] = acc;
    }
    const float sum = warp_transpose_sum(v, lane);
    if (lane < kPart) a.part[((size_t)t * nslices + s) * kPart + lane] = sum;
  }
}

__global__ void __launch_bounds__(256) seam_slice_kernel(const SeamArgs a) {
  __shared__ float smem[kSeamSliceSmem / 4];
  seam_slice_body(a, blockIdx.x, smem, true);
  pdl_launch();
}

// Store one row's 32-value group as MXFP8 (vLLM or aiter rule) from 8 values a lane; lanes
// 4 g .. 4 g + 3 of a warp hold group g.
__device__ __forceinline__ void mx_group_store(const float (&v)[8], bool vllm, uint8_t* q8,
                                               uint8_t* codes, __nv_bfloat16* deq, int col) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const int code = vllm ? mx_code_vllm(amax) : mx_code_aiter(amax);
  const float mul = mx_mul(code), sc = pow2c(code);
  uint32_t w0 = 0, w1 = 0;
  uint32_t d[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint8_t b = e4m3_byte(v[i] * mul);
    if (i < 4) w0 |= (uint32_t)b << (8 * i);
    else w1 |= (uint32_t)b << (8 * (i - 4));
    if (deq) {
      const float dv = e4m3_float(b) * sc;
      if (i & 1) d[i >> 1] |= (uint32_t)f2bfbits(dv) << 16;
      else d[i >> 1] = f2bfbits(dv);
    }
  }
  *reinterpret_cast<uint2*>(q8 + col) = make_uint2(w0, w1);
  if ((threadIdx.x & 3) == 0) codes[col / 32] = (uint8_t)code;
  if (deq) *reinterpret_cast<uint4*>(deq + col) = make_uint4(d[0], d[1], d[2], d[3]);
}

// Row t's gates and norm (a CTA of 256 threads).
__device__ __forceinline__ void seam_gate_norm_body(const SeamArgs& a, int t) {
  __shared__ double red[8];
  __shared__ float tot_s;
  __shared__ float gsum[8][kPart];
  const int H = a.H, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // ---- gate: the slices' partials summed in slice order (warp w: a contiguous eighth of the
  // slices, then the eight warp sums in warp order), then one warp computes the gates
  {
    const int nslices = H / kSliceCols;
    const int s0 = warp * nslices / 8, s1 = (warp + 1) * nslices / 8;
    if (lane < kPart) {
      // (eight slices' loads in flight, added in slice order)
      const float* pp = a.part + (size_t)t * nslices * kPart + lane;
      float acc = 0.f;
      int s = s0;
      for (; s + 8 <= s1; s += 8) {
        float u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) u[i] = pp[(size_t)(s + i) * kPart];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc += u[i];
      }
      for (; s < s1; ++s) acc += pp[(size_t)s * kPart];
      gsum[warp][lane] = acc;
    }
  }
  __syncthreads();
  if (warp == 0) {
    float mix = 0.f, sq = 0.f;
    for (int w = 0; w < 8; ++w) {
      mix += gsum[w][min(lane, kMix - 1)];
      sq += gsum[w][kMix];
    }
    const float v = mix * (1.0f / sqrtf(sq / (float)(kHC * H) + kRmsEps));
    const int j = min(lane, kMix - 1);
    if (lane < kHC) {
      a.pre_out[t * kHC + lane] = 1.0f / (1.0f + expf(-(v * a.hc_scale[0] + a.hc_base[j]))) + kHcEps;
    } else if (lane < 2 * kHC) {
      a.post_out[t * kHC + lane - kHC] = 2.0f / (1.0f + expf(-(v * a.hc_scale[1] + a.hc_base[j])));
    }
    // comb: lanes 8 .. 23 hold entry (r, c) = lane - 8 = 4 r + c; the 16-lane group 8..23 is
    // mapped onto lanes 0..15 by a shuffle so row / column partners are xor 1, 2 / 4, 8 apart
    float cv = v * a.hc_scale[2] + a.hc_base[j];
    cv = __shfl_sync(0xffffffffu, cv, (lane & 15) + 8);
    auto rsum = [&](float x) {
      const float p = x + __shfl_xor_sync(0xffffffffu, x, 1);
      return p + __shfl_xor_sync(0xffffffffu, p, 2);
    };
    auto csum = [&](float x) {
      const float p = x + __shfl_xor_sync(0xffffffffu, x, 4);
      return p + __shfl_xor_sync(0xffffffffu, p, 8);
    };
    float m = fmaxf(cv, __shfl_xor_sync(0xffffffffu, cv, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    cv = expf(cv - m);
    cv = cv / rsum(cv) + kHcEps;
    cv = cv / (csum(cv) + kHcEps);
    for (int it = 1; it < 20; ++it) {
      cv = cv / (rsum(cv) + kHcEps);
      cv = cv / (csum(cv) + kHcEps);
    }
    if (lane < 16) a.comb_out[t * 16 + lane] = cv;
  }
  // ---- norm: 8 consecutive columns a thread. The sum of squares is fp64 (each bf16 square
  // exact) in a fixed order -- a thread's columns in order, an xor-butterfly in each warp, the
  // warps in order -- and rounded once to fp32, so the scale and the normed row are bit-exact
  // (the oracle's seam_sumsq follows the same order).
  double ss = 0.0;
  for (int c = tid * 8; c < H; c += blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(a.lin + (size_t)t * H + c);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const double lo = __uint_as_float(ws[i] << 16), hi = __uint_as_float(ws[i] & 0xffff0000u);
      ss = __dadd_rn(ss, __dmul_rn(lo, lo));
      ss = __dadd_rn(ss, __dmul_rn(hi, hi));
    }
  }
  ss = warp_sum_d(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid == 0) {
    double s = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s = __dadd_rn(s, red[w]);
    tot_s = (float)s;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(tot_s / (float)H + kRmsEps);
  for (int c = tid * 8; c < H; c += blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(a.lin + (size_t)t * H + c);
    const uint4 nw = *reinterpret_cast<const uint4*>(a.norm_w + c);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    const uint32_t ns[4] = {nw.x, nw.y, nw.z, nw.w};
    float y[8];
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      y[2 * i] = bf16r((__uint_as_float(ws[i] << 16) * r) * __uint_as_float(ns[i] << 16));
      y[2 * i + 1] = bf16r((__uint_as_float(ws[i] & 0xffff0000u) * r) * __uint_as_float(ns[i] & 0xffff0000u));
      o[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
    }
    const size_t at = (size_t)t * H + c;
    *reinterpret_cast<uint4*>(a.normed + at) = make_uint4(o[0], o[1], o[2], o[3]);
    mx_group_store(y, true, a.x8 + (size_t)t * H, a.x8s + (size_t)t * (H / 32), a.xq + (size_t)t * H, c);
    if (a.aiter)
      mx_group_store(y, false, a.x8r + (size_t)t * H, a.x8rs + (size_t)t * (H / 32), nullptr, c);
  }
}

__global__ void __launch_bounds__(256) seam_gate_norm_kernel(const SeamArgs a) {
  pdl_wait();
  seam_gate_norm_body(a, blockIdx.x);
  pdl_launch();
}

}  // namespace dsv41
