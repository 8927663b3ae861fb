// K1 after the wqkv_a GEMV: the q / kv norms, the FP8 KV-record store, wq_b's epilogue
// (bf16 + GPT-J RoPE) and K2's key table. Restates front.py:117-355 of the reference.
#pragma once

#include "common.cuh"

namespace dsv41 {

struct FrontArgs {
  int M, QL, KVD, nope, rope;  // q_lora rank; kv latent dims (nope + rope)
  int kslices;                 // wqkv_a partial slices
  int index;                   // an index source: also write qr
  const float* qkv_part;       // [kslices][M][QL + KVD]
  const __nv_bfloat16* q_norm_w;   // [QL]
  const __nv_bfloat16* kv_norm_w;  // [KVD]
  const float* cos_sin;        // [positions, rope]: rope/2 cos, then rope/2 sin
  const int64_t* pos;          // [M]
  int64_t rope_rows;           // the table's positions (0: unchecked)
  const int64_t* slot;         // [M] KV slot (< 0: a pad row, nothing stored)
  uint8_t* cache;              // paged KV cache
  int64_t page_stride;         // bytes a page
  int blk;                     // slots a page
  // outputs
  __nv_bfloat16* qr;           // [M, QL] (index sources)
  uint8_t* qx8;                // [M, QL]
  uint8_t* qx8s;               // [M, QL / 32]
  __nv_bfloat16* qxq;          // [M, QL] qx8 dequantized (wq_b's input)
  float* qkv_out;              // optional [M, QL + KVD]: the summed fp32 projection
};

// A record: nope e4m3 bytes, rope bf16, then (in the page's scale rows) nope/64 E8M0 codes in
// an 8-byte slot. Page layout: blk data rows of (nope + 2 rope) bytes, then blk scale rows.
// Row t (a CTA of 256 threads).
__device__ __forceinline__ void front_qkv_body(const FrontArgs& a, int t) {
  __shared__ float red[8];
  __shared__ float tot_q;
  __shared__ double ssk[2];
  __shared__ float bmax[2][8];
  __shared__ int codes[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.QL + a.KVD;
  // the wqkv_a partials of this thread's values summed over the K slices in order, four slices'
  // loads in flight at a time: q values tid qper + i (qper = QL / 256 <= 4), kv values
  // QL + tid + 64 r (threads tid < 64, r < R <= 12)
  const int qper = a.QL / 256;
  const int R = a.KVD / 64;
  const bool kvt = tid < 64;
  float xq[4] = {0.f, 0.f, 0.f, 0.f};
  float xk[12];
#pragma unroll
  for (int r = 0; r < 12; ++r) xk[r] = 0.f;
  {
    const float* base = a.qkv_part + (size_t)t * W;
    const size_t sstride = (size_t)a.M * W;
    for (int s0 = 0; s0 < a.kslices; s0 += 4) {
      float uq[4][4], uk[4][12];
#pragma unroll
      for (int ds = 0; ds < 4; ++ds) {
        const bool in = s0 + ds < a.kslices;
        const float* b = base + (size_t)(s0 + ds) * sstride;
#pragma unroll
        for (int i = 0; i < 4; ++i) uq[ds][i] = (in && i < qper) ? b[tid * qper + i] : 0.f;
#pragma unroll
        for (int r = 0; r < 12; ++r) uk[ds][r] = (in && kvt && r < R) ? b[a.QL + tid + 64 * r] : 0.f;
      }
#pragma unroll
      for (int ds = 0; ds < 4; ++ds) {
        if (s0 + ds >= a.kslices) break;
#pragma unroll
        for (int i = 0; i < 4; ++i) xq[i] += uq[ds][i];
#pragma unroll
        for (int r = 0; r < 12; ++r) xk[r] += uk[ds][r];
      }
    }
    if (a.qkv_out) {
      for (int i = 0; i < qper; ++i) a.qkv_out[(size_t)t * W + tid * qper + i] = xq[i];
      if (kvt)
        for (int r = 0; r < R; ++r) a.qkv_out[(size_t)t * W + a.QL + tid + 64 * r] = xk[r];
    }
  }
  // ---- q: 4 consecutive values a thread (QL <= 1024), q_norm, bf16, vLLM MXFP8
  float ss = 0.f;
  for (int i = 0; i < qper; ++i) {
    xq[i] = bf16r(xq[i]);
    ss = fmaf(xq[i], xq[i], ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  // ---- kv: 64 threads, thread i holds dims i + 64 r (fixed-order fp64 sum of squares)
  if (kvt) {
    double acc = 0.0;
    for (int r = 0; r < R; ++r) {
      xk[r] = bf16r(xk[r]);
      acc = __dadd_rn(acc, __dmul_rn((double)xk[r], (double)xk[r]));
    }
    acc = warp_sum_d(acc);
    if (lane == 0) ssk[warp] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w];
    tot_q = s;
  }
  __syncthreads();
  // q_norm -> ys (bf16) -> MXFP8 (a 32-group = 32 / qper threads)
  {
    const float rq = 1.0f / sqrtf(tot_q / (float)a.QL + kRmsEps);
    float ys[4];
    float amax = 0.f;
    for (int i = 0; i < qper; ++i) {
      const int n = tid * qper + i;
      ys[i] = bf16r((xq[i] * rq) * bf2f(a.q_norm_w[n]));
      amax = fmaxf(amax, fabsf(ys[i]));
      if (a.index) a.qr[(size_t)t * a.QL + n] = __float2bfloat16_rn(ys[i]);
    }
    const int gthreads = 32 / qper;  // threads a group: 8, 16 or 32
    for (int d = 1; d < gthreads; d <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
    const int code = mx_code_vllm(amax);
    const float mul = mx_mul(code), sc = pow2c(code);
    for (int i = 0; i < qper; ++i) {
      const int n = tid * qper + i;
      const uint8_t b = e4m3_byte(ys[i] * mul);
      a.qx8[(size_t)t * a.QL + n] = b;
      a.qxq[(size_t)t * a.QL + n] = __float2bfloat16_rn(e4m3_float(b) * sc);
    }
    if ((tid * qper) % 32 == 0) a.qx8s[(size_t)t * (a.QL / 32) + tid * qper / 32] = (uint8_t)code;
  }
  // ---- kv record (bit-exact contract)
  const int64_t slot = a.slot[t];
  float e[12];
  if (tid < 64) {
    const float ssf = (float)__dadd_rn(ssk[0], ssk[1]);
    const float ms = __fadd_rn(__fdiv_rn(ssf, (float)a.KVD), kRmsEps);
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(ms));
    for (int q = 0; q < R; ++q) e[q] = __fmul_rn(__fmul_rn(xk[q], r), bf2f(a.kv_norm_w[tid + 64 * q]));
    // GPT-J RoPE of the dims past nope: pair (2j, 2j + 1) sits on threads 2j, 2j + 1 (r = R - 1)
    const int half = a.rope / 2;
    const int64_t p = rope_row(a.pos[t], a.rope_rows);
    for (int q = 0; q < R; ++q) {
      const int d = tid + 64 * q;
      if (d >= a.nope) {
        const int j = (d - a.nope) >> 1;
        const float c = a.cos_sin[p * a.rope + j], s = a.cos_sin[p * a.rope + half + j];
        const float mine = e[q];
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        if ((d & 1) == 0) e[q] = __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, s));
        else e[q] = __fadd_rn(__fmul_rn(other, s), __fmul_rn(mine, c));
      }
    }
    // 64-block amax of the nope dims: block q is dims 64 q .. 64 q + 63, one per thread
    for (int q = 0; q < a.nope / 64; ++q) {
      const float m = warp_max(fabsf(e[q]));
      if (lane == 0) bmax[warp][q] = m;
    }
  }
  __syncthreads();
  if (tid < a.nope / 64) {
    const float amax = fmaxf(bmax[0][tid], bmax[1][tid]);
    int c = code_ceil(__fdiv_rn(fmaxf(amax, 1e-4f), kFp8Max));
    codes[tid] = min(max(c, 0), 254);
  }
  __syncthreads();
  if (slot >= 0 && tid < 64) {
    const int data = a.nope + 2 * a.rope;
    uint8_t* page = a.cache + (slot / a.blk) * a.page_stride;
    const int off = (int)(slot % a.blk);
    uint8_t* rec = page + (size_t)off * data;
    for (int q = 0; q < R; ++q) {
      const int d = tid + 64 * q;
      if (d < a.nope) {
        rec[d] = e4m3_byte(e[q] * mx_mul(codes[q]));
      } else {
        *reinterpret_cast<uint16_t*>(rec + a.nope + 2 * (d - a.nope)) = f2bfbits(e[q]);
      }
    }
    if (tid < a.nope / 64) page[(size_t)a.blk * data + (size_t)off * 8 + tid] = (uint8_t)codes[tid];
  }
}

__global__ void __launch_bounds__(256) front_qkv_kernel(const FrontArgs a) {
  pdl_wait();
  front_qkv_body(a, blockIdx.x);
  pdl_launch();
}

struct QRopeArgs {
  int M, heads, D, nope, rope, kslices;
  const float* part;       // [kslices][M][heads * D]
  const float* cos_sin;    // [positions, rope]
  const int64_t* pos;      // [M]
  int64_t rope_rows;       // the table's positions (0: unchecked)
  __nv_bfloat16* q;        // [M, heads, D]
};

// q = bf16(wq_b partials summed); GPT-J RoPE of each head's dims past nope; bf16. A thread = 8
// consecutive dims (never across a head or the nope boundary: D and nope are multiples of 8).
// Block bx of gx along the row's dims, of row t.
__device__ __forceinline__ void q_rope_body(const QRopeArgs& a, int bx, int gx, int t) {
  const int N = a.heads * a.D;
  for (int g8 = bx * blockDim.x + threadIdx.x; g8 < N / 8; g8 += gx * blockDim.x) {
    const int n = 8 * g8;
    float v[8];
    sum_slices8(a.part + (size_t)t * N + n, (size_t)a.M * N, a.kslices, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = bf16r(v[q]);
    const int d = n % a.D;
    if (d >= a.nope) {
      const int64_t p = rope_row(a.pos[t], a.rope_rows);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const int j = (d + i - a.nope) >> 1;
        const float c = a.cos_sin[p * a.rope + j], s = a.cos_sin[p * a.rope + a.rope / 2 + j];
        const float e0 = __fsub_rn(__fmul_rn(v[i], c), __fmul_rn(v[i + 1], s));
        const float e1 = __fadd_rn(__fmul_rn(v[i], s), __fmul_rn(v[i + 1], c));
        v[i] = e0;
        v[i + 1] = e1;
      }
    }
    *reinterpret_cast<uint4*>(a.q + (size_t)t * N + n) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

__global__ void q_rope_kernel(const QRopeArgs a) {
  pdl_wait();
  q_rope_body(a, blockIdx.x, gridDim.x, blockIdx.y);
  pdl_launch();
}

struct KeyTableArgs {
  int M, swa_width, topk_width;
  const int64_t* slot;       // [M] (< 0: a pad row)
  const int32_t* swa_idx;    // [M, swa_width]
  const int32_t* swa_lens;   // [M]
  const int32_t* topk;       // [M, topk_width] (may be null when topk_width == 0)
  const int32_t* topk_lens;  // [M]
  int32_t* kt;               // [M, topk_width + swa_width]
  int32_t* klen;             // [2 M]: kv_len, then ntopk
};

// K2's key table (front.py:117-143): slot | 1 << 31 for the first ntopk keys (compressed
// rows), window slots for k in [ntopk, kv_len), -1 past them or for an invalid slot.
// Row t, block by of gy along its keys.
__device__ __forceinline__ void key_table_body(const KeyTableArgs& a, int t, int by, int gy) {
  const bool live = a.slot[t] >= 0;
  const int nswa = live ? min(a.swa_lens[t], a.swa_width) : 0;
  const int ntopk = (live && a.topk_width > 0) ? min(a.topk_lens[t], a.topk_width) : 0;
  const int kv = ntopk + nswa;
  const int keys = a.topk_width + a.swa_width;
  for (int k = by * blockDim.x + threadIdx.x; k < keys; k += gy * blockDim.x) {
    int v = -1;
    if (k < ntopk) {
      const int c = a.topk[(size_t)t * a.topk_width + k];
      v = c >= 0 ? (int)((uint32_t)c | 0x80000000u) : -1;
    } else if (k < kv) {
      const int s = a.swa_idx[(size_t)t * a.swa_width + (k - ntopk)];
      v = s >= 0 ? s : -1;
    }
    a.kt[(size_t)t * keys + k] = v;
  }
  if (threadIdx.x == 0 && by == 0) {
    a.klen[t] = kv;
    a.klen[a.M + t] = ntopk;
  }
}

__global__ void key_table_kernel(const KeyTableArgs a) {
  pdl_wait();
  key_table_body(a, blockIdx.x, blockIdx.y, gridDim.y);
  pdl_launch();
}

}  // namespace dsv41
