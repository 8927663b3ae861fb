// K2's sparse MLA-style attention over FP8 KV records (back.py:145-532 of the reference).
//
// split  : CTA = (row, key chunk, 16-head tile). Per 64-key sub-block the records are
//          fetched through the key table, dequantized (e4m3 x 2^(code-127), rope bf16) into an
//          fp16 tile in shared memory that serves as both K and V (exact for record values in
//          fp16's range); S = Q K^T and O += P V on mma.sync f16 with an online softmax in the
//          exp2 domain. P is rounded to fp16 (11 significant bits) for the PV product. Writes the chunk's
//          unnormalized O and (max, sum) per head.
// combine: a CTA per (row, head): chunks merged with the attention sink folded into the max
//          and the denominator, o = bf16(sum / l), inverse GPT-J RoPE of the dims past nope,
//          bf16 -> XO.
#pragma once

#include "common.cuh"

namespace dsv41 {

constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  int M, heads, D, nope, rope;
  int keys_ld;       // key-table row length
  int nchunks, chunk_keys, head_tiles;
  const __nv_bfloat16* q;  // [M, heads, D]
  const int32_t* kt;       // [M, keys_ld]
  const int32_t* klen;     // [2 M]
  const uint8_t* swa;
  int64_t swa_stride;
  int swa_blk;
  const uint8_t* comp;     // may be null (a window-only layer)
  int64_t comp_stride;
  int comp_blk;
  float scale_log2;        // D^-0.5 log2(e)
  float* part_o;           // [M][nchunks][heads][D]
  float* part_ml;          // [M][nchunks][heads][2]
};

constexpr int kSub = 64;  // keys a sub-block

__host__ __device__ inline int attn_smem_bytes(int D) {
  return 16 * (D + 8) * 2 + kSub * (D + 8) * 2 + 2 * 16 * (kSub + 8) * 2 + 2 * 8 * 16 * 4 +
         2 * kSub * 8 + 2 * kSub * 8;
}

__global__ void __launch_bounds__(256, 2) attn_split_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int D = a.D, ld = D + 8;
  __half* Qs = reinterpret_cast<__half*>(smem);
  __half* Ks = Qs + 16 * ld;
  __half* Ps = Ks + kSub * ld;
  __half* Pl = Ps + 16 * (kSub + 8);
  float* redm = reinterpret_cast<float*>(Pl + 16 * (kSub + 8));
  float* redl = redm + 8 * 16;
  const uint8_t** kdata = reinterpret_cast<const uint8_t**>(redl + 8 * 16);
  uint64_t* kcodes = reinterpret_cast<uint64_t*>(kdata + 2 * kSub);

  const int ht = blockIdx.x % a.head_tiles;
  const int ch = (blockIdx.x / a.head_tiles) % a.nchunks;
  const int t = blockIdx.x / (a.head_tiles * a.nchunks);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int h0 = ht * 16;

  pdl_wait();
  const int kv = a.klen[t];
  const int k0 = ch * a.chunk_keys, k1 = min(k0 + a.chunk_keys, kv);
  // Q tile (heads past the rank's count stay zero)
  for (int e = tid; e < 16 * (D / 8); e += blockDim.x) {
    const int h = e / (D / 8), c = e % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h0 + h < a.heads) {
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.heads + h0 + h) * D + 8 * c);
      v = make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
    }
    *reinterpret_cast<uint4*>(Qs + h * ld + 8 * c) = v;
  }
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int ntile = D / 8 / 8;  // PV n-tiles a warp (D / 64)
  float o[9][4];
#pragma unroll
  for (int n = 0; n < 9; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[n][i] = 0.f;
  const int data_bytes = a.nope + 2 * a.rope;

  // key k of the row -> its record's data pointer (null: masked) and its 8 scale codes
  auto resolve = [&](int k, const uint8_t*& dp, uint64_t& cw) {
    dp = nullptr;
    cw = 0;
    if (k >= k1) return;
    const int v = a.kt[(size_t)t * a.keys_ld + k];
    if (v == -1) return;
    const bool comp = v < 0 && a.comp != nullptr;
    if (v < 0 && !comp) return;
    const int s = v & 0x7fffffff;
    const int blk = comp ? a.comp_blk : a.swa_blk;
    const uint8_t* page = (comp ? a.comp : a.swa) + (int64_t)(s / blk) * (comp ? a.comp_stride : a.swa_stride);
    const int off = s % blk;
    dp = page + (size_t)off * data_bytes;
    cw = *reinterpret_cast<const uint64_t*>(page + (size_t)blk * data_bytes + (size_t)off * 8);
  };
  const uint8_t* ndp = nullptr;
  uint64_t ncw = 0;
  if (tid < kSub) resolve(k0 + tid, ndp, ncw);
  int buf = 0;
  for (int kb = k0; kb < k1; kb += kSub, buf ^= 1) {
    const uint8_t** kd = kdata + buf * kSub;
    const uint64_t* kc = kcodes + buf * kSub;
    if (tid < kSub) {
      kdata[buf * kSub + tid] = ndp;
      kcodes[buf * kSub + tid] = ncw;
    }
    __syncthreads();
    // ---- every record load of the sub-block in flight at once, then the next sub-block's keys
    const int chunks = data_bytes / 16;  // <= 40 (nope <= 512, rope 64)
    constexpr int kItems = kSub * 40 / 256;
    uint4 raw[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int e = tid + 256 * i;
      raw[i] = make_uint4(0, 0, 0, 0);
      if (e < kSub * chunks) {
        const uint8_t* dp = kd[e / chunks];
        if (dp) raw[i] = ldg16(dp + 16 * (e % chunks));
      }
    }
    if (tid < kSub) resolve(kb + kSub + tid, ndp, ncw);
    // ---- dequantize into the fp16 K/V tile
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int e = tid + 256 * i;
      if (e >= kSub * chunks) continue;
      const int k = e / chunks, c = e % chunks;
      const uint8_t* dp = kd[k];
      uint4 out0 = make_uint4(0, 0, 0, 0), out1 = make_uint4(0, 0, 0, 0);
      const int b0 = 16 * c;
      if (b0 < a.nope) {
        if (dp) {
          const int code = (int)((kc[k] >> (8 * (b0 / 64))) & 0xff);
          const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
          uint32_t r[8];
          if (code >= 113 && code <= 134) {
            // e4m3 -> f16 is exact, and so is the product by 2^(code-127) in this code range
            // (no f16 overflow; the smallest e4m3 subnormal stays on f16's subnormal grid)
            const uint32_t s1 = (uint32_t)(code - 112) << 10;
            const uint32_t s2 = s1 | (s1 << 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              r[2 * i] = hmul2_bits(e4m3x2_f16(w[i] & 0xffff), s2);
              r[2 * i + 1] = hmul2_bits(e4m3x2_f16(w[i] >> 16), s2);
            }
          } else {
            const float sc = pow2c(code);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 fl = e4m3x2_float2(w[i] & 0xffff), fh = e4m3x2_float2(w[i] >> 16);
              r[2 * i] = pack_f16x2(fl.x * sc, fl.y * sc);
              r[2 * i + 1] = pack_f16x2(fh.x * sc, fh.y * sc);
            }
          }
          out0 = make_uint4(r[0], r[1], r[2], r[3]);
          out1 = make_uint4(r[4], r[5], r[6], r[7]);
        }
        *reinterpret_cast<uint4*>(Ks + k * ld + b0) = out0;
        *reinterpret_cast<uint4*>(Ks + k * ld + b0 + 8) = out1;
      } else {
        if (dp) {
          out0 = make_uint4(bf16x2_to_f16x2(raw[i].x), bf16x2_to_f16x2(raw[i].y), bf16x2_to_f16x2(raw[i].z),
                            bf16x2_to_f16x2(raw[i].w));
        }
        *reinterpret_cast<uint4*>(Ks + k * ld + a.nope + (b0 - a.nope) / 2) = out0;
      }
    }
    __syncthreads();
    // ---- S = Q K^T: warp w takes keys 8 w .. 8 w + 7
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      // three independent accumulation chains over the head dims, summed at the end
      float s1[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t qa = smem_u32(Qs) + (uint32_t)((((lane & 7) + 8 * ((lane >> 3) & 1)) * ld + 8 * (lane >> 4)) * 2);
      const uint32_t kbase = smem_u32(Ks) + (uint32_t)(((8 * warp + (lane & 7)) * ld + 8 * ((lane >> 3) & 1)) * 2);
      int kk = 0;
      for (; kk + 2 < D / 16; kk += 3) {
        uint32_t af[3][4], bfr[3][2];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          ldmatrix_x4(af[j], qa + (kk + j) * 32);
          ldmatrix_x2(bfr[j], kbase + (kk + j) * 32);
        }
        mma_f16(s, af[0][0], af[0][1], af[0][2], af[0][3], bfr[0][0], bfr[0][1]);
        mma_f16(s1, af[1][0], af[1][1], af[1][2], af[1][3], bfr[1][0], bfr[1][1]);
        mma_f16(s2, af[2][0], af[2][1], af[2][2], af[2][3], bfr[2][0], bfr[2][1]);
      }
      for (; kk < D / 16; ++kk) {
        uint32_t af[4], bfr[2];
        ldmatrix_x4(af, qa + kk * 32);
        ldmatrix_x2(bfr, kbase + kk * 32);
        mma_f16(s1, af[0], af[1], af[2], af[3], bfr[0], bfr[1]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) s[i] = (s[i] + s1[i]) + s2[i];
    }
    // scale and mask; per-head max of this warp's keys
    float mx[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = 8 * warp + 2 * tq + (i & 1);
      s[i] = kd[key] ? s[i] * a.scale_log2 : -INFINITY;
    }
    mx[0] = fmaxf(s[0], s[1]);
    mx[1] = fmaxf(s[2], s[3]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    if (tq == 0) {
      redm[warp * 16 + g] = mx[0];
      redm[warp * 16 + g + 8] = mx[1];
    }
    __syncthreads();
    float mnew[2], alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float m = m_run[h];
      for (int w = 0; w < 8; ++w) m = fmaxf(m, redm[w * 16 + g + 8 * h]);
      mnew[h] = m;
      alpha[h] = (m_run[h] == -INFINITY) ? 0.f : exp2f(m_run[h] - m);
    }
    float p[4], ls[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int h = i >> 1;
      p[i] = (s[i] == -INFINITY) ? 0.f : exp2f(s[i] - mnew[h]);
      ls[h] += p[i];
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 1);
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 2);
    }
    {
      // P as an fp16 head plus an fp16 tail (p - head): the PV product sees ~22 bits of p
      float hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hi[i] = __half2float(__float2half_rn(p[i]));
        lo[i] = p[i] - hi[i];
      }
      *reinterpret_cast<uint32_t*>(Ps + g * (kSub + 8) + 8 * warp + 2 * tq) = pack_f16x2(hi[0], hi[1]);
      *reinterpret_cast<uint32_t*>(Ps + (g + 8) * (kSub + 8) + 8 * warp + 2 * tq) = pack_f16x2(hi[2], hi[3]);
      *reinterpret_cast<uint32_t*>(Pl + g * (kSub + 8) + 8 * warp + 2 * tq) = pack_f16x2(lo[0], lo[1]);
      *reinterpret_cast<uint32_t*>(Pl + (g + 8) * (kSub + 8) + 8 * warp + 2 * tq) = pack_f16x2(lo[2], lo[3]);
    }
    if (tq == 0) {
      redl[warp * 16 + g] = ls[0];
      redl[warp * 16 + g + 8] = ls[1];
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float l = 0.f;
      for (int w = 0; w < 8; ++w) l += redl[w * 16 + g + 8 * h];
      l_run[h] = l_run[h] * alpha[h] + l;
      m_run[h] = mnew[h];
    }
#pragma unroll
    for (int n = 0; n < 9; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // ---- O += P V: warp w takes dims 8 ntile w .. + 8 ntile
    {
      const uint32_t pa = smem_u32(Ps) + (uint32_t)((((lane & 7) + 8 * ((lane >> 3) & 1)) * (kSub + 8) + 8 * (lane >> 4)) * 2);
      const int dim0 = warp * 8 * ntile;
      const uint32_t pla = pa + (uint32_t)((Pl - Ps) * 2);
      for (int kk = 0; kk < kSub / 16; ++kk) {
        uint32_t af[4], al[4];
        ldmatrix_x4(af, pa + kk * 32);
        ldmatrix_x4(al, pla + kk * 32);
        const int key = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int n = 0; n + 1 < 9; n += 2) {
          if (n + 1 < ntile) {
            uint32_t b[4];
            ldmatrix_x4_trans(b, smem_u32(Ks) + (uint32_t)((key * ld + dim0 + 8 * n + 8 * (lane >> 4)) * 2));
            mma_f16(o[n], al[0], al[1], al[2], al[3], b[0], b[1]);
            mma_f16(o[n], af[0], af[1], af[2], af[3], b[0], b[1]);
            mma_f16(o[n + 1], al[0], al[1], al[2], al[3], b[2], b[3]);
            mma_f16(o[n + 1], af[0], af[1], af[2], af[3], b[2], b[3]);
          }
        }
        if (ntile & 1) {
          const int n = ntile - 1;
          uint32_t b[2];
          ldmatrix_x2_trans(b, smem_u32(Ks) + (uint32_t)((key * ld + dim0 + 8 * n) * 2));
#pragma unroll
          for (int q = 0; q < 9; ++q)
            if (q == n) {
              mma_f16(o[q], al[0], al[1], al[2], al[3], b[0], b[1]);
              mma_f16(o[q], af[0], af[1], af[2], af[3], b[0], b[1]);
            }
        }
      }
    }
    __syncthreads();
  }
  // ---- the chunk's partial
  const size_t base = ((size_t)t * a.nchunks + ch) * a.heads;
  const int dim0 = warp * 8 * ntile;
#pragma unroll
  for (int n = 0; n < 9; ++n) {
    if (n < ntile) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int h = h0 + g + 8 * hh;
        if (h < a.heads) {
          float2 v = make_float2(o[n][2 * hh], o[n][2 * hh + 1]);
          *reinterpret_cast<float2*>(a.part_o + (base + h) * D + dim0 + 8 * n + 2 * tq) = v;
        }
      }
    }
  }
  if (warp == 0 && tq == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int h = h0 + g + 8 * hh;
      if (h < a.heads) {
        a.part_ml[(base + h) * 2] = m_run[hh];
        a.part_ml[(base + h) * 2 + 1] = l_run[hh];
      }
    }
  }
  pdl_launch();
}

struct CombineArgs {
  int M, heads, D, nope, rope, nchunks;
  const float* part_o;
  const float* part_ml;
  const float* sink;       // [heads] (this rank's)
  const float* cos_sin;    // [positions, rope]
  const int64_t* pos;      // [M]
  int64_t rope_rows;       // the table's positions (0: unchecked)
  __nv_bfloat16* xo;       // [M, heads * D]
};

// One CTA a (row, head): the chunks' weights 2^(m_c - m) (0 for an empty chunk) go to shared
// memory first; then each thread sums 4 dims over the chunks in order, B chunks' loads a batch,
// while one otherwise idle thread sums the denominator in chunk order (the same sums, in the same
// order, as one chunk at a time, for either B).
// B = 16 (many CTAs: 12 resident an SM at ptxas's 32 registers, which keeps only a few of a
// thread's loads in flight; occupancy hides the rest). B = 32 when the grid is one CTA an SM or
// less and there are more than 16 chunks (M = 1: 64 CTAs over 57 chunks): one CTA an SM lets
// ptxas hold all 32 loads of a batch in registers (209): 2 batches of round trips a head.
constexpr int kCombineThreads = 160;
template <int B>
__global__ void __launch_bounds__(kCombineThreads, B == 32 ? 1 : 12) attn_combine_kernel(const CombineArgs a) {
  extern __shared__ float s_w[];  // [nchunks] weights, then [nchunks] the chunks' sums of p
  float* s_l = s_w + a.nchunks;
  __shared__ float s_red[kCombineThreads / 32];
  __shared__ float s_m, s_inv;
  pdl_wait();
  const int t = blockIdx.x / a.heads, h = blockIdx.x % a.heads, tid = threadIdx.x, lane = tid & 31;
  const int nw = (int)(blockDim.x >> 5);
  const float sink2 = a.sink[h] * kLog2e;
  const float* ml = a.part_ml + ((size_t)t * a.nchunks * a.heads + h) * 2;  // chunk c at + c * heads * 2
  float mx = sink2;
  for (int c = tid; c < a.nchunks; c += blockDim.x) mx = fmaxf(mx, ml[(size_t)c * a.heads * 2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[tid >> 5] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = s_red[0];
    for (int w = 1; w < nw; ++w) m = fmaxf(m, s_red[w]);
    s_m = m;
  }
  __syncthreads();
  const float m = s_m;
  for (int c = tid; c < a.nchunks; c += blockDim.x) {
    const float mc = ml[(size_t)c * a.heads * 2], lc = ml[(size_t)c * a.heads * 2 + 1];
    const float w = mc == -INFINITY ? 0.f : exp2f(mc - m);
    s_w[c] = w;
    s_l[c] = lc;
  }
  __syncthreads();
  // thread tid sums dims 4 tid .. 4 tid + 3 over the chunks (D <= 576: one column group a thread),
  // 16 chunks' loads in flight; meanwhile the last thread -- past the columns -- sums the
  // denominator in chunk order
  const int64_t p = rope_row(a.pos[t], a.rope_rows);
  const float* po = a.part_o + ((size_t)t * a.nchunks * a.heads + h) * a.D;  // chunk c at + c * heads * D
  const size_t cstride = (size_t)a.heads * a.D;
  const int d = 4 * tid;
  const bool col = d < a.D;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (col) {
    for (int c0 = 0; c0 < a.nchunks; c0 += B) {
      float4 ov[B];
      float wv[B];
      // (loads unconditional, so all B are in flight: a chunk past the end or without keys --
      // whose partial was never written, but is allocated -- reads its slot and is skipped below)
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const int c = min(c0 + u, a.nchunks - 1);
        wv[u] = c0 + u < a.nchunks ? s_w[c] : 0.f;
        const uint4 r = ldg_stream(po + c * cstride + d);  // (volatile: issued here, in order)
        ov[u] = make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z), __uint_as_float(r.w));
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {  // (selects, not branches: a skipped chunk leaves v as it is)
        const bool on = wv[u] != 0.f;
        v[0] = on ? fmaf(ov[u].x, wv[u], v[0]) : v[0];
        v[1] = on ? fmaf(ov[u].y, wv[u], v[1]) : v[1];
        v[2] = on ? fmaf(ov[u].z, wv[u], v[2]) : v[2];
        v[3] = on ? fmaf(ov[u].w, wv[u], v[3]) : v[3];
      }
    }
  }
  if (tid == (int)blockDim.x - 1) {
    float l = exp2f(sink2 - m);
    for (int c = 0; c < a.nchunks; ++c)
      if (s_w[c] != 0.f) l = fmaf(s_l[c], s_w[c], l);
    s_inv = 1.0f / l;
  }
  __syncthreads();
  if (col) {
    const float inv = s_inv;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bf16r(v[i] * inv);
    if (d >= a.nope) {
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        const int j = (d + i - a.nope) >> 1;
        const float c = a.cos_sin[p * a.rope + j], s = a.cos_sin[p * a.rope + a.rope / 2 + j];
        const float e0 = __fadd_rn(__fmul_rn(v[i], c), __fmul_rn(v[i + 1], s));
        const float e1 = __fsub_rn(__fmul_rn(v[i + 1], c), __fmul_rn(v[i], s));
        v[i] = e0;
        v[i + 1] = e1;
      }
    }
    uint2 pk;
    pk.x = pack_bf16x2(v[0], v[1]);
    pk.y = pack_bf16x2(v[2], v[3]);
    *reinterpret_cast<uint2*>(a.xo + ((size_t)t * a.heads + h) * a.D + d) = pk;
  }
  pdl_launch();
}

}  // namespace dsv41
