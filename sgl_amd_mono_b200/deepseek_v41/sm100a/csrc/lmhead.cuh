// The LM head and greedy selection of a decode / verify step: logits = x . W^T (W the bf16
// vocab-parallel head, [V, K] row-major, read in place), the argmax of every row (ties to the
// lower token id) fused into the GEMV's epilogue, and DSpark's greedy acceptance of a verify
// block (the roles of SGLang's logits processor and its greedy verify, spec.py:807-833 and
// draft.py:173-195 of the reference).
//
// Tensor cores: mma.sync m16n8k16 bf16 -> fp32, vocab rows as the A operand, tokens as B. A
// lane streams 16 contiguous bytes of its rows g and g + 8 per 32-K sub-chunk (ld.global.nc,
// no L1 allocation) and reads the same 16 bytes' K positions of its token g from shared
// memory; the 8 values serve two mma steps whose K slots {2t, 2t + 1, 2t + 8, 2t + 9} map to
// the same physical positions in A and B, so neither operand needs a permutation. x streams
// through shared memory in 128-K chunks (cp.async, double-buffered; rows padded to 160
// elements so the 16-byte reads are conflict-free) while every CTA keeps its 128 vocab rows'
// accumulators in registers over the whole K.
//
// Argmax: a row's candidates are packed into one int64 key -- the order-preserving 32 bits of
// the fp32 logit (NaN lowest, -0 as +0), then 0xFFFFFFFF - id -- biased into signed order, so
// the largest key is the largest logit and, among equal logits, the lowest id. Warps reduce
// by shuffles, the CTA through shared memory, and one atomicMax a token and CTA publishes
// it. Vocab-parallel ranks max-reduce their keys the same way (they carry the global id).
#pragma once

#include <climits>

#include "common.cuh"

namespace dsv41 {

constexpr int kLmRows = 128;   // vocab rows a CTA (8 warps x 16)
constexpr int kLmChunk = 128;  // K a pipeline stage
constexpr int kLmLd = kLmChunk + 32;

struct LmHeadArgs {
  const __nv_bfloat16* w;  // [V, K]
  const __nv_bfloat16* x;  // [M, K]
  float* logits;           // optional [M, V]
  long long* best;         // [M] keys
  int M, V, K, vbase;      // vbase: the global id of this rank's first row
};

__device__ __forceinline__ long long argmax_key(float v, uint32_t id) {
  uint32_t o = 0u;
  if (!isnan(v)) {
    const uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
    o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  const unsigned long long k = ((unsigned long long)o << 32) | (0xFFFFFFFFu - id);
  return (long long)(k ^ 0x8000000000000000ULL);
}

__device__ __forceinline__ float argmax_key_value(long long key, uint32_t* id) {
  const unsigned long long k = (unsigned long long)key ^ 0x8000000000000000ULL;
  *id = 0xFFFFFFFFu - (uint32_t)k;
  const uint32_t o = (uint32_t)(k >> 32);
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

__global__ void argmax_init_kernel(const LmHeadArgs a) {
  pdl_wait();
  for (int i = threadIdx.x; i < a.M; i += blockDim.x) a.best[i] = LLONG_MIN;
  pdl_launch();
}

template <int NT>
__global__ void __launch_bounds__(256, 2) lmhead_kernel(const LmHeadArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int MP = 8 * NT;
  __shared__ long long s_best[8][MP];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem);  // [2][MP][kLmLd]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * kLmRows + 16 * warp;
  const __nv_bfloat16* pa = a.w + (size_t)min(row0 + g, a.V - 1) * a.K + 8 * t;
  const __nv_bfloat16* pb = a.w + (size_t)min(row0 + g + 8, a.V - 1) * a.K + 8 * t;
  const int nchunks = a.K / kLmChunk;
  uint4 wa[4], wb[4], na[4], nb[4];
  // the weights wait on nothing: the first chunk streams before the dependency wait
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    wa[c] = ldg_stream(pa + 32 * c);
    wb[c] = ldg_stream(pb + 32 * c);
  }
  pdl_wait();
  // pad rows (tokens M .. MP - 1) of both buffers are zero; cp.async fills the rest
  for (int i = threadIdx.x; i < 2 * (MP - a.M) * (kLmLd / 8); i += blockDim.x) {
    const int buf = i / ((MP - a.M) * (kLmLd / 8)), r = i % ((MP - a.M) * (kLmLd / 8));
    const int m = a.M + r / (kLmLd / 8), q = r % (kLmLd / 8);
    *reinterpret_cast<uint4*>(xs + (buf * MP + m) * kLmLd + 8 * q) = make_uint4(0, 0, 0, 0);
  }
  auto stage_x = [&](int kc, int buf) {
    const uint32_t base = smem_u32(xs + buf * MP * kLmLd);
    for (int i = threadIdx.x; i < a.M * (kLmChunk / 8); i += blockDim.x) {
      const int m = i / (kLmChunk / 8), q = i % (kLmChunk / 8);
      cp_async16_stream(base + (m * kLmLd + 8 * q) * 2, a.x + (size_t)m * a.K + kc * kLmChunk + 8 * q);
    }
    cp_async_commit();
  };
  stage_x(0, 0);
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int kc = 0; kc < nchunks; ++kc) {
    const int cur = kc & 1;
    if (kc + 1 < nchunks) {
      stage_x(kc + 1, cur ^ 1);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        na[c] = ldg_stream(pa + (kc + 1) * kLmChunk + 32 * c);
        nb[c] = ldg_stream(pb + (kc + 1) * kLmChunk + 32 * c);
      }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t xb = smem_u32(xs + cur * MP * kLmLd) + (g * kLmLd + 8 * t) * 2;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4 X = lds16(xb + (8 * n * kLmLd + 32 * c) * 2);
        mma_bf16(acc[n], wa[c].x, wb[c].x, wa[c].y, wb[c].y, X.x, X.y);
        mma_bf16(acc[n], wa[c].z, wb[c].z, wa[c].w, wb[c].w, X.z, X.w);
      }
    }
    __syncthreads();  // the next stage overwrites this buffer
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      wa[c] = na[c];
      wb[c] = nb[c];
    }
  }
  // ---- epilogue: optional logits, then the argmax keys
  const int ida = row0 + g, idb = row0 + g + 8;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int tok = 8 * n + 2 * t + j;
      const float va = acc[n][j], vb = acc[n][2 + j];
      if (a.logits && tok < a.M) {
        if (ida < a.V) a.logits[(size_t)tok * a.V + ida] = va;
        if (idb < a.V) a.logits[(size_t)tok * a.V + idb] = vb;
      }
      long long k = LLONG_MIN;
      if (ida < a.V) k = argmax_key(va, (uint32_t)(a.vbase + ida));
      if (idb < a.V) k = max(k, argmax_key(vb, (uint32_t)(a.vbase + idb)));
      k = max(k, __shfl_xor_sync(0xffffffffu, k, 4));
      k = max(k, __shfl_xor_sync(0xffffffffu, k, 8));
      k = max(k, __shfl_xor_sync(0xffffffffu, k, 16));
      if (g == 0) s_best[warp][tok] = k;
    }
  }
  __syncthreads();
  for (int tok = threadIdx.x; tok < a.M; tok += blockDim.x) {
    long long k = s_best[0][tok];
#pragma unroll
    for (int w = 1; w < 8; ++w) k = max(k, s_best[w][tok]);
    atomicMax(a.best + tok, k);
  }
  pdl_launch();
}

// Keys -> ids and logits; with draft tokens, DSpark's greedy acceptance of each request's
// block of per_req verify rows: row j of a request scored the token after draft[j], so
// draft[j + 1] is accepted while it equals row j's argmax; accept[r] = the accepted count and
// next_tok[r] = the target's token after them.
struct ArgmaxArgs {
  const long long* best;
  int M;
  int32_t* ids;
  float* vals;
  const int32_t* draft;
  int per_req;
  int32_t* accept;
  int32_t* next_tok;
};

__global__ void argmax_decode_kernel(const ArgmaxArgs a) {
  pdl_wait();
  for (int i = threadIdx.x; i < a.M; i += blockDim.x) {
    uint32_t id;
    const float v = argmax_key_value(a.best[i], &id);
    if (a.ids) a.ids[i] = (int32_t)id;
    if (a.vals) a.vals[i] = v;
  }
  if (a.draft) {
    __syncthreads();
    for (int r = threadIdx.x; r < a.M / a.per_req; r += blockDim.x) {
      const int r0 = r * a.per_req;
      int n = 0;
      uint32_t id;
      while (n + 1 < a.per_req) {
        argmax_key_value(a.best[r0 + n], &id);
        if ((int32_t)id != a.draft[r0 + n + 1]) break;
        ++n;
      }
      argmax_key_value(a.best[r0 + n], &id);
      a.accept[r] = n;
      a.next_tok[r] = (int32_t)id;
    }
  }
  pdl_launch();
}

}  // namespace dsv41
