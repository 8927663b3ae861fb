// K2's MoE (stages/moe.py of the reference): router, routing, expert union, the MXFP4 routed
// experts, the shared expert's activation, and the top-k-order combine.
//
// Bit-exact contract for routing: the router logit of (row t, expert e) is the fp64 sum of
// the exact bf16 x bf16 products in a fixed order -- lane l of a warp owns k = 8 l + 256 i + j
// (j < 8), sums i-major / j-minor, then the 32 lanes fold by an xor-butterfly -- rounded once
// to fp32; scores use the deterministic fp64 softplus (detmath.cuh); the top-k takes the
// largest (score + bias), ties to the lower expert id.
//
// Routed experts (moe_tc.cuh) run on a one-time relayout of the MXFP4 weights into 256-row x
// 128-K tensor-core tiles (logged by the runner): tcgen05 block-scaled MMAs of e2m1 weights and
// e4m3 activations with their E8M0 codes.
#pragma once

#include "common.cuh"
#include "peer.cuh"
#include "detmath.cuh"

namespace dsv41 {

constexpr float kLimit = 10.0f;
constexpr float kRouteScale = 1.5f;

// ------------------------------------------------------------------ router
struct RouterArgs {
  int M, E, K;
  const __nv_bfloat16* x;     // [M, K] normed
  const __nv_bfloat16* gate;  // [E, K]
  float* logits;              // [M, E]
  int staged;                 // 1: the CTA's rows of x go to shared memory (2 K bytes a row and 1024 K)
};

// grid (E / 8, ceil(M / RPC)); warp w of CTA (ex, tg) = expert 8 ex + w, rows RPC tg .. + RPC - 1
// (RPC = 8, or 4 where a row group of 8 a CTA would leave the SMs short of CTAs: the sums are
// chains of dependent fp64 FMAs, so the kernel wants warps in flight more than rows a warp). A
// lane's weight loads go out ahead of their sums: all 16 batches of 256 K at once for 8 rows (the
// latency-bound small-M case), 4 at a time, double-buffered, for 4 rows (fewer registers, so three
// CTAs share an SM); the CTA's rows of x are staged once in shared memory when they fit. The
// arithmetic is the contract's, unchanged: per lane and row one fp64 chain over i, then j.
template <int RPC>
__global__ void __launch_bounds__(256, RPC == 4 ? 3 : 1) router_kernel(const RouterArgs a) {
  constexpr int kRouterChunk = RPC == 4 ? 4 : 16;  // 256-K iterations a batch of weight loads
  extern __shared__ __align__(16) uint8_t router_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  const bool live = e < a.E;
  const int iters = a.K / 256;
  const __nv_bfloat16* w = a.gate + (size_t)(live ? e : 0) * a.K + 8 * lane;
  uint4 wv[kRouterChunk], wn[kRouterChunk];
  auto load_chunk = [&](uint4 (&dst)[kRouterChunk], int i0) {
#pragma unroll
    for (int i = 0; i < kRouterChunk; ++i)
      dst[i] = (live && i0 + i < iters) ? ldg16(w + 256 * (i0 + i)) : make_uint4(0, 0, 0, 0);
  };
  load_chunk(wv, 0);  // the gate weights wait on nothing: stream them before the dependency wait
  if (kRouterChunk < 16) load_chunk(wn, kRouterChunk);
  pdl_wait();
  const int t0 = blockIdx.y * RPC, nt = min(RPC, a.M - t0);
  const __nv_bfloat16* xr = a.x + (size_t)t0 * a.K;
  if (a.staged) {
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(router_smem);
    for (int v = threadIdx.x; v < nt * (a.K / 8); v += blockDim.x)
      *reinterpret_cast<uint4*>(xs + 8 * (size_t)v) = *reinterpret_cast<const uint4*>(xr + 8 * (size_t)v);
    __syncthreads();
    xr = xs;
  }
  if (!live) return;
  // the rows' chains run side by side; each row's sum keeps the contract's order
  double acc[RPC];
#pragma unroll
  for (int r = 0; r < RPC; ++r) acc[r] = 0.0;
  for (int i0 = 0; i0 < iters; i0 += kRouterChunk) {
#pragma unroll
    for (int i = 0; i < kRouterChunk; ++i) {
      if (i0 + i >= iters) break;
      const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
      double wd[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        wd[j] = (double)__uint_as_float((j & 1) ? (ww[j >> 1] & 0xffff0000u) : (ww[j >> 1] << 16));
#pragma unroll
      for (int r = 0; r < RPC; ++r) {
        if (r < nt) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xr + (size_t)r * a.K + 8 * lane + 256 * (i0 + i));
          const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t xb = (j & 1) ? (xx[j >> 1] & 0xffff0000u) : (xx[j >> 1] << 16);
            acc[r] = __fma_rn((double)__uint_as_float(xb), wd[j], acc[r]);
          }
        }
      }
    }
    // the next batch (loaded a batch ahead when double-buffered); then the one after it
    if (kRouterChunk < 16) {
#pragma unroll
      for (int i = 0; i < kRouterChunk; ++i) wv[i] = wn[i];
      if (i0 + 2 * kRouterChunk < iters) load_chunk(wn, i0 + 2 * kRouterChunk);
    } else if (i0 + kRouterChunk < iters) {
      load_chunk(wv, i0 + kRouterChunk);
    }
  }
#pragma unroll
  for (int r = 0; r < RPC; ++r) {
    const double s = warp_sum_d(acc[r]);
    if (lane == 0 && r < nt) a.logits[(size_t)(t0 + r) * a.E + e] = (float)s;
  }
  pdl_launch();
}

// ------------------------------------------------------------------ routing
struct RouteArgs {
  int M, E, topk;
  int softmax;          // 1: softmax top-k; 0: sqrtsoftplus + bias
  const float* logits;  // [M, E]
  const float* bias;    // [E] fp32 (sqrtsoftplus)
  int32_t* ids;         // [M, topk], top-k order
  float* wts;           // [M, topk]
};

// The selection value (NaN -> -inf) and the original score of (row t, expert e) into the row's
// shared-memory arrays.
__device__ __forceinline__ void route_score_one(const RouteArgs& a, int t, int e, float* s_val, float* s_orig) {
  const float l = a.logits[(size_t)t * a.E + e];
  if (a.softmax) {
    s_val[e] = isnan(l) ? -INFINITY : l;
    s_orig[e] = l;
  } else {
    const float sc = route_score(l);
    s_orig[e] = isnan(sc) ? 0.f : sc;
    const float v = __fadd_rn(sc, a.bias[e]);
    s_val[e] = isnan(v) ? -INFINITY : v;
  }
}

// One warp selects row t's top-k from its scores (experts e = lane + 32 i, E <= 512) and writes
// ids / wts; lane k < topk also leaves its id in s_ids[k] when s_ids is given.
__device__ __forceinline__ void route_select(const RouteArgs& a, int t, const float* s_val, const float* s_orig,
                                             int lane, int* s_ids) {
  constexpr int kMaxPer = 16;  // E <= 512
  const int per = (a.E + 31) / 32;
  // (every loop over a lane's values runs to the compile-time kMaxPer, guarded by i < per, so
  // val / orig stay in registers instead of a local-memory frame indexed at run time)
  float val[kMaxPer], orig[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    const bool in = i < per && e < a.E;
    val[i] = in ? s_val[e] : -INFINITY;
    orig[i] = in ? s_orig[e] : 0.f;
  }
  float my_w = 0.f;
  int my_id = 0;
  float total = 0.f;
  double tot = 0.0, mine = 0.0;  // softmax: the picks' exps summed in pick order; lane k's own exp
  float first = 0.f;
  for (int k = 0; k < a.topk; ++k) {
    // the best (value, lowest id) of the lane, then of the warp
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (i < per && e < a.E && (val[i] > bv || (val[i] == bv && e < bi))) {
        bv = val[i];
        bi = e;
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, d);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // the winner's original value; retire it as NaN, which no comparison selects
    float ow = 0.f;
    if ((bi & 31) == lane) {
      const int i = bi >> 5;
#pragma unroll
      for (int q = 0; q < kMaxPer; ++q)
        if (q == i) {
          ow = orig[q];
          val[q] = __int_as_float(0x7fc00000);
        }
    }
    ow = __shfl_sync(0xffffffffu, ow, bi & 31);
    if (a.softmax) {
      if (k == 0) first = ow;
      const double ex = det_exp(__dadd_rn((double)ow, -(double)first));
      tot = __dadd_rn(tot, ex);
      if (lane == k) mine = ex;
    } else {
      total = __fadd_rn(total, ow);
    }
    if (lane == k) {
      my_w = ow;
      my_id = bi;
    }
  }
  if (a.softmax) {
    if (lane < a.topk) {
      a.ids[(size_t)t * a.topk + lane] = my_id;
      a.wts[(size_t)t * a.topk + lane] = (float)__ddiv_rn(mine, tot);
    }
  } else if (lane < a.topk) {
    const float scale = __fdiv_rn(kRouteScale, fmaxf(total, 1e-20f));
    a.ids[(size_t)t * a.topk + lane] = my_id;
    a.wts[(size_t)t * a.topk + lane] = __fmul_rn(my_w, scale);
  }
  if (s_ids != nullptr && lane < a.topk) s_ids[lane] = my_id;
}

// A CTA of 256 threads a row: the scores in parallel (one expert a thread, two when E > 256),
// then warp 0 selects the top-k.
__global__ void __launch_bounds__(256) route_kernel(const RouteArgs a) {
  __shared__ float s_val[512], s_orig[512];
  const int t = blockIdx.x;
  pdl_wait();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) route_score_one(a, t, e, s_val, s_orig);
  __syncthreads();
  if (threadIdx.x < 32) route_select(a, t, s_val, s_orig, threadIdx.x, nullptr);
  pdl_launch();
}

// ------------------------------------------------------------------ expert union and picks
struct PlanArgs {
  int M, E, topk;
  const int32_t* ids;  // [M, topk]
  int32_t* n_u;        // [1]
  int32_t* u_expert;   // [E]: the union's experts, ascending
  int32_t* u_off;      // [E + 1]: each union expert's first pick in ``picks``
  int32_t* picks;      // [M * topk]: natural pick indices t * topk + k, grouped by expert, ascending
};

// One CTA of 512 threads (E <= 512, M topk <= kPlanMaxPicks): counts by shared-memory atomics,
// a block-wide inclusive scan of (picks, union flag) an expert, then each pick's rank among the
// earlier picks of its expert from the ids staged in shared memory.
constexpr int kPlanMaxPicks = 48 * 32;
// The plan of the P = M topk picks whose ids sit in s_ids; s_ids filled and cnt zeroed by the
// caller before a barrier. 512 threads.
__device__ __forceinline__ void plan_picks(const PlanArgs& a, const int* s_ids, int* cnt, int* s_off, int* s_uf) {
  const int P = a.M * a.topk, tid = threadIdx.x;
  for (int p = tid; p < P; p += blockDim.x) atomicAdd(&cnt[s_ids[p]], 1);
  __syncthreads();
  // inclusive scans (Hillis-Steele) of the counts and of the union flags over experts
  const int c = tid < a.E ? cnt[tid] : 0;
  s_off[tid] = c;
  s_uf[tid] = c > 0;
  __syncthreads();
  for (int d = 1; d < 512; d <<= 1) {
    const int vo = tid >= d ? s_off[tid - d] : 0, vu = tid >= d ? s_uf[tid - d] : 0;
    __syncthreads();
    s_off[tid] += vo;
    s_uf[tid] += vu;
    __syncthreads();
  }
  const int first = s_off[tid] - c;  // this expert's first slot in picks
  if (tid < a.E && c > 0) {
    const int u = s_uf[tid] - 1;
    a.u_expert[u] = tid;
    a.u_off[u] = first;
  }
  if (tid == 0) {
    const int nu = s_uf[511];
    a.u_off[nu] = s_off[511];
    *a.n_u = nu;
  }
  cnt[tid] = first;  // reused: the experts' first slots
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    const int e = s_ids[p];
    int before = 0;
    for (int q = 0; q < p; ++q) before += (s_ids[q] == e);
    a.picks[cnt[e] + before] = p;
  }
}

__global__ void __launch_bounds__(512) moe_plan_kernel(const PlanArgs a) {
  __shared__ int cnt[512], s_off[512], s_uf[512];
  __shared__ int s_ids[kPlanMaxPicks];
  pdl_wait();
  const int P = a.M * a.topk, tid = threadIdx.x;
  cnt[tid] = 0;
  for (int p = tid; p < P; p += blockDim.x) s_ids[p] = a.ids[p];
  __syncthreads();
  plan_picks(a, s_ids, cnt, s_off, s_uf);
  pdl_launch();
}

// Routing and the plan in one CTA of 512 threads for M <= kRoutePlanRows (E <= 512, topk <= 32):
// every row's scores in parallel, warp t selects row t's top-k (ids into shared memory as well
// as global), then the plan of those picks. Saves the small-M decode one launch boundary; the
// arithmetic is route_kernel's and moe_plan_kernel's.
constexpr int kRoutePlanRows = 8;
__global__ void __launch_bounds__(512) route_plan_kernel(const RouteArgs r, const PlanArgs a) {
  __shared__ float s_val[kRoutePlanRows * 512], s_orig[kRoutePlanRows * 512];
  __shared__ int cnt[512], s_off[512], s_uf[512];
  __shared__ int s_ids[kRoutePlanRows * 32];
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5;
  cnt[tid] = 0;
  // M E <= 8 x 512: a thread's (up to) 8 scores unrolled, so their loads and math overlap
#pragma unroll
  for (int j = 0; j < kRoutePlanRows; ++j) {
    const int i = tid + 512 * j;
    if (i < r.M * r.E) {
      const int t = i / r.E;
      route_score_one(r, t, i - t * r.E, s_val + 512 * t, s_orig + 512 * t);
    }
  }
  __syncthreads();
  if (warp < r.M) route_select(r, warp, s_val + 512 * warp, s_orig + 512 * warp, tid & 31, s_ids + warp * r.topk);
  __syncthreads();
  plan_picks(a, s_ids, cnt, s_off, s_uf);
  pdl_launch();
}

// ------------------------------------------------------------------ routed expert plan
// The host's plan of one routed-expert GEMM (gate/up or down); expert_tc_kernel (moe_tc.cuh)
// runs it.
struct ExpertArgs {
  int M, topk, N, K;   // N rows of the expert matrix (2 I for gate/up, H for down), K
  int kslices, ks_len;  // K slices (ks_len a multiple of 128)
  int row_groups;       // 256-row tiles of N
  int max_units;        // union slots (min(E, M topk))
  const uint8_t* w;     // tensor-core tiles [E][N/256][K/128][256][64]
  const uint8_t* ws;    // codes [E][N/256][K/128][1024]
  const uint8_t* x;     // e4m3 [rows, K] activations: token rows (gate/up) or pick rows (down)
  const uint8_t* xs;    // codes [rows, K / 32]
  int x_by_pick;        // 1: x rows are natural pick indices; 0: token rows (pick / topk)
  const int32_t* n_u;
  const int32_t* u_expert;
  const int32_t* u_off;
  const int32_t* picks;
  float* out;           // [kslices][M * topk][N] fp32 partials, by natural pick index
};

// ------------------------------------------------------------------ routed activation
struct ExpertActArgs {
  int P, I, kslices;   // picks, intermediate width, gate/up K slices
  const float* part;   // [kslices][P][2 I]
  uint8_t* mid;        // [P, I] e4m3 (aiter rule)
  uint8_t* mids;       // [P, I / 32]
};

// v = bf16(gc sigmoid(gc) uc), gc = min(g, 10), uc = clamp(u, +-10); aiter MXFP8 a 32.
// Thread = 8 consecutive columns; 4 threads a group.
__global__ void expert_act_kernel(const ExpertActArgs a) {
  pdl_wait();
  const int groups8 = a.I / 8;
  const int total = a.P * groups8, padded = (total + 31) / 32 * 32;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < padded; i += gridDim.x * blockDim.x) {
    const bool live = i < total;
    const int p = live ? i / groups8 : 0, c = live ? (i % groups8) * 8 : 0;
    float v[8], gs[8], us[8];
    const float* row = a.part + (size_t)p * 2 * a.I;
    sum_slices8(row + c, (size_t)a.P * 2 * a.I, live ? a.kslices : 0, gs);
    sum_slices8(row + a.I + c, (size_t)a.P * 2 * a.I, live ? a.kslices : 0, us);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float gc = fminf(gs[q], kLimit), uc = fminf(fmaxf(us[q], -kLimit), kLimit);
      v[q] = bf16r(gc * (1.0f / (1.0f + expf(-gc))) * uc);
    }
    float amax = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(v[q]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const int code = mx_code_aiter(amax);
    const float mul = mx_mul(code);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t b = e4m3_byte(v[q] * mul);
      if (q < 4) w0 |= b << (8 * q);
      else w1 |= b << (8 * (q - 4));
    }
    if (!live) continue;
    *reinterpret_cast<uint2*>(a.mid + (size_t)p * a.I + c) = make_uint2(w0, w1);
    if ((c & 31) == 0) a.mids[(size_t)p * (a.I / 32) + c / 32] = (uint8_t)code;
  }
  pdl_launch();
}

// ------------------------------------------------------------------ shared expert activation
struct SharedActArgs {
  int M, SI, kslices;
  const float* part;      // [kslices][M][2 SI] (gate rows, then up rows)
  uint8_t* smq;           // [M, SI] e4m3 (vLLM rule)
  uint8_t* smqs;          // [M, SI / 32]
  __nv_bfloat16* smx;     // [M, SI] dequantized (the down GEMV's input)
};

// g = bf16(min(bf16(h_g), 10)), u = clamp(bf16(h_u), +-10), act = bf16(g / (1 + e^-g)),
// v = bf16(act u) (moe.py:502-507); vLLM MXFP8 a 32.
__global__ void shared_act_kernel(const SharedActArgs a) {
  pdl_wait();
  const int groups8 = a.SI / 8;
  const int total = a.M * groups8, padded = (total + 31) / 32 * 32;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < padded; i += gridDim.x * blockDim.x) {
    const bool live = i < total;
    const int t = live ? i / groups8 : 0, c = live ? (i % groups8) * 8 : 0;
    float v[8], gs[8], us[8];
    const float* row = a.part + (size_t)t * 2 * a.SI;
    sum_slices8(row + c, (size_t)a.M * 2 * a.SI, live ? a.kslices : 0, gs);
    sum_slices8(row + a.SI + c, (size_t)a.M * 2 * a.SI, live ? a.kslices : 0, us);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float gq = bf16r(fminf(bf16r(gs[q]), kLimit));
      const float uq = fminf(fmaxf(bf16r(us[q]), -kLimit), kLimit);
      const float act = bf16r(gq / (1.0f + expf(-gq)));
      v[q] = bf16r(act * uq);
    }
    float amax = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(v[q]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const int code = mx_code_vllm(amax);
    const float mul = mx_mul(code), sc = pow2c(code);
    uint32_t w0 = 0, w1 = 0, d[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint8_t b = e4m3_byte(v[q] * mul);
      if (q < 4) w0 |= (uint32_t)b << (8 * q);
      else w1 |= (uint32_t)b << (8 * (q - 4));
      d[q >> 1] |= (uint32_t)f2bfbits(e4m3_float(b) * sc) << (16 * (q & 1));
    }
    if (!live) continue;
    *reinterpret_cast<uint2*>(a.smq + (size_t)t * a.SI + c) = make_uint2(w0, w1);
    if ((c & 31) == 0) a.smqs[(size_t)t * (a.SI / 32) + c / 32] = (uint8_t)code;
    *reinterpret_cast<uint4*>(a.smx + (size_t)t * a.SI + c) = make_uint4(d[0], d[1], d[2], d[3]);
  }
  pdl_launch();
}

// ------------------------------------------------------------------ combine
struct CombineMoeArgs {
  int M, H, topk, routed_slices, shared_slices;
  const float* routed;   // [routed_slices][M * topk][H] down partials by natural pick
  const float* wts;      // [M, topk]
  const float* shared;   // [shared_slices][M][H] shared down partials
  __nv_bfloat16* out;    // [M, H]: bf16(routed + shared)
  PeerLL x;              // x.peers set: out is this rank's partial of the MoE all-reduce into x.reduced
};

// routed = bf16(routed + bf16(y_k w_k)) in top-k order; out = bf16(routed + bf16(shared)). A
// thread = 8 consecutive columns of a row; slice by slice, the loads of 8 picks are in flight
// together (each pick's slices still added in slice order).
__global__ void moe_combine_kernel(const CombineMoeArgs a) {
  pdl_wait();
  int xfail = 1;
  const uint32_t e = a.x.peers ? ll_begin(a.x, &xfail) : 0u;
  const int g8 = a.H / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.M * g8; i += gridDim.x * blockDim.x) {
    const int t = i / g8, n = (i % g8) * 8;
    float routed[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < a.topk; k0 += 8) {
      float y[8][8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int q = 0; q < 8; ++q) y[k][q] = 0.f;
      for (int s = 0; s < a.routed_slices; ++s) {
        float4 u[8][2];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k0 + k < a.topk) {
            const float4* p = reinterpret_cast<const float4*>(
                a.routed + ((size_t)s * a.M * a.topk + (size_t)t * a.topk + k0 + k) * a.H + n);
            u[k][0] = p[0];
            u[k][1] = p[1];
          }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k0 + k < a.topk) {
            y[k][0] += u[k][0].x; y[k][1] += u[k][0].y; y[k][2] += u[k][0].z; y[k][3] += u[k][0].w;
            y[k][4] += u[k][1].x; y[k][5] += u[k][1].y; y[k][6] += u[k][1].z; y[k][7] += u[k][1].w;
          }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k0 + k < a.topk) {
          const float w = a.wts[(size_t)t * a.topk + k0 + k];
#pragma unroll
          for (int q = 0; q < 8; ++q) routed[q] = bf16r(routed[q] + bf16r(y[k][q] * w));
        }
    }
    float sh[8];
    sum_slices8(a.shared + (size_t)t * a.H + n, (size_t)a.M * a.H, a.shared_slices, sh);
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = pack_bf16x2(routed[2 * q] + bf16r(sh[2 * q]), routed[2 * q + 1] + bf16r(sh[2 * q + 1]));
    *reinterpret_cast<uint4*>(a.out + (size_t)t * a.H + n) = make_uint4(o[0], o[1], o[2], o[3]);
    if (!xfail) ll_push(a.x, e, i, o);
  }
  // tp > 1: the MoE all-reduce of this kernel's groups (peer.cuh's fused exchange)
  if (a.x.peers) {
    if (!xfail)
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.M * g8; i += gridDim.x * blockDim.x) {
        uint32_t o[4];
        if (!ll_reduce(a.x, e, i, o)) break;
        reinterpret_cast<uint4*>(a.x.reduced)[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    ll_end(a.x, e);
  }
  pdl_launch();
}

}  // namespace dsv41
