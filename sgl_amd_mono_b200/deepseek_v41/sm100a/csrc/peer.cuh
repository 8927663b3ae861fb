// The TP all-reduce over peer memory: every rank pushes its bf16 partial into a slot of every
// rank's exchange region (NVLink stores through CUDA IPC mappings), raises a per-CTA arrival
// flag there, waits for every rank's flag in its own region, and sums the slots in rank order
// in fp32 before one rounding to bf16 -- the reference's one-shot push and fixed-order sum
// (seam.py:391-408, moe.py:1247-1268, ops.py:269-277), with its mailbox / guard / epoch roles
// (sync.py:29-197, guard.py:103-224, epoch.py:52-85) done by this layout:
//
//   [0, 256)      guard words (uint32): 0 the exchange sequence (epoch), 1 CTAs done with the
//                 current exchange, 3 the site (1-based) of the first wait on this GPU that ran
//                 past its deadline, 4 set when a wait saw another rank's failure flag, 5 set
//                 by the fault-injection hook (this rank stalled: no push, no flag)
//   [256, 288)    failure flags: rank r writes word r of every rank's region when it fails
//   [512, +4 * kPeerMaxTp * kArBlocks)   arrival flags [src rank][CTA], the sequence number
//   [kPeerDataOff, ...)  data slots [parity][src rank][cap] bf16
//   then LL slots [parity][src rank][cap / 2] 8-byte words {bf16x2, epoch}: the fused exchange
//
// The fused exchange (the wo_b epilogue and the MoE combine, ll_* below) needs no arrival flags:
// every 8-byte word carries its exchange's epoch beside two bf16 values, written by one 8-byte
// store, so a reader that sees the epoch sees the data (the reference's {value, tag} mailbox,
// sync.py:109-188). A producing thread stores its values into slot [e & 1][rank] of every rank's
// region, then polls its own region's slots of every rank for the same elements and sums them in
// rank order. Parity reuse is safe as above: a rank writes exchange e + 2 only after its kernel of
// exchange e + 1 completed, which needed every rank's pushes of e + 1, each made after that
// rank's kernel of exchange e (its reads included) completed.
//
// Sequence numbers only grow, so a waiter accepts any flag >= its own; the data of exchange e
// lives in parity e & 1, which no rank can overwrite before every rank has finished reading it
// (a rank reaches exchange e + 2 only after every rank raised its flag for e + 1, which each
// does after finishing e). A wait gives up after ``deadline_ns`` of %globaltimer: it records
// its site, raises this rank's failure flag in every region and returns -- a device-side
// failure is a status the host reads (dsv41_peer_status), never a fault. Failures are sticky:
// an exchange that starts on a failed region (any error word, or any rank's failure flag
// raised in it) does nothing.
#pragma once

#include "common.cuh"

namespace dsv41 {

constexpr int kPeerMaxTp = 8;
constexpr int kArBlocks = 128;     // CTAs an exchange at most (all resident: one an SM)
constexpr int kGuardSeq = 0, kGuardDone = 1, kErrDeadline = 3, kErrPeer = 4, kErrFault = 5;
constexpr int kFailOff = 256;
constexpr int kArriveOff = 512;
constexpr int kPeerDataOff = 8192;

__host__ __device__ inline int64_t peer_region_bytes(int tp, int64_t cap) {
  return kPeerDataOff + 2LL * tp * cap * 2 + 2LL * tp * cap * 4;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct AllReduceArgs {
  int n, tp, rank, nblk;        // n bf16 elements (a multiple of 8)
  const int64_t* peers;         // [tp] each rank's region as mapped in this process
  int64_t cap;                  // elements a data slot holds (a multiple of 8, >= n)
  const __nv_bfloat16* src;     // this rank's partial [n]
  __nv_bfloat16* dst;           // the reduced [n]
  int64_t deadline_ns;
  int site, skip_push;          // skip_push: the fault-injection hook (publish nothing)
};

__device__ __forceinline__ uint32_t* peer_words(int64_t base) { return reinterpret_cast<uint32_t*>(base); }
__device__ __forceinline__ uint32_t* arrive_flag(int64_t base, int src, int b) {
  return reinterpret_cast<uint32_t*>(base + kArriveOff) + src * kArBlocks + b;
}
__device__ __forceinline__ uint4* peer_slot(int64_t base, int par, int tp, int src, int64_t cap) {
  return reinterpret_cast<uint4*>(base + kPeerDataOff + ((int64_t)(par * tp + src) * cap) * 2);
}

// Wait until ``flag`` reaches epoch e, another rank fails, or the deadline passes (every
// 64 polls the failure flags and the clock are checked). Returns true on arrival.
__device__ inline bool wait_arrival(const AllReduceArgs& a, const uint32_t* flag, uint32_t e) {
  const int64_t me = a.peers[a.rank];
  uint64_t t0 = 0;
  for (uint32_t it = 1; it != 0; ++it) {
    if ((int)(ld_acquire_sys(flag) - e) >= 0) return true;
    if ((it & 63) != 0) continue;
    bool failed = false;
    for (int r = 0; r < a.tp; ++r)
      if (r != a.rank) failed |= ld_acquire_sys(peer_words(me + kFailOff) + r) != 0;
    if (failed) {
      atomicExch(peer_words(me) + kErrPeer, 1u);
      return false;
    }
    const uint64_t now = global_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > (uint64_t)a.deadline_ns) {
      atomicCAS(peer_words(me) + kErrDeadline, 0u, (uint32_t)a.site);
      for (int r = 0; r < a.tp; ++r) st_release_sys(peer_words(a.peers[r] + kFailOff) + a.rank, 1u);
      return false;
    }
  }
  atomicCAS(peer_words(me) + kErrDeadline, 0u, (uint32_t)a.site);  // 2^32 polls: give up too
  return false;
}

__global__ void __launch_bounds__(256) allreduce_kernel(const AllReduceArgs a) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  pdl_wait();
  const int tid = threadIdx.x, b = blockIdx.x;
  const int64_t me = a.peers[a.rank];
  uint32_t* words = peer_words(me);
  if (tid == 0) {
    s_epoch = __ldcg(words + kGuardSeq) + 1u;
    // sticky: this rank's earlier failure, or a failure flag another rank raised here
    uint32_t f = __ldcg(words + kErrDeadline) | __ldcg(words + kErrPeer) | __ldcg(words + kErrFault);
    for (int r = 0; r < a.tp; ++r) f |= __ldcg(peer_words(me + kFailOff) + r);
    s_fail = f != 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = (int)(e & 1u);
  const int nv = a.n / 8;
  const int per = (nv + a.nblk - 1) / a.nblk;
  const int v0 = min(nv, b * per), v1 = min(nv, v0 + per);
  if (!s_fail && a.skip_push) {
    // the fault-injection hook: this rank stalls -- it publishes nothing and raises no flag,
    // so the other ranks' waits run out -- and its exchange fails
    if (tid == 0) atomicExch(words + kErrFault, 1u);
  } else if (!s_fail) {
    const uint4* src = reinterpret_cast<const uint4*>(a.src);
    for (int v = v0 + tid; v < v1; v += blockDim.x) {
      const uint4 x = src[v];
      for (int r = 0; r < a.tp; ++r) peer_slot(a.peers[r], par, a.tp, a.rank, a.cap)[v] = x;
    }
    __threadfence_system();
    __syncthreads();
    if (tid < a.tp) st_release_sys(arrive_flag(a.peers[tid], a.rank, b), e);
    if (tid < a.tp && !wait_arrival(a, arrive_flag(me, tid, b), e)) atomicOr(&s_fail, 1);
    __syncthreads();
    if (!s_fail) {
      uint4* dst = reinterpret_cast<uint4*>(a.dst);
      for (int v = v0 + tid; v < v1; v += blockDim.x) {
        float acc[8];
        for (int r = 0; r < a.tp; ++r) {
          const uint4 x = __ldcg(peer_slot(me, par, a.tp, r, a.cap) + v);
          const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = __uint_as_float(w[q] << 16), hi = __uint_as_float(w[q] & 0xFFFF0000u);
            acc[2 * q] = r ? acc[2 * q] + lo : lo;
            acc[2 * q + 1] = r ? acc[2 * q + 1] + hi : hi;
          }
        }
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
        dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // the exchange's end: the last CTA advances the sequence
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(words + kGuardDone, 1u) == (uint32_t)(a.nblk - 1)) {
      atomicExch(words + kGuardDone, 0u);
      __threadfence();
      atomicExch(words + kGuardSeq, e);
    }
  }
  pdl_launch();
}

// ------------------------------------------------------------------ the fused (LL) exchange
struct PeerLL {
  const int64_t* peers;   // [tp] regions as mapped here; null: no exchange (tp 1, or a split phase)
  int tp, rank, site, skip;  // skip: the fault-injection hook (publish nothing at this site)
  int64_t cap;            // elements a slot holds (a multiple of 8, >= the exchange's elements)
  int64_t deadline_ns;
  __nv_bfloat16* reduced; // [n] the rank-order sum
};

__device__ __forceinline__ uint64_t* ll_slot(int64_t base, int par, int tp, int src, int64_t cap) {
  return reinterpret_cast<uint64_t*>(base + kPeerDataOff + 4LL * tp * cap) + (int64_t)(par * tp + src) * (cap / 2);
}
__device__ __forceinline__ void st_ll2(uint64_t* p, uint32_t w0, uint32_t w1, uint32_t e) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(((uint64_t)e << 32) | w0),
               "l"(((uint64_t)e << 32) | w1)
               : "memory");
}
__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// The CTA's view of the exchange: its epoch, and whether the region has failed (sticky: any
// error word or any rank's failure flag). Thread 0 reads, the block shares (a barrier inside).
__device__ inline uint32_t ll_begin(const PeerLL& x, int* fail) {
  __shared__ uint32_t s_e;
  __shared__ int s_f;
  if (threadIdx.x == 0) {
    const int64_t me = x.peers[x.rank];
    uint32_t* words = peer_words(me);
    s_e = __ldcg(words + kGuardSeq) + 1u;
    uint32_t f = __ldcg(words + kErrDeadline) | __ldcg(words + kErrPeer) | __ldcg(words + kErrFault);
    for (int r = 0; r < x.tp; ++r) f |= __ldcg(peer_words(me + kFailOff) + r);
    s_f = f != 0;
    if (!s_f && x.skip) atomicExch(words + kErrFault, 1u);  // the hook: this rank stalls
  }
  __syncthreads();
  *fail = s_f || x.skip;
  return s_e;
}

// This thread's 8 values (4 bf16x2 words) of element group i8 into slot [e & 1][rank] of every
// rank's region.
__device__ __forceinline__ void ll_push(const PeerLL& x, uint32_t e, int64_t i8, const uint32_t (&w)[4]) {
  const int par = (int)(e & 1u);
  for (int r = 0; r < x.tp; ++r) {
    uint64_t* p = ll_slot(x.peers[r], par, x.tp, x.rank, x.cap) + 4 * i8;
    st_ll2(p, w[0], w[1], e);
    st_ll2(p + 2, w[2], w[3], e);
  }
}

// Every rank's values of element group i8 from this rank's region, summed in rank order in fp32
// and rounded once to bf16, into o. Each wait gives up at the deadline or on another rank's
// failure flag (checked every 64 polls): it records the site, raises this rank's failure flag in
// every region and returns false.
__device__ inline bool ll_reduce(const PeerLL& x, uint32_t e, int64_t i8, uint32_t (&o)[4]) {
  const int par = (int)(e & 1u);
  const int64_t me = x.peers[x.rank];
  float acc[8];
  uint64_t t0 = 0;
  for (int r = 0; r < x.tp; ++r) {
    const uint64_t* p = ll_slot(me, par, x.tp, r, x.cap) + 4 * i8;
    uint64_t v[4];
    for (uint32_t it = 1;; ++it) {
      ld_ll2(p, v[0], v[1]);
      ld_ll2(p + 2, v[2], v[3]);
      if ((uint32_t)(v[0] >> 32) == e && (uint32_t)(v[1] >> 32) == e && (uint32_t)(v[2] >> 32) == e &&
          (uint32_t)(v[3] >> 32) == e)
        break;
      if ((it & 63) != 0) continue;
      // another rank failed (or another thread of this rank gave up: its flag is raised here too)
      bool failed = false;
      for (int q = 0; q < x.tp; ++q)
        if (q != x.rank) failed |= ld_acquire_sys(peer_words(me + kFailOff) + q) != 0;
      if (failed) {
        atomicExch(peer_words(me) + kErrPeer, 1u);
        return false;
      }
      if (ld_acquire_sys(peer_words(me + kFailOff) + x.rank) != 0) return false;
      const uint64_t now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > (uint64_t)x.deadline_ns || it == 0xffffffc0u) {
        atomicCAS(peer_words(me) + kErrDeadline, 0u, (uint32_t)x.site);
        for (int q = 0; q < x.tp; ++q) st_release_sys(peer_words(x.peers[q] + kFailOff) + x.rank, 1u);
        return false;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t d = (uint32_t)v[q];
      const float lo = __uint_as_float(d << 16), hi = __uint_as_float(d & 0xFFFF0000u);
      acc[2 * q] = r ? acc[2 * q] + lo : lo;
      acc[2 * q + 1] = r ? acc[2 * q + 1] + hi : hi;
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
  return true;
}

// The exchange's end: the last CTA of the grid advances the sequence (after every CTA's reads).
__device__ inline void ll_end(const PeerLL& x, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* words = peer_words(x.peers[x.rank]);
    __threadfence();
    if (atomicAdd(words + kGuardDone, 1u) == gridDim.x - 1) {
      atomicExch(words + kGuardDone, 0u);
      __threadfence();
      atomicExch(words + kGuardSeq, e);
    }
  }
}

// The standalone LL exchange (dsv41_allreduce_ll): dst = bf16(rank-order sum of every rank's src),
// a thread a group of 8 elements; every thread pushes all its groups before it waits for any.
__global__ void __launch_bounds__(256) allreduce_ll_kernel(const PeerLL x, const __nv_bfloat16* src, int n) {
  pdl_wait();
  int fail = 0;
  const uint32_t e = ll_begin(x, &fail);
  const int groups = n / 8;
  if (!fail) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < groups; i += gridDim.x * blockDim.x) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      ll_push(x, e, i, w);
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < groups; i += gridDim.x * blockDim.x) {
      uint32_t o[4];
      if (!ll_reduce(x, e, i, o)) break;
      reinterpret_cast<uint4*>(x.reduced)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  ll_end(x, e);
  pdl_launch();
}

// ------------------------------------------------------------------ row-parallel attention's exchanges
// With rows split over the ranks (rank r owns rows [r mr, min(M, (r + 1) mr))), every rank runs the
// attention of its rows for all heads. Two all-to-alls of bf16 blocks (one row's hl x D values of
// one rank's hl heads) over the LL slots carry what it needs:
//   mode 0 (queries): rank s sends peer p, for each of p's rows i, src[p mr + i][0 .. hl)[D] (its
//     heads' queries); p stores it at dst[i][s hl .. (s + 1) hl)[D] (all heads, rank-major);
//   mode 1 (outputs): rank s sends peer p, for each of its own rows i, src[i][p hl .. (p + 1) hl)[D];
//     p stores it at dst[s mr + i][0 .. hl)[D] (every row, its own heads).
// Block i from rank s is slot [e & 1][s] of the receiver at 8-value group i hl D / 8. Each thread
// pushes all its groups before it waits for any. Every rank must own at least one row (M >= tp):
// then every exchange waits on every rank, which keeps the slot parity reuse safe.
struct A2AArgs {
  int mode, M, mr, hl, D;
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
};

// Rank src's group i8 of this exchange from this rank's region, once its epoch is e (the waits and
// failure handling of ll_reduce).
__device__ inline bool ll_fetch(const PeerLL& x, uint32_t e, int src, int64_t i8, uint32_t (&o)[4]) {
  const int par = (int)(e & 1u);
  const int64_t me = x.peers[x.rank];
  const uint64_t* p = ll_slot(me, par, x.tp, src, x.cap) + 4 * i8;
  uint64_t v[4];
  uint64_t t0 = 0;
  for (uint32_t it = 1;; ++it) {
    ld_ll2(p, v[0], v[1]);
    ld_ll2(p + 2, v[2], v[3]);
    if ((uint32_t)(v[0] >> 32) == e && (uint32_t)(v[1] >> 32) == e && (uint32_t)(v[2] >> 32) == e &&
        (uint32_t)(v[3] >> 32) == e)
      break;
    if ((it & 63) != 0) continue;
    bool failed = false;
    for (int q = 0; q < x.tp; ++q)
      if (q != x.rank) failed |= ld_acquire_sys(peer_words(me + kFailOff) + q) != 0;
    if (failed) {
      atomicExch(peer_words(me) + kErrPeer, 1u);
      return false;
    }
    if (ld_acquire_sys(peer_words(me + kFailOff) + x.rank) != 0) return false;
    const uint64_t now = global_ns();
    if (t0 == 0) {
      t0 = now;
    } else if (now - t0 > (uint64_t)x.deadline_ns || it == 0xffffffc0u) {
      atomicCAS(peer_words(me) + kErrDeadline, 0u, (uint32_t)x.site);
      for (int q = 0; q < x.tp; ++q) st_release_sys(peer_words(x.peers[q] + kFailOff) + x.rank, 1u);
      return false;
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = (uint32_t)v[q];
  return true;
}

__global__ void __launch_bounds__(256) ll_a2a_kernel(const PeerLL x, const A2AArgs a) {
  pdl_wait();
  int fail = 0;
  const uint32_t e = ll_begin(x, &fail);
  const int par = (int)(e & 1u);
  const int G = a.hl * a.D / 8;  // 8-value groups a block
  auto rows_of = [&](int r) { return max(0, min(a.M, (r + 1) * a.mr) - r * a.mr); };
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nthr = (int64_t)gridDim.x * blockDim.x;
  const int hall = x.tp * a.hl;
  if (!fail) {
    for (int p = 0; p < x.tp; ++p) {
      const int64_t total = (int64_t)(a.mode == 0 ? rows_of(p) : rows_of(x.rank)) * G;
      uint64_t* slot = ll_slot(x.peers[p], par, x.tp, x.rank, x.cap);
      for (int64_t q = t0; q < total; q += nthr) {
        const int i = (int)(q / G), g = (int)(q % G);
        const __nv_bfloat16* s = a.mode == 0 ? a.src + ((size_t)(p * a.mr + i) * a.hl) * a.D + 8 * g
                                             : a.src + ((size_t)i * hall + p * a.hl) * a.D + 8 * g;
        const uint4 v = *reinterpret_cast<const uint4*>(s);
        st_ll2(slot + 4 * q, v.x, v.y, e);
        st_ll2(slot + 4 * q + 2, v.z, v.w, e);
      }
    }
    for (int s = 0; s < x.tp && !fail; ++s) {
      const int64_t total = (int64_t)(a.mode == 0 ? rows_of(x.rank) : rows_of(s)) * G;
      for (int64_t q = t0; q < total; q += nthr) {
        const int i = (int)(q / G), g = (int)(q % G);
        uint32_t o[4];
        if (!ll_fetch(x, e, s, q, o)) {
          fail = 1;
          break;
        }
        __nv_bfloat16* d = a.mode == 0 ? a.dst + ((size_t)i * hall + s * a.hl) * a.D + 8 * g
                                       : a.dst + ((size_t)(s * a.mr + i) * a.hl) * a.D + 8 * g;
        *reinterpret_cast<uint4*>(d) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  ll_end(x, e);
  pdl_launch();
}

// out = bf16(sum over ranks in rank order of parts[r]), fp32 accumulation: the reduction step
// of the NCCL variant (an all-gather of the partials, then this), bit-identical to the
// in-kernel exchange.
struct RankSumArgs {
  int n, tp;
  const __nv_bfloat16* parts;  // [tp][n]
  __nv_bfloat16* out;
};

__global__ void rank_sum_kernel(const RankSumArgs a) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
    float s = bf2f(a.parts[i]);
    for (int r = 1; r < a.tp; ++r) s += bf2f(a.parts[(size_t)r * a.n + i]);
    a.out[i] = __float2bfloat16_rn(s);
  }
  pdl_launch();
}

}  // namespace dsv41
