// K2's attention core on the 5th-generation tensor cores (tcgen05, accumulators in TMEM):
// the split step of back.py:189-435 of the reference, for every head of a row at once.
//
// CTA = (row, chunk of the row's keys, 32-head tile), 12 warps:
//   warps 0-3  softmax + epilogue (each owns the TMEM lane quarter of its warp index),
//   warp  4    TMEM allocation and the MMA issue (one elected thread),
//   warps 5-11 producers: 64-key sub-blocks of FP8 records -> an f16 tile in shared memory.
// Per sub-block j (tile buffer j & 1, S buffer j & 1):
//   S^T[64 keys x NH heads]  = K_tile . Q^T      tcgen05.mma M=64 (keys), N=NH, K=D: A = the tile
//                                                (K-major), B = Q (K-major), D in TMEM;
//   softmax over keys (the threads holding keys 16 w + lane, lane < 16, of warp w) with the
//   running max per head;
//   O_sub^T[D dims x NH heads] = V_tile^T . P^T  M=128 (dims, in 128-dim blocks), N=NH, K=64
//                                                keys: A = the same tile read MN-major, B = P^T
//                                                (MN-major, written by the softmax threads) --
//                                                twice: P's f16 head, then its f16 tail (two
//                                                buffers; p keeps ~22 bits, as the averages over
//                                                thousands of keys need);
//   O_acc = O_acc * alpha + O_sub by the softmax threads (one fp32 FMA an element): the
//   tensor core's accumulation into TMEM truncates, so a chunk's thousands of keys are summed
//   8 MMA steps at a time in hardware and across sub-blocks in round-to-nearest fp32.
// The tile is stored as 8 x 16-byte core matrices: element (key, d) at
//   (key / 8) * (D / 8) * 128 + (d / 8) * 128 + (key % 8) * 16 + (d % 8) * 2,
// which is the K-major layout of the QK operand (leading offset 128 B, stride (D / 8) * 128 B)
// and the MN-major layout of the PV operand (dims contiguous: stride 128 B, leading (D / 8)
// * 128 B); Q likewise ([head][d]), P^T as [key group][head group][8 keys][8 heads].
// Synchronization: mbarriers (producer -> MMA: tile full; MMA -> producer: tile free;
// MMA -> softmax: S ready, PV done; softmax -> MMA: P ready), tcgen05.commit for MMA
// completion; every wait is bounded and a timeout sets an error word and unwinds.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int kTcKeys = 64;                // keys a sub-block
constexpr int kTcThreads = 384;            // 12 warps
constexpr int kTcProducers = 7 * 32;       // warps 5..11
constexpr uint32_t kTcWaitPolls = 1u << 24;

__device__ int g_tc_error;  // set when a bounded wait gave up (a kernel bug, never a peer)

// Build-time role timeline of CTA 0 (clock64 at each role's milestones of each sub-block), for
// pipeline tuning: compiled only with -DDSV41_TC_TRACE.
#ifdef DSV41_TC_TRACE
__device__ long long g_tc_trace[64 * 8];
#define TC_TRACE(j, slot)                                                  \
  do {                                                                     \
    if (blockIdx.x == 0 && (j) < 64) g_tc_trace[(j) * 8 + (slot)] = clock64(); \
  } while (0)
#else
#define TC_TRACE(j, slot) \
  do {                    \
  } while (0)
#endif

struct AttnTcArgs {
  AttnArgs a;   // shapes, pointers, chunking (chunk_keys a multiple of kTcKeys)
  int nh;       // heads a tile, padded to the MMA's N (16 or 32)
  int head_tiles;
};

template <int D>
struct TcSmem {
  static constexpr int kTileBytes = kTcKeys * D * 2;
  static constexpr int kQBytes = 32 * D * 2;
  static constexpr int kPBytes = kTcKeys * 32 * 2;
  static constexpr int kTile0 = 0;
  static constexpr int kTile1 = kTileBytes;
  static constexpr int kQ = 2 * kTileBytes;
  static constexpr int kP = kQ + kQBytes;
  static constexpr int kRed = kP + 2 * kPBytes;      // float [4 warps][64 heads]
  static constexpr int kM = kRed + 4 * 64 * 4;       // float [64]: the used max of each head
  static constexpr int kAlpha = kM + 64 * 4;         // float [64]: this sub-block's rescale
  static constexpr int kMeta = kAlpha + 64 * 4;      // [2 stages][64 keys]: record pointer, then 8 codes
  static constexpr int kBar = kMeta + 2 * 64 * 16;   // uint64 mbarriers
  static constexpr int kNumBars = 9;
  static constexpr int kMisc = kBar + kNumBars * 8;  // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
};

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);  // sm100 version, no swizzle
}
// kind::f16 instruction descriptor: f16 x f16 -> f32, A / B major (0 K, 1 MN), N, M
__device__ __forceinline__ uint32_t umma_idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the abort flag raised) when it gave up or another role already had.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  for (uint32_t it = 0; it < kTcWaitPolls; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 255) == 255 && *abort) return false;
  }
  *abort = 1;
  atomicExch(&g_tc_error, 1);
  return false;
}
// AND / OR of a predicate over the 128 softmax threads (named barrier 1): keeps their control
// flow uniform, so no thread leaves while the others wait at the barrier.
__device__ __forceinline__ bool softmax_all(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, 1, 128, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ bool softmax_any(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, 1, 128, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 consecutive TMEM columns of this thread's lane (32x32b shape), raw bits
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Core-matrix byte offset of element (row r, column c) of a [rows][C] tile.
template <int C>
__device__ __forceinline__ int core_off(int r, int c) {
  return (r >> 3) * (C / 8) * 128 + (c >> 3) * 128 + (r & 7) * 16 + (c & 7) * 2;
}

template <int NOPE>
__global__ void __launch_bounds__(kTcThreads, 1) attn_tc_kernel(const AttnTcArgs A) {
  constexpr int D = NOPE + 64;
  constexpr int DG = D / 8;                 // 16-byte core columns a row
  constexpr int NBLK = (D + 127) / 128;     // 128-dim PV blocks
  constexpr int CHUNKS = (NOPE + 128) / 16; // 16-byte chunks of a record's data
  using L = TcSmem<D>;
  extern __shared__ __align__(16) uint8_t smem[];
  const AttnArgs& a = A.a;
  const int NH = A.nh;
  const int ht = blockIdx.x % A.head_tiles;
  const int ch = (blockIdx.x / A.head_tiles) % a.nchunks;
  const int t = blockIdx.x / (A.head_tiles * a.nchunks);
  const int h0 = 32 * ht;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // bars: 0,1 tile full; 2,3 tile free; 4 S ready; 5 S consumed; 6 P ready; 7 PV done; 8 MMA drain
  auto bar = [&](int i) { return smem_u32(bars + i); };
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* m_sm = reinterpret_cast<float*>(smem + L::kM);
  float* a_sm = reinterpret_cast<float*>(smem + L::kAlpha);
  const uint32_t s_tile0 = smem_u32(smem + L::kTile0);
  const uint32_t s_q = smem_u32(smem + L::kQ), s_p = smem_u32(smem + L::kP);

  pdl_wait();
  const int kv = a.klen[t];
  const int k0 = ch * a.chunk_keys, k1 = min(k0 + a.chunk_keys, kv);
  const int nsub = k1 > k0 ? (k1 - k0 + kTcKeys - 1) / kTcKeys : 0;

  // ---- Q (f16, core layout [head][d]; heads past the rank's count are zero), barriers, TMEM
  for (int e = tid; e < NH * DG; e += blockDim.x) {
    const int h = e / DG, c = e % DG;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h0 + h < a.heads) {
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.heads + h0 + h) * D + 8 * c);
      v = make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
    }
    *reinterpret_cast<uint4*>(smem + L::kQ + core_off<D>(h, 8 * c)) = v;
  }
  if (tid == 0) {
    mbar_init(bar(0), 7);
    mbar_init(bar(1), 7);
    mbar_init(bar(2), 1);
    mbar_init(bar(3), 1);
    mbar_init(bar(4), 1);
    mbar_init(bar(5), 4);
    mbar_init(bar(6), 4);
    mbar_init(bar(7), 1);
    mbar_init(bar(8), 1);
    *abort = 0;
  }
  if (tid < 64) {
    m_sm[tid] = -INFINITY;
    a_sm[tid] = 0.f;
  }
  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  // TMEM columns: S^T at 0 (NH); O_acc block b at 32 + 32 b (NH); O_sub block b at 192 + 64 b
  // (2 NH: the head pass's columns, then the tail pass's)
  const uint32_t tm_s0 = tmem, tm_o = tmem + 32, tm_sub = tmem + 192;

  if (warp >= 5) {
    // ================= producers
    // Per tile: producer threads 0..63 resolve their key (record pointer, the 8 scale codes;
    // null = masked) into shared memory; then each producer warp converts units of 8 keys x 4
    // consecutive 16-byte chunks (lane: key 8 g + lane % 8, chunk 4 q + lane / 8), so a warp's
    // loads are whole 64-byte runs of 8 records. The next tile's record loads are issued before
    // this tile's conversion.
    static_assert(CHUNKS % 4 == 0, "records are whole 64-byte runs");
    const int ptid = tid - 5 * 32, wp = warp - 5;
    const int data_bytes = NOPE + 128;
    const uint8_t** meta_p = reinterpret_cast<const uint8_t**>(smem + L::kMeta);  // [2][64] then codes
    uint64_t* meta_c = reinterpret_cast<uint64_t*>(smem + L::kMeta + 2 * 64 * 8);
    constexpr int kUnits = (kTcKeys / 8) * (CHUNKS / 4);
    constexpr int kItems = (kUnits + kTcProducers / 32 - 1) / (kTcProducers / 32);
    auto item = [&](int i, int& key, int& c) {  // this lane's (key, chunk) of its i-th unit
      const int u = wp + (kTcProducers / 32) * i;
      key = 8 * (u % 8) + (lane & 7);
      c = 4 * (u / 8) + (lane >> 3);
      return u < kUnits;
    };
    auto resolve = [&](int j) {
      // thread ptid < 64: key ptid of tile j into stage j & 1
      const int k = k0 + j * kTcKeys + ptid;
      const uint8_t* dp = nullptr;
      uint64_t cw = 0;
      if (k < k1) {
        const int v = a.kt[(size_t)t * a.keys_ld + k];
        const bool comp = v < 0 && v != -1 && a.comp != nullptr;
        if (v >= 0 || comp) {
          const int sl = v & 0x7fffffff;
          const int blk = comp ? a.comp_blk : a.swa_blk;
          const uint8_t* page = (comp ? a.comp : a.swa) + (int64_t)(sl / blk) * (comp ? a.comp_stride : a.swa_stride);
          const int off = sl % blk;
          dp = page + (size_t)off * data_bytes;
          cw = *reinterpret_cast<const uint64_t*>(page + (size_t)blk * data_bytes + (size_t)off * 8);
        }
      }
      meta_p[(j & 1) * 64 + ptid] = dp;
      meta_c[(j & 1) * 64 + ptid] = cw;
    };
    auto issue = [&](int j, uint4 (&raw)[kItems]) {
      const int s = j & 1;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        int key, c;
        raw[i] = make_uint4(0, 0, 0, 0);
        if (item(i, key, c)) {
          const uint8_t* dp = meta_p[s * 64 + key];
          if (dp) raw[i] = ldg16(dp + 16 * c);
        }
      }
    };
    uint4 cur[kItems], nxt[kItems];
    if (nsub > 0) {
      if (ptid < 64) resolve(0);
      asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
      issue(0, cur);
    }
    for (int j = 0; j < nsub; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait(bar(2 + s), ((j >> 1) - 1) & 1, abort)) break;
      if (ptid == 0) TC_TRACE(j, 0);
      // the next tile's keys and record loads (its stage's metadata was last read two tiles ago)
      if (j + 1 < nsub) {
        // every producer is past tile j - 1's conversion (the metadata stage being rewritten)
        asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
        if (ptid < 64) resolve(j + 1);
        asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
        issue(j + 1, nxt);
      }
      uint8_t* tile = smem + (s ? L::kTile1 : L::kTile0);
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        int key, c;
        if (!item(i, key, c)) continue;
        const int b0 = 16 * c;
        const bool live = meta_p[s * 64 + key] != nullptr;
        if (b0 < NOPE) {
          uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
          if (live) {
            const int cd = (int)((meta_c[s * 64 + key] >> (8 * (b0 / 64))) & 0xff);
            const uint32_t w[4] = {cur[i].x, cur[i].y, cur[i].z, cur[i].w};
            uint32_t r[8];
            if (cd >= 113 && cd <= 134) {
              const uint32_t s1 = (uint32_t)(cd - 112) << 10;
              const uint32_t s2 = s1 | (s1 << 16);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                r[2 * q] = hmul2_bits(e4m3x2_f16(w[q] & 0xffff), s2);
                r[2 * q + 1] = hmul2_bits(e4m3x2_f16(w[q] >> 16), s2);
              }
            } else {
              const float sc = pow2c(cd);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float2 fl = e4m3x2_float2(w[q] & 0xffff), fh = e4m3x2_float2(w[q] >> 16);
                r[2 * q] = pack_f16x2(fl.x * sc, fl.y * sc);
                r[2 * q + 1] = pack_f16x2(fh.x * sc, fh.y * sc);
              }
            }
            o0 = make_uint4(r[0], r[1], r[2], r[3]);
            o1 = make_uint4(r[4], r[5], r[6], r[7]);
          }
          *reinterpret_cast<uint4*>(tile + core_off<D>(key, b0)) = o0;
          *reinterpret_cast<uint4*>(tile + core_off<D>(key, b0 + 8)) = o1;
        } else {
          uint4 o0 = make_uint4(0, 0, 0, 0);
          if (live)
            o0 = make_uint4(bf16x2_to_f16x2(cur[i].x), bf16x2_to_f16x2(cur[i].y), bf16x2_to_f16x2(cur[i].z),
                            bf16x2_to_f16x2(cur[i].w));
          *reinterpret_cast<uint4*>(tile + core_off<D>(key, NOPE + (b0 - NOPE) / 2)) = o0;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(s));
      if (ptid == 0) TC_TRACE(j, 1);
#pragma unroll
      for (int i = 0; i < kItems; ++i) cur[i] = nxt[i];
    }
  } else if (warp == 4) {
    // ================= MMA issue (one elected thread)
    // QK(j) needs tile j and the S buffer consumed by softmax(j - 1); PV(j) needs P(j). QK(j + 1)
    // goes out as soon as both are ready, so it runs under softmax(j).
    if (lane == 0) {
      const uint32_t id_qk = umma_idesc(64, NH, 0, 0);
      const uint32_t id_pv = umma_idesc(128, 2 * NH, 1, 1);
      auto issue_qk = [&](int j) {
        const uint32_t tile = s_tile0 + ((j & 1) ? L::kTileBytes : 0);
#pragma unroll 4
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16(tm_s0, umma_sdesc(tile + 256 * ks, 128, DG * 128), umma_sdesc(s_q + 256 * ks, 128, DG * 128), id_qk,
                   ks > 0);
        umma_commit(bar(4));
      };
      auto qk_ready = [&](int j) {  // tile j loaded and S consumed by softmax(j - 1)
        return mbar_try(bar(j & 1), (j >> 1) & 1) && (j == 0 || mbar_try(bar(5), (j - 1) & 1));
      };
      auto wait_qk = [&](int j) {
        return mbar_wait(bar(j & 1), (j >> 1) & 1, abort) && (j == 0 || mbar_wait(bar(5), (j - 1) & 1, abort));
      };
      bool ok = true;
      if (nsub > 0) ok = wait_qk(0);
      if (ok && nsub > 0) issue_qk(0);
      for (int j = 0; ok && j < nsub; ++j) {
        const int s = j & 1;
        bool qk_done = j + 1 >= nsub;
        if (!qk_done && qk_ready(j + 1)) {
          issue_qk(j + 1);
          qk_done = true;
        }
        if (!qk_done) {
          // wait for whichever comes first: P(j) (then PV), or QK(j + 1)'s inputs
          for (uint32_t it = 0; !qk_done && it < kTcWaitPolls; ++it) {
            if (mbar_try(bar(6), j & 1)) break;
            if (qk_ready(j + 1)) {
              issue_qk(j + 1);
              qk_done = true;
            }
          }
        }
        TC_TRACE(j, 2);
        ok = mbar_wait(bar(6), j & 1, abort);
        if (!ok) break;
        TC_TRACE(j, 3);
        tc_fence_after();
        // PV: B = P^T with the f16 head of p in columns 0 .. NH - 1, its tail in NH .. 2 NH - 1
        const uint32_t tile = s_tile0 + (s ? L::kTileBytes : 0);
#pragma unroll
        for (int b = 0; b < NBLK; ++b) {
          const int d0 = min(128 * b, D - 128);
#pragma unroll
          for (int ks = 0; ks < kTcKeys / 16; ++ks)
            umma_f16(tm_sub + 64 * b, umma_sdesc(tile + (d0 / 8) * 128 + 2 * ks * DG * 128, DG * 128, 128),
                     umma_sdesc(s_p + 2 * ks * (2 * NH / 8) * 128, (2 * NH / 8) * 128, 128), id_pv, ks > 0);
        }
        umma_commit(bar(2 + s));  // the tile is free
        umma_commit(bar(7));      // P^T free; O_sub holds sub-block j
        if (!qk_done) {
          ok = wait_qk(j + 1);
          if (!ok) break;
          issue_qk(j + 1);
        }
      }
      // drain: every issued MMA complete before the TMEM is freed (also after an abort)
      umma_commit(bar(8));
      mbar_wait(bar(8), 0, abort);
    }
  } else {
    // ================= softmax + epilogue (warps 0-3: TMEM lanes 32 w .. 32 w + 31)
    // Thread (warp w, lane < 16) holds key 16 w + lane of a sub-block (S^T rows of an M = 64
    // MMA sit on the first 16 lanes of each 32-lane quarter). Heads go 16 at a time; the
    // running max of each head and the rescale factors live in shared memory (the same for
    // every thread); each key thread keeps its own partial sums of p.
    const int key = 16 * warp + (lane & 15);
    const bool has_key = lane < 16;
    const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;
    const int ngroups = NH / 16;
    float l_part[32];
#pragma unroll
    for (int h = 0; h < 32; ++h) l_part[h] = 0.f;
    bool ok = true;
    // O_acc = O_acc * alpha + O_sub for this thread's lane (dim) in every block: sub-block
    // jj's PV result joins the sum at jj's max (alpha: the rescale the sub-block made)
    auto fold = [&](int jj) {
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (g >= ngroups) break;
          uint32_t vh[16], vt[16], va[16];
          const uint32_t sub = tm_sub + 64 * b + lane_addr + 16 * g, acc = tm_o + 32 * b + lane_addr + 16 * g;
          tmem_ld16(sub, vh);
          tmem_ld16(sub + NH, vt);
          if (jj > 0) tmem_ld16(acc, va);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float x = __uint_as_float(vh[q]) + __uint_as_float(vt[q]);  // head + tail pass
            va[q] = __float_as_uint(jj > 0 ? fmaf(__uint_as_float(va[q]), a_sm[16 * g + q], x) : x);
          }
          tmem_st16(acc, va);
        }
      }
      tmem_wait_st();
    };
    for (int j = 0; ok && j < nsub; ++j) {
      bool w_ok = mbar_wait(bar(4), j & 1, abort);
      ok = softmax_all(w_ok);
      if (!ok) break;
      if (tid == 0) TC_TRACE(j, 5);
      tc_fence_after();
      const uint32_t src = tm_s0 + lane_addr;
      float sv[32];
      {
        uint32_t v[32];
        tmem_ld16(src, *reinterpret_cast<uint32_t(*)[16]>(v));
        if (NH > 16) tmem_ld16(src + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        // S is in registers: QK(j + 1) may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(5));
        // the previous sub-block's PV result joins O_acc (O_sub and P^T are then free)
        if (j > 0) {
          ok = softmax_all(mbar_wait(bar(7), (j - 1) & 1, abort));
          if (!ok) break;
          tc_fence_after();
          fold(j - 1);
        }
        const int k = k0 + j * kTcKeys + key;
        bool valid = has_key && k < k1;
        if (valid) {
          const int kv_ = a.kt[(size_t)t * a.keys_ld + k];
          valid = kv_ != -1 && (kv_ >= 0 || a.comp != nullptr);
        }
#pragma unroll
        for (int q = 0; q < 32; ++q) sv[q] = (valid && q < NH) ? __uint_as_float(v[q]) * a.scale_log2 : -INFINITY;
      }
      // per-head max of the sub-block: 16 key lanes, then the 4 warps (through red)
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        float x = sv[q];
        x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
        x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
        x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
        x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
        if (lane == 0) red[warp * 32 + q] = x;
      }
      softmax_bar();  // red complete; every thread is past its fold (a_sm may change)
      if (tid == 0) TC_TRACE(j, 6);
      if (tid < NH) {
        const float bx = fmaxf(fmaxf(red[tid], red[32 + tid]), fmaxf(red[64 + tid], red[96 + tid]));
        const float mu = m_sm[tid];
        const float mn = fmaxf(mu, bx);
        a_sm[tid] = (mu == -INFINITY) ? 0.f : exp2f(mu - mn);
        m_sm[tid] = mn;
      }
      softmax_bar();
      // p = 2^(s - m) (<= 1) into P^T as an f16 head and its f16 tail (the two PV passes see
      // ~22 bits of p); this thread's partial sums of p
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int q = 0; q < 32; q += 2) {
        const float p0 = sv[q] == -INFINITY ? 0.f : exp2f(sv[q] - m_sm[q]);
        const float p1 = sv[q + 1] == -INFINITY ? 0.f : exp2f(sv[q + 1] - m_sm[q + 1]);
        l_part[q] = l_part[q] * a_sm[q] + p0;
        l_part[q + 1] = l_part[q + 1] * a_sm[q + 1] + p1;
        const __half ph0 = __float2half_rn(p0), ph1 = __float2half_rn(p1);
        hi[q / 2] = pack_f16x2(p0, p1);
        lo[q / 2] = pack_f16x2(p0 - __half2float(ph0), p1 - __half2float(ph1));
      }
      if (has_key) {
        // P^T [key group][column group][8 keys][8 columns]: head groups 0 .. NH / 8 - 1, then tail
#pragma unroll
        for (int hg = 0; hg < 4; ++hg) {
          if (8 * hg >= NH) break;
          const int row = (key >> 3) * (2 * NH / 8);
          *reinterpret_cast<uint4*>(smem + L::kP + (row + hg) * 128 + (key & 7) * 16) =
              make_uint4(hi[4 * hg], hi[4 * hg + 1], hi[4 * hg + 2], hi[4 * hg + 3]);
          *reinterpret_cast<uint4*>(smem + L::kP + (row + NH / 8 + hg) * 128 + (key & 7) * 16) =
              make_uint4(lo[4 * hg], lo[4 * hg + 1], lo[4 * hg + 2], lo[4 * hg + 3]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(6));
      if (tid == 0) TC_TRACE(j, 7);
    }
    // ---- epilogue: the last sub-block folded in, then O_acc^T and (m, l) of the chunk
    if (ok && nsub > 0) ok = softmax_all(mbar_wait(bar(7), (nsub - 1) & 1, abort));
    const size_t base = ((size_t)t * a.nchunks + ch) * a.heads + h0;
    const int nh_live = min(NH, a.heads - h0);
    if (ok && nsub > 0) {
      tc_fence_after();
      fold(nsub - 1);
      // l: the partial sums of the 64 key threads (16 lanes x 4 warps)
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        if (h >= NH) break;
        float x = has_key ? l_part[h] : 0.f;
        x += __shfl_xor_sync(0xffffffffu, x, 1);
        x += __shfl_xor_sync(0xffffffffu, x, 2);
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        if (lane == 0) red[warp * 32 + h] = x;
      }
      softmax_bar();
      if (tid < nh_live) {
        a.part_ml[(base + tid) * 2] = m_sm[tid];
        a.part_ml[(base + tid) * 2 + 1] = (red[tid] + red[32 + tid]) + (red[64 + tid] + red[96 + tid]);
      }
      const int dl = 32 * warp + lane;  // this thread's dim within a block
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
        const int d0 = min(128 * b, D - 128);
        const int d = d0 + dl;
        const bool own = d >= 128 * b;  // the overlapping last block writes only its new dims
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (g >= ngroups) break;
          uint32_t v[16];
          tmem_ld16(tm_o + 32 * b + lane_addr + 16 * g, v);
          tmem_wait_ld();
          if (own)
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (16 * g + q < nh_live) a.part_o[(base + 16 * g + q) * D + d] = __uint_as_float(v[q]);
        }
      }
    } else if (nsub == 0 && tid < nh_live) {
      a.part_ml[(base + tid) * 2] = -INFINITY;
      a.part_ml[(base + tid) * 2 + 1] = 0.f;
    }
  }
  // ---- teardown: every role done (a timed-out one unwound); free the TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  pdl_launch();
}

}  // namespace dsv41
