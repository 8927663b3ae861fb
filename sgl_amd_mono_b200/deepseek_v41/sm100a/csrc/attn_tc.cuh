// K2's attention core on the 5th-generation tensor cores (tcgen05, accumulators in TMEM):
// the split step of back.py:189-435 of the reference, for every head of a row at once.
//
// CTA = (row, chunk of the row's keys, 32-head tile), 12 warps:
//   warps 0-3  softmax + epilogue (each owns the TMEM lane quarter of its warp index),
//   warp  4    TMEM allocation and the MMA issue (one elected thread),
//   warps 5-11 producers: 48-key sub-blocks of FP8 records -> an f16 tile in shared memory, in a
//              ring of 3 tiles (a 64-key tile is 73.7 KB and only two fit beside Q and P; three
//              48-key tiles let the producer run a tile further ahead of the QK -> softmax -> PV
//              chain).
// A row's two head tiles run as a cluster of two CTAs (PAIR) that share every key tile: each
// converts half of the tile's keys into its own shared memory and copies that half into the
// peer's with one cp.async.bulk, counted on the peer's tile-full mbarrier.
// Per sub-block j (tile j % 3; S and P buffers j & 1):
//   S^T[64 keys x NH heads] = K_tile . Q^T        tcgen05.mma M=64 (keys), N=NH, K=D: A = the tile
//                                                (K-major; its rows 48 .. 63 read whatever follows
//                                                the tile in shared memory, and those keys are
//                                                masked), B = Q (K-major), D in TMEM;
//   softmax over keys (the threads holding keys 16 w + lane, lane < 16, of warp w) against a
//   per-head reference max that moves only when a score passes it by more than 2^8 (then O is
//   rescaled in TMEM);
//   O^T[D dims x 2 NH] += V_tile^T . P^T          M=128 (dims, in 128-dim blocks), N=2 NH, K=48
//                                                keys: A = the same tile read MN-major, B = P^T
//                                                (MN-major, written by the softmax threads) whose
//                                                columns are p's f16 head (0 .. NH - 1), then its
//                                                f16 tail: p keeps ~22 bits, and head and tail
//                                                accumulate in separate TMEM columns, summed in
//                                                fp32 by the epilogue (the tensor core's fp32
//                                                accumulation truncates: a tail added into the
//                                                head's columns lost its precision).
// The tile and Q are stored in the 128-byte-swizzle layout: [64-dim chunk][8-row group][8 rows x
// 128 B] atoms of 1 KB, the 16-byte chunk q of row r at q ^ r (sw_off). For the tile this is at
// once the K-major operand of the QK (8-row groups 1 KB apart, a K step 32 B into the rows) and
// the MN-major operand V^T of the PV (64-dim atoms (kTcKeys / 8) KB apart, 8-key groups 1 KB
// apart); with the unswizzled core-matrix layout each MMA fetched its operands 128 B at a time.
// P^T is [key group][head group][8 keys][8 heads] (unswizzled, MN-major).
// Synchronization: mbarriers (producer -> MMA: tile full; MMA -> producer: tile free;
// MMA -> softmax: S ready, PV done; softmax -> MMA: S consumed, P ready), tcgen05.commit for MMA
// completion; every wait is bounded and a timeout sets an error word and unwinds.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int kTcKeys = 48;                // keys a sub-block (the QK's M = 64 rows: 16 padded)
constexpr int kTcStages = 3;               // key tiles in flight
constexpr int kTcThreads = 384;            // 12 warps
constexpr int kTcProducers = 7 * 32;       // warps 5..11
constexpr uint32_t kTcWaitPolls = 1u << 24;
constexpr float kTcSlack = 8.f;            // log2 headroom of p over the reference max

__device__ int g_tc_error;  // set when a bounded wait gave up (a kernel bug, never a peer)

// Build-time role timeline of CTA 0 (clock64 at each role's milestones of each sub-block), for
// pipeline tuning: compiled only with -DDSV41_TC_TRACE.
#ifdef DSV41_TC_TRACE
__device__ long long g_tc_trace[64 * 16];
#define TC_TRACE(j, slot)                                                  \
  do {                                                                     \
    if (blockIdx.x == 0 && (j) < 64) g_tc_trace[(j) * 16 + (slot)] = clock64(); \
  } while (0)
// every CTA's [start, end) in %globaltimer ns and its SM
__device__ long long g_tc_span[4096 * 3];
#define TC_SPAN(slot)                                                                       \
  do {                                                                                      \
    if (threadIdx.x == 0 && blockIdx.x < 4096) {                                            \
      unsigned long long ns;                                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns));                                \
      g_tc_span[blockIdx.x * 3 + (slot)] = (long long)ns;                                   \
      if ((slot) == 0) {                                                                    \
        unsigned sm;                                                                        \
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));                                     \
        g_tc_span[blockIdx.x * 3 + 2] = sm;                                                 \
      }                                                                                     \
    }                                                                                       \
  } while (0)
#else
#define TC_SPAN(slot) \
  do {                \
  } while (0)
#define TC_TRACE(j, slot) \
  do {                    \
  } while (0)
#endif

struct AttnTcArgs {
  AttnArgs a;   // shapes, pointers, chunking (chunk_keys a multiple of kTcKeys)
  int nh;       // heads a tile, padded to the MMA's N (16 or 32)
  int head_tiles;
};

// Shared memory of a CTA: TS f16 key tiles, Q, P, the softmax's reductions, the key metadata and
// (the staged producer, STG > 0) STG staging stages of raw FP8 records.
template <int D, int TS = kTcStages, int STG = 0>
struct TcSmem {
  static constexpr int kTileBytes = kTcKeys * D * 2;
  static constexpr int kQBytes = 32 * D * 2;
  static constexpr int kPBytes = kTcKeys * 32 * 2;
  static constexpr int kRecBytes = D - 64 + 128;       // a record's data row (nope e4m3, rope bf16)
  static constexpr int kStageBytes = kTcKeys * kRecBytes;
  static constexpr int kTile0 = 0;                      // TS tiles
  static constexpr int kQ = TS * kTileBytes;            // (the QK's padded rows of the last tile read Q)
  static constexpr int kP = kQ + kQBytes;
  static constexpr int kRed = kP + 4 * kPBytes;      // float [4 warps][64 heads]
  static constexpr int kM = kRed + 4 * 64 * 4;       // float [64]: the used max of each head
  static constexpr int kAlpha = kM + 64 * 4;         // float [64]: the rescale of the reference max
  static constexpr int kMetaStages = 3;
  static constexpr int kMeta = kAlpha + 64 * 4;      // [3 stages][64 keys]: record pointer, then 8 codes
  static constexpr int kStage = kMeta + kMetaStages * 64 * 16;  // STG staging stages (16-byte aligned)
  static constexpr int kBar = kStage + STG * kStageBytes;       // uint64 mbarriers
  static constexpr int kNumBars = 2 * TS + 9 + 2 * STG;
  static constexpr int kMisc = kBar + kNumBars * 8;  // tmem base, abort flag, then [STG] live-key masks
  static constexpr int kBytes = kMisc + 32 + 1024;  // + slack to align the base to 1 KB
  static_assert(kStage % 16 == 0 && kStageBytes % 16 == 0, "bulk copy destinations are 16-byte aligned");
};
constexpr int kTcBulkStages = 2;  // the staged producer: f16 tiles in flight
constexpr int kTcStaging = 2;     // and FP8 record staging stages

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);  // sm100 version, no swizzle
}
// The same with the 128-byte swizzle (layout type 2): K-major, sbo = the 8-row group stride (lbo
// unused); MN-major, lbo = the stride between 64-element (128-byte) atoms along MN, sbo = the
// 8-row group stride along K.
__device__ __forceinline__ uint64_t umma_sdesc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return umma_sdesc(addr, lbo, sbo) | ((uint64_t)2 << 61);
}
// Byte offset of element (row, d) of a [ROWS][D] f16 operand in the swizzled layout the tile and Q
// use: [64-dim chunk][8-row group][8 rows x 128 B] atoms of 1 KB, the 16-byte chunk q of row r at
// q ^ r (the 128-byte swizzle). It is at once the K-major operand of the QK and, for the tile, the
// MN-major operand V^T of the PV.
template <int ROWS>
__device__ __forceinline__ int sw_off(int row, int d) {
  return (d >> 6) * (ROWS / 8) * 1024 + (row >> 3) * 1024 + (row & 7) * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4) +
         (d & 7) * 2;
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
// Non-blocking tests (test_wait never suspends the thread, where a failed try_wait may for a while):
// for a thread that polls several barriers and must act on whichever completes first.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.test_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_test_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same with cluster-scope acquire: the arrivals come from the other CTA of a pair too (its
// producers' remote stores, its MMA completions).
__device__ __forceinline__ bool mbar_try_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, volatile int* abort) {
  for (uint32_t it = 0; it < kTcWaitPolls; ++it) {
    if (mbar_try_cl(bar, parity)) return true;
    if ((it & 255) == 255 && *abort) return false;
  }
  *abort = 1;
  atomicExch(&g_tc_error, 1);
  return false;
}
// Cluster plumbing for a CTA pair: the peer's address of a shared-memory location, both CTAs'
// barrier.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// An arrival on the peer's mbarrier that also raises its expected transaction bytes by tx.
__device__ __forceinline__ void mbar_arrive_tx_remote(uint32_t cluster_addr, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
               "r"(tx)
               : "memory");
}
// bytes of this CTA's shared memory into the peer's (cluster addresses dst, bar), counted on the
// peer's mbarrier bar as they land (a plain copy: no multicast)
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "r"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// the MMAs' completion arrives on the mbarrier at this offset in both CTAs of the pair
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
// AND of a predicate over the 224 producer threads (named barrier 2), for the same reason.
__device__ __forceinline__ bool producers_all(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, 2, %2, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v), "n"(kTcProducers) : "memory");
  return r != 0;
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
// One arrival on a CTA-local mbarrier that also raises its expected transaction bytes.
__device__ __forceinline__ void tc_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// bytes of global memory into this CTA's shared memory, counted on its mbarrier bar as they land
// (a plain bulk copy, no multicast; addresses and size multiples of 16 bytes)
__device__ __forceinline__ void tc_bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// The maximum of v over the warp's 32 lanes, in every lane (one instruction on sm_100a).
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

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

// 2^x by the SFU's ex2 instruction (PTX ex2.approx.ftz.f32: about 2 ulp; results below 2^-126
// flush to 0, far under what the f16 head/tail of p can hold).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// {lo, hi} -> f16x2 bits (round to nearest), one instruction.
__device__ __forceinline__ uint32_t cvt_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}


// PAIR: the row's two 32-head tiles run as a cluster of two CTAs that share every key tile:
// each CTA's producers gather and convert half of the tile's keys (key groups 3 r .. 3 r + 2 of
// CTA rank r) into its own tile, then one thread copies that half into the peer's; a tile is full
// after this CTA's 7 producer warps and the peer's copy (an arrival raising the expected bytes,
// then the bytes) arrived, and free after both CTAs' PV finished with it (2 commit arrivals).
//
// BULK (lone CTAs): the producer stages each tile's raw records in shared memory first. One warp
// reads the tile's key-table entries, finds the runs of consecutive slots of one page (a row's
// window keys are whole runs), and fetches each run with one cp.async.bulk into a staging stage
// (kTcStaging stages, counted on the stage's mbarrier); six warps convert the staged FP8 records
// into the f16 tile (kTcBulkStages tiles) with the same arithmetic as the gathering producers, so
// all three producers give the MMAs the same tiles and the outputs the same bits.
template <int NOPE, bool PAIR, bool BULK = false>
__global__ void __launch_bounds__(kTcThreads, 1) attn_tc_kernel(const AttnTcArgs A) {
  static_assert(!(PAIR && BULK), "the staged producer runs lone CTAs");
  constexpr int D = NOPE + 64;
  constexpr int DG = D / 8;                 // 16-byte core columns a row
  constexpr int NBLK = (D + 127) / 128;     // 128-dim PV blocks
  constexpr int CHUNKS = (NOPE + 128) / 16; // 16-byte chunks of a record's data
  constexpr int TS = BULK ? kTcBulkStages : kTcStages;  // f16 key tiles in flight
  constexpr int STG = BULK ? kTcStaging : 0;            // raw record staging stages
  using L = TcSmem<D, TS, STG>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);  // swizzle atoms: 1 KB
  const AttnArgs& a = A.a;
  const int NH = A.nh;
  const int ht = blockIdx.x % A.head_tiles;
  const int ch = (blockIdx.x / A.head_tiles) % a.nchunks;
  const int t = blockIdx.x / (A.head_tiles * a.nchunks);
  const int h0 = 32 * ht;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // bars: TS tile full; TS tile free; 2 S ready; 2 S consumed; 2 P ready; 2 PV done; 1 MMA
  // drain; STG staging full; STG staging empty (S and P pairs by the sub-block's parity)
  auto bar = [&](int i) { return smem_u32(bars + i); };
  // tile stage ts = j % TS (parity (j / TS) & 1); S and P buffers s = j & 1 (parity (j >> 1) & 1)
  auto b_full = [&](int ts) { return bar(ts); };                     // producers -> MMA
  auto b_free = [&](int ts) { return bar(TS + ts); };                // PV done with the tile
  auto b_sready = [&](int sb) { return bar(2 * TS + sb); };          // QK -> softmax
  auto b_scons = [&](int sb) { return bar(2 * TS + 2 + sb); };       // softmax holds S
  auto b_pready = [&](int sb) { return bar(2 * TS + 4 + sb); };      // softmax -> PV
  auto b_pvdone = [&](int sb) { return bar(2 * TS + 6 + sb); };      // PV(j) complete
  const uint32_t b_drain = bar(2 * TS + 8);
  auto b_sfull = [&](int st) { return bar(2 * TS + 9 + st); };       // staging: records landed
  auto b_sempty = [&](int st) { return bar(2 * TS + 9 + STG + st); };  // staging: converted
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* m_sm = reinterpret_cast<float*>(smem + L::kM);
  float* a_sm = reinterpret_cast<float*>(smem + L::kAlpha);
  const uint32_t s_tile0 = smem_u32(smem + L::kTile0);
  const uint32_t s_q = smem_u32(smem + L::kQ), s_p = smem_u32(smem + L::kP);

  pdl_wait();
  TC_SPAN(0);
  if (tid == 0) TC_TRACE(62, 0);  // timeline row 62: start, setup done; row 63: the epilogue
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
    *reinterpret_cast<uint4*>(smem + L::kQ + sw_off<32>(h, 8 * c)) = v;
  }
  if (tid == 0) {
    for (int ts = 0; ts < TS; ++ts) {
      // the producer warps (+ the peer's copy of its half; the staged producer's 6 converters)
      mbar_init(b_full(ts), BULK ? 6 : PAIR ? 8 : 7);
      mbar_init(b_free(ts), PAIR ? 2 : 1);
    }
    for (int st = 0; st < STG; ++st) {
      mbar_init(b_sfull(st), 1);   // the copy warp's arrival with the stage's bytes
      mbar_init(b_sempty(st), 6);  // the converters
    }
    for (int sb = 0; sb < 2; ++sb) {
      mbar_init(b_sready(sb), 1);
      mbar_init(b_scons(sb), 4);
      mbar_init(b_pready(sb), 4);
      mbar_init(b_pvdone(sb), 1);
    }
    mbar_init(b_drain, 1);
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
  // the peer's barriers are initialized before anything of this CTA reaches its shared memory
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  if (tid == 0) TC_TRACE(62, 1);
  const uint32_t tmem = *tmem_base;
  const int rank = PAIR ? ht : 0;  // head tile = rank in the pair (consecutive blocks form a cluster)
  const uint32_t peer_smem = PAIR ? cluster_map(smem_u32(smem), (uint32_t)(rank ^ 1)) : 0u;
  // TMEM columns: S^T[s] at 32 s (NH), s = the sub-block's parity; O^T block b at 64 + 64 b
  // (2 NH: the head pass's columns, then the tail pass's)
  const uint32_t tm_s = tmem, tm_o = tmem + 64;

  if (BULK && warp == 11) {
    // ================= staged producer: the record copies (one warp; lane l: keys l and 32 + l)
    // Per tile j: tile j + 1's records located (their scale-code words loaded), tile j + 2's
    // key-table entries loaded, then -- once stage j % STG is converted -- tile j's metadata
    // published and its runs fetched: a key starts a run unless it continues the previous key's
    // record (the next slot of the same page); a run's start lane copies the whole run.
    uint64_t* meta_c = reinterpret_cast<uint64_t*>(smem + L::kMeta + L::kMetaStages * 64 * 8);  // [stage][64]
    constexpr int RB = L::kRecBytes;
    const bool has_b = lane < kTcKeys - 32;
    uint64_t* live_mask = reinterpret_cast<uint64_t*>(smem + L::kMisc + 8);  // [STG] keys with a record
    auto kt_load = [&](int j, int i) {
      const int k = k0 + j * kTcKeys + i;
      return (i < kTcKeys && k < k1) ? a.kt[(size_t)t * a.keys_ld + k] : -1;
    };
    auto locate = [&](int v, const uint8_t*& p, uint64_t& c) {
      p = nullptr;
      c = 0;
      const bool comp = v < 0 && v != -1 && a.comp != nullptr;
      if (v >= 0 || comp) {
        const int sl = v & 0x7fffffff;
        const int blk = comp ? a.comp_blk : a.swa_blk;
        const uint8_t* page = (comp ? a.comp : a.swa) + (int64_t)(sl / blk) * (comp ? a.comp_stride : a.swa_stride);
        const int off = sl % blk;
        p = page + (size_t)off * RB;
        c = *reinterpret_cast<const uint64_t*>(page + (size_t)blk * RB + (size_t)off * 8);
      }
    };
    const uint8_t *pa = nullptr, *pb = nullptr;
    uint64_t ca = 0, cb = 0;
    int va = -1, vb = -1;
    if (nsub > 0) {
      locate(kt_load(0, lane), pa, ca);
      locate(kt_load(0, 32 + lane), pb, cb);
      va = kt_load(1, lane);
      vb = kt_load(1, 32 + lane);
    }
    int issued = 0;  // tiles whose copies went out
    for (int j = 0; j < nsub; ++j) {
      const int st = j % STG;
      const uint8_t *na = nullptr, *nb = nullptr;
      uint64_t nca = 0, ncb = 0;
      if (j + 1 < nsub) {
        locate(va, na, nca);
        locate(vb, nb, ncb);
        va = kt_load(j + 2, lane);
        vb = kt_load(j + 2, 32 + lane);
      }
      if (j >= STG && !__all_sync(0xffffffffu, mbar_wait(b_sempty(st), ((j / STG) - 1) & 1, abort))) break;
      if (lane == 0) TC_TRACE(j, 14);
      meta_c[st * 64 + lane] = ca;
      if (has_b) meta_c[st * 64 + 32 + lane] = cb;
      // runs: key i breaks a run when it is masked or does not continue key i - 1's record
      const uint8_t* prev_a = reinterpret_cast<const uint8_t*>(
          __shfl_up_sync(0xffffffffu, reinterpret_cast<unsigned long long>(pa), 1));
      const uint8_t* last_a = reinterpret_cast<const uint8_t*>(
          __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(pa), 31));
      const uint8_t* prev_b = reinterpret_cast<const uint8_t*>(
          __shfl_up_sync(0xffffffffu, reinterpret_cast<unsigned long long>(pb), 1));
      if (lane == 0) {
        prev_a = nullptr;
        prev_b = last_a;
      }
      const bool start_a = pa != nullptr && !(prev_a != nullptr && pa == prev_a + RB);
      const bool start_b = has_b && pb != nullptr && !(prev_b != nullptr && pb == prev_b + RB);
      const uint32_t brk_a = __ballot_sync(0xffffffffu, start_a || pa == nullptr);
      const uint32_t brk_b = __ballot_sync(0xffffffffu, !has_b || start_b || pb == nullptr);
      const uint64_t brk = (uint64_t)brk_a | ((uint64_t)brk_b << 32);  // bits kTcKeys .. 63 set
      const uint32_t va_mask = __ballot_sync(0xffffffffu, pa != nullptr);
      const uint32_t vb_mask = __ballot_sync(0xffffffffu, has_b && pb != nullptr);
      const uint32_t nvalid = __popc(va_mask) + __popc(vb_mask);
      if (lane == 0) live_mask[st] = (uint64_t)va_mask | ((uint64_t)vb_mask << 32);
      __syncwarp();
      if (lane == 0) tc_expect_tx(b_sfull(st), nvalid * (uint32_t)RB);  // (arrives: 0 bytes completes)
      __syncwarp();
      const uint32_t stage = smem_u32(smem + L::kStage + st * L::kStageBytes);
      auto run_copy = [&](int i, const uint8_t* p) {
        const uint64_t above = brk & ~((2ull << i) - 1);
        const int len = __ffsll((long long)above) - 1 - i;
        tc_bulk_load(stage + (uint32_t)(i * RB), p, (uint32_t)(len * RB), b_sfull(st));
      };
      if (start_a) run_copy(lane, pa);
      if (start_b) run_copy(32 + lane, pb);
      if (lane == 0) TC_TRACE(j, 15);
      issued = j + 1;
      pa = na;
      pb = nb;
      ca = nca;
      cb = ncb;
    }
    // no copy may still be landing when the CTA leaves (after an abort the converters stopped
    // consuming): wait, bounded, for the last issued phase of each stage
    for (int st = 0; st < STG; ++st) {
      const int last = issued - 1 - ((issued - 1 - st) % STG + STG) % STG;  // largest tile < issued in stage st
      if (last < 0) continue;
      for (uint32_t it = 0; it < kTcWaitPolls && !mbar_try(b_sfull(st), (last / STG) & 1); ++it) {
      }
    }
  } else if (BULK && warp >= 5) {
    // ================= staged producer: conversion (warps 5-10) of the staged records into the
    // f16 tile, the gathering producers' arithmetic; item e = (key e / CHUNKS, chunk e % CHUNKS),
    // consecutive threads on consecutive 16-byte chunks of a record
    const uint64_t* meta_c = reinterpret_cast<const uint64_t*>(smem + L::kMeta + L::kMetaStages * 64 * 8);
    const uint64_t* live_mask = reinterpret_cast<const uint64_t*>(smem + L::kMisc + 8);
    // warp w converts keys 8 w .. 8 w + 7: item i of a lane = flat index lane + 32 i of the warp's
    // 8 x CHUNKS chunks (key f / CHUNKS, chunk f % CHUNKS); all of a lane's loads go out first
    constexpr int kItemsB = 8 * CHUNKS / 32;
    static_assert(8 * CHUNKS % 32 == 0 && 6 * 8 == kTcKeys, "six warps of 8 keys, whole items");
    const int kbase = 8 * (warp - 5);
    for (int j = 0; j < nsub; ++j) {
      const int st = j % STG, ts = j % TS;
      if (!mbar_wait(b_sfull(st), (j / STG) & 1, abort)) break;
      if (tid == 160) TC_TRACE(j, 4);
      if (j >= TS && !mbar_wait(b_free(ts), ((j / TS) - 1) & 1, abort)) break;
      if (tid == 160) TC_TRACE(j, 0);
      const uint8_t* stage = smem + L::kStage + st * L::kStageBytes;
      uint8_t* tile = smem + L::kTile0 + ts * L::kTileBytes;
      const uint64_t live = live_mask[st];
      uint4 raw[kItemsB];
#pragma unroll
      for (int i = 0; i < kItemsB; ++i) {
        const int f = lane + 32 * i, key = kbase + f / CHUNKS, c = f % CHUNKS;
        raw[i] = ((live >> key) & 1) ? *reinterpret_cast<const uint4*>(stage + key * L::kRecBytes + 16 * c)
                                     : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < kItemsB; ++i) {
        const int f = lane + 32 * i, key = kbase + f / CHUNKS, c = f % CHUNKS;
        const int b0 = 16 * c;
        const bool is_live = (live >> key) & 1;
        if (b0 < NOPE) {
          uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
          if (is_live) {
            const int cd = (int)((meta_c[st * 64 + key] >> (8 * (b0 / 64))) & 0xff);
            const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
            uint32_t r[8];
            if (e4m3_f16_scale_ok(cd)) {
              const uint32_t s2 = e4m3_f16_scale(cd);
#pragma unroll
              for (int q = 0; q < 4; ++q) e4m3x4_f16x2_scaled(w[q], s2, r[2 * q], r[2 * q + 1]);
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
          *reinterpret_cast<uint4*>(tile + sw_off<kTcKeys>(key, b0)) = o0;
          *reinterpret_cast<uint4*>(tile + sw_off<kTcKeys>(key, b0 + 8)) = o1;
        } else {
          uint4 o0 = make_uint4(0, 0, 0, 0);
          if (is_live)
            o0 = make_uint4(bf16x2_to_f16x2(raw[i].x), bf16x2_to_f16x2(raw[i].y), bf16x2_to_f16x2(raw[i].z),
                            bf16x2_to_f16x2(raw[i].w));
          *reinterpret_cast<uint4*>(tile + sw_off<kTcKeys>(key, NOPE + (b0 - NOPE) / 2)) = o0;
        }
      }
      fence_async_smem();  // the MMA (async proxy) reads the tile
      __syncwarp();
      if (tid == 160) TC_TRACE(j, 1);
      if (lane == 0) {
        mbar_arrive(b_full(ts));
        mbar_arrive(b_sempty(st));
      }
    }
  } else if (warp >= 5) {
    if constexpr (!BULK) {
    // ================= producers
    // Per tile: the metadata threads publish their key (record pointer, the 8 scale codes;
    // null = masked) into shared memory; then each conversion warp converts units of 8 keys x 4
    // consecutive 16-byte chunks (lane: key 8 g + lane % 8, chunk 4 q + lane / 8) of its key
    // group g, so a warp's loads are whole 64-byte runs of 8 records. Loads run ahead of use:
    // while tile j converts, the record chunks of the next kAhead tiles and the following tiles'
    // scale codes and key-table entries are in flight.
    static_assert(CHUNKS % 4 == 0, "records are whole 64-byte runs");
    const int ptid = tid - 5 * 32, wp = warp - 5;
    const int data_bytes = NOPE + 128;
    // loads run kAhead tiles ahead of the conversion: two for a pair (its producers hold half a
    // tile's chunks, so three tiles' fit in registers), else one
    constexpr int kAhead = PAIR ? 2 : 1;
    constexpr int kStages = kAhead + 1;  // metadata stages: tiles j .. j + kAhead
    static_assert(kStages <= L::kMetaStages, "metadata stages");
    const uint8_t** meta_p = reinterpret_cast<const uint8_t**>(smem + L::kMeta);  // [stage][64] then codes
    uint64_t* meta_c = reinterpret_cast<uint64_t*>(smem + L::kMeta + L::kMetaStages * 64 * 8);
    constexpr int kGroups = PAIR ? kTcKeys / 16 : kTcKeys / 8;  // 8-key groups this CTA converts
    // 6 conversion warps, each on ONE key group (so its keys' metadata and the key part of every
    // store offset hold for all its items) and a run of chunk groups; the 7th warp does the
    // metadata (key table, record address, codes) and issues the pair's half-tile copies
    constexpr int kConvWarps = 6;
    static_assert(kConvWarps % kGroups == 0, "whole key groups a warp");
    constexpr int kWpg = kConvWarps / kGroups;                 // warps a key group
    constexpr int kItems = (CHUNKS / 4 + kWpg - 1) / kWpg;     // chunk groups a warp
    constexpr int kMetaKeys = 8 * kGroups;  // keys this CTA locates
    const int g0 = PAIR ? rank * kGroups : 0;
    // metadata threads: the 7th warp's first lanes (a pair: 24 keys), or the first 48 producer
    // threads (a lone CTA's 48 keys)
    const int meta_tid = PAIR ? ptid - 32 * kConvWarps : ptid;
    const bool is_meta = meta_tid >= 0 && meta_tid < kMetaKeys;
    constexpr uint32_t kHalfBytes = (uint32_t)(kGroups * 8 * DG * 16);  // a pair's half tile
    constexpr int kChunkT = (kTcKeys / 8) * 1024;                         // a 64-dim chunk of a tile
    const int mkey = 8 * g0 + meta_tid;  // a metadata thread's key of a tile
    auto item = [&](int i, int& key, int& c) {  // this lane's (key, chunk) of its i-th unit
      const int cg = (wp % kWpg) * kItems + i;
      key = 8 * (g0 + wp / kWpg) + (lane & 7);
      c = 4 * cg + (lane >> 3);
      return wp < kConvWarps && cg < CHUNKS / 4;
    };
    // key lookahead (metadata threads, key mkey of a tile)
    auto kt_load = [&](int j) {  // the key-table entry; -1 past the chunk
      const int k = k0 + j * kTcKeys + mkey;
      return k < k1 ? a.kt[(size_t)t * a.keys_ld + k] : -1;
    };
    const uint8_t* la_p = nullptr;  // tile j + 2's record and scale-code word (load in flight)
    uint64_t la_c = 0;
    auto locate = [&](int v) {
      la_p = nullptr;
      la_c = 0;
      const bool comp = v < 0 && v != -1 && a.comp != nullptr;
      if (v >= 0 || comp) {
        const int sl = v & 0x7fffffff;
        const int blk = comp ? a.comp_blk : a.swa_blk;
        const uint8_t* page = (comp ? a.comp : a.swa) + (int64_t)(sl / blk) * (comp ? a.comp_stride : a.swa_stride);
        const int off = sl % blk;
        la_p = page + (size_t)off * data_bytes;
        la_c = *reinterpret_cast<const uint64_t*>(page + (size_t)blk * data_bytes + (size_t)off * 8);
      }
    };
    auto publish = [&](int j) {
      meta_p[(j % kStages) * 64 + mkey] = la_p;
      meta_c[(j % kStages) * 64 + mkey] = la_c;
    };
    auto issue = [&](int j, uint4 (&raw)[kItems]) {
      const int ms = j % kStages;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        int key, c;
        raw[i] = make_uint4(0, 0, 0, 0);
        if (item(i, key, c)) {
          const uint8_t* dp = meta_p[ms * 64 + key];
          if (dp) raw[i] = ldg16(dp + 16 * c);
        }
      }
    };
    auto convert = [&](int j, const uint4 (&raw)[kItems]) {
      const int ts = j % TS, ms = j % kStages;
      const int tile_off = L::kTile0 + ts * L::kTileBytes;
      // into this CTA's tile (a pair's half then goes to the peer by one bulk copy, below)
      auto put = [&](int off, const uint4& v) { *reinterpret_cast<uint4*>(smem + tile_off + off) = v; };
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        int key, c;
        if (!item(i, key, c)) continue;
        const int b0 = 16 * c;
        const bool live = meta_p[ms * 64 + key] != nullptr;
        if (b0 < NOPE) {
          uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
          if (live) {
            const int cd = (int)((meta_c[ms * 64 + key] >> (8 * (b0 / 64))) & 0xff);
            const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
            uint32_t r[8];
            if (e4m3_f16_scale_ok(cd)) {
              const uint32_t s2 = e4m3_f16_scale(cd);
#pragma unroll
              for (int q = 0; q < 4; ++q) e4m3x4_f16x2_scaled(w[q], s2, r[2 * q], r[2 * q + 1]);
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
          put(sw_off<kTcKeys>(key, b0), o0);
          put(sw_off<kTcKeys>(key, b0 + 8), o1);
        } else {
          uint4 o0 = make_uint4(0, 0, 0, 0);
          if (live)
            o0 = make_uint4(bf16x2_to_f16x2(raw[i].x), bf16x2_to_f16x2(raw[i].y), bf16x2_to_f16x2(raw[i].z),
                            bf16x2_to_f16x2(raw[i].w));
          put(sw_off<kTcKeys>(key, NOPE + (b0 - NOPE) / 2), o0);
        }
      }
      fence_async_smem();  // the MMA and the bulk copy (async proxy) read these writes
      __syncwarp();
      if (lane == 0) mbar_arrive(b_full(ts));
      if (PAIR) {
        // this CTA's half (key groups g0 .. g0 + kGroups - 1: contiguous within each 64-dim
        // chunk) into the peer's tile once every producer warp has written it, a copy a chunk
        asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
        // (lane c of the metadata warp copies chunk c; lane 0 also raises the peer's
        // expected bytes -- the transaction count is signed, so a copy may land first)
        const int ct = ptid - 32 * kConvWarps;  // the metadata warp's lanes
        if (ct >= 0 && ct < D / 64) {
          const uint32_t peer_bar = cluster_map(b_full(ts), (uint32_t)(rank ^ 1));
          if (ct == 0) mbar_arrive_tx_remote(peer_bar, kHalfBytes);
          const uint32_t off = (uint32_t)(tile_off + ct * kChunkT + g0 * 1024);
          bulk_copy_to_peer(peer_smem + off, smem_u32(smem) + off, (uint32_t)(kGroups * 1024), peer_bar);
        }
      }
    };
    // one tile: free its stage, publish and issue the next tile, convert this one (cur holds its
    // chunks; nxt receives the next tile's)
    int la_v = -1;  // tile j + kAhead + 2's key-table entry (load in flight)
    // one tile: once its stage is free, convert it (a pair first: its chunks were loaded two
    // tiles ago), publish and issue tile j + kAhead's loads into nxt, locate tile j + kAhead + 1
    auto step = [&](int j, const uint4 (&cur)[kItems], uint4 (&nxt)[kItems]) {
      const int ts = j % TS, fpar = ((j / TS) - 1) & 1;
      // the stage is free (PV(j - 3) done), for every producer alike; and every producer is past
      // tile j - 1's conversion (its metadata stage is rewritten next)
      if (!producers_all(j < TS || (PAIR ? mbar_wait_cl(b_free(ts), fpar, abort)
                                                : mbar_wait(b_free(ts), fpar, abort))))
        return false;
      if (ptid == 0) TC_TRACE(j, 0);
      if (PAIR) {
        convert(j, cur);
        if (ptid == 0) TC_TRACE(j, 1);
        // the metadata before the records: publish and locate use loads issued before the last
        // record loads, so they wait for nothing newer (a use of a load waits for the loads issued
        // ahead of it); then the next key-table entry, then the records kAhead tiles on
        const bool more = j + kAhead < nsub;
        if (more && is_meta) publish(j + kAhead);
        if (is_meta) {
          locate(la_v);
          la_v = kt_load(j + kAhead + 2);
        }
        if (ptid == 0) TC_TRACE(j, 4);
        if (more) {
          asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
          if (ptid == 0) TC_TRACE(j, 14);
          issue(j + kAhead, nxt);
          if (ptid == 0) TC_TRACE(j, 15);
        }
        return true;
      }
      if (j + kAhead < nsub) {
        if (is_meta) publish(j + kAhead);
        asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
        if (ptid == 0) TC_TRACE(j, 14);
        issue(j + kAhead, nxt);
        if (ptid == 0) TC_TRACE(j, 15);
      }
      if (is_meta) {
        locate(la_v);
        la_v = kt_load(j + kAhead + 2);
      }
      if (ptid == 0) TC_TRACE(j, 4);
      convert(j, cur);
      if (ptid == 0) TC_TRACE(j, 1);
      return true;
    };
    uint4 buf0[kItems], buf1[kItems];
    if (nsub > 0) {
      if (is_meta) {
#pragma unroll
        for (int i = 0; i < kAhead; ++i) {
          locate(kt_load(i));
          publish(i);
        }
        const int v = kt_load(kAhead);
        la_v = kt_load(kAhead + 1);
        locate(v);
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kTcProducers) : "memory");
      issue(0, buf0);
    }
    if constexpr (PAIR) {
      uint4 buf2[kItems];
      if (nsub > 1) issue(1, buf1);
      for (int j = 0; j < nsub; j += 3) {
        if (!step(j, buf0, buf2)) break;
        if (j + 1 < nsub && !step(j + 1, buf1, buf0)) break;
        if (j + 2 < nsub && !step(j + 2, buf2, buf1)) break;
      }
    } else {
      for (int j = 0; j < nsub; j += 2) {
        if (!step(j, buf0, buf1)) break;
        if (j + 1 < nsub && !step(j + 1, buf1, buf0)) break;
      }
    }
    }  // !BULK
  } else if (warp == 4) {
    // ================= MMA issue (one elected thread)
    // QK(j) needs tile j and S[j & 1] consumed by softmax(j - 2); PV(j) needs P(j) (written
    // after softmax(j) rescaled O, when it had to). QK(j + 1) goes out as soon as its inputs are
    // ready, so it runs under softmax(j).
    if (lane == 0) {
      const uint32_t id_qk = umma_idesc(64, NH, 0, 0);
      const uint32_t id_pv = umma_idesc(128, 2 * NH, 1, 1);
      auto issue_qk = [&](int j) {
        const uint32_t tile = s_tile0 + (j % TS) * L::kTileBytes;
        const uint32_t dst = tm_s + 32 * (j & 1);
        // K-major, 128-byte swizzle: K step ks = 16 dims, byte 32 (ks % 4) of chunk ks / 4's rows
        // (tile chunks (kTcKeys / 8) KB apart, Q's 4 KB); 8-row groups 1 KB apart
#pragma unroll 4
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16(dst, umma_sdesc_sw128(tile + (ks >> 2) * ((kTcKeys / 8) * 1024) + (ks & 3) * 32, 16, 1024),
                   umma_sdesc_sw128(s_q + (ks >> 2) * 4096 + (ks & 3) * 32, 16, 1024), id_qk, ks > 0);
        umma_commit(b_sready(j & 1));
        TC_TRACE(j, 11);
      };
      auto qk_ready = [&](int j) {  // tile j loaded and S[j & 1] consumed by softmax(j - 2)
        const int ts = j % TS, tpar = (j / TS) & 1;
        return (PAIR ? mbar_test_cl(b_full(ts), tpar) : mbar_test(b_full(ts), tpar)) &&
               (j < 2 || mbar_test(b_scons(j & 1), ((j - 2) >> 1) & 1));
      };
      auto wait_qk = [&](int j) {
        const int ts = j % TS, tpar = (j / TS) & 1;
        return (PAIR ? mbar_wait_cl(b_full(ts), tpar, abort) : mbar_wait(b_full(ts), tpar, abort)) &&
               (j < 2 || mbar_wait(b_scons(j & 1), ((j - 2) >> 1) & 1, abort));
      };
      bool ok = true;
      if (nsub > 0) ok = wait_qk(0);
      if (ok && nsub > 0) issue_qk(0);
      for (int j = 0; ok && j < nsub; ++j) {
        const int s = j & 1;
        const uint32_t p_ready = b_pready(s), p_par = (j >> 1) & 1;
        bool qk_done = j + 1 >= nsub;
        if (!qk_done && qk_ready(j + 1)) {
          issue_qk(j + 1);
          qk_done = true;
        }
        if (!qk_done) {
          // wait for whichever comes first: P(j) (then PV), or QK(j + 1)'s inputs
          for (uint32_t it = 0; !qk_done && it < kTcWaitPolls; ++it) {
            if (mbar_test(p_ready, p_par)) break;
            if (qk_ready(j + 1)) {
              issue_qk(j + 1);
              qk_done = true;
            }
          }
        }
        TC_TRACE(j, 2);
        ok = mbar_wait(p_ready, p_par, abort);
        if (!ok) break;
        TC_TRACE(j, 3);
        tc_fence_after();
        // PV: O += V^T P^T, P^T's columns the f16 head of p (0 .. NH - 1), then its tail
        const uint32_t tile = s_tile0 + (j % TS) * L::kTileBytes;
        const uint32_t pt = s_p + 2 * s * L::kPBytes;
        // A = V^T, MN-major, 128-byte swizzle: a 128-dim block = 2 chunks (kTcKeys / 8) KB apart
        // (lbo), K step ks = key groups 2 ks, 2 ks + 1 (1 KB apart: sbo); B = P^T, no swizzle
        const uint64_t db0 = umma_sdesc(pt, (2 * NH / 8) * 128, 128);
        const uint32_t db_step = (uint32_t)(2 * (2 * NH / 8) * 128) >> 4;
#pragma unroll
        for (int b = 0; b < NBLK; ++b) {
          const int d0 = min(128 * b, D - 128);
#pragma unroll
          for (int ks = 0; ks < kTcKeys / 16; ++ks)
            umma_f16(tm_o + 64 * b,
                     umma_sdesc_sw128(tile + (d0 / 64) * ((kTcKeys / 8) * 1024) + ks * 2048, (kTcKeys / 8) * 1024, 1024),
                     db0 + (uint64_t)(ks * db_step), id_pv, j > 0 || ks > 0);
        }
        if (PAIR)
          umma_commit_pair(b_free(j % TS));  // the tile is free, in both CTAs
        else
          umma_commit(b_free(j % TS));  // the tile is free
        umma_commit(b_pvdone(s));  // P[s] free; O holds sub-blocks 0 .. j
        if (!qk_done) {
          ok = wait_qk(j + 1);
          if (!ok) break;
          issue_qk(j + 1);
        }
      }
      // drain: every issued MMA complete before the TMEM is freed (also after an abort)
      umma_commit(b_drain);
      mbar_wait(b_drain, 0, abort);
    }
  } else {
    // ================= softmax + epilogue (warps 0-3: TMEM lanes 32 w .. 32 w + 31)
    // Thread (warp w, lane < 16) holds key 16 w + lane of a sub-block (S^T rows of an M = 64
    // MMA sit on the first 16 lanes of each 32-lane quarter). p = 2^(s - m) against a per-head
    // reference m that moves only when a sub-block's max passes it by more than 2^kTcSlack
    // (p <= 2^kTcSlack stays well inside f16): then O and the partial sums are rescaled once.
    // Each key thread keeps its own partial sums of p.
    const int key = 16 * warp + (lane & 15);
    const bool has_key = lane < 16 && key < kTcKeys;  // keys 48 .. 63: the QK's padded rows
    const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;
    const int ngroups = NH / 16;
    float l_part[32];
#pragma unroll
    for (int h = 0; h < 32; ++h) l_part[h] = 0.f;
    bool ok = true;
    // O *= alpha (per head, head and tail columns) for this thread's lane (dim) in every block
    auto rescale_o = [&]() {
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (g >= ngroups) break;
          uint32_t vh[16], vt[16];
          const uint32_t col = tm_o + 64 * b + lane_addr + 16 * g;
          tmem_ld16(col, vh);
          tmem_ld16(col + NH, vt);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            vh[q] = __float_as_uint(__uint_as_float(vh[q]) * a_sm[16 * g + q]);
            vt[q] = __float_as_uint(__uint_as_float(vt[q]) * a_sm[16 * g + q]);
          }
          tmem_st16(col, vh);
          tmem_st16(col + NH, vt);
        }
      }
      tmem_wait_st();
    };
    // this thread's key-table entry, one sub-block ahead
    auto kt_entry = [&](int j) {
      const int k = k0 + j * kTcKeys + key;
      return (has_key && k < k1) ? a.kt[(size_t)t * a.keys_ld + k] : -1;
    };
    int kt_next = nsub > 0 ? kt_entry(0) : -1;
    for (int j = 0; ok && j < nsub; ++j) {
      const int s = j & 1;
      const int kv_ = kt_next;
      kt_next = j + 1 < nsub ? kt_entry(j + 1) : -1;
      const bool valid = kv_ != -1 && (kv_ >= 0 || a.comp != nullptr);
      ok = softmax_all(mbar_wait(b_sready(s), (j >> 1) & 1, abort));
      if (!ok) break;
      if (tid == 0) TC_TRACE(j, 5);
      tc_fence_after();
      float sv[32];
      {
        uint32_t v[32];
        tmem_ld16(tm_s + 32 * s + lane_addr, *reinterpret_cast<uint32_t(*)[16]>(v));
        if (NH > 16) tmem_ld16(tm_s + 32 * s + lane_addr + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        // S[s] is in registers: QK(j + 2) may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_scons(s));
        if (tid == 0) TC_TRACE(j, 8);
#pragma unroll
        for (int q = 0; q < 32; ++q) sv[q] = (valid && q < NH) ? __uint_as_float(v[q]) * a.scale_log2 : -INFINITY;
      }
      // The reference max moves only when a score passes it by more than the slack (in the
      // first sub-block with a valid key, rarely after): only then the sub-block's per-head max,
      // over the 16 key lanes and then the 4 warps (through red)
      bool exceed = false;
#pragma unroll
      for (int q = 0; q < 32; q += 4) {
        const float4 m4 = *reinterpret_cast<const float4*>(m_sm + q);
        exceed |= (sv[q] > m4.x + kTcSlack) | (sv[q + 1] > m4.y + kTcSlack) | (sv[q + 2] > m4.z + kTcSlack) |
                  (sv[q + 3] > m4.w + kTcSlack);
      }
      bool rescale = false;
      if (softmax_any(exceed)) {
        // (lanes 16 .. 31 hold no key: -inf)
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const float x = warp_max_f32(sv[q]);
          if (lane == q) red[warp * 32 + q] = x;
        }
        softmax_bar();  // red complete
        if (tid == 0) TC_TRACE(j, 6);
        bool moved = false;  // a head's reference moved while O already holds its sums
        if (tid < NH) {
          const float bx = fmaxf(fmaxf(red[tid], red[32 + tid]), fmaxf(red[64 + tid], red[96 + tid]));
          const float mu = m_sm[tid];
          float al = 1.f;
          if (bx > mu + kTcSlack) {
            al = (mu == -INFINITY) ? 0.f : exp2f(mu - bx);
            moved = mu != -INFINITY;
            m_sm[tid] = bx;
          }
          a_sm[tid] = al;
        }
        rescale = softmax_any(moved) && j > 0;  // also publishes m_sm / a_sm
      }
      if (tid == 0) TC_TRACE(j, 9);
      if (rescale) {
        // O must hold every issued PV before it is scaled
        ok = softmax_all(mbar_wait(b_pvdone((j - 1) & 1), ((j - 1) >> 1) & 1, abort));
        if (!ok) break;
        tc_fence_after();
        rescale_o();
        tc_fence_before();
#pragma unroll
        for (int q = 0; q < 32; ++q) l_part[q] *= a_sm[q];
        if (tid == 0) TC_TRACE(j, 10);
      }
      // p = 2^(s - m) into P^T[s] as an f16 head and its f16 tail (the PV sees ~22 bits of p);
      // this thread's partial sums of p
      // (the head keeps p's top 11 significant bits, exact in f16 for p >= 2^-14; the tail is
      // the exact remainder, rounded to f16)
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int q = 0; q < 32; q += 4) {
        const float4 m4 = *reinterpret_cast<const float4*>(m_sm + q);
        const float mq[4] = {m4.x, m4.y, m4.z, m4.w};
        float pq[4], hq[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pq[i] = sv[q + i] == -INFINITY ? 0.f : ex2_approx(sv[q + i] - mq[i]);
          l_part[q + i] += pq[i];
          hq[i] = __uint_as_float(__float_as_uint(pq[i]) & 0xffffe000u);
        }
        hi[q / 2] = cvt_f16x2(hq[0], hq[1]);
        hi[q / 2 + 1] = cvt_f16x2(hq[2], hq[3]);
        lo[q / 2] = cvt_f16x2(pq[0] - hq[0], pq[1] - hq[1]);
        lo[q / 2 + 1] = cvt_f16x2(pq[2] - hq[2], pq[3] - hq[3]);
      }
      if (tid == 0) TC_TRACE(j, 12);
      // P^T[s] is free once PV(j - 2) is done
      if (j >= 2) {
        ok = softmax_all(mbar_wait(b_pvdone(s), ((j - 2) >> 1) & 1, abort));
        if (!ok) break;
      }
      if (tid == 0) TC_TRACE(j, 13);
      if (has_key) {
        // P^T [key group][column group][8 keys][8 columns]: head groups 0 .. NH / 8 - 1, then tail
        uint8_t* pt = smem + L::kP + 2 * s * L::kPBytes;
        const int row = (key >> 3) * (2 * NH / 8);
#pragma unroll
        for (int hg = 0; hg < 4; ++hg) {
          if (8 * hg >= NH) break;
          *reinterpret_cast<uint4*>(pt + (row + hg) * 128 + (key & 7) * 16) =
              make_uint4(hi[4 * hg], hi[4 * hg + 1], hi[4 * hg + 2], hi[4 * hg + 3]);
          *reinterpret_cast<uint4*>(pt + (row + NH / 8 + hg) * 128 + (key & 7) * 16) =
              make_uint4(lo[4 * hg], lo[4 * hg + 1], lo[4 * hg + 2], lo[4 * hg + 3]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_pready(s));
      if (tid == 0) TC_TRACE(j, 7);
      // (the next update of red, m_sm and a_sm comes after the next sub-block's first barrier,
      // which every thread reaches only after this sub-block's reads)
    }
    // ---- epilogue: every PV done, then O^T (head + tail columns) and (m, l) of the chunk
    if (ok && nsub > 0) ok = softmax_all(mbar_wait(b_pvdone((nsub - 1) & 1), ((nsub - 1) >> 1) & 1, abort));
    if (tid == 0) TC_TRACE(63, 0);
    const size_t base = ((size_t)t * a.nchunks + ch) * a.heads + h0;
    const int nh_live = min(NH, a.heads - h0);
    if (ok && nsub > 0) {
      tc_fence_after();
      // l: the partial sums of the 64 key threads (16 lanes x 4 warps), lane h taking head h
#pragma unroll
      for (int h = 0; h < 32; ++h)
        if (!has_key || h >= NH) l_part[h] = 0.f;
      warp_transpose_sum(l_part, lane);
      red[warp * 32 + lane] = l_part[0];
      softmax_bar();
      if (tid < nh_live) {
        a.part_ml[(base + tid) * 2] = m_sm[tid];
        a.part_ml[(base + tid) * 2 + 1] = (red[tid] + red[32 + tid]) + (red[64 + tid] + red[96 + tid]);
      }
      if (tid == 0) TC_TRACE(63, 1);
      const int dl = 32 * warp + lane;  // this thread's dim within a block
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
        const int d0 = min(128 * b, D - 128);
        const int d = d0 + dl;
        const bool own = d >= 128 * b;  // the overlapping last block writes only its new dims
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          if (g >= ngroups) break;
          uint32_t vh[16], vt[16];
          tmem_ld16(tm_o + 64 * b + lane_addr + 16 * g, vh);
          tmem_ld16(tm_o + 64 * b + lane_addr + NH + 16 * g, vt);
          tmem_wait_ld();
          if (own)
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (16 * g + q < nh_live)
                a.part_o[(base + 16 * g + q) * D + d] = __uint_as_float(vh[q]) + __uint_as_float(vt[q]);
        }
      }
    } else if (nsub == 0 && tid < nh_live) {
      a.part_ml[(base + tid) * 2] = -INFINITY;
      a.part_ml[(base + tid) * 2 + 1] = 0.f;
    }
  }
  // ---- teardown: every role done (a timed-out one unwound); free the TMEM. A pair leaves
  // together: the peer's stores and MMA-completion arrivals target this CTA's shared memory
  // until its own roles are done.
  if (tid == 0) TC_TRACE(63, 2);
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();
  if (tid == 0) TC_TRACE(63, 3);
  if (warp == 4) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  TC_SPAN(1);
  pdl_launch();
}

}  // namespace dsv41
