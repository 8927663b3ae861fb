// K2's attention core for a row's 64 heads in one CTA (tcgen05, accumulators in TMEM): the split
// step of back.py:189-435 of the reference, with every MMA instruction covering all 64 heads.
//
// CTA = (row, chunk of the row's keys), 16 warps:
//   warps 0-7   softmax + epilogue: warp w owns TMEM lane quarter w % 4 and heads 32 (w / 4) ..
//   warp  8     TMEM allocation and the QK issue (one elected thread)
//   warp  9     copies: a tile's key-table entries -> runs of consecutive slots of one page -> one
//               cp.async.bulk a run into the staging buffer (a tile's 48 raw records); the scale
//               codes; and (lane 0) the PV issue: two issuing threads, because one thread's issue
//               rate (~70 cycles an MMA of these shapes) set the period
//   warps 10-15 conversion: staged FP8 records -> the f16 tile (two tiles in flight)
// Per 48-key tile j (tile, S and P buffers j & 1):
//   S^T[64 keys x 64 heads] = K_tile . Q^T   tcgen05.mma M=64 (keys; rows 48..63 read what follows
//                                            the tile and are masked), N=64, K=D: A the tile, B = Q
//                                            (both K-major, 128-byte swizzle), D in TMEM;
//   softmax over keys against a per-head reference max that moves only when a score passes it by
//   more than 2^8 (then O is rescaled in TMEM); p is stored as one f16, 2^(s - m + 7): at most 2^15,
//   and below f16's normal range only for p < 2^-21 of the row's largest;
//   O^T[D dims x 64 heads] += V_tile^T . P^T  M=128 (dims, 5 blocks: the last overlaps), N=64, K=48:
//                                            A the tile read MN-major, B = P^T (MN-major, written by
//                                            the softmax threads).
// The (m, l) written for the combine are in that shifted domain (m - 7), consistent with O.
//
// Shared memory conflicts: the staging buffer holds whole records (640 B apart); a converter lane
// reads 8 consecutive FP8 bytes (a warp: 256 contiguous bytes) and writes their 8 f16 values as
// one 16-byte unit of the swizzled tile (a warp: 32 units whose bank groups, (unit ^ row) % 8, take
// every value four times), so neither side serializes.
#pragma once

#include "attn_tc.cuh"

namespace dsv41 {

constexpr int kWdKeys = 48;     // keys a tile (the QK's M = 64: 16 padded rows)
constexpr int kWdNH = 64;       // heads a CTA: N of both MMAs
constexpr int kWdThreads = 512;  // 16 warps
constexpr int kWdConv = 6;      // converter warps (10..15)
constexpr float kWdShift = 7.f;  // log2 of p's storage scale


template <int D>
struct WdSmem {
  static constexpr int kRecBytes = D - 64 + 128;          // a record's data row: nope e4m3, rope bf16
  static constexpr int kTileBytes = kWdKeys * D * 2;       // f16, [64-dim chunk][8-key group][8 x 128 B]
  static constexpr int kTile0 = 0;                         // 2 tiles
  static constexpr int kQ = 2 * kTileBytes;                // (the QK's padded rows of tile 1 read Q)
  static constexpr int kQBytes = kWdNH * D * 2;
  static constexpr int kPBytes = kWdKeys * kWdNH * 2;      // P^T [key group][head group][8 keys][8 heads]
  static constexpr int kP = kQ + kQBytes;                  // 2 buffers
  static constexpr int kStage = kP + 2 * kPBytes;          // a tile's staged records
  static constexpr int kStageBytes = kWdKeys * kRecBytes;
  static constexpr int kRed = kStage + kStageBytes;        // float [8 warps][32]
  static constexpr int kM = kRed + 8 * 32 * 4;             // float [64]: reference max a head
  static constexpr int kAlpha = kM + 64 * 4;               // float [64]: its rescale factor
  static constexpr int kMeta = kAlpha + 64 * 4;            // uint64 [2][64] code words, then uint64 [2] live masks
  static constexpr int kBar = kMeta + 2 * 64 * 8 + 16;
  static constexpr int kNumBars = 16;
  static constexpr int kMisc = kBar + kNumBars * 8;        // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16 + 1024;         // + slack to align the base to 1 KB
  static_assert(kStage % 16 == 0 && kRecBytes % 16 == 0, "bulk copy destinations are 16-byte aligned");
  static_assert(kBytes <= 232448, "shared memory of one CTA");
};

// AND / OR / barrier over the 256 softmax threads (named barrier 1)
__device__ __forceinline__ bool wd_all(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, 1, 256, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ bool wd_any(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, 1, 256, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
__device__ __forceinline__ void wd_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Waits that park the thread: try_wait with a suspend-time hint lets the hardware suspend the
// waiting thread until the phase completes (or the hint runs out), so the roles that mostly wait
// (softmax, converters, copies) leave the issue slots of their scheduler to the MMA thread. Bounded
// by a %globaltimer deadline (2 s); on expiry the abort flag and the device error word are raised.
#ifndef DSV41_WD_SUSPEND_NS
#define DSV41_WD_SUSPEND_NS 20000
#endif
__device__ __forceinline__ bool wd_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(DSV41_WD_SUSPEND_NS)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t wd_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wd_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (wd_try(bar, parity)) return true;
  const uint64_t deadline = wd_now() + 2000000000ull;
  for (;;) {
    if (wd_try(bar, parity)) return true;
    if (*abort) return false;
    if (wd_now() > deadline) break;
  }
  *abort = 1;
  atomicExch(&g_tc_error, 1);
  return false;
}
// A warp's bounded wait on an mbarrier phase, warp-uniform. (Every lane waits: measured faster
// than lane 0 waiting alone and the others taking the completed phase after a shuffle.)
__device__ __forceinline__ bool wd_warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, wd_wait(bar, parity, abort));
}

// 8 e4m3 bytes (two words) -> 8 f16 of value x 2^(code - 127), as one 16-byte unit. For codes
// 113 .. 134 (2^(code - 127) a normal f16, and 448 x it at most 2^15) each pair converts exactly by
// cvt.rn.f16x2.e4m3x2 and one f16x2 multiply by the power of two rounds nothing; other codes take
// the integer bit placement (105 .. 134) or fp32.
__device__ __forceinline__ uint32_t wd_cvt2(uint32_t w16) {
  uint32_t r;
  asm("{\n\t.reg .b16 lo;\n\tcvt.u16.u32 lo, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, lo;\n\t}\n" : "=r"(r) : "r"(w16));
  return r;
}
__device__ __forceinline__ uint4 wd_convert8(uint2 w, int code) {
  uint32_t r[4];
  if (code >= 113 && code <= 134) {
    const uint32_t s1 = (uint32_t)(code - 112) << 10;  // f16 bits of 2^(code - 127)
    const uint32_t s2 = s1 | (s1 << 16);
    r[0] = hmul2_bits(wd_cvt2(w.x), s2);
    r[1] = hmul2_bits(wd_cvt2(w.x >> 16), s2);
    r[2] = hmul2_bits(wd_cvt2(w.y), s2);
    r[3] = hmul2_bits(wd_cvt2(w.y >> 16), s2);
  } else if (e4m3_f16_scale_ok(code)) {
    const uint32_t s2 = e4m3_f16_scale(code);
    e4m3x4_f16x2_scaled(w.x, s2, r[0], r[1]);
    e4m3x4_f16x2_scaled(w.y, s2, r[2], r[3]);
  } else {
    const float sc = pow2c(code);
    const uint32_t ww[2] = {w.x, w.y};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float2 fl = e4m3x2_float2(ww[q] & 0xffff), fh = e4m3x2_float2(ww[q] >> 16);
      r[2 * q] = pack_f16x2(fl.x * sc, fl.y * sc);
      r[2 * q + 1] = pack_f16x2(fh.x * sc, fh.y * sc);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

template <int NOPE>
__global__ void __launch_bounds__(kWdThreads, 1) attn_wide_kernel(const AttnArgs a) {
  constexpr int D = NOPE + 64;
  constexpr int DG = D / 8;              // 16-byte f16 units a row
  constexpr int NBLK = (D + 127) / 128;  // 128-dim PV blocks
  constexpr int RB = NOPE + 128;         // record data bytes
  constexpr int kChunkT = (kWdKeys / 8) * 1024;  // a 64-dim chunk of a tile
  using L = WdSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);  // swizzle atoms: 1 KB
  const int ch = blockIdx.x % a.nchunks;
  const int t = blockIdx.x / a.nchunks;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  auto b_full = [&](int s) { return bar(s); };        // converters -> MMA: tile s written
  auto b_free = [&](int s) { return bar(2 + s); };    // MMA -> converters: PV done with tile s
  const uint32_t b_sfull = bar(4);                     // copies landed in the staging buffer
  const uint32_t b_sempty = bar(5);                    // staging buffer converted
  auto b_sready = [&](int s) { return bar(6 + s); };  // QK -> softmax
  auto b_scons = [&](int s) { return bar(8 + s); };   // softmax holds S[s] in registers
  auto b_pready = [&](int s) { return bar(10 + s); }; // softmax -> PV
  auto b_pvdone = [&](int s) { return bar(12 + s); }; // PV done: P[s] free, O complete to here
  const uint32_t b_drain = bar(14);   // the QK thread's MMAs complete
  const uint32_t b_drain2 = bar(15);  // the PV thread's
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* m_sm = reinterpret_cast<float*>(smem + L::kM);
  float* a_sm = reinterpret_cast<float*>(smem + L::kAlpha);
  uint64_t* meta_c = reinterpret_cast<uint64_t*>(smem + L::kMeta);              // [2][64]
  uint64_t* live_mask = reinterpret_cast<uint64_t*>(smem + L::kMeta + 2 * 64 * 8);  // [2]
  const uint32_t s_tile0 = smem_u32(smem + L::kTile0);
  const uint32_t s_q = smem_u32(smem + L::kQ), s_p = smem_u32(smem + L::kP);

  pdl_wait();
  TC_SPAN(0);
  if (tid == 0) TC_TRACE(62, 0);
  const int kv = a.klen[t];
  const int k0 = ch * a.chunk_keys, k1 = min(k0 + a.chunk_keys, kv);
  const int nsub = k1 > k0 ? (k1 - k0 + kWdKeys - 1) / kWdKeys : 0;

  // ---- Q (f16, swizzled [head][d]; heads past the row's count are zero), barriers, TMEM
  for (int e = tid; e < kWdNH * DG; e += blockDim.x) {
    const int h = e / DG, c = e % DG;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < a.heads) {
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)t * a.heads + h) * D + 8 * c);
      v = make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
    }
    *reinterpret_cast<uint4*>(smem + L::kQ + sw_off<kWdNH>(h, 8 * c)) = v;
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(b_full(s), kWdConv);
      mbar_init(b_free(s), 1);
      mbar_init(b_sready(s), 1);
      mbar_init(b_scons(s), 8);
      mbar_init(b_pready(s), 8);
      mbar_init(b_pvdone(s), 1);
    }
    mbar_init(b_sfull, 1);
    mbar_init(b_sempty, kWdConv);
    mbar_init(b_drain, 1);
    mbar_init(b_drain2, 1);
    *abort = 0;
  }
  if (tid < 64) {
    m_sm[tid] = -INFINITY;
    a_sm[tid] = 0.f;
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  if (tid == 0) TC_TRACE(62, 1);
  // TMEM columns: S^T[s] at 64 s (64 heads); O^T block b at 128 + 64 b
  const uint32_t tm_s = tmem, tm_o = tmem + 128;

  if (warp == 9) {
    // ================= copies (lane l: keys l and 32 + l of a tile) and the PV issue (lane 0)
    // One polling loop over two event streams. Copies: once the converters hold tile jc - 1's
    // records in registers, tile jc's codes and live keys are published and its runs fetched (a
    // key starts a run unless it continues the previous key's record, the next slot of the same
    // page; a run's first lane copies it); then tile jc + 2 is located (its code words loaded) and
    // tile jc + 3's key-table entries loaded, in flight while the loop polls. PVs: once softmax(jp)
    // wrote P, PV(jp) -- its completion frees the tile for the conversion two tiles on.
    const uint32_t id_pv = umma_idesc(128, kWdNH, 1, 1);
    const bool has_b = lane < kWdKeys - 32;
    auto kt_load = [&](int j, int i) {
      const int k = k0 + j * kWdKeys + i;
      return (i < kWdKeys && k < k1) ? a.kt[(size_t)t * a.keys_ld + k] : -1;
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
    // PV(j): O += V^T P^T. A = V^T, MN-major, 128-byte swizzle: a 128-dim block = 2 chunks
    // kChunkT apart (lbo), K step ks = key groups 2 ks, 2 ks + 1 (1 KB apart: sbo); B = P^T.
    // K step outer, dim blocks inner: consecutive MMAs go to different accumulators
    auto issue_pv = [&](int j) {
      TC_TRACE(j, 3);
      tc_fence_after();
      const uint64_t da = umma_sdesc_sw128(s_tile0 + (j & 1) * L::kTileBytes, kChunkT, 1024);
      const uint64_t db0 = umma_sdesc(s_p + (j & 1) * L::kPBytes, (kWdNH / 8) * 128, 128);
      constexpr uint32_t db_step = (uint32_t)(2 * (kWdNH / 8) * 128) >> 4;
#pragma unroll
      for (int ks = 0; ks < kWdKeys / 16; ++ks)
#pragma unroll
        for (int b = 0; b < NBLK; ++b) {
          const int d0 = 128 * b < D - 128 ? 128 * b : D - 128;
          umma_f16(tm_o + 64 * b, da + (uint64_t)(((d0 / 64) * kChunkT + ks * 2048) >> 4),
                   db0 + (uint64_t)(ks * db_step), id_pv, j > 0 || ks > 0);
        }
      umma_commit(b_free(j & 1));    // the tile is free
      umma_commit(b_pvdone(j & 1));  // P[j & 1] free; O holds tiles 0 .. j
      TC_TRACE(j, 9);
    };
    const uint8_t *pa = nullptr, *pb = nullptr, *na = nullptr, *nb = nullptr;
    uint64_t ca = 0, cb = 0, nca = 0, ncb = 0;
    int va = -1, vb = -1;  // key-table entries of the tile after the located ones
    if (nsub > 0) {
      locate(kt_load(0, lane), pa, ca);
      locate(kt_load(0, 32 + lane), pb, cb);
      const int v1a = kt_load(1, lane), v1b = kt_load(1, 32 + lane);
      va = kt_load(2, lane);
      vb = kt_load(2, 32 + lane);
      locate(v1a, na, nca);
      locate(v1b, nb, ncb);
    }
    const uint32_t stage = smem_u32(smem + L::kStage);
    int jc = 0, jp = 0;  // next tile to copy, next tile to PV
    uint32_t idle = 0;
    uint64_t deadline = 0;
    bool ok = true;
    while (ok && (jc < nsub || jp < nsub)) {
      bool progress = false;
      if (jc < nsub) {
        bool go = true;
        if (jc >= 1) {
          go = __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(b_sempty, (jc - 1) & 1) : 0, 0) != 0;
          if (go) go = wd_warp_wait(b_sempty, (jc - 1) & 1, abort);  // (completes at once: each lane's acquire)
        }
        if (go) {
          if (lane == 0) TC_TRACE(jc, 14);
          meta_c[(jc & 1) * 64 + lane] = ca;
          if (has_b) meta_c[(jc & 1) * 64 + 32 + lane] = cb;
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
          const uint64_t brk = (uint64_t)brk_a | ((uint64_t)brk_b << 32);  // bits kWdKeys .. 63 set
          const uint32_t va_mask = __ballot_sync(0xffffffffu, pa != nullptr);
          const uint32_t vb_mask = __ballot_sync(0xffffffffu, has_b && pb != nullptr);
          const uint32_t nvalid = __popc(va_mask) + __popc(vb_mask);
          if (lane == 0) live_mask[jc & 1] = (uint64_t)va_mask | ((uint64_t)vb_mask << 32);
          __syncwarp();
          if (lane == 0) tc_expect_tx(b_sfull, nvalid * (uint32_t)RB);  // (0 bytes: the arrival completes it)
          __syncwarp();
          auto run_copy = [&](int i, const uint8_t* p) {
            const uint64_t above = brk & ~((2ull << i) - 1);
            const int len = __ffsll((long long)above) - 1 - i;
            tc_bulk_load(stage + (uint32_t)(i * RB), p, (uint32_t)(len * RB), b_sfull);
          };
          if (start_a) run_copy(lane, pa);
          if (start_b) run_copy(32 + lane, pb);
          if (lane == 0) TC_TRACE(jc, 15);
          ++jc;
          pa = na;
          pb = nb;
          ca = nca;
          cb = ncb;
          na = nb = nullptr;
          nca = ncb = 0;
          if (jc + 1 < nsub) {  // tile jc + 1 located, tile jc + 2's entries loaded
            locate(va, na, nca);
            locate(vb, nb, ncb);
            va = kt_load(jc + 2, lane);
            vb = kt_load(jc + 2, 32 + lane);
          }
          progress = true;
        }
      }
      if (jp < jc && jp < nsub) {
        // (P(jp) exists only after tile jp was copied, converted and its QK ran)
        const bool rdy = __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_test(b_pready(jp & 1), (jp >> 1) & 1) : 0, 0);
        if (rdy) {
          if (lane == 0) issue_pv(jp);
          __syncwarp();
          ++jp;
          progress = true;
        }
      }
      if (progress) {
        idle = 0;
        deadline = 0;
      } else if ((++idle & 255) == 0) {
        // bounded: another role gave up, or nothing arrived for 2 s
        if (*abort) {
          ok = false;
        } else {
          const uint64_t now = wd_now();
          if (deadline == 0) {
            deadline = now + 2000000000ull;
          } else if (now > deadline) {
            *abort = 1;
            atomicExch(&g_tc_error, 1);
            ok = false;
          }
        }
        ok = __all_sync(0xffffffffu, ok);
      }
    }
    if (lane == 0) {
      // every PV complete before the TMEM is freed (also after an abort)
      umma_commit(b_drain2);
      mbar_wait(b_drain2, 0, abort);
    }
    // no copy may still be landing when the CTA leaves (after an abort the converters stopped
    // consuming): wait, bounded, for the last issued tile's
    if (jc > 0)
      for (uint32_t it = 0; it < kTcWaitPolls && !mbar_try(b_sfull, (jc - 1) & 1); ++it) {
      }
  } else if (warp >= 10) {
    // ================= conversion (warps 10-15): nope item f = (key f / 64, 8-dim unit f % 64),
    // rope item f = (key f / 8, unit f % 8); consecutive lanes on consecutive units of one key
    const int ctid = tid - 32 * 10;
    constexpr int kNU = NOPE / 8;                              // nope units a key
    constexpr int kItems = kWdKeys * kNU / (32 * kWdConv);     // nope items a thread
    constexpr int kRItems = kWdKeys * 8 / (32 * kWdConv);      // rope items a thread
    static_assert(kWdKeys * kNU % (32 * kWdConv) == 0 && kWdKeys * 8 % (32 * kWdConv) == 0, "whole items");
    static_assert(kNU % 32 == 0, "a warp's nope items lie in one key");
    static_assert((32 * kWdConv) % kNU == 0 && (32 * kWdConv) % 8 == 0, "fixed units a thread");
    constexpr int kKStep = 32 * kWdConv / kNU, kRStep = 32 * kWdConv / 8;
    const int u = ctid % kNU, key0 = ctid / kNU;  // nope items: (key0 + kKStep i, unit u)
    const int ru = ctid % 8, rkey0 = ctid / 8;    // rope items: (rkey0 + kRStep i, unit ru)
    const int col_n = (u >> 3) * kChunkT;
    const uint8_t* stg = smem + L::kStage;
    for (int j = 0; j < nsub; ++j) {
      const int s = j & 1;
      if (!wd_warp_wait(b_sfull, j & 1, abort)) break;
      if (ctid == 0) TC_TRACE(j, 4);
      if (j >= 2 && !wd_warp_wait(b_free(s), ((j >> 1) - 1) & 1, abort)) break;
      if (ctid == 0) TC_TRACE(j, 0);
      uint8_t* tile = smem + L::kTile0 + s * L::kTileBytes;
      const uint64_t live = live_mask[s];
      const uint64_t* codes = meta_c + s * 64;  // (written before the copies' arrival, kept two tiles)
      // a thread's nope items share the unit u (32 kWdConv is a multiple of kNU) and step the key
      // by kKStep; its rope items likewise (unit ru, key step kRStep)
      uint2 raw[kItems];
#pragma unroll
      for (int i = 0; i < kItems; ++i)
        raw[i] = *reinterpret_cast<const uint2*>(stg + (key0 + kKStep * i) * RB + 8 * u);
      uint4 rr[kRItems];
#pragma unroll
      for (int i = 0; i < kRItems; ++i)
        rr[i] = *reinterpret_cast<const uint4*>(stg + (rkey0 + kRStep * i) * RB + NOPE + 16 * ru);
      // the records are in registers: the next tile's copies may land while these convert
      __syncwarp();
      if (lane == 0) mbar_arrive(b_sempty);
      if (ctid == 0) TC_TRACE(j, 6);
      // (sw_off of (key, d): 6144 (d / 64) + 128 key + 16 ((d / 8 % 8) ^ (key % 8)))
      const uint8_t* code_b = reinterpret_cast<const uint8_t*>(codes) + (u >> 3);
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int key = key0 + kKStep * i;
        uint4 o = make_uint4(0, 0, 0, 0);
        if ((live >> key) & 1) o = wd_convert8(raw[i], (int)code_b[8 * key]);
        *reinterpret_cast<uint4*>(tile + col_n + 128 * key + (((u & 7) ^ (key & 7)) << 4)) = o;
      }
#pragma unroll
      for (int i = 0; i < kRItems; ++i) {
        const int key = rkey0 + kRStep * i;
        uint4 o = make_uint4(0, 0, 0, 0);
        if ((live >> key) & 1)
          o = make_uint4(bf16x2_to_f16x2(rr[i].x), bf16x2_to_f16x2(rr[i].y), bf16x2_to_f16x2(rr[i].z),
                         bf16x2_to_f16x2(rr[i].w));
        *reinterpret_cast<uint4*>(tile + (NOPE / 64) * kChunkT + 128 * key + ((ru ^ (key & 7)) << 4)) = o;
      }
      fence_async_smem();  // the MMA (async proxy) reads the tile
      __syncwarp();
      if (lane == 0) mbar_arrive(b_full(s));
      if (ctid == 0) TC_TRACE(j, 1);
    }
  } else if (warp == 8) {
    // ================= QK issue (one elected thread): QK(j + 1) goes out as soon as its inputs are
    // ready, so it runs under softmax(j)
    if (lane == 0) {
      const uint32_t id_qk = umma_idesc(64, kWdNH, 0, 0);
      auto issue_qk = [&](int j) {
        TC_TRACE(j, 10);
        const uint32_t dst = tm_s + 64 * (j & 1);
        // K-major, 128-byte swizzle: K step ks = 16 dims, byte 32 (ks % 4) of chunk ks / 4's rows;
        // the descriptors' address fields (16-byte units) advanced from one base each
        const uint64_t da = umma_sdesc_sw128(s_tile0 + (j & 1) * L::kTileBytes, 16, 1024);
        const uint64_t db = umma_sdesc_sw128(s_q, 16, 1024);
#pragma unroll 4
        for (int ks = 0; ks < D / 16; ++ks)
          umma_f16(dst, da + (uint64_t)(((ks >> 2) * kChunkT + (ks & 3) * 32) >> 4),
                   db + (uint64_t)(((ks >> 2) * (kWdNH / 8) * 1024 + (ks & 3) * 32) >> 4), id_qk, ks > 0);
        umma_commit(b_sready(j & 1));
        TC_TRACE(j, 11);
      };
      auto wait_qk = [&](int j) {
        return mbar_wait(b_full(j & 1), (j >> 1) & 1, abort) &&
               (j < 2 || mbar_wait(b_scons(j & 1), ((j - 2) >> 1) & 1, abort));
      };
      // QK(j) once tile j is converted and S[j & 1] is free (softmax(j - 2) holds it in
      // registers); the PVs are warp 9's
      for (int j = 0; j < nsub; ++j) {
        if (!wait_qk(j)) break;
        tc_fence_after();
        issue_qk(j);
      }
      // every issued MMA complete before the TMEM is freed (also after an abort)
      umma_commit(b_drain);
      mbar_wait(b_drain, 0, abort);
    }
  }
  else if (warp < 8) {
    // ================= softmax + epilogue (warps 0-7)
    // Thread (warp w, lane < 16) holds key 16 (w % 4) + lane of a tile (S^T rows of an M = 64 MMA
    // sit on the first 16 lanes of each 32-lane quarter) for heads 32 (w / 4) .. + 31. p = 2^(s - m)
    // against a per-head reference m that moves only when a tile's max passes it by more than
    // 2^kTcSlack: then O and the partial sums are rescaled once. Each key thread keeps its own
    // partial sums of p.
    const int q4 = warp & 3, hb = 32 * (warp >> 2);
    const int key = 16 * q4 + (lane & 15);
    const bool has_key = lane < 16 && key < kWdKeys;  // keys 48 .. 63: the QK's padded rows
    const uint32_t lane_addr = (uint32_t)(32 * q4) << 16;
    float l_part[32];
#pragma unroll
    for (int h = 0; h < 32; ++h) l_part[h] = 0.f;
    bool ok = true;
    // O *= alpha (per head) for this thread's lane (dim) and head half, in every block
    auto rescale_o = [&]() {
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint32_t v[16];
          const uint32_t col = tm_o + 64 * b + lane_addr + hb + 16 * g;
          tmem_ld16(col, v);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = __float_as_uint(__uint_as_float(v[q]) * a_sm[hb + 16 * g + q]);
          tmem_st16(col, v);
        }
      }
      tmem_wait_st();
    };
    auto kt_entry = [&](int j) {
      const int k = k0 + j * kWdKeys + key;
      return (has_key && k < k1) ? a.kt[(size_t)t * a.keys_ld + k] : -1;
    };
    int kt_next = nsub > 0 ? kt_entry(0) : -1;
    for (int j = 0; ok && j < nsub; ++j) {
      const int s = j & 1;
      const int kv_ = kt_next;
      kt_next = j + 1 < nsub ? kt_entry(j + 1) : -1;
      const bool valid = kv_ != -1 && (kv_ >= 0 || a.comp != nullptr);
      ok = wd_all(wd_warp_wait(b_sready(s), (j >> 1) & 1, abort));
      if (!ok) break;
      if (tid == 0) TC_TRACE(j, 5);
      tc_fence_after();
      float sv[32];
      {
        uint32_t v[32];
        const uint32_t ts = tm_s + 64 * s + lane_addr + hb;
        tmem_ld16(ts, *reinterpret_cast<uint32_t(*)[16]>(v));
        tmem_ld16(ts + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_wait_ld();
        // S[s] is in registers: QK(j + 2) may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_scons(s));
        if (tid == 0) TC_TRACE(j, 8);
#pragma unroll
        for (int q = 0; q < 32; ++q) sv[q] = valid ? __uint_as_float(v[q]) * a.scale_log2 : -INFINITY;
      }
      // the reference max moves only when a score passes it by more than the slack: only then the
      // tile's per-head max, over the 16 key lanes and then the 4 warps of the head half (red)
      bool exceed = false;
#pragma unroll
      for (int q = 0; q < 32; q += 4) {
        const float4 m4 = *reinterpret_cast<const float4*>(m_sm + hb + q);
        exceed |= (sv[q] > m4.x + kTcSlack) | (sv[q + 1] > m4.y + kTcSlack) | (sv[q + 2] > m4.z + kTcSlack) |
                  (sv[q + 3] > m4.w + kTcSlack);
      }
      bool rescale = false;
      if (wd_any(exceed)) {
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const float x = warp_max_f32(sv[q]);  // (lanes 16 .. 31 hold no key: -inf)
          if (lane == q) red[warp * 32 + q] = x;
        }
        wd_bar();  // red complete
        bool moved = false;  // a head's reference moved while O already holds its sums
        if (tid < kWdNH) {
          const int w0 = 4 * (tid >> 5), hq = tid & 31;
          const float bx = fmaxf(fmaxf(red[w0 * 32 + hq], red[(w0 + 1) * 32 + hq]),
                                 fmaxf(red[(w0 + 2) * 32 + hq], red[(w0 + 3) * 32 + hq]));
          const float mu = m_sm[tid];
          float al = 1.f;
          if (bx > mu + kTcSlack) {
            al = (mu == -INFINITY) ? 0.f : exp2f(mu - bx);
            moved = mu != -INFINITY;
            m_sm[tid] = bx;
          }
          a_sm[tid] = al;
        }
        rescale = wd_any(moved) && j > 0;  // also publishes m_sm / a_sm
      }
      if (rescale) {
        // O must hold every issued PV before it is scaled
        ok = wd_all(wd_warp_wait(b_pvdone((j - 1) & 1), ((j - 1) >> 1) & 1, abort));
        if (!ok) break;
        tc_fence_after();
        rescale_o();
        tc_fence_before();
#pragma unroll
        for (int q = 0; q < 32; ++q) l_part[q] *= a_sm[hb + q];
      }
      // P^T[s] is free once PV(j - 2) is done
      if (j >= 2) {
        ok = wd_all(wd_warp_wait(b_pvdone(s), ((j - 2) >> 1) & 1, abort));
        if (!ok) break;
      }
      if (tid == 0) TC_TRACE(j, 13);
      // p' = 2^(s - m + 7) into P^T[s] as one f16 (<= 2^15), 8 heads (16 bytes) at a time; this
      // thread's partial sums of p'. P^T [key group][head group][8 keys][8 heads]: this half's
      // head groups hb / 8 ..
      uint8_t* prow = smem + L::kP + s * L::kPBytes + ((key >> 3) * (kWdNH / 8) + hb / 8) * 128 + (key & 7) * 16;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t hw[4];
#pragma unroll
        for (int q = 8 * g; q < 8 * g + 8; q += 4) {
          const float4 m4 = *reinterpret_cast<const float4*>(m_sm + hb + q);
          const float mq[4] = {m4.x, m4.y, m4.z, m4.w};
          float pq[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            pq[i] = sv[q + i] == -INFINITY ? 0.f : ex2_approx(sv[q + i] - mq[i] + kWdShift);
            l_part[q + i] += pq[i];
          }
          hw[(q - 8 * g) / 2] = cvt_f16x2(pq[0], pq[1]);
          hw[(q - 8 * g) / 2 + 1] = cvt_f16x2(pq[2], pq[3]);
        }
        if (has_key) *reinterpret_cast<uint4*>(prow + g * 128) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      }
      if (tid == 0) TC_TRACE(j, 12);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b_pready(s));
      if (tid == 0) TC_TRACE(j, 7);
    }
    // ---- epilogue: every PV done, then O^T and (m - 7, l) of the chunk
    if (ok && nsub > 0) ok = wd_all(wd_warp_wait(b_pvdone((nsub - 1) & 1), ((nsub - 1) >> 1) & 1, abort));
    const size_t base = ((size_t)t * a.nchunks + ch) * a.heads;
    const int nh = min(kWdNH, a.heads);
    if (ok && nsub > 0) {
      tc_fence_after();
      // l: the partial sums of the 64 key threads of each head half, lane q taking head hb + q
#pragma unroll
      for (int h = 0; h < 32; ++h)
        if (!has_key) l_part[h] = 0.f;
      warp_transpose_sum(l_part, lane);
      red[warp * 32 + lane] = l_part[0];
      wd_bar();
      if (tid < nh) {
        const int w0 = 4 * (tid >> 5), hq = tid & 31;
        a.part_ml[(base + tid) * 2] = m_sm[tid] - kWdShift;
        a.part_ml[(base + tid) * 2 + 1] =
            (red[w0 * 32 + hq] + red[(w0 + 1) * 32 + hq]) + (red[(w0 + 2) * 32 + hq] + red[(w0 + 3) * 32 + hq]);
      }
      const int dl = 32 * q4 + lane;  // this thread's dim within a block
#pragma unroll 1
      for (int b = 0; b < NBLK; ++b) {
        const int d0 = min(128 * b, D - 128);
        const int d = d0 + dl;
        const bool own = d >= 128 * b;  // the overlapping last block writes only its new dims
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          uint32_t v[16];
          tmem_ld16(tm_o + 64 * b + lane_addr + hb + 16 * g, v);
          tmem_wait_ld();
          if (own)
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (hb + 16 * g + q < nh) a.part_o[(base + hb + 16 * g + q) * D + d] = __uint_as_float(v[q]);
        }
      }
    } else if (nsub == 0 && tid < nh) {
      a.part_ml[(base + tid) * 2] = -INFINITY;
      a.part_ml[(base + tid) * 2 + 1] = 0.f;
    }
  }
  // ---- teardown: every role done (a timed-out one unwound); free the TMEM
  if (tid == 0) TC_TRACE(63, 2);
  tc_fence_before();
  __syncthreads();
  if (tid == 0) TC_TRACE(63, 3);
  if (warp == 8) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  TC_SPAN(1);
  pdl_launch();
}

}  // namespace dsv41
