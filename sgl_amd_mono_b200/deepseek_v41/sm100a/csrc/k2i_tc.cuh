// K2i's FP4 scorer on the 5th-generation tensor cores (score_fp4.py:221-441 of the reference):
// the same logits contract as k2i_score_kernel (bit for bit), with the integer chunk dots on
// tcgen05.mma.kind::mxf4.block_scale (block32) and the fp64 work mostly folded away.
//
// Operands, per 128-key tile: A = the keys (M = 128 rows, K = 128 dims of packed E2M1, K-major
// core matrices of 8 rows x 16 B: [chunk][key][16 B]), B = one row's query heads (N = heads, the
// same form); the E8M0 codes enter as the MMA's block scales (one per 32 dims), taken relative to
// each key's and each head's smallest code:
//   fast tile: D[k][h] = sum_c 2^(ke_kc - kref_k) 2^(qe_hc - qref_h) dot_c(k, h) in ONE accumulator,
//              exact when (max code spread of the tile's keys) + (of the piece's heads) <= 6:
//              every product is a multiple of 1/4 and |D| < 4608 * 2^6 < 2^19, so each partial sum
//              is an fp32 value and D has at most 21 significant bits. Then x_h = D 2^(qref_h +
//              kref_k - 254) exactly -- the oracle's fp64 chunk sum is exact too. The head sum:
//              * integer rows (the row's nonzero weights w_h = mw_h 2^ew_h span at most 18 in
//                E_h = ew_h + qref_h): T_h = 4 relu(D) < 2^21 and mult_h = +-mw_h 2^(E_h - Emin)
//                < 2^26, so sum_h mult_h T_h < 2^53 -- every partial sum of the contract's fp64
//                order is exact, the result is the exact sum, computed in int64 and rounded once;
//              * other rows: t = D + |D| (= 2 relu(D)) reinterpreted by a 3-bit shift of its fp32
//                bits is the fp64 t 2^-896 (its low word is zero); the contract's fp64 operations
//                in its order, scaled by 2^-(512 + kref_k): s_g = fma(w_h 2^(qref_h + 129),
//                t 2^-896, s_g) is RN(s_g + w_h x_h) scaled (the product is exact), the tree adds
//                likewise, and the final scale back is exact; nothing leaves fp64's normal range,
//                so the rounding is the oracle's.
//   slow tile: one accumulator a chunk (unit scales; the instruction's second K half multiplies a
//              zero chunk): D_c = dot_c exactly; the epilogue runs the contract's fp64 sequence
//              itself (x_h = sum_c D_c 2^(qe + ke - 254) in order, relu, s_g = s_g + w_h x_h with
//              separate rounding, the tree).
// Pieces (rows sharing a page table) put each row's item on the same key tile.
//
// CTA (one an SM, 14 warps): warps 0-7 the epilogue (two warpgroups taking alternate tiles; thread
// = TMEM lane = key), warps 8-11 the converters (thread = key: staged raw -> the tile, the codes ->
// kref / spread / the A scale atom), warp 12 the bulk copies of raw keys and codes into a 4-stage
// ring (and the TMEM allocation), warp 13 the MMA issue (one thread). TMEM: 7 accumulator slots
// of 64 columns (a fast item takes one, a slow item four), then the scale atoms. Every wait is
// bounded and parks the thread; a timeout sets the device error word and unwinds every role.
#pragma once

#include "attn_tc.cuh"
#include "attn_wide.cuh"
#include "k2i.cuh"
#include "moe_tc.cuh"

namespace dsv41 {

constexpr int kKtThreads = 448;   // 14 warps
constexpr int kKtStages = 4;      // raw key stages
constexpr int kKtBufs = 3;        // key tiles
constexpr int kKtMeta = 4;        // tile metadata ring (converters -> epilogue)
constexpr int kKtSlots = 7;       // TMEM accumulator slots of 64 columns
constexpr int kKtMaxSpan = kIdxMaxSpan;
constexpr int kKtFastSpread = 6;  // code spread bound of the folded-scale path
constexpr int kKtIntSpread = 18;  // exponent spread bound of a row's integer head sum
constexpr int kKtEntries = 2048;  // page-table entries a task caches in shared memory

struct KtSmem {
  static constexpr int kTileBytes = 4 * 128 * 16;           // [chunk][128 keys][16 B] packed E2M1
  static constexpr int kA = 0;                              // kKtBufs tiles
  static constexpr int kQBytes = 4 * 64 * 16;               // [chunk][64 heads][16 B], the same form
  static constexpr int kQ = kA + kKtBufs * kTileBytes;      // kKtMaxSpan rows, then a zero chunk
  static constexpr int kZero = kQ + kKtMaxSpan * kQBytes;   // 64 x 16 B of zeros
  static constexpr int kStKeys = 4 * 128 * 16;              // raw E2M1 of a tile's keys
  static constexpr int kStScales = 4 * 16 * 32;             // their codes
  static constexpr int kStMeta = 16 * 4;                    // [block] slot base | valid keys << 8
  static constexpr int kStBytes = kStKeys + kStScales + kStMeta;
  static constexpr int kSt = kZero + 1024;                  // kKtStages stages
  static constexpr int kSfA = kSt + kKtStages * kStBytes;   // kKtBufs A scale atoms (512 B)
  static constexpr int kSfB = kSfA + kKtBufs * 512;         // kKtMaxSpan B atoms, then the unit atom
  // a tile's codes [128] u32, kref [128] u8, then u32 flags: fast, first accumulator slot
  static constexpr int kMetaBytes = 128 * 4 + 128 + 16;
  static constexpr int kMeta = kSfB + (kKtMaxSpan + 1) * 512;
  static constexpr int kW3 = kMeta + kKtMeta * kMetaBytes;  // double [span][64]: w 2^(qref + 129)
  static constexpr int kW = kW3 + kKtMaxSpan * 64 * 8;      // double [span][64]: w
  static constexpr int kQe = kW + kKtMaxSpan * 64 * 8;      // u32 [span][64]: the 4 codes of a head
  static constexpr int kMult = kQe + kKtMaxSpan * 64 * 4;   // int [span][64]: integer head weights
  static constexpr int kEnt = kMult + kKtMaxSpan * 64 * 4;  // int [kKtEntries]: page-table entries
  static constexpr int kRed = kEnt + kKtEntries * 4;        // ints (see the kernel)
  static constexpr int kBar = kRed + 256;
  static constexpr int kNumBars = 2 * kKtStages + 2 * kKtBufs + 2 * kKtMeta + 2 * kKtSlots + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;         // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16 + 1024;          // + slack to align the base to 1 KB
  static_assert(kSt % 1024 == 0 && kStBytes % 16 == 0 && kSfA % 16 == 0, "alignment");
  static_assert(kMetaBytes % 16 == 0 && kW3 % 16 == 0 && kMult % 16 == 0, "alignment");
  static_assert(kBytes <= 232448, "shared memory of one CTA");
};

// kind::mxf4 instruction descriptor (block32: two E8M0 scales a row an instruction, K = 64): A and B
// E2M1 (format 1), K-major both, M = 128, N; scale-factor ids = the first of the two bytes used
__device__ __forceinline__ uint32_t kt_idesc(int id, int N) {
  return ((uint32_t)id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(128 >> 4) << 24) | ((uint32_t)id << 29);
}
__device__ __forceinline__ void kt_mma(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc,
                                       uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb));
}
// K-major, no swizzle: core matrices of 8 rows x 16 B (128 B contiguous), 8-row groups sbo apart,
// the instruction's two 16-byte K halves lbo apart
__device__ __forceinline__ uint64_t kt_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return umma_sdesc(addr, lbo, sbo);
}
// Bounded waits that park the thread (try_wait with a suspend-time hint, so the roles that mostly
// wait leave the issue slots to the MMA thread and the epilogue; 2 s %globaltimer deadline)
__device__ __forceinline__ bool kt_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  return wd_wait(bar, parity, abort);
}
__device__ __forceinline__ bool kt_warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, wd_wait(bar, parity, abort));
}
// AND over the 128 converter threads (named barrier 2)
__device__ __forceinline__ bool kt_conv_all(bool v) {
  uint32_t r;
  asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.and.pred q, 2, 128, p;\n\t"
               "selp.u32 %0, 1, 0, q;\n\t}\n"
               : "=r"(r) : "r"((uint32_t)v) : "memory");
  return r != 0;
}
// 2^e as a double (e within the normal range)
__device__ __forceinline__ double kt_pow2(int e) { return __hiloint2double((e + 1023) << 20, 0); }
// Staged raw bytes of key k (slot s of its page), chunk c. Whole plane pages: [page][chunk][slot]
// [16 B] and the page's codes [page][chunk][64 B] (one copy each a page); 8-key table blocks:
// [chunk][key][16 B] and [chunk][block][32-byte window of the page's 64 codes].
__device__ __forceinline__ int kt_key_off(bool full, int k, int c) {
  return full ? (k >> 6) * 4096 + c * 1024 + (k & 63) * 16 : c * 2048 + k * 16;
}
__device__ __forceinline__ int kt_scale_off(bool full, int k, int s, int c) {
  return full ? (k >> 6) * 256 + c * 64 + (s & 15) * 4 + (s >> 4)
              : c * 512 + (k >> 3) * 32 + (s & 7) * 4 + (s >> 4);
}

__global__ void __launch_bounds__(kKtThreads, 1) k2i_tc_kernel(const K2iArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  using L = KtSmem;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.heads;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  auto st_full = [&](int s) { return bar(s); };
  auto st_empty = [&](int s) { return bar(kKtStages + s); };
  auto a_full = [&](int b) { return bar(2 * kKtStages + b); };
  auto a_free = [&](int b) { return bar(2 * kKtStages + kKtBufs + b); };
  auto m_full = [&](int m) { return bar(2 * kKtStages + 2 * kKtBufs + m); };
  auto m_free = [&](int m) { return bar(2 * kKtStages + 2 * kKtBufs + kKtMeta + m); };
  auto s_ready = [&](int s) { return bar(2 * kKtStages + 2 * kKtBufs + 2 * kKtMeta + s); };
  auto s_free = [&](int s) { return bar(2 * kKtStages + 2 * kKtBufs + 2 * kKtMeta + kKtSlots + s); };
  const uint32_t drain = bar(L::kNumBars - 1);
  uint32_t* tmem_base = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  int* red = reinterpret_cast<int*>(smem + L::kRed);
  double* s_w3 = reinterpret_cast<double*>(smem + L::kW3);
  double* s_w = reinterpret_cast<double*>(smem + L::kW);
  uint32_t* s_qe = reinterpret_cast<uint32_t*>(smem + L::kQe);
  int* s_mult = reinterpret_cast<int*>(smem + L::kMult);
  int* s_ent = reinterpret_cast<int*>(smem + L::kEnt);
  // red: [0, 8) converter spreads (2 tiles x 4 warps), [8] the heads' code spread, [16 + r] row r's
  // smallest / [24 + r] largest weight exponent E, [32 + r] a non-finite weight, [40 + r] its bound

  pdl_wait();
  if (tid == 0) TC_TRACE(63, 0);
  // ---- the task: rows lead .. lead + span - 1 of one page table, key tiles ch0 .. ch1 - 1
  int lead, span, ch0, ch1;
  if (a.reindex) {
    const int per = max(1, (int)gridDim.x / a.rows);
    const int row = blockIdx.x / per, i = blockIdx.x % per;
    if (row >= a.rows) return;
    lead = row;
    span = 1;
    ch0 = i * a.reindex_chunks / per;
    ch1 = (i + 1) * a.reindex_chunks / per;
  } else {
    lead = a.plan[4 * blockIdx.x];
    span = a.plan[4 * blockIdx.x + 1];
    ch0 = a.plan[4 * blockIdx.x + 2];
    ch1 = a.plan[4 * blockIdx.x + 3];
  }
  if (span <= 0 || span > kKtMaxSpan || ch0 >= ch1) return;
  const int owner = a.owners[lead];
  int piece_bound = 0;
  for (int r = 0; r < span; ++r) piece_bound = max(piece_bound, a.bounds[lead + r]);
  const int nt = min(ch1, cdiv(piece_bound, kIdxChunk)) - ch0;  // key tiles with visible columns
  if (nt <= 0) return;
  const bool full_pages = a.entry_rows == kPlaneRows;

  // ---- barriers, TMEM and the shared scalars; then the copies start while the other warps stage
  // the piece's queries, their codes, weights and scale atoms, and each row's integer head weights:
  // w_h = mw_h 2^ew_h (mw_h the 8-bit significand), E_h = ew_h + qref_h, mult_h = +-mw_h 2^(E_h - Emin)
  // when the row's nonzero weights span at most kKtIntSpread in E
  if (tid < 8) {
    red[8 + tid] = 0;
    red[16 + tid] = 1 << 20;
    red[24 + tid] = -(1 << 20);
    red[32 + tid] = 0;
    red[40 + tid] = tid < span ? a.bounds[lead + tid] : 0;
  }
  if (tid == 0) {
    for (int s = 0; s < kKtStages; ++s) {
      mbar_init(st_full(s), 1);
      mbar_init(st_empty(s), 4);
    }
    for (int b = 0; b < kKtBufs; ++b) {
      mbar_init(a_full(b), 4);
      mbar_init(a_free(b), 1);
    }
    for (int m = 0; m < kKtMeta; ++m) {
      mbar_init(m_full(m), 4);
      mbar_init(m_free(m), 4);
    }
    for (int s = 0; s < kKtSlots; ++s) {
      mbar_init(s_ready(s), 1);
      mbar_init(s_free(s), 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 12) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  if (tid == 0) TC_TRACE(63, 1);
  // TMEM columns: accumulator slot s at 64 s; the unit scale atom at 448, A atoms 452 + 4 b, B atoms
  // 464 + 4 r (each scale operand on a 4-column boundary)
  const uint32_t t_sfu = tmem + 448, t_sfa = tmem + 452, t_sfb = tmem + 464;
  // every warp but the copy warp (12): thread pt of np, named barrier 3
  const int np = (int)blockDim.x - 32, pt = warp < 12 ? tid : tid - 32;
  auto rest_bar = [&]() { asm volatile("bar.sync 3, %0;" ::"r"(np) : "memory"); };
  if (warp != 12) {
    for (int e = pt; e < span * H; e += np) {
      const int r = e / H, h = e % H, row = lead + r;
      uint32_t codes = 0;
      int qref = 255, qmax = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int q = a.qscale[(size_t)row * 256 + c * 64 + (h % 16) * 4 + h / 16];
        codes |= (uint32_t)q << (8 * c);
        qref = min(qref, q);
        qmax = max(qmax, q);
      }
      const __nv_bfloat16 wbf = a.w[(size_t)row * H + h];
      const double w = (double)bf2f(wbf);
      {
        const uint32_t wb = __bfloat16_as_ushort(wbf);
        const int e8 = (int)((wb >> 7) & 0xffu), mw = e8 ? 128 + (int)(wb & 0x7fu) : (int)(wb & 0x7fu);
        if (e8 == 255) red[32 + r] = 1;
        if (mw != 0) {
          atomicMin(&red[16 + r], (e8 ? e8 - 134 : -133) + qref);
          atomicMax(&red[24 + r], (e8 ? e8 - 134 : -133) + qref);
        }
      }
      s_w[r * 64 + h] = w;
      s_w3[r * 64 + h] = __dmul_rn(w, kt_pow2(qref + 129));
      s_qe[r * 64 + h] = codes;
      atomicMax(&red[8], qmax - qref);
      uint32_t sb = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        sb |= (uint32_t)(127 + min((int)((codes >> (8 * c)) & 0xffu) - qref, kKtFastSpread)) << (8 * c);
      *reinterpret_cast<uint32_t*>(smem + L::kSfB + r * 512 + (h % 32) * 16 + (h / 32) * 4) = sb;
      const uint4* src = reinterpret_cast<const uint4*>(a.q + ((size_t)row * H + h) * 64);
      uint8_t* qrow = smem + L::kQ + r * L::kQBytes;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(qrow + c * 1024 + h * 16) = src[c];
    }
    for (int i = pt; i < 128; i += np) {
      reinterpret_cast<uint32_t*>(smem + L::kSfB + kKtMaxSpan * 512)[i] = 0x7f7f7f7fu;  // unit scales
      reinterpret_cast<uint2*>(smem + L::kZero)[i] = make_uint2(0, 0);
    }
    rest_bar();
    for (int e = pt; e < span * H; e += np) {
      const int r = e / H, h = e % H;
      const uint32_t wb = __bfloat16_as_ushort(a.w[(size_t)(lead + r) * H + h]);
      const uint32_t codes = s_qe[r * 64 + h];
      const int qref = min(min((int)(codes & 0xffu), (int)((codes >> 8) & 0xffu)),
                           min((int)((codes >> 16) & 0xffu), (int)(codes >> 24)));
      const int e8 = (int)((wb >> 7) & 0xffu), mw = e8 ? 128 + (int)(wb & 0x7fu) : (int)(wb & 0x7fu);
      const bool row_int = red[32 + r] == 0 && red[24 + r] - red[16 + r] <= kKtIntSpread;
      int m = 0;
      if (row_int && mw != 0) m = (mw << ((e8 ? e8 - 134 : -133) + qref - red[16 + r])) * ((wb >> 15) ? -1 : 1);
      s_mult[r * 64 + h] = m;
    }
    fence_async_smem();  // the queries and scale atoms are read by the MMA (async proxy)
    rest_bar();
  }
  const int qspread = red[8];  // the piece's largest head code spread (read after rest_bar)

  if (warp == 12) {
    // ================= copies: tile j's raw keys and codes into stage j % kKtStages. Lane b (< 16)
    // locates 8-key block b (its table entry, page, first slot, visible keys). The task's table
    // entries are contiguous: cp.async first brings them into shared memory (those of the first 4
    // tiles as one group, the rest as another), so no tile waits on a table load; a task with more
    // than kKtEntries of them reads the table directly.
    // Plane pages (64 keys an entry): a page's 4 chunks (4 KB) and its codes (256 B), one copy each;
    // 8-key table blocks: a block's chunk c is 128 B, its codes a 32-byte window of the page's 64.
    const int e_lo = (ch0 * kIdxChunk) / a.entry_rows;
    const int e_hi = min(a.itab_len, cdiv(min(piece_bound, (ch0 + nt) * kIdxChunk), a.entry_rows));
    const bool cached = e_hi - e_lo <= kKtEntries;
    const int* trow = a.itab + (size_t)owner * a.itab_stride;
    if (cached) {
      const int e_first = min(e_hi, cdiv(min(piece_bound, (ch0 + 4) * kIdxChunk), a.entry_rows));
      auto fetch = [&](int f0, int f1) {
        for (int e = f0 + lane; e < f1; e += 32)
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(s_ent + (e - e_lo))),
                       "l"(trow + e)
                       : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
      fetch(e_lo, e_first);
      fetch(e_first, e_hi);
    }
    int issued = 0;
    for (int j = 0; j < nt; ++j) {
      const int st = j % kKtStages;
      if (j >= kKtStages && !kt_warp_wait(st_empty(st), ((j / kKtStages) - 1) & 1, abort)) break;
      if (lane == 0) TC_TRACE(j, 0);
      if (cached && (j == 0 || j == 4)) {
        // tiles 0 .. 3: the first group landed; tile 4 on: every entry
        if (j == 0) asm volatile("cp.async.wait_group 1;" ::: "memory");
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
      }
      int page = 0, s0 = 0, nv = 0;
      {
        const int col = (ch0 + j) * kIdxChunk + 8 * (lane & 15);
        if (col < piece_bound && col / a.entry_rows < a.itab_len) {
          const int ei = col / a.entry_rows;
          const int entry = cached ? s_ent[ei - e_lo] : trow[ei];
          const long vrow = (long)entry * a.entry_rows + col % a.entry_rows;
          nv = min(8, piece_bound - col);
          page = (int)(vrow / kPlaneRows);
          s0 = (int)(vrow % kPlaneRows);
        }
      }
      uint8_t* stg = smem + L::kSt + st * L::kStBytes;
      const uint32_t s_stg = smem_u32(stg);
      if (lane < 16) reinterpret_cast<uint32_t*>(stg + L::kStKeys + L::kStScales)[lane] = (uint32_t)s0 | ((uint32_t)nv << 8);
      // full pages: lane p (< 2) copies page p (its 4 chunks, then its codes); blocks: lane l copies
      // chunks 2 (l / 16), + 1 of block l % 16
      const int src_lane = full_pages ? ((lane & 1) << 3) : (lane & 15);
      const int pg = __shfl_sync(0xffffffffu, page, src_lane);
      const int sb = __shfl_sync(0xffffffffu, s0, src_lane);
      const int nb = __shfl_sync(0xffffffffu, nv, src_lane);
      uint32_t bytes;
      if (full_pages) {
        const int n0 = __shfl_sync(0xffffffffu, nv, 0), n1 = __shfl_sync(0xffffffffu, nv, 8);
        bytes = (uint32_t)((n0 > 0) + (n1 > 0)) * (4096u + 256u);
      } else {
        bytes = (uint32_t)__popc(__ballot_sync(0xffffffffu, lane < 16 && nv > 0)) * 4u * (128u + 32u);
      }
      __syncwarp();
      if (lane == 0) tc_expect_tx(st_full(st), bytes);  // (0 bytes: the arrival completes it)
      __syncwarp();
      if (full_pages) {
        if (lane < 2 && nb > 0) {
          tc_bulk_load(s_stg + lane * 4096, a.payload + (size_t)pg * 4 * kPlaneRows * 16, 4096, st_full(st));
          tc_bulk_load(s_stg + L::kStKeys + lane * 256, a.kscale + (size_t)pg * 4 * kPlaneRows, 256, st_full(st));
        }
      } else if (nb > 0) {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * (lane >> 4) + cc, b = lane & 15;
          tc_bulk_load(s_stg + c * 2048 + b * 128, a.payload + (((size_t)pg * 4 + c) * kPlaneRows + sb) * 16, 128,
                       st_full(st));
          tc_bulk_load(s_stg + L::kStKeys + c * 512 + b * 32,
                       a.kscale + ((size_t)pg * 4 + c) * kPlaneRows + 32 * ((sb & 15) >> 3), 32, st_full(st));
        }
      }
      issued = j + 1;
      if (lane == 0) TC_TRACE(j, 1);
    }
    // no copy may still be landing when the CTA leaves (after an abort the converters stopped
    // consuming): wait, bounded, for the last stages issued
    if (lane == 0)
      for (int k = max(0, issued - kKtStages); k < issued; ++k)
        for (uint32_t it = 0; it < kTcWaitPolls && !mbar_try(st_full(k % kKtStages), (k / kKtStages) & 1); ++it) {
        }
    __syncwarp();
  } else if (warp >= 8 && warp < 12) {
    // ================= converters: thread k holds key k of the tile; the running count of
    // accumulator slots (a fast tile takes one a row, a slow tile four) goes into each tile's meta
    const int k = tid - 256, wc = warp - 8;
    int nslot = 0;
    for (int j = 0; j < nt; ++j) {
      const int st = j % kKtStages;
      bool ok = kt_warp_wait(st_full(st), (j / kKtStages) & 1, abort);
      if (k == 0) TC_TRACE(j, 2);
      uint4 raw[4];
      uint32_t codes = 0x7f7f7f7fu;
      int kref = 127, kspread = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) raw[c] = make_uint4(0, 0, 0, 0);
      if (ok) {
        const uint8_t* stg = smem + L::kSt + st * L::kStBytes;
        const uint32_t mw = reinterpret_cast<const uint32_t*>(stg + L::kStKeys + L::kStScales)[k >> 3];
        const int sb = (int)(mw & 0xffu), nvb = (int)((mw >> 8) & 0xffu);
        if ((k & 7) < nvb) {
          const int s = sb + (k & 7);
          int mn = 255, mx = 0;
          codes = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            raw[c] = *reinterpret_cast<const uint4*>(stg + kt_key_off(full_pages, k, c));
            const int code = stg[L::kStKeys + kt_scale_off(full_pages, k, s, c)];
            codes |= (uint32_t)code << (8 * c);
            mn = min(mn, code);
            mx = max(mx, code);
          }
          kref = mn;
          kspread = mx - mn;
        }
        // the stage is free once the warp's keys are in registers
        __syncwarp();
        if (lane == 0) mbar_arrive(st_empty(st));
      }
      const int wmax = __reduce_max_sync(0xffffffffu, kspread);
      if (lane == 0) red[(j & 1) * 4 + wc] = wmax;
      if (!kt_conv_all(ok)) break;
      if (k == 0) TC_TRACE(j, 3);
      const int* rj = red + (j & 1) * 4;
      const int ks = max(max(rj[0], rj[1]), max(rj[2], rj[3]));
      const bool fast = ks + qspread <= kKtFastSpread;
      const int b = j % kKtBufs, m = j % kKtMeta;
      ok = (j < kKtBufs || kt_warp_wait(a_free(b), ((j / kKtBufs) - 1) & 1, abort)) &&
           (j < kKtMeta || kt_warp_wait(m_free(m), ((j / kKtMeta) - 1) & 1, abort));
      if (!kt_conv_all(ok)) break;
      if (k == 0) TC_TRACE(j, 4);
      uint8_t* tile = smem + L::kA + b * L::kTileBytes;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(tile + c * 2048 + k * 16) = raw[c];
      uint32_t sa = 0x7f7f7f7fu;
      if (fast) {
        sa = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) sa |= (uint32_t)(127 + (int)((codes >> (8 * c)) & 0xffu) - kref) << (8 * c);
      }
      *reinterpret_cast<uint32_t*>(smem + L::kSfA + b * 512 + (k % 32) * 16 + (k / 32) * 4) = sa;
      uint8_t* meta = smem + L::kMeta + m * L::kMetaBytes;
      reinterpret_cast<uint32_t*>(meta)[k] = codes;
      meta[512 + k] = (uint8_t)kref;
      if (k == 0) {
        *reinterpret_cast<uint32_t*>(meta + 640) = fast ? 1u : 0u;
        *reinterpret_cast<uint32_t*>(meta + 644) = (uint32_t)nslot;
      }
      nslot += span * (fast ? 1 : 4);
      fence_async_smem();  // the tile and its scale atom are read by the MMA (async proxy)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(a_full(b));
        mbar_arrive(m_full(m));
      }
      if (k == 0) TC_TRACE(j, 5);
    }
  } else if (warp == 13) {
    // ================= MMA issue (one thread): per tile, each row of the piece -- fast: 2 K = 64
    // instructions into one slot with the tile's and the row's relative scales; slow: each chunk into
    // its own slot with unit scales
    if (lane == 0) {
      for (int r = 0; r < span; ++r) mx_cp_sf(t_sfb + 4 * r, smem_u32(smem + L::kSfB + r * 512));
      mx_cp_sf(t_sfu, smem_u32(smem + L::kSfB + kKtMaxSpan * 512));
      // descriptors built once, advanced by their 16-byte address field
      const uint64_t da0 = kt_sdesc(smem_u32(smem + L::kA), 2048, 128);
      const uint64_t db0 = kt_sdesc(smem_u32(smem + L::kQ), 1024, 128);
      const uint32_t id0 = kt_idesc(0, H), id2 = kt_idesc(2, H);
      const uint32_t s_zero = smem_u32(smem + L::kZero);
      int n = 0;
      bool ok = true;
      for (int j = 0; ok && j < nt; ++j) {
        const int b = j % kKtBufs;
        if (!(ok = kt_wait(a_full(b), (j / kKtBufs) & 1, abort))) break;
        TC_TRACE(j, 6);
        tc_fence_after();
        const bool fast =
            *reinterpret_cast<volatile const uint32_t*>(smem + L::kMeta + (j % kKtMeta) * L::kMetaBytes + 640) != 0;
        const uint64_t da = da0 + (uint64_t)((b * L::kTileBytes) >> 4);
        if (fast) mx_cp_sf(t_sfa + 4 * b, smem_u32(smem + L::kSfA + b * 512));
        for (int r = 0; ok && r < span; ++r) {
          const uint32_t sq = smem_u32(smem + L::kQ + r * L::kQBytes);
          const int parts = fast ? 1 : 4;
          for (int p = 0; p < parts; ++p, ++n) {
            const int s = n % kKtSlots;
            if (n >= kKtSlots && !(ok = kt_wait(s_free(s), ((n / kKtSlots) - 1) & 1, abort))) break;
            tc_fence_after();
            const uint32_t d = tmem + 64 * s;
            if (fast) {
              // chunks 0, 1 then 2, 3: their scale bytes 0, 1 then 2, 3
              const uint64_t db = db0 + (uint64_t)((r * L::kQBytes) >> 4);
              kt_mma(d, da, db, id0, 0, t_sfa + 4 * b, t_sfb + 4 * r);
              kt_mma(d, da + (4096 >> 4), db + (2048 >> 4), id2, 1, (t_sfa + 4 * b) | (2u << 30),
                     (t_sfb + 4 * r) | (2u << 30));
            } else {
              // chunk p alone: the query operand's second K half is the zero chunk (the key tile's
              // second half, chunk p + 1 or what follows the tile in shared memory, meets zeros)
              kt_mma(d, da + (uint64_t)((2048 * p) >> 4), kt_sdesc(sq + 1024 * p, s_zero - (sq + 1024 * p), 128),
                     id0, 0, t_sfu, t_sfu);
            }
            umma_commit(s_ready(s));
          }
        }
        if (!ok) break;
        umma_commit(a_free(b));
        TC_TRACE(j, 7);
      }
      // every issued MMA (and scale copy) complete before the TMEM is freed
      umma_commit(drain);
      mbar_wait(drain, 0, abort);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ================= epilogue: two warpgroups, tiles j = wg, wg + 2, ...; thread = key (TMEM lane)
    // of the tile; per row, the head sum (integer rows exactly, other rows in the contract's fp64
    // order: g = h % 8 chains in increasing h, then the tree)
    const int wg = warp >> 2;
    const uint32_t lane_addr = (uint32_t)(32 * (warp & 3)) << 16;
    const int kt = tid & 127;  // the key
    auto tree = [](const double (&s)[8]) {
      return __dadd_rn(__dadd_rn(__dadd_rn(s[0], s[4]), __dadd_rn(s[2], s[6])),
                       __dadd_rn(__dadd_rn(s[1], s[5]), __dadd_rn(s[3], s[7])));
    };
    bool ok = true;
    for (int j = wg; ok && j < nt; j += 2) {
      const int m = j % kKtMeta;
      if (!(ok = kt_warp_wait(m_full(m), (j / kKtMeta) & 1, abort))) break;
      if (kt == 0) TC_TRACE(j, 8);
      const uint8_t* meta = smem + L::kMeta + m * L::kMetaBytes;
      const bool fast = *reinterpret_cast<const uint32_t*>(meta + 640) != 0;
      int n = (int)*reinterpret_cast<const uint32_t*>(meta + 644);
      const uint32_t kc = reinterpret_cast<const uint32_t*>(meta)[kt];
      const int kref = meta[512 + kt];
      const int col = (ch0 + j) * kIdxChunk + kt;
      for (int r = 0; r < span; ++r) {
        float logit;
        if (fast) {
          const int s = n % kKtSlots;
          if (!(ok = kt_warp_wait(s_ready(s), (n / kKtSlots) & 1, abort))) break;
          if (kt == 0) TC_TRACE(j, 9);
          tc_fence_after();
          const uint32_t ta = tmem + 64 * s + lane_addr;
          const int emin = red[16 + r];
          const bool int_row = red[32 + r] == 0 && red[24 + r] - emin <= kKtIntSpread;
          // integer: T_h = 4 relu(D) < 2^21 (the low bits of the fp32 2^23 + T_h), |mult_h| < 2^26; 64
          // terms sum below 2^53, so the contract's fp64 head sum is exact in any order then
          long long acc[4] = {0, 0, 0, 0};
          double sg[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) sg[g] = 0.0;
          const int halves = (H + 31) / 32;
#pragma unroll 1
          for (int hf = 0; hf < halves; ++hf) {
            uint32_t v[32];
            tmem_ld16(ta + 32 * hf, *reinterpret_cast<uint32_t(*)[16]>(v));
            if (32 * hf + 16 < H) tmem_ld16(ta + 32 * hf + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
            tmem_wait_ld();
            if (hf == halves - 1) {  // the slot's columns are in registers
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(s_free(s));
            }
            if (int_row) {
              const int4* mr = reinterpret_cast<const int4*>(s_mult + r * 64 + 32 * hf);
#pragma unroll
              for (int h4 = 0; h4 < 8; ++h4) {
                if (32 * hf + 4 * h4 < H) {
                  const int4 mv = mr[h4];
                  const int mm[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float d = __uint_as_float(v[4 * h4 + e]);
                    const float t = d + fabsf(d);                  // 2 relu(D), exact
                    const float f = __fmaf_rn(t, 2.f, 8388608.f);  // 2^23 + T, exact
                    acc[e] += (long long)mm[e] * (long long)((int)__float_as_uint(f) - 0x4b000000);
                  }
                }
              }
              continue;
            }
            const double2* w3 = reinterpret_cast<const double2*>(s_w3 + r * 64 + 32 * hf);
#pragma unroll
            for (int h2 = 0; h2 < 16; ++h2) {
              if (32 * hf + 2 * h2 < H) {
                const double2 wv = w3[h2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int h = 2 * h2 + e;  // (32 hf + h) % 8 == h % 8
                  const float d = __uint_as_float(v[h]);
                  const float t = d + fabsf(d);  // 2 relu(D), exact
                  const double tt = __hiloint2double((int)(__float_as_uint(t) >> 3), 0);  // t 2^-896
                  sg[h & 7] = __fma_rn(e ? wv.y : wv.x, tt, sg[h & 7]);
                }
              }
            }
          }
          ++n;
          if (int_row) {
            // the sum is A 2^(Emin + kref - 256), rounded once to fp32 (A and the scaling exact in fp64)
            const long long A = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            logit = A == 0 ? 0.f : __double2float_rn(__dmul_rn(__ll2double_rn(A), kt_pow2(emin + kref - 256)));
          } else {
            logit = __double2float_rn(__dmul_rn(tree(sg), kt_pow2(kref + 512)));
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < 4 && ok; ++c) {
            const int s = (n + c) % kKtSlots;
            ok = kt_warp_wait(s_ready(s), ((n + c) / kKtSlots) & 1, abort);
          }
          if (!ok) break;
          tc_fence_after();
          double sg[8];
#pragma unroll
          for (int g = 0; g < 8; ++g) sg[g] = 0.0;
          const uint32_t* qe = s_qe + r * 64;
          const double* wr = s_w + r * 64;
#pragma unroll 1
          for (int q = 0; 16 * q < H; ++q) {
            double x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = 0.0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t v[16];
              tmem_ld16(tmem + 64 * ((n + c) % kKtSlots) + lane_addr + 16 * q, v);
              tmem_wait_ld();
              const int ke = (int)((kc >> (8 * c)) & 0xffu);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int qc = (int)((qe[16 * q + i] >> (8 * c)) & 0xffu);
                x[i] = __fma_rn((double)__uint_as_float(v[i]), kt_pow2(qc + ke - 254), x[i]);
              }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
              sg[i & 7] = __dadd_rn(sg[i & 7], __dmul_rn(wr[16 * q + i], fmax(x[i], 0.0)));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            for (int c = 0; c < 4; ++c) mbar_arrive(s_free((n + c) % kKtSlots));
          n += 4;
          logit = __double2float_rn(tree(sg));
        }
        const int row = lead + r;
        if (col < red[40 + r] && col < a.lstride) a.logits[(size_t)row * a.lstride + col] = logit;
        if (kt == 0) TC_TRACE(j, 10);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(m_free(m));
    }
  }
  // ---- teardown: every role done (a timed-out one unwound); free the TMEM
  tc_fence_before();
  __syncthreads();
  if (tid == 0) TC_TRACE(63, 2);
  if (warp == 12) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
  pdl_launch();
}

}  // namespace dsv41
