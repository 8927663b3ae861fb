// K2i, the index sources' FP4 scorer, and the index selection around it (the reference's
// gfx950/indexer/{index_plan,walk_plan,score_fp4,candidate_table}.py and SGLang's top-k
// kernels, which are absent here and restated).
//
// Logits (bit-exact contract, oracle/indexer.py:index_logits): for row t and column col,
//   x_h = sum_{c=0..3} I_{h,c} 2^(qe_{h,c} + ke_{col,c} - 256)   (fp64, c in order),
//   I_{h,c} = the integer dot of the 2 x E2M1 values of q_h and k_col over chunk c,
//   logit = fp32( tree-sum over heads of w_h relu(x_h) ) with the tree: s_g = terms of heads
//   g, g+8, g+16, ... in order, then ((s0 + s4) + (s2 + s6)) + ((s1 + s5) + (s3 + s7)).
// I_{h,c} comes from mma.sync m16n8k16 f16 on cvt.e2m1x2 operands (converted once a piece for the
// queries and once a chunk for the keys, read by ldmatrix): every product is a multiple of 1/4
// and a 32-dim sum stays below 2^11, so the fp32 accumulation is exact. The f16 operands carry
// the real E2M1 values (I / 4), so the scale exponent is qe + ke - 254.
#pragma once

#include "common.cuh"

namespace dsv41 {

constexpr int kPlaneRows = 64;   // keys an index-plane page
constexpr int kIdxChunk = 128;   // columns a score chunk
constexpr int kWalkRows = 6;     // rows a walk piece (one page table)
constexpr int kIdxMaxSpan = 6;

// ------------------------------------------------------------------ walk plan
struct WalkPlanArgs {
  int rows, ctas, topk;
  const int32_t* bounds;  // [rows]
  const int32_t* owners;  // [rows]: each row's request (page-table row)
  int32_t* plan;          // [ctas, 4]: (lead, span, ch0, ch1), zeros past the last task
};

// index_plan.py:42-82 restated: pieces of <= 6 adjacent rows of one owner; a piece needs
// ceil(max bound / 128) chunks when a row's bound exceeds topk; each piece gets
// ceil(need / width) tasks sharing its chunks evenly at the smallest width whose task count
// fits the CTAs. One warp plans (rows <= 64) with ballots and scans.
__global__ void walk_plan_kernel(const WalkPlanArgs a) {
  __shared__ int s_owner[64], s_bound[64];
  __shared__ int s_lead[64], s_span[64], s_need[64], s_k[64], s_first[65], s_pieces;
  pdl_wait();
  // the rows' owners and bounds in shared memory and the plan cleared, by the whole block
  for (int t = threadIdx.x; t < a.rows; t += blockDim.x) {
    s_owner[t] = a.owners[t];
    s_bound[t] = a.bounds[t];
  }
  for (int i = threadIdx.x; i < a.ctas * 4; i += blockDim.x) a.plan[i] = 0;
  __syncthreads();
  if (threadIdx.x < 32) {  // one warp plans (rows <= 64: lane l holds rows l and l + 32); the block writes the tasks
    const int lane = threadIdx.x;
    const uint32_t full = 0xffffffffu;
    auto below = [](int t) { return t >= 63 ? ~0ull : ((2ull << t) - 1); };  // bits 0 .. t
    // a run of one owner starts a piece, and so does every kWalkRows-th row of the run
    auto starts = [&](int t) { return t < a.rows && (t == 0 || s_owner[t] != s_owner[t - 1]); };
    const uint64_t smask = (uint64_t)__ballot_sync(full, starts(lane)) | ((uint64_t)__ballot_sync(full, starts(lane + 32)) << 32);
    auto leads = [&](int t) {
      if (t >= a.rows) return false;
      const int run_first = 63 - __clzll((long long)(smask & below(t)));
      return (t - run_first) % kWalkRows == 0;
    };
    const uint64_t lmask = (uint64_t)__ballot_sync(full, leads(lane)) | ((uint64_t)__ballot_sync(full, leads(lane + 32)) << 32);
    const int np = __popcll((long long)lmask);
    s_k[lane] = 0;  // (scratch: each piece's need, before the pieces without one are dropped)
    s_k[lane + 32] = 0;
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = lane + 32 * h;
      if (t < a.rows) {
        const int pc = __popcll((long long)(lmask & below(t))) - 1;
        const int b = s_bound[t];
        if (b > a.topk) atomicMax(&s_k[pc], (b + kIdxChunk - 1) / kIdxChunk);
        if ((lmask >> t) & 1) s_first[pc] = t;  // (scratch: the piece's first row)
      }
    }
    __syncwarp();
    // keep the pieces that need chunks, in order
    int pl[2], ps[2], pn[2];
    bool keep[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pc = lane + 32 * h;
      keep[h] = pc < np && s_k[pc] > 0;
      pl[h] = pc < np ? s_first[pc] : 0;
      ps[h] = pc < np ? (pc + 1 < np ? s_first[pc + 1] : a.rows) - pl[h] : 0;
      pn[h] = pc < np ? s_k[pc] : 0;
    }
    const uint64_t kmask = (uint64_t)__ballot_sync(full, keep[0]) | ((uint64_t)__ballot_sync(full, keep[1]) << 32);
    const int pieces = __popcll((long long)kmask);
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pc = lane + 32 * h;
      if (keep[h]) {
        const int i = __popcll((long long)(kmask & ((1ull << pc) - 1)));
        s_lead[i] = pl[h];
        s_span[i] = ps[h];
        s_need[i] = pn[h];
      }
    }
    __syncwarp();
    if (pieces == 0 || pieces >= a.ctas) {
      if (lane == 0) s_pieces = 0;
    } else {
      // the smallest width (chunks a task) whose task count fits the CTAs, from the total's share
      const int n0 = lane < pieces ? s_need[lane] : 0, n1 = lane + 32 < pieces ? s_need[lane + 32] : 0;
      const long total = __reduce_add_sync(full, n0 + n1);
      int width = (int)max((total + a.ctas - 1) / a.ctas, 1L);
      for (;; ++width) {
        const int tasks = __reduce_add_sync(full, (n0 + width - 1) / width + (n1 + width - 1) / width);
        if (tasks <= a.ctas) break;
      }
      // tasks a piece and their first index (exclusive scan over pieces 0 .. 31, then 32 ..)
      const int k0 = (n0 + width - 1) / width, k1 = (n1 + width - 1) / width;
      int c0 = k0, c1 = k1;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o0 = __shfl_up_sync(full, c0, d), o1 = __shfl_up_sync(full, c1, d);
        if (lane >= d) {
          c0 += o0;
          c1 += o1;
        }
      }
      const int tot0 = __shfl_sync(full, c0, 31);
      if (lane < pieces) {
        s_k[lane] = k0;
        s_first[lane] = c0 - k0;
      }
      if (lane + 32 < pieces) {
        s_k[lane + 32] = k1;
        s_first[lane + 32] = tot0 + c1 - k1;
      }
      const int tot1 = __shfl_sync(full, c1, 31);
      if (lane == 0) {
        s_first[pieces] = tot0 + tot1;
        s_pieces = pieces;
      }
    }
  }
  __syncthreads();
  // every thread writes its tasks: task r of piece i (r - first[i] = j of k)
  const int pieces = s_pieces;
  for (int r = threadIdx.x; pieces > 0 && r < s_first[pieces]; r += blockDim.x) {
    int i = 0;
    while (s_first[i + 1] <= r) ++i;
    const int j = r - s_first[i], k = s_k[i], nd = s_need[i];
    a.plan[4 * r + 0] = s_lead[i];
    a.plan[4 * r + 1] = s_span[i];
    a.plan[4 * r + 2] = j * nd / k;
    a.plan[4 * r + 3] = (j + 1) * nd / k;
  }
  pdl_launch();
}

// ------------------------------------------------------------------ scorer
struct K2iArgs {
  int rows, heads;
  const uint8_t* q;        // [rows, heads, 64] E2M1 pairs (128 dims a head)
  const uint8_t* qscale;   // [rows, 1, 4, 16, 4]: head h, chunk c at [c][h % 16][h / 16]
  const __nv_bfloat16* w;  // [rows, heads]
  const uint8_t* payload;  // [pages, 1, 4, 64, 16]
  const uint8_t* kscale;   // [pages, 1, 4, 64]: key s at (s % 16) * 4 + s / 16
  const int32_t* plan;     // FULL: [ctas, 4] walk plan
  const int32_t* itab;     // page table: row owners[t], entries of ``entry_rows`` keys
  int itab_stride, itab_len, entry_rows;  // 64 (plane pages) or 8 (a REINDEX table's blocks)
  const int32_t* owners;   // [rows]
  const int32_t* bounds;   // [rows]: columns a row sees
  float* logits;           // [rows, lstride]
  int lstride;
  int reindex;             // 1: CTA b scores chunk range b % per of row b / per (no plan)
  int reindex_chunks;      // a REINDEX row's chunks
};

// f16 operand rows: 128 dims (256 B) padded to 272 B so ldmatrix's 8 rows hit distinct banks
constexpr int kIdxRowBytes = 272;
__host__ __device__ inline int k2i_smem_bytes(int heads) {
  return kIdxMaxSpan * heads * 64 + heads * kIdxRowBytes + kIdxChunk * kIdxRowBytes + kIdxMaxSpan * 4 * heads +
         4 * kIdxChunk;
}

__global__ void __launch_bounds__(256) k2i_score_kernel(const K2iArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int H = a.heads, mtiles = H / 16;
  uint8_t* qraw = smem;                                  // [span][H][64] E2M1 bytes
  uint8_t* qf = qraw + kIdxMaxSpan * H * 64;             // [H] rows of 128 f16 dims: the current row
  uint8_t* kf = qf + H * kIdxRowBytes;                   // [128 columns] rows of 128 f16 dims
  uint8_t* qe = kf + kIdxChunk * kIdxRowBytes;           // [span][H][4]: a head's 4 chunk codes in a word
  uint8_t* ke = qe + kIdxMaxSpan * 4 * H;                // [4][128]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  pdl_wait();
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
  if (span <= 0 || ch0 >= ch1) return;
  const int owner = a.owners[lead];
  int piece_bound = 0;
  for (int r = 0; r < span; ++r) piece_bound = max(piece_bound, a.bounds[lead + r]);
  // the piece's queries: raw E2M1 bytes (each row goes to f16 once a chunk, below)
  for (int i = tid; i < span * H * 16; i += blockDim.x)
    reinterpret_cast<uint32_t*>(qraw)[i] = *reinterpret_cast<const uint32_t*>(a.q + (size_t)lead * H * 64 + 4 * i);
  for (int i = tid; i < span * 4 * H; i += blockDim.x) {
    const int r = i / (4 * H), h = (i / 4) % H, c = i % 4;
    qe[i] = a.qscale[(size_t)(lead + r) * 256 + c * 64 + (h % 16) * 4 + h / 16];
  }
  // a chunk's keys: 128 columns x 4 chunks x 16 B, zero past the piece's bound; this thread's
  // kKeyItems of them are loaded into registers one chunk ahead of their use
  constexpr int kKeyItems = 4 * kIdxChunk / 256;
  uint4 kv[kKeyItems];
  uint8_t ks[kKeyItems];
  auto load_keys = [&](int ch) {
#pragma unroll
    for (int u = 0; u < kKeyItems; ++u) {
      const int i = tid + 256 * u;
      const int c = i / kIdxChunk, cl = i % kIdxChunk, col = ch * kIdxChunk + cl;
      kv[u] = make_uint4(0, 0, 0, 0);
      ks[u] = 127;
      if (col < piece_bound && col / a.entry_rows < a.itab_len) {
        const int entry = a.itab[(size_t)owner * a.itab_stride + col / a.entry_rows];
        const long vrow = (long)entry * a.entry_rows + col % a.entry_rows;
        const long page = vrow / kPlaneRows;
        const int slot = (int)(vrow % kPlaneRows);
        kv[u] = ldg16(a.payload + ((page * 4 + c) * kPlaneRows + slot) * 16);
        ks[u] = a.kscale[(page * 4 + c) * kPlaneRows + (slot % 16) * 4 + slot / 16];
      }
    }
  };
  if (ch0 < ch1 && ch0 * kIdxChunk < piece_bound) load_keys(ch0);
  for (int ch = ch0; ch < ch1 && ch * kIdxChunk < piece_bound; ++ch) {
    __syncthreads();  // the previous chunk's readers are done
#pragma unroll
    for (int u = 0; u < kKeyItems; ++u) {
      // the 16 E2M1 bytes (32 dims) of chunk c of column cl, as f16 at dims 32 c ..
      const int i = tid + 256 * u;
      const int c = i / kIdxChunk, cl = i % kIdxChunk;
      const uint32_t w[4] = {kv[u].x, kv[u].y, kv[u].z, kv[u].w};
      uint8_t* dst = kf + cl * kIdxRowBytes + 64 * c;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(dst + 16 * q) =
            make_uint4(e2m1x2_f16(w[q] & 0xff), e2m1x2_f16((w[q] >> 8) & 0xff), e2m1x2_f16((w[q] >> 16) & 0xff),
                       e2m1x2_f16(w[q] >> 24));
      ke[c * kIdxChunk + cl] = ks[u];
    }
    __syncthreads();
    if (ch + 1 < ch1 && (ch + 1) * kIdxChunk < piece_bound) load_keys(ch + 1);
    // ldmatrix lane addresses: A rows 16 mt + lane % 16, dims + 8 (lane / 16); B columns
    // 16 warp + 8 (lane / 16) + lane % 8, dims + 8 ((lane / 8) % 2) -- both n-tiles at once
    const uint32_t qf_s = smem_u32(qf), kf_s = smem_u32(kf);
    const uint32_t a_lane = (uint32_t)((lane % 16) * kIdxRowBytes + 16 * (lane / 16));
    const uint32_t b_lane = (uint32_t)((16 * warp + 8 * (lane / 16) + lane % 8) * kIdxRowBytes + 16 * ((lane / 8) % 2));
    // this thread's key codes of the chunk: columns 16 warp + 8 nn + 2 t + j, byte 2 nn + j of
    // word c
    uint32_t kev[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint8_t* kc = ke + c * kIdxChunk + 16 * warp + 2 * t;
      kev[c] = (uint32_t)*reinterpret_cast<const uint16_t*>(kc) |
               ((uint32_t)*reinterpret_cast<const uint16_t*>(kc + 8) << 16);
    }
    for (int r = 0; r < span; ++r) {
      const int row = lead + r, bound = a.bounds[row];
      // row r's queries as f16 (exact: E2M1 values), once a chunk (a one-row piece: once)
      if (span > 1 || ch == ch0) {
        if (r > 0) __syncthreads();  // the previous row's readers are done
        for (int i = tid; i < H * 16; i += blockDim.x) {
          const int h = i / 16, wd = i % 16;
          const uint32_t v = reinterpret_cast<const uint32_t*>(qraw)[(r * H + h) * 16 + wd];
          *reinterpret_cast<uint4*>(qf + h * kIdxRowBytes + 16 * wd) =
              make_uint4(e2m1x2_f16(v & 0xff), e2m1x2_f16((v >> 8) & 0xff), e2m1x2_f16((v >> 16) & 0xff),
                         e2m1x2_f16(v >> 24));
        }
        __syncthreads();
      }
      double s2[2][2] = {{0.0, 0.0}, {0.0, 0.0}};  // [n-tile][column parity]
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        if (mt >= mtiles) break;
        // heads 16 mt + g (q = 0, 1) and 16 mt + g + 8 (q = 2, 3): their chunk codes and weights
        const uint32_t qw0 = *reinterpret_cast<const uint32_t*>(qe + (r * H + 16 * mt + g) * 4);
        const uint32_t qw1 = *reinterpret_cast<const uint32_t*>(qe + (r * H + 16 * mt + g + 8) * 4);
        const double wv0 = (double)bf2f(a.w[(size_t)row * H + 16 * mt + g]);
        const double wv1 = (double)bf2f(a.w[(size_t)row * H + 16 * mt + g + 8]);
        double x[2][4] = {{0.0, 0.0, 0.0, 0.0}, {0.0, 0.0, 0.0, 0.0}};
        const uint32_t qa = qf_s + (uint32_t)(16 * mt * kIdxRowBytes) + a_lane;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int ksp = 0; ksp < 2; ++ksp) {
            uint32_t af[4], bf[4];
            ldmatrix_x4(af, qa + (uint32_t)((32 * c + 16 * ksp) * 2));
            ldmatrix_x4(bf, kf_s + b_lane + (uint32_t)((32 * c + 16 * ksp) * 2));
            mma_f16(acc[0], af[0], af[1], af[2], af[3], bf[0], bf[1]);
            mma_f16(acc[1], af[0], af[1], af[2], af[3], bf[2], bf[3]);
          }
          const uint32_t qb0 = (qw0 >> (8 * c)) & 0xffu, qb1 = (qw1 >> (8 * c)) & 0xffu;
#pragma unroll
          for (int nn = 0; nn < 2; ++nn)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              // 2^(qe + ke - 254) as a double (biased exponent qe + ke + 769); acc times it is
              // exact, so the fused add rounds as the separate multiply and add would
              const uint32_t kb = (kev[c] >> (16 * nn + 8 * (q & 1))) & 0xffu;
              const double f = __hiloint2double((int)(((q >> 1) ? qb1 : qb0) + kb + 769u) << 20, 0);
              x[nn][q] = __fma_rn((double)acc[nn][q], f, x[nn][q]);
            }
        }
#pragma unroll
        for (int nn = 0; nn < 2; ++nn)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            // heads g + 16 mt (q = 0, 1), then g + 8 + 16 mt (q = 2, 3): the tree's order
            s2[nn][q & 1] = __dadd_rn(s2[nn][q & 1], __dmul_rn((q >> 1) ? wv1 : wv0, fmax(x[nn][q], 0.0)));
      }
#pragma unroll
      for (int nn = 0; nn < 2; ++nn) {
        const int nt = 2 * warp + nn;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          double v = s2[nn][j];
          v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 16));
          v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
          v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
          const int col = ch * kIdxChunk + 8 * nt + 2 * t + j;
          if (g == 0 && col < bound && col < a.lstride) a.logits[(size_t)row * a.lstride + col] = (float)v;
        }
      }
    }
  }
  pdl_launch();
}

// ------------------------------------------------------------------ top-k
// The k largest of each row's first n values, ties to the lower position, written as
// positions in ascending order (-1 padded); every position when n <= k. Radix select on an
// order-preserving 32-bit key (NaN lowest, -0 equal to +0), then an ordered compaction.
__device__ __forceinline__ uint32_t order_key(float v) {
  if (isnan(v)) return 0u;
  const uint32_t b = v == 0.f ? 0u : __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct TopkArgs {
  int rows, k;
  const float* vals;       // [rows, vstride]
  int vstride;
  const int32_t* n;        // [rows] values a row considers
  int group;               // 1: values as is; G > 1: a candidate's score is the max of G values
  int32_t* out;            // [rows, k] positions (or groups)
  // optional paged outputs: page_out[t][j] = table[owner][pos / page] * page + pos % page
  int32_t* page_out;
  const int32_t* table;
  int table_stride, page;
  const int32_t* owners;
  int cap;                 // keys the dynamic shared memory holds (a multiple of 4; the row is staged
                           // when n <= cap); a 4096-bin histogram follows them
};

constexpr int kTopkBins = 4096;  // 12-bit digits (bits 31..20, then 19..8), then 8 bits (7..0)

__global__ void __launch_bounds__(1024) topk_kernel(const TopkArgs a) {
  extern __shared__ __align__(16) uint32_t s_keys[];  // [cap], then the histogram
  int* hist = reinterpret_cast<int*>(s_keys + a.cap);
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  __shared__ int s_warp[32], s_warp2[32];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = (int)blockDim.x, nwarps = nthr >> 5;
  pdl_wait();
  const int nval = a.n[row];
  const int n = a.group > 1 ? (nval + a.group - 1) / a.group : nval;
  int32_t* out = a.out + (size_t)row * a.k;
  const float* vrow = a.vals + (size_t)row * a.vstride;
  auto key_of = [&](int i) -> uint32_t {
    if (a.group <= 1) return order_key(vrow[i]);
    uint32_t m = 0;
    for (int j = 0; j < a.group; ++j) {
      const int p = i * a.group + j;
      if (p < nval) m = max(m, order_key(vrow[p]));
    }
    return m;
  };
  // the row's keys go to shared memory once when they fit: the passes below read them there,
  // four a thread at a time
  const bool staged = n <= a.cap;
  if (tid == 0) {
    s_prefix = 0;
    s_need = a.k;
  }
  if (staged && n > a.k)
#pragma unroll 4
    for (int i = tid; i < n; i += nthr) s_keys[i] = key_of(i);
  __syncthreads();  // the staged keys and the radix state are visible to every thread
  const int32_t* tbl = a.page_out ? a.table + (size_t)__ldg(a.owners + row) * a.table_stride : nullptr;
  auto emit = [&](int j, int pos) {
    out[j] = pos;
    if (a.page_out) a.page_out[(size_t)row * a.k + j] = pos >= 0 ? __ldg(tbl + pos / a.page) * a.page + pos % a.page : -1;
  };
  if (n <= a.k) {
    for (int j = tid; j < a.k; j += nthr) emit(j, j < n ? j : -1);
    return;
  }
  // keys p .. p + 3 (p a multiple of 4; past `end` read as 0 and flagged out)
  auto load4 = [&](int p, int end, uint32_t (&kq)[4]) {
    if (staged) {
      const uint4 v = *reinterpret_cast<const uint4*>(s_keys + p);
      kq[0] = v.x;
      kq[1] = v.y;
      kq[2] = v.z;
      kq[3] = v.w;
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) kq[q] = p + q < end ? key_of(p + q) : 0u;
    }
  };
  // ---- radix select: the threshold key T, count(key > T) < k <= count(key >= T), in three
  // passes (12, 12, 8 bits); a 12-bit first digit spreads even logits of a few exponents over
  // many bins, so plain shared atomics do
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 8 : 0);
    const int nb = pass == 2 ? 256 : kTopkBins;
    const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (pass == 1 ? 20 : 8));
    const uint32_t prefix = s_prefix;
    const int need = s_need;
    for (int i = tid; i < nb; i += nthr) hist[i] = 0;
    __syncthreads();
    for (int p = 4 * tid; p < n; p += 4 * nthr) {
      uint32_t kq[4];
      load4(p, n, kq);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (p + q < n && (kq[q] & pmask) == prefix) atomicAdd(&hist[(kq[q] >> shift) & (nb - 1)], 1);
    }
    __syncthreads();
    // the digit d with S(d + 1) < need <= S(d), S(d) = count of bins >= d: thread t holds bins
    // 4 t .. 4 t + 3; a block-wide suffix sum finds the one thread the crossing falls in
    int c[4], own = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      c[q] = 4 * tid + q < nb ? hist[4 * tid + q] : 0;
      own += c[q];
    }
    int incl = own;  // this thread's bins and every higher lane's of the warp
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_down_sync(0xffffffffu, incl, d);
      if (lane + d < 32) incl += o;
    }
    if (lane == 0) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int wt = lane < nwarps ? s_warp[lane] : 0;
      int ws = wt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_down_sync(0xffffffffu, ws, d);
        if (lane + d < 32) ws += o;
      }
      if (lane < nwarps) s_warp2[lane] = ws - wt;  // the warps above
    }
    __syncthreads();
    incl += s_warp2[warp];
    const int above = incl - own;
    if (above < need && need <= incl) {
      int acc = above, d = 4 * tid;
#pragma unroll
      for (int q = 3; q >= 0; --q) {
        if (acc + c[q] >= need) {
          d = 4 * tid + q;
          break;
        }
        acc += c[q];
      }
      s_need = need - acc;
      s_prefix = prefix | ((uint32_t)d << shift);
    }
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int ties_taken = s_need;  // how many keys equal to T are selected (lowest positions)
  // ---- ordered compaction (exactly k selections): warp w walks positions [w seg, (w + 1) seg)
  // 128 at a time, lane l holding positions + 4 l .. + 3; counts, then emits in order by scans
  const int seg = ((n + nwarps - 1) / nwarps + 127) / 128 * 128;
  const int p0 = min(n, warp * seg), p1 = min(n, p0 + seg);
  int cnt_gt = 0, cnt_eq = 0;
  for (int base = p0; base < p1; base += 128) {
    const int p = base + 4 * lane;
    if (p >= p1) continue;
    uint32_t kq[4];
    load4(p, p1, kq);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (p + q < p1) {
        cnt_gt += kq[q] > T;
        cnt_eq += kq[q] == T;
      }
  }
  cnt_gt = __reduce_add_sync(0xffffffffu, cnt_gt);
  cnt_eq = __reduce_add_sync(0xffffffffu, cnt_eq);
  // exclusive scans over the warps: of the ties (for the tie budget), then of the selections
  if (lane == 0) {
    s_warp[warp] = cnt_gt;
    s_warp2[warp] = cnt_eq;
  }
  __syncthreads();
  if (warp == 0) {
    const int te = lane < nwarps ? s_warp2[lane] : 0, ge = lane < nwarps ? s_warp[lane] : 0;
    int ti = te;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, ti, d);
      if (lane >= d) ti += o;
    }
    const int eq_mine = max(0, min(te, ties_taken - (ti - te)));
    const int sel = ge + eq_mine;
    int si = sel;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, si, d);
      if (lane >= d) si += o;
    }
    if (lane < nwarps) {
      s_warp2[lane] = eq_mine;  // this warp's ties to take
      s_warp[lane] = si - sel;  // this warp's first output slot
    }
  }
  __syncthreads();
  const int eq_mine = s_warp2[warp];
  int j = s_warp[warp], eq_seen = 0;  // warp-uniform
  for (int base = p0; base < p1; base += 128) {
    const int p = base + 4 * lane;
    uint32_t kq[4] = {0u, 0u, 0u, 0u};
    if (p < p1) load4(p, p1, kq);
    bool gt[4], eq[4];
    int ne = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      gt[q] = p + q < p1 && kq[q] > T;
      eq[q] = p + q < p1 && kq[q] == T;
      ne += eq[q];
    }
    int ei = ne;  // ties at this lane's positions and the lanes' below
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, ei, d);
      if (lane >= d) ei += o;
    }
    int seen = eq_seen + ei - ne, nt = 0;
    bool take[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      take[q] = gt[q] || (eq[q] && seen < eq_mine);
      seen += eq[q];
      nt += take[q];
    }
    int tsum = nt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, tsum, d);
      if (lane >= d) tsum += o;
    }
    int slot = j + tsum - nt;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (take[q]) emit(slot++, p + q);
    j += __shfl_sync(0xffffffffu, tsum, 31);
    eq_seen += __shfl_sync(0xffffffffu, ei, 31);
  }
  pdl_launch();
}

// ------------------------------------------------------------------ candidate tables
struct ReindexArgs {
  int rows, topk_blocks, units, block_rows;  // units: 8-row blocks a 64-row page
  const int32_t* ids;       // [rows, ids_stride] candidate blocks, -1 after the kept ones
  int ids_stride;
  const int32_t* page_table;  // [owner][page_stride]
  int page_stride;
  const int32_t* owners;
  const int32_t* visible;   // [rows] bounds
  int32_t* ids_out;         // [rows, ids_stride]
  int32_t* table;           // [rows, ids_stride] virtual 8-row pages
  int32_t* context;         // [rows]
};

// candidate_table.py:19-66 restated: the newest block (holding position visible - 1) moved to
// the last kept slot; each kept block's virtual 8-row page; the context.
__global__ void reindex_kernel(const ReindexArgs a) {
  pdl_wait();
  const int t = blockIdx.x;
  if (threadIdx.x != 0) return;
  const int32_t* ids = a.ids + (size_t)t * a.ids_stride;
  int32_t* io = a.ids_out + (size_t)t * a.ids_stride;
  int32_t* tb = a.table + (size_t)t * a.ids_stride;
  int kept = 0;
  for (int s = 0; s < a.topk_blocks; ++s) kept += ids[s] >= 0;
  const int seen = a.visible[t];
  const int newest = seen >= 1 ? (seen - 1) / a.block_rows : -1;  // floor division
  int at = -1;
  for (int s = 0; s < a.topk_blocks; ++s)
    if (ids[s] >= 0 && ids[s] == newest) at = s;
  const int last = kept - 1;
  const int moved = last >= 0 ? ids[last] : 0;
  for (int s = 0; s < a.topk_blocks; ++s) {
    int c = ids[s];
    if (at >= 0 && s == at) c = moved;
    else if (at >= 0 && s == last) c = newest;
    io[s] = c;
    const bool live = c >= 0;
    const int cc = live ? c : 0;
    tb[s] = live ? a.page_table[(size_t)a.owners[t] * a.page_stride + cc / a.units] * a.units + cc % a.units : 0;
  }
  const int tail = last >= 0 ? io[last] : 0;
  const int span = min(max(seen - tail * a.block_rows, 0), a.block_rows);
  a.context[t] = kept > 0 ? (kept - 1) * a.block_rows + span : 0;
  pdl_launch();
}

struct MapCompactArgs {
  int rows, topk, block_rows, page;
  const int32_t* compact;   // [rows, topk]
  const int32_t* ids;       // [rows, ids_stride] (reindex_kernel's ids_out)
  int ids_stride;
  const int32_t* page_table;
  int table_stride;
  const int32_t* owners;
  int32_t* raw_out;         // [rows, out_stride]
  int32_t* page_out;
  int out_stride;
};

// candidate_table.py:103-134 restated: compact column c -> position ids[c / 8] * 8 + c % 8
// -> pool slot page_table[pos / 64] * 64 + pos % 64; -1 stays -1.
__global__ void map_compact_kernel(const MapCompactArgs a) {
  pdl_wait();
  const int t = blockIdx.x;
  for (int j = threadIdx.x; j < a.topk; j += blockDim.x) {
    const int c = a.compact[(size_t)t * a.topk + j];
    int raw = -1, pg = -1;
    if (c >= 0) {
      raw = a.ids[(size_t)t * a.ids_stride + c / a.block_rows] * a.block_rows + c % a.block_rows;
      pg = a.page_table[(size_t)a.owners[t] * a.table_stride + raw / a.page] * a.page + raw % a.page;
    }
    a.raw_out[(size_t)t * a.out_stride + j] = raw;
    a.page_out[(size_t)t * a.out_stride + j] = pg;
  }
  pdl_launch();
}

}  // namespace dsv41
