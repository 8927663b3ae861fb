// The top-k of k2i.cuh's topk_kernel (the same selection: the k largest of a row's first n
// values, ties to the lower position, positions ascending, -1 padded; optional groups and paged
// twin) with each row spread over a cluster of kTopkCl CTAs, so a step's few rows occupy more
// than one SM each. CTA rank r of a row's cluster stages the row's r-th segment of keys; each
// radix pass builds per-CTA histograms that every CTA then sums over the cluster through
// distributed shared memory (the same digit decision in every CTA); the ordered compaction
// offsets each CTA by the selections and ties of the CTAs before it.
#pragma once

#include "attn_tc.cuh"
#include "k2i.cuh"

namespace dsv41 {

constexpr int kTopkCl = 8;             // CTAs a row
constexpr int kTopkClThreads = 512;    // 16 warps
constexpr int kTopkClMinCands = 2048;  // rows of fewer candidates take the one-CTA kernel

__device__ __forceinline__ uint32_t tk_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint4 tk_ld_dsmem4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ int tk_ld_dsmem(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// a.cap: keys a CTA stages (a multiple of 128); kTopkBins ints of histogram follow them
__global__ void __launch_bounds__(kTopkClThreads, 1) topk_cluster_kernel(const TopkArgs a) {
  extern __shared__ __align__(16) uint32_t s_keys[];
  int* hist = reinterpret_cast<int*>(s_keys + a.cap);
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  __shared__ int s_warp[32], s_warp2[32];
  __shared__ int s_cnt[2];  // this CTA's keys > T and == T
  const uint32_t cr = tk_ctarank();
  const int row = blockIdx.x / kTopkCl, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = (int)blockDim.x, nwarps = nthr >> 5;
  pdl_wait();
  if (tid == 0) TC_TRACE(0, 0);
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
  const int32_t* tbl = a.page_out ? a.table + (size_t)__ldg(a.owners + row) * a.table_stride : nullptr;
  auto emit = [&](int j, int pos) {
    out[j] = pos;
    if (a.page_out) a.page_out[(size_t)row * a.k + j] = pos >= 0 ? __ldg(tbl + pos / a.page) * a.page + pos % a.page : -1;
  };
  if (n <= a.k) {  // every position in order (the whole cluster returns here, before any barrier)
    for (int j = (int)cr * nthr + tid; j < a.k; j += kTopkCl * nthr) emit(j, j < n ? j : -1);
    pdl_launch();
    return;
  }
  // this CTA's segment [q0, q1) of the candidates, staged when it fits
  const int seg = cdiv(cdiv(n, kTopkCl), 128) * 128;
  const int q0 = min(n, (int)cr * seg), q1 = min(n, q0 + seg), len = q1 - q0;
  const bool staged = seg <= a.cap;
  if (tid == 0) {
    s_prefix = 0;
    s_need = a.k;
  }
  if (staged)
#pragma unroll 4
    for (int i = tid; i < len; i += nthr) s_keys[i] = key_of(q0 + i);
  // local keys p .. p + 3 (p a multiple of 4; past len flagged out by the callers)
  auto load4 = [&](int p, uint32_t (&kq)[4]) {
    if (staged) {
      const uint4 v = *reinterpret_cast<const uint4*>(s_keys + p);
      kq[0] = v.x;
      kq[1] = v.y;
      kq[2] = v.z;
      kq[3] = v.w;
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) kq[q] = p + q < len ? key_of(q0 + p + q) : 0u;
    }
  };
  const uint32_t hist_s = smem_u32(hist);
  if (tid == 0) TC_TRACE(0, 1);
  // ---- radix select over the cluster (12, 12, 8 bits): T with count(key > T) < k <= count(key >= T)
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 8 : 0);
    const int nb = pass == 2 ? 256 : kTopkBins;
    const uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (pass == 1 ? 20 : 8));
    __syncthreads();  // the staged keys, s_prefix / s_need of the previous pass
    const uint32_t prefix = s_prefix;
    const int need = s_need;
    for (int i = tid; i < nb; i += nthr) hist[i] = 0;
    __syncthreads();
    for (int p = 4 * tid; p < len; p += 4 * nthr) {
      uint32_t kq[4];
      load4(p, kq);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (p + q < len && (kq[q] & pmask) == prefix) atomicAdd(&hist[(kq[q] >> shift) & (nb - 1)], 1);
    }
    if (tid == 0) TC_TRACE(1 + pass, 0);
    cluster_sync_all();  // every CTA's histogram complete
    if (tid == 0) TC_TRACE(1 + pass, 1);
    // this CTA's slice of the bins, [sl0, sl0 + sw): thread t < sw sums bin sl0 + t over the cluster
    const int sw = nb / kTopkCl, sl0 = (int)cr * sw;
    int mine = 0;
    if (tid < sw) {
      int v[kTopkCl];
#pragma unroll
      for (int r = 0; r < kTopkCl; ++r) v[r] = tk_ld_dsmem(cluster_map(hist_s + 4u * (uint32_t)(sl0 + tid), (uint32_t)r));
#pragma unroll
      for (int r = 0; r < kTopkCl; ++r) mine += v[r];
    }
    // suffix sums within the slice (bins >= sl0 + t), and the slice's total
    int incl = mine;
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
      if (lane == 0) s_cnt[0] = ws;                // the slice's total
    }
    __syncthreads();
    incl += s_warp2[warp];
    if (tid == 0) TC_TRACE(1 + pass, 2);
    cluster_sync_all();  // every slice total published (and every read of the histograms done)
    // the slices above this one (higher ranks hold higher bins)
    int higher = 0;
    for (int r = (int)cr + 1; r < kTopkCl; ++r) higher += tk_ld_dsmem(cluster_map(smem_u32(s_cnt), (uint32_t)r));
    const int above = higher + incl - mine;
    if (tid < sw && above < need && need <= higher + incl) {
      // the crossing bin: every CTA of the cluster gets the digit and what remains to take
      const uint32_t np = prefix | ((uint32_t)(sl0 + tid) << shift);
      const int nn = need - above;
      for (int r = 0; r < kTopkCl; ++r) {
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_map(smem_u32(&s_prefix), (uint32_t)r)), "r"(np)
                     : "memory");
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_map(smem_u32(&s_need), (uint32_t)r)), "r"(nn)
                     : "memory");
      }
    }
    if (tid == 0) TC_TRACE(1 + pass, 3);
    cluster_sync_all();  // the digit in every CTA; the slice totals read before they are rewritten
    if (tid == 0) TC_TRACE(1 + pass, 4);
  }
  __syncthreads();
  const uint32_t T = s_prefix;
  const int ties_taken = s_need;  // keys equal to T selected over the row (the lowest positions)
  // ---- ordered compaction: warp w walks local positions [w wseg, (w + 1) wseg) 128 at a time
  const int wseg = cdiv(cdiv(max(len, 1), nwarps), 128) * 128;
  const int p0 = min(len, warp * wseg), p1 = min(len, p0 + wseg);
  int cnt_gt = 0, cnt_eq = 0;
  for (int base = p0; base < p1; base += 128) {
    const int p = base + 4 * lane;
    if (p >= p1) continue;
    uint32_t kq[4];
    load4(p, kq);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (p + q < p1) {
        cnt_gt += kq[q] > T;
        cnt_eq += kq[q] == T;
      }
  }
  cnt_gt = __reduce_add_sync(0xffffffffu, cnt_gt);
  cnt_eq = __reduce_add_sync(0xffffffffu, cnt_eq);
  if (lane == 0) {
    s_warp[warp] = cnt_gt;
    s_warp2[warp] = cnt_eq;
  }
  __syncthreads();
  if (tid == 0) {
    int g = 0, e = 0;
    for (int w = 0; w < nwarps; ++w) {
      g += s_warp[w];
      e += s_warp2[w];
    }
    s_cnt[0] = g;
    s_cnt[1] = e;
  }
  if (tid == 0) TC_TRACE(4, 0);
  cluster_sync_all();  // every CTA's counts published
  if (tid == 0) TC_TRACE(4, 1);
  // the CTAs before this one: their selections (keys > T and their share of the ties) and ties
  int sel_before = 0, eq_before = 0;
  for (int r = 0; r < (int)cr; ++r) {
    const uint32_t ra = cluster_map(smem_u32(s_cnt), (uint32_t)r);
    const int g = tk_ld_dsmem(ra), e = tk_ld_dsmem(ra + 4);
    sel_before += g + max(0, min(e, ties_taken - eq_before));
    eq_before += e;
  }
  const int ties_here = max(0, min(s_cnt[1], ties_taken - eq_before));
  if (tid == 0) TC_TRACE(4, 2);
  cluster_sync_all();  // the reads of the others' counts done before any CTA leaves
  if (tid == 0) TC_TRACE(4, 3);
  if (warp == 0) {
    const int te = lane < nwarps ? s_warp2[lane] : 0, ge = lane < nwarps ? s_warp[lane] : 0;
    int ti = te;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, ti, d);
      if (lane >= d) ti += o;
    }
    const int eq_mine = max(0, min(te, ties_here - (ti - te)));
    const int sel = ge + eq_mine;
    int si = sel;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, si, d);
      if (lane >= d) si += o;
    }
    __syncwarp();
    if (lane < nwarps) {
      s_warp2[lane] = eq_mine;               // this warp's ties to take
      s_warp[lane] = sel_before + si - sel;  // this warp's first output slot
    }
  }
  __syncthreads();
  const int eq_mine = s_warp2[warp];
  int j = s_warp[warp], eq_seen = 0;  // warp-uniform
  for (int base = p0; base < p1; base += 128) {
    const int p = base + 4 * lane;
    uint32_t kq[4] = {0u, 0u, 0u, 0u};
    if (p < p1) load4(p, kq);
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
      if (take[q]) emit(slot++, q0 + p + q);
    j += __shfl_sync(0xffffffffu, tsum, 31);
    eq_seen += __shfl_sync(0xffffffffu, ei, 31);
  }
  if (tid == 0) TC_TRACE(4, 4);
  pdl_launch();
}

}  // namespace dsv41
