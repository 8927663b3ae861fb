// extern "C" entry points (include/dsv41_b200.h): argument checks, scratch carving, and the
// launch sequences of K1 and K2. Every launch goes on the caller's stream with programmatic
// dependent launch, so a kernel's CTAs are resident (and its weight-independent prologue runs)
// while the previous kernel drains; each kernel waits (griddepcontrol.wait) before reading
// what the previous one wrote.
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <map>
#include <tuple>
#include <mutex>
#include <cstdlib>

#include "../../../../include/dsv41_b200.h"
#include "attention.cuh"
#include "attn_tc.cuh"
#include "attn_wide.cuh"
#include "k2i_tc.cuh"
#include "topk_cl.cuh"
#include "common.cuh"
#include "epilogue.cuh"
#include "front.cuh"
#include "gemv.cuh"
#include "gemv_entry.cuh"
#include "index_query.cuh"
#include "k1_persistent.cuh"
#include "k2i.cuh"
#include "lmhead.cuh"
#include "moe.cuh"
#include "moe_tc.cuh"
#include "dense_tc.cuh"
#include "peer.cuh"
#include "seam.cuh"

using namespace dsv41;

cudaError_t dsv41::ensure_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[key] = bytes;
  return e;
}

namespace {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// Tuning switches: read once from the environment, overridable through dsv41_set_option.
struct Option {
  const char* name;  // dsv41_set_option's name
  const char* env;
  int64_t dflt;
  std::atomic<int64_t> value;
  std::atomic<bool> set;
};
// The attention core: tcgen05 (1, default) or the mma.sync split kernel (0; DSV41_ATTN=mma).
// A row's two 32-head tiles as one CTA pair sharing key tiles (1, default), or two lone CTAs that
// each gather every key (0; DSV41_ATTN_PAIR=0), for comparison.
// The smallest M whose MXFP8-input GEMVs run on the tcgen05 dense kernel (DSV41_DENSE_MIN_M, 16).
// Programmatic dependent launch between the layer's kernels (DSV41_PDL=0 turns it off).
// The tcgen05 attention's producer staging each tile's records by bulk copies (1; lone CTAs), or
// gathering them into registers (0, default; DSV41_ATTN_BULK=1 turns staging on). Measured at
// config 2, M = 48: staged 469 us against the gathering pair's 386 us (two f16 tile stages beside
// the staging ring put each tile's conversion on the MMA's critical path).
Option g_options[] = {
    {"attn_tc", "DSV41_ATTN", 1, {0}, {false}},
    {"attn_pair", "DSV41_ATTN_PAIR", 1, {0}, {false}},
    {"dense_min_m", "DSV41_DENSE_MIN_M", 16, {0}, {false}},
    {"pdl", "DSV41_PDL", 1, {0}, {false}},
    {"attn_bulk", "DSV41_ATTN_BULK", 0, {0}, {false}},
    {"fused_allreduce", "DSV41_FUSED_AR", 1, {0}, {false}},
    {"k1_persistent", "DSV41_K1_PERSISTENT", 0, {0}, {false}},
    {"attn_wide", "DSV41_ATTN_WIDE", 1, {0}, {false}},
    {"k2i_tc", "DSV41_K2I_TC", 1, {0}, {false}},
    {"topk_cluster", "DSV41_TOPK_CLUSTER", 1, {0}, {false}},
    {"row_attn", "DSV41_ROW_ATTN", 1, {0}, {false}},
};
enum {
  kOptAttnTc, kOptAttnPair, kOptDenseMinM, kOptPdl, kOptAttnBulk, kOptFusedAr, kOptK1Persistent, kOptAttnWide,
  kOptK2iTc, kOptTopkCluster, kOptRowAttn
};

int64_t option(int i) {
  Option& o = g_options[i];
  if (!o.set.load(std::memory_order_acquire)) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (!o.set.load(std::memory_order_relaxed)) {
      int64_t v = o.dflt;
      if (const char* e = getenv(o.env)) {
        if (i == kOptAttnTc) v = e[0] == 'm' ? 0 : 1;
        else if (i == kOptDenseMinM) v = std::max(1, atoi(e));
        else if (i == kOptAttnBulk || i == kOptK1Persistent) v = e[0] == '1' ? 1 : 0;
        else v = e[0] == '0' ? 0 : 1;
      }
      o.value.store(v, std::memory_order_relaxed);
      o.set.store(true, std::memory_order_release);
    }
  }
  return o.value.load(std::memory_order_relaxed);
}

bool use_tc_attention() { return option(kOptAttnTc) == 1; }
bool use_attn_pair() { return option(kOptAttnPair) == 1; }
int dense_min_rows() { return (int)option(kOptDenseMinM); }
bool use_pdl() { return option(kOptPdl) == 1; }
bool use_attn_bulk() { return option(kOptAttnBulk) == 1; }
// A row's 64 heads in one tcgen05 attention CTA (attn_wide_kernel: N = 64 MMAs, staged records,
// one f16 p) (1, default), or the 32-head kernels above (0; DSV41_ATTN_WIDE=0). Measured at config
// 2, M = 48: 243 us against the CTA pair's 392 us.
bool use_attn_wide() { return option(kOptAttnWide) == 1; }
// K2i's scorer on tcgen05 block-scaled MMAs (k2i_tc_kernel, 1, default) or on mma.sync with the fp64
// chunk epilogue (k2i_score_kernel, 0; DSV41_K2I_TC=0). Both give the contract's bits.
bool use_k2i_tc() { return option(kOptK2iTc) == 1; }
// Top-k rows of at least kTopkClMinCands candidates over a cluster of 8 CTAs each
// (topk_cluster_kernel, 1, default) or one CTA a row (topk_kernel, 0; DSV41_TOPK_CLUSTER=0).
bool use_topk_cluster() { return option(kOptTopkCluster) == 1; }
// TP > 1: each rank attends its share of the rows for all heads, the rows' queries and outputs
// exchanged in-kernel (1, default, when the caller passes every head's sinks), or its own heads for
// every row over the replicated KV cache (0; DSV41_ROW_ATTN=0).
bool use_row_attn() { return option(kOptRowAttn) == 1; }
// TP > 1: both all-reduces fused into the kernels that produce the partials (wo_b's epilogue, the
// MoE combine) as LL peer stores (1, default), or the standalone exchange kernel after each (0;
// DSV41_FUSED_AR=0).
bool use_fused_allreduce() { return option(kOptFusedAr) == 1; }
// K1 as one persistent launch when both its projections run on the CUDA-core GEMV (M below
// dense_min_rows) (1; DSV41_K1_PERSISTENT=1), or its seven launches (0, default). Measured at
// config 2 (CUDA-graph replay): K1 47-50 us persistent against 42 us for the seven launches
// chained by programmatic dependent launch, and the layer 24 us slower at M = 1 -- the five grid
// barriers cost what the launch boundaries did, and the resident grid keeps K2's first kernel
// from starting its prologue early.
bool use_k1_persistent() { return option(kOptK1Persistent) == 1; }

// CTAs of the persistent K1 an SM can hold (0: none fit), a cache per (NT, shared memory).
int k1p_blocks_per_sm(int nt, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(dev, nt, smem);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  const void* k = nt == 1 ? reinterpret_cast<const void*>(k1_persistent_kernel<1>)
                          : reinterpret_cast<const void*>(k1_persistent_kernel<2>);
  int n = 0;
  if (ensure_smem(k, smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, 256, smem) != cudaSuccess)
    n = 0;
  cudaGetLastError();
  done[key] = std::min(n, 2);
  return done[key];
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "dsv41: launch failed: %s\n", cudaGetErrorString(e));
    return DSV41_ELAUNCH;
  }
  return DSV41_OK;
}

std::atomic<int64_t> g_launches{0};

// Record stage-boundary event i of an optional host array of cudaEvent_t.
void mark(int64_t events, int i, cudaStream_t st) {
  if (events) cudaEventRecord(reinterpret_cast<cudaEvent_t*>(events)[i], st);
}

cudaError_t gemv_go(const GemvArgs& g, cudaStream_t st) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return gemv_launch(g, st, use_pdl());
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// The tensor map of a relayout expert weight: `tiles` 256-row x 128-K tiles of packed e2m1 (16 KB
// each), read as unpacked FP4 (16U4_ALIGN16B) with the 128-byte swizzle, one tile a copy.
bool expert_weight_map(CUtensorMap* m, const void* w, int64_t tiles) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc || !w || reinterpret_cast<uintptr_t>(w) % 32) return false;
  const cuuint64_t dims[3] = {128, kMxRows, (cuuint64_t)tiles};
  const cuuint64_t strides[2] = {64, 64 * kMxRows};
  const cuuint32_t box[3] = {128, kMxRows, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<void*>(w), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor map of a dense FP8 weight [N, K] read in place: 256-row x 128-K boxes, 128-byte
// swizzle, rows past N read as zeros.
bool dense_weight_map(CUtensorMap* m, const void* w, int N, int K) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc || !w || reinterpret_cast<uintptr_t>(w) % 16 || K % 16) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128, 256};
  const cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether a planned GEMV with an MXFP8 input runs on the tcgen05 dense kernel: 16 <= M <= 48
// (below, the persistent kernel's per-item latency loses to gemv_fp8_kernel: at M = 1 and 4 its
// wq_b is ~2 us faster, its shared expert ~7 us slower, and front_qkv has 16 partial slices to
// sum instead of the GEMV's few), ungrouped, N >= 256,
// K a multiple of 128, the weight 16-byte aligned. (Independent of the activation pointers, which
// are null while the scratch is only being measured.)
bool dense_eligible(const GemvArgs& g) {
  return g.M >= dense_min_rows() && g.M <= kDnMaxRows && g.N >= 256 && g.K % 128 == 0 && g.x_group_rows == g.N &&
         reinterpret_cast<uintptr_t>(g.w) % 16 == 0;
}
// Its K slicing: the longest slice (<= kDnKsMax, dividing K) that still gives a (256-row tile,
// slice) pair to every SM, at most 16 slices (the consumer sums the slices' partials); and the
// row-tile groups an item covers.
DenseTcArgs dense_args(const GemvArgs& g, const uint8_t* x8, const uint8_t* xs, int sms) {
  DenseTcArgs d = {};
  d.M = g.M; d.N = g.N; d.K = g.K;
  int ks = std::min(g.K, kDnKsMax) / 128 * 128;
  while (g.K % ks) ks -= 128;
  d.rtiles = cdiv(g.N, 256);
  while (ks > 128 && d.rtiles * (g.K / ks) < sms && g.K / ks < 16 && (ks / 2) % 128 == 0 && g.K % (ks / 2) == 0)
    ks /= 2;
  d.ks_len = ks;
  d.kslices = g.K / ks;
  d.row_groups = std::max(1, std::min(d.rtiles, cdiv(sms, d.kslices)));
  d.codes = g.codes; d.x = x8; d.xs = xs; d.x_ld = g.K; d.out = g.out;
  return d;
}
// Plan time: a dense-eligible GEMV takes the dense kernel's K slice count (its partials' count).
void dense_replan(GemvArgs& g, int sms) {
  if (dense_eligible(g)) g.kslices = dense_args(g, nullptr, nullptr, sms).kslices;
}

// cluster_x > 1: consecutive blocks along x form clusters of that size
template <typename Kern, typename Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, int smem, cudaStream_t st, const Args& args,
                   int cluster_x = 1) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (smem > 48 * 1024) {
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kernel), smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = use_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args);
}

// The same with any kernel parameters (no cluster).
template <typename... Exp, typename... Act>
cudaError_t launch_n(void (*kernel)(Exp...), dim3 grid, dim3 block, int smem, cudaStream_t st, Act&&... args) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = use_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// The same with two kernel parameters (a tensor map, then the arguments).
template <typename Kern, typename A0, typename A1>
cudaError_t launch2(Kern kernel, dim3 grid, dim3 block, int smem, cudaStream_t st, const A0& a0, const A1& a1) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (smem > 48 * 1024) {
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kernel), smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = use_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a0, a1);
}

// A planned GEMV: the tcgen05 dense kernel when its input is MXFP8, else gemv_fp8_kernel.
cudaError_t dense_go(const GemvArgs& g, const uint8_t* x8, const uint8_t* xs, cudaStream_t st) {
  if (!dense_eligible(g)) return gemv_go(g, st);
  if (!x8 || !xs) return cudaErrorInvalidValue;
  const DenseTcArgs d = dense_args(g, x8, xs, sm_count());
  CUtensorMap m;
  if (!dense_weight_map(&m, g.w, g.N, g.K)) {
    fprintf(stderr, "dsv41: dense weight tensor map failed (driver entry point or alignment)\n");
    return cudaErrorInvalidValue;
  }
  return launch2(dense_tc_kernel, dim3(std::min(sm_count(), d.kslices * d.row_groups)), dim3(kDnThreads),
                 DnSmem::kBytes, st, m, d);
}

// Bump allocation over the caller's scratch; with a null base it only measures.
struct Carver {
  uint8_t* base;
  int64_t off = 0;
  template <class T>
  T* take(int64_t count) {
    off = (off + 255) & ~(int64_t)255;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * (int64_t)sizeof(T);
    return p;
  }
};

template <class T>
T* ptr(int64_t v) {
  return reinterpret_cast<T*>(v);
}

int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > 4 * 148 * 8) g = 4 * 148 * 8;
  return (int)g;
}

#define DSV41_TRY(expr)                       \
  do {                                        \
    if ((expr) != cudaSuccess) return launch_status(); \
  } while (0)

// ------------------------------------------------------------------ K1
bool k1_ok(const Dsv41K1Args* a) {
  if (!a || a->M < 1 || a->M > 48 || a->hidden % 256 || a->hidden > 16384) return false;
  if (!(a->q_lora == 256 || a->q_lora == 512 || a->q_lora == 1024)) return false;
  if (a->nope % 64 || a->rope != 64 || a->nope < 64 || a->nope > 512) return false;
  if (a->heads < 1 || (a->heads * (a->nope + a->rope)) % 16) return false;
  if (!a->res_in || !a->hc_fn || !a->norm_w || !a->wqkv || !a->wqb || !a->q || !a->cache) return false;
  if (a->fold && (!a->x_in || !a->post_in || !a->comb_in)) return false;
  if (!a->first && !a->pre_in) return false;
  if (a->build_kt && (!a->kt || !a->klen || !a->swa_idx || !a->swa_lens)) return false;
  if (a->build_kt && a->topk_width > 0 && (!a->topk_idx || !a->topk_lens)) return false;
  if (a->index && !a->qr) return false;
  if (a->hidden % 128 || a->q_lora % 128) return false;
  if (a->q % 16) return false;  // q_rope stores 8 bf16 (16 bytes) at a time
  return true;
}

int k1_run(const Dsv41K1Args* a, cudaStream_t st, bool go, int64_t* need) {
  if (!k1_ok(a)) return DSV41_EINVAL;
  const int M = (int)a->M, H = (int)a->hidden, QL = (int)a->q_lora;
  const int nope = (int)a->nope, rope = (int)a->rope, D = nope + rope, heads = (int)a->heads;
  const int QKV = QL + D;
  const int sms = sm_count();
  Carver c{go ? ptr<uint8_t>(a->scratch) : nullptr};
  auto* k1p_bar = c.take<unsigned>(64);  // the persistent launch's grid-barrier word
  auto* lin = c.take<__nv_bfloat16>((int64_t)M * H);
  auto* part = c.take<float>((int64_t)M * (H / 32) * kPart);
  auto* xq = c.take<__nv_bfloat16>((int64_t)M * H);
  auto* x8 = a->x8 ? ptr<uint8_t>(a->x8) : c.take<uint8_t>((int64_t)M * H);
  auto* x8s = a->x8s ? ptr<uint8_t>(a->x8s) : c.take<uint8_t>((int64_t)M * H / 32);
  auto* normed = a->normed ? ptr<__nv_bfloat16>(a->normed) : c.take<__nv_bfloat16>((int64_t)M * H);
  auto* res_out = a->res_out ? ptr<__nv_bfloat16>(a->res_out) : c.take<__nv_bfloat16>((int64_t)M * 4 * H);
  auto* post_out = a->post_out ? ptr<float>(a->post_out) : c.take<float>(M * 4);
  auto* comb_out = a->comb_out ? ptr<float>(a->comb_out) : c.take<float>(M * 16);
  auto* pre_out = a->pre_out ? ptr<float>(a->pre_out) : c.take<float>(M * 4);
  GemvArgs g1 = gemv_plan(ptr<const uint8_t>(a->wqkv), ptr<const uint8_t>(a->wqkv_codes), xq, nullptr,
                          M, QKV, H, H, 0, sms);
  dense_replan(g1, sms);
  g1.out = c.take<float>((int64_t)g1.kslices * M * QKV);
  auto* qxq = c.take<__nv_bfloat16>((int64_t)M * QL);
  auto* qx8 = a->qx8 ? ptr<uint8_t>(a->qx8) : c.take<uint8_t>((int64_t)M * QL);
  auto* qx8s = a->qx8s ? ptr<uint8_t>(a->qx8s) : c.take<uint8_t>((int64_t)M * QL / 32);
  GemvArgs g2 = gemv_plan(ptr<const uint8_t>(a->wqb), ptr<const uint8_t>(a->wqb_codes), qxq, nullptr,
                          M, heads * D, QL, QL, 0, sms);
  dense_replan(g2, sms);
  g2.out = c.take<float>((int64_t)g2.kslices * M * heads * D);
  *need = c.off;
  if (!go) return DSV41_OK;
  if (!a->scratch || a->scratch_bytes < c.off) return DSV41_ESCRATCH;

  SeamArgs s = {};
  s.M = M; s.H = H; s.fold = (int)a->fold; s.first = (int)a->first; s.aiter = 0;
  s.res_in = ptr<const __nv_bfloat16>(a->res_in); s.x = ptr<const __nv_bfloat16>(a->x_in);
  s.post_in = ptr<const float>(a->post_in); s.comb_in = ptr<const float>(a->comb_in);
  s.pre_in = ptr<const float>(a->pre_in); s.hc_fn = ptr<const float>(a->hc_fn);
  s.hc_scale = ptr<const float>(a->hc_scale); s.hc_base = ptr<const float>(a->hc_base);
  s.norm_w = ptr<const __nv_bfloat16>(a->norm_w);
  s.res_out = res_out; s.pre_out = pre_out; s.post_out = post_out; s.comb_out = comb_out;
  s.normed = normed; s.x8 = x8; s.x8s = x8s; s.xq = xq; s.lin = lin; s.part = part;
  FrontArgs f = {};
  f.M = M; f.QL = QL; f.KVD = D; f.nope = nope; f.rope = rope; f.kslices = g1.kslices;
  f.index = (int)a->index; f.qkv_part = g1.out;
  f.q_norm_w = ptr<const __nv_bfloat16>(a->q_norm); f.kv_norm_w = ptr<const __nv_bfloat16>(a->kv_norm);
  f.cos_sin = ptr<const float>(a->cos_sin); f.pos = ptr<const int64_t>(a->pos); f.rope_rows = a->rope_rows;
  f.slot = ptr<const int64_t>(a->slot); f.cache = ptr<uint8_t>(a->cache);
  f.page_stride = a->page_stride; f.blk = (int)a->blk;
  f.qr = ptr<__nv_bfloat16>(a->qr); f.qx8 = qx8; f.qx8s = qx8s; f.qxq = qxq;
  f.qkv_out = ptr<float>(a->qkv_out);
  KeyTableArgs k = {};
  k.M = M; k.swa_width = (int)a->swa_width; k.topk_width = (int)a->topk_width;
  k.slot = ptr<const int64_t>(a->slot); k.swa_idx = ptr<const int32_t>(a->swa_idx);
  k.swa_lens = ptr<const int32_t>(a->swa_lens); k.topk = ptr<const int32_t>(a->topk_idx);
  k.topk_lens = ptr<const int32_t>(a->topk_lens); k.kt = ptr<int32_t>(a->kt);
  k.klen = ptr<int32_t>(a->klen);
  const int kt_keys = (int)(a->swa_width + a->topk_width);
  const int kt_y = std::max(1, std::min(cdiv(kt_keys, 1024), 16));
  QRopeArgs qr = {};
  qr.M = M; qr.heads = heads; qr.D = D; qr.nope = nope; qr.rope = rope; qr.kslices = g2.kslices;
  qr.part = g2.out; qr.cos_sin = ptr<const float>(a->cos_sin); qr.pos = ptr<const int64_t>(a->pos);
  qr.rope_rows = a->rope_rows;
  qr.q = ptr<__nv_bfloat16>(a->q);
  const int qr_x = cdiv(heads * D / 8, 256);

  // ---- the persistent K1 (both projections on the CUDA-core GEMV)
  const int nt = cdiv(M, 8);
  const int p_smem = std::max(kSeamSliceSmem, std::max(gemv_smem_bytes(M, g1.ks_blocks), gemv_smem_bytes(M, g2.ks_blocks)));
  const int p_bps = use_k1_persistent() && !dense_eligible(g1) && !dense_eligible(g2) && nt <= 2
                        ? k1p_blocks_per_sm(nt, p_smem) : 0;
  if (p_bps > 0) {
    K1PArgs kp = {};
    kp.s = s; kp.k = k; kp.kt_rows = a->build_kt ? M : 0; kp.kt_y = kt_y;
    kp.g1 = g1; kp.f = f; kp.g2 = g2; kp.qr = qr; kp.qr_x = qr_x; kp.bar = k1p_bar;
    const bool aligned = reinterpret_cast<uintptr_t>(g1.w) % 16 == 0 && reinterpret_cast<uintptr_t>(g2.w) % 16 == 0;
    kp.pf[0] = aligned ? g1.w : nullptr; kp.pf_bytes[0] = (int64_t)QKV * H;
    kp.pf[1] = aligned ? g2.w : nullptr; kp.pf_bytes[1] = (int64_t)heads * D * QL;
    mark(a->events, 0, st);
    DSV41_TRY(cudaMemsetAsync(k1p_bar, 0, 4, st));
    const dim3 grid(p_bps * sms), block(256);
    DSV41_TRY(nt == 1 ? launch(k1_persistent_kernel<1>, grid, block, p_smem, st, kp)
                      : launch(k1_persistent_kernel<2>, grid, block, p_smem, st, kp));
    for (int i = 1; i <= 4; ++i) mark(a->events, i, st);
    return launch_status();
  }

  mark(a->events, 0, st);
  DSV41_TRY(launch(seam_slice_kernel, dim3(H / kSliceCols), dim3(256), 0, st, s));
  DSV41_TRY(launch(seam_gate_norm_kernel, dim3(M), dim3(256), 0, st, s));
  mark(a->events, 1, st);
  DSV41_TRY(dense_go(g1, x8, x8s, st));
  mark(a->events, 2, st);
  DSV41_TRY(launch(front_qkv_kernel, dim3(M), dim3(256), 0, st, f));
  if (a->build_kt) DSV41_TRY(launch(key_table_kernel, dim3(M, kt_y), dim3(256), 0, st, k));
  mark(a->events, 3, st);
  DSV41_TRY(dense_go(g2, qx8, qx8s, st));
  DSV41_TRY(launch(q_rope_kernel, dim3(qr_x, M), dim3(256), 0, st, qr));
  mark(a->events, 4, st);
  return launch_status();
}

// ------------------------------------------------------------------ K2
bool k2_ok(const Dsv41K2Args* a) {
  if (!a || a->M < 1 || a->M > 48 || a->hidden % 256 || a->hidden > 16384) return false;
  if (a->nope % 64 || a->rope != 64 || a->nope > 512 || a->heads < 1) return false;
  if (a->o_groups < 1 || a->o_rank % 128 || a->heads % a->o_groups) return false;
  if (((a->heads / a->o_groups) * (a->nope + a->rope)) % 128) return false;
  if (a->experts < 1 || a->experts > 512 || a->topk < 1 || a->topk > 32) return false;
  if (a->inter % 128 || a->shared_inter % 128 || a->tp < 1 || a->tp > kPeerMaxTp) return false;
  if (a->rank < 0 || a->rank >= a->tp || a->phase < 0 || a->phase > 2 || a->inject < 0 || a->inject > 2)
    return false;
  if (a->tp > 1 && a->phase == 0 && (!a->peers || a->peer_cap < a->M * a->hidden || a->peer_cap % 8))
    return false;
  if (a->phase == 2 && (!a->attn || !a->moe_part)) return false;
  if (a->moe_part % 16) return false;  // the MoE combine stores 8 bf16 (16 bytes) at a time
  if (a->phase == 1 && !a->attn_part) return false;
  if (!a->q || !a->kt || !a->klen || !a->swa || !a->sink || !a->woa || !a->wob) return false;
  // KV records are fetched by bulk copies: page bases and strides 16-byte aligned
  if (a->swa % 16 || a->swa_stride % 16 || (a->comp && (a->comp % 16 || a->comp_stride % 16))) return false;
  if (!a->res_in || !a->post_in || !a->comb_in || !a->pre_in || !a->hc_fn || !a->norm_w) return false;
  if (!a->gate_w || !a->w13 || !a->w2 || !a->sgu || !a->sw2 || !a->out || !a->ids || !a->wts) return false;
  if (!a->route_softmax && !a->bias) return false;
  if (a->hidden % 1024 && a->hidden > 1024) return false;
  return true;
}

int64_t deadline_or_default(int64_t ns) { return ns > 0 ? ns : 5000000000LL; }

// One in-kernel exchange: CTAs of 256 threads, a thread a 16-byte vector, at most kArBlocks
// (every CTA resident, so each CTA's wait only needs the same CTA on the other ranks).
cudaError_t allreduce_go(int n, int tp, int rank, int64_t peers, int64_t cap, const void* src, void* dst,
                         int64_t deadline_ns, int site, int skip, cudaStream_t st) {
  AllReduceArgs r = {};
  r.n = n; r.tp = tp; r.rank = rank;
  r.nblk = std::max(1, std::min(kArBlocks, cdiv(n / 8, 256)));
  r.peers = ptr<const int64_t>(peers); r.cap = cap;
  r.src = reinterpret_cast<const __nv_bfloat16*>(src); r.dst = reinterpret_cast<__nv_bfloat16*>(dst);
  r.deadline_ns = deadline_or_default(deadline_ns); r.site = site; r.skip_push = skip;
  return launch(allreduce_kernel, dim3(r.nblk), dim3(256), 0, st, r);
}

struct K2Plan {
  int head_tiles, nchunks, chunk_keys;
  GemvArgs ga, gb, gs, gd;
  ExpertArgs eu, ed;
};

int k2_run(const Dsv41K2Args* a, cudaStream_t st, bool go, int64_t* need) {
  if (!k2_ok(a)) return DSV41_EINVAL;
  const int M = (int)a->M, H = (int)a->hidden, nope = (int)a->nope, rope = (int)a->rope;
  const int D = nope + rope, heads = (int)a->heads, G = (int)a->o_groups, O = (int)a->o_rank;
  const int E = (int)a->experts, TK = (int)a->topk, I = (int)a->inter, SI = (int)a->shared_inter;
  const int P = M * TK, keys = (int)a->keys_ld;
  const int sms = sm_count();
  Carver c{go ? ptr<uint8_t>(a->scratch) : nullptr};
  // row-parallel attention (TP > 1): this rank's rows [row0, row0 + Mr) for all Ha heads
  const int tpn = (int)a->tp, mr = cdiv(M, tpn);
  const bool rowattn = tpn > 1 && a->phase == 0 && a->sink_all != 0 && use_row_attn() && use_fused_allreduce() &&
                       M >= tpn && (int64_t)mr * heads * D <= a->peer_cap;
  const int Ma = rowattn ? mr : M, Ha = rowattn ? heads * tpn : heads;
  const int row0 = rowattn ? (int)a->rank * mr : 0, Mr = rowattn ? std::min(M, row0 + mr) - row0 : M;
  // attention split plan: the tcgen05 kernel takes every head of a row (one CTA an SM in
  // total), the mma.sync kernel 16-head tiles (two CTAs an SM)
  const bool tc = use_tc_attention() && (nope == 512 || nope == 448);
  const bool wide = tc && nope == 512 && Ha == kWdNH && use_attn_wide();
  const int head_tiles = wide ? 1 : tc ? cdiv(Ha, 32) : cdiv(Ha, 16);
  const int units = Ma * head_tiles;
  int nchunks = cdiv(2 * sms, units);
  const int sub = tc ? kTcKeys : kSub;  // keys a sub-block
  if (tc) {
    // one CTA an SM: the split with the fewest sub-block periods over all waves, a CTA's start
    // and drain counted as 4 periods (ties: fewer chunks, so fewer partials for the combine)
    int64_t best = INT64_MAX;
    for (int c = 1; c <= cdiv(keys, sub); ++c) {
      const int64_t cost = (int64_t)cdiv(units * c, sms) * (cdiv(cdiv(keys, c), sub) + 4);
      if (cost < best) best = cost, nchunks = c;
    }
  }
  nchunks = std::max(1, std::min(nchunks, cdiv(keys, sub)));
  const int chunk_keys = cdiv(cdiv(keys, nchunks), sub) * sub;
  nchunks = cdiv(keys, chunk_keys);
  auto* part_o = c.take<float>((int64_t)Ma * nchunks * Ha * D);
  auto* part_ml = c.take<float>((int64_t)Ma * nchunks * Ha * 2);
  auto* xo = a->xo ? ptr<__nv_bfloat16>(a->xo) : c.take<__nv_bfloat16>((int64_t)M * heads * D);
  // row-parallel attention: this rank's rows' queries and outputs for every head
  auto* q_all = rowattn ? c.take<__nv_bfloat16>((int64_t)Ma * Ha * D) : nullptr;
  auto* xo_rows = rowattn ? c.take<__nv_bfloat16>((int64_t)Ma * Ha * D) : nullptr;
  const int gk = heads / G * D;  // wo_a's K a group
  GemvArgs ga = gemv_plan(ptr<const uint8_t>(a->woa), ptr<const uint8_t>(a->woa_codes), xo, nullptr,
                          M, G * O, gk, heads * D, O, sms);
  ga.out = c.take<float>((int64_t)ga.kslices * M * G * O);
  auto* x8bq = c.take<__nv_bfloat16>((int64_t)M * G * O);
  auto* x8b = a->x8b ? ptr<uint8_t>(a->x8b) : c.take<uint8_t>((int64_t)M * G * O);
  auto* x8bs = a->x8bs ? ptr<uint8_t>(a->x8bs) : c.take<uint8_t>((int64_t)M * G * O / 32);
  GemvArgs gb = gemv_plan(ptr<const uint8_t>(a->wob), ptr<const uint8_t>(a->wob_codes), x8bq, nullptr,
                          M, H, G * O, G * O, 0, sms);
  dense_replan(gb, sms);
  gb.out = c.take<float>((int64_t)gb.kslices * M * H);
  auto* attn_part = a->attn_part ? ptr<__nv_bfloat16>(a->attn_part) : c.take<__nv_bfloat16>((int64_t)M * H);
  auto* attn = a->attn ? ptr<__nv_bfloat16>(a->attn) : c.take<__nv_bfloat16>((int64_t)M * H);
  // FFN seam
  auto* lin = c.take<__nv_bfloat16>((int64_t)M * H);
  auto* spart = c.take<float>((int64_t)M * (H / 32) * kPart);
  auto* xq = c.take<__nv_bfloat16>((int64_t)M * H);
  auto* x8 = c.take<uint8_t>((int64_t)M * H);
  auto* x8s = c.take<uint8_t>((int64_t)M * H / 32);
  auto* x8r = c.take<uint8_t>((int64_t)M * H);
  auto* x8rs = c.take<uint8_t>((int64_t)M * H / 32);
  auto* normed = a->normed ? ptr<__nv_bfloat16>(a->normed) : c.take<__nv_bfloat16>((int64_t)M * H);
  auto* res_out = a->res_out ? ptr<__nv_bfloat16>(a->res_out) : c.take<__nv_bfloat16>((int64_t)M * 4 * H);
  auto* post_out = a->post_out ? ptr<float>(a->post_out) : c.take<float>(M * 4);
  auto* comb_out = a->comb_out ? ptr<float>(a->comb_out) : c.take<float>(M * 16);
  auto* pre_out = a->pre_out ? ptr<float>(a->pre_out) : c.take<float>(M * 4);
  // MoE
  auto* logits = a->logits ? ptr<float>(a->logits) : c.take<float>((int64_t)M * E);
  auto* n_u = c.take<int32_t>(1);
  auto* u_expert = c.take<int32_t>(E);
  auto* u_off = c.take<int32_t>(E + 1);
  auto* picks = c.take<int32_t>(P);
  GemvArgs gs = gemv_plan(ptr<const uint8_t>(a->sgu), ptr<const uint8_t>(a->sgu_codes), xq, nullptr,
                          M, 2 * SI, H, H, 0, sms);
  dense_replan(gs, sms);
  gs.out = c.take<float>((int64_t)gs.kslices * M * 2 * SI);
  auto* smq = c.take<uint8_t>((int64_t)M * SI);
  auto* smqs = c.take<uint8_t>((int64_t)M * SI / 32);
  auto* smx = c.take<__nv_bfloat16>((int64_t)M * SI);
  GemvArgs gd = gemv_plan(ptr<const uint8_t>(a->sw2), ptr<const uint8_t>(a->sw2_codes), smx, nullptr,
                          M, H, SI, SI, 0, sms);
  dense_replan(gd, sms);
  gd.out = c.take<float>((int64_t)gd.kslices * M * H);
  const int max_units = std::min(E, P);
  ExpertArgs eu = {};
  eu.M = M; eu.topk = TK; eu.N = 2 * I; eu.K = H; eu.ks_len = std::min(H, 1024);
  eu.kslices = cdiv(H, eu.ks_len); eu.row_groups = cdiv(2 * I, kMxRows); eu.max_units = max_units;
  eu.w = ptr<const uint8_t>(a->w13); eu.ws = ptr<const uint8_t>(a->w13_codes);
  eu.x = x8r; eu.xs = x8rs; eu.x_by_pick = 0;
  eu.n_u = n_u; eu.u_expert = u_expert; eu.u_off = u_off; eu.picks = picks;
  eu.out = c.take<float>((int64_t)eu.kslices * P * 2 * I);
  auto* mid = c.take<uint8_t>((int64_t)P * I);
  auto* mids = c.take<uint8_t>((int64_t)P * I / 32);
  ExpertArgs ed = eu;
  ed.N = H; ed.K = I; ed.ks_len = std::min(I, 1024); ed.kslices = cdiv(I, ed.ks_len);
  ed.row_groups = cdiv(H, kMxRows); ed.w = ptr<const uint8_t>(a->w2); ed.ws = ptr<const uint8_t>(a->w2_codes);
  ed.x = mid; ed.xs = mids; ed.x_by_pick = 1;
  ed.out = c.take<float>((int64_t)ed.kslices * P * H);
  auto* moe_part = a->moe_part ? ptr<__nv_bfloat16>(a->moe_part) : c.take<__nv_bfloat16>((int64_t)M * H);
  *need = c.off;
  if (!go) return DSV41_OK;
  if (!a->scratch || a->scratch_bytes < c.off) return DSV41_ESCRATCH;
  if (eu.ks_len % 128 || ed.ks_len % 128 || H % eu.ks_len || I % ed.ks_len || eu.ks_len > kMxKsMax ||
      ed.ks_len > kMxKsMax)
    return DSV41_EINVAL;

  const int phase = (int)a->phase, tp = (int)a->tp, rank = (int)a->rank;
  const __nv_bfloat16* reduced = attn;
  // the fused exchanges: every CTA resident (a thread pushes all its groups before it waits)
  const bool fused = tp > 1 && phase == 0 && use_fused_allreduce();
  auto exchange = [&](int site, __nv_bfloat16* dst) {
    PeerLL x = {};
    x.peers = ptr<const int64_t>(a->peers); x.tp = tp; x.rank = rank; x.site = site;
    x.skip = a->inject == site; x.cap = a->peer_cap; x.deadline_ns = deadline_or_default(a->deadline_ns);
    x.reduced = dst;
    return x;
  };
  const int xgrid = std::min(grid_for((int64_t)M * H / 8, 256), 4 * sms);
  if (phase != 2) {
  // ---- attention
  mark(a->events, 0, st);
  const int a2a_grid = std::min(grid_for((int64_t)mr * heads * D / 8, 256), 4 * sms);
  if (rowattn) {
    // the rows' queries of every rank's heads (exchange site 3)
    A2AArgs qa = {0, M, mr, heads, D, ptr<const __nv_bfloat16>(a->q), q_all};
    DSV41_TRY(launch2(ll_a2a_kernel, dim3(a2a_grid), dim3(256), 0, st, exchange(3, nullptr), qa));
  }
  AttnArgs at = {};
  at.M = Mr; at.heads = Ha; at.D = D; at.nope = nope; at.rope = rope; at.keys_ld = keys;
  at.nchunks = nchunks; at.chunk_keys = chunk_keys; at.head_tiles = head_tiles;
  at.q = rowattn ? q_all : ptr<const __nv_bfloat16>(a->q);
  at.kt = ptr<const int32_t>(a->kt) + (int64_t)row0 * keys; at.klen = ptr<const int32_t>(a->klen) + row0;
  at.swa = ptr<const uint8_t>(a->swa); at.swa_stride = a->swa_stride; at.swa_blk = (int)a->swa_blk;
  at.comp = ptr<const uint8_t>(a->comp); at.comp_stride = a->comp_stride; at.comp_blk = (int)(a->comp_blk ? a->comp_blk : 1);
  at.scale_log2 = (float)(1.0 / sqrt((double)D) * 1.4426950408889634);
  at.part_o = part_o; at.part_ml = part_ml;
  if (wide) {
    DSV41_TRY(launch(attn_wide_kernel<512>, dim3(Mr * nchunks), dim3(kWdThreads), WdSmem<576>::kBytes, st, at));
  } else if (tc) {
    AttnTcArgs ta = {at, Ha >= 32 ? 32 : std::max(16, cdiv(Ha, 16) * 16), head_tiles};
    // the staged producer (lone CTAs), or a row's two head tiles sharing their key tiles as a
    // CTA pair, or lone gathering CTAs
    const bool bulk = use_attn_bulk();
    const bool pair = !bulk && head_tiles == 2 && use_attn_pair();
    const dim3 grid(Mr * nchunks * head_tiles), block(kTcThreads);
    using S576 = TcSmem<576, kTcBulkStages, kTcStaging>;
    using S512 = TcSmem<512, kTcBulkStages, kTcStaging>;
    if (nope == 512)
      DSV41_TRY(bulk ? launch(attn_tc_kernel<512, false, true>, grid, block, S576::kBytes, st, ta)
                : pair ? launch(attn_tc_kernel<512, true>, grid, block, TcSmem<576>::kBytes, st, ta, 2)
                       : launch(attn_tc_kernel<512, false>, grid, block, TcSmem<576>::kBytes, st, ta));
    else
      DSV41_TRY(bulk ? launch(attn_tc_kernel<448, false, true>, grid, block, S512::kBytes, st, ta)
                : pair ? launch(attn_tc_kernel<448, true>, grid, block, TcSmem<512>::kBytes, st, ta, 2)
                       : launch(attn_tc_kernel<448, false>, grid, block, TcSmem<512>::kBytes, st, ta));
  } else {
    DSV41_TRY(launch(attn_split_kernel, dim3(Mr * nchunks * head_tiles), dim3(256), attn_smem_bytes(D), st, at));
  }
  CombineArgs cb = {};
  cb.M = Mr; cb.heads = Ha; cb.D = D; cb.nope = nope; cb.rope = rope; cb.nchunks = nchunks;
  cb.part_o = part_o; cb.part_ml = part_ml;
  cb.sink = ptr<const float>(rowattn ? a->sink_all : a->sink);
  cb.cos_sin = ptr<const float>(a->cos_sin); cb.pos = ptr<const int64_t>(a->pos) + row0;
  cb.xo = rowattn ? xo_rows : xo;
  cb.rope_rows = a->rope_rows;
  DSV41_TRY(nchunks > 16 && Mr * Ha <= sms
                ? launch(attn_combine_kernel<32>, dim3(Mr * Ha), dim3(kCombineThreads), nchunks * 8, st, cb)
                : launch(attn_combine_kernel<16>, dim3(Mr * Ha), dim3(kCombineThreads), nchunks * 8, st, cb));
  if (rowattn) {
    // every row's output for this rank's heads (exchange site 4)
    A2AArgs oa = {1, M, mr, heads, D, xo_rows, xo};
    DSV41_TRY(launch2(ll_a2a_kernel, dim3(a2a_grid), dim3(256), 0, st, exchange(4, nullptr), oa));
  }
  // ---- wo_a -> X8B -> wo_b -> partial -> reduce
  mark(a->events, 1, st);
  DSV41_TRY(gemv_go(ga, st));
  FinalizeArgs fa = {M, G * O, ga.kslices, ga.out, x8bq, x8b, x8bs};
  DSV41_TRY(launch(finalize_kernel, dim3(grid_for((int64_t)M * G * O / 8, 256)), dim3(256), 0, st, fa));
  DSV41_TRY(dense_go(gb, x8b, x8bs, st));
  FinalizeArgs fb = {M, H, gb.kslices, gb.out, attn_part, nullptr, nullptr};
  if (fused) fb.x = exchange(1, attn);  // + the attention all-reduce into attn
  DSV41_TRY(launch(finalize_kernel, dim3(fused ? xgrid : grid_for((int64_t)M * H / 8, 256)), dim3(256), 0, st, fb));
  mark(a->events, 2, st);
  if (phase == 1) return launch_status();
  if (fused) {
    // reduced in the wo_b epilogue
  } else if (tp > 1) {
    // the attention all-reduce (site 1)
    DSV41_TRY(allreduce_go(M * H, tp, rank, a->peers, a->peer_cap, attn_part, attn, a->deadline_ns, 1,
                           a->inject == 1, st));
  } else if (attn != attn_part) {
    // tp == 1: the all-reduce of one rank's bf16 partial is the partial itself
    DSV41_TRY(cudaMemcpyAsync(attn, attn_part, (size_t)M * H * 2, cudaMemcpyDeviceToDevice, st));
  } else {
    reduced = attn_part;
  }
  }
  // ---- FFN seam
  SeamArgs s = {};
  s.M = M; s.H = H; s.fold = 1; s.first = 0; s.aiter = 1;
  s.res_in = ptr<const __nv_bfloat16>(a->res_in); s.x = reduced;
  s.post_in = ptr<const float>(a->post_in); s.comb_in = ptr<const float>(a->comb_in);
  s.pre_in = ptr<const float>(a->pre_in); s.hc_fn = ptr<const float>(a->hc_fn);
  s.hc_scale = ptr<const float>(a->hc_scale); s.hc_base = ptr<const float>(a->hc_base);
  s.norm_w = ptr<const __nv_bfloat16>(a->norm_w);
  s.res_out = res_out; s.pre_out = pre_out; s.post_out = post_out; s.comb_out = comb_out;
  s.normed = normed; s.x8 = x8; s.x8s = x8s; s.xq = xq; s.x8r = x8r; s.x8rs = x8rs;
  s.lin = lin; s.part = spart;
  DSV41_TRY(launch(seam_slice_kernel, dim3(H / kSliceCols), dim3(256), 0, st, s));
  DSV41_TRY(launch(seam_gate_norm_kernel, dim3(M), dim3(256), 0, st, s));
  // ---- router, routing, union
  // rows a CTA: 4 once 8 would leave the SMs short of CTAs (M > 8)
  const int rpc = M > 8 ? 4 : 8;
  const int router_smem = 2 * rpc * H <= 200 * 1024 ? 2 * rpc * H : 0;
  RouterArgs ra = {M, E, H, normed, ptr<const __nv_bfloat16>(a->gate_w), logits, router_smem > 0};
  mark(a->events, 3, st);
  DSV41_TRY(rpc == 4 ? launch(router_kernel<4>, dim3(cdiv(E, 8), cdiv(M, 4)), dim3(256), router_smem, st, ra)
                     : launch(router_kernel<8>, dim3(cdiv(E, 8), cdiv(M, 8)), dim3(256), router_smem, st, ra));
  RouteArgs rt = {M, E, TK, (int)a->route_softmax, logits, ptr<const float>(a->bias),
                  ptr<int32_t>(a->ids), ptr<float>(a->wts)};
  PlanArgs pl = {M, E, TK, ptr<const int32_t>(a->ids), n_u, u_expert, u_off, picks};
  if (M <= kRoutePlanRows) {
    DSV41_TRY(launch2(route_plan_kernel, dim3(1), dim3(512), 0, st, rt, pl));
  } else {
    DSV41_TRY(launch(route_kernel, dim3(M), dim3(256), 0, st, rt));
    DSV41_TRY(launch(moe_plan_kernel, dim3(1), dim3(512), 0, st, pl));
  }
  // ---- shared expert
  mark(a->events, 4, st);
  DSV41_TRY(dense_go(gs, x8, x8s, st));
  SharedActArgs sa = {M, SI, gs.kslices, gs.out, smq, smqs, smx};
  DSV41_TRY(launch(shared_act_kernel, dim3(grid_for((int64_t)M * SI / 8, 256)), dim3(256), 0, st, sa));
  DSV41_TRY(dense_go(gd, smq, smqs, st));
  mark(a->events, 5, st);
  // ---- routed experts: persistent tcgen05 grouped GEMMs, one CTA an SM
  {
    CUtensorMap m13, m2;
    if (!expert_weight_map(&m13, ptr<const void>(a->w13), (int64_t)E * eu.row_groups * (H / 128)) ||
        !expert_weight_map(&m2, ptr<const void>(a->w2), (int64_t)E * ed.row_groups * (I / 128))) {
      fprintf(stderr, "dsv41: expert weight tensor map failed (driver entry point or alignment)\n");
      return DSV41_ELAUNCH;
    }
    const ExpertTcArgs tu = {M, TK, 2 * I, H, eu.kslices, eu.ks_len, eu.row_groups, eu.ws, eu.x, eu.xs, 0,
                             n_u, u_expert, u_off, picks, eu.out};
    const ExpertTcArgs td = {M, TK, H, I, ed.kslices, ed.ks_len, ed.row_groups, ed.ws, ed.x, ed.xs, 1,
                             n_u, u_expert, u_off, picks, ed.out};
    DSV41_TRY(launch2(expert_tc_kernel, dim3(std::min(sms, max_units * eu.kslices * eu.row_groups)),
                      dim3(kMxThreads), MxSmem::kBytes, st, m13, tu));
    ExpertActArgs ea = {P, I, eu.kslices, eu.out, mid, mids};
    DSV41_TRY(launch(expert_act_kernel, dim3(grid_for((int64_t)P * I / 8, 256)), dim3(256), 0, st, ea));
    DSV41_TRY(launch2(expert_tc_kernel, dim3(std::min(sms, max_units * ed.kslices * ed.row_groups)),
                      dim3(kMxThreads), MxSmem::kBytes, st, m2, td));
  }
  CombineMoeArgs cm = {M, H, TK, ed.kslices, gd.kslices, ed.out, ptr<const float>(a->wts), gd.out, moe_part};
  if (fused) cm.x = exchange(2, ptr<__nv_bfloat16>(a->out));  // + the MoE all-reduce into out
  mark(a->events, 6, st);
  DSV41_TRY(launch(moe_combine_kernel, dim3(fused ? xgrid : grid_for((int64_t)M * H / 8, 256)), dim3(256), 0, st, cm));
  if (phase == 2) return launch_status();
  if (fused) {
    // reduced in the combine
  } else if (tp > 1) {
    // the MoE all-reduce (site 2)
    DSV41_TRY(allreduce_go(M * H, tp, rank, a->peers, a->peer_cap, moe_part, ptr<void>(a->out), a->deadline_ns,
                           2, a->inject == 2, st));
  } else if (ptr<__nv_bfloat16>(a->out) != moe_part) {
    // tp == 1: the MoE all-reduce of one partial is the partial
    DSV41_TRY(cudaMemcpyAsync(ptr<void>(a->out), moe_part, (size_t)M * H * 2, cudaMemcpyDeviceToDevice, st));
  }
  mark(a->events, 7, st);
  return launch_status();
}

}  // namespace

extern "C" {

int64_t dsv41_launch_count(void) { return g_launches.load(); }

int dsv41_device_error(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, dsv41::g_tc_error, sizeof(v)) != cudaSuccess) return launch_status();
  return v ? DSV41_EDEVICE : DSV41_OK;
}

int dsv41_version(void) { return 1; }

int dsv41_set_option(const char* name, int64_t value) {
  if (!name) return DSV41_EINVAL;
  for (int i = 0; i < (int)(sizeof(g_options) / sizeof(g_options[0])); ++i) {
    Option& o = g_options[i];
    if (strcmp(name, o.name) != 0) continue;
    if (i == kOptDenseMinM ? value < 1 : (value != 0 && value != 1)) return DSV41_EINVAL;
    o.value.store(value, std::memory_order_relaxed);
    o.set.store(true, std::memory_order_release);
    return DSV41_OK;
  }
  return DSV41_EINVAL;
}
int dsv41_arch(void) { return 100; }

int64_t dsv41_gemv_fp8_scratch_bytes(const Dsv41GemvArgs* a) {
  if (!gemv_entry_args_ok(a)) return DSV41_EINVAL;
  return gemv_entry_partials_bytes(gemv_entry_plan(a, sm_count()));
}

int dsv41_gemv_fp8(const Dsv41GemvArgs* a, void* stream) {
  if (!gemv_entry_args_ok(a)) return DSV41_EINVAL;
  const GemvArgs g = gemv_entry_plan(a, sm_count());
  const int64_t need = gemv_entry_partials_bytes(g);
  if (need > 0 && (!a->scratch || a->scratch_bytes < need)) return DSV41_ESCRATCH;
  if (gemv_entry_launch(g, ptr<float>(a->y), ptr<float>(a->scratch), reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return launch_status();
  return launch_status();
}

static bool index_query_ok(const Dsv41IndexQueryArgs* a) {
  return a && a->M >= 1 && a->M <= 48 && a->heads >= 16 && a->heads <= 64 && a->heads % 16 == 0 && a->dim == 128 &&
         a->rope >= 2 && a->rope % 2 == 0 && a->rope <= a->dim && a->hidden >= 256 && a->hidden % 256 == 0 &&
         a->hidden <= 16384 && a->q && a->cos_sin && a->rope_rows >= 1 && a->pos && a->x && a->wp && a->q_out &&
         a->qscale && a->w_out && a->q % 16 == 0 && a->x % 16 == 0 && a->wp % 16 == 0 && a->q_out % 16 == 0;
}

int64_t dsv41_index_query_scratch_bytes(const Dsv41IndexQueryArgs* a) {
  if (!index_query_ok(a)) return DSV41_EINVAL;
  return a->M * a->heads * 4;
}

int dsv41_index_query(const Dsv41IndexQueryArgs* a, void* stream) {
  if (!index_query_ok(a)) return DSV41_EINVAL;
  if (!a->scratch || a->scratch_bytes < a->M * a->heads * 4 || a->scratch % 16) return DSV41_ESCRATCH;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int M = (int)a->M, heads = (int)a->heads, hidden = (int)a->hidden;
  float* hw = ptr<float>(a->scratch);
  // the head weights' dots: the router's exact fixed-order fp64 sums, heads as its experts
  const int smem = 16 * hidden <= 200 * 1024 ? 16 * hidden : 0;
  RouterArgs ra = {M, heads, hidden, ptr<const __nv_bfloat16>(a->x), ptr<const __nv_bfloat16>(a->wp), hw, smem > 0};
  DSV41_TRY(launch(router_kernel<8>, dim3(cdiv(heads, 8), cdiv(M, 8)), dim3(256), smem, st, ra));
  float scale;
  const uint32_t sb = (uint32_t)a->weight_scale_f32;
  memcpy(&scale, &sb, 4);
  IndexQueryArgs q = {M, heads, (int)a->dim, (int)a->rope, ptr<const __nv_bfloat16>(a->q), ptr<const float>(a->cos_sin),
                      a->rope_rows, ptr<const int64_t>(a->pos), hw, scale, ptr<uint8_t>(a->q_out),
                      ptr<uint8_t>(a->qscale), ptr<__nv_bfloat16>(a->w_out)};
  DSV41_TRY(launch(index_query_kernel, dim3(M), dim3(256), 0, st, q));
  return launch_status();
}

int dsv41_walk_plan(const Dsv41WalkPlanArgs* a, void* stream) {
  if (!a || a->rows < 1 || a->rows > 48 || a->ctas < 1 || a->ctas > 4096 || !a->bounds || !a->owners ||
      !a->plan)
    return DSV41_EINVAL;
  WalkPlanArgs w = {(int)a->rows, (int)a->ctas, (int)a->topk, ptr<const int32_t>(a->bounds),
                    ptr<const int32_t>(a->owners), ptr<int32_t>(a->plan)};
  DSV41_TRY(launch(walk_plan_kernel, dim3(1), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), w));
  return launch_status();
}

int dsv41_k2i(const Dsv41K2iArgs* a, void* stream) {
  if (!a || a->rows < 1 || a->rows > 48 || a->heads < 16 || a->heads > 64 || a->heads % 16 || !a->q ||
      !a->qscale || !a->w || !a->payload || !a->kscale || !a->itab || !a->owners || !a->bounds ||
      !a->logits || a->ctas < 1 || (!a->reindex && !a->plan) ||
      !(a->entry_rows == 64 || a->entry_rows == 8) || a->lstride < 1 || a->payload % 16)
    return DSV41_EINVAL;
  K2iArgs k = {};
  k.rows = (int)a->rows; k.heads = (int)a->heads;
  k.q = ptr<const uint8_t>(a->q); k.qscale = ptr<const uint8_t>(a->qscale);
  k.w = ptr<const __nv_bfloat16>(a->w); k.payload = ptr<const uint8_t>(a->payload);
  k.kscale = ptr<const uint8_t>(a->kscale); k.plan = ptr<const int32_t>(a->plan);
  k.itab = ptr<const int32_t>(a->itab); k.itab_stride = (int)a->itab_stride; k.itab_len = (int)a->itab_len;
  k.entry_rows = (int)a->entry_rows; k.owners = ptr<const int32_t>(a->owners);
  k.bounds = ptr<const int32_t>(a->bounds); k.logits = ptr<float>(a->logits); k.lstride = (int)a->lstride;
  k.reindex = (int)a->reindex; k.reindex_chunks = (int)a->reindex_chunks;
  // the tensor-core scorer reads queries as 16-byte vectors and copies code bytes in bulk
  if (use_k2i_tc() && a->q % 16 == 0 && a->kscale % 16 == 0)
    DSV41_TRY(launch(k2i_tc_kernel, dim3((int)a->ctas), dim3(kKtThreads), KtSmem::kBytes,
                     reinterpret_cast<cudaStream_t>(stream), k));
  else
    DSV41_TRY(launch(k2i_score_kernel, dim3((int)a->ctas), dim3(256), k2i_smem_bytes(k.heads),
                     reinterpret_cast<cudaStream_t>(stream), k));
  return launch_status();
}

int dsv41_topk(const Dsv41TopkArgs* a, void* stream) {
  if (!a || a->rows < 1 || a->k < 1 || a->k > 65536 || !a->vals || !a->n || !a->out || a->group < 1 ||
      (a->page_out && (!a->table || !a->owners || a->page < 1)))
    return DSV41_EINVAL;
  // a row has at most vstride values, hence at most ceil(vstride / group) candidates (rounded up
  // to a multiple of 4: the kernel reads the staged keys four at a time)
  const int cands = ((int)a->vstride + (int)a->group - 1) / (int)a->group;
  if (use_topk_cluster() && cands >= kTopkClMinCands) {
    // a CTA stages its eighth of a row (rows past 8 x 8192 candidates read theirs from global memory)
    const int cap_cl = std::min(8192, (cands + kTopkCl - 1) / kTopkCl + 127) / 128 * 128;
    TopkArgs t = {(int)a->rows, (int)a->k, ptr<const float>(a->vals), (int)a->vstride, ptr<const int32_t>(a->n),
                  (int)a->group, ptr<int32_t>(a->out), ptr<int32_t>(a->page_out), ptr<const int32_t>(a->table),
                  (int)a->table_stride, (int)a->page, ptr<const int32_t>(a->owners), cap_cl};
    DSV41_TRY(launch(topk_cluster_kernel, dim3((int)a->rows * kTopkCl), dim3(kTopkClThreads),
                     cap_cl * 4 + kTopkBins * 4, reinterpret_cast<cudaStream_t>(stream), t, kTopkCl));
    return launch_status();
  }
  const int cap = (std::min<int>(40960, cands) + 3) / 4 * 4;
  TopkArgs t = {(int)a->rows, (int)a->k, ptr<const float>(a->vals), (int)a->vstride, ptr<const int32_t>(a->n),
                (int)a->group, ptr<int32_t>(a->out), ptr<int32_t>(a->page_out), ptr<const int32_t>(a->table),
                (int)a->table_stride, (int)a->page, ptr<const int32_t>(a->owners), cap};
  DSV41_TRY(launch(topk_kernel, dim3((int)a->rows), dim3(1024), cap * 4 + kTopkBins * 4,
                   reinterpret_cast<cudaStream_t>(stream), t));
  return launch_status();
}

int dsv41_reindex_table(const Dsv41ReindexArgs* a, void* stream) {
  if (!a || a->rows < 1 || a->topk_blocks < 1 || a->units < 1 || a->block_rows < 1 || !a->ids ||
      !a->page_table || !a->owners || !a->visible || !a->ids_out || !a->table || !a->context)
    return DSV41_EINVAL;
  ReindexArgs r = {(int)a->rows, (int)a->topk_blocks, (int)a->units, (int)a->block_rows,
                   ptr<const int32_t>(a->ids), (int)a->ids_stride, ptr<const int32_t>(a->page_table),
                   (int)a->page_stride, ptr<const int32_t>(a->owners), ptr<const int32_t>(a->visible),
                   ptr<int32_t>(a->ids_out), ptr<int32_t>(a->table), ptr<int32_t>(a->context)};
  DSV41_TRY(launch(reindex_kernel, dim3((int)a->rows), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream), r));
  return launch_status();
}

int dsv41_map_compact(const Dsv41MapCompactArgs* a, void* stream) {
  if (!a || a->rows < 1 || a->topk < 1 || !a->compact || !a->ids || !a->page_table || !a->owners ||
      !a->raw_out || !a->page_out || a->block_rows < 1 || a->page < 1)
    return DSV41_EINVAL;
  MapCompactArgs m = {(int)a->rows, (int)a->topk, (int)a->block_rows, (int)a->page,
                      ptr<const int32_t>(a->compact), ptr<const int32_t>(a->ids), (int)a->ids_stride,
                      ptr<const int32_t>(a->page_table), (int)a->table_stride, ptr<const int32_t>(a->owners),
                      ptr<int32_t>(a->raw_out), ptr<int32_t>(a->page_out), (int)a->out_stride};
  DSV41_TRY(launch(map_compact_kernel, dim3((int)a->rows), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), m));
  return launch_status();
}

int64_t dsv41_peer_region_bytes(int64_t tp, int64_t cap) {
  if (tp < 1 || tp > kPeerMaxTp || cap < 8 || cap % 8) return DSV41_EINVAL;
  return peer_region_bytes((int)tp, cap);
}

int dsv41_peer_alloc(int64_t bytes, int64_t* region, uint8_t* handle) {
  if (bytes < kPeerDataOff || !region || !handle) return DSV41_EINVAL;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return launch_status();
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return launch_status();
  }
  static_assert(sizeof(h) == DSV41_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *region = reinterpret_cast<int64_t>(p);
  return DSV41_OK;
}

int dsv41_peer_open(const uint8_t* handle, int64_t* region) {
  if (!handle || !region) return DSV41_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return launch_status();
  *region = reinterpret_cast<int64_t>(p);
  return DSV41_OK;
}

int dsv41_peer_close(int64_t region) {
  if (!region) return DSV41_EINVAL;
  if (cudaIpcCloseMemHandle(reinterpret_cast<void*>(region)) != cudaSuccess) return launch_status();
  return DSV41_OK;
}

int dsv41_peer_free(int64_t region) {
  if (!region) return DSV41_EINVAL;
  if (cudaFree(reinterpret_cast<void*>(region)) != cudaSuccess) return launch_status();
  return DSV41_OK;
}

int dsv41_peer_status(int64_t region, int32_t* words) {
  if (!region || !words) return DSV41_EINVAL;
  if (cudaMemcpy(words, reinterpret_cast<const void*>(region), DSV41_GUARD_WORDS * 4, cudaMemcpyDeviceToHost) !=
      cudaSuccess)
    return launch_status();
  return (words[kErrDeadline] | words[kErrPeer] | words[kErrFault]) ? DSV41_EDEVICE : DSV41_OK;
}

int dsv41_allreduce(const Dsv41AllReduceArgs* a, void* stream) {
  if (!a || a->tp < 1 || a->tp > kPeerMaxTp || a->rank < 0 || a->rank >= a->tp || !a->peers || !a->src ||
      !a->dst || a->n < 8 || a->n % 8 || a->cap < a->n || a->cap % 8 || a->n > (1LL << 30) || a->src % 16 ||
      a->dst % 16)
    return DSV41_EINVAL;
  DSV41_TRY(allreduce_go((int)a->n, (int)a->tp, (int)a->rank, a->peers, a->cap, ptr<const void>(a->src),
                         ptr<void>(a->dst), a->deadline_ns, (int)a->site, (int)a->skip_push,
                         reinterpret_cast<cudaStream_t>(stream)));
  return launch_status();
}

int dsv41_allreduce_ll(const Dsv41AllReduceArgs* a, void* stream) {
  if (!a || a->tp < 1 || a->tp > kPeerMaxTp || a->rank < 0 || a->rank >= a->tp || !a->peers || !a->src ||
      !a->dst || a->n < 8 || a->n % 8 || a->cap < a->n || a->cap % 8 || a->n > (1LL << 30) || a->src % 16 ||
      a->dst % 16)
    return DSV41_EINVAL;
  PeerLL x = {};
  x.peers = ptr<const int64_t>(a->peers); x.tp = (int)a->tp; x.rank = (int)a->rank; x.site = (int)a->site;
  x.skip = (int)a->skip_push; x.cap = a->cap; x.deadline_ns = deadline_or_default(a->deadline_ns);
  x.reduced = ptr<__nv_bfloat16>(a->dst);
  const int grid = std::min(grid_for(a->n / 8, 256), 4 * sm_count());
  DSV41_TRY(launch_n(allreduce_ll_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), x,
                     ptr<const __nv_bfloat16>(a->src), (int)a->n));
  return launch_status();
}

int dsv41_rank_sum(const Dsv41RankSumArgs* a, void* stream) {
  if (!a || a->n < 1 || a->tp < 1 || a->tp > kPeerMaxTp || !a->parts || !a->out || a->n > (1LL << 30))
    return DSV41_EINVAL;
  RankSumArgs r = {(int)a->n, (int)a->tp, ptr<const __nv_bfloat16>(a->parts), ptr<__nv_bfloat16>(a->out)};
  DSV41_TRY(launch(rank_sum_kernel, dim3(grid_for(a->n, 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                   r));
  return launch_status();
}

int dsv41_lmhead_argmax(const Dsv41LmHeadArgs* a, void* stream) {
  if (!a || a->M < 1 || a->M > 48 || a->V < 1 || a->V > (1LL << 30) || a->K < kLmChunk || a->K % kLmChunk ||
      a->vbase < 0 || a->vbase + a->V > (1LL << 31) || !a->w || !a->x || !a->best || a->w % 16 || a->x % 16)
    return DSV41_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  LmHeadArgs l = {ptr<const __nv_bfloat16>(a->w), ptr<const __nv_bfloat16>(a->x), ptr<float>(a->logits),
                  ptr<long long>(a->best), (int)a->M, (int)a->V, (int)a->K, (int)a->vbase};
  if (a->init) DSV41_TRY(launch(argmax_init_kernel, dim3(1), dim3(64), 0, st, l));
  const dim3 grid(cdiv(l.V, kLmRows));
  const int nt = cdiv(l.M, 8);
  const int smem = 2 * 8 * nt * kLmLd * 2;
  switch (nt) {
    case 1: DSV41_TRY(launch(lmhead_kernel<1>, grid, dim3(256), smem, st, l)); break;
    case 2: DSV41_TRY(launch(lmhead_kernel<2>, grid, dim3(256), smem, st, l)); break;
    case 3: DSV41_TRY(launch(lmhead_kernel<3>, grid, dim3(256), smem, st, l)); break;
    case 4: DSV41_TRY(launch(lmhead_kernel<4>, grid, dim3(256), smem, st, l)); break;
    case 5: DSV41_TRY(launch(lmhead_kernel<5>, grid, dim3(256), smem, st, l)); break;
    default: DSV41_TRY(launch(lmhead_kernel<6>, grid, dim3(256), smem, st, l)); break;
  }
  return launch_status();
}

int dsv41_argmax_decode(const Dsv41ArgmaxArgs* a, void* stream) {
  if (!a || a->M < 1 || a->M > 4096 || !a->best ||
      (a->draft && (a->per_req < 1 || a->M % a->per_req || !a->accept || !a->next_tok)))
    return DSV41_EINVAL;
  ArgmaxArgs d = {ptr<const long long>(a->best), (int)a->M, ptr<int32_t>(a->ids), ptr<float>(a->vals),
                  ptr<const int32_t>(a->draft), (int)a->per_req, ptr<int32_t>(a->accept), ptr<int32_t>(a->next_tok)};
  DSV41_TRY(launch(argmax_decode_kernel, dim3(1), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), d));
  return launch_status();
}

int dsv41_relayout_mxfp4(const Dsv41RelayoutArgs* a, void* stream) {
  if (!a || !a->src || !a->src_codes || !a->dst || !a->dst_codes || a->E < 1 || a->N % 16 ||
      a->K % 128 || a->N < 16 || a->src % 16 || a->dst % 16 || a->src_codes % 4 || a->dst_codes % 4)
    return DSV41_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  relayout_mxfp4_kernel<<<4 * 148 * 4, 256, 0, st>>>(ptr<const uint8_t>(a->src), ptr<const uint8_t>(a->src_codes),
                                                     ptr<uint8_t>(a->dst), ptr<uint8_t>(a->dst_codes), a->E,
                                                     (int)a->N, (int)a->K);
  return launch_status();
}

int64_t dsv41_k1_scratch_bytes(const Dsv41K1Args* a) {
  int64_t need = 0;
  const int rc = k1_run(a, nullptr, false, &need);
  return rc < 0 ? rc : need;
}

int dsv41_k1(const Dsv41K1Args* a, void* stream) {
  int64_t need = 0;
  return k1_run(a, reinterpret_cast<cudaStream_t>(stream), true, &need);
}

int64_t dsv41_k2_scratch_bytes(const Dsv41K2Args* a) {
  int64_t need = 0;
  const int rc = k2_run(a, nullptr, false, &need);
  return rc < 0 ? rc : need;
}

int dsv41_k2(const Dsv41K2Args* a, void* stream) {
  int64_t need = 0;
  return k2_run(a, reinterpret_cast<cudaStream_t>(stream), true, &need);
}

}  // extern "C"
