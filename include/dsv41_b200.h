/* C ABI of the DeepSeek-V4.1 decode / verify monokernel backend for B200 (sm_100a).
 *
 * Every entry point takes a POD argument struct whose fields are all 64-bit (device
 * pointers as int64, sizes and flags as int64), plus a cudaStream_t passed as void*, and
 * returns 0 or a negative DSV41_E* status. Nothing throws across the boundary; nothing but
 * dsv41_peer_alloc (the TP exchange regions) allocates device memory: scratch is
 * caller-owned, sized by the *_scratch_bytes queries.
 * Launches go on the given stream only, so every call is CUDA-graph capturable.
 *
 * The reference (omirosh/sgl-amd-mono) binds the same launches through its FlyDSL JIT
 * entry points, which take raw int64 device pointers and a stream; each declaration below
 * names the reference interface it replaces (file:line in the reference).
 */
#ifndef DSV41_B200_H
#define DSV41_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV41_OK 0
#define DSV41_EINVAL (-1)   /* an argument is out of range or misaligned */
#define DSV41_ELAUNCH (-2)  /* a CUDA launch failed (cudaGetLastError) */
#define DSV41_ESCRATCH (-3) /* the caller's scratch is smaller than required */
#define DSV41_EDEVICE (-4)  /* a device-side guard fired (deadline, peer failure) */

/* Library version and the compute capability it was built for (100 for sm_100a). */
int dsv41_version(void);
int dsv41_arch(void);

/* Tuning switches of the launch sequences, for comparisons and tests (each also read once
 * from its environment variable): "attn_tc" 1/0 (DSV41_ATTN=mma: 0) the tcgen05 attention core
 * or the mma.sync one; "attn_pair" 1/0 (DSV41_ATTN_PAIR) a row's two 32-head tiles as one CTA
 * pair sharing key tiles, or two lone CTAs; "dense_min_m" >= 1 (DSV41_DENSE_MIN_M, 16) the
 * smallest M whose MXFP8-input projections run on the tcgen05 dense kernel; "pdl" 1/0
 * (DSV41_PDL) programmatic dependent launch; "fused_allreduce" 1/0 (DSV41_FUSED_AR) K2's two
 * TP all-reduces fused into the kernels producing their partials, or the standalone exchange
 * kernel after each; "k1_persistent" 0/1 (DSV41_K1_PERSISTENT) K1 as one persistent launch
 * when M is below "dense_min_m" (its six stages separated by grid barriers), or its launch
 * sequence (default); "attn_bulk" 0/1 (DSV41_ATTN_BULK) the tcgen05 attention's producer
 * gathering each key tile's records into registers (default; "attn_pair" then chooses pair or
 * lone CTAs), or staging them in shared memory by bulk copies (lone CTAs); "attn_wide" 1/0
 * (DSV41_ATTN_WIDE) a row's 64 heads in one tcgen05 attention CTA (default when a rank holds 64
 * heads of 512 + 64 dims), or the 32-head kernels above; "k2i_tc" 1/0 (DSV41_K2I_TC) K2i's scorer
 * on tcgen05 block-scaled MMAs (default; needs q and kscale 16-byte aligned) or on mma.sync with
 * the fp64 chunk epilogue, the same logits either way; "topk_cluster" 1/0 (DSV41_TOPK_CLUSTER)
 * dsv41_topk rows of at least 2048 candidates over an 8-CTA cluster each (default) or one CTA a
 * row, the same selection either way; "row_attn" 1/0 (DSV41_ROW_ATTN) at TP > 1 each rank attends
 * ceil(M / tp) rows for all heads (default; needs sink_all, M >= tp and the peer capacity) or its
 * own heads for every row. Takes effect at the
 * next launch; DSV41_EINVAL for an unknown name or value. No counterpart in the reference (its variants are build keys). */
int dsv41_set_option(const char* name, int64_t value);

/* ---------------------------------------------------------------- FP8 GEMV
 * y[m][n] = sum_k x[m][k] * dequant(W)[n][k] in fp32: W e4m3 [N, K] row-major with one
 * E8M0 code per 128 x 128 block, x bf16 [M, x_ld]. Rows n use x columns
 * (n / x_group_rows) * K .. + K (a grouped projection, wo_a); x_group_rows = 0: N.
 * Replaces the GEMV tiles of attention/gemv.py:141-194 (chain_mfmas), stages/gemv.py:182-214. */
typedef struct {
  int64_t w, codes, x, y;             /* device pointers */
  int64_t M, N, K, x_ld, x_group_rows;
  int64_t scratch, scratch_bytes;     /* caller-owned device scratch */
} Dsv41GemvArgs;
int64_t dsv41_gemv_fp8_scratch_bytes(const Dsv41GemvArgs* a);
int dsv41_gemv_fp8(const Dsv41GemvArgs* a, void* stream);

/* The same GEMV for callers that cannot allocate device memory (a server whose KV-cache pool
 * took the spare HBM at start-up, a foreign runtime without a device allocator): the K-slice
 * partials go to a library-owned device array of DSV41_NOALLOC_SCRATCH_BYTES (held by every
 * GPU that loads the library until exit) instead of caller scratch; scratch and
 * scratch_bytes are ignored. A shape whose partials exceed the array returns DSV41_ESCRATCH.
 * The first call in each CUDA context (each device's primary context, a driver-API caller's
 * own context, a new primary context after cudaDeviceReset) resolves the array's address in
 * that context, so make the first call in a context before any stream capture in it. All
 * calls share the array: calls that overlap on the GPU race. No counterpart in the reference
 * (its launches take caller buffers only). */
#define DSV41_NOALLOC_SCRATCH_BYTES (4 << 20)
int dsv41_gemv_fp8_noalloc(const Dsv41GemvArgs* a, void* stream);

/* ---------------------------------------------------------------- MXFP4 expert relayout
 * One-time copy of routed-expert weights from the checkpoint layout -- w [E, N, K/2] E2M1
 * (even K in the low nibble) with E8M0 codes [E, N, K/32] -- into the tensor-core tiles the
 * expert kernel streams: dst [E][ceil(N/256)][K/128][256 rows][64 B] (rows past N zero),
 * dst_codes [E][ceil(N/256)][K/128][1024 B]: two 512-byte atoms (rows 0..127, 128..255), row r's
 * code of K block b at (r / 128) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + b. dst holds
 * E * ceil(N/256) * 256 * K/2 bytes, dst_codes E * ceil(N/256) * 256 * K/32. N % 16 == 0,
 * K % 128 == 0; src, dst 16-byte aligned (dst 32-byte aligned for the kernels' tensor maps),
 * codes 4-byte aligned.
 * Replaces the reader of aiter's shuffle_weight / shuffle_scale layout (common/mx.py:35-50,
 * stages/moe.py:567-607); the runner logs the copy as the reference logs its copies
 * (deepseek_v41/spec.py:34-41). */
typedef struct {
  int64_t src, src_codes, dst, dst_codes;
  int64_t E, N, K;
} Dsv41RelayoutArgs;
int dsv41_relayout_mxfp4(const Dsv41RelayoutArgs* a, void* stream);

/* ---------------------------------------------------------------- K1
 * The attention seam and front of one layer (gfx950/layer.py:189-468, launch args
 * layer.py:223-263; host runner.py:512-622): mHC seam, wqkv_a GEMV, q_norm -> MXFP8 q,
 * kv_norm + RoPE -> the FP8 KV record at the row's slot, the key table for K2, wq_b GEMV +
 * RoPE -> q. Shapes: hidden % 256 == 0; q_lora in {256, 512, 1024}; nope % 64 == 0,
 * rope == 64; heads * (nope + rope) % 16 == 0. Inputs and outputs are row-major. */
typedef struct {
  int64_t M, hidden, q_lora, nope, rope, heads, swa_width, topk_width;
  int64_t fold, first, index, build_kt;
  /* seam */
  int64_t res_in, x_in, post_in, comb_in, pre_in, hc_fn, hc_scale, hc_base, norm_w;
  int64_t res_out, post_out, comb_out, pre_out, normed, x8, x8s;
  /* projections, norms, positions */
  int64_t wqkv, wqkv_codes, q_norm, kv_norm, cos_sin, pos, rope_rows;
  /* KV store */
  int64_t slot, cache, page_stride, blk;
  /* key table */
  int64_t swa_idx, swa_lens, topk_idx, topk_lens, kt, klen;
  /* wq_b and outputs */
  int64_t wqb, wqb_codes, q, qr, qx8, qx8s, qkv_out;
  /* optional host array of DSV41_K1_STAGES + 1 cudaEvent_t recorded at stage boundaries
   * (seam, wqkv_a, q/kv, wq_b) for profiling; 0 = none */
  int64_t events;
  int64_t scratch, scratch_bytes;
} Dsv41K1Args;
#define DSV41_K1_STAGES 4
int64_t dsv41_k1_scratch_bytes(const Dsv41K1Args* a);
int dsv41_k1(const Dsv41K1Args* a, void* stream);

/* ---------------------------------------------------------------- K2
 * The attention core, wo_a, wo_b, the attention all-reduce, the FFN seam, the router and
 * routing, the shared and routed experts and the MoE all-reduce of one layer
 * (gfx950/layer.py:773-1072, launch args layer.py:802-854; host runner.py:624-728).
 * route_softmax = 1: softmax top-k routing; 0: sqrtsoftplus + bias, renormalized x 1.5.
 * heads, o_groups, inter and shared_inter are this rank's (local) widths.
 * tp > 1: peers is a device array of tp int64 -- each rank's exchange region
 * (dsv41_peer_alloc / dsv41_peer_open) as mapped in this process -- whose data slots hold
 * peer_cap bf16 elements (>= M * hidden); both all-reduces run in-kernel through it, with
 * waits that give up after deadline_ns (0: 5 s) and leave the failure in the guard words
 * (dsv41_peer_status). phase 0: the whole layer; phase 1: stop at this rank's attention
 * partial (attn_part); phase 2: start from the reduced attention output in attn and stop at
 * this rank's MoE partial (moe_part) -- the caller reduces in between (the NCCL variant:
 * an all-gather, then dsv41_rank_sum). inject = s (1 attention, 2 MoE): skip this rank's
 * push at site s (the reference's SGLANG_AMD_MONO_FAULT_INJECT test hook, guard.py:80-100),
 * so the peers' waits run out. */
typedef struct {
  int64_t M, hidden, nope, rope, heads, o_groups, o_rank;
  int64_t experts, topk, inter, shared_inter, route_softmax, tp, rank, keys_ld;
  /* attention */
  int64_t q, kt, klen, swa, swa_stride, swa_blk, comp, comp_stride, comp_blk, sink, cos_sin, pos, rope_rows;
  int64_t woa, woa_codes, wob, wob_codes;
  /* FFN seam */
  int64_t res_in, post_in, comb_in, pre_in, hc_fn, hc_scale, hc_base, norm_w;
  int64_t res_out, post_out, comb_out, pre_out, normed;
  /* MoE */
  int64_t gate_w, bias, w13, w13_codes, w2, w2_codes, sgu, sgu_codes, sw2, sw2_codes;
  /* outputs (xo, x8b, x8bs, attn_part, attn, logits: optional inspection copies) */
  int64_t out, ids, wts, xo, x8b, x8bs, attn_part, attn, logits, moe_part;
  /* tensor parallelism (sink_all: the sinks of every rank's heads in rank order, float [tp * heads],
   * or 0; with it, phase 0, the in-kernel exchanges, M >= tp and peer_cap >= ceil(M / tp) * heads *
   * (nope + rope), each rank runs the attention of its ceil(M / tp) rows for all heads -- the rows'
   * queries and outputs exchanged through the peer region -- instead of its heads for all rows) */
  int64_t peers, peer_cap, deadline_ns, phase, inject, sink_all;
  /* optional host array of DSV41_K2_STAGES + 1 cudaEvent_t recorded at stage boundaries
   * (attention, wo_a + wo_b, all-reduce + FFN seam, router + routing, shared expert,
   * routed experts, combine + all-reduce); 0 = none */
  int64_t events;
  int64_t scratch, scratch_bytes;
} Dsv41K2Args;
#define DSV41_K2_STAGES 7

/* ---------------------------------------------------------------- K2i and the index selection
 * The FULL walk plan from device bounds: pieces of <= 6 rows of one owner (page-table row),
 * [ctas, 4] int32 (lead, span, ch0, ch1). Replaces walk_plan.fill_walk_plan_device
 * (gfx950/indexer/walk_plan.py:32-87; host twin index_plan.py:42-82). */
typedef struct {
  int64_t rows, ctas, topk, bounds, owners, plan;
} Dsv41WalkPlanArgs;
int dsv41_walk_plan(const Dsv41WalkPlanArgs* a, void* stream);

/* K2i: index logits [rows, lstride] f32 of the FP4 query (q [rows, heads, 64] E2M1 pairs,
 * qscale [rows, 1, 4, 16, 4], w [rows, heads] bf16) against the FP4 index plane (payload
 * [pages, 1, 4, 64, 16], kscale [pages, 1, 4, 64]) through a page table of entry_rows keys an
 * entry (64: plane pages; 8: a REINDEX table's blocks). FULL (reindex 0) follows the walk
 * plan (grid = ctas); REINDEX scores reindex_chunks 128-column chunks a row (grid = ctas).
 * heads % 16 == 0, heads <= 64. Replaces build_k2i's launch (gfx950/indexer/k2i.py:39-85,
 * called from indexer/runner.py:228-251). */
typedef struct {
  int64_t rows, heads, q, qscale, w, payload, kscale;
  int64_t plan, ctas, itab, itab_stride, itab_len, entry_rows, owners, bounds;
  int64_t logits, lstride, reindex, reindex_chunks;
} Dsv41K2iArgs;
int dsv41_k2i(const Dsv41K2iArgs* a, void* stream);

/* The indexer's FP4 query of decode rows, K2i's q / qscale / w inputs, from wq_b's output q
 * [M, heads, 128] bf16, the layer's RoPE table cos_sin [rope_rows, rope] fp32 (rope / 2 cos, then
 * rope / 2 sin) at positions pos [M] int64, the normed rows x [M, hidden] bf16 and the head weight
 * projection wp [heads, hidden] bf16 with its scale (weight_scale_f32: the fp32 bit pattern):
 * head weights w_out [M, heads] bf16 = bf16(fp32(x . wp[h]) * scale), the dot summed as the
 * router's logits (exact products, fp64 in a fixed order); GPT-J RoPE on each head's last rope
 * dims (separate fp32 products); MXFP4 per 32 dims (E8M0 = the ceiling power of two of
 * amax / 6, E2M1 round to nearest even) into q_out [M, heads, 64] and qscale [M, 1, 4, 16, 4]
 * (head h's chunk c at [c, h % 16, h / 16]). heads 16..64 in 16s, dim 128; scratch >= M * heads
 * * 4 bytes. Replaces SGLang's index_q_rope_pack_weights with its split-K head-weight GEMV
 * (called at deepseek_v41/spec.py:744-763 of the reference). */
typedef struct {
  int64_t M, heads, dim, rope, hidden;
  int64_t q, cos_sin, rope_rows, pos, x, wp, weight_scale_f32;
  int64_t q_out, qscale, w_out;
  int64_t scratch, scratch_bytes;
} Dsv41IndexQueryArgs;
int64_t dsv41_index_query_scratch_bytes(const Dsv41IndexQueryArgs* a);
int dsv41_index_query(const Dsv41IndexQueryArgs* a, void* stream);

/* Top-k of each row's first n[t] values (group > 1: of the maxima of groups of `group`
 * values -- candidate blocks), ties to the lower position, written in ascending position
 * order, -1 padded; optional paged twin page_out = table[owners[t]][pos / page] * page +
 * pos % page. Replaces SGLang's topk_transform_paged(_hip) and select_candidate_blocks_hip
 * (called at indexer/runner.py:158-190, deepseek_v41/spec.py:697-706). */
typedef struct {
  int64_t rows, k, vals, vstride, n, group, out, page_out, table, table_stride, page, owners;
} Dsv41TopkArgs;
int dsv41_topk(const Dsv41TopkArgs* a, void* stream);

/* A REINDEX layer's candidate table (indexer/candidate_table.py:19-99). */
typedef struct {
  int64_t rows, topk_blocks, units, block_rows, ids, ids_stride, page_table, page_stride;
  int64_t owners, visible, ids_out, table, context;
} Dsv41ReindexArgs;
int dsv41_reindex_table(const Dsv41ReindexArgs* a, void* stream);

/* A REINDEX layer's compact selection mapped back to positions and pool slots
 * (indexer/candidate_table.py:103-163). */
typedef struct {
  int64_t rows, topk, block_rows, page, compact, ids, ids_stride, page_table, table_stride;
  int64_t owners, raw_out, page_out, out_stride;
} Dsv41MapCompactArgs;
int dsv41_map_compact(const Dsv41MapCompactArgs* a, void* stream);

/* ---------------------------------------------------------------- TP exchange regions
 * One region a rank (guard words, failure flags, per-CTA arrival flags, two parities of
 * tp data slots of cap bf16 elements, then two parities of tp LL slots of cap / 2 8-byte
 * words); replaces common/peer.py:114-156 (PeerBuffer) and the
 * guard block of common/guard.py:20-40. Construction is collective in the caller: every
 * rank allocates its region, the 64-byte IPC handles are exchanged, and every rank opens the
 * others'. dsv41_peer_region_bytes: the size of a region for tp ranks and cap elements. */
#define DSV41_IPC_HANDLE_BYTES 64
#define DSV41_PEER_MAX_TP 8
#define DSV41_GUARD_WORDS 8
int64_t dsv41_peer_region_bytes(int64_t tp, int64_t cap);
/* cudaMalloc + zero fill + cudaIpcGetMemHandle on the current device: *region and the
 * handle's DSV41_IPC_HANDLE_BYTES bytes. */
int dsv41_peer_alloc(int64_t bytes, int64_t* region, uint8_t* handle);
/* Map another rank's region (cudaIpcOpenMemHandle, lazy peer access). */
int dsv41_peer_open(const uint8_t* handle, int64_t* region);
int dsv41_peer_close(int64_t region);
int dsv41_peer_free(int64_t region);
/* Synchronous read of a region's DSV41_GUARD_WORDS guard words (0 sequence, 1 CTAs done,
 * 3 deadline site, 4 peer failure seen, 5 fault injected); DSV41_EDEVICE when one of the
 * error words is set. */
int dsv41_peer_status(int64_t region, int32_t* words);

/* One in-kernel TP all-reduce (seam.py:391-408, moe.py:1247-1268): dst = bf16(rank-order
 * fp32 sum of every rank's src), n bf16 elements (a multiple of 8, <= cap). site: the
 * 1-based number a timed-out wait records; skip_push: the fault-injection hook. */
typedef struct {
  int64_t n, tp, rank, peers, cap, src, dst, deadline_ns, site, skip_push;
} Dsv41AllReduceArgs;
int dsv41_allreduce(const Dsv41AllReduceArgs* a, void* stream);

/* The same all-reduce as LL stores: every 8-byte word of the exchange carries an epoch beside two
 * bf16 values, so a reader polls the data itself -- no fence and arrival-flag round trip. The
 * exchange K2 fuses into its two producing kernels at tp > 1 (wo_b's epilogue, the MoE combine);
 * this entry runs it alone. Same arguments, result bits and guard words as dsv41_allreduce. The
 * reference's {value, tag} mailbox (common/sync.py:109-188) and its in-kernel pushes
 * (stages/seam.py:382-425, stages/moe.py:1156-1184, 1247-1268). */
int dsv41_allreduce_ll(const Dsv41AllReduceArgs* a, void* stream);

/* out = bf16(rank-order fp32 sum of parts[r]), parts [tp][n] bf16 contiguous: the reduction
 * step of the NCCL variant (all-gather, then this); bit-identical to dsv41_allreduce.
 * No counterpart kernel in the reference (its comparison path is NCCL's all_reduce). */
typedef struct {
  int64_t n, tp, parts, out;
} Dsv41RankSumArgs;
int dsv41_rank_sum(const Dsv41RankSumArgs* a, void* stream);

/* ---------------------------------------------------------------- LM head and greedy selection
 * logits = x . W^T for this rank's vocab rows W [V, K] bf16 (row-major, read in place; vocab
 * row i is global token vbase + i) and x [M, K] bf16, M <= 48, K a multiple of 128; the
 * argmax of each row (ties to the lower token id) as int64 keys in best [M] (init = 1:
 * reset first; 0: max-merge into best, e.g. a second vocab shard); optional fp32 logits
 * [M, V]. Vocab-parallel ranks max-reduce best (int64 MAX) and decode with
 * dsv41_argmax_decode. Replaces SGLang's logits processor + greedy sampling on the verify
 * path (reference spec.py:807-833, draft.py:173-195); the fused argmax has no kernel
 * counterpart in the reference. */
typedef struct {
  int64_t M, V, K, vbase, w, x, logits, best, init;
} Dsv41LmHeadArgs;
int dsv41_lmhead_argmax(const Dsv41LmHeadArgs* a, void* stream);

/* best [M] keys -> ids [M] int32 and vals [M] fp32 (each optional); with draft [M] int32 (the
 * verify rows' input tokens, per_req rows a request): accept [M / per_req] = the accepted
 * draft tokens of each request (draft[j + 1] accepted while it equals row j's argmax) and
 * next_tok [M / per_req] = the target's token after them. */
typedef struct {
  int64_t M, best, ids, vals, draft, per_req, accept, next_tok;
} Dsv41ArgmaxArgs;
int dsv41_argmax_decode(const Dsv41ArgmaxArgs* a, void* stream);

/* DSV41_EDEVICE once a kernel's bounded internal wait gave up in this process (the tcgen05
 * attention's and the routed experts' pipeline barriers; sticky), else 0. Synchronizes with the device. */
int dsv41_device_error(void);

/* Kernels this library has launched in this process (all entry points): for profiling. */
int64_t dsv41_launch_count(void);
int64_t dsv41_k2_scratch_bytes(const Dsv41K2Args* a);
int dsv41_k2(const Dsv41K2Args* a, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV41_B200_H */
