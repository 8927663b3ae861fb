"""ctypes mirrors of the C-ABI argument structs (``include/dsv41_b200.h``), field for field;
``tests/test_abi.py`` checks them against the header."""

from __future__ import annotations

from ...common.ext import struct

GemvArgs = struct("Dsv41GemvArgs", [
    "w", "codes", "x", "y", "M", "N", "K", "x_ld", "x_group_rows", "scratch", "scratch_bytes",
])

RelayoutArgs = struct("Dsv41RelayoutArgs", ["src", "src_codes", "dst", "dst_codes", "E", "N", "K"])

K1Args = struct("Dsv41K1Args", [
    "M", "hidden", "q_lora", "nope", "rope", "heads", "swa_width", "topk_width",
    "fold", "first", "index", "build_kt",
    "res_in", "x_in", "post_in", "comb_in", "pre_in", "hc_fn", "hc_scale", "hc_base", "norm_w",
    "res_out", "post_out", "comb_out", "pre_out", "normed", "x8", "x8s",
    "wqkv", "wqkv_codes", "q_norm", "kv_norm", "cos_sin", "pos", "rope_rows",
    "slot", "cache", "page_stride", "blk",
    "swa_idx", "swa_lens", "topk_idx", "topk_lens", "kt", "klen",
    "wqb", "wqb_codes", "q", "qr", "qx8", "qx8s", "qkv_out", "events",
    "scratch", "scratch_bytes",
])
K1_STAGES = ("seam", "wqkv_a", "q/kv", "wq_b")

K2Args = struct("Dsv41K2Args", [
    "M", "hidden", "nope", "rope", "heads", "o_groups", "o_rank",
    "experts", "topk", "inter", "shared_inter", "route_softmax", "tp", "rank", "keys_ld",
    "q", "kt", "klen", "swa", "swa_stride", "swa_blk", "comp", "comp_stride", "comp_blk", "sink",
    "cos_sin", "pos", "rope_rows",
    "woa", "woa_codes", "wob", "wob_codes",
    "res_in", "post_in", "comb_in", "pre_in", "hc_fn", "hc_scale", "hc_base", "norm_w",
    "res_out", "post_out", "comb_out", "pre_out", "normed",
    "gate_w", "bias", "w13", "w13_codes", "w2", "w2_codes", "sgu", "sgu_codes", "sw2", "sw2_codes",
    "out", "ids", "wts", "xo", "x8b", "x8bs", "attn_part", "attn", "logits", "moe_part",
    "peers", "peer_cap", "deadline_ns", "phase", "inject", "sink_all", "events",
    "scratch", "scratch_bytes",
])
K2_STAGES = ("attention", "wo_a+wo_b", "reduce+ffn seam", "router", "shared expert", "routed experts",
             "combine+reduce")

WalkPlanArgs = struct("Dsv41WalkPlanArgs", ["rows", "ctas", "topk", "bounds", "owners", "plan"])

K2iArgs = struct("Dsv41K2iArgs", [
    "rows", "heads", "q", "qscale", "w", "payload", "kscale",
    "plan", "ctas", "itab", "itab_stride", "itab_len", "entry_rows", "owners", "bounds",
    "logits", "lstride", "reindex", "reindex_chunks",
])

IndexQueryArgs = struct("Dsv41IndexQueryArgs", [
    "M", "heads", "dim", "rope", "hidden",
    "q", "cos_sin", "rope_rows", "pos", "x", "wp", "weight_scale_f32",
    "q_out", "qscale", "w_out",
    "scratch", "scratch_bytes",
])

TopkArgs = struct("Dsv41TopkArgs", [
    "rows", "k", "vals", "vstride", "n", "group", "out", "page_out", "table", "table_stride", "page",
    "owners",
])

ReindexArgs = struct("Dsv41ReindexArgs", [
    "rows", "topk_blocks", "units", "block_rows", "ids", "ids_stride", "page_table", "page_stride",
    "owners", "visible", "ids_out", "table", "context",
])

MapCompactArgs = struct("Dsv41MapCompactArgs", [
    "rows", "topk", "block_rows", "page", "compact", "ids", "ids_stride", "page_table", "table_stride",
    "owners", "raw_out", "page_out", "out_stride",
])

AllReduceArgs = struct("Dsv41AllReduceArgs", [
    "n", "tp", "rank", "peers", "cap", "src", "dst", "deadline_ns", "site", "skip_push",
])

RankSumArgs = struct("Dsv41RankSumArgs", ["n", "tp", "parts", "out"])

LmHeadArgs = struct("Dsv41LmHeadArgs", ["M", "V", "K", "vbase", "w", "x", "logits", "best", "init"])

ArgmaxArgs = struct("Dsv41ArgmaxArgs", ["M", "best", "ids", "vals", "draft", "per_req", "accept", "next_tok"])

STRUCTS = {
    "Dsv41GemvArgs": GemvArgs,
    "Dsv41RelayoutArgs": RelayoutArgs,
    "Dsv41K1Args": K1Args,
    "Dsv41K2Args": K2Args,
    "Dsv41WalkPlanArgs": WalkPlanArgs,
    "Dsv41K2iArgs": K2iArgs,
    "Dsv41IndexQueryArgs": IndexQueryArgs,
    "Dsv41TopkArgs": TopkArgs,
    "Dsv41ReindexArgs": ReindexArgs,
    "Dsv41MapCompactArgs": MapCompactArgs,
    "Dsv41AllReduceArgs": AllReduceArgs,
    "Dsv41RankSumArgs": RankSumArgs,
    "Dsv41LmHeadArgs": LmHeadArgs,
    "Dsv41ArgmaxArgs": ArgmaxArgs,
}
