"""DeepSeek-V4.1 on sm_100a: the monokernel spec and its forward (the reference's
``deepseek_v41/spec.py``, same interface, CUDA kernels).

SGLang's runtime switches the model's forward at attach: a routed decode or DSpark verify
step runs ``_Built.forward``, which takes and returns what ``DeepseekV4ForCausalLM.forward``
does: SGLang's input preparation, the embedding, every layer as K1 then K2 (the C-ABI
launches of ``sm100a``), the head's combine and norm, and SGLang's logits processor.

- K1 folds the previous layer's pending post into the residual (none is owed on the first
  layer's broadcast embedding or after an Engram write) and writes the step's SWA KV records
  and K2's key table; K2 runs the attention core over the window (and, at compress ratio 1
  or 2, the layer's sparse top-k of the compressed cache), wo_a, wo_b, both all-reduces, the
  FFN seam and the MoE.
- An index source: SGLang's compressor runs on K1's normed input between the launches, then
  K2i scores the index keys and its top-k writes SGLang's sparse indices of the layer's ratio
  (``_select``), as SGLang's decode indexer decides.

The kernels read SGLang's weights in place, except the copies logged in ``ctx.copies``: each
covered layer's FP8 shared expert (this rank's shard, kept at load), the E8M0 codes of the
power-of-two fp32 block scales, the f32 router bias and attention sinks, the RoPE table, and
the routed experts in the kernels' MXFP4 tensor-core tile order.
"""

from __future__ import annotations

import re

import torch
from sglang.srt.monokernels.spec import (
    DeviceLimits,
    Feature,
    MonoSpec,
    Numerics,
    NumericsKind,
    Requirements,
    StepMetadata,
)

from . import CANDIDATES, ENVELOPE, HF_CONFIG

MAX_ROWS = 48  # the rows a launch takes at most
ISA = "sm_100a"
RESIDENT_BLOCKS = 2 * 148  # DeviceLimits.resident_blocks: CTAs a launch keeps resident (two an SM)

_SHARED = ("gate_proj", "up_proj", "down_proj")
# the checkpoint's shared expert tensors, as the model loader names them
_CKPT_SHARED = re.compile(r"layers\.(?P<i>\d+)\.ffn\.shared_experts\.(?P<w>w[123])\.(?P<kind>weight|scale)")
_CKPT_PROJ = {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}

# The SGLang names this glue reads, by file under the sglang package (``f(p)``: a parameter,
# ``"x"``: a string literal); tests/test_spec.py pins them against this module's imports.
SGLANG_READS = {
    "srt/monokernels/spec.py": (
        "MONOKERNEL_API_VERSION", "DeviceLimits", "Feature", "MonoSpec", "Numerics", "NumericsKind",
        "Requirements", "StepMetadata", "tokens_per_request", "unread_metadata",
    ),
    "kernels/ops/layernorm/mhc.py": ("hc_broadcast", "hc_combine"),
    "srt/layers/attention/deepseek_v4_backend.py": (
        "forward_low_ratio_sources(layer)", "forward_low_ratio_sources(x)",
        "forward_low_ratio_sources(q_lora)", "forward_low_ratio_sources(positions)",
        "forward_low_ratio_sources(forward_batch)", "forward_low_ratio_sources(run_indexer)",
        "forward_metadata", "core_attn_metadata", "get_swa_out_cache_loc", "swa_page_indices",
        "swa_topk_lengths", "sparse_page_indices", "sparse_topk_lengths", "low_ratio_indexer_metadata",
        "sparse_raw_indices", "drop_folded_sparse_indices",
    ),
    "srt/layers/attention/dsv4/metadata.py": ("page_table", "compressed_seq_lens", "compressed_page_size"),
    "srt/layers/attention/dsv4/low_ratio_backend.py": (
        "low_ratio_decode_rows_are_identity", "low_ratio_decode_rows_are_identity(backend)",
        "low_ratio_decode_rows_are_identity(forward_batch)", "low_ratio_decode_rows_are_identity(ratio)",
        "low_ratio_decode_rows_fit_candidate_span", "low_ratio_decode_rows_fit_candidate_span(backend)",
        "low_ratio_decode_rows_fit_candidate_span(forward_batch)",
    ),
    "srt/layers/attention/dsv4/dsv41_sparse.py": (
        "is_candidate_source", "uses_candidates", "candidate_topk_blocks", "candidate_block_size",
        "n_heads", "wq_b", "weights_proj", "rope_head_dim", "head_weight_scale",
    ),
    "srt/mem_cache/deepseek_v4_memory_pool.py": (
        "get_swa_raw_buffer", "get_swa_key_page_size", "get_extra_key_buffer", "get_extra_key_page_size",
        "get_index_k_fp4_payload_buffer", "get_index_k_fp4_scale_buffer", "low_ratio_index_k_is_split",
        "get_index_k_page_size",
    ),
    "srt/model_executor/forward_context.py": ("get_attn_backend", "get_token_to_kv_pool"),
    "srt/models/deepseek_v4.py": (
        "freqs_cis", "o_groups", "o_lora_rank", "head_dim", "q_lora_rank", "hidden_size",
        "moe_intermediate_size", "num_experts_per_tok", "max_position_embeddings",
        "prepare_language_model_inputs", "logits_processor", "lm_head", "model", "forward(input_ids)",
        "forward(positions)", "forward(forward_batch)", "forward(input_embeds)", "embed_tokens", "hc_mult",
        "norm", "start_layer", "end_layer", "layers", "config", "self_attn", "mlp", "engram", "hc_attn_fn",
        "hc_attn_scale", "hc_attn_base", "hc_ffn_fn", "hc_ffn_scale", "hc_ffn_base", "input_layernorm",
        "post_attention_layernorm", "hc_post", "compressor", "indexer", "q_head_norm", "fuse_wqa_wkv",
        "n_local_heads", "wqkv_a", "wq_b", "wo_a", "wo_b", "q_norm", "kv_norm", "attn_sink",
        "compress_ratio", "weight_scale_inv",
    ),
    "srt/models/deepseek_v2.py": ("experts", "gate", "e_score_correction_bias", "is_nextn", "is_hash"),
    "srt/layers/quantization/mxfp4.py": ("w13_weight", "w2_weight", "w13_weight_scale", "w2_weight_scale"),
    "srt/runtime_context.py": ("get_parallel", "get_model", '"tp_rank"', '"tp_size"', '"tp_group"'),
}

# Per-launch output bounds against the oracle on the same inputs (tests/test_*_gpu.py); the
# north star's contract: integer outputs bit-exact, hidden states within 2e-2 x RMS
NUMERICS = Numerics(
    NumericsKind.TOLERANCE,
    {
        "k1.kv.max_abs": 0.0,          # the SWA KV records' bytes
        "k1.mix.max_abs": 0.0,         # the seam's mixes (the kernels' fixed order)
        "k2.route.ids.max_abs": 0.0,   # routing ids
        "k2.route.wts.max_abs": 0.0,   # routing weights (fp64 fixed-order logits)
        "k2.attn_out.rel": 1e-4,
        "layer.hidden.max_abs_rms": 2e-2,
        "k2i.logits.max_abs": 0.0,     # the kernels' fixed-order logit contract
        "k2i.sel.max_abs": 0.0,        # top-k sets, ties to the lower position
        "head.greedy.agree": 0.995,    # greedy ids agree on at least this share of rows
    },
)


def _covered_layers(config) -> list[int]:
    """The layers K1 and K2 can run: not hash-routed, compress ratio 0, 1 or 2."""
    first = getattr(config, "num_hash_layers", 0) or 0
    return [i for i in range(first, config.num_hidden_layers) if config.compress_ratios[i] in (0, 1, 2)]


def _envelope_reasons(hf_config) -> list[str]:
    reasons = []
    for key, (ok, want) in ENVELOPE.items():
        v = getattr(hf_config, key, None)
        if v is not None and not ok(v):
            reasons.append(f"{key} = {v}: the kernels take {want}")
    return reasons


def _config_disable_reasons(cfg, hf_config) -> list[str]:
    """What ``SPEC.requires`` cannot state: the widths against the kernels' envelope, and
    the built sm_100a library."""
    from ..common import ext

    reasons = _envelope_reasons(hf_config)
    if not ext.LIB_PATH.exists():
        reasons.append("needs the sm_100a library (python -m sgl_amd_mono_b200.deepseek_v41.sm100a.build)")
    return reasons


def _model_disable_reasons(model, hf_config, copies: dict) -> list[str]:
    from sglang.srt.runtime_context import get_parallel

    tp = get_parallel().tp_size
    heads = getattr(hf_config, "num_attention_heads", None)
    covered = _covered_layers(hf_config)
    other = sorted(set(range(hf_config.num_hidden_layers)) - set(covered))
    reasons = [f"layers {other}: no kernels (hash-routed, or another compress ratio)"] if other else []
    unseen = []
    for i in covered:
        layer = model.model.layers[i]
        a, moe = layer.self_attn, layer.mlp
        if moe.is_nextn or moe.is_hash:
            reasons.append(f"layer {i}: needs a routed MoE")
        if any(("shared expert fp8", i, p, k) not in copies for p in _SHARED for k in ("weight", "scale")):
            unseen.append(i)
        if a.q_head_norm or not a.fuse_wqa_wkv or (heads is not None and a.n_local_heads * tp != heads):
            reasons.append(f"layer {i}: K1 needs the fused wqkv_a, heads / tp local heads and no q head norm")
        if (a.compressor is not None or a.indexer is not None) and a.compress_ratio not in (1, 2):
            reasons.append(
                f"layer {i}: a compressor or indexer at compress ratio {a.compress_ratio}; "
                "SGLang's low-ratio sources serve ratio 1 or 2")
        reasons += _indexer_reasons(i=i, attn=a)
    if unseen:
        reasons.append(f"the shared expert's FP8 checkpoint tensors were not seen at load (layers {unseen})")
    return reasons


def _indexer_reasons(*, i: int, attn) -> list[str]:
    ix = attn.indexer
    if ix is None:
        return []
    if (ix.is_candidate_source or ix.uses_candidates) and (ix.candidate_topk_blocks, ix.candidate_block_size) != (
            CANDIDATES["candidate_topk_blocks"], CANDIDATES["candidate_block_size"]):
        return [f"layer {i}: K2i scores candidate blocks of 2048 x 8 rows"]
    if ix.n_heads % 16 or not 16 <= ix.n_heads <= 64:
        return [f"layer {i}: K2i takes 16 to 64 index heads in groups of 16, not {ix.n_heads}"]
    return []


def _load_tensor(copies: dict, model, name: str, tensor: torch.Tensor) -> None:
    """Keep this rank's shard of each covered layer's FP8 shared expert by its checkpoint name
    (the TP-sharded dimension: rows of w1 / w3, columns of w2)."""
    from sglang.srt.runtime_context import get_parallel

    m = _CKPT_SHARED.fullmatch(name)
    if m is None or int(m["i"]) not in _covered_layers(model.config):
        return
    i, proj = int(m["i"]), _CKPT_PROJ[m["w"]]
    p = get_parallel()
    dim = 1 if proj == "down_proj" else 0
    t = tensor.view(torch.uint8)
    n = t.shape[dim] // p.tp_size
    shard = t.narrow(dim, p.tp_rank * n, n)
    if torch.cuda.is_available():
        shard = shard.to(torch.cuda.current_device())
    copies["shared expert fp8", i, proj, m["kind"]] = shard.contiguous()


def e8m0_codes(scale_inv: torch.Tensor, what: str) -> torch.Tensor:
    """fp32 power-of-two block scales -> their E8M0 codes (uint8); other scales refuse."""
    s = scale_inv.float()
    m, e = torch.frexp(s)
    if not bool(((m == 0.5) & (s > 0)).all()):
        raise RuntimeError(f"{what}: block scales must be positive powers of two")
    codes = e.to(torch.int32) - 1 + 127
    if int(codes.min()) < 1 or int(codes.max()) > 254:
        raise RuntimeError(f"{what}: block scale outside E8M0's range")
    return codes.to(torch.uint8).contiguous()


def _keep(copies: dict, t: torch.Tensor, *key) -> torch.Tensor:
    copies[key] = t
    return t


def layer_weights(copies: dict, layer, i: int, tp_rank: int, rope_tables: dict) -> dict:
    """Layer i's tensors as ``MonoRunner.bind`` reads them (read in place where the layout
    allows; the logged copies otherwise)."""
    a, moe = layer.self_attn, layer.mlp
    e, u8 = moe.experts, torch.uint8
    n = moe.gate.weight.shape[0]  # the routed experts

    def codes(name, lin):
        return _keep(copies, e8m0_codes(lin.weight_scale_inv, f"layer {i} {name}"), "e8m0 scale codes", i, name)

    def shared(kind):
        parts = [copies.pop(("shared expert fp8", i, q, kind)) for q in _SHARED[:2]]
        return _keep(copies, torch.cat(parts), "shared expert fp8", i, "gate_up", kind)

    down_w = copies["shared expert fp8", i, "down_proj", "weight"]
    down_s = copies["shared expert fp8", i, "down_proj", "scale"]
    heads = a.n_local_heads
    sink = a.attn_sink.detach()[tp_rank * heads:(tp_rank + 1) * heads].float().contiguous()
    key = id(a.freqs_cis)
    if key not in rope_tables:  # [positions, rope] fp32: cos, then sin
        fc = a.freqs_cis
        rope_tables[key] = torch.cat([fc.real, fc.imag], -1).float().contiguous()
    return {
        "hc_attn_fn": layer.hc_attn_fn, "hc_attn_scale": layer.hc_attn_scale, "hc_attn_base": layer.hc_attn_base,
        "attn_norm": layer.input_layernorm.weight,
        "wqkv": a.wqkv_a.weight.view(u8), "wqkv_s": codes("wqkv_a", a.wqkv_a),
        "q_norm": a.q_norm.weight, "kv_norm": a.kv_norm.weight,
        "wqb": a.wq_b.weight.view(u8), "wqb_s": codes("wq_b", a.wq_b),
        "sink": _keep(copies, sink, "f32 attention sinks", i),
        "woa": a.wo_a.weight.view(u8), "woa_s": codes("wo_a", a.wo_a),
        "wob": a.wo_b.weight.view(u8), "wob_s": codes("wo_b", a.wo_b),
        "hc_ffn_fn": layer.hc_ffn_fn, "hc_ffn_scale": layer.hc_ffn_scale, "hc_ffn_base": layer.hc_ffn_base,
        "ffn_norm": layer.post_attention_layernorm.weight,
        "gate_w": moe.gate.weight,
        "bias": _keep(copies, moe.gate.e_score_correction_bias.float().contiguous(), "f32 router bias", i),
        "w13": e.w13_weight[:n].view(u8), "s13": e.w13_weight_scale[:n].view(u8),
        "w2": e.w2_weight[:n].view(u8), "s2": e.w2_weight_scale[:n].view(u8),
        "sgu": shared("weight"), "sgu_s": shared("scale"),
        "sw2": down_w, "sw2_s": down_s,
        "cos_sin": rope_tables[key],
    }


class _Layer:
    """One covered layer: its module, its bound weights and (at its first launch) caches."""

    def __init__(self, i: int, module, bound, ratio: int, index: bool):
        self.i, self.module, self.w, self.ratio, self.index = i, module, bound, ratio, index
        self.swa = self.comp = self.plane = None
        self.swa_block = self.comp_block = 0


def _launch(runner, L: _Layer, plan, positions, forward_batch, pending, prev_pre, M: int):
    """K1, then K2, of layer ``L``: the previous layer's pending post (x, residual, post, comb)
    and pre in; K2's (x, residual, post, comb, pre) out, this layer's post pending."""
    from sglang.srt.model_executor.forward_context import get_attn_backend, get_token_to_kv_pool

    x, residual, post, comb = pending
    if L.swa is None:  # the layer's caches, at its first launch
        pool = get_token_to_kv_pool()
        L.swa, L.swa_block = pool.get_swa_raw_buffer(L.i), pool.get_swa_key_page_size()
        if L.ratio:
            L.comp = pool.get_extra_key_buffer(L.i).view(torch.uint8)
            L.comp_block = pool.get_extra_key_page_size(L.i)
    backend = get_attn_backend()
    if "k1" not in plan.state:  # the forward's first K1 converts them; a graph records the copies
        slot = backend.get_swa_out_cache_loc(forward_batch)
        plan.state["k1"] = (positions[:M].long().contiguous(), slot[:M].long().contiguous())
    pos, slot = plan.state["k1"]
    md = backend.forward_metadata.core_attn_metadata
    swa_idx, swa_lens = md.swa_page_indices, md.swa_topk_lengths
    topk = dict(topk_width=0)
    if L.ratio:
        idx = md.sparse_page_indices(L.ratio)
        topk = dict(topk_width=idx.shape[1], topk_idx=idx, topk_lens=md.sparse_topk_lengths(L.ratio))
    dummy = runner.zeros_like_pending(M)
    step = dict(res=residual.contiguous(), x=x if x is not None else dummy["x"],
                post=post if post is not None else dummy["post"], comb=comb if comb is not None else dummy["comb"],
                pre=prev_pre if prev_pre is not None else dummy["pre"], pos=pos, slot=slot,
                swa_idx=swa_idx, swa_lens=swa_lens, cache=L.swa, blk=L.swa_block, page_stride=L.swa.stride(0))
    b = runner.k1(L.w, step, M, fold=x is not None, first=prev_pre is None, index=L.index,
                  swa_width=swa_idx.shape[1], **topk)
    if L.index:
        _select(runner=runner, L=L, plan=plan, backend=backend, positions=positions, pos=pos,
                forward_batch=forward_batch, M=M, b=b)
    comp = dict(comp=L.comp, comp_stride=L.comp.stride(0), comp_blk=L.comp_block) if L.ratio else {}
    runner.k2(L.w, step, M, b, **comp)
    return b["out"], b["res2"], b["post_f"], b["comb_f"], b["pre_f"]


def select_kind(ix, fits_candidate_span: bool) -> str:
    """The K2i selection of an index source on a step where SGLang scores rows: every column
    (``full``), or on a two-level step the candidate source (``producer``) and the layers that
    read its blocks (``reindex``) -- SGLang's decode indexer's rule."""
    two_level = (ix.is_candidate_source or ix.uses_candidates) and not fits_candidate_span
    return "full" if not two_level else "reindex" if ix.uses_candidates else "producer"


def _select(*, runner, L, plan, backend, positions, pos, forward_batch, M, b) -> None:
    """An index source between K1 and K2: SGLang's compressor on K1's normed input, then the
    layer's top-k into SGLang's sparse indices of its ratio, from K2i's logits of SGLang's
    query (``K2iRunner.select``)."""
    from sglang.srt.layers.attention.dsv4.low_ratio_backend import (
        low_ratio_decode_rows_are_identity,
        low_ratio_decode_rows_fit_candidate_span,
    )

    attn, r = L.module.self_attn, L.ratio
    if attn.compressor is not None:
        backend.forward_low_ratio_sources(layer=attn, x=b["normed_a"][:M], q_lora=None, positions=positions,
                                          forward_batch=forward_batch, run_indexer=False)
    ix = attn.indexer
    if ix is None:
        return
    fm = backend.forward_metadata
    core, meta = fm.core_attn_metadata, fm.low_ratio_indexer_metadata(r)
    page_idx, raw_idx = core.sparse_page_indices(r), core.sparse_raw_indices(r)
    core.drop_folded_sparse_indices(r)
    bounds = meta.compressed_seq_lens.to(torch.int32).contiguous()
    k2i, per_req = runner.k2i, plan.key.tokens_per_request
    if low_ratio_decode_rows_are_identity(backend=backend, forward_batch=forward_batch, ratio=r):
        # every row sees at most index_topk rows: its top-k is every row, in order
        k2i.identity(rows=M, bounds=bounds, page_table=meta.page_table, raw_out=raw_idx, page_out=page_idx)
        return
    kind = select_kind(ix, low_ratio_decode_rows_fit_candidate_span(backend=backend, forward_batch=forward_batch))
    if L.plane is None:
        L.plane = _index_plane(L, M, meta)
    if kind != "reindex" and ("k2i plan", r) not in plan.state:
        k2i.walk_plan(ratio=r, bounds=bounds, rows=M, per_req=per_req)
        plan.state["k2i plan", r] = True
    published = k2i.select(kind=kind, rows=M, per_req=per_req, ratio=r,
                           query=_index_query(k2i, attn, L, b["normed_a"][:M], b["qr"][:M], pos), plane=L.plane,
                           page_table=meta.page_table, bounds=bounds, raw_out=raw_idx, page_out=page_idx,
                           candidates=plan.state.get("k2i candidates") if kind == "reindex" else None)
    if kind == "producer":
        plan.state["k2i candidates"] = published


def _index_query(k2i, attn, L: _Layer, x: torch.Tensor, q_lora: torch.Tensor, pos: torch.Tensor) -> tuple:
    """The indexer's FP4 query of decode rows, as K2i reads it (the reference's
    ``_index_query``, ``spec.py:744-763``): q = SGLang's wq_b(q_lora), then one C-ABI call
    (``dsv41_index_query``) in place of SGLang's fused ``index_q_rope_pack_weights`` and its
    split-K head-weight GEMV: GPT-J RoPE on each head's last rope_head_dim dims, MXFP4 per 32
    dims, head weights = weights_proj(x) x head_weight_scale in bf16."""
    ix = attn.indexer
    if ix.rope_head_dim != L.w["cos_sin"].shape[1]:
        raise RuntimeError(f"monokernel: layer {L.i}: index RoPE of {ix.rope_head_dim} dims, the layer's table "
                           f"{L.w['cos_sin'].shape[1]}")
    q = ix.wq_b(q_lora)
    q = q[0] if isinstance(q, tuple) else q
    return k2i.query(q=q.contiguous(), cos_sin=L.w["cos_sin"], pos=pos, x=x, wp=ix.weights_proj.weight,
                     scale=ix.head_weight_scale)


def _index_plane(L: _Layer, M: int, meta) -> tuple:
    """The layer's FP4 index plane, after the checks K2i needs of SGLang's index cache."""
    from sglang.srt.model_executor.forward_context import get_token_to_kv_pool

    from .sm100a.indexer import PLANE_ROWS, check_plane

    pool = get_token_to_kv_pool()
    reasons = []
    if not pool.low_ratio_index_k_is_split(L.i):
        reasons.append("the index keys are not in the split FP4 plane")
    if pool.get_index_k_page_size(L.ratio) != PLANE_ROWS:
        reasons.append(f"index pages of {pool.get_index_k_page_size(L.ratio)} rows")
    if meta.compressed_page_size != PLANE_ROWS or meta.page_table.shape[0] != M:
        reasons.append(f"an index page table of {tuple(meta.page_table.shape)} at {meta.compressed_page_size} rows")
    if reasons:
        raise RuntimeError(f"monokernel: layer {L.i}: K2i needs SGLang's FP4 index plane of {PLANE_ROWS}-row "
                           "pages: " + "; ".join(reasons))
    payload = pool.get_index_k_fp4_payload_buffer(L.i)
    scale = pool.get_index_k_fp4_scale_buffer(L.i)
    check_plane(payload, scale)
    return payload.view(torch.uint8), scale


class _Built:
    """One rank's monokernels: the runner, each covered layer, and the forward."""

    def __init__(self, lm, runner, layers: dict):
        self.lm, self.model, self.runner, self._layers = lm, lm.model, runner, layers

    def forward(self, plan, input_ids, positions, forward_batch, input_embeds=None, *_, **__):
        """``DeepseekV4ForCausalLM.forward`` for a routed step: SGLang's input preparation and
        logits processor around the backbone."""
        lm = self.lm
        input_ids, input_embeds = lm.prepare_language_model_inputs(input_ids, forward_batch, input_embeds)
        hidden, pre_hc_head = self.backbone(plan, input_ids, positions, forward_batch, input_embeds)
        return lm.logits_processor(input_ids, hidden, lm.lm_head, forward_batch,
                                   hidden_states_before_norm=pre_hc_head)

    def backbone(self, plan, input_ids, positions, forward_batch, input_embeds):
        """``DeepseekV4Model.forward``: the embedding, each layer as K1 and K2, SGLang's Engram
        writes, then the head's combine and norm."""
        from sglang.kernels.ops.layernorm.mhc import hc_broadcast, hc_combine

        m = self.model
        x = m.embed_tokens(input_ids) if input_embeds is None else input_embeds
        M = x.shape[0]
        if M > MAX_ROWS:
            raise RuntimeError(f"monokernel: {M} rows, at most {MAX_ROWS}")
        pending, pre = (None, hc_broadcast(x, m.hc_mult), None, None), None
        for i in range(m.start_layer, m.end_layer):
            engram = getattr(m.layers[i], "engram", None)
            if engram is not None:
                raise RuntimeError(f"monokernel: layer {i}: Engram writes are not covered")
            out, res, post, comb, pre = _launch(self.runner, self._layers[i], plan, positions, forward_batch,
                                                pending, pre, M)
            if i + 1 < m.end_layer:
                pending = (out, res, post, comb)
            else:
                pending = (None, m.layers[i].hc_post(out, res, post, comb), None, None)
        residual = pending[1]
        pre_hc_head = residual.flatten(1)
        hidden = m.norm(hc_combine(pre_hc_head.float(), pre, m.hc_mult, residual.dtype))
        return hidden, pre_hc_head


def _build(model, hf_config, ctx) -> _Built:
    from sglang.srt.runtime_context import get_parallel

    from ..common.peer import PeerBuffer
    from .shapes import LayerShape
    from .sm100a.indexer import K2iRunner
    from .sm100a.runner import MonoRunner, peer_cap

    p = get_parallel()
    layers0 = model.model.layers
    covered = _covered_layers(hf_config)
    a0, moe0 = layers0[covered[0]].self_attn, layers0[covered[0]].mlp
    shape = LayerShape(
        hidden=hf_config.hidden_size, heads=a0.n_local_heads * p.tp_size,
        nope=hf_config.head_dim - HF_CONFIG["qk_rope_head_dim"], rope=HF_CONFIG["qk_rope_head_dim"],
        q_lora=hf_config.q_lora_rank, o_groups=hf_config.o_groups, o_rank=hf_config.o_lora_rank,
        experts=moe0.gate.weight.shape[0], topk=hf_config.num_experts_per_tok,
        inter=hf_config.moe_intermediate_size, shared_inter=hf_config.moe_intermediate_size,
        tp=p.tp_size)
    device = layers0[covered[0]].input_layernorm.weight.device
    # the peer handshake is collective: every rank gets here (attach agreed first)
    peers = (PeerBuffer(peer_cap(shape, MAX_ROWS), p.tp_group.cpu_group, p.tp_rank, p.tp_size, device)
             if p.tp_size > 1 else None)
    runner = MonoRunner(shape, device, ctx.copies, rank=p.tp_rank, peers=peers, group=p.tp_group.cpu_group,
                        deadline_s=ctx.deadline_s)
    tables: dict = {}
    layers = {}
    for i in covered:
        a = layers0[i].self_attn
        w = layer_weights(ctx.copies, layers0[i], i, p.tp_rank, tables)
        index = a.compressor is not None or a.indexer is not None
        layers[i] = _Layer(i, layers0[i], runner.bind(w, tag=f"layer {i}"), a.compress_ratio, index)
    for n, t in enumerate(tables.values()):
        ctx.copies["rope table", n] = t
    if any(L.module.self_attn.indexer is not None for L in layers.values()):
        ctx_len = getattr(hf_config, "max_position_embeddings", 0) + 2 * MAX_ROWS
        runner.k2i = K2iRunner(device, ctx_len)
    return _Built(model, runner, layers)


SPEC = MonoSpec(
    name="deepseek_v41_cuda",
    devices={ISA: DeviceLimits(widths=tuple(range(1, MAX_ROWS + 1)), tp_sizes=(1, 2, 4, 8),
                               resident_blocks=RESIDENT_BLOCKS)},
    features=frozenset({Feature.SPECULATIVE_DECODING}),
    requires=Requirements(
        dtypes=frozenset({"bfloat16"}),
        attention_backends=frozenset({"dsv4"}),
        server_args={
            "kv_cache_dtype": frozenset({"fp8_e4m3"}),
            # DSpark's target steps are uniform verify steps; other drafts differ
            "speculative_algorithm": frozenset({None, "DSPARK"}),
            # the paged SWA cache, not a request window
            "enable_encoder_swa_bounded_replay": frozenset({False}),
        },
        hf_config={**HF_CONFIG, "model_type": "deepseek_v41"},
        env={
            # MXFP4 experts row-major (relaid once, logged), fp8 nope + bf16 rope records
            "SGLANG_DSV4_FP4_EXPERTS": True,
            "SGLANG_DSV4_FP4_DEQUANT": False,
            "SGLANG_DSV4_KV_LAYOUT": "v4",
        },
    ),
    numerics=NUMERICS,
    model_disable_reasons=_model_disable_reasons,
    build=_build,
    api_version=1,  # sglang.srt.monokernels.spec.MONOKERNEL_API_VERSION
    config_disable_reasons=_config_disable_reasons,
    load_tensor=_load_tensor,
    # a routed step scores every index source with K2i (_select)
    unread_metadata=frozenset({StepMetadata.LOW_RATIO_DECODE_SCHEDULE}),
)
