"""The DSpark draft of DeepSeek-V4.1 on sm_100a: the draft model's spec and forward, behind the
interface of the reference's ``deepseek_v41/draft.py``.

The draft runs as its own routed step: SGLang hands ``_Draft.forward`` a verify-shaped batch
(each request contributes its block of draft rows) and expects back what
``DeepseekV4ForCausalLMDSpark.forward`` would return. Here every draft stage is one K1 + K2
launch pair -- the target's own kernels, given the draft's expert count, top-k and attention
window as launch-time widths -- followed by SGLang's ``hc_post``; the head then combines the
last stage's residual copies with that stage's pre, as SGLang does. No kernel is specific to
the draft.
"""

from __future__ import annotations

import re

import torch
from sglang.srt.monokernels.spec import DeviceLimits, Feature, MonoSpec, Requirements

from . import spec as target

# the checkpoint's draft stages are mtp.{stage}
_CKPT_SHARED = re.compile(r"mtp\.(?P<i>\d+)\.ffn\.shared_experts\.(?P<w>w[123])\.(?P<kind>weight|scale)")

# The SGLang names this module reads, by file under the sglang package (``f(p)``: a parameter,
# ``"x"``: a string literal); tests/test_spec.py pins them against this module's imports.
SGLANG_READS = {
    "srt/monokernels/spec.py": ("DeviceLimits", "Feature", "MonoSpec", "Requirements"),
    "kernels/ops/layernorm/mhc.py": ("hc_combine",),
    "srt/layers/logits_processor.py": ("LogitsProcessorOutput", "next_token_logits", "hidden_states"),
    "srt/models/deepseek_v4_dspark.py": (
        "forward(input_ids)", "forward(positions)", "forward(forward_batch)", "forward(input_embeds)",
        "stages", "forward_embed", "hc_mult", "hc_pre_from_prev_sublayer", "sample_from_anchor",
        '"dspark_n_routed_experts"', '"dspark_num_experts_per_tok"',
    ),
    "srt/runtime_context.py": ("get_parallel", "get_spec", '"tp_group"'),
    "srt/speculative/dspark_components/dspark_config.py": ("dspark_gamma_from_num_draft_tokens",),
}


def _tokens_per_request(model) -> int:
    """A draft block's rows a request: gamma, or gamma + 1 without the anchor."""
    from sglang.srt.runtime_context import get_spec
    from sglang.srt.speculative.dspark_components.dspark_config import dspark_gamma_from_num_draft_tokens

    gamma = dspark_gamma_from_num_draft_tokens(int(get_spec().speculative_num_draft_tokens))
    return gamma if model.sample_from_anchor else gamma + 1


def _model_disable_reasons(model, hf_config, copies: dict) -> list[str]:
    from sglang.srt.runtime_context import get_parallel

    reasons, unseen = [], []
    experts = getattr(hf_config, "dspark_n_routed_experts", None)
    topk = getattr(hf_config, "dspark_num_experts_per_tok", None)
    if experts is None or not 1 <= experts <= 512 or topk is None or not 1 <= topk <= 32:
        reasons.append(f"draft route ({experts}, {topk}): the kernels take 1..512 experts, top-1..32")
    rows = _tokens_per_request(model)
    if rows > target.MAX_ROWS:
        reasons.append(f"a draft block of {rows} rows past {target.MAX_ROWS}")
    if not getattr(model, "hc_pre_from_prev_sublayer", False):
        reasons.append("needs V4.1's mHC hand-off between stages")
    tp = get_parallel().tp_size
    heads = getattr(hf_config, "num_attention_heads", None)
    for i, stage in enumerate(model.stages):
        a = stage.self_attn
        if a.compress_ratio != 0 or a.q_head_norm or (heads is not None and a.n_local_heads * tp != heads):
            reasons.append(f"stage {i}: needs a window-only attention with heads / tp local heads and no q head "
                           "norm")
        if any(("shared expert fp8", i, p, k) not in copies for p in target._SHARED for k in ("weight", "scale")):
            unseen.append(i)
    if unseen:
        reasons.append(f"the shared expert's FP8 checkpoint tensors were not seen at load (stages {unseen})")
    return reasons


def _load_tensor(copies: dict, model, name: str, tensor: torch.Tensor) -> None:
    """Keep this rank's shard of each stage's FP8 shared expert, by its checkpoint name
    (``mtp.{stage}.ffn.shared_experts.{w1,w2,w3}.{weight,scale}``)."""
    from sglang.srt.runtime_context import get_parallel

    m = _CKPT_SHARED.fullmatch(name)
    if m is None or int(m["i"]) >= len(model.stages):
        return
    i, proj = int(m["i"]), target._CKPT_PROJ[m["w"]]
    p = get_parallel()
    dim = 1 if proj == "down_proj" else 0
    t = tensor.view(torch.uint8)
    n = t.shape[dim] // p.tp_size
    shard = t.narrow(dim, p.tp_rank * n, n)
    if torch.cuda.is_available():
        shard = shard.to(torch.cuda.current_device())
    copies["shared expert fp8", i, proj, m["kind"]] = shard.contiguous()


class _Draft:
    """One rank's draft monokernels: its runner, each stage's weights, the forward."""

    def __init__(self, lm, runner, stages: list):
        self.lm, self.runner, self.stages = lm, runner, stages

    def forward(self, plan, input_ids, positions, forward_batch, input_embeds=None, *_, **__):
        """``DeepseekV4ForCausalLMDSpark.forward`` for a routed draft step."""
        from sglang.kernels.ops.layernorm.mhc import hc_combine
        from sglang.srt.layers.logits_processor import LogitsProcessorOutput

        lm = self.lm
        x = lm.forward_embed(input_ids) if input_embeds is None else input_embeds
        M, pre = x.shape[0], None
        for L in self.stages:  # each stage settles its post: what SGLang's returns
            out, res, post, comb, pre = target._launch(self.runner, L, plan, positions, forward_batch,
                                                       (None, x, None, None), pre, M)
            x = L.module.hc_post(out, res, post, comb)
        x = hc_combine(x.flatten(1).float(), pre, lm.hc_mult, x.dtype)
        return LogitsProcessorOutput(next_token_logits=None, hidden_states=x)


def _build(model, hf_config, ctx) -> _Draft:
    from sglang.srt.runtime_context import get_parallel

    from ..common.peer import PeerBuffer
    from .shapes import LayerShape
    from .sm100a.runner import MonoRunner, peer_cap

    p = get_parallel()
    s0 = model.stages[0]
    shape = LayerShape(
        hidden=hf_config.hidden_size, heads=s0.self_attn.n_local_heads * p.tp_size,
        nope=hf_config.head_dim - target.HF_CONFIG["qk_rope_head_dim"], rope=target.HF_CONFIG["qk_rope_head_dim"],
        q_lora=hf_config.q_lora_rank, o_groups=hf_config.o_groups, o_rank=hf_config.o_lora_rank,
        experts=hf_config.dspark_n_routed_experts, topk=hf_config.dspark_num_experts_per_tok,
        inter=hf_config.moe_intermediate_size, shared_inter=hf_config.moe_intermediate_size, tp=p.tp_size)
    device = s0.input_layernorm.weight.device
    peers = (PeerBuffer(peer_cap(shape, target.MAX_ROWS), p.tp_group.cpu_group, p.tp_rank, p.tp_size, device)
             if p.tp_size > 1 else None)
    runner = MonoRunner(shape, device, ctx.copies, rank=p.tp_rank, peers=peers, group=p.tp_group.cpu_group,
                        deadline_s=ctx.deadline_s)
    tables: dict = {}
    stages = []
    for i, stage in enumerate(model.stages):
        w = target.layer_weights(ctx.copies, stage, i, p.tp_rank, tables)
        stages.append(target._Layer(i, stage, runner.bind(w, tag=f"draft stage {i}"), 0, False))
    for n, t in enumerate(tables.values()):
        ctx.copies["draft rope table", n] = t
    return _Draft(model, runner, stages)


SPEC = MonoSpec(
    name="deepseek_v41_dspark_draft_cuda",
    devices={target.ISA: DeviceLimits(widths=tuple(range(1, target.MAX_ROWS + 1)), tp_sizes=(1, 2, 4, 8),
                                      resident_blocks=target.RESIDENT_BLOCKS)},
    features=frozenset({Feature.SPECULATIVE_DECODING}),
    # the launcher checks the target's requirements; the capture check, this
    requires=Requirements(attention_backends=target.SPEC.requires.attention_backends),
    numerics=target.NUMERICS,
    model_disable_reasons=_model_disable_reasons,
    build=_build,
    api_version=1,  # sglang.srt.monokernels.spec.MONOKERNEL_API_VERSION
    load_tensor=_load_tensor,
    tokens_per_request=_tokens_per_request,
)
