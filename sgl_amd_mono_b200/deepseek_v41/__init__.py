"""DeepSeek-V4.1 monokernels for B200: the spec and its SGLang glue in ``spec`` / ``draft``,
and the sm_100a kernels and host runner in ``sm100a``.

The reference builds for DeepSeek-V4.1-Flash's exact widths; these kernels take every width
as a launch argument, so the spec pins the model's arithmetic (routing, activation, mHC,
norms, RoPE width) and checks its widths against the kernels' envelope instead
(``ENVELOPE``, ``spec._config_disable_reasons``).
"""

# DeepSeek-V4.1's routing, activation and mixing, which the kernels build in
# (reference ``deepseek_v41/__init__.py:12-39`` without its widths)
HF_CONFIG = dict(
    n_shared_experts=1,
    routed_scaling_factor=1.5,
    scoring_func="sqrtsoftplus",
    norm_topk_prob=True,
    topk_method="noaux_tc",
    hidden_act="silu",
    swiglu_limit=10.0,
    hc_mult=4,
    hc_sinkhorn_iters=20,
    hc_eps=1e-6,
    rms_norm_eps=1e-20,
    hc_pre_from_prev_sublayer=True,
    qk_rope_head_dim=64,
)
# the widths the kernels take (``sm100a/csrc/capi.cu`` argument checks)
ENVELOPE = dict(
    hidden_size=(lambda v: v % 1024 == 0 and 1024 <= v <= 16384, "a multiple of 1024 up to 16384"),
    q_lora_rank=(lambda v: v in (256, 512, 1024), "256, 512 or 1024"),
    head_dim=(lambda v: v % 64 == 0 and 128 <= v <= 576, "nope + 64 RoPE dims, nope a multiple of 64 <= 512"),
    moe_intermediate_size=(lambda v: v % 128 == 0, "a multiple of 128 a rank"),
    n_routed_experts=(lambda v: 1 <= v <= 512, "1..512"),
    num_experts_per_tok=(lambda v: 1 <= v <= 32, "1..32"),
    index_n_heads=(lambda v: v in (16, 32, 48, 64), "16, 32, 48 or 64"),
    index_head_dim=(lambda v: v == 128, "128"),
)
# a candidate source's (``candidate_source_layer_id``) top blocks, which K2i scores
CANDIDATES = dict(candidate_topk_blocks=2048, candidate_block_size=8)
