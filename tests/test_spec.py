"""The plugin surface on CPU against a stand-in of SGLang's monokernel interface: the entry
point registers both specs and the registry finds them for sm_100a; the layers the forward
covers on DeepSeek-V4.1-Flash's layer structure; the numeric bounds; the model and config
refusal reasons; the load hook keeping this rank's shared-expert shard; the E8M0 scale codes;
K2i's selection kinds; and every SGLang name a module imports is declared in its
SGLANG_READS. The reference's ``test/unit/test_deepseek_v41_spec.py`` and
``test/unit/test_contract.py`` are the model."""

import ast
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

import sgl_amd_mono_b200

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "sgl_amd_mono_b200"

HF = dict(scoring_func="sqrtsoftplus", hc_mult=4, hidden_size=4096, q_lora_rank=1024, head_dim=576,
          moe_intermediate_size=2048, n_routed_experts=256, num_experts_per_tok=8, index_n_heads=64,
          index_head_dim=128)
# DeepSeek-V4.1-Flash's layer structure (its config.json), with config-2 widths
FLASH = SimpleNamespace(num_hidden_layers=40, compress_ratios=[0, 0] + [2] * 18 + [1] * 20 + [0, 0, 0],
                        model_type="deepseek_v41", num_attention_heads=64, **HF)


def test_covered_layers(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import spec
    assert spec._covered_layers(FLASH) == list(range(40))
    hashed = SimpleNamespace(**{**vars(FLASH), "num_hash_layers": 4})
    assert spec._covered_layers(hashed) == list(range(4, 40))
    ratio4 = SimpleNamespace(**{**vars(FLASH), "compress_ratios": [4] * 43})
    assert spec._covered_layers(ratio4) == []


def test_the_plugin_registers_both_specs(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import draft, spec
    sgl_amd_mono_b200.register_specs()
    for arch, want in (("DeepseekV4ForCausalLM", spec.SPEC), ("DeepseekV4ForCausalLMDSpark", draft.SPEC)):
        found, why = fake_sglang.find_spec(backend=sgl_amd_mono_b200.BACKEND, architectures=[arch], isa="sm_100a")
        assert found is want, why
    found, why = fake_sglang.find_spec(backend=sgl_amd_mono_b200.BACKEND, architectures=["DeepseekV4ForCausalLM"],
                                       isa="gfx950")
    assert found is None and "no kernels" in why
    assert spec.SPEC.devices["sm_100a"].tp_sizes == (1, 2, 4, 8)
    assert spec.SPEC.devices["sm_100a"].widths == tuple(range(1, 49))


def test_numerics_pin_the_bit_exact_outputs(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import draft, spec
    for s in (spec.SPEC, draft.SPEC):
        for name in ("k1.kv.max_abs", "k2.route.ids.max_abs", "k2i.sel.max_abs"):
            assert s.numerics.bound(name) == 0.0
        assert s.numerics.bound("layer.hidden.max_abs_rms") == 2e-2
        assert s.numerics.bound("head.greedy.agree") == 0.995


def _layer(i, **attn):
    attn = {"compressor": None, "indexer": None, "q_head_norm": False, "fuse_wqa_wkv": True, "n_local_heads": 16,
            "compress_ratio": 0 if i < 2 else 2 if i < 20 else 1, **attn}
    return SimpleNamespace(self_attn=SimpleNamespace(**attn), mlp=SimpleNamespace(is_nextn=False, is_hash=False))


def test_model_reasons(fake_sglang):
    import sglang.srt.runtime_context as rc

    from sgl_amd_mono_b200.deepseek_v41 import CANDIDATES, spec
    rc.PARALLEL = SimpleNamespace(tp_size=4, tp_rank=0, tp_group=None)
    layers = [_layer(i) for i in range(40)]
    model = SimpleNamespace(model=SimpleNamespace(layers=layers))
    seen = {("shared expert fp8", i, p, k): None for i in range(40) for p in spec._SHARED for k in ("weight", "scale")}
    assert spec.SPEC.model_disable_reasons(model, FLASH, seen) == []
    layers[1] = _layer(1, compress_ratio=0, compressor=SimpleNamespace())
    layers[5] = _layer(5, q_head_norm=True)
    seen = {k: v for k, v in seen.items() if k[1] != 7}
    reasons = spec.SPEC.model_disable_reasons(model, FLASH, seen)
    assert len(reasons) == 3, reasons
    assert reasons[0].startswith("layer 1: a compressor or indexer at compress ratio 0")
    assert reasons[1].startswith("layer 5: K1 needs the fused wqkv_a")
    assert "(layers [7])" in reasons[2]
    hashed = SimpleNamespace(**{**vars(FLASH), "num_hash_layers": 2})
    assert spec.SPEC.model_disable_reasons(model, hashed, seen)[0].startswith("layers [0, 1]: no kernels")
    # K2i's indexers: the candidate blocks and the index heads
    layers[1], layers[5] = _layer(1), _layer(5)
    seen |= {("shared expert fp8", 7, p, k): None for p in spec._SHARED for k in ("weight", "scale")}
    ix = SimpleNamespace(is_candidate_source=True, uses_candidates=False, n_heads=64, **CANDIDATES)
    layers[20] = _layer(20, indexer=ix)
    assert spec.SPEC.model_disable_reasons(model, FLASH, seen) == []
    layers[20] = _layer(20, indexer=SimpleNamespace(**{**vars(ix), "candidate_topk_blocks": 1024}))
    layers[24] = _layer(24, indexer=SimpleNamespace(**{**vars(ix), "n_heads": 40}))
    reasons = spec.SPEC.model_disable_reasons(model, FLASH, seen)
    assert [r.split(":")[0] for r in reasons] == ["layer 20", "layer 24"], reasons
    rc.PARALLEL = SimpleNamespace(tp_size=1, tp_rank=0, tp_group=None)


def test_config_reasons_check_the_kernel_envelope(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import spec
    assert spec._envelope_reasons(FLASH) == []
    odd = SimpleNamespace(**{**vars(FLASH), "q_lora_rank": 1280, "index_n_heads": 40})
    r = spec._envelope_reasons(odd)
    assert [x.split(" =")[0] for x in r] == ["q_lora_rank", "index_n_heads"]


def test_load_tensor_keeps_this_ranks_shard(fake_sglang):
    import sglang.srt.runtime_context as rc

    from sgl_amd_mono_b200.deepseek_v41 import draft, spec
    rc.PARALLEL = SimpleNamespace(tp_size=2, tp_rank=1, tp_group=None)
    model = SimpleNamespace(config=FLASH, stages=[None])
    copies = {}
    w1 = torch.arange(8 * 6, dtype=torch.uint8).view(8, 6)
    w2 = torch.arange(6 * 8, dtype=torch.uint8).view(6, 8)
    spec.SPEC.load_tensor(copies, model, "layers.3.ffn.shared_experts.w1.weight", w1)
    spec.SPEC.load_tensor(copies, model, "layers.3.ffn.shared_experts.w2.weight", w2)
    spec.SPEC.load_tensor(copies, model, "layers.3.attn.wq_b.weight", w1)  # not a shared expert
    spec.SPEC.load_tensor(copies, model, "mtp.0.ffn.shared_experts.w1.weight", w1)  # the draft's
    assert set(copies) == {("shared expert fp8", 3, "gate_proj", "weight"), ("shared expert fp8", 3, "down_proj", "weight")}
    assert torch.equal(copies["shared expert fp8", 3, "gate_proj", "weight"], w1[4:])
    assert torch.equal(copies["shared expert fp8", 3, "down_proj", "weight"], w2[:, 4:])
    dc = {}
    draft.SPEC.load_tensor(dc, model, "mtp.0.ffn.shared_experts.w3.weight", w1)
    draft.SPEC.load_tensor(dc, model, "mtp.1.ffn.shared_experts.w3.weight", w1)  # no stage 1
    assert set(dc) == {("shared expert fp8", 0, "up_proj", "weight")}
    rc.PARALLEL = SimpleNamespace(tp_size=1, tp_rank=0, tp_group=None)


def test_e8m0_codes(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import spec
    s = torch.tensor([[2.0 ** -7, 1.0], [2.0 ** 5, 0.25]])
    assert spec.e8m0_codes(s, "w").tolist() == [[120, 127], [132, 125]]
    with pytest.raises(RuntimeError, match="powers of two"):
        spec.e8m0_codes(torch.tensor([0.3]), "w")


def test_select_kinds(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import spec
    ix = lambda src, uses: SimpleNamespace(is_candidate_source=src, uses_candidates=uses)  # noqa: E731
    assert spec.select_kind(ix(False, False), False) == "full"
    assert spec.select_kind(ix(True, False), False) == "producer"
    assert spec.select_kind(ix(False, True), False) == "reindex"
    assert spec.select_kind(ix(True, False), True) == "full"  # the rows fit one candidate span


def test_draft_tokens_per_request(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import draft
    assert draft.SPEC.tokens_per_request(SimpleNamespace(sample_from_anchor=True)) == 5
    assert draft.SPEC.tokens_per_request(SimpleNamespace(sample_from_anchor=False)) == 6


def _declared(tree):
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "SGLANG_READS" for t in node.targets):
            return ast.literal_eval(node.value)
    return {}


def test_every_sglang_import_is_declared():
    """A module that imports from sglang lists every imported name in its SGLANG_READS, so a
    rename in SGLang is found by a static check instead of at a server's startup."""
    readers = 0
    for path in sorted(PACKAGE.rglob("*.py")):
        tree = ast.parse(path.read_text())
        imported = {a.asname or a.name for n in ast.walk(tree) if isinstance(n, ast.ImportFrom)
                    and (n.module or "").startswith("sglang.") for a in n.names}
        if not imported:
            continue
        readers += 1
        declared = {name for names in _declared(tree).values() for name in names}
        assert imported <= declared, (path.name, imported - declared)
    assert readers == 3  # the package entry, the spec and the draft
