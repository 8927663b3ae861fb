"""The routed forward on the GPU: a two-layer DeepSeek-V4.1 model made of stand-in SGLang modules
(seeded synthetic weights in SGLang's layouts: FP8 linears with fp32 power-of-two block
scales, MXFP4 experts, the shared expert through the load hook), attached with
``SPEC.build`` and run by ``_Built.forward`` -- K1 and K2 of each layer through the C-ABI --
against the oracle: layer 0 from the step's inputs, layer 1 from the GPU's own layer-0 outputs
(a one-layer run of the same weights; teacher forcing), so every layer's KV records are
bit-exact; the head's hidden state and logits within the reference's MoE bound (rel 1.5e-2:
element-wise bounds stop at the MXFP8 requantization of each layer's attention output, where a
one-step bf16 difference flips e4m3 codes). The DSpark draft's forward likewise, one stage."""

from types import SimpleNamespace

import pytest
import torch

from oracle import layer as OL

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SHAPE = dict(hidden=1024, heads=8, nope=512, rope=64, q_lora=256, o_groups=1, o_rank=1024, experts=16, topk=4,
             inter=512, shared_inter=512)
M, CTX, VOCAB = 4, 256, 3000


def _shape():
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    return LayerShape(**SHAPE)


def _fp8_lin(u8, codes):
    return SimpleNamespace(weight=u8.view(torch.float8_e4m3fn),
                           weight_scale_inv=torch.ldexp(torch.ones(codes.shape, device=codes.device), codes.int() - 127))


def _rms_norm(w):
    def norm(x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(torch.bfloat16)
    return norm


def _module(w, s):
    """One decoder layer as SGLang's modules hold it."""
    cs = w["cos_sin"]
    attn = SimpleNamespace(
        wqkv_a=_fp8_lin(w["wqkv"], w["wqkv_s"]), wq_b=_fp8_lin(w["wqb"], w["wqb_s"]),
        wo_a=_fp8_lin(w["woa"], w["woa_s"]), wo_b=_fp8_lin(w["wob"], w["wob_s"]),
        q_norm=SimpleNamespace(weight=w["q_norm"]), kv_norm=SimpleNamespace(weight=w["kv_norm"]),
        attn_sink=w["sink"], freqs_cis=torch.complex(cs[:, :32], cs[:, 32:]), n_local_heads=s.heads,
        compress_ratio=0, compressor=None, indexer=None, q_head_norm=False, fuse_wqa_wkv=True)
    experts = SimpleNamespace(w13_weight=w["w13"], w13_weight_scale=w["s13"], w2_weight=w["w2"],
                              w2_weight_scale=w["s2"])
    mlp = SimpleNamespace(gate=SimpleNamespace(weight=w["gate_w"], e_score_correction_bias=w["bias"]),
                          experts=experts, is_nextn=False, is_hash=False)
    return SimpleNamespace(
        self_attn=attn, mlp=mlp, engram=None,
        hc_attn_fn=w["hc_attn_fn"], hc_attn_scale=w["hc_attn_scale"], hc_attn_base=w["hc_attn_base"],
        hc_ffn_fn=w["hc_ffn_fn"], hc_ffn_scale=w["hc_ffn_scale"], hc_ffn_base=w["hc_ffn_base"],
        input_layernorm=SimpleNamespace(weight=w["attn_norm"]),
        post_attention_layernorm=SimpleNamespace(weight=w["ffn_norm"]),
        hc_post=lambda x, res, post, comb: OL.fold_post(res.cpu(), x.cpu(), post.cpu(), comb.cpu()).to(
            torch.bfloat16).to(x.device))


def _load_shared(load, copies, lm, w, prefix, s):
    SI = s.shared_inter
    parts = {"w1": (w["sgu"][:SI], w["sgu_s"][:SI // 128]), "w3": (w["sgu"][SI:], w["sgu_s"][SI // 128:]),
             "w2": (w["sw2"], w["sw2_s"])}
    for n, (wt, sc) in parts.items():
        load(copies, lm, f"{prefix}.ffn.shared_experts.{n}.weight", wt.view(torch.float8_e4m3fn))
        load(copies, lm, f"{prefix}.ffn.shared_experts.{n}.scale", sc)


def _to(d, dev):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in d.items()}


def _world(fake, n_layers, draft=False):
    """Weights, the step, the stand-in model and the SGLang context, on the GPU."""
    import sglang.srt.model_executor.forward_context as fc

    from sgl_amd_mono_b200.deepseek_v41 import synth
    s = _shape()
    ws = [synth.make_layer(s, 41 + i, "cpu", positions=CTX + 8) for i in range(n_layers)]
    S = synth.make_step(s, M, CTX, 51, "cpu")
    g = torch.Generator().manual_seed(61)
    emb = torch.randn(VOCAB, s.hidden, generator=g).to(torch.bfloat16)
    head = (torch.randn(VOCAB, s.hidden, generator=g) * 0.02).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(s.hidden, generator=g)).to(torch.bfloat16)
    ids = torch.randint(0, VOCAB, (M,), generator=g)
    modules = [_module(_to(w, DEV), s) for w in ws]
    hf = SimpleNamespace(num_hidden_layers=n_layers, compress_ratios=[0] * n_layers, hidden_size=s.hidden,
                         head_dim=s.head_dim, q_lora_rank=s.q_lora, o_groups=s.o_groups, o_lora_rank=s.o_rank,
                         num_experts_per_tok=s.topk, moe_intermediate_size=s.inter, num_attention_heads=s.heads,
                         max_position_embeddings=CTX + 8, dspark_n_routed_experts=s.experts,
                         dspark_num_experts_per_tok=s.topk)
    embd, headd = emb.to(DEV), head.to(DEV)
    m = SimpleNamespace(layers=modules, embed_tokens=lambda t: embd[t], hc_mult=4, norm=_rms_norm(norm_w.to(DEV)),
                        start_layer=0, end_layer=n_layers)
    lm = SimpleNamespace(
        model=m, config=hf, lm_head=SimpleNamespace(weight=headd), stages=modules, hc_mult=4,
        hc_pre_from_prev_sublayer=True, sample_from_anchor=True,
        forward_embed=lambda t: embd[t][:, None, :].expand(t.shape[0], 4, s.hidden).contiguous(),
        prepare_language_model_inputs=lambda i, fb, e: (i, e),
        logits_processor=lambda i, h, head, fb, **kw: SimpleNamespace(next_token_logits=h.float() @ head.weight.float().T))
    caches = [S["cache"].clone().to(DEV) for _ in range(n_layers)]
    Sd = _to(S, DEV)
    md = SimpleNamespace(swa_page_indices=Sd["swa_idx"], swa_topk_lengths=Sd["swa_lens"])
    fc.BACKEND = SimpleNamespace(forward_metadata=SimpleNamespace(core_attn_metadata=md),
                                 get_swa_out_cache_loc=lambda fb: Sd["slot"])
    fc.POOL = SimpleNamespace(get_swa_raw_buffer=lambda i: caches[i], get_swa_key_page_size=lambda: S["blk"])
    return dict(s=s, ws=ws, S=S, emb=emb, head=head, norm_w=norm_w, ids=ids, lm=lm, hf=hf, caches=caches,
                positions=Sd["pos"])


def _oracle(wd, draft=False, forced=None):
    """The oracle over the layers; ``forced`` (the GPU's layer-0 outputs) feeds layer 1."""
    s, S = wd["s"], wd["S"]
    x0 = wd["emb"][wd["ids"]]
    res = x0[:, None, :].expand(M, 4, s.hidden).contiguous()
    zero = dict(x=torch.zeros(M, s.hidden), post=torch.zeros(M, 4), comb=torch.zeros(M, 4, 4), pre=torch.zeros(M, 4))
    pend, caches = None, []
    for i, w in enumerate(wd["ws"]):
        cache = S["cache"].clone()
        if i == 1 and forced is not None:
            pend = forced
        if pend is None or draft:
            Si = dict(S, res=res, **zero)
            o = OL.decode_layer([w], Si, s, cache=cache, fold=False, first=pend is None)
        else:
            Si = dict(S, res=pend["res2"], x=pend["out"], post=pend["post2"], comb=pend["comb2"], pre=pend["pre2"])
            o = OL.decode_layer([w], Si, s, cache=cache, fold=True, first=False)
        caches.append(cache)
        pend = o
        if draft:
            res = OL.fold_post(o["res2"], o["out"], o["post2"], o["comb2"])
    if not draft:
        res = OL.fold_post(pend["res2"], pend["out"], pend["post2"], pend["comb2"])
    flat = res.reshape(M, -1).float()
    acc = torch.zeros(M, s.hidden)
    for h in range(4):
        acc = acc + pend["pre2"][:, h, None] * flat.view(M, 4, -1)[:, h]
    return acc.to(torch.bfloat16), caches


def _close(got, ref, tol=1.5e-2):
    got, ref = got.float().cpu(), ref.float()
    assert (got - ref).norm() / ref.norm() < tol, float((got - ref).norm() / ref.norm())


def test_target_forward_two_layers(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import spec
    wd = _world(fake_sglang, 2)
    copies = {}
    for i, w in enumerate(wd["ws"]):
        _load_shared(spec.SPEC.load_tensor, copies, wd["lm"], _to(w, DEV), f"layers.{i}", wd["s"])
    assert spec.SPEC.model_disable_reasons(wd["lm"], wd["hf"], copies) == []
    built = spec.SPEC.build(wd["lm"], wd["hf"], SimpleNamespace(copies=copies, deadline_s=5.0, widths=range(1, 49)))
    assert any(k[0] == "mxfp4 tensor-core tile relayout" for k in copies) and ("e8m0 scale codes", 0, "wq_b") in copies
    plan = SimpleNamespace(state={}, key=SimpleNamespace(tokens_per_request=1))
    ids = wd["ids"].to(DEV)
    hidden, _ = built.backbone(plan, ids, wd["positions"], None, None)
    out = built.forward(SimpleNamespace(state={}, key=plan.key), ids, wd["positions"], None)
    torch.cuda.synchronize()
    caches2 = [c.clone() for c in wd["caches"]]
    # the GPU's layer-0 outputs: a one-layer model of the same first layer, same step
    wd1 = _world(fake_sglang, 1)
    copies1 = {}
    _load_shared(spec.SPEC.load_tensor, copies1, wd1["lm"], _to(wd1["ws"][0], DEV), "layers.0", wd1["s"])
    built1 = spec.SPEC.build(wd1["lm"], wd1["hf"], SimpleNamespace(copies=copies1, deadline_s=5.0,
                                                                      widths=range(1, 49)))
    built1.backbone(SimpleNamespace(state={}, key=plan.key), ids, wd1["positions"], None, None)
    torch.cuda.synchronize()
    b0 = built1.runner.buffers(M, wd["S"]["swa_idx"].shape[1])
    forced = dict(res2=b0["res2"].cpu(), out=b0["out"].cpu().float(), post2=b0["post_f"].cpu(),
                  comb2=b0["comb_f"].cpu(), pre2=b0["pre_f"].cpu())
    ref_x, ref_caches = _oracle(wd, forced=forced)
    ref_hidden = _rms_norm(wd["norm_w"])(ref_x)
    for got, want in zip(caches2, ref_caches):
        assert torch.equal(got.cpu(), want)  # every layer's KV records
    _close(hidden, ref_hidden)
    logits = out.next_token_logits.cpu()
    want = ref_hidden.float() @ wd["head"].float().T
    _close(logits, want)


def test_draft_forward_one_stage(fake_sglang):
    from sgl_amd_mono_b200.deepseek_v41 import draft
    wd = _world(fake_sglang, 1, draft=True)
    copies = {}
    _load_shared(draft.SPEC.load_tensor, copies, wd["lm"], _to(wd["ws"][0], DEV), "mtp.0", wd["s"])
    assert draft.SPEC.model_disable_reasons(wd["lm"], wd["hf"], copies) == []
    built = draft.SPEC.build(wd["lm"], wd["hf"], SimpleNamespace(copies=copies, deadline_s=5.0, widths=range(1, 49)))
    plan = SimpleNamespace(state={}, key=SimpleNamespace(tokens_per_request=6))
    out = built.forward(plan, wd["ids"].to(DEV), wd["positions"], None)
    torch.cuda.synchronize()
    ref_x, ref_caches = _oracle(wd, draft=True)
    assert torch.equal(wd["caches"][0].cpu(), ref_caches[0])
    assert out.next_token_logits is None
    _close(out.hidden_states, ref_x)
