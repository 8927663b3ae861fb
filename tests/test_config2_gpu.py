"""K1 + K2 at BASELINE config-2 shapes -- the kernel configurations ``bench.py`` times -- on the
GPU against the CPU oracle, stage by stage.

Config 2 is hidden 4096, 64 heads of 512 + 64 dims (so the tcgen05 attention runs over the
row's 64 heads in one CTA, ``attn_wide_kernel<512>``, the default, and over its two 32-head
tiles, ``attn_tc_kernel<512, ...>``), q_lora 1024, 8 wo_a
groups of 1024, 256 routed experts top-8 with intermediate 2048 (the expert kernel's K slices
and row groups) and a shared expert of 2048. Rows M = 1 (the CUDA-core GEMVs), 16 and 48 (the
tcgen05 dense projections), at KV context 1536.

Bounds are the reference's (``deepseek_v41/spec.py:287-318``, ``check_k1.py:305-330``): the
folded residual, the MXFP8 input of wqkv_a and the KV record bytes bit-exact; the seam's
gates (pre, post, comb) within 1e-6; q cos 0.99999 / rel 5e-3; the attention output cos
0.9998 (and rel 1e-3) against the exact oracle attention of the GPU's own q; wo_a rel 5e-3,
wo_b rel 1e-3; the FFN seam's gates rel 1e-4; router logits, routing ids and weights
bit-exact; the MoE partial cos 0.9999 / rel 1.5e-2. Each stage's oracle runs on the GPU's own
inputs to that stage. The attention's three 32-head producers -- records gathered by a CTA pair,
staged by bulk copies, or gathered by lone CTAs -- give the same bits; the 64-head CTAs (one f16
p instead of a head and tail) meet the same oracle bounds, and every later stage runs on their
output.
Every check runs and the failures are reported together.
"""

import pytest
import torch

from oracle import layer as OL
from oracle import numerics as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
CTX = 1536


def cos(a, b):
    return torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0).item()


def rel(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return ((a - b).norm() / b.norm()).item()


def maxabs(a, b):
    return (a.double() - b.double()).abs().max().item()


def cpu(d):
    return {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.items()}


class Checks:
    def __init__(self, what):
        self.what, self.failed, self.seen = what, [], {}

    def __call__(self, name, ok, value=None):
        self.seen[name] = value
        if not ok:
            self.failed.append(f"{name}: {value}")

    def done(self):
        print(f"\n{self.what}: " + ", ".join(f"{k}={v}" for k, v in self.seen.items()))
        assert not self.failed, f"{self.what}: " + "; ".join(self.failed)


@pytest.fixture(scope="module")
def layer2():
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner
    s = CONFIG2
    w = synth.make_layer(s, 5, DEV, positions=CTX + 8)
    r = MonoRunner(s, DEV)
    L = r.bind(w)
    W = cpu(w)
    yield s, r, L, W
    ext.set_option("attn_pair", 1)
    ext.set_option("attn_bulk", 0)
    ext.set_option("attn_wide", 1)


@pytest.mark.parametrize("M", [1, 16, 48])
def test_config2_stages(layer2, M):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    s, r, L, W = layer2
    step = synth.make_step(s, M, CTX, 900 + M, DEV)
    cache0 = step["cache"].clone()
    ext.set_option("attn_bulk", 0)
    ext.set_option("attn_pair", 1)
    ext.set_option("attn_wide", 0)
    b = r.k1(L, step, M)
    r.k2(L, step, M, b)
    torch.cuda.synchronize()
    pair = cpu(b)
    # the same K2 with the other 32-head producers: records staged by bulk copies, then gathered
    # by lone CTAs
    ext.set_option("attn_bulk", 1)
    r.k2(L, step, M, b)
    torch.cuda.synchronize()
    staged = cpu(b)
    ext.set_option("attn_bulk", 0)
    ext.set_option("attn_pair", 0)
    r.k2(L, step, M, b)
    torch.cuda.synchronize()
    lone = cpu(b)
    ext.set_option("attn_pair", 1)
    # the default at 64 heads, the one bench.py times: the 64-head CTAs (one f16 p); every stage
    # below checks this run
    ext.set_option("attn_wide", 1)
    r.k2(L, step, M, b)
    torch.cuda.synchronize()
    B = cpu(b)
    assert ext.lib().dsv41_device_error() == 0
    S = cpu(step)
    H, QL, D, nope = s.hidden, s.q_lora, s.head_dim, s.nope
    cs = W["cos_sin"][S["pos"]]
    cosv, sinv = cs[:, :32], cs[:, 32:]
    c = Checks(f"config2 M={M}")

    # ---- K1 seam: residual, normed, MXFP8 bit-exact; gates within 1e-6
    rn, normed, pre, post, comb = OL.seam(S["res"].float(), S["x"].float(), S["post"], S["comb"], S["pre"],
                                          W["hc_attn_fn"], W["hc_attn_scale"], W["hc_attn_base"], W["attn_norm"])
    c("res1 exact", torch.equal(B["res1"].float(), rn), maxabs(B["res1"], rn))
    c("normed exact", torch.equal(B["normed_a"].float(), normed), maxabs(B["normed_a"], normed))
    q8, q8s = N.mxfp8_quant(normed, "vllm")  # from the oracle's own normed row
    c("x8 exact", torch.equal(q8, B["x8"]) and torch.equal(q8s, B["x8s"]),
      int((q8 != B["x8"]).sum()) + int((q8s != B["x8s"]).sum()))
    gate = max(maxabs(B["pre_a"], pre), maxabs(B["post_a"], post), maxabs(B["comb_a"], comb))
    c("k1 gates max_abs <= 1e-6", gate <= 1e-6, gate)
    # ---- wqkv_a
    qkv = OL.gemv_x8_fp8(B["x8"], B["x8s"], W["wqkv"], W["wqkv_s"])
    c("wqkv rel < 1e-5", rel(B["qkv"], qkv) < 1e-5, rel(B["qkv"], qkv))
    # ---- the KV record: bit-exact
    nb, rb, codes = OL.kv_record(B["qkv"][:, QL:], W["kv_norm"], cosv, sinv, nope)
    data, sc = OL.record_bytes(nb, rb, codes, 8)
    ref_cache = cache0.cpu().clone()
    OL.write_records(ref_cache, S["slot"], data, sc, S["blk"])
    c("kv bytes exact", torch.equal(S["cache"], ref_cache), int((S["cache"] != ref_cache).sum()))
    # ---- q path, wq_b + RoPE (64 heads x 576)
    ys, qx8, qx8s = OL.q_path(B["qkv"][:, :QL], W["q_norm"])
    qr = rel(N.mxfp8_dequant(B["qx8"], B["qx8s"]), N.mxfp8_dequant(qx8, qx8s))
    c("q_norm mxfp8 rel < 4e-3", qr < 4e-3, qr)
    v = OL.bf(OL.gemv_x8_fp8(B["qx8"], B["qx8s"], W["wqb"], W["wqb_s"])).view(M, -1, D)
    q = OL.rope_q(v, cosv, sinv, nope)
    c("q cos/rel", cos(B["q"].float(), q) > 0.99999 and rel(B["q"].float(), q) < 5e-3,
      (cos(B["q"].float(), q), rel(B["q"].float(), q)))
    kt, klen = OL.key_table(S["slot"], S["swa_idx"], S["swa_lens"], None, torch.zeros(M, dtype=torch.int32),
                            S["swa_idx"].shape[1], 0)
    c("key table exact", torch.equal(B["kt"], kt) and torch.equal(B["klen"], klen))
    # ---- attention: the CTA pair, the lone CTAs, the exact oracle of the GPU's q
    xo = OL.attention(B["q"].float(), B["kt"], B["klen"], S["cache"], S["blk"], None, 1, W["sink"], cosv, sinv,
                      nope, s.rope, 8)
    gx = B["xo"].float()
    c("attention (64-head CTAs) cos >= 0.9998, rel < 1e-3", cos(gx, xo) >= 0.9998 and rel(gx, xo) < 1e-3,
      (cos(gx, xo), rel(gx, xo)))
    px = pair["xo"].float()
    c("attention (CTA pair) cos >= 0.9998, rel < 1e-3", cos(px, xo) >= 0.9998 and rel(px, xo) < 1e-3,
      (cos(px, xo), rel(px, xo)))
    for name, other in (("staged", staged), ("lone", lone)):
        c(f"pair == {name} CTAs", torch.equal(pair["xo"], other["xo"]) and torch.equal(pair["out"], other["out"]),
          maxabs(pair["xo"], other["xo"]))
    # ---- wo_a -> X8B, wo_b
    _, x8b, x8bs = OL.wo_a(gx, W["woa"], W["woa_s"], s.groups_local, s.o_rank)
    wr = rel(N.mxfp8_dequant(B["x8b"], B["x8bs"]), N.mxfp8_dequant(x8b, x8bs))
    c("wo_a rel < 5e-3", wr < 5e-3, wr)
    part = OL.wo_b(B["x8b"], B["x8bs"], W["wob"], W["wob_s"])
    c("wo_b rel < 1e-3", rel(B["attn_part"].float(), part) < 1e-3, rel(B["attn_part"].float(), part))
    # ---- FFN seam from the GPU's own attention output and K1 state: residual and normed exact
    rn2, normed2, pre2, post2, comb2 = OL.seam(B["res1"].float(), B["attn"].float(), B["post_a"], B["comb_a"],
                                               B["pre_a"], W["hc_ffn_fn"], W["hc_ffn_scale"], W["hc_ffn_base"],
                                               W["ffn_norm"])
    c("res2 exact", torch.equal(B["res2"].float(), rn2), maxabs(B["res2"], rn2))
    c("normed_f exact", torch.equal(B["normed_f"].float(), normed2), maxabs(B["normed_f"], normed2))
    fm = max(rel(B["pre_f"], pre2), rel(B["post_f"], post2), rel(B["comb_f"], comb2))
    c("ffn gates rel < 1e-4", fm < 1e-4, fm)
    # ---- router logits and routing: bit-exact (256 experts, top-8, sqrtsoftplus + bias)
    logits = OL.router_logits(B["normed_f"].float(), W["gate_w"])
    c("router logits exact", torch.equal(B["logits"], logits), maxabs(B["logits"], logits))
    ids, wts = OL.route(B["logits"], W.get("bias"), s.topk, s.route)
    c("ids exact", torch.equal(B["ids"], ids))
    c("weights exact", torch.equal(B["wts"], wts))
    # ---- the MoE partial (shared + routed over the GPU's routing)
    moe, _, _, _ = OL.moe_partial(B["normed_f"].float(), W, s.route, s.topk)
    mo = B["out"].float()
    c("moe cos/rel", cos(mo, moe) > 0.9999 and rel(mo, moe) < 0.015, (cos(mo, moe), rel(mo, moe)))
    c.done()


@pytest.mark.parametrize("M", [1, 8, 15])
def test_k1_persistent_equals_launch_sequence(layer2, M):
    """K1 as one persistent launch (M below the tcgen05 dense threshold) against K1's seven
    launches: every output bit for bit (the same stage functions, in the same order)."""
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    s, r, L, W = layer2
    step = synth.make_step(s, M, CTX, 700 + M, DEV)
    cache0 = step["cache"].clone()
    keys = ("res1", "post_a", "comb_a", "pre_a", "normed_a", "x8", "x8s", "qkv", "q", "qx8", "qx8s", "kt", "klen")
    outs = {}
    for persistent in (1, 0):
        ext.set_option("k1_persistent", persistent)
        step["cache"].copy_(cache0)
        b = r.k1(L, step, M)
        torch.cuda.synchronize()
        outs[persistent] = {k: b[k].clone() for k in keys}
        outs[persistent]["cache"] = step["cache"].clone()
    ext.set_option("k1_persistent", 0)
    assert ext.lib().dsv41_device_error() == 0
    for k in keys + ("cache",):
        assert torch.equal(outs[1][k], outs[0][k]), k
