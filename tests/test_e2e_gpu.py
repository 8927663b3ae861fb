"""The north star's end-to-end criterion, measured as written: a chain of decode layers on the GPU
(K1 + K2 of each, layer j + 1 fed by layer j's outputs, every layer with its own KV cache), then
the head (the last layer's pending post folded, the copies collapsed with its pre, an RMSNorm)
and the 129280-token LM head with its argmax (``dsv41_lmhead_argmax``).

Two oracles run beside it. Per layer, the oracle runs the whole layer from the GPU's own inputs
to that layer (the reference's per-launch comparison, ``deepseek_v41/spec.py:287-318``): the
layer's hidden state -- the residual stream with its MoE output folded in -- must be within
max-abs 2e-2 of the oracle's RMS on >= 99 % of the rows the two route alike and within 5e-2 on
all of them, and at most 1 % of rows may route differently. (Measured: 11 rows in 1440 pass
2e-2, the largest 2.8e-2. The attention output agrees with the exact one to ~5e-5 relative -- the tensor core's
fp32 accumulation truncates -- so ~1 % of its bf16 outputs land one rounding step apart; wo_a's
output is requantized to MXFP8, where such a step can move an element to the next e4m3 code, an
eighth of its value; a row with a few such moves in large elements carries them into its hidden
state.) (The router sees the layer's attention output, bf16 after an MXFP8
requantization: the GPU's and the oracle's agree to ~1e-6 before rounding, yet a row whose 8th
and 9th expert scores lie that close can pick another expert, and then its MoE output differs
by that expert's whole contribution.) End to end, a fully independent oracle runs the chain from
the same first inputs, nothing of the GPU's fed back: the greedy next-token ids must agree on
>= 99.5 % of rows (BASELINE config 1 shapes, 3 layers, 10 steps of 48 rows: 480 rows). The
independent chain's hidden-state and logit max-abs are reported, not bounded: they grow layer
by layer, because each layer requantizes its bf16 attention output and its normed input to
MXFP8 -- one bf16 step in an element can move it to the next e4m3 code -- and a differently
routed row carries its difference into every later layer.
"""

import pytest
import torch

from oracle import layer as OL

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
LAYERS, STEPS, M, CTX, VOCAB = 3, 10, 48, 256, 129280


def cpu(d):
    return {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.items()}


def head_input(res, out, post, comb, pre, norm_w):
    """The model head's input from the last layer's outputs: its pending post folded into the
    residual copies, the copies collapsed with its pre (h in order), RMSNorm (fp32, eps 1e-20)."""
    rn = OL.fold_post(res.float(), out.float(), post, comb)
    acc = torch.zeros(rn.shape[0], rn.shape[2])
    for h in range(rn.shape[1]):
        acc = acc + pre[:, h, None].float() * rn[:, h, :]
    lin = OL.bf(acc)
    r = 1.0 / torch.sqrt(OL.seam_sumsq(lin).float() / float(lin.shape[1]) + OL.RMS_EPS)
    return rn, OL.bf((lin * r[:, None]) * norm_w.float())


def test_layer_chain_hidden_logits_and_greedy_ids():
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG1
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner
    s = CONFIG1
    Ws = [synth.make_layer(s, 40 + j, "cpu", positions=CTX + 8) for j in range(LAYERS)]
    r = MonoRunner(s, DEV)
    Ls = [r.bind({k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in w.items()}, tag=f"l{j}")
          for j, w in enumerate(Ws)]
    g = torch.Generator().manual_seed(77)
    head_w = (torch.randn(VOCAB, s.hidden, generator=g) * 0.02).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(s.hidden, generator=g)).to(torch.bfloat16)
    head_dev = head_w.to(DEV)
    worst = {"layer": 0.0, "layer_all_rows": 0.0, "hidden": 0.0, "head": 0.0, "logits": 0.0}
    over = 0  # rows routed alike whose hidden state is beyond 2e-2 x RMS
    chain_by_layer = [0.0] * LAYERS
    same = total = flips = layer_flips = layer_rows = 0
    for t in range(STEPS):
        steps = [synth.make_step(s, M, CTX, 500 + 10 * t + j, "cpu") for j in range(LAYERS)]
        # ---- GPU chain
        b = None
        for j, st in enumerate(steps):
            sd = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in st.items()}
            if j > 0:
                sd = dict(sd, res=b["res2"], x=b["out"], post=b["post_f"], comb=b["comb_f"], pre=b["pre_f"])
            b = r.k1(Ls[j], sd, M)
            r.k2(Ls[j], sd, M, b)
            torch.cuda.synchronize()
            # ---- the oracle's own chain, layer by layer beside it
            if j == 0:
                so = st
            else:
                so = dict(st, res=ref["res2"], x=ref["out"], post=ref["post2"], comb=ref["comb2"], pre=ref["pre2"])
            ref = OL.decode_layer([Ws[j]], so, s)
            B = cpu(b)
            hg = OL.fold_post(B["res2"].float(), B["out"].float(), B["post_f"], B["comb_f"])
            ho = OL.fold_post(ref["res2"].float(), ref["out"].float(), ref["post2"], ref["comb2"])
            rms = ho.pow(2).mean().sqrt().item()
            e = (hg - ho).abs().max().item() / rms
            worst["hidden"] = max(worst["hidden"], e)
            chain_by_layer[j] = max(chain_by_layer[j], e)
            flips += int((B["ids"].sort(1).values != ref["ids"].sort(1).values).any(1).sum())
            # the same layer from the GPU's own inputs to it
            sg = dict(st) if j == 0 else dict(st, res=prev["res2"], x=prev["out"], post=prev["post_f"],
                                              comb=prev["comb_f"], pre=prev["pre_f"])
            one = OL.decode_layer([Ws[j]], sg, s)
            h1 = OL.fold_post(one["res2"].float(), one["out"].float(), one["post2"], one["comb2"])
            rms1 = h1.pow(2).mean().sqrt().item()
            alike = (B["ids"].sort(1).values == one["ids"].sort(1).values).all(1)
            per_row = (hg - h1).abs().flatten(1).amax(1) / rms1
            worst["layer_all_rows"] = max(worst["layer_all_rows"], per_row.max().item())
            if bool(alike.any()):
                worst["layer"] = max(worst["layer"], per_row[alike].max().item())
                over += int((per_row[alike] > 2e-2).sum())
            layer_flips += int((~alike).sum())
            layer_rows += M
            prev = B
        # ---- the head on the GPU's outputs and on the oracle's
        _, xg = head_input(B["res2"], B["out"], B["post_f"], B["comb_f"], B["pre_f"], norm_w)
        _, xo = head_input(ref["res2"], ref["out"], ref["post2"], ref["comb2"], ref["pre2"], norm_w)
        worst["head"] = max(worst["head"], (xg - xo).abs().max().item() / xo.pow(2).mean().sqrt().item())
        best = torch.empty(M, dtype=torch.int64, device=DEV)
        logits = torch.empty(M, VOCAB, dtype=torch.float32, device=DEV)
        xg_dev = xg.to(torch.bfloat16).to(DEV)
        a = abi.LmHeadArgs(M=M, V=VOCAB, K=s.hidden, vbase=0, w=head_dev.data_ptr(), x=xg_dev.data_ptr(),
                           logits=logits.data_ptr(), best=best.data_ptr(), init=1)
        ext.call("dsv41_lmhead_argmax", a, torch.cuda.current_stream().cuda_stream)
        ids = torch.empty(M, dtype=torch.int32, device=DEV)
        d = abi.ArgmaxArgs(M=M, best=best.data_ptr(), ids=ids.data_ptr(), vals=0, draft=0, per_req=1, accept=0,
                           next_tok=0)
        ext.call("dsv41_argmax_decode", d, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        ref_logits, ref_ids = OL.lm_head_argmax(xo, head_w)
        lg = logits.cpu()
        worst["logits"] = max(worst["logits"],
                              (lg - ref_logits).abs().max().item() / ref_logits.pow(2).mean().sqrt().item())
        same += int((ids.cpu() == ref_ids).sum())
        total += M
    agree = same / total
    print(f"\nper layer from its own inputs: max-abs/RMS {worst['layer']:.3e} on rows routed alike, "
          f"{over} of them beyond 2e-2 "
          f"({worst['layer_all_rows']:.3e} on all), {layer_flips} of {layer_rows} rows routed differently; "
          f"independent chain of {LAYERS} "
          f"layers, {total} rows: hidden {worst['hidden']:.3e} (by layer "
          f"{', '.join(f'{v:.2e}' for v in chain_by_layer)}), head input {worst['head']:.3e}, logits "
          f"{worst['logits']:.3e}, rows routed differently {flips}; greedy ids agree {agree:.4f}")
    assert over <= 0.01 * layer_rows and worst["layer"] <= 5e-2, (over, worst)
    assert layer_flips <= 0.01 * layer_rows, (layer_flips, layer_rows)
    assert agree >= 0.995, agree
