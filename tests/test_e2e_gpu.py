"""The north star's end-to-end criterion, measured as written: a chain of decode layers on the GPU
(K1 + K2 of each, layer j + 1 fed by layer j's outputs, every layer with its own KV cache)
against a fully independent oracle run of the same chain from the same inputs -- nothing of
the GPU's fed back into the oracle -- then the head (the last layer's pending post folded,
the copies collapsed with its pre, an RMSNorm) and the 129280-token LM head with its argmax
(``dsv41_lmhead_argmax``) on the GPU against the oracle's fp64 logits.

Reported and bounded: the hidden state (the folded residual stream after each layer, and the
head's normed input) within max-abs 2e-2 of the oracle's RMS; the logits within max-abs 2e-2
of their RMS; the greedy next-token ids equal on >= 99.5 % of rows (BASELINE config 1
shapes, 3 layers, 5 steps of 48 rows: 240 rows).
"""

import pytest
import torch

from oracle import layer as OL

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
LAYERS, STEPS, M, CTX, VOCAB = 3, 5, 48, 256, 129280


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
    worst = {"hidden": 0.0, "head": 0.0, "logits": 0.0}
    same = total = 0
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
            worst["hidden"] = max(worst["hidden"], (hg - ho).abs().max().item() / rms)
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
    print(f"\nchain of {LAYERS} layers, {total} rows: max-abs/RMS hidden {worst['hidden']:.3e}, "
          f"head input {worst['head']:.3e}, logits {worst['logits']:.3e}; greedy ids agree {agree:.4f}")
    assert worst["hidden"] <= 2e-2, worst
    assert worst["head"] <= 2e-2, worst
    assert worst["logits"] <= 2e-2, worst
    assert agree >= 0.995, agree
