"""BASELINE config 3's pipeline on the GPU (at test size): K2i scores every row's compressed
keys from the FP4 index plane, the top-2048 (ties to the lower position) become the pool slots
K1 writes into K2's key table beside the SWA window, and K2 attends over both caches. Against
the oracle: the selection bit-exact, the step's KV record bytes exact, the reduced attention
output within 2e-2 x RMS + one bf16 step element-wise, and the MoE output within the reference's
ffn.moe.rel bound (1.5e-2) with identical routing (element-wise bounds stop at the MXFP8
requantization of the attention's bf16 output, where a one-step difference flips e4m3 codes)."""

import pytest
import torch

from oracle import indexer as OI
from oracle import layer as OL

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SMALL = dict(hidden=1024, heads=8, nope=512, rope=64, q_lora=256, o_groups=1, o_rank=1024, experts=16, topk=4,
             inter=512, shared_inter=512)


def _rel(got, ref, tol):
    got, ref = got.float().cpu(), ref.float()
    assert (got - ref).norm() / ref.norm() < tol


def _close(got, ref, tol=2e-2):
    got, ref = got.float().cpu(), ref.float()
    rms = ref.pow(2).mean().sqrt()
    ulp = torch.ldexp(torch.ones_like(ref), torch.frexp(ref.abs())[1] - 8)
    assert ((got - ref).abs() - ulp).clamp_min(0).max() <= tol * rms
    assert (got - ref).norm() / ref.norm() < 1e-2


@pytest.mark.parametrize("M,ctx,topk", [(4, 4096, 2048), (3, 1500, 2048)])
def test_k2i_topk_sparse_attention_layer(M, ctx, topk):
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    from sgl_amd_mono_b200.deepseek_v41.sm100a.indexer import K2iRunner
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner
    s = LayerShape(**SMALL)
    w = synth.make_layer(s, 71, "cpu", positions=512)
    S = synth.make_step(s, M, 128, 72, "cpu")
    sp = synth.make_sparse(s, M, ctx, 73, "cpu", index_heads=32)
    gpu = lambda d: {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}  # noqa: E731
    Sd, spd = gpu(S), gpu(sp)
    runner = MonoRunner(s, DEV)
    L = runner.bind(gpu(w))
    k2i = K2iRunner(DEV, ctx, topk=topk)
    k2i.walk_plan(ratio=1, bounds=spd["bounds"], rows=M, per_req=1)
    raw = torch.empty(M, topk, dtype=torch.int32, device=DEV)
    page = torch.empty_like(raw)
    k2i.select(kind="full", rows=M, per_req=1, ratio=1, query=(spd["q"], spd["qscale"], spd["w"]),
               plane=(spd["payload"], spd["kscale"]), page_table=spd["page_table"], bounds=spd["bounds"],
               raw_out=raw, page_out=page)
    lens = torch.clamp(spd["bounds"], max=topk).to(torch.int32)
    b = runner.k1(L, Sd, M, topk_width=topk, topk_idx=page, topk_lens=lens)
    runner.k2(L, Sd, M, b, comp=spd["comp"], comp_stride=spd["comp"].stride(0), comp_blk=sp["comp_blk"])
    torch.cuda.synchronize()
    # the selection, bit-exact
    for t in range(M):
        n = int(sp["bounds"][t])
        lg = OI.index_logits(sp["q"], sp["qscale"], sp["w"], sp["payload"], sp["kscale"], sp["page_table"], t,
                             torch.arange(n))
        want = OI.topk_rows(lg, n, topk)
        assert torch.equal(raw[t].cpu(), want), t
        assert torch.equal(page[t].cpu(), OI.page_indices(want, sp["page_table"][t], 64)), t
    # the layer over the window and the selected compressed keys
    ref = OL.decode_layer([w], S, s, topk=page.cpu(), topk_lens=lens.cpu(), comp=sp["comp"], comp_blk=sp["comp_blk"])
    assert torch.equal(Sd["cache"].cpu(), ref["cache"])
    assert int(b["klen"][:M].sum()) == int((lens + 128).sum())
    _close(b["attn"], ref["attn"])
    _rel(b["out"], ref["out"], 1.5e-2)
    assert torch.equal(b["ids"].cpu(), ref["ids"])


def test_verify_blocks_causal_layer():
    """BASELINE config 5's rows: verify blocks of 6 rows a request sharing its cache, row j
    seeing the causal prefix up to its own token (written by the same K1 launch)."""
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner
    s = LayerShape(**SMALL)
    M, P, ctx = 12, 6, 700
    w = synth.make_layer(s, 81, "cpu", positions=ctx + 8)
    S = synth.make_step(s, M, ctx, 82, "cpu", per_req=P)
    gpu = lambda d: {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}  # noqa: E731
    Sd = gpu(S)
    runner = MonoRunner(s, DEV)
    L = runner.bind(gpu(w))
    b = runner.k1(L, Sd, M)
    runner.k2(L, Sd, M, b)
    torch.cuda.synchronize()
    ref = OL.decode_layer([w], S, s)
    assert torch.equal(Sd["cache"].cpu(), ref["cache"])
    assert b["klen"][:M].tolist() == S["swa_lens"].tolist()
    _close(b["attn"], ref["attn"])
    _rel(b["out"], ref["out"], 1.5e-2)
