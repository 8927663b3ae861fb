"""K2i and the index selection on the GPU against the oracle: the device walk plan equals the
host plan (the reference's own fixtures, and seeded steps); the FP4 index logits are
bit-identical to the oracle's contract (and within 1e-6 of the reference's fp64 logits); the
top-k (ties to the lower position), the candidate blocks and the REINDEX candidate pipeline
are exact. ``test_deepseek_v41_k2i.py`` and ``test_deepseek_v41_index_plan.py`` of the
reference are the model."""

import numpy as np
import pytest
import torch

from oracle import indexer as OI

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _runner(bound_max=1 << 15, topk=512, ctas=None):
    from sgl_amd_mono_b200.deepseek_v41.sm100a.indexer import K2iRunner
    return K2iRunner(DEV, bound_max, topk=topk, ctas=ctas)


def fp4_case(ctxs, per_req, heads, seed):
    """Synthetic FP4 index inputs in SGLang's layouts (``test_deepseek_v41_k2i.py:107-134``):
    request r sees ctxs[r] columns on its last row (one fewer each row before)."""
    g = torch.Generator().manual_seed(seed)
    rows = len(ctxs) * per_req
    ppr = -(-max(ctxs) // 64)
    pages = len(ctxs) * ppr + 3
    u8 = dict(generator=g, dtype=torch.uint8)
    payload = torch.randint(0, 256, (pages, 1, 4, 64, 16), **u8)
    kscale = torch.randint(123, 130, (pages, 1, 4, 64), **u8)
    perm = torch.randperm(pages, generator=g).to(torch.int32)
    table = perm[: len(ctxs) * ppr].view(len(ctxs), ppr).repeat_interleave(per_req, 0).contiguous()
    q = torch.randint(0, 256, (rows, heads, 64), **u8)
    qscale = torch.randint(123, 130, (rows, 1, 4, 16, 4), **u8)
    w = (torch.randn(rows, heads, generator=g) * 0.05).to(torch.bfloat16)
    bounds = torch.tensor([max(c - (per_req - 1 - i), 0) for c in ctxs for i in range(per_req)], dtype=torch.int32)
    return dict(q=q, qscale=qscale, w=w, payload=payload, kscale=kscale, table=table, bounds=bounds)


def _gpu(case):
    return {k: v.to(DEV) for k, v in case.items()}


def test_walk_plan_device_equals_reference_plans(golden):
    r = _runner(ctas=256)
    for bounds, owners, plan in golden("walk_plan")["plans"]:
        n = bounds.shape[0]
        # the fixture's owners are arbitrary runs: pass them through the runner's owner table
        r.owners[0, :n] = torch.from_numpy(owners.astype(np.int32)).to(DEV)
        got = r.walk_plan(ratio=1, bounds=torch.from_numpy(bounds.astype(np.int32)).to(DEV), rows=n, per_req=1)
        assert np.array_equal(got.cpu().numpy(), plan), (bounds, owners)
    r.owners[0] = torch.arange(48, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("seed", range(3))
def test_walk_plan_device_equals_host_b200_grid(seed):
    rng = np.random.default_rng(seed)
    r = _runner()
    for _ in range(60):
        per_req = int(rng.choice([1, 2, 4, 6]))
        n = per_req * int(rng.integers(1, 48 // per_req + 1))
        ctx = rng.integers(0, 1 << 16, size=n // per_req)
        bounds = np.array([max(int(c) - (per_req - 1 - i), 0) for c in ctx for i in range(per_req)], np.int32)
        owners = (np.arange(n) // per_req * per_req).astype(np.int32)
        got = r.walk_plan(ratio=2, bounds=torch.from_numpy(bounds).to(DEV), rows=n, per_req=per_req)
        want = OI.fill_walk_plan(bounds, owners, r.ctas)
        assert np.array_equal(got.cpu().numpy(), want)


def _logits_case(case, per_req, topk_plan):
    r = _runner(topk=topk_plan)
    c = _gpu(case)
    rows = c["q"].shape[0]
    r.walk_plan(ratio=1, bounds=c["bounds"], rows=rows, per_req=per_req)
    lg = r.score(rows=rows, per_req=per_req, ratio=1, query=(c["q"], c["qscale"], c["w"]),
                 plane=(c["payload"], c["kscale"]), page_table=c["table"], bounds=c["bounds"])
    torch.cuda.synchronize()
    return lg.cpu()


def test_index_logits_golden_case_bit_exact(golden):
    g = golden("k2i")
    case = {k: g["case"][k] for k in ("q", "qscale", "w", "payload", "kscale", "table", "bounds")}
    lg = _logits_case(case, g["case"]["per_req"], topk_plan=0)
    for t, ref in enumerate(g["logits"]):
        n = ref.numel()
        if n == 0:
            continue
        want = OI.index_logits(case["q"], case["qscale"], case["w"], case["payload"], case["kscale"],
                               case["table"], t, torch.arange(n))
        assert torch.equal(lg[t, :n], want), (t, (lg[t, :n] - want).abs().max().item())
        assert ((lg[t, :n].double() - ref).abs().max() / ref.abs().max()).item() < 1e-6


@pytest.mark.parametrize("heads,ctxs,per_req", [(64, [4096, 1000, 2500], 2), (32, [700, 3000], 6)])
def test_index_logits_bit_exact(heads, ctxs, per_req):
    case = fp4_case(ctxs, per_req, heads, seed=heads + per_req)
    lg = _logits_case(case, per_req, topk_plan=0)
    for t in range(case["q"].shape[0]):
        n = int(case["bounds"][t])
        want = OI.index_logits(case["q"], case["qscale"], case["w"], case["payload"], case["kscale"],
                               case["table"], t, torch.arange(n))
        assert torch.equal(lg[t, :n], want), t


def quantized_case(ctxs, per_req, heads, seed, spread_keys=0):
    """fp4_case's layouts with SGLang-like MXFP4 data: N(0, 1) keys and queries quantized per 32
    dims (small code spreads: the tensor-core scorer's folded-scale tiles). ``spread_keys`` keys
    get one chunk's code raised by 9, so their 128-key tiles take the per-chunk path."""
    from sgl_amd_mono_b200.deepseek_v41 import quant
    case = fp4_case(ctxs, per_req, heads, seed)
    g = torch.Generator().manual_seed(seed + 1000)
    pages = case["payload"].shape[0]
    packed, codes = quant.quant_mxfp4(torch.randn(pages * 64, 128, generator=g))
    case["payload"] = packed.view(pages, 64, 4, 16).permute(0, 2, 1, 3).contiguous().view(pages, 1, 4, 64, 16)
    slot = torch.arange(64)
    ks = torch.empty(pages, 1, 4, 64, dtype=torch.uint8)
    ks[:, 0, :, (slot % 16) * 4 + slot // 16] = codes.view(pages, 64, 4).permute(0, 2, 1)
    for _ in range(spread_keys):
        p, s = int(torch.randint(0, pages, (1,), generator=g)), int(torch.randint(0, 64, (1,), generator=g))
        ks[p, 0, 1, (s % 16) * 4 + s // 16] += 9
    case["kscale"] = ks
    rows = case["q"].shape[0]
    qp, qc = quant.quant_mxfp4(torch.randn(rows * heads, 128, generator=g))
    case["q"] = qp.view(rows, heads, 64).contiguous()
    qs = torch.zeros(rows, 1, 4, 16, 4, dtype=torch.uint8)
    h = torch.arange(heads)
    qs[:, 0, :, h % 16, h // 16] = qc.view(rows, heads, 4).permute(0, 2, 1)
    case["qscale"] = qs
    return case


@pytest.mark.parametrize("heads,ctxs,per_req,spread", [(64, [5000, 2100], 1, 0), (64, [3000, 700], 3, 0),
                                                        (32, [4100, 1900], 2, 0), (64, [6000, 2500], 2, 12)])
def test_index_logits_quantized_bit_exact(heads, ctxs, per_req, spread):
    """Folded-scale tiles (and, with spread keys, per-chunk tiles among them) equal the contract."""
    case = quantized_case(ctxs, per_req, heads, seed=heads + per_req + spread, spread_keys=spread)
    lg = _logits_case(case, per_req, topk_plan=0)
    for t in range(case["q"].shape[0]):
        n = int(case["bounds"][t])
        want = OI.index_logits(case["q"], case["qscale"], case["w"], case["payload"], case["kscale"],
                               case["table"], t, torch.arange(n))
        assert torch.equal(lg[t, :n], want), (t, (lg[t, :n] - want).abs().max().item())


def test_topk_ties_and_pages():
    g = torch.Generator().manual_seed(5)
    rows, width, k = 6, 5000, 512
    vals = torch.randint(-40, 40, (rows, width), generator=g).float() / 8  # many exact ties
    n = torch.tensor([5000, 512, 100, 4999, 513, 0], dtype=torch.int32)
    table = torch.randperm(600, generator=g)[: rows * 80].view(rows, 80).to(torch.int32)
    owners = torch.arange(rows, dtype=torch.int32)
    r = _runner()
    out = torch.empty(rows, k, dtype=torch.int32, device=DEV)
    pages = torch.empty_like(out)
    r.topk_of(vals.to(DEV), n.to(DEV), k, out, page_out=pages, table=table.to(DEV), owners=owners.to(DEV))
    torch.cuda.synchronize()
    for t in range(rows):
        want = OI.topk_rows(vals[t], int(n[t]), k)
        assert torch.equal(out[t].cpu(), want), t
        assert torch.equal(pages[t].cpu(), OI.page_indices(want, table[t], 64)), t


def test_candidate_blocks_and_reindex_pipeline():
    heads, per_req = 32, 2
    case = fp4_case([20000, 17000], per_req, heads, seed=9)
    rows = case["q"].shape[0]
    r = _runner()
    c = _gpu(case)
    r.walk_plan(ratio=1, bounds=c["bounds"], rows=rows, per_req=per_req)
    raw = torch.empty(rows, 512, dtype=torch.int32, device=DEV)
    page = torch.empty_like(raw)
    query, plane = (c["q"], c["qscale"], c["w"]), (c["payload"], c["kscale"])
    cand = r.select(kind="producer", rows=rows, per_req=per_req, ratio=1, query=query, plane=plane,
                    page_table=c["table"], bounds=c["bounds"], raw_out=raw, page_out=page)
    torch.cuda.synchronize()
    lg = r.ilog[: rows * c["table"].shape[1] * 64].view(rows, -1).cpu()
    for t in range(rows):
        n = int(case["bounds"][t])
        assert torch.equal(cand.ids[t].cpu(), OI.candidate_blocks(lg[t], n)), t
        want = OI.topk_rows(lg[t], n, 512)
        assert torch.equal(raw[t].cpu(), want), t
        assert torch.equal(page[t].cpu(), OI.page_indices(want, case["table"][t], 64)), t
    # a consumer layer (another query) reads only the producer's candidate blocks
    g2 = torch.Generator().manual_seed(10)
    q2 = torch.randint(0, 256, case["q"].shape, generator=g2, dtype=torch.uint8)
    w2 = (torch.randn(rows, heads, generator=g2) * 0.05).to(torch.bfloat16)
    ids_in = cand.ids.clone()
    raw2 = torch.empty_like(raw)
    page2 = torch.empty_like(raw)
    r.select(kind="reindex", rows=rows, per_req=per_req, ratio=1, query=(q2.to(DEV), c["qscale"], w2.to(DEV)),
             plane=plane, page_table=c["table"], bounds=c["bounds"], raw_out=raw2, page_out=page2,
             candidates=type(cand)(ids_in))
    torch.cuda.synchronize()
    for t in range(rows):
        owner = t // per_req * per_req
        ids_o, tab_o, ctx_o = OI.reindex_table(ids_in[t].cpu(), case["table"][owner], int(case["bounds"][t]))
        assert torch.equal(r.cand_ids[t].cpu(), ids_o) and int(r.cand_bound[t]) == ctx_o, t
        assert torch.equal(r.cand_table[t].cpu(), tab_o), t
        comp = OI.index_logits(q2, case["qscale"], w2, case["payload"], case["kscale"],
                               tab_o[None].expand(rows, -1), t, torch.arange(ctx_o), entry_rows=8)
        sel = OI.topk_rows(comp, ctx_o, 512)
        want_raw, want_page = OI.map_compact(sel, ids_o, case["table"][owner])
        assert torch.equal(raw2[t].cpu(), want_raw), t
        assert torch.equal(page2[t].cpu(), want_page), t
