"""Seeded synthetic layers and decode steps with the BASELINE configs' shapes and value
distributions (random-init weights; no checkpoint or dataset is available here).

Weights: N(0, 0.02) quantized to MXFP4 for the routed experts, FP8 e4m3
with power-of-two 128 x 128 block scales for the dense projections and the shared expert;
router gate N(0, 0.02) bf16, router bias N(0, 0.02) (kept in bf16 by SGLang, widened to
fp32); mHC weights as the reference's kernel test draws them (``check_ffn.py:129-184``).
Steps: residual streams with unit-RMS rows, N(0, 1) bf16 activations, Sinkhorn-normalized
comb, and a paged FP8 KV cache prefilled from N(0, 1) rows.
"""

from __future__ import annotations

import torch

from . import quant
from .shapes import HC, LayerShape

MIX = HC * (HC + 2)


def _rng(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def rope_table(positions: int, rope: int, device, theta: float = 10000.0) -> torch.Tensor:
    """[positions, rope] fp32: rope/2 cos, then rope/2 sin (``weights.py:34-43``)."""
    half = rope // 2
    j = torch.arange(half, device=device, dtype=torch.float64)
    ang = torch.arange(positions, device=device, dtype=torch.float64)[:, None] * theta ** (-j / half)
    return torch.cat([ang.cos(), ang.sin()], -1).float().contiguous()


def _fp8(n, k, g, device, std=0.02):
    return quant.quant_fp8_block(torch.randn(n, k, generator=g, device=device) * std)


def make_layer(s: LayerShape, seed: int, device, positions: int = 65536, rank: int = 0) -> dict:
    """One layer's weights for TP rank ``rank`` of ``s.tp`` (full tensors drawn with the seed,
    then this rank's shard sliced, so every rank sees one model)."""
    g = _rng(seed, device)
    H, D, tp = s.hidden, s.head_dim, s.tp
    w: dict = {}
    for seam in ("attn", "ffn"):
        w[f"hc_{seam}_fn"] = torch.randn(MIX, HC * H, generator=g, device=device) * 0.01
        w[f"hc_{seam}_scale"] = torch.randn(3, generator=g, device=device).abs() * 0.5 + 0.5
        w[f"hc_{seam}_base"] = torch.randn(MIX, generator=g, device=device) * 0.1
        w[f"{seam}_norm"] = (1 + 0.1 * torch.randn(H, generator=g, device=device)).to(torch.bfloat16)
    w["wqkv"], w["wqkv_s"] = _fp8(s.q_lora + D, H, g, device)
    w["q_norm"] = (1 + 0.1 * torch.randn(s.q_lora, generator=g, device=device)).to(torch.bfloat16)
    w["kv_norm"] = (1 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
    hl = s.heads_local
    wqb, wqbs = _fp8(s.heads * D, s.q_lora, g, device)
    w["wqb"], w["wqb_s"] = _rows(wqb, wqbs, rank * hl * D, hl * D)
    sink = torch.randn(s.heads, generator=g, device=device)
    w["sink"] = sink[rank * hl:(rank + 1) * hl].contiguous()
    gl, O = s.groups_local, s.o_rank
    woa, woas = _fp8(s.o_groups * O, s.group_k, g, device)
    w["woa"], w["woa_s"] = _rows(woa, woas, rank * gl * O, gl * O)
    wob, wobs = _fp8(H, s.o_groups * O, g, device)
    w["wob"], w["wob_s"] = _cols(wob, wobs, rank * gl * O, gl * O)
    w["gate_w"] = (torch.randn(s.experts, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    w["bias"] = (torch.randn(s.experts, generator=g, device=device) * 0.02).to(torch.bfloat16).float()
    I, Il = s.inter, s.inter_local
    w13 = torch.empty(s.experts, 2 * Il, H // 2, dtype=torch.uint8, device=device)
    s13 = torch.empty(s.experts, 2 * Il, H // 32, dtype=torch.uint8, device=device)
    w2 = torch.empty(s.experts, H, Il // 2, dtype=torch.uint8, device=device)
    s2 = torch.empty(s.experts, H, Il // 32, dtype=torch.uint8, device=device)
    for e in range(s.experts):
        gu_p, gu_s = quant.quant_mxfp4(torch.randn(2 * I, H, generator=g, device=device) * 0.02)
        for half in range(2):
            src = slice(half * I + rank * Il, half * I + (rank + 1) * Il)
            w13[e, half * Il:(half + 1) * Il] = gu_p[src]
            s13[e, half * Il:(half + 1) * Il] = gu_s[src]
        d_p, d_s = quant.quant_mxfp4(torch.randn(H, I, generator=g, device=device) * 0.02)
        w2[e] = d_p[:, rank * Il // 2:(rank + 1) * Il // 2]
        s2[e] = d_s[:, rank * Il // 32:(rank + 1) * Il // 32]
    w["w13"], w["s13"], w["w2"], w["s2"] = w13, s13, w2, s2
    SI, SIl = s.shared_inter, s.shared_local
    sgu, sgus = _fp8(2 * SI, H, g, device)
    gate_r, gate_c = _rows(sgu, sgus, rank * SIl, SIl)
    up_r, up_c = _rows(sgu, sgus, SI + rank * SIl, SIl)
    w["sgu"] = torch.cat([gate_r, up_r]).contiguous()
    w["sgu_s"] = torch.cat([gate_c, up_c]).contiguous()
    sw2, sw2s = _fp8(H, SI, g, device)
    w["sw2"], w["sw2_s"] = _cols(sw2, sw2s, rank * SIl, SIl)
    w["cos_sin"] = rope_table(positions, s.rope, device)
    return w


def _rows(q, codes, r0, n):
    assert r0 % 128 == 0 and (n % 128 == 0 or r0 + n == q.shape[0])
    return q[r0:r0 + n].contiguous(), codes[r0 // 128:(r0 + n + 127) // 128].contiguous()


def _cols(q, codes, c0, n):
    assert c0 % 128 == 0 and n % 128 == 0
    return q[:, c0:c0 + n].contiguous(), codes[:, c0 // 128:(c0 + n) // 128].contiguous()


def make_step(s: LayerShape, M: int, ctx: int, seed: int, device, blk: int = 64, per_req: int = 1) -> dict:
    """A decode step of M rows, each its own request with ``ctx`` keys (the row's own token
    last), over a paged SWA-layout cache of ``blk``-slot pages scattered by a page table.
    The key table is the rows' window of ``ctx`` slots (K1 builds it). With ``per_req`` > 1,
    rows come in verify blocks: the per_req rows of a request share its cache and row j of the
    block sees the causal prefix ending at its own token, ctx - per_req + j + 1 keys."""
    if per_req > 1:
        return _make_verify_step(s, M, ctx, seed, device, blk, per_req)
    g = _rng(seed, device)
    H = s.hidden
    res = torch.randn(M, HC, H, generator=g, device=device)
    res = (res * torch.rsqrt(res.pow(2).mean(-1, keepdim=True))).to(torch.bfloat16)
    x = torch.randn(M, H, generator=g, device=device).to(torch.bfloat16)
    comb = torch.rand(M, HC, HC, generator=g, device=device) + 0.1
    for _ in range(20):
        comb = comb / comb.sum(-1, keepdim=True)
        comb = comb / comb.sum(-2, keepdim=True)
    post = torch.sigmoid(torch.randn(M, HC, generator=g, device=device)) * 2
    pre = torch.sigmoid(torch.randn(M, HC, generator=g, device=device)) + 1e-6
    pages_per_row = -(-ctx // blk)
    pages = M * pages_per_row
    perm = torch.randperm(pages, generator=g, device=device)
    page_table = perm.view(M, pages_per_row)
    posn = torch.arange(ctx, device=device)
    slots = (page_table[:, posn // blk] * blk + posn % blk).to(torch.int32)  # [M, ctx]
    data_b = s.record_data
    page_stride = -(-blk * (data_b + 8) // 16) * 16
    cache = torch.zeros(pages, page_stride, dtype=torch.uint8, device=device)
    # prefill every key but the row's own (K1 writes it)
    for t in range(M):
        e = torch.randn(ctx - 1, s.head_dim, generator=g, device=device)
        data, sc = quant.kv_records(e, s.nope)
        sl = slots[t, : ctx - 1].long()
        p, o = sl // blk, sl % blk
        col = o[:, None] * data_b + torch.arange(data_b, device=device)
        cache[p[:, None].expand_as(col), col] = data
        scol = blk * data_b + o[:, None] * 8 + torch.arange(8, device=device)
        cache[p[:, None].expand_as(scol), scol] = sc
    return dict(
        res=res, x=x.contiguous(), post=post.contiguous(), comb=comb.contiguous(), pre=pre.contiguous(),
        pos=torch.full((M,), ctx - 1, dtype=torch.int64, device=device),
        slot=slots[:, ctx - 1].long().contiguous(),
        swa_idx=slots.contiguous(), swa_lens=torch.full((M,), ctx, dtype=torch.int32, device=device),
        cache=cache, blk=blk, page_stride=page_stride, ctx=ctx,
    )


def _make_verify_step(s: LayerShape, M: int, ctx: int, seed: int, device, blk: int, per_req: int) -> dict:
    g = _rng(seed, device)
    H, R = s.hidden, M // per_req
    assert M % per_req == 0 and ctx >= per_req
    res = torch.randn(M, HC, H, generator=g, device=device)
    res = (res * torch.rsqrt(res.pow(2).mean(-1, keepdim=True))).to(torch.bfloat16)
    x = torch.randn(M, H, generator=g, device=device).to(torch.bfloat16)
    comb = torch.rand(M, HC, HC, generator=g, device=device) + 0.1
    for _ in range(20):
        comb = comb / comb.sum(-1, keepdim=True)
        comb = comb / comb.sum(-2, keepdim=True)
    post = torch.sigmoid(torch.randn(M, HC, generator=g, device=device)) * 2
    pre = torch.sigmoid(torch.randn(M, HC, generator=g, device=device)) + 1e-6
    ppr = -(-ctx // blk)
    page_table = torch.randperm(R * ppr, generator=g, device=device).view(R, ppr)
    posn = torch.arange(ctx, device=device)
    req_slots = (page_table[:, posn // blk] * blk + posn % blk).to(torch.int32)  # [R, ctx]
    slots = req_slots.repeat_interleave(per_req, 0)  # [M, ctx]
    j = torch.arange(M, device=device) % per_req
    lens = (ctx - per_req + j + 1).to(torch.int32)
    data_b = s.record_data
    page_stride = -(-blk * (data_b + 8) // 16) * 16
    cache = torch.zeros(R * ppr, page_stride, dtype=torch.uint8, device=device)
    # prefill every key before the block (K1 writes the block's own)
    for r in range(R):
        data, sc = quant.kv_records(torch.randn(ctx - per_req, s.head_dim, generator=g, device=device), s.nope)
        sl = req_slots[r, : ctx - per_req].long()
        p, o = sl // blk, sl % blk
        col = o[:, None] * data_b + torch.arange(data_b, device=device)
        cache[p[:, None].expand_as(col), col] = data
        scol = blk * data_b + o[:, None] * 8 + torch.arange(8, device=device)
        cache[p[:, None].expand_as(scol), scol] = sc
    pos = (lens - 1).long()
    return dict(
        res=res, x=x.contiguous(), post=post.contiguous(), comb=comb.contiguous(), pre=pre.contiguous(),
        pos=pos, slot=slots.gather(1, pos[:, None])[:, 0].long().contiguous(),
        swa_idx=slots.contiguous(), swa_lens=lens, cache=cache, blk=blk, page_stride=page_stride, ctx=ctx,
    )


def make_sparse(s: LayerShape, M: int, ctx: int, seed: int, device, index_heads: int = 64, blk: int = 64) -> dict:
    """BASELINE config 3's compressed side of a decode step, every row its own request with
    ``ctx`` compressed keys: the compressed KV cache (records of N(0, 1) rows in ``blk``-slot
    pages scattered by the request's page table), the FP4 index plane on the same page table
    (N(0, 1) keys of 128 dims as E2M1 + E8M0 per 32, SGLang's split layout), and the rows' FP4
    index queries (N(0, 1), ``index_heads`` heads) with N(0, 0.05) bf16 head weights."""
    g = _rng(seed, device)
    ppr = -(-ctx // blk)
    pages = M * ppr
    pt = torch.randperm(pages, generator=g, device=device).to(torch.int32).view(M, ppr).contiguous()
    data_b = s.record_data
    page_stride = -(-blk * (data_b + 8) // 16) * 16
    comp = torch.zeros(pages, page_stride, dtype=torch.uint8, device=device)
    posn = torch.arange(ctx, device=device)
    for t in range(M):
        data, sc = quant.kv_records(torch.randn(ctx, s.head_dim, generator=g, device=device), s.nope)
        sl = pt[t, posn // blk].long() * blk + posn % blk
        p, o = sl // blk, sl % blk
        col = o[:, None] * data_b + torch.arange(data_b, device=device)
        comp[p[:, None].expand_as(col), col] = data
        scol = blk * data_b + o[:, None] * 8 + torch.arange(8, device=device)
        comp[p[:, None].expand_as(scol), scol] = sc
    packed, codes = quant.quant_mxfp4(torch.randn(pages * blk, 128, generator=g, device=device))
    payload = packed.view(pages, blk, 4, 16).permute(0, 2, 1, 3).contiguous().view(pages, 1, 4, blk, 16)
    slot = torch.arange(blk, device=device)
    kscale = torch.empty(pages, 1, 4, blk, dtype=torch.uint8, device=device)
    kscale[:, 0, :, (slot % 16) * 4 + slot // 16] = codes.view(pages, blk, 4).permute(0, 2, 1)
    qp, qc = quant.quant_mxfp4(torch.randn(M * index_heads, 128, generator=g, device=device))
    qs = torch.zeros(M, 1, 4, 16, 4, dtype=torch.uint8, device=device)
    h = torch.arange(index_heads, device=device)
    qs[:, 0, :, h % 16, h // 16] = qc.view(M, index_heads, 4).permute(0, 2, 1)
    w = (torch.randn(M, index_heads, generator=g, device=device) * 0.05).to(torch.bfloat16)
    return dict(comp=comp, comp_blk=blk, page_table=pt, payload=payload, kscale=kscale,
                q=qp.view(M, index_heads, 64).contiguous(), qscale=qs, w=w,
                bounds=torch.full((M,), ctx, dtype=torch.int32, device=device))
