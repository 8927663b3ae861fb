"""CPU restatement of one DeepSeek-V4.1 decoder layer's decode step (oracle; tests only).

Stage by stage, in the order the kernels run them (K1, then K2). Each function takes
and returns CPU tensors; "bf16-valued" fp32 tensors hold values already rounded to
bf16. Integer / byte outputs (KV records, routing ids) follow the bit-exact contracts
stated in each docstring, which the CUDA kernels implement identically. Citations
are to omirosh/sgl-amd-mono.
"""

from __future__ import annotations

import numpy as np
import torch

from . import numerics as N

HC = 4
MIX = HC * (HC + 2)  # 24 mix projections: pre 4 | post 4 | comb 16
RMS_EPS = 1e-20
HC_EPS = 1e-6
SINKHORN = 20
LIMIT = 10.0  # swiglu_limit
ROUTE_SCALE = 1.5  # routed_scaling_factor


def bf(x):
    return N.bf16_round(x)


def f32(x):
    return x.to(torch.float32)


# ---------------------------------------------------------------- mHC seam
def fold_post(res, x, post, comb):
    """The pending post folded into the residual (``seam.py:137-157``): R_new[o] =
    bf16(fma(c3 r3, ((post x + r0 c0) + c1 r1) + c2 r2)), res [M, HC, H], x [M, H]."""
    res, x, c = f32(res), f32(x), f32(comb)
    v = f32(post)[:, :, None] * x[:, None, :] + res[:, 0:1, :] * c[:, 0, :, None]
    v = v + c[:, 1, :, None] * res[:, 1:2, :]
    v = v + c[:, 2, :, None] * res[:, 2:3, :]
    # the last term as one fused multiply-add: the exact product plus v, rounded once
    v = N.fma_f32(c[:, 3, :, None], res[:, 3:4, :], v)
    return bf(v)


def seam(res, x, post, comb, pre_prev, hc_fn, hc_scale, hc_base, norm_w, *, fold=True,
         first=False):
    """One hyper-connection boundary (``seam.py:137-378``).

    res [M, HC, H] bf16-valued; x [M, H] bf16-valued (the pending sublayer output);
    post [M, HC], comb [M, HC(src), HC(dst)], pre_prev [M, HC] fp32.
    R_new[o] = bf16(fma(c3 r3, ((post x + r0 c0) + c1 r1) + c2 r2)) when a post is owed
    (``fold``), else R (``seam.py:137-157``); the layer input collapses R_new with the
    previous pre (copy 0 on the first layer, ``check_k1.py:228-245``); 24 mixes and the
    sum of squares of R_new feed the gate (sigmoid pre/post, softmax + Sinkhorn comb,
    ``seam.py:260-321``); RMSNorm of the layer input (``seam.py:325-378``).
    Returns (res_out, normed, pre, post, comb)."""
    M, _, H = res.shape
    rn = fold_post(res, x, post, comb) if fold else f32(res).clone()
    if first:
        lin = rn[:, 0, :].clone()
    else:
        acc = torch.zeros(M, H)
        for h in range(HC):
            acc = acc + f32(pre_prev)[:, h, None] * rn[:, h, :]
        lin = bf(acc)
    flat = rn.reshape(M, HC * H).double()
    mix = (flat @ f32(hc_fn).double().T).float()
    sq = (flat * flat).sum(1).float()
    rstd = 1.0 / torch.sqrt(sq / float(HC * H) + RMS_EPS)
    v = mix * rstd[:, None]
    sc, base = f32(hc_scale), f32(hc_base)
    pre = torch.sigmoid(v[:, :HC] * sc[0] + base[:HC]) + HC_EPS
    post_o = 2.0 * torch.sigmoid(v[:, HC:2 * HC] * sc[1] + base[HC:2 * HC])
    cv = (v[:, 2 * HC:] * sc[2] + base[2 * HC:]).view(M, HC, HC)
    cv = torch.exp(cv - cv.amax(2, keepdim=True))
    cv = cv / cv.sum(2, keepdim=True) + HC_EPS
    cv = cv / (cv.sum(1, keepdim=True) + HC_EPS)
    for _ in range(SINKHORN - 1):
        cv = cv / (cv.sum(2, keepdim=True) + HC_EPS)
        cv = cv / (cv.sum(1, keepdim=True) + HC_EPS)
    r = 1.0 / torch.sqrt(seam_sumsq(lin).float() / float(H) + RMS_EPS)
    normed = bf((lin * r[:, None]) * f32(norm_w))
    return rn, normed, pre, post_o, cv


def seam_sumsq(lin, threads=256):
    """fp64 sum of squares of the bf16-valued rows of lin [M, H] (H a multiple of 8) in the
    seam norm's fixed order: thread t of ``threads`` takes the 8 columns at 8 t + 8 threads k
    for k = 0, 1, ... in column order; each 32-thread warp folds by an xor-butterfly; the warp
    sums add in warp order from 0. The squares are exact, so only the order is pinned (the
    reference's norm, ``seam.py:325-378``, sums in its own lane order)."""
    M, H = lin.shape
    v = lin.double().numpy() ** 2
    per = threads * 8
    acc = np.zeros((M, threads))
    for k in range(-(-H // per)):
        chunk = np.zeros((M, per))
        c0 = k * per
        chunk[:, : min(per, H - c0)] = v[:, c0:c0 + per]
        chunk = chunk.reshape(M, threads, 8)
        for i in range(8):
            acc = acc + chunk[:, :, i]
    warps = butterfly32(acc.reshape(M, threads // 32, 32))
    tot = np.zeros(M)
    for w in range(threads // 32):
        tot = tot + warps[:, w]
    return torch.from_numpy(tot)


# ---------------------------------------------------------------- dense GEMVs
def gemv_x8_fp8(x8, x8s, w8, wcodes, block=128):
    """fp32 [M, N] = dequant(MXFP8 x) . dequant(FP8 W, E8M0 per block x block)^T, accumulated in
    fp64 (the GEMVs sum in another order: tolerance parity; ``attention/gemv.py:141-194``)."""
    x = N.mxfp8_dequant(x8, x8s).double()
    w = N.deq_fp8_block(w8, wcodes, block, block).double()
    return (x @ w.T).float()


def gemv_bf16_fp8(x, w8, wcodes, block=128):
    """fp32 [M, N] = bf16 x . dequant(FP8 W)^T (wo_a: bf16 activations, ``back.py:538-575``)."""
    w = N.deq_fp8_block(w8, wcodes, block, block).double()
    return (f32(x).double() @ w.T).float()


# ---------------------------------------------------------------- K1: q / kv
def q_path(qkv_q, q_norm_w):
    """q_norm of the q_lora part (bf16 in) -> bf16 ys (``qr``) and vLLM MXFP8 QX8
    (``front.py:189-244``). Returns (ys, qx8, qx8s)."""
    xq = bf(qkv_q)
    ss = (xq.double() ** 2).sum(1).float()
    r = 1.0 / torch.sqrt(ss / float(xq.shape[1]) + RMS_EPS)
    ys = bf((xq * r[:, None]) * f32(q_norm_w))
    q8, q8s = N.mxfp8_quant(ys, "vllm")
    return ys, q8, q8s


def butterfly32(lanes):
    """The value an xor-butterfly (16, 8, 4, 2, 1) of fp64 lane values [..., 32] leaves."""
    for d in (16, 8, 4, 2, 1):
        lanes = lanes[..., :d] + lanes[..., d:2 * d]
    return lanes[..., 0]


def sumsq_fixed(x):
    """fp64 sum of squares of the rows of x [M, D] (D a multiple of 64) in the kernel's order:
    lane i of 64 sums x[i + 64 r]^2 over r sequentially; each 32-lane half folds by an
    xor-butterfly; the two halves add. Exact products, so only the order is pinned."""
    M, D = x.shape
    v = x.double().numpy() ** 2
    v = v.reshape(M, D // 64, 64)
    acc = np.zeros((M, 64))
    for r in range(D // 64):
        acc = acc + v[:, r, :]
    w = acc.reshape(M, 2, 32)
    return torch.from_numpy(butterfly32(w[:, 0]) + butterfly32(w[:, 1]))


def kv_record(qkv_kv, kv_norm_w, cos, sin, nope):
    """The FP8 KV record of each row (``front.py:246-300``), bit-exact contract:
    x = bf16(kv); ss = fp32(sum of x^2 in fp64, in ``sumsq_fixed``'s order); ms = fp32(ss / D) + eps;
    r = 1 / sqrt(ms) (IEEE fp32, two roundings); k = (x r) w (fp32, two roundings);
    GPT-J RoPE of the dims past ``nope``: e0 = k0 c - k1 s, e1 = k0 s + k1 c (separate
    fp32 products, then the sum); per 64 nope dims: code = code_ceil(max(amax, 1e-4) / 448),
    byte = e4m3(clamp(e 2^(127 - code))). Returns (nope bytes [M, nope] u8, rope bf16 bytes
    [M, 2 * rope] u8, codes [M, nope / 64] u8)."""
    x = bf(qkv_kv)
    M, D = x.shape
    ss = sumsq_fixed(x).float()
    ms = ss / torch.tensor(float(D), dtype=torch.float32) + torch.tensor(RMS_EPS, dtype=torch.float32)
    r = torch.tensor(1.0, dtype=torch.float32) / torch.sqrt(ms)
    k = (x * r[:, None]) * f32(kv_norm_w)
    e = k.clone()
    k0, k1 = k[:, nope::2], k[:, nope + 1::2]
    c, s = f32(cos), f32(sin)
    e[:, nope::2] = k0 * c - k1 * s
    e[:, nope + 1::2] = k0 * s + k1 * c
    blocks = e[:, :nope].reshape(M, nope // 64, 64)
    amax = blocks.abs().amax(-1)
    code = N.code_ceil(amax.clamp_min(1e-4) / torch.tensor(448.0)).clamp(0, 254)
    q = N.e4m3_encode((blocks * N.mx_mul(code)[..., None]).clamp(-448, 448)).reshape(M, nope)
    rope = e[:, nope:].to(torch.bfloat16).view(torch.uint8).reshape(M, -1)
    return q, rope, code.to(torch.uint8)


def record_bytes(nope_b, rope_b, codes, scale_bytes):
    """[M, data] and [M, scale_bytes] byte rows of the record (codes then zero padding)."""
    M = nope_b.shape[0]
    data = torch.cat([nope_b, rope_b], 1)
    sc = torch.zeros(M, scale_bytes, dtype=torch.uint8)
    sc[:, : codes.shape[1]] = codes
    return data, sc


def write_records(cache, slot, data, sc, blk):
    """Store records at ``slot`` into a paged cache [pages, page bytes]: a page holds ``blk``
    data rows, then ``blk`` scale rows (``check_k1.py:166-176``). Negative slots store nothing."""
    D, S = data.shape[1], sc.shape[1]
    for t, s in enumerate(slot.tolist()):
        if s < 0:
            continue
        p, o = s // blk, s % blk
        cache[p, o * D:(o + 1) * D] = data[t]
        cache[p, blk * D + o * S: blk * D + (o + 1) * S] = sc[t]


def read_records(cache, slots, blk, nope, rope, scale_bytes):
    """Dequantized keys [n, nope + rope] fp32 of ``slots`` (``check_k2.py:39-64``)."""
    D = nope + 2 * rope
    slots = torch.as_tensor(slots, dtype=torch.long)
    p, o = slots // blk, slots % blk
    cols = o[:, None] * D + torch.arange(D)
    raw = cache[p[:, None].expand_as(cols), cols]
    scol = blk * D + o[:, None] * scale_bytes + torch.arange(nope // 64)
    codes = cache[p[:, None].expand_as(scol), scol]
    kn = N.e4m3_decode(raw[:, :nope]).reshape(-1, nope // 64, 64) * N.pow2(codes.int())[..., None]
    kr = raw[:, nope:].contiguous().view(torch.bfloat16).float()
    return torch.cat([kn.reshape(-1, nope), kr], 1)


def rope_q(v, cos, sin, nope):
    """GPT-J RoPE of dims past ``nope`` of [M, heads, D] bf16-valued q (``front.py:325-355``)."""
    out = v.clone()
    v0, v1 = v[..., nope::2], v[..., nope + 1::2]
    c, s = f32(cos)[:, None, :], f32(sin)[:, None, :]
    out[..., nope::2] = v0 * c - v1 * s
    out[..., nope + 1::2] = v0 * s + v1 * c
    return bf(out)


def key_table(slot, swa_idx, swa_lens, topk, topk_lens, swa_width, topk_width):
    """K2's key table (``front.py:117-143``): kt[t][k] = slot | 1 << 31 for the first ntopk
    keys (k < ntopk, compressed rows), window slots for k in [ntopk, kv_len), -1 past them or
    for an invalid slot; klen[t] = kv_len (0 for a pad row: slot < 0), klen[M + t] = ntopk."""
    M = slot.shape[0]
    keys = topk_width + swa_width
    kt = torch.full((M, keys), -1, dtype=torch.int32)
    klen = torch.zeros(2 * M, dtype=torch.int32)
    for t in range(M):
        live = int(slot[t]) >= 0
        nswa = min(int(swa_lens[t]), swa_width) if live else 0
        ntopk = min(int(topk_lens[t]), topk_width) if live else 0
        for k in range(ntopk + nswa):
            if k < ntopk:
                v = int(topk[t, k])
                kt[t, k] = (v | -(2**31)) if v >= 0 else -1
            else:
                s = int(swa_idx[t, k - ntopk])
                kt[t, k] = s if s >= 0 else -1
        klen[t], klen[M + t] = ntopk + nswa, ntopk
    return kt, klen


# ---------------------------------------------------------------- K2: attention
def attention(q, kt, klen, swa, swa_blk, comp, comp_blk, sink, cos, sin, nope, rope,
              scale_bytes):
    """XO [M, heads * D] bf16-valued (``check_k2.py:120-139``): each row's keys from the
    key table (bit 31: the compressed cache; -1: masked), exact softmax of q.k D^-0.5 with
    the sink folded into the max and the denominator, o = sum p k / l rounded to bf16, then
    the inverse GPT-J RoPE of dims past ``nope``, bf16. A row with no keys is zero."""
    M, Hh, D = q.shape
    xo = torch.zeros(M, Hh, D)
    for t in range(M):
        n = int(klen[t])
        vals = kt[t, :n].long()
        vals = vals[vals != -1]
        if vals.numel() == 0:
            continue
        is_c = vals < 0
        parts = []
        if bool(is_c.any()):
            parts.append(read_records(comp, (vals[is_c] & 0x7FFFFFFF), comp_blk, nope, rope, scale_bytes))
        if bool((~is_c).any()):
            parts.append(read_records(swa, vals[~is_c], swa_blk, nope, rope, scale_bytes))
        # the key order inside a row does not change the softmax; keep compressed keys first
        k = torch.cat(parts).double()
        s = (f32(q[t]).double() @ k.T) * (D ** -0.5)
        m = torch.maximum(s.amax(1), f32(sink).double())
        p = torch.exp(s - m[:, None])
        o = (p @ k) / (p.sum(1) + torch.exp(f32(sink).double() - m))[:, None]
        xo[t] = o.float()
    xo = bf(xo)
    e, od = xo[..., nope::2], xo[..., nope + 1::2]
    c, s = f32(cos)[:, None, :], f32(sin)[:, None, :]
    out = xo.clone()
    out[..., nope::2] = e * c + od * s
    out[..., nope + 1::2] = od * c - e * s
    return bf(out).reshape(M, Hh * D)


def wo_a(xo, woa8, woa_codes, groups, o_rank):
    """X8B: per local group g, bf16(XO_g . wo_a_g^T), then vLLM MXFP8 (``back.py:538-575``).
    Returns (ya bf16-valued [M, groups * o_rank], x8b, x8bs)."""
    M = xo.shape[0]
    w = N.deq_fp8_block(woa8, woa_codes, 128, 128).double().view(groups, o_rank, -1)
    ya = torch.einsum("tgk,grk->tgr", f32(xo).double().view(M, groups, -1), w).float()
    ya = bf(ya.reshape(M, groups * o_rank))
    q, s = N.mxfp8_quant(ya, "vllm")
    return ya, q, s


def wo_b(x8b, x8bs, wob8, wob_codes):
    """This rank's attention partial bf16(X8B . wo_b^T) (``back.py:592-617``)."""
    return bf(gemv_x8_fp8(x8b, x8bs, wob8, wob_codes))


def all_reduce(parts):
    """fp32 sum of the ranks' bf16 partials in rank order, rounded to bf16
    (``ops.py:269-277``, ``check_ffn.py:254-261``)."""
    acc = f32(parts[0]).clone()
    for p in parts[1:]:
        acc = acc + f32(p)
    return bf(acc)


# ---------------------------------------------------------------- K2: MoE
def router_logits(x, gate_w):
    """Router logits, bit-exact contract: fp32 of an fp64 sum of the exact bf16 x bf16
    products in a fixed order. Lane l of 32 owns k = 8 l + 256 i + j (j < 8); it sums
    i-major, j-minor, sequentially in fp64; the 32 lane sums then fold by xor-butterfly
    16, 8, 4, 2, 1 (lane 0's value). (The reference sums 4 fp32 K-parts in part order,
    ``moe.py:279-301``, ``moe.py:334-341``; this order is our kernel's.)"""
    xd = f32(x).double().numpy()
    wd = f32(gate_w).double().numpy()
    M, K = xd.shape
    E = wd.shape[0]
    xs = xd.reshape(M, K // 256, 32, 8)  # [t, i, lane, j]
    ws = wd.reshape(E, K // 256, 32, 8)
    lanes = np.zeros((M, E, 32))
    for i in range(K // 256):
        for j in range(8):
            lanes = lanes + xs[:, None, i, :, j] * ws[None, :, i, :, j]
    for d in (16, 8, 4, 2, 1):
        lanes = lanes[..., :d] + lanes[..., d:2 * d]
    return torch.from_numpy(lanes[..., 0].astype(np.float32))


def _topk_ids(vals, k):
    """Top-k column ids of each row, descending, ties to the lower id (-inf / NaN last)."""
    v = vals.double().numpy().copy()
    v[np.isnan(v)] = -np.inf
    idx = np.arange(v.shape[1])
    order = np.lexsort((np.broadcast_to(idx, v.shape), -v), axis=1)
    return torch.from_numpy(order[:, :k].astype(np.int32))


def route(logits, bias, topk, kind="sqrtsoftplus"):
    """Routing ids [M, k] int32 and weights [M, k] fp32, in top-k order.

    "sqrtsoftplus" (``moe.py:305-391``): score = sqrt(softplus(x)) (x > 20 passes through,
    ``numerics.route_score``), NaN scores weigh 0; the top-k of score + bias (NaN -> -inf),
    ties to the lower id; weights = score * 1.5 / max(sum of the k scores in top-k order,
    1e-20), all fp32.
    "softmax": the top-k of the logits, ties to the lower id; weights =
    e^(l - lmax) / sum over the k of e^(l - lmax), computed with the deterministic fp64 exp
    and rounded once to fp32."""
    M, E = logits.shape
    if kind == "softmax":
        ids = _topk_ids(logits, topk)
        sel = logits.gather(1, ids.long()).double().numpy()
        ex = N.det_exp(sel - sel[:, :1])
        tot = np.zeros(M)
        for j in range(topk):
            tot = tot + ex[:, j]
        w = (ex / tot[:, None]).astype(np.float32)
        return ids, torch.from_numpy(w)
    sc = N.route_score(logits)
    orig = torch.where(torch.isnan(sc), torch.zeros_like(sc), sc)
    vals = sc + f32(bias)[None, :]
    vals = torch.where(torch.isnan(vals), torch.full_like(vals, -float("inf")), vals)
    ids = _topk_ids(vals, topk)
    w = orig.gather(1, ids.long())
    total = torch.zeros(M)
    for j in range(topk):
        total = total + w[:, j]
    scale = torch.tensor(ROUTE_SCALE, dtype=torch.float32) / total.clamp_min(1e-20)
    return ids, w * scale[:, None]


def shared_expert(x8, x8s, sgu8, sgu_codes, sw28, sw2_codes, block=128):
    """Shared expert (``moe.py:502-563``, ``moe.py:1133-1153``): h = X8 . sgu^T; g = bf16(min(
    bf16(h_gate), 10)), u = clamp(bf16(h_up), +-10), act = bf16(g / (1 + e^-g)), v = bf16(act u);
    vLLM MXFP8 of v, then bf16(. sw2^T)."""
    h = gemv_x8_fp8(x8, x8s, sgu8, sgu_codes, block)
    si = h.shape[1] // 2
    g = bf(torch.clamp(bf(h[:, :si]), max=LIMIT))
    u = bf(h[:, si:]).clamp(-LIMIT, LIMIT)
    act = bf(g / (1.0 + torch.exp(-g)))
    v = bf(act * u)
    q, s = N.mxfp8_quant(v, "vllm")
    return bf(gemv_x8_fp8(q, s, sw28, sw2_codes, block))


def routed_experts(x8r, x8rs, ids, wts, w13, s13, w2, s2):
    """Routed experts (``check_ffn.py:209-232``, ``moe.py:907-947``, ``moe.py:1156-1184``):
    per pick, h = X8R . dequant(w13_e)^T; v = bf16(gc sigmoid(gc) uc) with gc = min(g, 10),
    uc = clamp(u, +-10); aiter MXFP8 of v; y = . dequant(w2_e)^T; contribution bf16(y w);
    summed in top-k order with a bf16 rounding at every add. Returns bf16-valued [M, H]."""
    M, K = ids.shape
    H = w2.shape[1]
    x = N.mxfp8_dequant(x8r, x8rs).double()
    per_k = torch.zeros(M, K, H)
    for e in torch.unique(ids).tolist():
        rows, ks = (ids == e).nonzero(as_tuple=True)
        wg = N.deq_fp4(w13[e], s13[e]).double()
        h = (x[rows] @ wg.T).float()
        inter = h.shape[1] // 2
        gc = h[:, :inter].clamp(max=LIMIT)
        uc = h[:, inter:].clamp(-LIMIT, LIMIT)
        v = bf(gc * torch.sigmoid(gc) * uc)
        q, s = N.mxfp8_quant(v, "aiter")
        y = (N.mxfp8_dequant(q, s).double() @ N.deq_fp4(w2[e], s2[e]).double().T).float()
        per_k[rows, ks] = bf(y * wts[rows, ks, None])
    routed = torch.zeros(M, H)
    for k in range(K):
        routed = bf(routed + per_k[:, k])
    return routed


def moe_partial(normed, w, route_kind, topk, block=128):
    """This rank's MoE partial bf16(routed + shared) and its routing (``check_ffn.py:209-232``)."""
    x8r, x8rs = N.mxfp8_quant(normed, "aiter")
    x8, x8s = N.mxfp8_quant(normed, "vllm")
    logits = router_logits(normed, w["gate_w"])
    ids, wts = route(logits, w.get("bias"), topk, route_kind)
    routed = routed_experts(x8r, x8rs, ids, wts, w["w13"], w["s13"], w["w2"], w["s2"])
    shared = shared_expert(x8, x8s, w["sgu"], w["sgu_s"], w["sw2"], w["sw2_s"], block)
    return bf(routed + shared), ids, wts, logits


# ---------------------------------------------------------------- the whole layer over tp ranks
def decode_layer(ws, S, shape, cache=None, fold=True, first=False, topk=None, topk_lens=None, comp=None,
                 comp_blk=1):
    """One decode layer of M rows over ``len(ws)`` TP ranks (``ws[r]``: rank r's weight shards;
    replicated tensors are read from ws[0]), from a step ``S`` (``synth.make_step``'s keys):
    the attention seam, wqkv_a, the q path and KV record (written into ``cache``, a copy of
    S["cache"] unless given), then per rank its heads' attention, wo_a and wo_b partial; the
    attention all-reduce; the FFN seam; per rank its expert-slice MoE partial; the MoE
    all-reduce (``layer.py:773-1072``). Returns a dict of the intermediate and final tensors."""
    W = ws[0]
    M = S["res"].shape[0]
    cs = W["cos_sin"][S["pos"]]
    cosv, sinv = cs[:, :32], cs[:, 32:]
    QL, D, nope = shape.q_lora, shape.head_dim, shape.nope
    cache = S["cache"].clone() if cache is None else cache
    rn, normed, pre, post, comb = seam(S["res"].float(), S["x"].float(), S["post"], S["comb"], S["pre"],
                                       W["hc_attn_fn"], W["hc_attn_scale"], W["hc_attn_base"], W["attn_norm"],
                                       fold=fold, first=first)
    x8, x8s = N.mxfp8_quant(normed, "vllm")
    qkv = gemv_x8_fp8(x8, x8s, W["wqkv"], W["wqkv_s"])
    _, qx8, qx8s = q_path(qkv[:, :QL], W["q_norm"])
    nb, rb, codes = kv_record(qkv[:, QL:], W["kv_norm"], cosv, sinv, nope)
    data, sc = record_bytes(nb, rb, codes, 8)
    write_records(cache, S["slot"], data, sc, S["blk"])
    if topk is None:
        kt, klen = key_table(S["slot"], S["swa_idx"], S["swa_lens"], None, torch.zeros(M, dtype=torch.int32),
                             S["swa_idx"].shape[1], 0)
    else:
        kt, klen = key_table(S["slot"], S["swa_idx"], S["swa_lens"], topk, topk_lens, S["swa_idx"].shape[1],
                             topk.shape[1])
    attn_parts = []
    for w in ws:
        q = rope_q(bf(gemv_x8_fp8(qx8, qx8s, w["wqb"], w["wqb_s"])).view(M, -1, D), cosv, sinv, nope)
        xo = attention(q, kt, klen, cache, S["blk"], comp, comp_blk, w["sink"], cosv, sinv, nope, shape.rope, 8)
        _, x8b, x8bs = wo_a(xo, w["woa"], w["woa_s"], shape.groups_local, shape.o_rank)
        attn_parts.append(wo_b(x8b, x8bs, w["wob"], w["wob_s"]))
    attn = all_reduce(attn_parts)
    rn2, normed2, pre2, post2, comb2 = seam(rn, attn, post, comb, pre, W["hc_ffn_fn"], W["hc_ffn_scale"],
                                            W["hc_ffn_base"], W["ffn_norm"])
    moe_parts, ids = [], None
    for w in ws:
        part, ids, _, _ = moe_partial(normed2, w, shape.route, shape.topk)
        moe_parts.append(part)
    return dict(cache=cache, attn_parts=attn_parts, attn=attn, res2=rn2, normed2=normed2, pre2=pre2,
                post2=post2, comb2=comb2, moe_parts=moe_parts, out=all_reduce(moe_parts), ids=ids)


# ---------------------------------------------------------------- LM head and greedy selection
def lm_head_argmax(x, w):
    """fp32 logits x . W^T (exact bf16 products summed in fp64, rounded once) and each row's
    greedy id, ties to the lower id (the north star's rule for SGLang's greedy sampling)."""
    logits = (f32(x).double() @ f32(w).double().T).float()
    return logits, _topk_ids(logits, 1)[:, 0]


def greedy_accept(ids, draft, per_req):
    """DSpark's greedy verify of blocks of ``per_req`` rows: row j of a request scored the token
    after draft[j]; draft[j + 1] is accepted while it equals row j's greedy id. Returns
    (accepted count, the target's next token) per request."""
    acc, nxt = [], []
    for r0 in range(0, ids.numel(), per_req):
        n = 0
        while n + 1 < per_req and int(ids[r0 + n]) == int(draft[r0 + n + 1]):
            n += 1
        acc.append(n)
        nxt.append(int(ids[r0 + n]))
    return torch.tensor(acc, dtype=torch.int32), torch.tensor(nxt, dtype=torch.int32)
