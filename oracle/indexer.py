"""CPU restatement of the indexer path: K2i FP4 logits, the top-k, the walk plan and the
candidate-block helpers (oracle; tests only). Citations are to omirosh/sgl-amd-mono.

FP4 plane layout (SGLang's, ``score_fp4.py:12-16``, ``indexer/runner.py:63-79``):
payload [pages, 1, 4, 64, 16] u8 -- a 64-key page, 4 chunks of 32 dims, a key's chunk as
16 bytes of E2M1 (even dim in the low nibble); kscale [pages, 1, 4, 64] u8 E8M0 with key s
of a page at (s % 16) * 4 + s // 16. Query: q [rows, heads, 64] u8 (128 E2M1 a head),
qscale [rows, 1, 4, 16, 4] u8 with head h's chunk c at [c, h % 16, h // 16], head weights
w [rows, heads] bf16. Column col of row t is key col % 64 of page table[t][col // 64].
"""

from __future__ import annotations

import numpy as np
import torch

from .numerics import E2M1

PAGE = 64  # keys an index-plane page
TOPK = 512
TOPK_BLOCKS = 2048
BLOCK_ROWS = 8
CHUNK = 128


def _e2m1_x2(b: torch.Tensor) -> torch.Tensor:
    """Bytes -> [.., 2 * n] int64 of 2 * E2M1 value (exact small integers)."""
    lut = torch.tensor([int(2 * v) for v in E2M1], dtype=torch.int64)
    b = b.to(torch.int64)
    return torch.stack([lut[b & 15], lut[b >> 4]], -1).flatten(-2)


def key_dims(payload, kscale, page, slot):
    """Keys at (page, slot) -> (2 * E2M1 ints [n, 4, 32], E8M0 codes [n, 4])."""
    k = _e2m1_x2(payload[page, 0, :, slot, :])  # [n, 4, 32]
    kidx = ((slot % 16) * 4 + slot // 16)
    ke = kscale[page[:, None], 0, torch.arange(4)[None], kidx[:, None]]
    return k, ke.to(torch.int64)


def index_logits(q, qscale, w, payload, kscale, table, t, cols, entry_rows=PAGE):
    """fp32 logits of row t at ``cols`` (``test_deepseek_v41_k2i.py:148-171``), bit-exact
    contract: per (head h, chunk c) the exact integer dot I of the 2 * E2M1 values; x_h =
    sum over c = 0..3 (sequential, fp64) of I 2^(qe + ke - 256); relu; the head terms
    w_h x_h (exact in fp64) summed in the kernel's tree: for g = 0..7, s_g = the terms of
    heads g, g + 8, g + 16, ... added in that order; then ((s0 + s4) + (s2 + s6)) +
    ((s1 + s5) + (s3 + s7)); rounded once to fp32."""
    cols = torch.as_tensor(cols, dtype=torch.long)
    heads = q.shape[1]
    # a table entry covers ``entry_rows`` keys: 64 (plane pages) or 8 (a REINDEX table's blocks)
    vrow = table[t][cols // entry_rows].long() * entry_rows + cols % entry_rows
    page = vrow // PAGE
    slot = vrow % PAGE
    k, ke = key_dims(payload, kscale, page, slot)  # [n, 4, 32], [n, 4]
    qv = _e2m1_x2(q[t].view(heads, 4, 16))  # [heads, 4, 32]
    h = torch.arange(heads)
    qe = qscale[t, 0][:, h % 16, h // 16].T.to(torch.int64)  # [heads, 4]
    dots = torch.einsum("hcd,ncd->hnc", qv, k)  # exact int64
    x = torch.zeros(heads, cols.numel(), dtype=torch.float64)
    for c in range(4):
        x = x + torch.ldexp(dots[:, :, c].double(), (qe[:, c, None] + ke[None, :, c] - 256))
    x = x.clamp_min(0.0)
    wd = w[t].float().double()
    s = torch.zeros(8, cols.numel(), dtype=torch.float64)
    for j in range(heads // 8):
        for g in range(8):
            s[g] = s[g] + wd[g + 8 * j] * x[g + 8 * j]
    s = s[:4] + s[4:]
    s = s[:2] + s[2:]
    return (s[0] + s[1]).float()


# E2M1 magnitudes by code, and the rounding boundaries between neighbours: a value exactly on a
# boundary goes to the neighbour with the even code (round to nearest even)
E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)
_E2M1_LOW_TIES = (0.25, 1.25, 2.5, 5.0)   # ties go down (to codes 0, 2, 4, 6)
_E2M1_HIGH_TIES = (0.75, 1.75, 3.5)       # ties go up (to codes 2, 4, 6)


def e2m1_rne(y: np.ndarray) -> np.ndarray:
    """fp32 values -> E2M1 codes (0..15): magnitude by round to nearest even, saturating at 6;
    the sign bit from the value's sign (a negative value that rounds to zero is -0), as
    cvt.rn.satfinite.e2m1x2.f32 encodes."""
    y = np.asarray(y, dtype=np.float32)
    m = np.abs(y).astype(np.float64)
    idx = np.zeros(y.shape, dtype=np.int64)
    for b in _E2M1_LOW_TIES:
        idx += m > b
    for b in _E2M1_HIGH_TIES:
        idx += m >= b
    return (idx | (np.signbit(y).astype(np.int64) << 3)).astype(np.uint8)


def index_query(q, cos_sin, pos, rope, x, wp, scale):
    """K2i's FP4 query of decode rows, the contract ``dsv41_index_query`` implements (restating
    SGLang's ``index_q_rope_pack_weights`` with its split-K head-weight GEMV, called at
    ``deepseek_v41/spec.py:744-763``; SGLang is absent here, so this contract is ours):
    head weights bf16(fp32(x . wp[h]) * scale), the dot as ``layer.router_logits`` sums it;
    GPT-J RoPE on the last ``rope`` dims of each head (e0 = k0 c - k1 s, e1 = k0 s + k1 c, fp32,
    each product and sum rounded); per 32 dims code = the E8M0 ceiling of fp32(max(amax, 2^-126)
    / 6) (at most 253), E2M1 of v 2^(127 - code) by ``e2m1_rne``, even dims in the low nibble.
    q [M, H, 128] bf16-valued, cos_sin [rows, rope] fp32, pos [M], x [M, hidden], wp [H, hidden].
    Returns (q_out [M, H, 64] u8, qscale [M, 1, 4, 16, 4] u8, w [M, H] bf16)."""
    from . import layer as OL
    M, H, D = q.shape
    hw = OL.router_logits(x, wp)
    w = (hw * torch.tensor(float(scale), dtype=torch.float32)).to(torch.bfloat16)
    v = q.float().clone()
    cs = cos_sin[torch.as_tensor(pos).long().clamp(0, cos_sin.shape[0] - 1)].float()
    c, s = cs[:, None, : rope // 2], cs[:, None, rope // 2:]
    k0, k1 = v[..., D - rope::2].clone(), v[..., D - rope + 1::2].clone()
    v[..., D - rope::2] = k0 * c - k1 * s
    v[..., D - rope + 1::2] = k0 * s + k1 * c
    chunks = v.view(M, H, D // 32, 32)
    q6 = chunks.abs().amax(-1).clamp_min(2.0**-126) / torch.tensor(6.0, dtype=torch.float32)
    bits = q6.view(torch.int32)
    code = (((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0).int()).clamp(max=253)
    mul = ((254 - code) << 23).view(torch.float32)
    codes4 = torch.from_numpy(e2m1_rne((chunks * mul[..., None]).numpy())).view(M, H, D // 2, 2)
    packed = (codes4[..., 0] | (codes4[..., 1] << 4)).contiguous()
    qs = torch.zeros(M, 1, 4, 16, 4, dtype=torch.uint8)
    h = torch.arange(H)
    qs[:, 0, :, h % 16, h // 16] = code.to(torch.uint8).permute(0, 2, 1)
    return packed, qs, w


def topk_rows(logits, bound, k):
    """The k largest of one row's logits[:bound], ties to the lower position (the north
    star's rule for SGLang's ``topk_transform_paged``), as positions in ascending order; every
    position when bound <= k; -1 padded to k. int32 [k]."""
    out = torch.full((k,), -1, dtype=torch.int32)
    if bound <= k:
        out[:bound] = torch.arange(bound, dtype=torch.int32)
        return out
    v = logits[:bound].double().numpy()
    order = np.lexsort((np.arange(bound), -v))[:k]
    out[:] = torch.from_numpy(np.sort(order).astype(np.int32))
    return out


def page_indices(raw, table_row, page_size):
    """Raw positions -> pool slots: table[pos // page] * page + pos % page; -1 stays -1."""
    valid = raw >= 0
    pos = torch.where(valid, raw, torch.zeros_like(raw)).long()
    slot = table_row[pos // page_size].long() * page_size + pos % page_size
    return torch.where(valid, slot.int(), torch.full_like(raw, -1))


def candidate_blocks(logits, bound, nblocks=TOPK_BLOCKS, rows=BLOCK_ROWS):
    """A producer row's candidate blocks: block b covers positions [8 b, 8 b + 8) of the
    row's bound; its score is the largest logit in it; the top ``nblocks`` blocks by
    score, ties to the lower block, in ascending block order, -1 padded (restating SGLang's
    ``select_candidate_blocks``, absent here, from its use at ``indexer/runner.py:158-190``)."""
    nb = -(-bound // rows)
    out = torch.full((nblocks,), -1, dtype=torch.int32)
    if nb == 0:
        return out
    v = torch.full((nb * rows,), -float("inf"), dtype=torch.float64)
    v[:bound] = logits[:bound].double()
    score = v.view(nb, rows).amax(1).numpy()
    order = np.sort(np.lexsort((np.arange(nb), -score))[:nblocks])
    out[: order.size] = torch.from_numpy(order.astype(np.int32))
    return out


def reindex_table(ids, page_table_row, visible, units=PAGE // BLOCK_ROWS, rows=BLOCK_ROWS):
    """One row of ``candidate_table.reindex_table`` (``candidate_table.py:19-66``): the
    newest block (holding position visible - 1) moved to the last kept slot; each kept
    block's virtual 8-row page; the context (full kept blocks, then the newest one's
    visible rows). Returns (ids_out, table, context)."""
    cand = ids.clone()
    live = cand >= 0
    kept = int(live.sum())
    newest = (int(visible) - 1) // rows
    at = -1
    for s in range(cand.numel()):
        if live[s] and int(cand[s]) == newest:
            at = s
    last = kept - 1
    moved = int(cand[last]) if last >= 0 else 0
    if at >= 0:
        cand[at], cand[last] = moved, newest
    live = cand >= 0
    table = torch.where(live, page_table_row[torch.where(live, cand, 0).long() // units].int() * units
                        + torch.where(live, cand, 0) % units, torch.zeros_like(cand))
    tail = int(cand[last]) if last >= 0 else 0
    last_span = min(max(int(visible) - tail * rows, 0), rows)
    context = (kept - 1) * rows + last_span if kept > 0 else 0
    return cand, table, context


def map_compact(compact_pos, ids_row, page_table_row, rows=BLOCK_ROWS, page=PAGE):
    """``candidate_table.map_compact_selection`` for one row (``candidate_table.py:103-134``):
    compact column c -> position ids[c // 8] * 8 + c % 8 -> pool slot; -1 stays -1."""
    valid = compact_pos >= 0
    col = torch.where(valid, compact_pos, torch.zeros_like(compact_pos)).long()
    pos = ids_row[col // rows].long() * rows + col % rows
    slot = page_table_row[pos // page].long() * page + pos % page
    raw = torch.where(valid, pos.int(), torch.full_like(compact_pos, -1))
    pg = torch.where(valid, slot.int(), torch.full_like(compact_pos, -1))
    return raw, pg


def fill_walk_plan(bounds, owners, ctas, walk_rows=6, chunk=CHUNK, topk=TOPK):
    """The FULL layer's score tasks (``index_plan.py:42-82``): pieces of at most
    ``walk_rows`` adjacent rows of one owner; a piece needs ceil(max bound / chunk) chunks
    (0 when no row's bound exceeds topk); every piece gets ceil(need / width) tasks sharing
    its chunks evenly, at the smallest width whose task count fits ``ctas``. Returns
    [ctas, 4] int32 of (lead, span, ch0, ch1), zeros past the last task."""
    bounds = np.asarray(bounds, dtype=np.int64)
    owners = np.asarray(owners, dtype=np.int64)
    plan = np.zeros((ctas, 4), dtype=np.int32)
    n = bounds.shape[0]
    leads, run_first = [], 0
    for t in range(n):
        if t == 0 or owners[t] != owners[t - 1]:
            run_first = t
            leads.append(t)
        elif (t - run_first) % walk_rows == 0:
            leads.append(t)
    pieces = []
    for i, lead in enumerate(leads):
        end = leads[i + 1] if i + 1 < len(leads) else n
        need = max(((b + chunk - 1) // chunk) if b > topk else 0 for b in bounds[lead:end])
        if need > 0:
            pieces.append((lead, end - lead, need))
    if not pieces:
        return plan
    assert len(pieces) < ctas
    total = sum(p[2] for p in pieces)
    width = max(-(-total // ctas), 1)
    while sum(-(-p[2] // width) for p in pieces) > ctas:
        width += 1
    r = 0
    for lead, span, need in pieces:
        k = -(-need // width)
        for i in range(k):
            plan[r] = (lead, span, i * need // k, (i + 1) * need // k)
            r += 1
    return plan
