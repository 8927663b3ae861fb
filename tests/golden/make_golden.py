"""Generate the golden fixtures that pin the oracle to the reference's own Python.

Run in a container that has the reference checkout (omirosh/sgl-amd-mono) at
``REFERENCE`` (default: the ``SGL_AMD_MONO_REF`` environment variable):

    SGL_AMD_MONO_REF=<path to the reference> python tests/golden/make_golden.py

It imports the reference's torch golden models and helpers -- the MX codecs and MoE
golden model of ``test/kernels/deepseek_v41/check_ffn.py``, the query reference of
``check_k1.py``, the attention reference and paged-cache builder of ``check_k2.py``,
the FP4 index-logit reference of ``test/kernels/test_deepseek_v41_k2i.py``, the weight
helpers of ``sgl_amd_mono/deepseek_v41/gfx950/weights.py`` and the walk plan of
``gfx950/indexer/index_plan.py`` -- runs them on small seeded CPU inputs and saves
inputs and outputs to ``tests/golden/*.pt``. SGLang, aiter and FlyDSL are absent, so
the reference's ``spec`` module (imported by the test files only for their numeric
bounds) is replaced by a stub carrying ``NUMERICS.bound``; nothing else is stubbed.
The fixtures are committed; the tests read only them, never the reference.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("SGL_AMD_MONO_REF", "/nonexistent"))


def _import_reference():
    if not REFERENCE.is_dir():
        raise SystemExit(f"reference checkout not found at {REFERENCE}")
    sys.path.insert(0, str(REFERENCE))
    sys.path.insert(0, str(REFERENCE / "test" / "kernels" / "deepseek_v41"))
    sys.path.insert(0, str(REFERENCE / "test" / "kernels"))
    import sgl_amd_mono.deepseek_v41  # noqa: F401  (pure Python)

    bounds = {
        "k1.kv.max_abs": 0.0, "k1.mix.max_abs": 1e-6, "k1.q.cosine": 0.99999, "k1.q.rel": 5e-3,
        "k1.normed.max_abs": 0.0, "k1.qr.rel": 4e-3, "k2.attn_out.cosine": 0.9998,
        "k2.wo_a.rel": 5e-3, "k2.wo_b.rel": 1e-3, "ffn.mix.rel": 1e-4,
        "ffn.normed.cosine": 0.9999, "ffn.normed.rel": 0.012, "ffn.moe.cosine": 0.9999,
        "ffn.moe.rel": 0.015, "k2i.logits.rel": 1e-5, "k2i.sel.max_abs": 0.0,
    }
    spec = types.ModuleType("sgl_amd_mono.deepseek_v41.spec")
    spec.NUMERICS = types.SimpleNamespace(bound=bounds.__getitem__)
    sys.modules["sgl_amd_mono.deepseek_v41.spec"] = spec
    import check_ffn
    import check_k1
    import check_k2
    import test_deepseek_v41_k2i as k2i
    from sgl_amd_mono.deepseek_v41.gfx950 import weights
    from sgl_amd_mono.deepseek_v41.gfx950.indexer import index_plan

    return check_ffn, check_k1, check_k2, k2i, weights, index_plan


def main():
    check_ffn, check_k1, check_k2, k2i, weights, index_plan = _import_reference()
    g = torch.Generator().manual_seed(20261201)

    # ---- MX codecs (check_ffn.py:87-121)
    x = torch.cat([torch.randn(64, 256, generator=g) * 3.0,
                   torch.randn(8, 256, generator=g) * 1e-3,
                   torch.zeros(1, 256)]).to(torch.bfloat16).float()
    pk = torch.randint(0, 256, (48, 64), generator=g, dtype=torch.uint8)
    pks = torch.randint(110, 135, (48, 4), generator=g, dtype=torch.uint8)
    w8 = (torch.randn(64, 96, generator=g) * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    w8s = torch.randint(110, 135, (2, 3), generator=g, dtype=torch.uint8)
    v = torch.rand(4096, generator=g) * torch.exp2(torch.randint(-40, 40, (4096,), generator=g).float())
    mx = dict(
        x=x,
        qdq_aiter=check_ffn.mxfp8_qdq(x, "aiter"),
        qdq_vllm=check_ffn.mxfp8_qdq(x, "vllm"),
        v=v, code_ceil=check_ffn.code_ceil(v),
        fp4_packed=pk, fp4_codes=pks, deq_fp4=check_ffn.deq_fp4(pk, pks),
        fp8_w=w8.view(torch.uint8), fp8_codes=w8s, deq_fp8=check_ffn.deq_fp8_block(w8, w8s),
    )
    torch.save(mx, OUT / "mx.pt")

    # ---- MoE golden model (check_ffn.py:201-232), small shapes, 32 x 32 shared blocks
    H, E, TOPK, INTER = 256, 16, 4, 128
    check_ffn.HIDDEN, check_ffn.E, check_ffn.TOPK = H, E, TOPK
    gm = torch.Generator().manual_seed(7)
    u8 = torch.uint8
    w = dict(
        gate_w=(torch.randn(E, H, generator=gm) * 0.05).to(torch.bfloat16),
        bias=(torch.randn(E, generator=gm) * 0.02).to(torch.bfloat16),
        w13_raw=torch.randint(0, 256, (E, 2 * INTER, H // 2), generator=gm, dtype=u8),
        s13_raw=torch.randint(118, 123, (E, 2 * INTER, H // 32), generator=gm, dtype=u8),
        w2_raw=torch.randint(0, 256, (E, H, INTER // 2), generator=gm, dtype=u8),
        s2_raw=torch.randint(118, 123, (E, H, INTER // 32), generator=gm, dtype=u8),
        sgu=torch.randn(2 * INTER, H, generator=gm).clamp(-6, 6).to(torch.float8_e4m3fn),
        sgu_s=torch.randint(118, 123, (2 * INTER // 32, H // 32), generator=gm, dtype=u8),
        sw2=torch.randn(H, INTER, generator=gm).clamp(-6, 6).to(torch.float8_e4m3fn),
        sw2_s=torch.randint(118, 123, (H // 32, INTER // 32), generator=gm, dtype=u8),
    )
    xm = (torch.randn(12, H, generator=gm)).to(torch.bfloat16)
    ids_r, wts_r = check_ffn.routing(xm, w)
    ids_g, part = check_ffn.golden_partial(xm, w, INTER, INTER)
    moe = {k: (t.view(u8) if t.dtype == torch.float8_e4m3fn else t) for k, t in w.items()}
    moe.update(x=xm, ids=ids_r, wts=wts_r, ids_golden=ids_g, partial=part, topk=TOPK)
    torch.save(moe, OUT / "moe.pt")

    # ---- weights.py: E8M0 codes, exact MXFP8 of a bf16 weight, the RoPE table
    sc = torch.exp2(torch.randint(-12, 4, (8, 6), generator=g).float())
    wq = (torch.randn(64, 96, generator=g) * 20).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    bl = torch.exp2(torch.randint(-8, 0, (2, 3), generator=g).float())
    wbf = (wq * bl.repeat_interleave(32, 0).repeat_interleave(32, 1)).to(torch.bfloat16)
    q8, codes = weights.mxfp8_exact(wbf, "golden")
    ang = torch.outer(torch.arange(16).double(), 10000.0 ** (-torch.arange(32).double() / 32))
    freqs = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    torch.save(dict(scale=sc, e8m0=weights.e8m0(sc, "golden"), wbf=wbf,
                    mx_q=q8.view(torch.uint8), mx_codes=codes, freqs=freqs,
                    rope=weights.rope_table(freqs, [])), OUT / "weights.pt")

    # ---- K1 query reference (check_k1.py:91-119), reference shapes at 2 heads
    check_k1.POSITIONS = 256
    gq = torch.Generator().manual_seed(11)
    heads = 2
    a = dict(
        q_norm=(1 + 0.1 * torch.randn(1280, generator=gq)).to(torch.bfloat16),
        wqb=(torch.randn(heads * 512, 1280, generator=gq) * 0.5).to(torch.float8_e4m3fn),
        wqb_s=torch.randint(121, 123, (heads * 512 // 32, 1280 // 32), generator=gq, dtype=u8),
    )
    qkv = (torch.randn(5, 1792, generator=gq) * 2).to(torch.bfloat16)
    pos = torch.tensor([0, 3, 77, 255, 128])
    cos_sin = check_k1.rope_table("cpu")
    qref = check_k1.query_ref(qkv, a, cos_sin, pos)
    torch.save(dict(qkv=qkv, q_norm=a["q_norm"], wqb=a["wqb"].view(u8), wqb_s=a["wqb_s"],
                    pos=pos, cos_sin=cos_sin, q=qref.float()), OUT / "k1_query.pt")

    # ---- K2 attention reference (check_k2.py:39-139): paged caches, key lists, XO
    gc = torch.Generator().manual_seed(5)
    check_k2.POSITIONS = 256
    swa_raw, swa_keys = check_k2.make_cache(4, 64, gc, "cpu")
    comp_raw, comp_keys = check_k2.make_cache(4, 128, gc, "cpu")
    # key_lists draws up to 512 top-k rows and 128 window rows from these pools
    check_k2.SWA_PAGES, check_k2.COMP_PAGES = 4, 4
    gk = torch.Generator().manual_seed(1006)
    M, Hh = 6, 4
    kt, klen, lists = check_k2.key_lists(M, gk, "cpu", pad_rows=(5,))
    qa = (torch.randn(M, Hh, 512, generator=gk) * 0.05).bfloat16()
    sink = torch.randn(Hh, generator=gk)
    posa = torch.randint(0, 256, (M,), generator=gk)
    freqs2 = torch.outer(torch.arange(256).float(), 1.0 / 10000 ** (torch.arange(32).float() / 32))
    cs2 = torch.cat([freqs2.cos(), freqs2.sin()], -1).contiguous()
    xo = check_k2.attention_xo(qa, swa_keys, comp_keys, lists, sink, posa, cs2)
    slot, keys = check_k2.source_keys(M, lists, "cpu")
    torch.save(dict(swa=swa_raw, comp=comp_raw, kt=kt, klen=klen, q=qa, sink=sink, pos=posa,
                    cos_sin=cs2, xo=xo, slot=slot, swa_idx=keys[0], swa_lens=keys[1],
                    topk=keys[2], topk_lens=keys[3]), OUT / "k2_attention.pt")

    # ---- K2i FP4 index logits (test_deepseek_v41_k2i.py:107-171)
    case = k2i.fp4_case(ctxs=[300, 129], seed=3, per_req=2, dev="cpu")
    rows = case["q"].shape[0]
    logits = []
    for t in range(rows):
        n = int(case["bounds"][t])
        cols = torch.arange(n)
        logits.append(k2i.ref_logits(case=case, t=t, cols=cols) if n else torch.zeros(0, dtype=torch.float64))
    torch.save(dict(case=case, logits=logits), OUT / "k2i.pt")

    # ---- walk plan (index_plan.py:42-82) on seeded steps
    rng = np.random.default_rng(0)
    plans = []
    for _ in range(40):
        n = int(rng.integers(1, 49))
        bounds, owners = k2i._walk_case(rng=rng, n=n)
        plan = np.zeros((256, 4), dtype=np.int32)
        index_plan.fill_walk_plan(bounds=bounds, owners=owners, plan=plan)
        plans.append((bounds, owners, plan))
    torch.save(dict(plans=plans), OUT / "walk_plan.pt")
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
