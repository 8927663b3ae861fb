"""The LM head + fused argmax and DSpark's greedy acceptance on the GPU against the oracle
(fp64-summed logits, greedy ids with ties to the lower id): ids identical, logits within
1e-5 of the oracle's largest magnitude; exact ties resolved to the lower id; two vocab shards
max-merged into one key array equal the full head; the acceptance of verify blocks."""

import pytest
import torch

from oracle import layer as OL

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _call(x, w, best, *, logits=None, vbase=0, init=1):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    a = abi.LmHeadArgs(M=x.shape[0], V=w.shape[0], K=w.shape[1], vbase=vbase, w=w.data_ptr(), x=x.data_ptr(),
                       logits=0 if logits is None else logits.data_ptr(), best=best.data_ptr(), init=init)
    ext.call("dsv41_lmhead_argmax", a, torch.cuda.current_stream().cuda_stream)


def _decode(best, *, draft=None, per_req=1):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    M = best.numel()
    ids = torch.empty(M, dtype=torch.int32, device=DEV)
    vals = torch.empty(M, dtype=torch.float32, device=DEV)
    R = M // per_req
    acc = torch.empty(R, dtype=torch.int32, device=DEV)
    nxt = torch.empty(R, dtype=torch.int32, device=DEV)
    a = abi.ArgmaxArgs(M=M, best=best.data_ptr(), ids=ids.data_ptr(), vals=vals.data_ptr(),
                       draft=0 if draft is None else draft.data_ptr(), per_req=per_req, accept=acc.data_ptr(),
                       next_tok=nxt.data_ptr())
    ext.call("dsv41_argmax_decode", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return ids.cpu(), vals.cpu(), acc.cpu(), nxt.cpu()


def _inputs(M, V, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(V, K, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    return x, w


@pytest.mark.parametrize("M,V,K", [(48, 20000, 4096), (1, 1000, 4096), (13, 777, 1024), (8, 129, 128)])
def test_lmhead_argmax_matches_oracle(M, V, K):
    x, w = _inputs(M, V, K, seed=M + V)
    best = torch.empty(M, dtype=torch.int64, device=DEV)
    logits = torch.empty(M, V, dtype=torch.float32, device=DEV)
    _call(x.to(DEV), w.to(DEV), best, logits=logits)
    ids, vals, _, _ = _decode(best)
    ref, ref_ids = OL.lm_head_argmax(x, w)
    assert torch.equal(ids, ref_ids)
    scale = ref.abs().max()
    assert (logits.cpu() - ref).abs().max() <= 1e-5 * scale
    assert torch.equal(vals, logits.cpu().gather(1, ids.long()[:, None])[:, 0])


def test_lmhead_full_vocab_against_fp32_torch():
    """BASELINE config 5's head (129280 x 4096): greedy ids against a torch fp32 GEMM on the
    GPU, on >= 99.5 % of rows (both sum in fp32, in different orders)."""
    M, V, K = 48, 129280, 4096
    g = torch.Generator(device=DEV).manual_seed(4)
    w = (torch.randn(V, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    best = torch.empty(M, dtype=torch.int64, device=DEV)
    _call(x, w, best)
    ids, _, _, _ = _decode(best)
    ref = (x.float() @ w.float().T).argmax(1).int().cpu()
    assert (ids == ref).float().mean() >= 0.995


def test_lmhead_ties_go_to_the_lower_id():
    M, V, K = 16, 3000, 512
    x, w = _inputs(M, V, K, seed=7)
    # rows 2900 and 100 become copies of the row each token likes best: equal logits
    _, ref_ids = OL.lm_head_argmax(x, w)
    w[2900] = w[int(ref_ids[0])]
    lo = int(ref_ids[0])
    best = torch.empty(M, dtype=torch.int64, device=DEV)
    _call(x.to(DEV), w.to(DEV), best)
    ids, _, _, _ = _decode(best)
    _, want = OL.lm_head_argmax(x, w)
    assert torch.equal(ids, want)
    assert int(ids[0]) == min(lo, 2900)


def test_vocab_shards_max_merge():
    M, V, K = 24, 5000, 2048
    x, w = _inputs(M, V, K, seed=11)
    xd, wd = x.to(DEV), w.to(DEV)
    best = torch.empty(M, dtype=torch.int64, device=DEV)
    _call(xd, wd[:2600], best, vbase=0, init=1)
    _call(xd, wd[2600:], best, vbase=2600, init=0)
    ids, _, _, _ = _decode(best)
    assert torch.equal(ids, OL.lm_head_argmax(x, w)[1])


def test_greedy_acceptance():
    M, V, K, P = 48, 4000, 1024, 6
    x, w = _inputs(M, V, K, seed=13)
    _, ref_ids = OL.lm_head_argmax(x, w)
    # request r's draft agrees with the target for its first r % P tokens
    draft = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    for r in range(M // P):
        for j in range(r % P):
            draft[r * P + j + 1] = ref_ids[r * P + j]
        if r % P + 1 < P:
            draft[r * P + r % P + 1] = (ref_ids[r * P + r % P] + 1) % V
    best = torch.empty(M, dtype=torch.int64, device=DEV)
    _call(x.to(DEV), w.to(DEV), best)
    ids, _, acc, nxt = _decode(best, draft=draft.to(DEV), per_req=P)
    want_acc, want_next = OL.greedy_accept(ref_ids, draft, P)
    assert torch.equal(acc, want_acc) and torch.equal(nxt, want_next)
    assert acc.tolist() == [r % P for r in range(M // P)]
