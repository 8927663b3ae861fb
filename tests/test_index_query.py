"""The indexer's FP4 query (K2i's input): the oracle's contract on the CPU -- E2M1 round to
nearest even at every rounding boundary, and agreement with the torch restatement the spec glue
ran before (the same RoPE, layout and codes, but for its rounding of exact ties and of -0) -- and ``dsv41_index_query`` on the GPU bit for bit against the oracle."""

import numpy as np
import pytest
import torch

from oracle import indexer as OI


def test_e2m1_rne_boundaries():
    vals = np.array([0.0, 0.1, 0.25, 0.26, 0.74, 0.75, 1.0, 1.25, 1.3, 1.75, 2.4, 2.5, 2.6, 3.5, 4.9, 5.0, 5.1, 6.0,
                     100.0, -0.1, -0.75, -6.5], dtype=np.float32)
    want = [0, 0, 0, 1, 1, 2, 2, 2, 3, 4, 4, 4, 5, 6, 6, 6, 7, 7, 7, 8 | 0, 8 | 2, 8 | 7]
    assert OI.e2m1_rne(vals).tolist() == want
    # every code's magnitude encodes to itself
    assert OI.e2m1_rne(OI.E2M1_MAG.astype(np.float32)).tolist() == list(range(8))


def _case(M, H, hidden, seed, positions=4096):
    from sgl_amd_mono_b200.deepseek_v41 import synth
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(M, H, 128, generator=g).to(torch.bfloat16)
    x = torch.randn(M, hidden, generator=g).to(torch.bfloat16)
    wp = (torch.randn(H, hidden, generator=g) * 0.02).to(torch.bfloat16)
    pos = torch.randint(0, positions, (M,), generator=g)
    cs = synth.rope_table(positions, 64, "cpu")
    return q, x, wp, pos, cs


def _torch_restatement(q, freqs_cis, pos, rope_dim, w):
    """The torch restatement the spec glue ran before the kernel: complex RoPE, then the weight
    quantizer's MXFP4 (log2-ceiling codes, E2M1 ties toward zero, -0 stored as +0)."""
    from sgl_amd_mono_b200.deepseek_v41 import quant
    M, H, D = q.shape
    q = q.clone()
    f = freqs_cis[pos.long()][:, None, : rope_dim // 2]
    r = q[..., D - rope_dim:].reshape(M, H, rope_dim // 2, 2)
    rc = torch.view_as_complex(r.contiguous()) * f
    q[..., D - rope_dim:] = torch.view_as_real(rc).reshape(M, H, rope_dim)
    packed, codes = quant.quant_mxfp4(q.reshape(M * H, D))
    qs = torch.zeros(M, 1, 4, 16, 4, dtype=torch.uint8)
    h = torch.arange(H)
    qs[:, 0, :, h % 16, h // 16] = codes.view(M, H, 4).permute(0, 2, 1)
    return packed.view(M, H, D // 2).contiguous(), qs, w.to(torch.bfloat16).contiguous()


def test_oracle_query_matches_torch_restatement():
    q, x, wp, pos, cs = _case(4, 32, 1024, 1)
    scale = 0.125
    packed, qs, w = OI.index_query(q, cs, pos, 64, x, wp, scale)
    # the earlier restatement: complex RoPE on the same table, quant_mxfp4, bf16 head weights
    fc = torch.complex(cs[:, :32], cs[:, 32:])
    hw = (x.float().double() @ wp.float().double().T).float()
    p2, qs2, w2 = _torch_restatement(q.float(), fc, pos, 64, hw * scale)
    assert torch.equal(qs, qs2)
    assert torch.equal(w, w2)
    # the same codes but at the two places the earlier restatement's rounding differs: it stored
    # -0 as +0, and it sent a value exactly between two E2M1 magnitudes to the lower one (round to
    # nearest even picks the even code, the upper one at 0.75, 1.75 and 3.5 times the scale)
    a = torch.stack([packed & 15, packed >> 4], -1).flatten().numpy().astype(np.int64)
    b = torch.stack([p2 & 15, p2 >> 4], -1).flatten().numpy().astype(np.int64)
    diff = a != b
    neg_zero = (a == 8) & (b == 0)
    tie_up = ((a & 8) == (b & 8)) & ((a & 7) == (b & 7) + 1) & np.isin(a & 7, [2, 4, 6])
    assert np.all(~diff | neg_zero | tie_up)
    assert tie_up.sum() < 0.02 * diff.size


@pytest.mark.gpu
@pytest.mark.parametrize("M,H,hidden", [(16, 64, 4096), (5, 32, 1024), (1, 16, 2048)])
def test_index_query_gpu_bit_exact(M, H, hidden):
    import struct

    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    dev = torch.device("cuda", 0)
    q, x, wp, pos, cs = _case(M, H, hidden, M + H)
    scale = 0.0883883
    want = OI.index_query(q, cs, pos, 64, x, wp, scale)
    d = {k: v.to(dev) for k, v in dict(q=q, x=x, wp=wp, pos=pos, cs=cs).items()}
    q_out = torch.empty(M, H, 64, dtype=torch.uint8, device=dev)
    qscale = torch.zeros(M, 1, 4, 16, 4, dtype=torch.uint8, device=dev)
    w_out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    scratch = torch.empty(M * H * 4, dtype=torch.uint8, device=dev)
    bits = struct.unpack("<I", struct.pack("<f", scale))[0]
    a = abi.IndexQueryArgs(M=M, heads=H, dim=128, rope=64, hidden=hidden, q=d["q"].data_ptr(),
                           cos_sin=d["cs"].data_ptr(), rope_rows=d["cs"].shape[0], pos=d["pos"].data_ptr(),
                           x=d["x"].data_ptr(), wp=d["wp"].data_ptr(), weight_scale_f32=bits, q_out=q_out.data_ptr(),
                           qscale=qscale.data_ptr(), w_out=w_out.data_ptr(), scratch=scratch.data_ptr(),
                           scratch_bytes=scratch.numel())
    assert ext.query("dsv41_index_query_scratch_bytes", a) == M * H * 4
    ext.call("dsv41_index_query", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(qscale.cpu(), want[1])
    assert torch.equal(q_out.cpu(), want[0]), int((q_out.cpu() != want[0]).sum())
    assert torch.equal(w_out.cpu(), want[2])
