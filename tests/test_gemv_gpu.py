"""The FP8 weight-streaming GEMV against the oracle (fp64 dequantized product)."""

import pytest
import torch

from oracle import numerics as N

pytestmark = pytest.mark.gpu


def _case(M, Nn, K, seed, groups=1):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(Nn, K, generator=g) * 60).clamp(-448, 448)
    w8 = N.e4m3_encode(w)
    w8[0, :7] = torch.tensor([0, 1, 2, 7, 0x80, 0x81, 0x87], dtype=torch.uint8)  # zero and subnormals
    codes = torch.randint(110, 134, ((Nn + 127) // 128, K // 128), generator=g, dtype=torch.uint8)
    x = (torch.randn(M, K * groups, generator=g) * 3).to(torch.bfloat16)
    return w8, codes, x


@pytest.mark.parametrize("M,Nn,K,groups", [(1, 1600, 4096, 1), (5, 4096, 8192, 1), (16, 2304, 1024, 1),
                                          (48, 1600, 4096, 1), (33, 512, 2048, 1), (1, 8192, 4608, 8),
                                          (48, 8192, 4608, 8), (8, 4096, 256, 1)])
def test_gemv_fp8_matches_oracle(M, Nn, K, groups):
    from sgl_amd_mono_b200.deepseek_v41.sm100a import ops
    w8, codes, x = _case(M, Nn, K, 1000 + M + K, groups)
    wd = N.deq_fp8_block(w8, codes, 128, 128).double()
    xd = x.double()
    if groups > 1:
        gr = Nn // groups
        ref = torch.cat([xd[:, g * K:(g + 1) * K] @ wd[g * gr:(g + 1) * gr].T for g in range(groups)], 1)
    else:
        ref = xd @ wd.T
    dev = torch.device("cuda")
    y = ops.gemv_fp8(x.to(dev), w8.to(dev), codes.to(dev), x_group_rows=Nn // groups if groups > 1 else 0)
    torch.cuda.synchronize()
    err = (y.cpu().double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-6, err
