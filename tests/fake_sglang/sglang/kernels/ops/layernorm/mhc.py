"""SGLang's mHC helpers the forward calls around the kernels (a test stand-in)."""

import torch


def hc_broadcast(x: torch.Tensor, hc_mult: int) -> torch.Tensor:
    """The embedding as every residual copy: [M, H] -> [M, hc, H]."""
    return x[:, None, :].expand(x.shape[0], hc_mult, x.shape[1]).contiguous()


def hc_combine(flat: torch.Tensor, pre: torch.Tensor, hc_mult: int, dtype) -> torch.Tensor:
    """The head's collapse of the residual copies with the last pre: sum_h pre[h] R[h]."""
    M = flat.shape[0]
    r = flat.view(M, hc_mult, -1)
    acc = torch.zeros_like(r[:, 0])
    for h in range(hc_mult):
        acc = acc + pre[:, h, None].float() * r[:, h]
    return acc.to(dtype)
