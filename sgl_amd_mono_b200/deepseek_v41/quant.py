"""Weight quantizers for synthetic layers and checkpoint conversion (torch, any device).

The formats are the ones the kernels read: FP8 e4m3 with one power-of-two scale (stored as
an E8M0 code) per 128 x 128 block, and MXFP4 (E2M1, even K in the low nibble) with an E8M0
code per 32 values along K. Scales are the smallest powers of two that keep each block in
range, as V4 checkpoints store them (ue8m0). Also the KV-record quantizer used to fill
synthetic caches (``front.py:246-300`` of the reference).
"""

from __future__ import annotations

import torch

FP8_MAX = 448.0
E2M1_MAGS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _pow2_code(amax: torch.Tensor, fmax: float) -> torch.Tensor:
    """E8M0 code of the smallest power of two s with amax / s <= fmax."""
    e = torch.ceil(torch.log2(amax.clamp_min(2.0**-126) / fmax)).clamp(-127, 127)
    return (e + 127).to(torch.int32)


def quant_fp8_block(w: torch.Tensor, block: int = 128):
    """fp32 [N, K] -> (e4m3 bytes [N, K], E8M0 codes [ceil(N / block), K / block])."""
    N, K = w.shape
    Np = -(-N // block) * block
    wp = torch.zeros(Np, K, device=w.device, dtype=torch.float32)
    wp[:N] = w
    blocks = wp.view(Np // block, block, K // block, block)
    code = _pow2_code(blocks.abs().amax(dim=(1, 3)), FP8_MAX)
    scale = torch.ldexp(torch.ones_like(code, dtype=torch.float32), code - 127)
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(Np, K)[:N].contiguous().view(torch.uint8), code.to(torch.uint8)


def e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    """fp32 values already divided by their block scale -> E2M1 codes 0..15 (nearest)."""
    mids = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=x.device)
    mag = torch.bucketize(x.abs(), mids)
    sign = ((x < 0) & (mag > 0)).to(torch.int64) << 3
    return (mag | sign).to(torch.uint8)


def quant_mxfp4(w: torch.Tensor):
    """fp32 [..., N, K] -> (packed [..., N, K / 2] uint8, E8M0 codes [..., N, K / 32])."""
    *lead, N, K = w.shape
    g = w.reshape(*lead, N, K // 32, 32)
    code = _pow2_code(g.abs().amax(-1), 6.0)
    scale = torch.ldexp(torch.ones_like(code, dtype=torch.float32), code - 127)
    c = e2m1_codes(g / scale[..., None]).reshape(*lead, N, K // 2, 2)
    return (c[..., 0] | (c[..., 1] << 4)).contiguous(), code.to(torch.uint8)


def kv_records(e: torch.Tensor, nope: int):
    """Post-norm, post-RoPE KV rows [T, nope + rope] fp32 -> (data bytes [T, nope + 2 rope],
    scale bytes [T, 8]): per 64 nope dims code = ceil_pow2(max(amax, 1e-4) / 448)."""
    T = e.shape[0]
    blocks = e[:, :nope].reshape(T, nope // 64, 64)
    amax = blocks.abs().amax(-1).clamp_min(1e-4)
    q = amax / FP8_MAX
    bits = q.view(torch.int32)
    code = ((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0).int()
    mul = ((254 - code) << 23).view(torch.float32)
    b = (blocks * mul[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    rope = e[:, nope:].to(torch.bfloat16).view(torch.uint8).reshape(T, -1)
    sc = torch.zeros(T, 8, dtype=torch.uint8, device=e.device)
    sc[:, : nope // 64] = code.to(torch.uint8)
    return torch.cat([b.reshape(T, nope), rope], 1), sc
