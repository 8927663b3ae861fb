"""Thin torch-facing wrappers of single C-ABI launches (tests and the runner use them)."""

from __future__ import annotations

import torch

from ...common import ext
from . import abi


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def gemv_fp8(x: torch.Tensor, w: torch.Tensor, codes: torch.Tensor, x_group_rows: int = 0,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [M, N] = x (bf16 [M, >= K]) . dequant(W e4m3 [N, K], E8M0 128 x 128 codes)^T."""
    M, N, K = x.shape[0], w.shape[0], w.shape[1]
    y = out if out is not None else torch.empty(M, N, dtype=torch.float32, device=w.device)
    a = abi.GemvArgs(w=_ptr(w), codes=_ptr(codes), x=_ptr(x), y=_ptr(y), M=M, N=N, K=K,
                     x_ld=x.stride(0), x_group_rows=x_group_rows, scratch=0, scratch_bytes=0)
    need = ext.query("dsv41_gemv_fp8_scratch_bytes", a)
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=w.device)
    a.scratch, a.scratch_bytes = _ptr(scratch), need
    ext.call("dsv41_gemv_fp8", a, _stream())
    return y
