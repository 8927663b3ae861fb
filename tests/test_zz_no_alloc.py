"""The GEMV entry point for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: a serving process that gave all spare
HBM to its KV-cache pool at start-up, or a runtime binding the C ABI without a device
allocator. ``dsv41_gemv_fp8_noalloc`` serves them by keeping the GEMV's K-slice partials in a
library-owned device array. This file checks it through the C ABI against
``dsv41_gemv_fp8`` (caller scratch) on two calls in a row, and that a shape whose partials do
not fit the array is refused. It is named so pytest collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DSV41_ESCRATCH = -3


def _noalloc(args):
    from sgl_amd_mono_b200.common import ext
    f = ext.lib().dsv41_gemv_fp8_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return f(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _case(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randint(0, 256, (N, K), generator=g, device="cuda", dtype=torch.uint8)
    w[(w & 0x7F) == 0x7F] = 0  # no e4m3 NaN codes
    codes = torch.randint(115, 130, ((N + 127) // 128, K // 128), generator=g, device="cuda", dtype=torch.uint8)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    return w, codes, x


def _args(w, codes, x, y):
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    M, N, K = x.shape[0], w.shape[0], w.shape[1]
    return abi.GemvArgs(w=w.data_ptr(), codes=codes.data_ptr(), x=x.data_ptr(), y=y.data_ptr(), M=M, N=N, K=K,
                        x_ld=x.stride(0), x_group_rows=0, scratch=0, scratch_bytes=0)


def test_noalloc_matches_scratch_entry_two_calls():
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import ops
    # two shapes whose plans split K (partials in the library array), back to back
    for M, N, K, seed in ((16, 1600, 4096, 1), (8, 4096, 8192, 2)):
        w, codes, x = _case(M, N, K, seed)
        a = _args(w, codes, x, torch.empty(1, device="cuda"))
        assert ext.query("dsv41_gemv_fp8_scratch_bytes", a) > 0, "the case must use K-slice partials"
        want = ops.gemv_fp8(x, w, codes)
        got = torch.full((M, N), float("nan"), device="cuda")
        rc = _noalloc(_args(w, codes, x, got))
        torch.cuda.synchronize()
        assert rc == 0, rc
        # the same kernel, plan and slice order: the same bits
        assert torch.equal(got, want), (got - want).abs().max().item()


def test_noalloc_refuses_partials_over_the_array():
    M, N, K = 48, 65536, 8192  # partials far above the 4 MiB array
    w, codes, x = _case(M, N, K, 3)
    y = torch.zeros(M, N, device="cuda")
    rc = _noalloc(_args(w, codes, x, y))
    torch.cuda.synchronize()
    assert rc == DSV41_ESCRATCH
    assert bool((y == 0).all())
