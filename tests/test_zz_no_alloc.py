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
ARRAY_BYTES = 4 << 20  # DSV41_NOALLOC_SCRATCH_BYTES


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
    # two shapes whose plans split K (partials in the library array), queued back to back on one
    # stream with no host sync between them -- the ordering the shared array is safe under --
    # then one sync and both compared
    cases = [(16, 1600, 4096, 1), (8, 4096, 8192, 2)]
    inputs, wants, gots = [], [], []
    for M, N, K, seed in cases:
        w, codes, x = _case(M, N, K, seed)
        a = _args(w, codes, x, torch.empty(1, device="cuda"))
        assert ext.query("dsv41_gemv_fp8_scratch_bytes", a) > 0, "the case must use K-slice partials"
        wants.append(ops.gemv_fp8(x, w, codes))
        inputs.append((w, codes, x))
    torch.cuda.synchronize()
    for (w, codes, x), (M, N, K, _) in zip(inputs, cases):
        got = torch.full((M, N), float("nan"), device="cuda")
        rc = _noalloc(_args(w, codes, x, got))
        assert rc == 0, rc
        gots.append(got)
    torch.cuda.synchronize()
    for got, want in zip(gots, wants):
        # the same kernel, plan and slice order: the same bits
        assert torch.equal(got, want), (got - want).abs().max().item()


def test_noalloc_array_edge():
    """A shape whose partials fill the array exactly is served (and equals the scratch entry);
    one 8 rows wider is refused before any launch."""
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import ops
    M, N, K = 32, 8192, 4096
    w, codes, x = _case(M, N, K, 4)
    need = ext.query("dsv41_gemv_fp8_scratch_bytes", _args(w, codes, x, torch.empty(1, device="cuda")))
    assert need == ARRAY_BYTES, (need, "the plan of this shape no longer fills the array exactly")
    want = ops.gemv_fp8(x, w, codes)
    got = torch.full((M, N), float("nan"), device="cuda")
    assert _noalloc(_args(w, codes, x, got)) == 0
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    N2 = N + 8
    w2, codes2, x2 = _case(M, N2, K, 5)
    assert ext.query("dsv41_gemv_fp8_scratch_bytes", _args(w2, codes2, x2, torch.empty(1, device="cuda"))) > ARRAY_BYTES
    y = torch.zeros(M, N2, device="cuda")
    assert _noalloc(_args(w2, codes2, x2, y)) == DSV41_ESCRATCH
    torch.cuda.synchronize()
    assert bool((y == 0).all())


def test_noalloc_refuses_partials_over_the_array():
    M, N, K = 48, 65536, 8192  # partials far above the 4 MiB array
    w, codes, x = _case(M, N, K, 3)
    y = torch.zeros(M, N, device="cuda")
    rc = _noalloc(_args(w, codes, x, y))
    torch.cuda.synchronize()
    assert rc == DSV41_ESCRATCH
    assert bool((y == 0).all())
