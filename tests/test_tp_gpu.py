"""The TP exchange on the GPU.

One GPU: ``dsv41_allreduce`` (and ``dsv41_allreduce_ll``, the LL exchange K2 fuses into its
producing kernels) as rank 0 of 2 with the other rank emulated by the host (its slot and arrival
flags, or its tagged LL words, written before the launch, so no kernel waits on another kernel):
the result is the rank-order fp32 sum rounded once, bit for bit, over consecutive exchanges
of both parities; a wait that nothing satisfies gives up at its deadline, records its site,
raises the failure flags, and later exchanges on the failed region do nothing; the context
stays usable. ``dsv41_rank_sum`` (the NCCL variant's sum) is the same sum.

Two GPUs (skipped with fewer): K1 + K2 at tp=2 with the in-kernel all-reduces against the
oracle layer over both ranks' shards, bit-identical to the NCCL variant, the attention
output bit-identical to the rank-order sum of the ranks' partials; and the fault-injection
hook (rank 1 stalls at its attention exchange) ending in guard errors on both ranks -- rank 0's
wait runs past its deadline -- not a hang.
"""

import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import layer as OL

pytestmark = pytest.mark.gpu


def _native():
    from sgl_amd_mono_b200.common.peer import Native
    return Native()


def _regions(tp, cap, dev):
    n = _native().region_bytes(tp, cap)
    return [torch.zeros(n, dtype=torch.uint8, device=dev) for _ in range(tp)]


def _words(region):
    return region[:32].view(torch.int32).cpu().tolist()


def _slot(region, par, tp, src, cap):
    off = 8192 + (par * tp + src) * cap * 2
    return region[off:off + cap * 2].view(torch.bfloat16)


def _arrive(region):
    return region[512:512 + 4 * 8 * 128].view(torch.int32).view(8, 128)


def _allreduce(table, tp, rank, cap, src, dst, deadline_ns=2_000_000_000, site=1, skip=0):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    a = abi.AllReduceArgs(n=src.numel(), tp=tp, rank=rank, peers=table.data_ptr(), cap=cap, src=src.data_ptr(),
                          dst=dst.data_ptr(), deadline_ns=deadline_ns, site=site, skip_push=skip)
    ext.call("dsv41_allreduce", a, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n", [4096, 48 * 4096, 8])
def test_allreduce_emulated_peer_bit_exact(n):
    dev = torch.device("cuda", 0)
    cap = 48 * 4096
    r0, r1 = _regions(2, cap, dev)
    table = torch.tensor([r0.data_ptr(), r1.data_ptr()], dtype=torch.int64, device=dev)
    g = torch.Generator(device=dev).manual_seed(n)
    for e in (1, 2, 3):
        p0 = (torch.randn(n, generator=g, device=dev) * 3).to(torch.bfloat16)
        p1 = (torch.randn(n, generator=g, device=dev) * 3).to(torch.bfloat16)
        # rank 1, emulated: its partial in rank 0's slot of parity e & 1, its flags raised
        _slot(r0, e & 1, 2, 1, cap)[:n] = p1
        _arrive(r0)[1] = e
        dst = torch.empty(n, dtype=torch.bfloat16, device=dev)
        _allreduce(table, 2, 0, cap, p0, dst)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), OL.all_reduce([p0.cpu(), p1.cpu()])), e
        assert torch.equal(_slot(r1, e & 1, 2, 0, cap)[:n], p0)  # pushed into the peer's slot
        nblk = max(1, min(128, -(-n // 8 // 256)))
        assert (_arrive(r1)[0, :nblk] == e).all()
        w = _words(r0)
        assert w[0] == e and w[1] == 0 and w[3:6] == [0, 0, 0]


def test_allreduce_deadline_gives_up_and_sticks():
    from sgl_amd_mono_b200.common.peer import Native
    dev = torch.device("cuda", 0)
    cap = 4096
    r0, r1 = _regions(2, cap, dev)
    table = torch.tensor([r0.data_ptr(), r1.data_ptr()], dtype=torch.int64, device=dev)
    src = torch.ones(cap, dtype=torch.bfloat16, device=dev)
    dst = torch.full((cap,), 7.0, dtype=torch.bfloat16, device=dev)
    t0 = time.perf_counter()
    _allreduce(table, 2, 0, cap, src, dst, deadline_ns=200_000_000, site=7)  # nothing raises rank 1's flag
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert 0.15 < took < 5.0, took
    w = _words(r0)
    assert w[3] == 7 and w[0] == 1  # the site; the sequence still advanced
    fail0 = r0[256:288].view(torch.int32).cpu()
    fail1 = r1[256:288].view(torch.int32).cpu()
    assert fail0[0] == 1 and fail1[0] == 1  # rank 0's failure flag in every region
    assert (dst.cpu() == 7.0).all()  # no reduce after a failed wait
    rc, words = Native().status(r0.data_ptr())
    assert rc == -4 and words[3] == 7
    # sticky: the next exchange on the failed region does nothing and returns at once
    _arrive(r0)[1] = 2
    t0 = time.perf_counter()
    _allreduce(table, 2, 0, cap, src, dst, deadline_ns=200_000_000, site=8)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.15
    assert (dst.cpu() == 7.0).all() and _words(r0)[3] == 7
    # the context is still usable
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 499500.0


def _ll_slot_words(region, par, tp, src, cap):
    off = 8192 + 4 * tp * cap + (par * tp + src) * (cap // 2) * 8
    return region[off:off + (cap // 2) * 8].view(torch.int64)


def _ll_words(vals_bf16, tag):
    """LL words of a bf16 vector: {bf16x2 of elements 2k, 2k + 1 (low 32 bits), tag (high)}."""
    bits = vals_bf16.view(torch.int16).to(torch.int64) & 0xFFFF
    pair = bits[0::2] | (bits[1::2] << 16)
    return pair | (int(tag) << 32)


def _allreduce_ll(table, tp, rank, cap, src, dst, deadline_ns=2_000_000_000, site=1, skip=0):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    a = abi.AllReduceArgs(n=src.numel(), tp=tp, rank=rank, peers=table.data_ptr(), cap=cap, src=src.data_ptr(),
                          dst=dst.data_ptr(), deadline_ns=deadline_ns, site=site, skip_push=skip)
    ext.call("dsv41_allreduce_ll", a, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n", [4096, 48 * 4096, 8])
def test_allreduce_ll_emulated_peer_bit_exact(n):
    """The fused exchange's LL protocol as rank 0 of 2, rank 1 emulated by the host: its words
    (tag = the exchange's epoch) written into rank 0's LL slot before the launch."""
    dev = torch.device("cuda", 0)
    cap = 48 * 4096
    r0, r1 = _regions(2, cap, dev)
    table = torch.tensor([r0.data_ptr(), r1.data_ptr()], dtype=torch.int64, device=dev)
    g = torch.Generator(device=dev).manual_seed(n + 1)
    for e in (1, 2, 3):
        p0 = (torch.randn(n, generator=g, device=dev) * 3).to(torch.bfloat16)
        p1 = (torch.randn(n, generator=g, device=dev) * 3).to(torch.bfloat16)
        _ll_slot_words(r0, e & 1, 2, 1, cap)[: n // 2] = _ll_words(p1, e)
        dst = torch.empty(n, dtype=torch.bfloat16, device=dev)
        _allreduce_ll(table, 2, 0, cap, p0, dst)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), OL.all_reduce([p0.cpu(), p1.cpu()])), e
        # pushed into the peer's slot (and its own), tagged with the epoch
        assert torch.equal(_ll_slot_words(r1, e & 1, 2, 0, cap)[: n // 2], _ll_words(p0, e))
        assert torch.equal(_ll_slot_words(r0, e & 1, 2, 0, cap)[: n // 2], _ll_words(p0, e))
        w = _words(r0)
        assert w[0] == e and w[1] == 0 and w[3:6] == [0, 0, 0]


def test_allreduce_ll_deadline_gives_up_and_sticks():
    from sgl_amd_mono_b200.common.peer import Native
    dev = torch.device("cuda", 0)
    cap = 4096
    r0, r1 = _regions(2, cap, dev)
    table = torch.tensor([r0.data_ptr(), r1.data_ptr()], dtype=torch.int64, device=dev)
    src = torch.ones(cap, dtype=torch.bfloat16, device=dev)
    dst = torch.full((cap,), 7.0, dtype=torch.bfloat16, device=dev)
    t0 = time.perf_counter()
    _allreduce_ll(table, 2, 0, cap, src, dst, deadline_ns=200_000_000, site=7)  # rank 1 never writes
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert 0.15 < took < 5.0, took
    w = _words(r0)
    assert w[3] == 7 and w[0] == 1
    assert r0[256:288].view(torch.int32).cpu()[0] == 1 and r1[256:288].view(torch.int32).cpu()[0] == 1
    assert (dst.cpu() == 7.0).all()
    rc, words = Native().status(r0.data_ptr())
    assert rc == -4 and words[3] == 7
    # sticky: the next exchange on the failed region does nothing and returns at once
    _ll_slot_words(r0, 0, 2, 1, cap)[: cap // 2] = _ll_words(src, 2)
    t0 = time.perf_counter()
    _allreduce_ll(table, 2, 0, cap, src, dst, deadline_ns=200_000_000, site=8)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.15
    assert (dst.cpu() == 7.0).all() and _words(r0)[3] == 7
    x = torch.arange(1000, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 499500.0


def test_rank_sum_matches_rank_order():
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(3)
    parts = (torch.randn(4, 16 * 4096, generator=g, device=dev) * 5).to(torch.bfloat16)
    out = torch.empty(16 * 4096, dtype=torch.bfloat16, device=dev)
    a = abi.RankSumArgs(n=out.numel(), tp=4, parts=parts.data_ptr(), out=out.data_ptr())
    ext.call("dsv41_rank_sum", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), OL.all_reduce(list(parts.cpu())))


# ---------------------------------------------------------------- two GPUs
SMALL_TP = dict(hidden=1024, heads=8, nope=512, rope=64, q_lora=256, o_groups=2, o_rank=1024, experts=16,
                topk=4, inter=512, shared_inter=512, route="softmax")
M_ROWS, CTX = 4, 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q, inject):
    import faulthandler
    import sys
    import traceback

    import torch.distributed as dist
    faulthandler.dump_traceback_later(150, exit=True)  # a stuck rank prints where it is, then exits
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if inject:
        os.environ["SGLANG_AMD_MONO_FAULT_INJECT"] = inject
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=dev)
    from sgl_amd_mono_b200.common.peer import DeviceGuardError, PeerBuffer
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner, peer_cap
    s = LayerShape(**SMALL_TP).sharded(world)
    peers = PeerBuffer(peer_cap(s, M_ROWS), None, rank, world, dev)
    # drawn on the CPU (the oracle's generator), then moved
    w = {k: (v.to(dev) if torch.is_tensor(v) else v)
         for k, v in synth.make_layer(s, 31, "cpu", positions=CTX + 8, rank=rank).items()}
    S = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in synth.make_step(s, M_ROWS, CTX, 32, "cpu").items()}
    from sgl_amd_mono_b200.common import ext
    res = {"error": None}
    # peer: row-parallel attention (each rank attends its rows for all heads); peer_heads: each rank
    # its heads for every row; nccl: the same split as peer_heads, the all-reduces through NCCL
    for mode in ("peer", "peer_heads", "nccl"):
        dist.barrier()
        try:
            ext.set_option("row_attn", 0 if mode == "peer_heads" else 1)
            rn = MonoRunner(s, dev, rank=rank, peers=peers, allreduce="nccl" if mode == "nccl" else "peer",
                            deadline_s=0.5 if inject else 5.0)
            L = rn.bind(w)
            step = dict(S, cache=S["cache"].clone())
            torch.cuda.synchronize()
            b = rn.k1(L, step, M_ROWS)
            rn.k2(L, step, M_ROWS, b)
            torch.cuda.synchronize()
            res[mode + "_words"] = peers.words()
            if inject:
                try:
                    rn.check()
                    res["guard"] = None
                except DeviceGuardError as e:
                    res["guard"] = str(e)
                break
            rn.check()
            res[mode] = {k: b[k].float().cpu().numpy() for k in ("out", "attn", "attn_part", "ids")}
            res[mode]["cache"] = step["cache"].cpu().numpy()
        except Exception:  # noqa: BLE001 -- reported through the gather below
            res["error"] = f"rank {rank} ({mode}): " + traceback.format_exc()
            print(res["error"], file=sys.stderr, flush=True)
        print(f"rank {rank} {mode}: guard words {peers.words()}", file=sys.stderr, flush=True)
        failed = [None] * world
        dist.all_gather_object(failed, res["error"] is not None or bool(inject))
        if any(failed):
            break
    got = [None] * world
    dist.all_gather_object(got, res)
    if rank == 0:
        q.put(got)
    torch.cuda.synchronize()
    dist.barrier()
    peers.close()
    dist.destroy_process_group()
    faulthandler.cancel_dump_traceback_later()


def _run_tp(inject=""):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    pc = mp.start_processes(_tp_worker, args=(2, _free_port(), q, inject), nprocs=2, start_method="spawn",
                            join=False)
    got = q.get()  # read before joining: the results fill more than a pipe buffer
    while not pc.join():
        pass
    return got


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_k2_tp2_in_kernel_allreduce_two_gpus():
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    got = _run_tp()
    assert not any(g["error"] for g in got), [g["error"] for g in got]
    r0, r1 = got[0], got[1]
    for k in ("out", "attn", "ids"):
        assert np.array_equal(r0["peer_heads"][k], r0["nccl"][k]), k  # both exchanges: the same bits
        for mode in ("peer", "peer_heads"):
            assert np.array_equal(r0[mode][k], r1[mode][k]), (mode, k)  # every rank: the same result
    for mode in ("peer", "peer_heads"):
        parts = [torch.from_numpy(r[mode]["attn_part"]).to(torch.bfloat16) for r in got]
        assert np.array_equal(OL.all_reduce(parts).float().numpy(), r0[mode]["attn"]), mode
    # the row split attends with other kernels / chunkings than the head split: close, same routing
    assert np.array_equal(r0["peer"]["ids"], r0["peer_heads"]["ids"])
    a, b = r0["peer"]["attn"], r0["peer_heads"]["attn"]
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-2
    # the oracle over both ranks' shards
    s = LayerShape(**SMALL_TP).sharded(2)
    ws = [synth.make_layer(s, 31, "cpu", positions=CTX + 8, rank=r) for r in range(2)]
    S = synth.make_step(s, M_ROWS, CTX, 32, "cpu")
    ref = OL.decode_layer(ws, S, s)
    assert np.array_equal(ref["cache"].numpy(), r0["peer"]["cache"])
    assert np.array_equal(ref["ids"].numpy(), r0["peer"]["ids"].astype(np.int32))
    out, want = torch.from_numpy(r0["peer"]["out"]), ref["out"].float()
    rms = want.pow(2).mean().sqrt()
    assert (out - want).norm() / want.norm() < 1e-2
    assert (out - want).abs().max() < 2e-2 * rms + want.abs().max() * 2 ** -7


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fault_injection_ends_in_guard_errors_two_gpus():
    got = _run_tp(inject="1:1")
    assert not any(g["error"] for g in got), [g["error"] for g in got]
    g0, g1 = got[0]["guard"], got[1]["guard"]
    assert g0 and "attention all-reduce ran past its deadline" in g0, g0
    assert g1 and "fault-injection" in g1 and "deadline" not in g1, g1
    assert got[0]["peer_words"][3] == 1 and got[1]["peer_words"][5] == 1
