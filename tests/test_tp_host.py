"""The TP host path on CPU with world_size-2 ``gloo`` ranks: the peer-region handshake (handles
exchanged in rank order, every rank refusing together when one fails, everything released),
the fault-injection hook's parsing, and the TP-sharded oracle layer (each rank's partials
gathered and summed in rank order equal the single-process sum, and tp=2 agrees with tp=1
within the bf16 rounding of the partials). The reference's ``test/multi_gpu`` suite and
``common/peer.py`` construction are the model."""

import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sgl_amd_mono_b200.common import peer as P


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))


class FakeNative:
    """The region calls without a GPU: regions are numbers, handles name their rank."""

    def __init__(self, rank, fail_alloc=False, fail_open=False):
        self.rank, self.fail_alloc, self.fail_open = rank, fail_alloc, fail_open
        self.freed, self.closed, self.opened = [], [], []

    def region_bytes(self, tp, cap):
        return 8192 + 4 * tp * cap

    def alloc(self, nbytes):
        if self.fail_alloc:
            raise RuntimeError("out of device memory")
        return 0x1000 * (self.rank + 1), bytes([self.rank + 1]) * P.IPC_HANDLE_BYTES

    def open(self, handle):
        if self.fail_open:
            raise RuntimeError("peer access unavailable")
        assert len(handle) == P.IPC_HANDLE_BYTES
        self.opened.append(0x100000 * handle[0])
        return 0x100000 * handle[0]

    def close(self, region):
        self.closed.append(region)

    def free(self, region):
        self.freed.append(region)

    def status(self, region):
        return 0, [0] * P.GUARD_WORDS


def _handshake(rank, world, port):
    _init(rank, world, port)
    try:
        nat = FakeNative(rank)
        pb = P.PeerBuffer(1000, None, rank, world, "cpu", native=nat)
        assert pb.cap == 1000 and pb.nbytes == 8192 + 4 * world * 1000
        want = [0x1000 * (rank + 1) if r == rank else 0x100000 * (r + 1) for r in range(world)]
        assert pb.table.tolist() == want and pb.table.dtype == torch.int64
        pb.check()
        pb.close()
        assert sorted(nat.closed) == sorted(nat.opened) and nat.freed == [0x1000 * (rank + 1)]
    finally:
        dist.destroy_process_group()


def _refuse(rank, world, port, where):
    _init(rank, world, port)
    try:
        nat = FakeNative(rank, fail_alloc=(where == "alloc" and rank == 1), fail_open=(where == "open" and rank == 0))
        with pytest.raises(P.PeerMemoryError) as e:
            P.PeerBuffer(64, None, rank, world, "cpu", native=nat)
        culprit = 1 if where == "alloc" else 0
        assert f"rank {culprit}" in str(e.value)
        # everything this rank made is released
        if not (where == "alloc" and rank == 1):
            assert nat.freed == [0x1000 * (rank + 1)]
        assert sorted(nat.closed) == sorted(nat.opened)
    finally:
        dist.destroy_process_group()


def _close_order(rank, world, port, q):
    import time
    _init(rank, world, port)
    try:
        nat = FakeNative(rank)
        pb = P.PeerBuffer(64, None, rank, world, "cpu", native=nat)
        if rank == 1:
            time.sleep(1.0)  # rank 1's last exchange is still queued when rank 0 closes
        entered = time.time()
        pb.close()
        released = time.time()
        q.put((rank, entered, released, list(nat.freed)))
    finally:
        dist.destroy_process_group()


def test_peer_close_waits_for_every_rank_gloo():
    """No rank frees its region before every rank has reached close()."""
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    pc = mp.start_processes(_close_order, args=(2, _free_port(), q), nprocs=2, start_method="spawn", join=False)
    got = sorted([q.get(), q.get()])
    while not pc.join():
        pass
    (_, e0, r0, f0), (_, e1, r1, f1) = got
    assert f0 == [0x1000] and f1 == [0x2000]
    assert r0 >= e1 - 0.05, (r0, e1)  # rank 0 released only after rank 1 arrived (clock slack)
    assert r0 - e0 > 0.5


def test_peer_handshake_gloo():
    mp.start_processes(_handshake, args=(2, _free_port()), nprocs=2, start_method="spawn")


@pytest.mark.parametrize("where", ["alloc", "open"])
def test_peer_ranks_refuse_together(where):
    mp.start_processes(_refuse, args=(2, _free_port(), where), nprocs=2, start_method="spawn")


def test_peer_rejects_bad_widths():
    with pytest.raises(P.PeerMemoryError):
        P.PeerBuffer(64, None, 0, 1, "cpu", native=FakeNative(0))
    with pytest.raises(P.PeerMemoryError):
        P.PeerBuffer(64, None, 9, 9, "cpu", native=FakeNative(0))


def test_fault_injection_parse(monkeypatch):
    monkeypatch.delenv("SGLANG_AMD_MONO_FAULT_INJECT", raising=False)
    assert P.fault_injection(0) is None
    monkeypatch.setenv("SGLANG_AMD_MONO_FAULT_INJECT", "1:2:3")
    assert P.fault_injection(1) == (2, 3) and P.fault_injection(0) is None
    monkeypatch.setenv("SGLANG_AMD_MONO_FAULT_INJECT", "0:1")
    assert P.fault_injection(0) == (1, 0)
    for bad in ("x", "1", "1:9", "1:a"):
        monkeypatch.setenv("SGLANG_AMD_MONO_FAULT_INJECT", bad)
        with pytest.raises(ValueError):
            P.fault_injection(1)


def test_guard_messages():
    assert P.guard_message([0] * 8) is None
    w = [0] * 8
    w[P.W_DEADLINE] = 1
    assert "attention all-reduce" in P.guard_message(w)
    w[P.W_DEADLINE], w[P.W_PEER], w[P.W_FAULT] = 2, 1, 1
    m = P.guard_message(w)
    assert "MoE all-reduce" in m and "failure flag" in m and "fault-injection" in m


def test_guard_messages_name_the_row_attention_exchanges():
    w = [0] * 8
    w[P.W_DEADLINE] = 3
    assert "query exchange" in P.guard_message(w)
    w[P.W_DEADLINE] = 4
    assert "output exchange" in P.guard_message(w)



def test_fault_injection_takes_the_all_reduce_sites_only(monkeypatch):
    monkeypatch.setenv("SGLANG_AMD_MONO_FAULT_INJECT", "0:3")
    with pytest.raises(ValueError):
        P.fault_injection(0)


def test_peer_cap_covers_both_exchange_kinds():
    """A slot holds rows x hidden (the all-reduces) and ceil(rows / tp) x local heads x head_dim
    (the row-parallel attention's all-to-alls); K2 falls back to the head split when it cannot."""
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import peer_cap
    for tp in (2, 4, 8):
        s = CONFIG2.sharded(tp)
        for rows in (1, 4, 7, 16, 48):
            c = peer_cap(s, rows)
            assert c >= rows * s.hidden
            assert c >= -(-rows // tp) * s.heads_local * s.head_dim


def test_runner_refuses_tp_without_peers():
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner
    s = CONFIG2.sharded(2)
    with pytest.raises(RuntimeError, match="PeerBuffer"):
        MonoRunner(s, "cpu", rank=0)
    with pytest.raises(RuntimeError, match="rank"):
        MonoRunner(s, "cpu", rank=2, allreduce="nccl")
    with pytest.raises(RuntimeError, match="deadline"):
        MonoRunner(s, "cpu", rank=0, allreduce="nccl", deadline_s=0.0)


# ---------------------------------------------------------------- the sharded oracle layer
SMALL_TP = dict(hidden=1024, heads=8, nope=512, rope=64, q_lora=256, o_groups=2, o_rank=1024, experts=16,
                topk=4, inter=512, shared_inter=512, route="softmax")
M_ROWS, CTX = 2, 48


def _small(tp):
    from sgl_amd_mono_b200.deepseek_v41.shapes import LayerShape
    return LayerShape(**SMALL_TP).sharded(tp)


def _layer_inputs(tp, rank):
    from sgl_amd_mono_b200.deepseek_v41 import synth
    s = _small(tp)
    w = synth.make_layer(s, 21, "cpu", positions=CTX + 8, rank=rank)
    S = synth.make_step(s, M_ROWS, CTX, 22, "cpu")
    return s, w, S


def _sharded_layer(rank, world, port, q):
    torch.set_num_threads(2)
    _init(rank, world, port)
    try:
        from oracle import layer as OL
        s, w, S = _layer_inputs(world, rank)
        mine = OL.decode_layer([w], S, s)
        # this rank's partials, gathered in rank order over gloo, then the rank-order sum
        parts = [torch.empty_like(mine["attn_parts"][0]) for _ in range(world)]
        dist.all_gather(parts, mine["attn_parts"][0])
        attn = OL.all_reduce(parts)
        if rank == 0:
            q.put(attn.float().numpy())  # a numpy copy: no tensor sharing across the exit
    finally:
        dist.destroy_process_group()


def test_tp2_sharded_oracle_layer_gloo():
    from oracle import layer as OL
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    pc = mp.start_processes(_sharded_layer, args=(2, _free_port(), q), nprocs=2, start_method="spawn", join=False)
    attn_gloo = torch.from_numpy(q.get())  # read before joining
    while not pc.join():
        pass
    s2, w0, S = _layer_inputs(2, 0)
    _, w1, _ = _layer_inputs(2, 1)
    tp2 = OL.decode_layer([w0, w1], S, s2)
    assert torch.equal(attn_gloo, tp2["attn"].float())
    # the sharding is one model: tp=2 agrees with tp=1 up to the bf16 rounding of each partial
    s1, wf, _ = _layer_inputs(1, 0)
    tp1 = OL.decode_layer([wf], S, s1)
    assert torch.equal(tp1["cache"], tp2["cache"])
    for key in ("attn", "out"):
        a, b = tp2[key].float(), tp1[key].float()
        rms = b.pow(2).mean().sqrt()
        assert (a - b).norm() / b.norm() < 2e-2, key
        assert (a - b).abs().max() < 0.1 * rms + 0.02 * b.abs().max(), key
