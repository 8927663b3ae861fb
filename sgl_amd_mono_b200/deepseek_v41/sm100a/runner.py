"""Host runner of the sm_100a kernels: per-width buffers, tensor checks, and the K1 / K2
launches through the C-ABI (the role of the reference's ``gfx950/runner.py:250-728``).

Weights are read in place (row-major FP8 dense projections, bf16 router, fp32 mHC weights);
the routed experts get one logged copy in the kernels' MXFP4 tensor-core tile order. Activations and
scratch belong to the runner and are allocated per width outside graph capture
(``buffers``); every launch goes on the current stream, so a step can be captured in a CUDA
graph and replayed. Host-side argument errors raise ``RuntimeError``; a launch's negative
status raises ``ExtError``.

Tensor parallelism (tp > 1): the weights are this rank's shards (``synth.make_layer`` with
``rank``), and K2's two all-reduces run either in-kernel through a ``PeerBuffer`` (the
default, ``allreduce="peer"``) or as the NCCL variant (``allreduce="nccl"``: K2 in two
phases around an all-gather of the bf16 partials and the same rank-order fp32 sum, so both
give identical bits). ``check()`` raises if a device-side guard fired.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ...common import ext
from ...common.peer import MIN_DEADLINE_S, PeerBuffer, fault_injection
from ..shapes import LayerShape
from . import abi


def _p(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check(t: torch.Tensor, name: str, shape: tuple, dtype: torch.dtype, device) -> None:
    if tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name}: must be contiguous")
    if t.device != device:
        raise RuntimeError(f"{name}: on {t.device}, expected {device}")


class Layer:
    """One layer's weights as the kernels read them."""

    def __init__(self, w: dict, relayout: dict):
        self.w = w
        self.r = relayout

    def __getitem__(self, k):
        return self.r[k] if k in self.r else self.w[k]


def peer_cap(shape: LayerShape, rows: int) -> int:
    """bf16 elements a PeerBuffer slot needs for launches of up to ``rows`` rows: the all-reduces'
    rows x hidden, and the row-parallel attention's exchanges (ceil(rows / tp) rows x this rank's
    heads x head_dim)."""
    return max(rows * shape.hidden, -(-rows // max(shape.tp, 1)) * shape.heads_local * shape.head_dim)


class MonoRunner:
    MAX_ROWS = 48

    def __init__(self, shape: LayerShape, device: torch.device, copies: dict | None = None, *,
                 rank: int = 0, peers: PeerBuffer | None = None, group=None, allreduce: str = "peer",
                 deadline_s: float = 5.0):
        shape.check()
        if not 0 <= rank < shape.tp:
            raise RuntimeError(f"rank {rank} outside tp {shape.tp}")
        if allreduce not in ("peer", "nccl"):
            raise RuntimeError(f"allreduce {allreduce!r}: 'peer' or 'nccl'")
        if shape.tp > 1 and allreduce == "peer" and peers is None:
            raise RuntimeError("tp > 1 with the in-kernel all-reduce needs a PeerBuffer")
        if deadline_s < MIN_DEADLINE_S:
            raise RuntimeError(f"deadline {deadline_s} s under {MIN_DEADLINE_S} s")
        self.rank, self.peers, self.group, self.allreduce = rank, peers, group, allreduce
        self.deadline_ns = int(deadline_s * 1e9)
        self._inject = fault_injection(rank) if shape.tp > 1 else None
        self._k2_count = 0
        self.s = shape
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.copies = copies if copies is not None else {}
        self._bufs: dict[int, dict] = {}
        self._scratch: dict[tuple, torch.Tensor] = {}
        self._pending_zeros: dict[int, dict] = {}
        self.k2i = None  # an indexer's K2iRunner (a model with index sources)

    # ------------------------------------------------------------ weights
    def bind(self, w: dict, tag: str = "layer") -> Layer:
        s, d = self.s, self.dev
        H, D, Il, SIl = s.hidden, s.head_dim, s.inter_local, s.shared_local
        E = s.experts
        checks = {
            "wqkv": ((s.q_lora + D, H), torch.uint8), "wqb": ((s.heads_local * D, s.q_lora), torch.uint8),
            "woa": ((s.groups_local * s.o_rank, s.group_k), torch.uint8),
            "wob": ((H, s.groups_local * s.o_rank), torch.uint8),
            "gate_w": ((E, H), torch.bfloat16), "w13": ((E, 2 * Il, H // 2), torch.uint8),
            "s13": ((E, 2 * Il, H // 32), torch.uint8), "w2": ((E, H, Il // 2), torch.uint8),
            "s2": ((E, H, Il // 32), torch.uint8), "sgu": ((2 * SIl, H), torch.uint8),
            "sw2": ((H, SIl), torch.uint8), "sink": ((s.heads_local,), torch.float32),
        }
        for k, (shape, dt) in checks.items():
            _check(w[k], k, shape, dt, d)
        r = {}
        for name, (src, codes, N, K) in {"w13": ("w13", "s13", 2 * Il, H), "w2": ("w2", "s2", H, Il)}.items():
            rows = (N + 255) // 256 * 256  # whole 256-row tensor-core tiles
            dst = torch.empty(E * rows * K // 2, dtype=torch.uint8, device=d)
            dcodes = torch.empty(E * rows * K // 32, dtype=torch.uint8, device=d)
            a = abi.RelayoutArgs(src=_p(w[src]), src_codes=_p(w[codes]), dst=_p(dst), dst_codes=_p(dcodes),
                                 E=E, N=N, K=K)
            ext.call("dsv41_relayout_mxfp4", a, _stream())
            r[name], r[name + "_codes"] = dst, dcodes
            self.copies[("mxfp4 tensor-core tile relayout", tag, name)] = (dst, dcodes)
        if s.tp > 1 and self.allreduce == "peer":
            # every rank's head sinks in rank order, for the row-parallel attention (each rank
            # attends its rows for all heads); a collective over the ranks, once a bound layer
            if dist.is_initialized() and dist.get_world_size(self.group) == s.tp:
                src = w["sink"].contiguous()
                if dist.get_backend(self.group) == "gloo":
                    src = src.cpu()
                parts = [torch.empty_like(src) for _ in range(s.tp)]
                dist.all_gather(parts, src, group=self.group)
                r["sink_all"] = torch.cat(parts).to(d)
                self.copies[("every rank's attention sinks", tag, "sink_all")] = (r["sink_all"],)
        return Layer(w, r)

    # ------------------------------------------------------------ buffers
    def buffers(self, M: int, keys: int) -> dict:
        if not 1 <= M <= self.MAX_ROWS:
            raise RuntimeError(f"rows {M} outside 1..{self.MAX_ROWS}")
        key = (M, keys)
        if key not in self._bufs:
            s, d = self.s, self.dev
            H, D = s.hidden, s.head_dim
            f32, bf, u8, i32 = torch.float32, torch.bfloat16, torch.uint8, torch.int32

            def z(*shape, dt=f32):
                return torch.zeros(*shape, dtype=dt, device=d)

            self._bufs[key] = dict(
                res1=z(M, 4, H, dt=bf), post_a=z(M, 4), comb_a=z(M, 4, 4), pre_a=z(M, 4),
                normed_a=z(M, H, dt=bf), x8=z(M, H, dt=u8), x8s=z(M, H // 32, dt=u8),
                qkv=z(M, s.q_lora + D), q=z(M, s.heads_local, D, dt=bf), qr=z(M, s.q_lora, dt=bf),
                qx8=z(M, s.q_lora, dt=u8), qx8s=z(M, s.q_lora // 32, dt=u8),
                kt=z(M, keys, dt=i32), klen=z(2 * M, dt=i32),
                res2=z(M, 4, H, dt=bf), post_f=z(M, 4), comb_f=z(M, 4, 4), pre_f=z(M, 4),
                normed_f=z(M, H, dt=bf), out=z(M, H, dt=bf), ids=z(M, s.topk, dt=i32),
                wts=z(M, s.topk), xo=z(M, s.heads_local * D, dt=bf),
                x8b=z(M, s.groups_local * s.o_rank, dt=u8), x8bs=z(M, s.groups_local * s.o_rank // 32, dt=u8),
                attn_part=z(M, H, dt=bf), logits=z(M, s.experts),
            )
            b = self._bufs[key]
            # one rank: the reduced attention output is the partial, the MoE output its partial
            b["attn"] = b["attn_part"] if s.tp == 1 else z(M, H, dt=bf)
            b["moe_part"] = b["out"] if s.tp == 1 else z(M, H, dt=bf)
            if s.tp > 1:
                if self.peers is not None and self.peers.cap < M * H:
                    raise RuntimeError(f"peer slots of {self.peers.cap} elements < {M} x {H}")
                b["gathered"] = z(s.tp, M, H, dt=bf)  # the NCCL variant's all-gather
        return self._bufs[key]

    def zeros_like_pending(self, M: int) -> dict:
        """Stand-ins for a pending post that is not owed (K1 with fold = 0 reads none of them;
        with first = 1 it reads no pre)."""
        if M not in self._pending_zeros:
            H, d = self.s.hidden, self.dev
            self._pending_zeros[M] = dict(
                x=torch.zeros(M, H, dtype=torch.bfloat16, device=d), post=torch.zeros(M, 4, device=d),
                comb=torch.zeros(M, 4, 4, device=d), pre=torch.zeros(M, 4, device=d))
        return self._pending_zeros[M]

    def _scratch_for(self, kind: str, M: int, need: int) -> torch.Tensor:
        k = (kind, M)
        t = self._scratch.get(k)
        if t is None or t.numel() < need:
            t = torch.empty(max(need, 256), dtype=torch.uint8, device=self.dev)
            self._scratch[k] = t
        return t

    # ------------------------------------------------------------ K1
    def k1_args(self, L: Layer, step: dict, M: int, *, fold=True, first=False, index=False,
                build_kt=True, swa_width=None, topk_width=0, topk_idx=None, topk_lens=None, events=0):
        s = self.s
        keys = (swa_width or step["swa_idx"].shape[1]) + topk_width
        b = self.buffers(M, keys)
        w = L
        a = abi.K1Args(
            M=M, hidden=s.hidden, q_lora=s.q_lora, nope=s.nope, rope=s.rope, heads=s.heads_local,
            swa_width=swa_width or step["swa_idx"].shape[1], topk_width=topk_width,
            fold=int(fold), first=int(first), index=int(index), build_kt=int(build_kt),
            res_in=_p(step["res"]), x_in=_p(step["x"]), post_in=_p(step["post"]), comb_in=_p(step["comb"]),
            pre_in=_p(step["pre"]), hc_fn=_p(w["hc_attn_fn"]), hc_scale=_p(w["hc_attn_scale"]),
            hc_base=_p(w["hc_attn_base"]), norm_w=_p(w["attn_norm"]),
            res_out=_p(b["res1"]), post_out=_p(b["post_a"]), comb_out=_p(b["comb_a"]), pre_out=_p(b["pre_a"]),
            normed=_p(b["normed_a"]), x8=_p(b["x8"]), x8s=_p(b["x8s"]),
            wqkv=_p(w["wqkv"]), wqkv_codes=_p(w["wqkv_s"]), q_norm=_p(w["q_norm"]), kv_norm=_p(w["kv_norm"]),
            cos_sin=_p(w["cos_sin"]), pos=_p(step["pos"]), rope_rows=w["cos_sin"].shape[0],
            slot=_p(step["slot"]), cache=_p(step["cache"]), page_stride=step["page_stride"], blk=step["blk"],
            swa_idx=_p(step["swa_idx"]), swa_lens=_p(step["swa_lens"]), topk_idx=_p(topk_idx),
            topk_lens=_p(topk_lens), kt=_p(b["kt"]), klen=_p(b["klen"]),
            wqb=_p(w["wqb"]), wqb_codes=_p(w["wqb_s"]), q=_p(b["q"]), qr=_p(b["qr"]),
            qx8=_p(b["qx8"]), qx8s=_p(b["qx8s"]), qkv_out=_p(b["qkv"]), events=events, scratch=0,
            scratch_bytes=0,
        )
        need = ext.query("dsv41_k1_scratch_bytes", a)
        sc = self._scratch_for("k1", M, need)
        a.scratch, a.scratch_bytes = _p(sc), sc.numel()
        return a, b

    def k1(self, L: Layer, step: dict, M: int, **kw) -> dict:
        a, b = self.k1_args(L, step, M, **kw)
        ext.call("dsv41_k1", a, _stream())
        return b

    # ------------------------------------------------------------ K2
    def k2_args(self, L: Layer, step: dict, M: int, b: dict, *, comp=None, comp_stride=0, comp_blk=0,
                events=0, phase=0, inject=0):
        s = self.s
        w = L
        peers = self.peers if s.tp > 1 else None
        a = abi.K2Args(
            M=M, hidden=s.hidden, nope=s.nope, rope=s.rope, heads=s.heads_local, o_groups=s.groups_local,
            o_rank=s.o_rank, experts=s.experts, topk=s.topk, inter=s.inter_local,
            shared_inter=s.shared_local, route_softmax=int(s.route == "softmax"), tp=s.tp, rank=self.rank,
            keys_ld=b["kt"].shape[1],
            q=_p(b["q"]), kt=_p(b["kt"]), klen=_p(b["klen"]), swa=_p(step["cache"]),
            swa_stride=step["page_stride"], swa_blk=step["blk"], comp=_p(comp), comp_stride=comp_stride,
            comp_blk=comp_blk, sink=_p(w["sink"]), sink_all=_p(L.r.get("sink_all")),
            cos_sin=_p(w["cos_sin"]), pos=_p(step["pos"]),
            rope_rows=w["cos_sin"].shape[0],
            woa=_p(w["woa"]), woa_codes=_p(w["woa_s"]), wob=_p(w["wob"]), wob_codes=_p(w["wob_s"]),
            res_in=_p(b["res1"]), post_in=_p(b["post_a"]), comb_in=_p(b["comb_a"]), pre_in=_p(b["pre_a"]),
            hc_fn=_p(w["hc_ffn_fn"]), hc_scale=_p(w["hc_ffn_scale"]), hc_base=_p(w["hc_ffn_base"]),
            norm_w=_p(w["ffn_norm"]),
            res_out=_p(b["res2"]), post_out=_p(b["post_f"]), comb_out=_p(b["comb_f"]), pre_out=_p(b["pre_f"]),
            normed=_p(b["normed_f"]),
            gate_w=_p(w["gate_w"]), bias=_p(w["bias"]), w13=_p(w["w13"]), w13_codes=_p(w["w13_codes"]),
            w2=_p(w["w2"]), w2_codes=_p(w["w2_codes"]), sgu=_p(w["sgu"]), sgu_codes=_p(w["sgu_s"]),
            sw2=_p(w["sw2"]), sw2_codes=_p(w["sw2_s"]),
            out=_p(b["out"]), ids=_p(b["ids"]), wts=_p(b["wts"]), xo=_p(b["xo"]), x8b=_p(b["x8b"]),
            x8bs=_p(b["x8bs"]), attn_part=_p(b["attn_part"]), attn=_p(b["attn"]), logits=_p(b["logits"]),
            moe_part=_p(b["moe_part"]), peers=_p(peers.table) if peers else 0,
            peer_cap=peers.cap if peers else 0, deadline_ns=self.deadline_ns, phase=phase, inject=inject,
            events=events,
            scratch=0, scratch_bytes=0,
        )
        need = ext.query("dsv41_k2_scratch_bytes", a)
        sc = self._scratch_for("k2", M, need)
        a.scratch, a.scratch_bytes = _p(sc), sc.numel()
        return a

    def k2(self, L: Layer, step: dict, M: int, b: dict, **kw) -> dict:
        s = self.s
        if s.tp > 1 and self.allreduce == "nccl":
            for phase, part, dst in ((1, "attn_part", "attn"), (2, "moe_part", "out")):
                ext.call("dsv41_k2", self.k2_args(L, step, M, b, phase=phase, **kw), _stream())
                self._nccl_reduce(b[part], b["gathered"], b[dst])
            return b
        inject = 0
        if self._inject is not None and self._k2_count == self._inject[1]:
            inject = self._inject[0]
        self._k2_count += 1
        a = self.k2_args(L, step, M, b, inject=inject, **kw)
        ext.call("dsv41_k2", a, _stream())
        return b

    def _nccl_reduce(self, part: torch.Tensor, gathered: torch.Tensor, out: torch.Tensor) -> None:
        """The NCCL variant of an all-reduce: all-gather the bf16 partials, then the rank-order
        fp32 sum (``dsv41_rank_sum``)."""
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        a = abi.RankSumArgs(n=part.numel(), tp=self.s.tp, parts=_p(gathered), out=_p(out))
        ext.call("dsv41_rank_sum", a, _stream())

    def check(self) -> None:
        """Raise ``DeviceGuardError`` if a device-side guard fired on this rank (synchronizes)."""
        if self.peers is not None:
            self.peers.check()
