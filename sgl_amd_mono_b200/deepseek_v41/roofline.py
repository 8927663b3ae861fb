"""Algorithmic bytes of a decode step: what a step must read from HBM once, per rank.

Per layer (the numerator of the HBM weight-streaming roofline): every dense weight and its
scales (wqkv_a, wq_b, wo_a, wo_b, both mHC projections, the router gate and bias, the shared
expert, the norms), the routed experts the step actually selected (|U| of them, with their
E8M0 scales), and the KV records the step's key tables read (data + scale row each).
Activations and all-reduce traffic are excluded (all-reduce bytes are reported apart).
"""

from __future__ import annotations

from .shapes import HC, LayerShape

MIX = HC * (HC + 2)


def _fp8(n: int, k: int) -> int:
    return n * k + (-(-n // 128)) * (k // 128)


def dense_bytes(s: LayerShape) -> dict:
    H, D = s.hidden, s.head_dim
    return {
        "wqkv_a": _fp8(s.q_lora + D, H),
        "wq_b": _fp8(s.heads_local * D, s.q_lora),
        "wo_a": _fp8(s.groups_local * s.o_rank, s.group_k),
        "wo_b": _fp8(H, s.groups_local * s.o_rank),
        "shared": _fp8(2 * s.shared_local, H) + _fp8(H, s.shared_local),
        "router": s.experts * H * 2 + s.experts * 4,
        "hc_fn": 2 * MIX * HC * H * 4,
        "norms": 2 * H * 2 + s.q_lora * 2 + D * 2,
    }


def expert_bytes(s: LayerShape) -> int:
    """One routed expert's MXFP4 weights and E8M0 scales on one rank."""
    H, I = s.hidden, s.inter_local
    return 2 * I * H // 2 + 2 * I * H // 32 + H * I // 2 + H * I // 32


def layer_bytes(s: LayerShape, union: int, keys_read: int) -> dict:
    d = dense_bytes(s)
    out = dict(d)
    out["experts"] = union * expert_bytes(s)
    out["kv"] = keys_read * (s.record_data + 8)
    out["total"] = sum(d.values()) + out["experts"] + out["kv"]
    return out
