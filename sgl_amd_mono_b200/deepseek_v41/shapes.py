"""Layer shapes the kernels are built for: the reference model's and the BASELINE configs'.

The reference (omirosh/sgl-amd-mono, ``deepseek_v41/__init__.py:12-39``) builds for
DeepSeek-V4.1-Flash; the benchmark configs use other widths, so every width is a field.
The widths the benchmark configs leave open are chosen here: q_lora 1024 (hidden / 4, as the
reference model), wo_a in 8 groups of 1024, 64 bf16 RoPE dims beside the 512 FP8 latent dims of
a KV record, an FP8 shared expert, and power-of-two (E8M0) scales per 128 x 128 block of the
dense FP8 weights.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

HC = 4  # hc_mult


@dataclass(frozen=True)
class LayerShape:
    hidden: int
    heads: int          # query heads (all ranks)
    nope: int           # FP8 latent dims of a KV record / head
    rope: int           # RoPE dims (bf16 in the record)
    q_lora: int
    o_groups: int       # wo_a groups (all ranks)
    o_rank: int
    experts: int
    topk: int
    inter: int          # routed expert intermediate (all ranks)
    shared_inter: int
    route: str = "sqrtsoftplus"  # or "softmax"
    tp: int = 1

    @property
    def head_dim(self) -> int:
        return self.nope + self.rope

    @property
    def heads_local(self) -> int:
        return self.heads // self.tp

    @property
    def groups_local(self) -> int:
        return self.o_groups // self.tp

    @property
    def inter_local(self) -> int:
        return self.inter // self.tp

    @property
    def shared_local(self) -> int:
        return self.shared_inter // self.tp

    @property
    def group_k(self) -> int:
        """wo_a's K a group: its heads' outputs."""
        return self.heads // self.o_groups * self.head_dim

    @property
    def record_data(self) -> int:
        """Bytes of a KV record's data row (nope e4m3, rope bf16)."""
        return self.nope + 2 * self.rope

    def sharded(self, tp: int) -> "LayerShape":
        for name, v in (("heads", self.heads), ("o_groups", self.o_groups),
                        ("inter", self.inter), ("shared_inter", self.shared_inter)):
            if v % tp:
                raise ValueError(f"{name}={v} does not split over tp={tp}")
        return replace(self, tp=tp)

    def check(self) -> None:
        if self.hidden % 256 or self.nope % 64 or self.rope != 64:
            raise ValueError(f"unsupported shape {self}")
        if self.q_lora not in (256, 512, 1024):
            raise ValueError(f"q_lora {self.q_lora} unsupported")
        if self.inter_local % 128 or self.shared_local % 128:
            raise ValueError("expert widths must be multiples of 128 a rank")


# the CPU reference layer (softmax top-4 routing)
CONFIG1 = LayerShape(hidden=1024, heads=8, nope=512, rope=64, q_lora=256, o_groups=1, o_rank=1024,
                     experts=16, topk=4, inter=512, shared_inter=512, route="softmax")
# the full-size synthetic MoE decode layer
CONFIG2 = LayerShape(hidden=4096, heads=64, nope=512, rope=64, q_lora=1024, o_groups=8, o_rank=1024,
                     experts=256, topk=8, inter=2048, shared_inter=2048)
# the reference model (DeepSeek-V4.1-Flash), for the record
FLASH = LayerShape(hidden=5120, heads=64, nope=448, rope=64, q_lora=1280, o_groups=8, o_rank=1024,
                   experts=384, topk=6, inter=2304, shared_inter=2304)
