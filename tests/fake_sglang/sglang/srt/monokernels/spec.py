"""The monokernel registry and spec types, as the plugin uses them (a test stand-in)."""

from __future__ import annotations

import enum
import importlib
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

MONOKERNEL_API_VERSION = 1


class Feature(enum.Enum):
    SPECULATIVE_DECODING = "speculative_decoding"


class NumericsKind(enum.Enum):
    TOLERANCE = "tolerance"
    EXACT = "exact"


class StepMetadata(enum.Enum):
    LOW_RATIO_DECODE_SCHEDULE = "low_ratio_decode_schedule"


@dataclass(frozen=True)
class DeviceLimits:
    widths: tuple
    tp_sizes: tuple
    resident_blocks: int


@dataclass(frozen=True)
class Requirements:
    dtypes: frozenset = frozenset()
    attention_backends: frozenset = frozenset()
    server_args: dict = field(default_factory=dict)
    hf_config: dict = field(default_factory=dict)
    env: dict = field(default_factory=dict)


@dataclass(frozen=True)
class Numerics:
    kind: NumericsKind
    bounds: dict

    def bound(self, name: str) -> float:
        return self.bounds[name]


@dataclass(frozen=True)
class MonoSpec:
    name: str
    devices: dict
    features: frozenset
    requires: Requirements
    numerics: Numerics
    model_disable_reasons: Callable
    build: Callable
    api_version: int = MONOKERNEL_API_VERSION
    config_disable_reasons: Optional[Callable] = None
    load_tensor: Optional[Callable] = None
    unread_metadata: frozenset = frozenset()
    tokens_per_request: Optional[Callable] = None


_REGISTRY: dict = {}


def register(*, backend: str, architecture: str, path: str) -> None:
    _REGISTRY[(backend, architecture)] = path


def find_spec(*, backend: str, architectures: list, isa: str) -> tuple[Any, str]:
    """(the spec, "") or (None, why)."""
    for arch in architectures:
        path = _REGISTRY.get((backend, arch))
        if path is None:
            continue
        mod, _, attr = path.partition(":")
        spec = getattr(importlib.import_module(mod), attr)
        if spec.api_version != MONOKERNEL_API_VERSION:
            return None, f"{spec.name}: api_version {spec.api_version}"
        if isa not in spec.devices:
            return None, f"{spec.name}: no kernels for {isa}"
        return spec, ""
    return None, f"no {backend} spec for {architectures}"
