"""The runtime context the plugin reads (a test stand-in): set ``PARALLEL`` / ``MODEL``."""

from types import SimpleNamespace

PARALLEL = SimpleNamespace(tp_size=1, tp_rank=0, tp_group=SimpleNamespace(cpu_group=None))
MODEL = SimpleNamespace(context_length=None)


def get_parallel():
    return PARALLEL


def get_model():
    return MODEL

SPEC = SimpleNamespace(speculative_num_draft_tokens=6)


def get_spec():
    return SPEC
