"""A CUDA backend for SGLang's monokernel plugin interface on NVIDIA B200 (sm_100a).

It runs DeepSeek-V4.1's decode and speculative-verify layers through hand-written sm_100a
kernels, a handful of launches a layer with both tensor-parallel all-reduces done inside the
kernels over NVLink peer memory, and registers under the backend name ``"cuda"`` through the
same plugin surface the reference project exposes (omirosh/sgl-amd-mono,
``sgl_amd_mono/__init__.py``): ``BACKEND``, ``SPECS`` keyed by Hugging Face architecture, and
``register_specs``, which SGLang calls through the ``sglang.srt.plugins`` entry point declared
in ``pyproject.toml``.

Layout: ``common/`` holds what every model shares (the ctypes loader of the C-ABI library, the
peer-memory exchange regions); ``deepseek_v41/`` holds the model's specs, forwards and glue, with
its kernels, C-ABI and launch runner under ``deepseek_v41/sm100a/``.
"""

__version__ = "0.1.0.dev0"

# The --monokernel-backend name this package registers
BACKEND = "cuda"
# Each spec by the model's HF architecture; a spec module imports only when a server runs
# this backend
SPECS = {
    "DeepseekV4ForCausalLM": "sgl_amd_mono_b200.deepseek_v41.spec:SPEC",
    "DeepseekV4ForCausalLMDSpark": "sgl_amd_mono_b200.deepseek_v41.draft:SPEC",
}

# The SGLang names this module reads (tests/test_spec.py pins them against the imports)
SGLANG_READS = {"srt/monokernels/spec.py": ("register",)}


def register_specs() -> None:
    """The plugin entry point, which SGLang runs in every process."""
    from sglang.srt.monokernels.spec import register

    for architecture, path in SPECS.items():
        register(backend=BACKEND, architecture=architecture, path=path)
