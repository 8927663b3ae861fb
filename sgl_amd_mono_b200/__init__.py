"""Monokernels for SGLang on NVIDIA B200 (sm_100a): the DeepSeek-V4.1 decode and
speculative-verify layer as a few hand-written CUDA launches a layer, including both TP
all-reduces, behind the reference plugin's surface (omirosh/sgl-amd-mono,
``sgl_amd_mono/__init__.py``).

SGLang holds the interface (``sglang.srt.monokernels``). This package holds the CUDA device
runtime (``common``: the C-ABI loader, peer exchange regions) and, per model, its specs and
their forwards (``<model>/spec.py``, ``<model>/draft.py``) and its kernels per ISA
(``<model>/sm100a/``). SGLang loads the package as a general plugin (``pyproject.toml``: the
``sglang.srt.plugins`` entry point), which registers each spec with SGLang's monokernel
framework.
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
