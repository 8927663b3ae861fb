import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import torch

    def load(name):
        return torch.load(ROOT / "tests" / "golden" / f"{name}.pt", weights_only=False)

    return load


@pytest.fixture
def fake_sglang():
    """SGLang's monokernel interface as a test stand-in (tests/fake_sglang): importable as
    ``sglang`` for the test, then removed with every module that imported it."""
    path = str(ROOT / "tests" / "fake_sglang")
    sys.path.insert(0, path)
    before = set(sys.modules)
    try:
        import sglang.srt.monokernels.spec as registry
        registry._REGISTRY.clear()
        yield registry
    finally:
        sys.path.remove(path)
        for name in set(sys.modules) - before:
            if name.startswith(("sglang", "sgl_amd_mono_b200.deepseek_v41.spec",
                                "sgl_amd_mono_b200.deepseek_v41.draft")):
                del sys.modules[name]
        pkg = sys.modules.get("sgl_amd_mono_b200.deepseek_v41")
        for attr in ("spec", "draft"):
            if pkg is not None and hasattr(pkg, attr):
                delattr(pkg, attr)
