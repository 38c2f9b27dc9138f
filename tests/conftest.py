import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); parity tests through the C ABI")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on a CPU-only host)")
    return torch.device("cuda:0")


FAKES = os.path.join(REPO, "tests", "fakes")


@pytest.fixture
def fake_kitchen(monkeypatch):
    """Put the comfy_kitchen test double (tests/fakes) on the path with a fresh registry."""
    monkeypatch.syspath_prepend(FAKES)
    for name in [m for m in sys.modules if m == "comfy_kitchen" or m.startswith("comfy_kitchen.")]:
        monkeypatch.delitem(sys.modules, name)
    import comfy_kitchen.registry as reg

    from tilegen_b200.comfyui import backend

    monkeypatch.setattr(backend, "_INSTALLED", False)
    monkeypatch.setattr(backend, "_FAILED_FHT_SHAPES", set())
    yield reg.registry
