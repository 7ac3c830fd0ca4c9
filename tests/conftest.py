import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "thompiler-emmy-hackathon_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden" / "packages"
PACKAGES = sorted(d.name for d in GOLDEN.iterdir() if (d / "meta.json").exists())


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
