import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_PARENT = ROOT / "vllm-inference-engine_b200"
for p in (str(ROOT), str(PKG_PARENT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; parity tests of the CUDA path")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    gdir = ROOT / "tests" / "golden"
    arrays = dict(np.load(gdir / "golden.npz"))
    manifest = json.loads((gdir / "manifest.json").read_text())
    return arrays, manifest


@pytest.fixture(scope="session")
def cuda_ready():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import pagedkv._native as native

    native.lib()  # raises if the library is missing: no fallback
    return torch.device("cuda", 0)
