"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on
CPU (oracle, host logic, the C-ABI library's exports and error paths)."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

PKG_NAME = "yallma3-mini-inference_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    config.addinivalue_line("markers", "slow: long-running parity case")


def load_package():
    lib = ROOT / PKG_NAME / "libyallma3_b200.so"
    if not lib.exists():
        build = importlib.import_module(f"{PKG_NAME}.build")
        build.build()
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def yl():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    import pyoracle
    pyoracle.build()
    return pyoracle


@pytest.fixture(scope="session")
def model_factory(tmp_path_factory, yl):
    """model_factory(preset, **overrides) -> path of a cached synthetic GGUF."""
    root = tmp_path_factory.mktemp("models")
    cache: dict = {}

    def make(preset: str, **over) -> str:
        key = (preset, tuple(sorted(over.items())))
        if key not in cache:
            name = preset + "".join(f"_{k}{int(v) if isinstance(v, bool) else v}" for k, v in sorted(over.items()))
            path = root / f"{name}.gguf"
            yl.synth_preset(preset, str(path), **over)
            cache[key] = str(path)
        return cache[key]

    return make


@pytest.fixture(scope="session")
def golden():
    g = ROOT / "tests" / "golden"
    return {"quant": np.load(g / "quantize_q8.npz"), "matmul": np.load(g / "matmul_q8.npz")}


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    torch.cuda.init()
    return torch
