"""Shared test setup: import paths, the `gpu` marker and seeded random-init model fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "mac-gpu-compiler_b200"
for p in (PKG, ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def tiny_model_path():
    import randmodel
    return randmodel.make_model("tiny", 0)


@pytest.fixture(scope="session")
def mid_model_path():
    import randmodel
    return randmodel.make_model("mid", 0)


@pytest.fixture(scope="session")
def full_model_path():
    import randmodel
    return randmodel.make_model("qwen3-0.6b", 0)
