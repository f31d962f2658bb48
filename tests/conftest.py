"""Shared fixtures.  Tests marked ``gpu`` need a B200 and the built library."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built library")
    config.addinivalue_line("markers", "slow: takes tens of seconds of CPU")


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory) -> Path:
    from breezetoken_b200.synth import QWEN35_TINY, write_qwen35_gguf

    return write_qwen35_gguf(tmp_path_factory.mktemp("tiny") / "tiny.gguf", QWEN35_TINY, seed=0)


@pytest.fixture(scope="session")
def gguf_0_8b(tmp_path_factory) -> Path:
    from breezetoken_b200.synth import QWEN35_0_8B, write_qwen35_gguf

    return write_qwen35_gguf(tmp_path_factory.mktemp("q35") / "q35.gguf", QWEN35_0_8B, seed=0)


@pytest.fixture(scope="session")
def qwen36_tiny_gguf(tmp_path_factory) -> Path:
    from breezetoken_b200.synth import QWEN36_TINY, write_qwen36_gguf

    return write_qwen36_gguf(tmp_path_factory.mktemp("q36") / "q36.gguf", QWEN36_TINY, seed=4)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    from breezetoken_b200 import _native

    _native.load()
    return torch.device("cuda")
