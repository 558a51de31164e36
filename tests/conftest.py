"""Shared test setup: marker registration and fixture paths.

`-m gpu` tests need a CUDA device (B200) and call the engine through its C ABI; everything
else runs on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

FIXTURES = ["tiny_llama_q8_0", "tiny_llama_q4_0", "tiny_gpt2_q8_0"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; runs the engine through its C ABI")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN
