"""Shared fixtures. `-m gpu` tests need a CUDA device (a B200); everything else runs on CPU."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

# Test model shapes: dims of nibblemac_b200.pq presets, random init with a larger weight scale
# than the benchmark's 0.02 so that greedy decoding does not settle on one repeated token.
TEST_STD = 0.05


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (NVIDIA B200)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lib():
    from nibblemac_b200._lib import load_library
    return load_library()


@pytest.fixture(scope="session")
def q4k_oracle():
    from oracle import Q4KOracle
    return Q4KOracle()


def _model(name: str, seed: int, std: float, out_scale: float = 1.0) -> Path:
    from nibblemac_b200 import pq
    root = Path(os.environ.get("NB_MODEL_CACHE", ROOT / "_models"))
    tag = "" if out_scale == 1.0 else f"-out{out_scale}"
    path = root / f"test-{name}-s{seed}-std{std}{tag}.pq"
    if not path.exists():
        pq.make_synthetic(path, pq.PRESETS[name], seed, std=std, out_scale=out_scale)
    return path


@pytest.fixture(scope="session")
def looping_model() -> Path:
    """TINY dims with the residual-stream projections scaled down: greedy decoding repeats
    itself, so prompt lookup finds matches."""
    return _model("tiny", 3, TEST_STD, out_scale=0.02)


@pytest.fixture(scope="session")
def tiny_model() -> Path:
    return _model("tiny", 1, TEST_STD)


@pytest.fixture(scope="session")
def small_model() -> Path:
    return _model("small", 2, TEST_STD)


@pytest.fixture(scope="session")
def model_08b() -> Path:
    return _model("0.8b", 0, 0.02)


def ref_available() -> bool:
    return (ROOT / "oracle" / "_ref" / "libpinfer_ref.so").exists()
