"""Shared test setup: the ``gpu`` marker, import paths and golden fixtures."""

from __future__ import annotations

import hashlib
import importlib
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def pkg():
    """The product package (its directory name is not an identifier)."""
    return importlib.import_module("praxis-1-oss_b200")


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def routing_inputs(seed: int, tokens: int, dim: int, experts: int, bias_scale: float):
    """Same recipe as tests/golden/make_golden.py."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, dim, generator=g).to(torch.bfloat16)
    w = (torch.randn(experts, dim, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.randn(experts, generator=g) * bias_scale
    return x, w, bias


_GOLDEN_CACHE: dict = {}


def golden() -> dict:
    if "ref" not in _GOLDEN_CACHE:
        _GOLDEN_CACHE["ref"] = torch.load(GOLDEN / "reference_cpu.pt", weights_only=False)
    return _GOLDEN_CACHE["ref"]


def assert_bytes_equal(actual: torch.Tensor, expected: torch.Tensor) -> None:
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    assert actual.dtype == expected.dtype, (actual.dtype, expected.dtype)
    a = actual.detach().cpu().contiguous().view(torch.uint8)
    b = expected.detach().cpu().contiguous().view(torch.uint8)
    if not torch.equal(a, b):
        diff = (a != b).nonzero()
        raise AssertionError(f"{diff.shape[0]} bytes differ; first at {diff[:5].tolist()}")


@pytest.fixture
def cuda_lib():
    """The loaded C-ABI library on a B200; skips without a GPU."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    lib = pkg().capi.load()
    return lib
