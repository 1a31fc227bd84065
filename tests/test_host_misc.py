"""Host-side checks that need no GPU: argument validation of the
expert-parallel helpers and the bench's algorithmic-byte bookkeeping."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest
from conftest import pkg

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("bench_module", mod)
    spec.loader.exec_module(mod)
    return mod


def test_peer_exchange_rejects_a_bad_sm_copy_fraction():
    P = pkg()
    for frac in (-0.1, 1.5):
        with pytest.raises(ValueError):
            P.expert_parallel.PeerExchange(None, "cpu", sm_copy_fraction=frac)


def test_gate_up_algorithmic_bytes_match_the_config_2_budget():
    b = _bench()
    t, k, c, f, e = 16384, 4, 3072, 1536, 64
    got = b.gemm1_bytes(t, k, c, f, e)
    weights = e * 2 * f * c // 2 + e * 2 * f * c // 16
    rows = t * k * c // 2 + t * k * c // 16 + t * k * f * 2
    assert got == weights + rows == 654_311_424
    # the measured DRAM traffic of one launch reads every byte about once:
    # within the replicated scale layout's extra scale bytes and the padding
    # rows (at most 127 per expert) of the activations
    traffic = b.GEMM1_TRAFFIC[("2", t)]
    extra = 3 * (e * 2 * f * c // 16 + t * k * c // 16)
    padding = e * 127 * (c // 2 + 4 * c // 16)
    assert got * 0.9 < traffic < got + extra + padding


def test_bench_configs_cover_the_baseline_shapes():
    b = _bench()
    for name in ("1", "2", "3", "4", "5", "ckpt"):
        cfg = b.CONFIGS[name]
        assert cfg["dim"] % 64 == 0 and cfg["hidden"] % 128 == 0 and cfg["top_k"] <= cfg["experts"]
