"""Routing + dispatch against the reference's own sm_100 kernel pair on the
same GPU: ``router_fused.route_dispatch`` (praxis/kernels/router_fused.py:
738-804, CuTe DSL, E = 128, top-8, P = 1 or 2), imported from the offline
install of the reference under ``baseline/_ref`` when that install and the
CUTLASS DSL are present (skipped otherwise).

Bar: bit-exact on identical fp32 logits for every output of the reference's
``Routing`` (top_idx, gate, order, inverse, sorted_gate, tokens, tokens32,
seg_csr, offsets), with and without tie-heavy logits.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from conftest import assert_bytes_equal, pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


@pytest.fixture(scope="module")
def rf():
    if not (REF / "praxis" / "kernels" / "router_fused.py").is_file():
        pytest.skip("the reference install (baseline/_ref) is absent")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    try:
        import cutlass.cute  # noqa: F401
        from praxis.kernels import router_fused
    except Exception as exc:  # the CUTLASS DSL or a reference dependency is missing
        pytest.skip(f"reference router_fused not importable: {type(exc).__name__}: {exc}")
    try:  # the kernel imports more of the DSL when it is first compiled
        router_fused.route_dispatch(torch.zeros(64, 128, device=DEV), torch.zeros(128, device=DEV), (64,))
    except ImportError as exc:
        pytest.skip(f"reference router_fused does not build with this CUTLASS DSL: {exc}")
    return router_fused


@pytest.mark.parametrize("rows", [(4096,), (1000, 3000), (16384,), (1, 777)])
@pytest.mark.parametrize("ties", [False, True])
def test_route_dispatch_bit_exact_vs_reference_kernel(P, rf, rows, ties):
    t = sum(rows)
    g = torch.Generator().manual_seed(t + int(ties))
    logits = torch.randn(t, 128, generator=g)
    if ties:
        logits = (logits * 4).round() / 4  # many equal scores per row
    bias = (torch.randn(128, generator=g) * 0.05).float()
    if ties:
        bias = (bias * 8).round() / 8
    logits, bias = logits.to(DEV).contiguous(), bias.to(DEV).contiguous()
    ref = rf.route_dispatch(logits, bias, rows)
    ours = P.ops.route_dispatch(logits, bias, rows, top_k=8)
    for name in ("top_idx", "gate", "order", "inverse", "sorted_gate", "tokens", "tokens32", "seg_csr"):
        assert_bytes_equal(getattr(ours, name), getattr(ref, name))
    assert_bytes_equal(ours.offsets.contiguous(), ref.offsets)
