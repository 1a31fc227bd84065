"""The C ABI library and the host-side logic, without a GPU.

The library loads on a machine without a GPU (static CUDA runtime); host-only
entry points are called, device entry points are not.
"""

from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch
from conftest import ROOT, pkg

HEADER = ROOT / "include" / "praxis_b200_moe.h"


@pytest.fixture(scope="module")
def lib():
    p = pkg()
    p.build.build()
    return p.capi.load()


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(praxis_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    # the ctypes stub binds exactly the declared functions
    assert sorted(pkg().capi.SIGNATURES) == names


def test_library_is_built_for_sm100a_only():
    text = Path(pkg().build.__file__).read_text()
    assert "arch=compute_100a,code=sm_100a" in text


def test_host_helpers(lib):
    assert lib.praxis_b200_abi_version() == pkg().capi.ABI_VERSION == 4
    assert lib.praxis_b200_padded_rows(65536, 64) == (65536 + 127 * 64) // 128 * 128
    assert pkg().ops.padded_rows(512, 8) == lib.praxis_b200_padded_rows(512, 8)
    ws = lib.praxis_b200_moe_workspace_size(16384, 4, 64, 3072, 1536, 1, 1)
    assert ws > 16384 * 4 * 3072 * 2  # holds the routed output rows
    # a lockstep pair pads every (expert, input) group on its own
    ws2 = lib.praxis_b200_moe_workspace_size(16384, 4, 64, 3072, 1536, 1, 2)
    assert ws2 > ws
    assert lib.praxis_b200_dispatch_passes_workspace_size(16384, 4, 64, 2) == \
        lib.praxis_b200_dispatch_workspace_size(16384, 4, 128)


def test_argument_errors_before_launch(lib):
    # Null args are rejected before any device work (device 0 may not exist).
    rc = lib.praxis_b200_moe_forward(None)
    assert rc == pkg().capi.EINVAL
    assert b"null" in lib.praxis_b200_last_error()


def test_router_weight_split_is_exact():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(64, 512, generator=g) * 0.02
    terms = pkg().ops.split_router_weight(w)
    assert terms.shape == (3, 64, 512) and terms.dtype == torch.bfloat16
    recon = terms[0].double() + terms[1].double() + terms[2].double()
    assert torch.equal(recon.float(), w)
    assert pkg().ops.split_router_weight(w.to(torch.bfloat16)).shape == (1, 64, 512)


def packed_state(e=2, c=128, h=128):
    return {
        "gate_up_q": torch.zeros(e, 2 * h, c // 2, dtype=torch.uint8),
        "gate_up_sf": torch.zeros(e, 2 * h, c // 16, dtype=torch.uint8),
        "gate_up_global": torch.ones(e),
        "down_q": torch.zeros(e, c, h // 2, dtype=torch.uint8),
        "down_sf": torch.zeros(e, c, h // 16, dtype=torch.uint8),
        "down_global": torch.ones(e),
        "_unit_alpha": torch.ones(e),
    }


@pytest.mark.parametrize(
    "kind", ["missing", "extra", "shape", "dtype", "global_nan", "global_zero", "scale_nan", "scale_negative", "alpha"]
)
def test_bank_rejects_corrupt_packed_state(kind):
    # tests/test_nvfp4.py:108-134 of the reference, against this bank.
    state = packed_state()
    if kind == "missing":
        del state["down_q"]
    elif kind == "extra":
        state["bf16_master"] = torch.ones(1)
    elif kind == "shape":
        state["down_q"] = state["down_q"][:, :, :1].contiguous()
    elif kind == "dtype":
        state["gate_up_global"] = state["gate_up_global"].to(torch.bfloat16)
    elif kind.startswith("global"):
        state["gate_up_global"][0] = float("nan") if kind == "global_nan" else 0
    elif kind.startswith("scale"):
        state["down_sf"].flatten()[0] = 127 if kind == "scale_nan" else 184
    else:
        state["_unit_alpha"][0] = 2
    with pytest.raises(ValueError):
        pkg().B200NVFP4RoutedExperts.from_packed(state)


def test_bank_is_inference_only_and_dtype_rejection_is_atomic():
    # tests/test_nvfp4.py:137-162 of the reference, against this bank.
    bank = pkg().B200NVFP4RoutedExperts.from_packed(packed_state())
    originals = dict(bank.named_buffers())
    assert bank.to("cpu") is bank
    with pytest.raises(TypeError, match="dtype"):
        bank.to(torch.bfloat16)
    assert all(bank.get_buffer(name) is value for name, value in originals.items())
    with pytest.raises(RuntimeError, match="inference"):
        bank.train()
    x = torch.ones(3, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA BF16"):
        bank.routed_forward(x, torch.zeros(3, 1, dtype=torch.int64), torch.ones(3, 1, dtype=torch.bfloat16),
                            scaling=2.5, chunk_size=2)
    with pytest.raises(RuntimeError, match="inference"):
        bank.routed_forward(x.requires_grad_(), torch.zeros(3, 1, dtype=torch.int64),
                            torch.ones(3, 1, dtype=torch.bfloat16), scaling=2.5, chunk_size=2)
    assert set(bank.state_dict()) == set(packed_state())


@pytest.mark.parametrize("kind", ["float32", "noncontiguous", "gradient"])
def test_shared_output_fallback_preserves_native_addition(monkeypatch, kind):
    # tests/test_nvfp4.py:242-269 of the reference, against this bank.
    bank = pkg().B200NVFP4RoutedExperts.from_packed(packed_state())
    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    routed = torch.randn_like(x)
    shared = torch.randn_like(x)
    if kind == "float32":
        shared = shared.float()
    elif kind == "noncontiguous":
        shared = torch.randn(128, 2, dtype=torch.bfloat16).T
    else:
        shared.requires_grad_(True)
    monkeypatch.setattr(bank, "routed_forward", lambda *a, **kw: routed)
    actual = bank.routed_forward_with_shared(x, torch.zeros(2, 1, dtype=torch.int64),
                                             torch.ones(2, 1, dtype=torch.bfloat16), scaling=2.5, chunk_size=2,
                                             shared=shared)
    expected = routed + shared
    assert actual.dtype == expected.dtype
    assert torch.equal(actual.view(torch.uint8), expected.view(torch.uint8))


def test_ops_refuse_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        pkg().ops.row_amax(torch.zeros(4, 128, dtype=torch.bfloat16))


def test_from_packed_requires_cpu_buffers_like_the_reference():
    # praxis/quantization/nvfp4.py:163-177: reconstruction starts from CPU buffers
    state = {name: v.to("meta") for name, v in packed_state().items()}
    with pytest.raises(ValueError, match="CPU"):
        pkg().B200NVFP4RoutedExperts.from_packed(state)
    assert pkg().B200NVFP4RoutedExperts.ACCEPTS_DISPATCH is False


@pytest.mark.parametrize("rows,ok", [
    ((0, 4, 4), True), ((2, 6, 10), True), ((3, 2, 10), False), ((0, 4, 3), False), ((0, 5, 8), False),
    ([0, 4, 4], False), ((0, 4), False), ((0.0, 4, 4), False),
])
def test_module_router_rows_keyword(rows, ok):
    """``forward(x, router_rows=(r0, r1, total))`` as the reference's block
    calls it (praxis/layers.py:2515): x holds r1 - r0 query rows."""
    x = torch.zeros(2, 4, 128, dtype=torch.bfloat16)
    check = pkg().B200MoEFeedForward._check_router_rows
    if ok:
        check(x, rows)
    else:
        with pytest.raises(ValueError):
            check(x, rows)


def test_module_forward_signature_matches_the_reference():
    import inspect

    sig = inspect.signature(pkg().B200MoEFeedForward.forward)
    assert list(sig.parameters) == ["self", "x", "router_rows"]
    assert sig.parameters["router_rows"].kind is inspect.Parameter.KEYWORD_ONLY
    assert pkg().B200MoEFeedForward.routing_hook is None
