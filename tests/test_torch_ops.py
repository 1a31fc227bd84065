"""The torch operator registrations (``torch.ops.praxis_b200.*``).

CPU: the operators exist and their fake implementations give the real
outputs' shapes and dtypes without a device (FakeTensorMode on "cuda").
GPU: each operator returns the bits of the direct ``ops`` call, and
``torch.library.opcheck`` accepts the schema and the fake implementation.
"""

from __future__ import annotations

import pytest
import torch
from conftest import pkg
from torch._subclasses.fake_tensor import FakeTensorMode

BF16 = torch.bfloat16


def test_operators_are_registered():
    pkg()
    for name in ("router_logits", "route", "moe_forward", "moe_forward_routed"):
        assert hasattr(torch.ops.praxis_b200, name), name


def test_fake_shapes_without_a_device():
    pkg()
    t, c, e, k, f = 100, 512, 8, 2, 256
    with FakeTensorMode():
        x = torch.empty(t, c, dtype=BF16, device="cuda")
        terms = torch.empty(3, e, c, dtype=BF16, device="cuda")
        logits, amax = torch.ops.praxis_b200.router_logits(x, terms)
        assert (logits.shape, logits.dtype, amax.shape, amax.dtype) == ((t, e), torch.float32, (t,), BF16)
        top, gate = torch.ops.praxis_b200.route(logits, None, k, "sigmoid")
        assert (top.shape, top.dtype, gate.shape, gate.dtype) == ((t, k), torch.int64, (t, k), BF16)
        bank = (torch.empty(e, 2 * f, c // 2, dtype=torch.uint8, device="cuda"),
                torch.empty(e, 2 * f, c // 16, dtype=torch.uint8, device="cuda"),
                torch.empty(e, device="cuda"),
                torch.empty(e, c, f // 2, dtype=torch.uint8, device="cuda"),
                torch.empty(e, c, f // 16, dtype=torch.uint8, device="cuda"),
                torch.empty(e, device="cuda"))
        y = torch.ops.praxis_b200.moe_forward(x, top, gate, *bank, 2.5, None, 0, 0)
        assert (y.shape, y.dtype) == ((t, c), BF16)
        y2, top2, gate2 = torch.ops.praxis_b200.moe_forward_routed(x, terms, None, k, "sigmoid", *bank, 2.5, None,
                                                                   0, 0)
        assert (y2.shape, top2.shape, top2.dtype, gate2.shape) == ((t, c), (t, k), torch.int64, (t, k))


@pytest.mark.gpu
def test_operators_match_direct_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    P = pkg()
    P.capi.load()
    dev = "cuda"
    t, c, e, k, f = 300, 512, 8, 2, 256
    g = torch.Generator().manual_seed(61)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(BF16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(BF16)
    bank = P.pack_routed_experts(gu.to(dev), down.to(dev), keep_on_device=True)
    bank.prepare()
    kw = bank.kernel_weights()
    x = torch.randn(t, c, generator=g).to(BF16).to(dev)
    terms = P.ops.split_router_weight((torch.randn(e, c, generator=g) * 0.05).to(dev))
    bias = torch.zeros(e, device=dev)
    weights = (kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q, kw.down_sf, bank.down_global)
    layouts = (kw.gate_up_sf_layout, kw.down_sf_layout)

    logits, amax = torch.ops.praxis_b200.router_logits(x, terms)
    want_l, want_a = P.ops.router_logits(x, terms)
    assert torch.equal(logits, want_l) and torch.equal(amax.view(torch.int16), want_a.view(torch.int16))
    top, gate = torch.ops.praxis_b200.route(logits, bias, k, "sigmoid")
    want_t, want_g = P.ops.route(logits, bias, k, "sigmoid")
    assert torch.equal(top, want_t) and torch.equal(gate.view(torch.int16), want_g.view(torch.int16))
    y = torch.ops.praxis_b200.moe_forward(x, top, gate, *weights, 2.5, None, *layouts)
    want_y = P.ops.moe_forward(x, top, gate, *weights, 2.5, None, gate_up_sf_layout=layouts[0],
                               down_sf_layout=layouts[1])
    assert torch.equal(y.view(torch.int16), want_y.view(torch.int16))
    y2, top2, gate2 = torch.ops.praxis_b200.moe_forward_routed(x, terms, bias, k, "sigmoid", *weights, 2.5, None,
                                                               *layouts)
    assert torch.equal(top2, top) and torch.equal(y2.view(torch.int16), want_y.view(torch.int16))

    torch.library.opcheck(torch.ops.praxis_b200.route.default, (logits, bias, k, "sigmoid"),
                          test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(torch.ops.praxis_b200.moe_forward.default, (x, top, gate, *weights, 2.5, None, *layouts),
                          test_utils=("test_schema", "test_faketensor"))
