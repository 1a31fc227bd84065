"""The hot-path entry points registered as torch operators
(``torch.ops.praxis_b200.*``), for callers that trace or compile around
them (torch.compile, torch.export, FX) or want them in profiler traces by
name.

Each operator calls the C ABI through :mod:`ops` (no work in Python beyond
argument checks and output allocation) and has a fake implementation that
returns outputs of the right shapes and dtypes without touching a device, so
shape inference needs neither a GPU nor the library. The operators are
functional: they allocate their outputs and mutate none of their inputs.

    praxis_b200::router_logits(x, terms) -> (logits fp32 [T, E], row max bf16 [T])
    praxis_b200::route(logits, bias?, top_k, activation) -> (top_idx int64 [T, k], gate bf16 [T, k])
    praxis_b200::moe_forward(x, top_idx, gate, <bank>, scaling, shared?, layouts) -> bf16 [T, C]
    praxis_b200::moe_forward_routed(x, terms, bias?, top_k, activation, <bank>, scaling, shared?, layouts)
        -> (bf16 [T, C], top_idx, gate)

``<bank>`` is the kernel-layout bank of ``B200NVFP4RoutedExperts.kernel_weights()``
and its global scales: gate_up_q, gate_up_sf, gate_up_global, down_q, down_sf,
down_global. Layouts are the ``capi.SF_*`` values of the two scale buffers.
"""

# no postponed annotations here: torch.library reads the signatures
from typing import Optional

import torch
from torch import Tensor

from . import ops

BF16 = torch.bfloat16


@torch.library.custom_op("praxis_b200::router_logits", mutates_args=())
def router_logits(x: Tensor, terms: Tensor) -> tuple[Tensor, Tensor]:
    return ops.router_logits(x, terms)


@router_logits.register_fake
def _router_logits_fake(x: Tensor, terms: Tensor) -> tuple[Tensor, Tensor]:
    t, e = x.shape[0], terms.shape[1]
    return x.new_empty(t, e, dtype=torch.float32), x.new_empty(t, dtype=BF16)


@torch.library.custom_op("praxis_b200::route", mutates_args=())
def route(logits: Tensor, bias: Optional[Tensor], top_k: int, activation: str) -> tuple[Tensor, Tensor]:
    return ops.route(logits, bias, top_k, activation)


@route.register_fake
def _route_fake(logits: Tensor, bias: Optional[Tensor], top_k: int, activation: str) -> tuple[Tensor, Tensor]:
    t = logits.shape[0]
    return logits.new_empty(t, top_k, dtype=torch.int64), logits.new_empty(t, top_k, dtype=BF16)


@torch.library.custom_op("praxis_b200::moe_forward", mutates_args=())
def moe_forward(x: Tensor, top_idx: Tensor, gate: Tensor, gate_up_q: Tensor, gate_up_sf: Tensor,
                gate_up_global: Tensor, down_q: Tensor, down_sf: Tensor, down_global: Tensor, scaling: float,
                shared: Optional[Tensor], gate_up_sf_layout: int, down_sf_layout: int) -> Tensor:
    return ops.moe_forward(x, top_idx, gate, gate_up_q, gate_up_sf, gate_up_global, down_q, down_sf, down_global,
                           scaling, shared, gate_up_sf_layout=gate_up_sf_layout, down_sf_layout=down_sf_layout)


@moe_forward.register_fake
def _moe_forward_fake(x: Tensor, top_idx: Tensor, gate: Tensor, gate_up_q: Tensor, gate_up_sf: Tensor,
                      gate_up_global: Tensor, down_q: Tensor, down_sf: Tensor, down_global: Tensor, scaling: float,
                      shared: Optional[Tensor], gate_up_sf_layout: int, down_sf_layout: int) -> Tensor:
    return torch.empty_like(x)


@torch.library.custom_op("praxis_b200::moe_forward_routed", mutates_args=())
def moe_forward_routed(x: Tensor, terms: Tensor, bias: Optional[Tensor], top_k: int, activation: str,
                       gate_up_q: Tensor, gate_up_sf: Tensor, gate_up_global: Tensor, down_q: Tensor,
                       down_sf: Tensor, down_global: Tensor, scaling: float, shared: Optional[Tensor],
                       gate_up_sf_layout: int, down_sf_layout: int) -> tuple[Tensor, Tensor, Tensor]:
    return ops.moe_forward(x, None, None, gate_up_q, gate_up_sf, gate_up_global, down_q, down_sf, down_global,
                           scaling, shared, router_terms=terms, router_bias=bias, top_k=top_k, activation=activation,
                           gate_up_sf_layout=gate_up_sf_layout, down_sf_layout=down_sf_layout)


@moe_forward_routed.register_fake
def _moe_forward_routed_fake(x: Tensor, terms: Tensor, bias: Optional[Tensor], top_k: int, activation: str,
                             gate_up_q: Tensor, gate_up_sf: Tensor, gate_up_global: Tensor, down_q: Tensor,
                             down_sf: Tensor, down_global: Tensor, scaling: float, shared: Optional[Tensor],
                             gate_up_sf_layout: int, down_sf_layout: int) -> tuple[Tensor, Tensor, Tensor]:
    t = x.shape[0]
    return (torch.empty_like(x), x.new_empty(t, top_k, dtype=torch.int64), x.new_empty(t, top_k, dtype=BF16))


__all__ = ["moe_forward", "moe_forward_routed", "route", "router_logits"]
