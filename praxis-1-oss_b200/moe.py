"""``B200MoEFeedForward``: the MoE module of praxis/layers.py:1584-1631 with
the router and the routed experts on this library's sm_100a kernels.

Constructor, state-dict keys (``router.weight``, ``expert_bias``,
``routed.*`` packed NVFP4 buffers, ``shared.gate_up``, ``shared.down``) and the
forward contract follow the reference module; the routed bank is a
``B200NVFP4RoutedExperts``. The shared expert stays a torch bf16 SwiGLU (the
reference's ``SharedExpert``, praxis/layers.py:1033-1089), added after the
routed sum is rounded to bf16.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import ops
from .bank import B200NVFP4RoutedExperts, pack_routed_experts, routed_forward_tail
from .ops import Tail

_NVTX = os.environ.get("PRAXIS_NVTX", "0") not in ("", "0")


class _Range:
    """``praxis::moe:<name>`` NVTX range (praxis/nvtx.py naming) when PRAXIS_NVTX=1."""

    def __init__(self, name: str) -> None:
        self.name = name

    def __enter__(self):
        if _NVTX:
            torch.cuda.nvtx.range_push(f"praxis::moe:{self.name}")

    def __exit__(self, *exc):
        if _NVTX:
            torch.cuda.nvtx.range_pop()


class SharedExpert(nn.Module):
    """The always-on dense SwiGLU expert (praxis/layers.py:1033-1089)."""

    def __init__(self, dim: int, hidden: int) -> None:
        super().__init__()
        self.gate_up = nn.Parameter(torch.empty(dim, 2 * hidden))
        self.down = nn.Parameter(torch.empty(hidden, dim))

    def forward(self, x: Tensor, out: Tensor | None = None) -> Tensor:
        """``out``: a [rows, C] destination for 2-D ``x`` (the same GEMM)."""
        gate, up = (x @ self.gate_up).chunk(2, dim=-1)
        if out is not None:
            return torch.mm(F.silu(gate) * up, self.down, out=out)
        return (F.silu(gate) * up) @ self.down


class B200MoEFeedForward(nn.Module):
    """Router (sigmoid or softmax) + top-k routed NVFP4 experts + optional
    shared expert, inference only.

    ``routing_hook`` (praxis/layers.py:1595-1602): None at inference; a
    callable ``hook(layer, logits, top_idx)`` set by training or diagnostics
    code is called after the routing and before the experts with the float32
    router logits and the picked experts.
    """

    expert_bias: Tensor
    routing_hook = None

    def __init__(
        self,
        dim: int = 3072,
        hidden: int = 1280,
        num_experts: int = 128,
        top_k: int = 8,
        routed_scaling_factor: float = 2.5,
        dispatch_chunk_size: int | None = None,
        *,
        router_activation: str = "sigmoid",
        shared_expert: bool = True,
    ) -> None:
        super().__init__()
        if dispatch_chunk_size is not None and dispatch_chunk_size <= 0:
            raise ValueError("dispatch_chunk_size must be positive")
        if router_activation not in ("sigmoid", "softmax"):
            raise ValueError("router_activation must be 'sigmoid' or 'softmax'")
        self.dim, self.hidden = dim, hidden
        self.dispatch_chunk_size = dispatch_chunk_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.routed_scaling_factor = routed_scaling_factor
        self.router_activation = router_activation
        self.router = nn.Linear(dim, num_experts, bias=False)
        self.routed: B200NVFP4RoutedExperts | None = None
        self.shared = SharedExpert(dim, hidden) if shared_expert else None
        self.register_buffer("expert_bias", torch.zeros(num_experts))
        self._router_terms: Tensor | None = None

    def _apply(self, fn, recurse: bool = True):
        bias = self.expert_bias
        super()._apply(fn, recurse)
        # The routing bias stays float32 under dtype casts (praxis/layers.py:1617-1622).
        self.expert_bias = bias.to(device=self.expert_bias.device)
        self._router_terms = None
        return self

    def set_routed_weights(self, gate_up_weight: Tensor, down_weight: Tensor) -> None:
        """Pack expert-first bf16 banks [E,C,2H] / [E,H,C] on the GPU."""
        self.routed = pack_routed_experts(gate_up_weight, down_weight, keep_on_device=True)

    @classmethod
    def from_reference(cls, layer: nn.Module) -> B200MoEFeedForward:
        """Build from a reference ``praxis.layers.MoEFeedForward`` whose routed
        bank is either ``RoutedExperts`` (bf16, packed here on the GPU) or
        ``NVFP4RoutedExperts`` (buffers reused as they are)."""
        router_w = layer.router.weight
        e, c = router_w.shape
        routed = layer.routed
        if hasattr(routed, "gate_up_q"):
            h = routed.down_q.shape[2] * 2
        else:
            h = routed.gate_up_weight.shape[2] // 2
        new = cls(c, h, e, layer.top_k, layer.routed_scaling_factor, layer.dispatch_chunk_size,
                  shared_expert=getattr(layer, "shared", None) is not None)
        with torch.no_grad():
            new.router.weight = nn.Parameter(router_w.detach().clone(), requires_grad=False)
            new.expert_bias = layer.expert_bias.detach().clone().float()
            if new.shared is not None:
                new.shared.gate_up = nn.Parameter(layer.shared.gate_up.detach().clone(), requires_grad=False)
                new.shared.down = nn.Parameter(layer.shared.down.detach().clone(), requires_grad=False)
        if hasattr(routed, "gate_up_q"):
            state = {name: buf.detach().cpu().contiguous() for name, buf in routed.named_buffers()
                     if name in ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf",
                                 "down_global", "_unit_alpha")}
            new.routed = B200NVFP4RoutedExperts.from_packed(state)
        else:
            new.set_routed_weights(routed.gate_up_weight.detach().to(torch.bfloat16),
                                   routed.down_weight.detach().to(torch.bfloat16))
        return new

    def router_terms(self) -> Tensor:
        """The router weight as bf16 terms for the tensor-core logits kernel."""
        w = self.router.weight
        if self._router_terms is None or self._router_terms.device != w.device:
            self._router_terms = ops.split_router_weight(w.detach())
        return self._router_terms

    @torch.no_grad()
    def route(self, x_flat: Tensor) -> tuple[Tensor, Tensor]:
        """(top_idx, gate) of ``MoEFeedForward._route`` (praxis/layers.py:1632-1655)."""
        with _Range("router"):
            logits, _ = ops.router_logits(x_flat, self.router_terms())
        with _Range("topk_dispatch"):
            bias = self.expert_bias.to(device=x_flat.device, dtype=torch.float32).contiguous()
            top_idx, gate = ops.route(logits, bias, self.top_k, self.router_activation)
        if self.routing_hook is not None:
            self.routing_hook(self, logits, top_idx)
        return top_idx, gate

    @staticmethod
    def _check_router_rows(x: Tensor, router_rows) -> None:
        """``router_rows = (r0, r1, total)`` (praxis/layers.py:2122-2165): x
        holds query rows r0..r1 of a sequence of ``total`` tokens whose context
        rows were left out. The reference pads x back to ``total`` rows with
        zeros so that its fp32 router GEMM keeps the full call's row-chunk
        shapes; the logits kernel here computes every row on its own, in an
        order that does not depend on the number of rows, so the query rows'
        logits are those of the padded call and no padding is needed."""
        if (
            not isinstance(router_rows, tuple)
            or len(router_rows) != 3
            or not all(isinstance(v, int) and not isinstance(v, bool) for v in router_rows)
        ):
            raise ValueError("router_rows must be a tuple (r0, r1, total) of ints")
        r0, r1, total = router_rows
        if not 0 <= r0 <= r1 <= total:
            raise ValueError(f"router_rows {router_rows}: need 0 <= r0 <= r1 <= total")
        if x.dim() < 2 or x.shape[-2] != r1 - r0:
            raise ValueError(f"router_rows {router_rows}: x must hold r1 - r0 = {r1 - r0} rows per sequence")

    @torch.no_grad()
    def forward_tail(self, x: Tensor, residual: Tensor, norm: nn.Module | None = None, scale=None, *,
                     mod: Tensor | None = None, modfma: bool = True, geom=None
                     ) -> tuple[Tensor, Tensor | None]:
        """``forward(x)`` fused into what follows it in the reference's
        MOE_TAIL_NORM path (praxis/layers.py:429-441): the residual add
        ``residual + y`` and, with ``norm`` (the reference's zero-centred
        RMSNorm: ``weight``, ``eps``) and ``scale``, the next block's
        ``norm(residual + y) * scale`` — with ``mod`` ([R, 2C] shift | scale
        rows, ``geom`` the (RF, RC, NREG, PW, WD, PH) of ``CompactMod`` or
        None) its modulation in between — as ``tail_residual_add``,
        ``tail_add_norm_scale`` and ``tail_add_mod_norm_scale`` of
        praxis/kernels/moe_tail_triton.py:329-445 compute them. Returns
        ``(new residual, normed rows or None)`` with the eager bits; the
        routed combine, the shared add, the residual add, the modulation and
        the norm run as the last kernel of the routed forward."""
        if self.routed is None:
            raise RuntimeError("routed experts are not set (set_routed_weights / from_reference)")
        if (norm is None) != (scale is None):
            raise ValueError("norm and scale go together")
        shape = x.shape
        c = x.size(-1)
        x_flat = x.reshape(-1, c).contiguous()
        top_idx, gate = self.route(x_flat)
        y_shared = self.shared(x_flat).contiguous() if self.shared is not None else None
        tail = Tail(residual=residual.reshape(-1, c).contiguous())
        if norm is not None:
            tail = tail._replace(norm_weight=(1 + norm.weight.detach().to(torch.float32)).contiguous(),
                                 eps=float(norm.eps), norm_scale=float(torch.as_tensor(scale).float()))
        if mod is not None:
            tail = tail._replace(mod=mod.reshape(-1, 2 * c).contiguous(), mod_fma=bool(modfma),
                                 mod_geom=None if geom is None else tuple(int(v) for v in geom))
        chunk = self.dispatch_chunk_size or max(1, x_flat.shape[0])
        with _Range("routed"):
            xo, h = routed_forward_tail(self.routed, x_flat, top_idx, gate, scaling=self.routed_scaling_factor,
                                        chunk_size=chunk, tail=tail, shared=y_shared)
        return xo.reshape(shape), None if h is None else h.reshape(shape)

    @torch.no_grad()
    def forward_pair(self, xs) -> list[Tensor]:
        """``[self(x) for x in xs]`` with one routed-expert pass for both
        inputs of a classifier-free-guidance pair (``MoEFeedForward.forward_pair``,
        praxis/layers.py:1779-1853): the router and the gates run on both
        inputs' rows at once (row-wise kernels, so each row's bits are those
        of its own call), the shared expert per input, and the routed bank's
        ``routed_forward_pair`` sends both inputs' routed rows through the
        expert GEMMs once, grouped per (expert, input) so that every output
        has the bits of ``forward``. Falls back to one forward per input where
        the pair does not apply (the reference's conditions: two inputs, each
        one dispatch chunk, no routing hook)."""
        xs = list(xs)
        if self.routed is None:
            raise RuntimeError("routed experts are not set (set_routed_weights / from_reference)")
        flats = [x.reshape(-1, x.size(-1)) for x in xs]
        chunk = self.dispatch_chunk_size
        if (
            len(xs) != 2
            or self.routing_hook is not None
            or any(not f.is_cuda or f.dtype != torch.bfloat16 or f.device != flats[0].device for f in flats)
            or any(not 0 < f.shape[0] <= (chunk or f.shape[0]) for f in flats)
        ):
            return [self(x) for x in xs]
        from .bank import _adjacent

        flats = [f.contiguous() for f in flats]
        t0 = flats[0].shape[0]
        x = _adjacent(flats)
        top_idx, gate = self.route(x)
        shared = None
        if self.shared is not None:
            y_sh = torch.empty_like(x)
            self.shared(flats[0], out=y_sh[:t0])
            self.shared(flats[1], out=y_sh[t0:])
            shared = [y_sh[:t0], y_sh[t0:]]
        with _Range("routed"):
            ys = self.routed.routed_forward_pair(
                [x[:t0], x[t0:]], [top_idx[:t0], top_idx[t0:]], [gate[:t0], gate[t0:]],
                scaling=self.routed_scaling_factor, shared=shared)
        return [y.reshape(xi.shape) for y, xi in zip(ys, xs, strict=True)]

    @torch.no_grad()
    def forward(self, x: Tensor, *, router_rows: tuple[int, int, int] | None = None) -> Tensor:
        """``MoEFeedForward.forward`` (praxis/layers.py:2122-2199), the same
        keyword (called as ``self.ffn(normed, router_rows=rows)`` by the
        reference's transformer block, praxis/layers.py:2515)."""
        if self.routed is None:
            raise RuntimeError("routed experts are not set (set_routed_weights / from_reference)")
        if router_rows is not None:
            self._check_router_rows(x, router_rows)
        shape = x.shape
        x_flat = x.reshape(-1, x.size(-1)).contiguous()
        top_idx, gate = self.route(x_flat)
        y_shared = self.shared(x_flat) if self.shared is not None else None
        chunk = self.dispatch_chunk_size or max(1, x_flat.shape[0])
        with _Range("routed"):
            if y_shared is None:
                out = self.routed.routed_forward(x_flat, top_idx, gate, scaling=self.routed_scaling_factor,
                                                 chunk_size=chunk)
            else:
                out = self.routed.routed_forward_with_shared(
                    x_flat, top_idx, gate, scaling=self.routed_scaling_factor, chunk_size=chunk,
                    shared=y_shared.contiguous())
        return out.reshape(shape)
