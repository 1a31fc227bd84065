"""Expert parallelism for the routed NVFP4 bank (one process per GPU).

Rank r of R owns experts [r * E/R, (r + 1) * E/R); the router weights, the
expert bias and the shared expert are replicated. One layer forward on each
rank (its own tokens are one dispatch chunk):

1. route + row max |x| of the local tokens, dispatch into the expert-major
   padded layout (expert-major = destination-rank-major, since each rank's
   experts are contiguous), per-expert activation global scales of the local
   tokens (the reference's per-expert, per-chunk scale);
2. NVFP4 quantization of the outbound rows on the source rank;
3. exchange of the per-(destination, expert) counts, padded offsets and
   global scales (one small all-to-all), then of the FP4 rows and their
   compact scale atoms: destination d receives rows
   [pcsr[d * E/R], pcsr[(d + 1) * E/R]) of every source, whole 128-row tiles,
   so the swizzled scale atoms travel as contiguous bytes;
4. on the expert rank: gate/up GEMM + SwiGLU, hidden quantize with one global
   scale per (source, expert) segment, down GEMM + rescale
   (``praxis_b200_expert_forward``);
5. the bf16 rows travel back (the reverse all-to-all) into the source's own
   padded layout, and the source combines its tokens with the reference's
   four-accumulator order.

Every row meets the same arithmetic as on one GPU, so a rank's output equals
the single-GPU layer on that rank's tokens bit for bit. The exchange step
needs one device-to-host read of the split sizes per forward.

The compute steps go through a backend object (``CudaBackend``: this
library's kernels); the exchange logic is backend-independent so that it can
be exercised with CPU tensors over gloo.
"""

from __future__ import annotations

from collections.abc import Mapping

import torch
import torch.distributed as dist
from torch import Tensor

from . import ops
from .bank import B200NVFP4RoutedExperts


def shard_packed_state(state: Mapping[str, Tensor], rank: int, world: int) -> dict[str, Tensor]:
    """The packed buffers of experts [rank * E/world, (rank + 1) * E/world)."""
    e = state["gate_up_q"].shape[0]
    if e % world:
        raise ValueError(f"{e} experts do not shard evenly over {world} ranks")
    lo, hi = rank * e // world, (rank + 1) * e // world
    return {name: value[lo:hi].contiguous() for name, value in state.items()}


class CudaBackend:
    """The compute steps on this library's sm_100a kernels."""

    def __init__(self, bank: B200NVFP4RoutedExperts) -> None:
        self.bank = bank

    def route_rows(self, x: Tensor, top_idx: Tensor, gate: Tensor, num_experts: int):
        return ops.dispatch(top_idx, gate, num_experts, ops.row_amax(x), full=False)

    def quantize(self, x: Tensor, routing) -> tuple[Tensor, Tensor]:
        return ops.quantize_gather(x, routing, routing.act_global)

    def experts(self, q: Tensor, sf: Tensor, counts: Tensor, starts: Tensor, act_global: Tensor) -> Tensor:
        kw = self.bank.kernel_weights()
        b = self.bank
        return ops.expert_forward(q, sf, counts, starts, act_global, kw.gate_up_q, kw.gate_up_sf, b.gate_up_global,
                                  b.down_q, kw.down_sf, b.down_global, weight_sf_layout=kw.sf_layout)

    def combine(self, rows: Tensor, routing, scaling: float, shared: Tensor | None) -> Tensor:
        return ops.combine(rows, routing, scaling, rows_rescaled=True, shared=shared)


def exchange_forward(x: Tensor, top_idx: Tensor, gate: Tensor, *, num_experts: int, scaling: float,
                     backend, group=None, shared: Tensor | None = None) -> Tensor:
    """One expert-parallel layer forward of this rank's tokens (see the module
    docstring). Every rank of ``group`` must call it the same number of times."""
    world = dist.get_world_size(group)
    e_local = num_experts // world
    if e_local * world != num_experts:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    dev = x.device

    routing = backend.route_rows(x, top_idx, gate, num_experts)
    q, sf = backend.quantize(x, routing)
    csr = routing.csr.to(torch.int64)
    pcsr = routing.pcsr.to(torch.int64)

    # per destination: counts, padded starts relative to its block, global
    # scales (fp32 bits), block rows
    counts = (csr[1:] - csr[:-1]).view(world, e_local)
    bounds = pcsr[::e_local]  # [world + 1]
    rel = pcsr[:-1].view(world, e_local) - bounds[:-1].unsqueeze(1)
    block = (bounds[1:] - bounds[:-1]).unsqueeze(1)
    ag_bits = routing.act_global.contiguous().view(torch.int32).view(world, e_local).to(torch.int64)
    meta_send = torch.cat([counts, rel, ag_bits, block], dim=1).to(torch.int32).contiguous()
    meta_recv = torch.empty_like(meta_send)
    dist.all_to_all_single(meta_recv, meta_send, group=group)

    sizes = torch.stack([block.squeeze(1), meta_recv[:, -1].to(torch.int64)]).cpu()
    send_rows = sizes[0].tolist()
    recv_rows = sizes[1].tolist()
    total_send, total_recv = sum(send_rows), sum(recv_rows)

    q_recv = _exchange_rows(q[:total_send], total_recv, recv_rows, send_rows, group)
    sf_recv = _exchange_rows(sf[:total_send], total_recv, recv_rows, send_rows, group)

    # received segments: source s, local expert e -> segment s * e_local + e
    base = torch.zeros(world, dtype=torch.int64)
    if world > 1:
        base[1:] = torch.tensor(recv_rows[:-1], dtype=torch.int64).cumsum(0)
    base = base.to(dev)
    seg_counts = meta_recv[:, :e_local].reshape(-1).contiguous()
    seg_starts = torch.cat([(base.unsqueeze(1) + meta_recv[:, e_local:2 * e_local].to(torch.int64)).reshape(-1),
                            torch.tensor([total_recv], dtype=torch.int64, device=dev)]).to(torch.int32)
    seg_global = meta_recv[:, 2 * e_local:3 * e_local].reshape(-1).contiguous().view(torch.float32)
    rows_out = backend.experts(q_recv, sf_recv, seg_counts, seg_starts, seg_global)

    rows_back = _exchange_rows(rows_out, total_send, send_rows, recv_rows, group)
    return backend.combine(rows_back, routing, scaling, shared)


def _exchange_rows(src: Tensor, out_rows: int, out_splits: list[int], in_splits: list[int], group) -> Tensor:
    """all_to_all of whole rows, moved as bytes (any dtype, any backend)."""
    src = src.contiguous()
    width = src.shape[1]
    out = torch.empty(out_rows, width, dtype=src.dtype, device=src.device)
    dist.all_to_all_single(out.view(torch.uint8), src.view(torch.uint8), out_splits, in_splits, group=group)
    return out


class ExpertParallelRoutedExperts(torch.nn.Module):
    """The routed-bank protocol (``routed_forward`` /
    ``routed_forward_with_shared``) over an expert-sharded bank: this rank holds
    ``bank`` = its E/R experts; each forward processes the rank's batch as one
    dispatch chunk and exchanges rows with the other ranks of ``group``."""

    format = "nvfp4"
    backend = "b200_sm100a_tcgen05_nvfp4_expert_parallel"
    ACCEPTS_DISPATCH = False

    def __init__(self, bank: B200NVFP4RoutedExperts, num_experts: int, group=None) -> None:
        super().__init__()
        world = dist.get_world_size(group)
        if bank.num_experts * world != num_experts:
            raise ValueError("the local bank must hold num_experts / world experts")
        self.bank = bank
        self.num_experts = num_experts
        self.group = group
        self._backend = CudaBackend(bank)

    @classmethod
    def from_packed(cls, state: Mapping[str, Tensor], group=None) -> ExpertParallelRoutedExperts:
        """Shard a full packed bank (reference buffer layout) over ``group``."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        e = state["gate_up_q"].shape[0]
        return cls(B200NVFP4RoutedExperts.from_packed(shard_packed_state(state, rank, world)), e, group)

    def prepare(self) -> None:
        self.bank.prepare()

    def routed_forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float, chunk_size: int = 0,
                       dispatch=None) -> Tensor:
        self.bank._check(x, top_idx, gate, scaling, max(chunk_size, x.shape[0], 1))
        return exchange_forward(x, top_idx, gate, num_experts=self.num_experts, scaling=float(scaling),
                                backend=self._backend, group=self.group)

    def routed_forward_with_shared(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float,
                                   chunk_size: int = 0, shared: Tensor, dispatch=None) -> Tensor:
        self.bank._check(x, top_idx, gate, scaling, max(chunk_size, x.shape[0], 1))
        return exchange_forward(x, top_idx, gate, num_experts=self.num_experts, scaling=float(scaling),
                                backend=self._backend, group=self.group, shared=shared)


__all__ = ["CudaBackend", "ExpertParallelRoutedExperts", "exchange_forward", "shard_packed_state"]
