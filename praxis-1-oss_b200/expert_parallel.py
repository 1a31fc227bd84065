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
   compact scale atoms: destination d receives rows [pcsr[d * E/R],
   pcsr[(d + 1) * E/R]) of every source, whole 128-row tiles, so the
   swizzled scale atoms travel as contiguous bytes; the rank's own rows for
   its own experts do not move and are computed while the transfers run.
   ``exchange_forward_peer`` (the default on GPUs) writes the rows with the
   copy engines into the destinations' IPC-mapped buffers
   (``PeerExchange``); ``exchange_forward`` uses NCCL point-to-point
   transfers (and runs over gloo for the CPU tests);
4. on the expert rank, per source: gate/up GEMM + SwiGLU, hidden quantize with
   one global scale per (source, expert) segment (``praxis_b200_expert_forward``
   in hidden-output mode);
5. the FP4 hidden rows, their scale atoms and the segments' hidden maxima
   travel back into the source's own padded layout (F/2 + F/16 bytes a row
   instead of 2 C bytes of bf16: 7x fewer at C = 3072, F = 1536): sources are
   taken in rotating order (step j: compute for rank + j, receive from
   rank - j), so each return transfer overlaps the next source's compute;
6. the source runs the down GEMM + rescale of all its rows against every
   expert's down weights (replicated on every rank: E * C * F / 2 bytes of
   FP4 plus scales) and combines its tokens with the reference's
   four-accumulator order.

Every row meets the same arithmetic as on one GPU, so a rank's output equals
the single-GPU layer on that rank's tokens bit for bit. The exchange step
needs one device-to-host read of the split sizes per forward.

The compute steps go through a backend object (``CudaBackend``: this
library's kernels); the exchange logic is backend-independent so that it can
be exercised with CPU tensors over gloo.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

import torch
import torch.distributed as dist
from torch import Tensor

import ctypes as C

from . import capi, ops
from .bank import B200NVFP4RoutedExperts


def shard_packed_state(state: Mapping[str, Tensor], rank: int, world: int) -> dict[str, Tensor]:
    """The packed buffers of experts [rank * E/world, (rank + 1) * E/world)."""
    e = state["gate_up_q"].shape[0]
    if e % world:
        raise ValueError(f"{e} experts do not shard evenly over {world} ranks")
    lo, hi = rank * e // world, (rank + 1) * e // world
    return {name: value[lo:hi].contiguous() for name, value in state.items()}


class CudaBackend:
    """The compute steps on this library's sm_100a kernels. ``transfer_sms``
    SMs are left out of the expert GEMMs' persistent grids so that the
    transfer kernels of the exchange run beside them. ``down_full``: every
    expert's (down_q, down_sf, down_global), for the down GEMM of the
    source's own rows."""

    def __init__(self, bank: B200NVFP4RoutedExperts, transfer_sms: int = 16, down_full=None) -> None:
        self.bank = bank
        self.down_full = down_full
        self.hidden_features = bank.hidden_features
        props = torch.cuda.get_device_properties(bank.gate_up_q.device)
        self.sm_limit = max(2, props.multi_processor_count - transfer_sms) if transfer_sms > 0 else 0

    def route_rows(self, x: Tensor, top_idx: Tensor, gate: Tensor, num_experts: int):
        return ops.dispatch(top_idx, gate, num_experts, ops.row_amax(x), full=False)

    def quantize(self, x: Tensor, routing) -> tuple[Tensor, Tensor]:
        return ops.quantize_gather(x, routing, routing.act_global)

    def _part(self, t: Tensor, first: int, last: int) -> Tensor:
        """Experts [first, last) of a per-expert buffer (flat when replicated)."""
        return t[first:last] if t.dim() > 1 else t.view(self.bank.num_experts, -1)[first:last].reshape(-1)

    def hidden(self, q: Tensor, sf: Tensor, counts: Tensor, starts: Tensor, act_global: Tensor, first: int,
               last: int, out=None) -> tuple[Tensor, Tensor, Tensor]:
        """Segments of local experts [first, last) (segment v: expert first +
        v % (last - first)) -> FP4 hidden rows, their scales and the
        segments' hidden maxima (written into ``out`` when given)."""
        kw = self.bank.kernel_weights()
        b = self.bank
        return ops.expert_hidden(q, sf, counts, starts, act_global, self._part(kw.gate_up_q, first, last),
                                 self._part(kw.gate_up_sf, first, last), b.gate_up_global[first:last],
                                 hidden=b.hidden_features, gate_up_sf_layout=kw.gate_up_sf_layout,
                                 sm_limit=self.sm_limit, out=out)

    def down(self, hq: Tensor, hsf: Tensor, hamax: Tensor, routing) -> Tensor:
        """Down GEMM + rescale of the source's padded rows (all experts)."""
        dq, dsf, dg = self.down_full
        return ops.grouped_gemm(hq, hsf, dq, dsf, routing, epilogue=capi.EPI_RESCALE, act_amax=hamax, w_global=dg)

    def experts(self, q: Tensor, sf: Tensor, counts: Tensor, starts: Tensor, act_global: Tensor,
                first: int, last: int, out_ptr: int | None = None) -> Tensor | None:
        """Both GEMMs of segments of local experts [first, last) on this rank
        (one launch sequence; the compute of a rank's share of the layer, for
        timing); with ``out_ptr`` the rows are written to that address."""
        kw = self.bank.kernel_weights()
        b = self.bank
        return ops.expert_forward(q, sf, counts, starts, act_global, self._part(kw.gate_up_q, first, last),
                                  self._part(kw.gate_up_sf, first, last), b.gate_up_global[first:last],
                                  self._part(b.down_q, first, last), self._part(kw.down_sf, first, last),
                                  b.down_global[first:last], gate_up_sf_layout=kw.gate_up_sf_layout,
                                  down_sf_layout=kw.down_sf_layout, sm_limit=self.sm_limit, out_ptr=out_ptr)

    def combine(self, rows: Tensor, routing, scaling: float, shared: Tensor | None) -> Tensor:
        return ops.combine(rows, routing, scaling, rows_rescaled=True, shared=shared)


def exchange_forward(x: Tensor, top_idx: Tensor, gate: Tensor, *, num_experts: int, scaling: float,
                     backend, group=None, shared: Tensor | None = None, chunks: int | None = None) -> Tensor:
    """One expert-parallel layer forward of this rank's tokens (see the module
    docstring). Every rank of ``group`` must call it the same number of times
    with the same ``chunks`` (expert groups per source for the return
    pipeline; default 1: on 2 GPUs the split launches cost more than the
    overlap wins)."""
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
    rank = dist.get_rank(group)
    peer = [dist.get_global_rank(group, i) if group is not None else i for i in range(world)]
    lo = [int(v) for v in bounds.cpu().tolist()]

    # outbound rows and scale atoms of every other rank, as one batch
    recv_q: list[Tensor | None] = [None] * world
    recv_sf: list[Tensor | None] = [None] * world
    p2p = []
    for s in range(world):
        if s == rank or recv_rows[s] == 0:
            continue
        recv_q[s] = torch.empty(recv_rows[s], q.shape[1], dtype=q.dtype, device=dev)
        recv_sf[s] = torch.empty(recv_rows[s], sf.shape[1], dtype=sf.dtype, device=dev)
        p2p += [dist.P2POp(dist.irecv, recv_q[s].view(torch.uint8), peer[s], group),
                dist.P2POp(dist.irecv, recv_sf[s].view(torch.uint8), peer[s], group)]
    for d in range(world):
        if d == rank or send_rows[d] == 0:
            continue
        p2p += [dist.P2POp(dist.isend, q[lo[d]:lo[d + 1]].contiguous().view(torch.uint8), peer[d], group),
                dist.P2POp(dist.isend, sf[lo[d]:lo[d + 1]].contiguous().view(torch.uint8), peer[d], group)]
    outbound = dist.batch_isend_irecv(p2p) if p2p else []

    # the source's return buffers: FP4 hidden rows, their scale atoms (tile
    # rows of F/16 bytes) and the hidden maxima of every expert's segment
    f = backend.hidden_features
    hq_back = torch.empty(lo[world], f // 2, dtype=torch.uint8, device=dev)
    hsf_back = torch.empty(lo[world], f // 16, dtype=torch.uint8, device=dev)
    hamax = torch.zeros(num_experts, dtype=torch.int32, device=dev)
    chunks = max(1, min(e_local, chunks or 1))
    # every source's segments in one go: counts, starts (relative to its
    # block, then the block end) and global scales, one row per source
    seg_counts = meta_recv[:, :e_local].contiguous()
    seg_starts = torch.cat([meta_recv[:, e_local:2 * e_local], meta_recv[:, -1:]], dim=1).contiguous()
    seg_global = meta_recv[:, 2 * e_local:3 * e_local].contiguous().view(torch.float32)
    if chunks > 1:
        rel_host = meta_recv[:, e_local:2 * e_local].cpu().tolist()
        first = (torch.arange(num_experts + 1, device=dev) // e_local).clamp_max(world - 1) * e_local
        mine = (pcsr - pcsr[first]).cpu()

    def segments(s: int, a: int, b: int):
        """Received segments of source s for local experts [a, b), rows
        relative to the first one, and that row range in the source block."""
        if chunks == 1:
            return (seg_counts[s], seg_starts[s], seg_global[s]), 0, recv_rows[s]
        r0 = int(rel_host[s][a])
        r1 = int(rel_host[s][b]) if b < e_local else recv_rows[s]
        starts_s = torch.tensor([int(v) - r0 for v in rel_host[s][a:b]] + [r1 - r0], dtype=torch.int32, device=dev)
        return (seg_counts[s, a:b].contiguous(), starts_s, seg_global[s, a:b].contiguous()), r0, r1

    # this rank's own rows for its own experts: computed while the exchange runs
    if send_rows[rank]:
        seg, _, _ = segments(rank, 0, e_local)
        backend.hidden(q[lo[rank]:lo[rank + 1]], sf[lo[rank]:lo[rank + 1]], *seg, 0, e_local,
                       out=(hq_back[lo[rank]:lo[rank + 1]], hsf_back[lo[rank]:lo[rank + 1]],
                            hamax[rank * e_local:(rank + 1) * e_local]))
    for w in outbound:
        w.wait()

    # the other sources in rotating order: at step j this rank computes the
    # hidden rows of source (rank + j) and returns them while it receives its
    # own from rank (rank - j), which computes them at the same step; each
    # source's experts go in `chunks` groups so the return transfers pipeline
    groups = [(c * e_local // chunks, (c + 1) * e_local // chunks) for c in range(chunks)]
    keep = []
    returns = []
    for j in range(1, world):
        s, d = (rank + j) % world, (rank - j) % world
        for a, b in groups:
            p2p = []
            if recv_rows[s]:
                seg, r0, r1 = segments(s, a, b)
                if r1 > r0:
                    res = backend.hidden(recv_q[s][r0:r1], recv_sf[s][r0:r1], *seg, a, b)
                    keep.append(res)
                    p2p += [dist.P2POp(dist.isend, t_.contiguous().view(torch.uint8), peer[s], group) for t_ in res]
            if send_rows[d]:
                g0 = 0 if chunks == 1 else int(mine[d * e_local + a])
                g1 = send_rows[d] if chunks == 1 or b == e_local else int(mine[d * e_local + b])
                if g1 > g0:
                    p2p += [dist.P2POp(dist.irecv, dst.view(torch.uint8), peer[d], group) for dst in (
                        hq_back[lo[d] + g0:lo[d] + g1], hsf_back[lo[d] + g0:lo[d] + g1],
                        hamax[d * e_local + a:d * e_local + b])]
            if p2p:
                returns += dist.batch_isend_irecv(p2p)
    for w in returns:
        w.wait()
    rows = backend.down(hq_back, hsf_back, hamax, routing)
    return backend.combine(rows, routing, scaling, shared)


def _padded(rows: int) -> int:
    return (rows + 127) // 128 * 128


class _DeviceBytes:
    """A raw device allocation seen by torch as a uint8 tensor (no copy)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


class PeerExchange:
    """Buffers of this rank that every other rank of ``group`` writes into
    directly (CUDA IPC mappings), and the copy streams that move rows between
    ranks on the GPUs' copy engines, so the expert GEMMs keep every SM.

    * ``recv``: one slot per source rank for the FP4 rows and compact scale
      atoms that source sends to this rank's experts;
    * ``back``: this rank's padded routed rows as FP4 hidden rows and their
      scale atoms, plus every expert's hidden maximum, written by the expert
      ranks with their results.

    Buffers grow (collectively: every rank derives the same capacity from the
    exchanged token counts) and are never shrunk. Ordering between ranks uses
    two one-element all-reduces per forward: after them every rank's copies
    into this rank's buffers have landed, and every reader of the previous
    forward's data is done.
    """

    def __init__(self, group, device: torch.device, copy_streams: int = 4, sm_copy_fraction: float = 0.0,
                 copy_ctas: int = 16) -> None:
        """``sm_copy_fraction`` of every transfer's bytes go through a copy
        kernel on ``copy_ctas`` CTAs (SM-driven NVLink writes) beside the copy
        engines, which move the rest."""
        if not 0.0 <= sm_copy_fraction <= 1.0:
            raise ValueError("sm_copy_fraction must be in [0, 1]")
        self.group = group
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slot_rows = 0
        self.back_rows = 0
        self.q_cols = self.sf_cols = self.hq_cols = self.hsf_cols = self.experts = 0
        self._local: dict[str, tuple[int, int]] = {}  # name -> (pointer, bytes)
        self._peer: dict[str, list[int]] = {}  # name -> pointer per rank (own rank: local)
        self.streams = [torch.cuda.Stream(self.device) for _ in range(copy_streams)]
        self.sm_copy_fraction = float(sm_copy_fraction)
        self.copy_ctas = int(copy_ctas)
        self.sm_stream = torch.cuda.Stream(self.device) if sm_copy_fraction > 0 else None
        self.flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ready: torch.cuda.Event | None = None  # the previous forward's last barrier
        # per-source arrival flags: a source's copy stream writes the
        # forward's epoch into the destination's flag after the rows
        self.epoch = 0
        self.epoch_buf = torch.zeros(1, dtype=torch.int32, device=self.device)
        # this rank's results for the other sources before they travel back:
        # one region per source (like the receive slots), kept across
        # forwards so the return copies need no per-call allocation or
        # stream bookkeeping (each forward ends with the compute stream
        # waiting for every copy stream)
        self.res_hq = self.res_hsf = self.res_amax = None

    # -- buffers ------------------------------------------------------------
    def _release(self) -> None:
        lib = capi.load()
        dev = self.device.index
        if self._local:
            # this rank's copies into the peers' buffers are done before the
            # mappings go away
            torch.cuda.synchronize(self.device)
        for name, ptrs in self._peer.items():
            for r, ptr in enumerate(ptrs):
                if r != self.rank and ptr:
                    capi.check(lib.praxis_b200_ipc_close(C.c_void_p(ptr), dev))
        self._peer = {}
        if self._local:
            dist.barrier(group=self.group)  # every peer has closed its mappings
            for ptr, _ in self._local.values():
                capi.check(lib.praxis_b200_ipc_free(C.c_void_p(ptr), dev))
        self._local = {}

    def ensure(self, slot_rows: int, back_rows: int, q_cols: int, sf_cols: int, hq_cols: int, hsf_cols: int,
               experts: int) -> None:
        """Collective when the buffers grow: every rank must call it with the
        same arguments."""
        shape = (q_cols, sf_cols, hq_cols, hsf_cols, experts)
        if (slot_rows <= self.slot_rows and back_rows <= self.back_rows and shape ==
                (self.q_cols, self.sf_cols, self.hq_cols, self.hsf_cols, self.experts)):
            return
        self._release()
        lib = capi.load()
        dev = self.device.index
        sizes = {"recv": self.world * slot_rows * (q_cols + sf_cols),
                 "back": back_rows * (hq_cols + hsf_cols) + experts * 4, "flags": self.world * 4}
        handles = {}
        for name, nbytes in sizes.items():
            ptr = C.c_void_p()
            capi.check(lib.praxis_b200_ipc_alloc(nbytes, dev, C.byref(ptr)))
            self._local[name] = (int(ptr.value), nbytes)
            if name == "flags":  # no epoch yet
                torch.as_tensor(_DeviceBytes(int(ptr.value), nbytes), device=self.device).zero_()
                torch.cuda.synchronize(self.device)
            h = (C.c_ubyte * capi.IPC_HANDLE_BYTES)()
            capi.check(lib.praxis_b200_ipc_handle(ptr, dev, h))
            handles[name] = bytes(h)
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, handles, group=self.group)
        for name in sizes:
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._local[name][0])
                    continue
                h = (C.c_ubyte * capi.IPC_HANDLE_BYTES).from_buffer_copy(gathered[r][name])
                ptr = C.c_void_p()
                capi.check(lib.praxis_b200_ipc_open(h, dev, C.byref(ptr)))
                ptrs.append(int(ptr.value))
            self._peer[name] = ptrs
        self.slot_rows, self.back_rows = slot_rows, back_rows
        self.q_cols, self.sf_cols, self.hq_cols, self.hsf_cols, self.experts = shape
        u8 = dict(dtype=torch.uint8, device=self.device)
        self.res_hq = torch.empty(self.world, slot_rows, hq_cols, **u8)
        self.res_hsf = torch.empty(self.world, slot_rows, hsf_cols, **u8)
        self.res_amax = torch.empty(self.world, experts, dtype=torch.int32, device=self.device)
        self.ready = None

    def recv_views(self, s: int, rows: int) -> tuple[Tensor, Tensor]:
        """The FP4 rows and scale atoms source ``s`` wrote into this rank's slot."""
        ptr, _ = self._local["recv"]
        base = ptr + s * self.slot_rows * (self.q_cols + self.sf_cols)
        q = torch.as_tensor(_DeviceBytes(base, rows * self.q_cols), device=self.device)
        sf = torch.as_tensor(_DeviceBytes(base + self.slot_rows * self.q_cols, rows * self.sf_cols),
                             device=self.device)
        return q.view(rows, self.q_cols), sf.view(rows, self.sf_cols)

    def back_views(self, rows: int) -> tuple[Tensor, Tensor, Tensor]:
        """This rank's returned FP4 hidden rows, their scale atoms and the
        experts' hidden maxima (int32 bits)."""
        ptr, _ = self._local["back"]
        hq = torch.as_tensor(_DeviceBytes(ptr, rows * self.hq_cols), device=self.device)
        hsf = torch.as_tensor(_DeviceBytes(ptr + self.back_rows * self.hq_cols, rows * self.hsf_cols),
                              device=self.device)
        amax = torch.as_tensor(_DeviceBytes(ptr + self.back_rows * (self.hq_cols + self.hsf_cols), self.experts * 4),
                               device=self.device)
        return hq.view(rows, self.hq_cols), hsf.view(rows, self.hsf_cols), amax.view(torch.int32)

    def result_views(self, s: int, r0: int, r1: int, a: int, b: int) -> tuple[Tensor, Tensor, Tensor]:
        """Where this rank computes source s's hidden rows [r0, r1) and the
        maxima of its segments [a, b) before they travel back."""
        return self.res_hq[s, r0:r1], self.res_hsf[s, r0:r1], self.res_amax[s, a:b]

    def recv_slot(self, d: int, s: int) -> tuple[int, int]:
        """Device addresses (on this rank) of rank d's slot for source s: rows, scales."""
        base = self._peer["recv"][d] + s * self.slot_rows * (self.q_cols + self.sf_cols)
        return base, base + self.slot_rows * self.q_cols

    def back_ptrs(self, d: int, row: int, expert: int) -> tuple[int, int, int]:
        """Device addresses (on this rank) of rank d's returned hidden row
        ``row``, its scales, and its maximum of expert ``expert``."""
        base = self._peer["back"][d]
        return (base + row * self.hq_cols, base + self.back_rows * self.hq_cols + row * self.hsf_cols,
                base + self.back_rows * (self.hq_cols + self.hsf_cols) + expert * 4)

    def signal(self, d: int, stream: torch.cuda.Stream) -> None:
        """After everything queued for rank d on ``stream`` (and on the SM copy
        stream): write this forward's epoch into d's flag for this source."""
        lib = capi.load()
        if self.sm_stream is not None:
            ev = torch.cuda.Event()
            ev.record(self.sm_stream)
            stream.wait_event(ev)
        dst = self._peer["flags"][d] + 4 * self.rank
        capi.check(lib.praxis_b200_copy_async(C.c_void_p(dst), C.c_void_p(self.epoch_buf.data_ptr()), 4,
                                               self.device.index, C.c_void_p(stream.cuda_stream)))

    def wait_source(self, s: int, stream: torch.cuda.Stream, timeout_s: float = 10.0) -> None:
        """``stream`` waits (bounded, on the GPU) until source s's rows of this
        forward have landed in this rank's slot."""
        flag = self._local["flags"][0] + 4 * s
        capi.check(capi.load().praxis_b200_wait_value(C.c_void_p(flag), self.epoch, int(timeout_s * 1e9),
                                                       self.device.index, C.c_void_p(stream.cuda_stream)))

    def copy(self, dst: int, src: int, nbytes: int, stream: torch.cuda.Stream,
             after: Sequence[torch.cuda.Event] = ()) -> None:
        """``nbytes`` from ``src`` to ``dst`` once the ``after`` events have
        completed: the copy engines on ``stream``, and the ``sm_copy_fraction``
        head of it by the copy kernel on the SM copy stream."""
        lib = capi.load()
        dev = self.device.index
        for ev in after:
            stream.wait_event(ev)
        head = 0
        if self.sm_stream is not None:
            head = int(nbytes * self.sm_copy_fraction) // 16 * 16
            if head:
                for ev in after:
                    self.sm_stream.wait_event(ev)
                capi.check(lib.praxis_b200_sm_copy(C.c_void_p(dst), C.c_void_p(src), head, self.copy_ctas, dev,
                                                   C.c_void_p(self.sm_stream.cuda_stream)))
        capi.check(lib.praxis_b200_copy_async(C.c_void_p(dst + head), C.c_void_p(src + head), nbytes - head, dev,
                                               C.c_void_p(stream.cuda_stream)))

    def copy_many(self, items: Sequence[tuple[int, int, int]], stream: torch.cuda.Stream,
                  after: Sequence[torch.cuda.Event] = ()) -> None:
        """``copy`` of several (dst, src, nbytes) on one stream behind the
        same events (each waited for once)."""
        for ev in after:
            stream.wait_event(ev)
        for dst, src, nbytes in items:
            self.copy(dst, src, nbytes, stream, () if self.sm_stream is None else after)

    def copy_streams(self) -> list[torch.cuda.Stream]:
        """Every stream the copies run on."""
        return self.streams + ([self.sm_stream] if self.sm_stream is not None else [])

    def barrier(self, stream: torch.cuda.Stream) -> None:
        """All ranks' work enqueued before this point (on ``stream``) is done
        when ``stream`` continues."""
        with torch.cuda.stream(stream):
            dist.all_reduce(self.flag, group=self.group)

    def close(self) -> None:
        self._release()
        self.slot_rows = self.back_rows = 0


def exchange_forward_peer(x: Tensor, top_idx: Tensor, gate: Tensor, *, num_experts: int, scaling: float,
                          backend, peers: PeerExchange, shared: Tensor | None = None, chunks: int = 2) -> Tensor:
    """``exchange_forward`` with the rows moved by copy engines into the
    peers' mapped buffers (``PeerExchange``) instead of NCCL point-to-point
    transfers: the same routing, segments, arithmetic and results. Collective
    over ``peers.group``; ``chunks`` expert groups per source (same on every
    rank)."""
    world, rank = peers.world, peers.rank
    e_local = num_experts // world
    if e_local * world != num_experts:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    dev = x.device
    compute = torch.cuda.current_stream(dev)
    top_k = top_idx.shape[1]
    chunks = max(1, min(e_local, chunks))

    routing = backend.route_rows(x, top_idx, gate, num_experts)
    csr = routing.csr.to(torch.int64)
    pcsr = routing.pcsr.to(torch.int64)
    counts = (csr[1:] - csr[:-1]).view(world, e_local)
    bounds = pcsr[::e_local]  # [world + 1]
    rel = pcsr[:-1].view(world, e_local) - bounds[:-1].unsqueeze(1)
    block = (bounds[1:] - bounds[:-1]).unsqueeze(1)
    ag_bits = routing.act_global.contiguous().view(torch.int32).view(world, e_local).to(torch.int64)
    # per destination: counts, padded starts in the block, global scales,
    # block rows, the block's first row here (where the results go back) and
    # this rank's token count (buffer capacity)
    tok = torch.full((world, 1), x.shape[0], dtype=torch.int64, device=dev)
    meta_send = torch.cat([counts, rel, ag_bits, block, bounds[:-1].unsqueeze(1), tok], dim=1)
    meta_send = meta_send.to(torch.int32).contiguous()
    meta_recv = torch.empty_like(meta_send)
    dist.all_to_all_single(meta_recv, meta_send, group=peers.group)
    # one device-to-host read: block rows to each destination, rows from each
    # source, where they go back in the source, token counts, block bounds,
    # and each source's per-expert row starts inside its block
    host = torch.cat([block.squeeze(1), meta_recv[:, 3 * e_local:].t().reshape(-1).to(torch.int64), bounds,
                      meta_recv[:, e_local:2 * e_local].reshape(-1).to(torch.int64)]).cpu().tolist()
    send_rows, recv_rows = host[:world], host[world:2 * world]
    src_row0, tokens_all = host[2 * world:3 * world], host[3 * world:4 * world]
    lo = host[4 * world:5 * world + 1]
    rel_host = [host[5 * world + 1 + i * e_local:5 * world + 1 + (i + 1) * e_local] for i in range(world)]
    max_tokens = max(tokens_all)
    f = backend.hidden_features
    # the quantize is queued after the host read, so the GPU runs it while
    # the host queues the transfers and the expert groups below
    q, sf = backend.quantize(x, routing)
    peers.ensure(_padded(max_tokens * top_k + 127 * e_local), _padded(max_tokens * top_k + 127 * num_experts),
                 q.shape[1], sf.shape[1], f // 2, f // 16, num_experts)

    # outbound rows, on the copy engines, into every destination's slot for
    # this rank, each destination's rows followed by this forward's epoch in
    # its flag for this rank (destinations in rotating order, so each expert
    # rank's sources land spread out in time)
    peers.epoch = (peers.epoch + 1) & 0x7FFFFFFF
    peers.epoch_buf.fill_(peers.epoch)
    quantized = torch.cuda.Event()
    quantized.record(compute)
    streams = peers.streams
    after = [quantized] + ([peers.ready] if peers.ready is not None else [])
    for k, d in enumerate((rank + j) % world for j in range(1, world)):
        st = streams[k % len(streams)]
        if send_rows[d]:
            dq, dsf = peers.recv_slot(d, rank)
            peers.copy(dq, q.data_ptr() + lo[d] * q.shape[1], send_rows[d] * q.shape[1], st, after)
            peers.copy(dsf, sf.data_ptr() + lo[d] * sf.shape[1], send_rows[d] * sf.shape[1], st, after)
        else:
            for ev in after:
                st.wait_event(ev)
        peers.signal(d, st)
    for st in peers.copy_streams():
        q.record_stream(st)
        sf.record_stream(st)

    # per source and expert group: segment counts, segment starts relative
    # to the group's first row, and global scales, as contiguous rows (a few
    # batched ops here instead of three small copies per source and group)
    seg_counts = meta_recv[:, :e_local].contiguous()
    seg_starts = torch.cat([meta_recv[:, e_local:2 * e_local], meta_recv[:, 3 * e_local:3 * e_local + 1]], dim=1)
    seg_global = meta_recv[:, 2 * e_local:3 * e_local].contiguous().view(torch.float32)
    groups = [(c * e_local // chunks, (c + 1) * e_local // chunks) for c in range(chunks)]
    # this rank's own rows: most of them while its rows travel out (half on
    # 2 ranks, three quarters on more, where more rows leave), the rest last
    half = e_local - e_local // (2 if world <= 2 else 4)
    group_starts = {(a, b): (seg_starts[:, a:b + 1] - seg_starts[:, a:a + 1]).to(torch.int32).contiguous()
                    for a, b in set(groups + [(0, half), (half, e_local)]) if a < b}
    hq_back, hsf_back, hamax = peers.back_views(lo[world])
    returned = [0]

    def run(src: int, a: int, b: int) -> None:
        """Local experts [a, b) on the rows of source ``src``: the FP4 hidden
        rows, their scales and the segments' maxima go to the source's
        return buffers."""
        if a >= b:
            return
        r0 = rel_host[src][a]
        r1 = rel_host[src][b] if b < e_local else recv_rows[src]
        if r1 <= r0:
            return
        if src == rank:
            sq, ssf = q[lo[rank] + r0:lo[rank] + r1], sf[lo[rank] + r0:lo[rank] + r1]
        else:
            rq, rsf = peers.recv_views(src, recv_rows[src])
            sq, ssf = rq[r0:r1], rsf[r0:r1]
        counts, starts, ag = seg_counts[src, a:b], group_starts[(a, b)][src], seg_global[src, a:b]
        if src == rank:  # own rows: straight into this rank's return buffers
            row = lo[rank] + r0
            backend.hidden(sq, ssf, counts, starts, ag, a, b,
                           out=(hq_back[row:row + r1 - r0], hsf_back[row:row + r1 - r0],
                                hamax[rank * e_local + a:rank * e_local + b]))
            return
        # other sources: the result in this rank's region for the source,
        # then a copy engine writes it into the source's mapped buffers while
        # the next group computes
        hq, hsf, amax = peers.result_views(src, r0, r1, a, b)
        backend.hidden(sq, ssf, counts, starts, ag, a, b, out=(hq, hsf, amax))
        done = torch.cuda.Event()
        done.record(compute)
        st = streams[returned[0] % len(streams)]
        returned[0] += 1
        d_hq, d_hsf, d_amax = peers.back_ptrs(src, src_row0[src] + r0, rank * e_local + a)
        peers.copy_many([(d_hq, hq.data_ptr(), hq.numel()), (d_hsf, hsf.data_ptr(), hsf.numel()),
                         (d_amax, amax.data_ptr(), amax.numel() * 4)], st, [done])

    # the own rows' first part; the other sources in rotating order, in
    # `chunks` expert groups so each result travels back while the next
    # group computes; the rest of the own rows last, while the final results
    # travel; then the down GEMM of all this rank's rows and the combine
    run(rank, 0, half)
    for j in range(1, world):
        src = (rank - j) % world  # the source whose rows were sent to this rank j-th
        if recv_rows[src]:
            peers.wait_source(src, compute)
        for a, b in groups:
            run(src, a, b)
    run(rank, half, e_local)
    for st in peers.copy_streams():
        compute.wait_stream(st)
    peers.barrier(compute)  # every result for this rank's rows has landed
    rows = backend.down(hq_back, hsf_back, hamax, routing)
    peers.ready = torch.cuda.Event()
    peers.ready.record(compute)
    return backend.combine(rows, routing, scaling, shared)


def chunked_forward(one_chunk, x: Tensor, top_idx: Tensor, gate: Tensor, shared: Tensor | None, chunk_size: int,
                    group=None) -> Tensor:
    """The dispatch-chunk loop of ``NVFP4RoutedExperts._routed_forward``
    (praxis/quantization/nvfp4.py:683-747) over an expert-parallel exchange:
    each rank splits its own tokens into chunks of ``chunk_size`` and every
    chunk is one exchange, so activation and hidden global scales are taken
    per (chunk, expert) as on one GPU. Ranks may hold different token counts;
    they agree on the largest chunk count (one all-reduce) and a rank with
    fewer chunks joins the remaining exchanges with an empty chunk, so every
    rank runs the same collectives in the same order. ``chunk_size <= 0``
    takes each rank's whole batch as one chunk (no agreement needed)."""
    t = x.shape[0]
    if chunk_size <= 0:
        return one_chunk(x, top_idx, gate, shared)
    mine = -(-t // chunk_size)
    count = torch.tensor([mine], dtype=torch.int64, device=x.device)
    dist.all_reduce(count, op=dist.ReduceOp.MAX, group=group)
    n = int(count.item())
    if n <= 1:
        return one_chunk(x, top_idx, gate, shared)
    out = torch.empty_like(x)
    for i in range(n):
        a, b = min(i * chunk_size, t), min((i + 1) * chunk_size, t)
        res = one_chunk(x[a:b], top_idx[a:b], gate[a:b], None if shared is None else shared[a:b])
        if b > a:
            out[a:b] = res
    return out


class ExpertParallelRoutedExperts(torch.nn.Module):
    """The routed-bank protocol (``routed_forward`` /
    ``routed_forward_with_shared``) over an expert-sharded bank: this rank holds
    ``bank`` = its E/R experts; each forward processes the rank's batch as one
    dispatch chunk and exchanges rows with the other ranks of ``group``."""

    format = "nvfp4"
    backend = "b200_sm100a_tcgen05_nvfp4_expert_parallel"
    ACCEPTS_DISPATCH = False

    def __init__(self, bank: B200NVFP4RoutedExperts, num_experts: int, group=None, *,
                 down_full: tuple[Tensor, Tensor, Tensor], transport: str = "peer", transfer_sms: int = 16,
                 chunks: int | None = None, copy_streams: int = 4, sm_copy_fraction: float = 0.0) -> None:
        """``transport="peer"``: rows move on the copy engines into the peers'
        mapped buffers (``exchange_forward_peer``); ``"nccl"``: NCCL
        point-to-point transfers (``exchange_forward``), with ``transfer_sms``
        SMs kept free of the expert GEMMs for NCCL's kernels. With the peer
        transport, ``sm_copy_fraction`` > 0 moves that share of the bytes with
        a copy kernel on ``transfer_sms`` CTAs beside the copy engines (and
        keeps those SMs free of the GEMMs). ``down_full``: every expert's
        (down_q, down_sf, down_global) in the reference's layout (the down
        GEMM of this rank's rows runs here)."""
        super().__init__()
        world = dist.get_world_size(group)
        if bank.num_experts * world != num_experts:
            raise ValueError("the local bank must hold num_experts / world experts")
        dq, dsf, dg = down_full
        if (dq.shape[0] != num_experts or dsf.shape[0] != num_experts or dg.numel() != num_experts
                or dq.shape[1:] != bank.down_q.shape[1:] or dsf.shape[1:] != bank.down_sf.shape[1:]):
            raise ValueError("down_full must hold the down weights of every expert")
        self.register_buffer("down_q_full", dq.detach().contiguous())
        self.register_buffer("down_sf_full", dsf.detach().contiguous())
        self.register_buffer("down_global_full", dg.detach().contiguous())
        if transport not in ("peer", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.bank = bank
        self.num_experts = num_experts
        self.group = group
        self.chunks = chunks
        self.transport = transport if world > 1 else "nccl"
        reserve = self.transport == "nccl" or sm_copy_fraction > 0
        self._backend = CudaBackend(bank, transfer_sms if world > 1 and reserve else 0,
                                    (self.down_q_full, self.down_sf_full, self.down_global_full))
        self._peers = (PeerExchange(group, bank.gate_up_q.device, copy_streams, sm_copy_fraction, transfer_sms)
                       if self.transport == "peer" else None)

    @classmethod
    def from_packed(cls, state: Mapping[str, Tensor], group=None, **kwargs) -> ExpertParallelRoutedExperts:
        """Shard a full packed bank (reference buffer layout) over ``group``."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        e = state["gate_up_q"].shape[0]
        shard = shard_packed_state(state, rank, world)
        on_host = all(v.device.type == "cpu" for v in shard.values())
        bank = (B200NVFP4RoutedExperts.from_packed(shard) if on_host
                else B200NVFP4RoutedExperts.from_device_state(shard))
        down_full = tuple(state[n].to(bank.down_q.device) for n in ("down_q", "down_sf", "down_global"))
        return cls(bank, e, group, down_full=down_full, **kwargs)

    def prepare(self) -> None:
        self.bank.prepare()

    def _forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, scaling: float, shared: Tensor | None) -> Tensor:
        self._backend.down_full = (self.down_q_full, self.down_sf_full, self.down_global_full)  # after moves
        if self._peers is not None:
            return exchange_forward_peer(x, top_idx, gate, num_experts=self.num_experts, scaling=scaling,
                                         backend=self._backend, peers=self._peers, shared=shared,
                                         chunks=self.chunks or 2)
        return exchange_forward(x, top_idx, gate, num_experts=self.num_experts, scaling=scaling,
                                backend=self._backend, group=self.group, shared=shared, chunks=self.chunks)

    def routed_forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float, chunk_size: int = 0,
                       dispatch=None) -> Tensor:
        """The bank protocol's ``routed_forward``; ``chunk_size`` splits this
        rank's tokens into dispatch chunks as the reference does (see
        ``chunked_forward``; 0 = the whole batch is one chunk)."""
        return self._chunked(x, top_idx, gate, scaling, chunk_size, None)

    def routed_forward_with_shared(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float,
                                   chunk_size: int = 0, shared: Tensor, dispatch=None) -> Tensor:
        return self._chunked(x, top_idx, gate, scaling, chunk_size, shared)

    def _chunked(self, x, top_idx, gate, scaling, chunk_size, shared) -> Tensor:
        if type(chunk_size) is not int or chunk_size < 0:
            raise ValueError("chunk_size must be a non-negative int (0: one chunk per rank)")
        self.bank._check(x, top_idx, gate, scaling, chunk_size if chunk_size > 0 else max(x.shape[0], 1))
        scaling = float(scaling)
        return chunked_forward(lambda xc, tc, gc, sc: self._forward(xc, tc, gc, scaling, sc), x, top_idx, gate,
                               shared, chunk_size, self.group)

    def close(self) -> None:
        """Unmap and free the peer buffers (collective over ``group``)."""
        if self._peers is not None:
            self._peers.close()


__all__ = ["CudaBackend", "ExpertParallelRoutedExperts", "PeerExchange", "chunked_forward", "exchange_forward",
           "exchange_forward_peer", "shard_packed_state"]
