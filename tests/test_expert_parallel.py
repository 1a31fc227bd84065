"""Expert-parallel exchange logic on CPU ranks (gloo, world size 2 and 4).

The product's exchange (``praxis_b200.expert_parallel.exchange_forward``:
metadata all-to-all, row/scale all-to-all, segment bookkeeping, return
all-to-all, combine) runs with the oracle's CPU restatement as the compute
backend. Each rank's output must equal the single-rank oracle layer on that
rank's tokens, bit for bit: expert parallelism changes where rows are
computed, not how. A rank that fails before the exchange must make the other
ranks' collectives end with an error (short process-group timeout), not hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from conftest import pkg

from oracle import nvfp4_moe_oracle as O

BF16 = torch.bfloat16


class OracleBackend:
    """The compute steps of ``CudaBackend`` restated on the CPU."""

    def __init__(self, local_bank: dict, top_k: int, full_bank: dict):
        self.bank = local_bank
        self.full = full_bank
        self.top_k = top_k
        self.hidden_features = local_bank["down_q"].shape[2] * 2

    def route_rows(self, x, top_idx, gate, num_experts):
        order, inverse, tokens, _sg, offsets, csr = O.dispatch(top_idx, gate, num_experts)
        pcsr = O.pad_csr(csr)
        ag = O.segment_global_scales(O.row_amax(x), csr, tokens)
        return SimpleNamespace(csr=csr.to(torch.int32), pcsr=pcsr.to(torch.int32), act_global=ag.to(torch.float32),
                               inverse=inverse, top_idx=top_idx, gate=gate, tokens=tokens, experts=num_experts)

    def quantize(self, x, r):
        rows = O.padded_rows(r.tokens.numel(), r.experts)
        return O.quantize_activations(x, r.csr.long(), r.pcsr.long(), rows, r.act_global, row_indices=r.tokens)

    def experts(self, q, sf, counts, starts, ag, first, last):
        b = {name: v[first:last] for name, v in self.bank.items()}
        e_local = last - first
        f = b["down_q"].shape[2] * 2
        c = q.shape[1] * 2
        rows = q.shape[0]
        seg = torch.arange(counts.numel()) % e_local
        vb = {k: b[k][seg] for k in ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf",
                                     "down_global")}
        pc = starts.long()
        gu = O.grouped_gemm(q, sf, vb["gate_up_q"], vb["gate_up_sf"], pc, c, 2 * f)
        hidden, rowmax = O.rescale_swiglu_maximum(gu, pc, ag, vb["gate_up_global"])
        hg = O.segment_global_scales(rowmax, pc)
        hq, hsf = O.quantize_activations(hidden, pc, pc, rows, hg)
        raw = O.grouped_gemm(hq, hsf, vb["down_q"], vb["down_sf"], pc, f, c)
        ex = O.expert_of_rows(pc, torch.arange(rows))
        mult = O.bf16_round(hg[ex] * vb["down_global"][ex]).unsqueeze(1)
        return (raw.to(torch.float32) * mult).to(BF16)

    def hidden(self, q, sf, counts, starts, ag, first, last, out=None):
        b = {name: v[first:last] for name, v in self.bank.items()}
        e_local = last - first
        f = self.hidden_features
        c = q.shape[1] * 2
        rows = q.shape[0]
        seg = torch.arange(counts.numel()) % e_local
        vb = {k: b[k][seg] for k in ("gate_up_q", "gate_up_sf", "gate_up_global")}
        pc = starts.long()
        gu = O.grouped_gemm(q, sf, vb["gate_up_q"], vb["gate_up_sf"], pc, c, 2 * f)
        hidden, rowmax = O.rescale_swiglu_maximum(gu, pc, ag, vb["gate_up_global"])
        # each segment's max |hidden| (rows past the last segment count for it)
        ex = O.expert_of_rows(pc, torch.arange(rows))
        amax = torch.zeros(counts.numel(), dtype=torch.float32)
        amax.scatter_reduce_(0, ex, rowmax.to(torch.float32), "amax")
        hg = O.global_scale_from_amax(amax.to(BF16))
        hq, hsf = O.quantize_activations(hidden, pc, pc, rows, hg)
        res = (hq, hsf, amax.view(torch.int32))
        if out is not None:
            for dst, src in zip(out, res, strict=True):
                dst.copy_(src)
            return out
        return res

    def down(self, hq, hsf, hamax, r):
        f = self.hidden_features
        c = self.full["down_q"].shape[1]
        pc = r.pcsr.long()
        raw = O.grouped_gemm(hq, hsf, self.full["down_q"], self.full["down_sf"], pc, f, c)
        ex = O.expert_of_rows(pc, torch.arange(hq.shape[0]))
        hg = O.global_scale_from_amax(hamax.view(torch.float32).to(BF16))
        mult = O.bf16_round(hg[ex] * self.full["down_global"][ex]).unsqueeze(1)
        return (raw.to(torch.float32) * mult).to(BF16)

    def combine(self, rows, r, scaling, shared):
        ones = torch.ones(r.experts, dtype=torch.float32)
        return O.rescale_combine(rows, r.inverse, r.top_idx, r.gate, r.csr.long(), r.pcsr.long(), ones, ones,
                                 scaling, shared)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(rank: int, t: int, c: int, e: int, k: int, f: int):
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(t, c, generator=g).to(BF16)
    logits = torch.randn(t, e, generator=g)
    if rank == 1:
        logits[:, 0] += 3.0  # one rank concentrates on expert 0
    top_idx = logits.topk(k, -1).indices.contiguous()
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(BF16)
    shared = (torch.randn(t, c, generator=g) * 0.1).to(BF16)
    return x, top_idx, gate, shared


def _bank(e: int, c: int, f: int):
    g = torch.Generator().manual_seed(77)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(BF16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(BF16)
    return O.pack_routed_experts(gu, down)


def _worker(rank, world, port, shape, fail_rank, results, chunks=None, chunk_size=None, tokens=None):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        ep = pkg().expert_parallel
        t, c, e, k, f = shape
        if tokens is not None:
            t = tokens[rank]
        bank = _bank(e, c, f)
        local = ep.shard_packed_state(bank, rank, world)
        x, top_idx, gate, shared = _case(rank, t, c, e, k, f)
        if rank == fail_rank:
            raise RuntimeError("planted failure before the exchange")
        backend = OracleBackend(local, k, bank)

        def one(xc, tc, gc, sc):
            return ep.exchange_forward(xc, tc, gc, num_experts=e, scaling=2.5, backend=backend, shared=sc,
                                       chunks=chunks)

        if chunk_size is None:
            out = one(x, top_idx, gate, shared)
        else:
            out = ep.chunked_forward(one, x, top_idx, gate, shared, chunk_size)
        want = O.routed_forward(x, top_idx, gate, bank, 2.5, chunk_size or t, shared=shared)
        results.put((rank, "ok", bool(torch.equal(out.view(torch.int16), want.view(torch.int16))),
                     float(O.rel_l2(out, want))))
    except Exception as exc:  # reported to the parent
        results.put((rank, "error", type(exc).__name__, str(exc)[:200] + traceback.format_exc()[-300:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, shape, fail_rank=-1, chunks=None, chunk_size=None, tokens=None):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, fail_rank, results, chunks, chunk_size, tokens))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, *rest = results.get(timeout=240)
        out[rank] = rest
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,shape,chunks", [
    (2, (64, 256, 8, 2, 128), None),
    (2, (64, 256, 8, 2, 128), 2),      # return transfers in two expert groups per source
    (2, (40, 256, 4, 2, 256), None),   # two experts per rank, ragged counts
    (4, (48, 128, 8, 3, 128), None),
])
def test_exchange_matches_single_rank_layer(world, shape, chunks):
    res = _run(world, shape, chunks=chunks)
    for rank in range(world):
        status, *info = res[rank]
        assert status == "ok", info
        equal, err = info
        assert equal, (rank, err)


@pytest.mark.parametrize("world,tokens,chunk_size", [
    (2, (70, 40), 32),       # 3 chunks on rank 0, 2 on rank 1: rank 1 joins the last exchange empty
    (2, (50, 50), 64),       # one chunk each
    (4, (33, 0, 65, 17), 16),  # a rank without tokens joins every exchange empty
])
def test_dispatch_chunks_match_the_single_rank_chunk_loop(world, tokens, chunk_size):
    """Each rank's tokens go through the reference's dispatch-chunk loop
    (global scales per chunk and expert); ranks with fewer chunks still take
    part in every exchange, so no collective is left unmatched."""
    res = _run(world, (max(tokens), 256, 8, 2, 128), chunk_size=chunk_size, tokens=tokens)
    for rank in range(world):
        status, *info = res[rank]
        assert status == "ok", info
        equal, err = info
        assert equal, (rank, err)


def test_a_failing_rank_ends_the_others_with_an_error():
    res = _run(2, (32, 128, 4, 2, 128), fail_rank=1)
    assert res[1][0] == "error" and "planted failure" in res[1][2], res[1]
    assert res[0][0] == "error", res[0]  # the survivor's collective timed out or saw the peer leave
