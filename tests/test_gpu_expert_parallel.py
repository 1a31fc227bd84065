"""Expert parallelism on the GPU kernels.

* two ranks emulated on one GPU: each "rank" runs ``praxis_b200_expert_forward``
  on the rows it would receive (segments of two sources, weights = its half of
  the bank); after the emulated return and combine, every source's output must
  equal the single-GPU bank forward of its tokens bit for bit;
* the real exchange (``exchange_forward``) over NCCL with one rank;
* the real exchange over NCCL with two ranks when two GPUs are visible;
* the copy-engine exchange into IPC-mapped peer buffers with two ranks when
  two GPUs are visible, alone and with half of every transfer done by the SM
  copy kernel: several forwards with changing token counts (buffer reuse and
  growth), each bit for bit equal to the single-GPU bank.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from conftest import pkg

from oracle import nvfp4_moe_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


def _tokens(seed, t, c, e, k, skew=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, c, generator=g).to(BF16)
    logits = torch.randn(t, e, generator=g)
    if skew:
        logits[:, 1] += 2.5
    top = logits.topk(k, -1).indices.contiguous()
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(BF16)
    shared = (torch.randn(t, c, generator=g) * 0.1).to(BF16)
    return x, top, gate, shared


def _packed(e, c, f, seed=5):
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(BF16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(BF16)
    return O.pack_routed_experts(gu, down)


@pytest.mark.parametrize("t,c,e,k,f", [(300, 512, 8, 2, 256), (1000, 256, 16, 4, 384), (64, 256, 4, 1, 128)])
def test_two_rank_exchange_emulated_on_one_gpu(P, t, c, e, k, f):
    world = 2
    el = e // world
    state = _packed(e, c, f)
    full = P.B200NVFP4RoutedExperts.from_packed({n: v.clone() for n, v in state.items()}).to(DEV)
    local = [P.B200NVFP4RoutedExperts.from_packed(P.expert_parallel.shard_packed_state(state, r, world)).to(DEV)
             for r in range(world)]
    sources = []
    for s in range(world):
        x, top, gate, shared = (v.to(DEV) for v in _tokens(10 + s, t, c, e, k, skew=s == 1))
        r = P.ops.dispatch(top, gate, e, P.ops.row_amax(x), full=False)
        q, sf = P.ops.quantize_gather(x, r, r.act_global)
        sources.append((x, top, gate, shared, r, q, sf, r.pcsr.cpu().long(), r.csr.cpu().long()))
    rows_back = [torch.empty(int(src[7][-1]), c, dtype=BF16, device=DEV) for src in sources]
    for d in range(world):  # expert rank d
        qs, sfs, counts, starts, ags, base = [], [], [], [], [], 0
        for s, (_x, _t, _g, _sh, r, q, sf, pcsr, csr) in enumerate(sources):
            lo, hi = int(pcsr[d * el]), int(pcsr[(d + 1) * el])
            qs.append(q[lo:hi])
            sfs.append(sf[lo:hi])
            for e_loc in range(el):
                ge = d * el + e_loc
                counts.append(int(csr[ge + 1] - csr[ge]))
                starts.append(base + int(pcsr[ge]) - lo)
                ags.append(r.act_global[ge].item())
            base += hi - lo
        starts.append(base)
        kw = local[d].kernel_weights()
        b = local[d]
        out = P.ops.expert_forward(
            torch.cat(qs), torch.cat(sfs), torch.tensor(counts, dtype=torch.int32, device=DEV),
            torch.tensor(starts, dtype=torch.int32, device=DEV), torch.tensor(ags, dtype=torch.float32, device=DEV),
            kw.gate_up_q, kw.gate_up_sf, b.gate_up_global, b.down_q, kw.down_sf, b.down_global,
            gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout)
        off = 0
        for s, src in enumerate(sources):
            pcsr = src[7]
            lo, hi = int(pcsr[d * el]), int(pcsr[(d + 1) * el])
            rows_back[s][lo:hi] = out[off:off + hi - lo]
            off += hi - lo
    for s, (x, top, gate, shared, r, *_rest) in enumerate(sources):
        got = P.ops.combine(rows_back[s], r, 2.5, rows_rescaled=True, shared=shared)
        want = full.routed_forward_with_shared(x, top, gate, scaling=2.5, chunk_size=t, shared=shared)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), s
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_exchange_forward_one_rank_nccl(P):
    t, c, e, k, f = 700, 512, 8, 2, 256
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    try:
        state = _packed(e, c, f)
        ep = P.expert_parallel.ExpertParallelRoutedExperts.from_packed({n: v.to(DEV) for n, v in state.items()})
        full = P.B200NVFP4RoutedExperts.from_packed({n: v.clone() for n, v in state.items()}).to(DEV)
        x, top, gate, shared = (v.to(DEV) for v in _tokens(3, t, c, e, k))
        got = ep.routed_forward_with_shared(x, top, gate, scaling=2.5, shared=shared)
        want = full.routed_forward_with_shared(x, top, gate, scaling=2.5, chunk_size=t, shared=shared)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    finally:
        dist.destroy_process_group()


def _nccl_worker(rank, world, port, results):
    try:
        torch.cuda.set_device(rank)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        p = pkg()
        t, c, e, k, f = 900, 512, 8, 2, 256
        state = _packed(e, c, f)
        dev = torch.device("cuda", rank)
        ep = p.expert_parallel.ExpertParallelRoutedExperts.from_packed({n: v.to(dev) for n, v in state.items()},
                                                                      transport="nccl")
        full = p.B200NVFP4RoutedExperts.from_packed({n: v.clone() for n, v in state.items()}).to(dev)
        x, top, gate, shared = (v.to(dev) for v in _tokens(20 + rank, t, c, e, k, skew=rank == 1))
        got = ep.routed_forward_with_shared(x, top, gate, scaling=2.5, shared=shared)
        want = full.routed_forward_with_shared(x, top, gate, scaling=2.5, chunk_size=t, shared=shared)
        torch.cuda.synchronize()
        results.put((rank, bool(torch.equal(got.view(torch.int16), want.view(torch.int16))), ""))
        dist.barrier()
    except Exception:
        results.put((rank, False, traceback.format_exc()[-600:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_exchange_forward_two_ranks_nccl(P):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, results)) for r in range(2)]
    for proc in procs:
        proc.start()
    res = {}
    for _ in range(2):
        rank, ok, info = results.get(timeout=300)
        res[rank] = (ok, info)
    for proc in procs:
        proc.join(timeout=120)
    assert all(ok for ok, _ in res.values()), res


def _peer_worker(rank, world, port, results, sm_copy_fraction=0.0):
    try:
        torch.cuda.set_device(rank)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
        dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        p = pkg()
        c, e, k, f = 512, 8, 2, 256
        state = _packed(e, c, f)
        dev = torch.device("cuda", rank)
        ep = p.expert_parallel.ExpertParallelRoutedExperts.from_packed({n: v.to(dev) for n, v in state.items()},
                                                                      sm_copy_fraction=sm_copy_fraction)
        assert ep.transport == "peer"
        full = p.B200NVFP4RoutedExperts.from_packed({n: v.clone() for n, v in state.items()}).to(dev)
        ok = True
        # token counts differ between ranks and grow (buffer growth), then shrink (reuse)
        for it, t in enumerate([(900, 700), (640, 1500), (300, 200), (1500, 1500)]):
            x, top, gate, shared = (v.to(dev) for v in _tokens(40 + 7 * it + rank, t[rank], c, e, k, skew=rank == 1))
            got = ep.routed_forward_with_shared(x, top, gate, scaling=2.5, shared=shared)
            want = full.routed_forward_with_shared(x, top, gate, scaling=2.5, chunk_size=t[rank], shared=shared)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(got.view(torch.int16), want.view(torch.int16)))
        ep.close()
        results.put((rank, ok and p.capi.device_error(rank) == 0, ""))
        dist.barrier()
    except Exception:
        results.put((rank, False, traceback.format_exc()[-600:]))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("sm_copy_fraction", [0.0, 0.5])
def test_peer_exchange_two_ranks(P, sm_copy_fraction):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, results, sm_copy_fraction)) for r in range(2)]
    for proc in procs:
        proc.start()
    res = {}
    for _ in range(2):
        rank, ok, info = results.get(timeout=300)
        res[rank] = (ok, info)
    for proc in procs:
        proc.join(timeout=120)
    assert all(ok for ok, _ in res.values()), res


def test_peer_flag_wait_is_bounded(P):
    """The exchange's arrival wait (``praxis_b200_wait_value``): a flag that
    is already set passes; a flag that nothing sets gives up after its limit
    with the peer-timeout error code instead of hanging the stream."""
    import ctypes as C

    lib = P.capi.load()
    dev = torch.cuda.current_device()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    flag = torch.tensor([7], dtype=torch.int32, device=DEV)
    P.capi.device_error(dev)  # clear
    P.capi.check(lib.praxis_b200_wait_value(C.c_void_p(flag.data_ptr()), 7, 1_000_000_000, dev, stream))
    torch.cuda.synchronize()
    assert P.capi.device_error(dev) == 0
    P.capi.check(lib.praxis_b200_wait_value(C.c_void_p(flag.data_ptr()), 8, 2_000_000, dev, stream))
    torch.cuda.synchronize()
    assert P.capi.device_error(dev) == 5
    assert P.capi.device_error(dev) == 0  # read and cleared
    with pytest.raises(ValueError):  # a wait must have a limit
        P.capi.check(lib.praxis_b200_wait_value(C.c_void_p(flag.data_ptr()), 7, 0, dev, stream))
