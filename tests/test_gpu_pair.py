"""Lockstep pairs (classifier-free guidance): ``MoEFeedForward.forward_pair``
(praxis/layers.py:1779-1853), the bank's ``routed_forward_pair``
(praxis/quantization/nvfp4.py:467-488) and the P = 2 dispatch of
``router_fused.route_dispatch`` / ``dispatch_ref``
(praxis/kernels/router_fused.py:738-852), through the C ABI.

Bars: the P = 2 dispatch metadata bit-exact against the oracle's restatement
of ``dispatch_ref`` (order, inverse, tokens, sorted gates, seg_csr, offsets),
the per-(expert, input) padding and global scales against the per-group
formulas; every paired output bit-exact against the same input run alone
(the reference's contract: ``[self(x) for x in xs]``).
"""

from __future__ import annotations

import pytest
import torch
from conftest import assert_bytes_equal, pkg

from oracle import nvfp4_moe_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


def routing(t, e, k, seed):
    g = torch.Generator().manual_seed(seed)
    top = torch.randn(t, e, generator=g).topk(k, -1).indices.contiguous()
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(torch.bfloat16)
    return top, gate


@pytest.mark.parametrize("t0,t1,e,k", [(300, 200, 8, 2), (1, 1000, 64, 4), (513, 513, 128, 8), (0, 77, 16, 3),
                                       (90, 0, 16, 3), (4099, 2000, 64, 4)])
def test_dispatch_pair_bit_exact(P, t0, t1, e, k):
    t = t0 + t1
    top, gate = routing(t, e, k, seed=t + e)
    x = (torch.randn(t, 128, generator=torch.Generator().manual_seed(3)) * 3).to(torch.bfloat16)
    amax = O.row_amax(x)
    r = P.ops.dispatch(top.to(DEV), gate.to(DEV), e, amax.to(DEV), rows=(t0, t1))
    order, inverse, tokens, sorted_gate, seg_csr, offsets = O.dispatch_passes(top, gate, e, (t0, t1))
    assert r.rows == (t0, t1)
    assert_bytes_equal(r.order.cpu(), order)
    assert_bytes_equal(r.inverse.cpu(), inverse)
    assert_bytes_equal(r.tokens.cpu(), tokens)
    assert_bytes_equal(r.sorted_gate.cpu(), sorted_gate)
    assert_bytes_equal(r.seg_csr.cpu(), seg_csr)
    assert_bytes_equal(r.offsets.cpu().contiguous(), offsets)
    pcsr = O.pad_csr(seg_csr)
    assert_bytes_equal(r.pcsr.cpu(), pcsr)
    # per (expert, input) group: the global scale of that group's rows alone
    assert_bytes_equal(r.act_global.cpu(), O.segment_global_scales(amax, seg_csr, tokens))
    counts = (seg_csr[1:] - seg_csr[:-1]).long()
    n, npairs = r.num_tiles.cpu().tolist()
    assert n == int(((counts + 127) // 128).sum()) and npairs == int(((counts + 255) // 256).sum())
    tiles = r.tiles[:n].cpu()
    i = 0
    for grp in range(2 * e):
        for j in range((int(counts[grp]) + 127) // 128):
            assert tiles[i].tolist() == [grp, int(pcsr[grp]) + 128 * j, min(128, int(counts[grp]) - 128 * j), 0]
            i += 1


def test_route_dispatch_pair(P):
    t0, t1, e, k = 200, 300, 128, 8
    g = torch.Generator().manual_seed(8)
    logits = torch.randn(t0 + t1, e, generator=g).to(DEV)
    bias = (torch.randn(e, generator=g) * 0.1).to(DEV)
    r = P.ops.route_dispatch(logits, bias, (t0, t1), top_k=k)
    top, gate = P.ops.route(logits, bias, k)
    assert_bytes_equal(r.top_idx, top)
    assert_bytes_equal(r.gate, gate)
    order, inverse, _, _, seg_csr, offsets = O.dispatch_passes(top.cpu(), gate.cpu(), e, (t0, t1))
    assert_bytes_equal(r.order.cpu(), order)
    assert_bytes_equal(r.seg_csr.cpu(), seg_csr)
    assert_bytes_equal(r.offsets.cpu().contiguous(), offsets)
    with pytest.raises(ValueError):
        P.ops.route_dispatch(logits, bias, (t0, t1 + 1), top_k=k)


def _bank(P, e, c, f, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gu = (torch.randn(e, c, 2 * f, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    bank = P.pack_routed_experts(gu, down, keep_on_device=True)
    bank.prepare()
    return bank, gu, down


@pytest.mark.parametrize("t0,t1,c,e,k,f,adjacent", [
    (256, 256, 512, 8, 2, 1024, True),
    (300, 129, 1024, 64, 4, 512, False),
    (1, 700, 512, 32, 2, 256, True),
    (512, 512, 3072, 128, 8, 1280, True),  # the checkpoint shape (E=128, top-8, F=1280)
])
def test_routed_forward_pair_equals_each_input_alone(P, t0, t1, c, e, k, f, adjacent):
    bank, _, _ = _bank(P, e, c, f, seed=c + e)
    g = torch.Generator().manual_seed(t0 + t1)
    buf = torch.randn(t0 + t1, c, generator=g).to(torch.bfloat16).to(DEV)
    xs = [buf[:t0], buf[t0:]] if adjacent else [buf[:t0].clone(), buf[t0:].clone()]
    top, gate = routing(t0 + t1, e, k, seed=5)
    tops, gates = [top[:t0].to(DEV), top[t0:].to(DEV)], [gate[:t0].to(DEV), gate[t0:].to(DEV)]
    shb = (torch.randn(t0 + t1, c, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    sh = [shb[:t0], shb[t0:]]
    ys = bank.routed_forward_pair(xs, tops, gates, scaling=2.5, shared=sh)
    for x, tp, gt, s, y in zip(xs, tops, gates, sh, ys, strict=True):
        alone = bank.routed_forward_with_shared(x, tp, gt, scaling=2.5, chunk_size=x.shape[0], shared=s)
        assert_bytes_equal(y, alone)
    ys2 = bank.routed_forward_pair(xs, tops, gates, scaling=2.5)
    for x, tp, gt, y in zip(xs, tops, gates, ys2, strict=True):
        assert_bytes_equal(y, bank.routed_forward(x, tp, gt, scaling=2.5, chunk_size=x.shape[0]))
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def test_routed_forward_pair_with_tail(P):
    t0, t1, c, e, k, f = 200, 300, 1024, 16, 4, 512
    bank, _, _ = _bank(P, e, c, f, seed=12)
    g = torch.Generator().manual_seed(13)
    x = torch.randn(t0 + t1, c, generator=g).to(torch.bfloat16).to(DEV)
    resid = torch.randn(t0 + t1, c, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (1 + torch.randn(c, generator=g) * 0.1).float().to(DEV)
    top, gate = routing(t0 + t1, e, k, seed=14)
    top, gate = top.to(DEV), gate.to(DEV)
    tail = P.ops.Tail(resid, w1, 1e-6, 0.5)
    out = bank.routed_forward_pair([x[:t0], x[t0:]], [top[:t0], top[t0:]], [gate[:t0], gate[t0:]], scaling=2.5,
                                   tail=tail)
    for i, (a, b) in enumerate(((0, t0), (t0, t0 + t1))):
        want = P.routed_forward_tail(bank, x[a:b], top[a:b], gate[a:b], scaling=2.5, chunk_size=b - a,
                                     tail=P.ops.Tail(resid[a:b], w1, 1e-6, 0.5))
        assert_bytes_equal(out[i][0], want[0])
        assert_bytes_equal(out[i][1], want[1])


def test_router_logits_do_not_depend_on_row_position(P):
    """A token's logits are the same wherever its row sits in the call: what
    lets a pair, a router_rows slice and a lone call route alike."""
    g = torch.Generator().manual_seed(41)
    x = torch.randn(1000, 3072, generator=g).to(torch.bfloat16).to(DEV)
    terms = P.ops.split_router_weight((torch.randn(128, 3072, generator=g) * 0.02).to(DEV))
    full, amax = P.ops.router_logits(x, terms)
    for a, b in ((0, 1000), (5, 600), (128, 1000), (777, 778), (300, 428)):
        part, pamax = P.ops.router_logits(x[a:b], terms)
        assert_bytes_equal(part, full[a:b])
        assert_bytes_equal(pamax, amax[a:b])


@pytest.mark.parametrize("t0,t1,c,e,k,f", [(384, 128, 512, 32, 4, 256), (2048, 2048, 1024, 128, 8, 512)])
def test_moe_forward_pair_with_router(P, t0, t1, c, e, k, f):
    """The whole chunk with the router inside (one C call for both inputs)
    against the same call per input."""
    bank, _, _ = _bank(P, e, c, f, seed=21)
    kw = bank.kernel_weights()
    g = torch.Generator().manual_seed(22)
    x = torch.randn(t0 + t1, c, generator=g).to(torch.bfloat16).to(DEV)
    terms = P.ops.split_router_weight((torch.randn(e, c, generator=g) * 0.05).to(DEV))
    bias = torch.zeros(e, device=DEV)
    args = (kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q, kw.down_sf, bank.down_global, 2.5)
    out, top, gate = P.ops.moe_forward(x, None, None, *args, router_terms=terms, router_bias=bias, top_k=k,
                                       rows=(t0, t1))
    for a, b in ((0, t0), (t0, t0 + t1)):
        o1, tp1, g1 = P.ops.moe_forward(x[a:b], None, None, *args, router_terms=terms, router_bias=bias, top_k=k)
        assert_bytes_equal(out[a:b], o1)
        assert_bytes_equal(top[a:b], tp1)
        assert_bytes_equal(gate[a:b], g1)


def test_module_forward_pair_equals_forward(P):
    t, c, e, k, f = 256, 512, 16, 2, 512
    g = torch.Generator().manual_seed(31)
    mod = P.B200MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=t).to(DEV)
    with torch.no_grad():
        mod.router.weight.copy_((torch.randn(e, c, generator=g) * 0.05).to(DEV))
        mod.shared.gate_up.copy_((torch.randn(c, 2 * f, generator=g) * 0.02).to(DEV))
        mod.shared.down.copy_((torch.randn(f, c, generator=g) * 0.02).to(DEV))
    mod = mod.to(torch.bfloat16)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(torch.bfloat16)
    mod.set_routed_weights(gu.to(DEV), down.to(DEV))
    xs = [torch.randn(2, t // 2, c, generator=g).to(torch.bfloat16).to(DEV),
          torch.randn(1, 100, c, generator=g).to(torch.bfloat16).to(DEV)]
    ys = mod.forward_pair(xs)
    for x, y in zip(xs, ys, strict=True):
        assert y.shape == x.shape
        assert_bytes_equal(y, mod(x))
    # over the dispatch chunk: falls back to one forward per input
    big = torch.randn(t + 1, c, generator=g).to(torch.bfloat16).to(DEV)
    ys = mod.forward_pair([big, xs[1]])
    assert_bytes_equal(ys[0], mod(big))
