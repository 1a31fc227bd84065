"""The MoE tail fused into what follows it (praxis.layers.MOE_TAIL_NORM:
praxis/kernels/moe_tail_triton.py:329-445 tail_add_norm_scale,
tail_add_mod_norm_scale, tail_residual_add), through the C ABI.

Bars: the new residual (with its modulation) bit-exact against the CPU
oracle; the whole tail (new residual and normalised rows) bit-exact against
the reference's eager path run by torch on the GPU (``x + y``, the modulation
``x * bf16(scale + 1) + shift``, the zero-centred RMSNorm as ``F.rms_norm``
in float32 with weight ``1 + w``, cast back, times the bf16 block scale),
whose reduction order and hardware reciprocal square root the kernel
reproduces; the normalised rows within one bf16 ulp of the oracle, whose
reciprocal square root is the correctly rounded one.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F
from conftest import assert_bytes_equal, pkg

from oracle import nvfp4_moe_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
GEOM = (26, 8, 2, 2, 3, 2)  # RF, RC, NREG, PW, WD, PH: 2 registers + (f y)=2, i<2, x<3, j<2


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


def eager_tail(x, y, w1=None, eps=1e-6, s=1.0, mod=None, mrow=None):
    """The reference's unfused path on the GPU (praxis/layers.py:214-224,
    :201-213; the modulation of praxis/kernels/moe_tail_triton.py:257-266)."""
    xo = x + y
    if mod is not None:
        c = x.shape[1]
        m = mod[mrow.to(mod.device)]
        sc1 = (m[:, c:].float() + 1.0).to(torch.bfloat16).float()
        xo = torch.addcmul(m[:, :c].float(), xo.float(), sc1).to(torch.bfloat16)
    if w1 is None:
        return xo, None
    h = F.rms_norm(xo.float(), (x.shape[1],), weight=w1, eps=eps).to(torch.bfloat16)
    return xo, h * torch.tensor(s, dtype=torch.bfloat16, device=x.device)


def routed_case(P, t, e, k, c, seed, shared=True):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(t, e, generator=g)
    top = logits.topk(k, -1).indices.contiguous().to(DEV)
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(torch.bfloat16).to(DEV)
    r = P.ops.dispatch(top, gate, e)
    rp = P.ops.padded_rows(t * k, e)
    rows = (torch.randn(rp, c, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16).to(DEV)
    sh = (torch.randn(t, c, generator=g) * 0.1).to(torch.bfloat16).to(DEV) if shared else None
    w1 = (1 + torch.randn(c, generator=g) * 0.1).float().to(DEV)
    mod = (torch.randn(64, 2 * c, generator=g) * 0.2).to(torch.bfloat16).to(DEV)
    return r, rows, x, sh, w1, mod


def oracle_y(r, rows, e, sh):
    ones = torch.ones(e)
    return O.rescale_combine(rows.cpu(), r.inverse.cpu(), r.top_idx.cpu(), r.gate.cpu(), r.csr.cpu().long(),
                             r.pcsr.cpu().long(), ones, ones, 2.5, None if sh is None else sh.cpu())


def check_h_vs_oracle(h, h_o):
    d = (h.cpu().view(torch.int16).int() - h_o.view(torch.int16).int()).abs()
    assert d.max().item() <= 1 and (d != 0).float().mean().item() < 1e-2


CASES = [(300, 8, 2, 512, True), (257, 64, 4, 3072, True), (64, 128, 8, 1024, False), (33, 16, 3, 3068, True),
         (52, 8, 1, 128, False), (9, 8, 8, 4, True)]


@pytest.mark.parametrize("t,e,k,c,shared", CASES)
def test_tail_add_norm_scale(P, t, e, k, c, shared):
    r, rows, x, sh, w1, _ = routed_case(P, t, e, k, c, seed=t + c, shared=shared)
    eps, s = 1e-6, 0.8125
    xo, h = P.ops.combine_tail(rows, r, 2.5, P.ops.Tail(x, w1, eps, s), shared=sh, rows_rescaled=True)
    y_o = oracle_y(r, rows, e, sh)
    if c % 8 == 0:  # the stock combine kernel of the library agrees with the oracle
        assert_bytes_equal(P.ops.combine(rows, r, 2.5, rows_rescaled=True, shared=sh), y_o)
    xo_e, h_e = eager_tail(x, y_o.to(DEV), w1, eps, s)
    assert_bytes_equal(xo, xo_e)
    assert_bytes_equal(h, h_e)
    xo_o, h_o = O.tail_add_norm_scale(y_o, x.cpu(), w1.cpu(), eps, s)
    assert_bytes_equal(xo.cpu(), xo_o)
    check_h_vs_oracle(h, h_o)


@pytest.mark.parametrize("t,e,k,c,shared", CASES[:4])
def test_tail_residual_add(P, t, e, k, c, shared):
    r, rows, x, sh, _, _ = routed_case(P, t, e, k, c, seed=3 * t + c, shared=shared)
    xo, h = P.ops.combine_tail(rows, r, 2.5, P.ops.Tail(x), shared=sh, rows_rescaled=True)
    assert h is None
    assert_bytes_equal(xo.cpu(), O.tail_residual_add(oracle_y(r, rows, e, sh), x.cpu()))


@pytest.mark.parametrize("geom", [None, GEOM])
@pytest.mark.parametrize("fma", [True, False])
@pytest.mark.parametrize("t,e,k,c,shared", [(52, 8, 2, 512, True), (41, 64, 8, 3072, True), (30, 16, 4, 1020, False)])
def test_tail_add_mod_norm_scale(P, t, e, k, c, shared, geom, fma):
    r, rows, x, sh, w1, mod = routed_case(P, t, e, k, c, seed=5 * t + c, shared=shared)
    eps, s = 1e-6, 1.25
    tail = P.ops.Tail(x, w1, eps, s, mod=mod, mod_fma=fma, mod_geom=geom)
    xo, h = P.ops.combine_tail(rows, r, 2.5, tail, shared=sh, rows_rescaled=True)
    y_o = oracle_y(r, rows, e, sh)
    mrow = O.mod_row_map(t, geom)
    xo_e, h_e = eager_tail(x, y_o.to(DEV), w1, eps, s, mod, mrow)
    assert_bytes_equal(xo, xo_e)
    assert_bytes_equal(h, h_e)
    xo_o, h_o = O.tail_add_norm_scale(y_o, x.cpu(), w1.cpu(), eps, s, mod=mod.cpu(), geom=geom)
    assert_bytes_equal(xo.cpu(), xo_o)
    check_h_vs_oracle(h, h_o)


def test_tail_rejects_bad_requests(P):
    r, rows, x, sh, w1, mod = routed_case(P, 16, 8, 2, 512, seed=9)
    with pytest.raises(ValueError):  # the modulation needs the norm
        P.ops.combine_tail(rows, r, 2.5, P.ops.Tail(x, mod=mod), shared=sh, rows_rescaled=True)
    with pytest.raises(ValueError):  # too few modulation rows for the row map
        P.ops.combine_tail(rows, r, 2.5, P.ops.Tail(x, w1, mod=mod[:3]), shared=sh, rows_rescaled=True)
    with pytest.raises(ValueError):
        P.ops.combine_tail(rows, r, 2.5, P.ops.Tail(x[:, :256].contiguous(), w1), shared=sh, rows_rescaled=True)


def _bank(P, e, c, f, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gu = (torch.randn(e, c, 2 * f, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    bank = P.pack_routed_experts(gu, down, keep_on_device=True)
    bank.prepare()
    return bank


@pytest.mark.parametrize("with_mod", [False, True])
def test_routed_forward_tail_equals_unfused(P, with_mod):
    """The whole routed forward with the fused tail, several dispatch chunks
    (the compact modulation rows keep their global row map across chunks)."""
    t, c, e, k, f = 520, 1024, 32, 2, 2048
    bank = _bank(P, e, c, f, 61)
    gh = torch.Generator().manual_seed(62)
    x = torch.randn(t, c, generator=gh).to(torch.bfloat16).to(DEV)
    resid = torch.randn(t, c, generator=gh).to(torch.bfloat16).to(DEV)
    sh = (torch.randn(t, c, generator=gh) * 0.1).to(torch.bfloat16).to(DEV)
    top = torch.randn(t, e, generator=gh).topk(k, -1).indices.contiguous().to(DEV)
    gate = torch.softmax(torch.randn(t, k, generator=gh), -1).to(torch.bfloat16).to(DEV)
    w1 = (1 + torch.randn(c, generator=gh) * 0.1).float().to(DEV)
    mod = (torch.randn(160, 2 * c, generator=gh) * 0.2).to(torch.bfloat16).to(DEV) if with_mod else None
    y = bank.routed_forward_with_shared(x, top, gate, scaling=2.5, chunk_size=200, shared=sh)
    xo_e, h_e = eager_tail(resid, y, w1, 1e-6, 1.25, mod, O.mod_row_map(t, GEOM) if with_mod else None)
    tail = P.ops.Tail(resid, w1, 1e-6, 1.25, mod=mod, mod_geom=GEOM if with_mod else None)
    xo, h = P.routed_forward_tail(bank, x, top, gate, scaling=2.5, chunk_size=200, tail=tail, shared=sh)
    assert_bytes_equal(xo, xo_e)
    assert_bytes_equal(h, h_e)
    xo2, h2 = P.routed_forward_tail(bank, x, top, gate, scaling=2.5, chunk_size=200, tail=P.ops.Tail(resid),
                                    shared=sh)
    assert h2 is None
    assert_bytes_equal(xo2, resid + y)
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def test_module_forward_tail(P):
    t, c, e, k, f = 256, 512, 8, 2, 1024
    g = torch.Generator().manual_seed(71)
    mod_ = P.B200MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=t, shared_expert=False).to(DEV)
    with torch.no_grad():
        mod_.router.weight.copy_((torch.randn(e, c, generator=g) * 0.02).to(DEV))
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(torch.bfloat16)
    mod_.set_routed_weights(gu.to(DEV), down.to(DEV))

    class Norm(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = torch.nn.Parameter(torch.randn(c, generator=g) * 0.1)
            self.eps = 1e-6

    norm = Norm().to(DEV)
    x = torch.randn(2, t // 2, c, generator=g).to(torch.bfloat16).to(DEV)
    resid = torch.randn(2, t // 2, c, generator=g).to(torch.bfloat16).to(DEV)
    scale = torch.tensor(0.75, dtype=torch.bfloat16)
    y = mod_(x)
    xo, h = mod_.forward_tail(x, resid, norm, scale)
    xo_e, h_e = eager_tail(resid.reshape(t, c), y.reshape(t, c), 1 + norm.weight.detach().float(), 1e-6, 0.75)
    assert_bytes_equal(xo, xo_e.reshape(xo.shape))
    assert_bytes_equal(h, h_e.reshape(h.shape))
    xo2, h2 = mod_.forward_tail(x, resid)
    assert h2 is None
    assert_bytes_equal(xo2, resid + y)
