"""The calibrated FC1 FP4-output path (praxis/kernels/
nvfp4_swiglu.py:40-74, praxis/quantization/nvfp4.py:235-260, :327-339),
through the C ABI.

The reference's path runs a FlashInfer act-fusion kernel (flashinfer
0.6.18, not installed here) whose bits are its own; this library's path
quantizes the dynamic path's SwiGLU hidden values with the reference's
quantize recipe at the frozen global. Bars: the fused epilogue's FP4 codes
and scale bytes bit-exact against the hidden quantize kernel at that global;
the layer bit-exact against the same chain run stage by stage, and within
rel-L2 1e-2 of the oracle's dequantised chain with that hidden global.
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


def _case(P, t, c, e, k, f, seed):
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(torch.bfloat16)
    bank = P.pack_routed_experts(gu.to(DEV), down.to(DEV), keep_on_device=True)
    bank.prepare()
    x = torch.randn(t, c, generator=g).to(torch.bfloat16).to(DEV)
    top = torch.randn(t, e, generator=g).topk(k, -1).indices.contiguous().to(DEV)
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(torch.bfloat16).to(DEV)
    return bank, x, top, gate, gu, down


def _live_rows(r) -> torch.Tensor:
    n = int(r.num_tiles[0])
    row0 = r.tiles[:n, 1].cpu().long()
    return (row0.unsqueeze(1) + torch.arange(128)).reshape(-1)


@pytest.mark.parametrize("t,c,e,k,f", [(512, 1024, 16, 4, 512), (300, 3072, 64, 4, 1536)])
@pytest.mark.parametrize("factor", [0.25, 1.0, 4.0])
def test_fp4_epilogue_equals_hidden_quantize_at_the_frozen_global(P, t, c, e, k, f, factor):
    bank, x, top, gate, _, _ = _case(P, t, c, e, k, f, seed=t + c)
    kw = bank.kernel_weights()
    amax = P.ops.row_amax(x)
    r = P.ops.dispatch(top, gate, e, amax)
    aq, asf = P.ops.quantize_gather(x, r, r.act_global)
    hamax = torch.zeros(e, dtype=torch.int32, device=DEV)
    hidden = P.ops.grouped_gemm(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, epilogue=P.capi.EPI_SWIGLU,
                                act_global=r.act_global, w_global=bank.gate_up_global, amax_out=hamax)
    # a calibrated-style global: 2 * max |hidden| / 2688, scaled (some blocks saturate at 0.25)
    g = float(2.0 * hidden.float().abs().max() / 2688.0 * factor)
    hq_ref, hsf_ref = P.ops.quantize_rows(hidden, r, torch.full((e,), g, device=DEV))
    hq, hsf = P.ops.grouped_gemm_swiglu_fp4(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, act_global=r.act_global,
                                            w_global=bank.gate_up_global, hidden_global=g)
    rows = _live_rows(r)
    assert_bytes_equal(hq.cpu()[rows], hq_ref.cpu()[rows])
    kb = f // 16
    rp = hq.shape[0]
    assert_bytes_equal(O.unswizzle_scales(hsf.cpu().reshape(-1), rp, kb)[rows],
                       O.unswizzle_scales(hsf_ref.cpu().reshape(-1), rp, kb)[rows])
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def test_calibrated_bank_forward(P):
    t, c, e, k, f = 400, 1024, 32, 4, 512
    bank, x, top, gate, gu, down = _case(P, t, c, e, k, f, seed=7)
    dynamic = bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t)
    g = 0.01
    bank.set_fused_swiglu_scale(g)
    y = bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=150)
    # the same chain stage by stage (per dispatch chunk)
    kw = bank.kernel_weights()
    for a in range(0, t, 150):
        b = min(a + 150, t)
        amax = P.ops.row_amax(x[a:b])
        r = P.ops.dispatch(top[a:b].contiguous(), gate[a:b].contiguous(), e, amax)
        aq, asf = P.ops.quantize_gather(x[a:b], r, r.act_global)
        hq, hsf = P.ops.grouped_gemm_swiglu_fp4(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, act_global=r.act_global,
                                                w_global=bank.gate_up_global, hidden_global=g)
        rows = P.ops.grouped_gemm(hq, hsf, bank.down_q, kw.down_sf, r, epilogue=P.capi.EPI_RESCALE,
                                  act_global=torch.full((e,), g, device=DEV), w_global=bank.down_global)
        want = P.ops.combine(rows, r, 2.5, rows_rescaled=True)
        assert_bytes_equal(y[a:b], want)
    # against the oracle's chain with the frozen hidden global
    obank = {name: buf.cpu() for name, buf in bank.named_buffers()}
    ref = O.routed_forward(x.cpu(), top.cpu(), gate.cpu(), obank, 2.5, 150, hidden_global=g)
    assert O.rel_l2(y.cpu(), ref) <= 1e-2
    # back to dynamic scales
    bank.set_fused_swiglu_scale(None)
    assert_bytes_equal(bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t), dynamic)
    with pytest.raises(ValueError):
        bank.set_fused_swiglu_scale(-1.0)
    with pytest.raises(ValueError):
        bank.set_fused_swiglu_scale(float("inf"))
