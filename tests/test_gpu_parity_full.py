"""Parity at the BASELINE shapes, every stage through the C ABI.

The small-shape tests in test_gpu_parity.py pin each kernel's arithmetic;
this file runs the same checks on the shapes every bench number is measured
on, where K = 3072 (gate/up GEMM) and K = 1536 (down GEMM), the padding and
tile tables of 16,384 tokens, and skewed routing exercise code paths the
small shapes do not reach:

  config 2  T=16384, C=3072, E=64, k=4, F=1536
  config 3  config 2 with Zipf(1.2) expert popularity (top expert picked by
            about 30% of tokens, through the routing bias)
  config 5  T=512, C=1024, E=32, k=2, F=2048

For each: the measured fused path (praxis_b200_moe_forward with the router)
equals the stage-by-stage ops bit for bit; routing on identical logits is
bit-exact against the reference's stock routing ops run by torch on the GPU
(and the CPU oracle, up to picks its CPU sigmoid flips within an ulp);
dispatch, the FP4 codes and scale bytes of both quantizations, the hidden
global scales and the combine are bit-exact against the CPU oracle; both
GEMMs are checked on a sample of rows of every expert against exact
dequantised products (float64 accumulation, then the tensor core's
float32 -> bf16 rounding: at most 1% of elements one bf16 ulp apart,
relative L2 below 2e-3); the layer output is within relative L2 1e-2 of the
oracle's dequantised chain on the same routing.
"""

from __future__ import annotations

import importlib.util
import sys

import pytest
import torch
from conftest import ROOT, assert_bytes_equal, pkg

from oracle import nvfp4_moe_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
SHAPES = {
    # tokens, dim, experts, top_k, hidden, skewed routing
    "2": (16384, 3072, 64, 4, 1536, False),
    "3": (16384, 3072, 64, 4, 1536, True),
    "5": (512, 1024, 32, 2, 2048, False),
}
SCALING = 2.5


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_tests", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("bench_for_tests", mod)
    spec.loader.exec_module(mod)
    return mod


def ulp_mismatch(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().cpu().view(torch.int16).int()
    b = b.detach().cpu().view(torch.int16).int()
    return (a != b).float().mean().item()


def dequant_rows_sample(q: torch.Tensor, sf: torch.Tensor, rows: torch.Tensor, k: int) -> torch.Tensor:
    """float64 values of the listed rows of a padded [Rp, K/2] FP4 matrix with
    compact swizzled scales [Rp, K/16] (the oracle's formats, row by row)."""
    rp = q.shape[0]
    scales = O.e4m3_values(O.unswizzle_scales(sf, rp, k // 16)[rows]).to(torch.float64)
    vals = O.e2m1_values(O.unpack_nibbles(q[rows])).to(torch.float64)
    return vals * scales.repeat_interleave(16, dim=1)


def sample_rows(pcsr: torch.Tensor, csr: torch.Tensor, per_expert: int, seed: int) -> torch.Tensor:
    """Up to ``per_expert`` routed rows of every expert (first, last and
    random ones), as padded row indices."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for ex in range(csr.numel() - 1):
        n = int(csr[ex + 1] - csr[ex])
        if n == 0:
            continue
        pick = {0, n - 1} | set(torch.randint(0, n, (per_expert,), generator=g).tolist())
        out.extend(int(pcsr[ex]) + i for i in sorted(pick))
    return torch.tensor(out, dtype=torch.int64)


def gemm_rows_oracle(a: torch.Tensor, experts: torch.Tensor, b_q: torch.Tensor, b_sf: torch.Tensor, n: int,
                     k: int) -> torch.Tensor:
    """bf16(f32(a @ W_e^T)) per row with float64 products of the dequantised
    operands (praxis/kernels/nvfp4.py:355-419, alpha = 1)."""
    out = torch.empty(a.shape[0], n, dtype=torch.bfloat16)
    for ex in experts.unique().tolist():
        sel = (experts == ex).nonzero().flatten()
        w = O.dequant_matrix(b_q[ex], b_sf[ex], n, k).to(torch.float64)
        out[sel] = (a[sel] @ w.t()).to(torch.float32).to(torch.bfloat16)
    return out


@pytest.fixture(scope="module", params=sorted(SHAPES))
def layer(request):
    """One layer forward of a BASELINE shape on the GPU, stage by stage and
    fused, with every intermediate copied to the host."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    P = pkg()
    P.capi.load()
    ops, capi = P.ops, P.capi
    name = request.param
    t, c, e, k, f, skew = SHAPES[name]
    g = torch.Generator().manual_seed(2000 + int(name))
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    router = torch.randn(e, c, generator=g) * (1.0 / c) ** 0.5
    bias = _bench().zipf_selection_bias(e) if skew else torch.zeros(e)
    gw = torch.Generator(device=DEV).manual_seed(3000 + int(name))
    gu_w = (torch.randn(e, c, 2 * f, generator=gw, device=DEV) * 0.02).to(torch.bfloat16)
    dn_w = (torch.randn(e, f, c, generator=gw, device=DEV) * 0.02).to(torch.bfloat16)
    bank = P.pack_routed_experts(gu_w, dn_w, keep_on_device=True)
    bank.prepare()
    kw = bank.kernel_weights()
    # two experts' bf16 weights, to pin the full-size packing against the oracle
    probe = {ex: (gu_w[ex].cpu(), dn_w[ex].cpu()) for ex in (0, e - 1)}
    del gu_w, dn_w

    xd = x.to(DEV)
    terms = ops.split_router_weight(router.to(DEV))
    bias_d = bias.to(DEV)
    logits, amax = ops.router_logits(xd, terms)
    top, gate = ops.route(logits, bias_d, k)
    r = ops.dispatch(top, gate, e, amax)
    aq, asf = ops.quantize_gather(xd, r, r.act_global)
    hamax = torch.zeros(e, dtype=torch.int32, device=DEV)
    a_sf = ops.replicate_scales(asf, 128) if kw.gate_up_sf_layout == capi.SF_REPLICATED else asf
    hidden = ops.grouped_gemm(aq, a_sf, kw.gate_up_q, kw.gate_up_sf, r,
                              epilogue=capi.EPI_SWIGLU, act_global=r.act_global, w_global=bank.gate_up_global,
                              amax_out=hamax, sf_layout=kw.gate_up_sf_layout)
    hq, hsf = ops.quantize_rows(hidden, r, amax_bits=hamax)
    raw = ops.grouped_gemm(hq, hsf, bank.down_q, bank.down_sf, r, epilogue=capi.EPI_PLAIN)
    rows = ops.grouped_gemm(hq, hsf, bank.down_q, kw.down_sf, r, epilogue=capi.EPI_RESCALE, act_amax=hamax,
                            w_global=bank.down_global, sf_layout=kw.down_sf_layout)
    out_stage = ops.combine(rows, r, SCALING, rows_rescaled=True)
    out_fused, top_f, gate_f = ops.moe_forward(
        xd, None, None, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q, kw.down_sf, bank.down_global,
        SCALING, router_terms=terms, router_bias=bias_d, top_k=k, gate_up_sf_layout=kw.gate_up_sf_layout,
        down_sf_layout=kw.down_sf_layout)
    torch.cuda.synchronize()
    assert capi.device_error(torch.cuda.current_device()) == 0
    host = {n: v.cpu() for n, v in dict(
        logits=logits, amax=amax, top=top, gate=gate, order=r.order, inverse=r.inverse, tokens=r.tokens,
        sorted_gate=r.sorted_gate, offsets=r.offsets, csr=r.csr, pcsr=r.pcsr, act_global=r.act_global, aq=aq,
        asf=asf, hidden=hidden, hamax=hamax, hq=hq, hsf=hsf, raw=raw, rows=rows, out_stage=out_stage,
        out_fused=out_fused, top_f=top_f, gate_f=gate_f).items()}
    state = {n: getattr(bank, n).cpu() for n in ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf",
                                                 "down_global", "_unit_alpha")}
    yield dict(name=name, shape=SHAPES[name], x=x, router=router, bias=bias, probe=probe, state=state, **host)
    del bank, kw
    torch.cuda.empty_cache()


def test_measured_fused_path_equals_stage_by_stage_ops(layer):
    assert_bytes_equal(layer["top_f"], layer["top"])
    assert_bytes_equal(layer["gate_f"], layer["gate"])
    assert_bytes_equal(layer["out_fused"], layer["out_stage"])


def test_full_size_packing_matches_oracle(layer):
    st = layer["state"]
    for ex, (gu, dn) in layer["probe"].items():
        for prefix, w in (("gate_up", gu), ("down", dn)):
            q, sf, gg = O.pack_matrix(w.t().contiguous())
            assert_bytes_equal(st[prefix + "_q"][ex], q)
            assert_bytes_equal(st[prefix + "_sf"][ex], sf)
            assert st[prefix + "_global"][ex].item() == gg.item()


def test_router_logits_and_routing(layer):
    t, c, e, k, f, _ = layer["shape"]
    ref = layer["x"].double() @ layer["router"].double().t()
    err = (layer["logits"].double() - ref).abs().max().item()
    assert err < 2e-5 * ref.abs().max().item()
    assert_bytes_equal(layer["amax"], O.row_amax(layer["x"]))
    # routing on identical logits, bit for bit against the reference's stock
    # routing ops (praxis/layers.py:2167-2173) run by torch on this GPU
    lg, bias = layer["logits"].to(DEV), layer["bias"].to(DEV)
    scores = torch.sigmoid(lg)
    ref_top = torch.topk(scores + bias, k, dim=-1).indices
    picked = scores.gather(-1, ref_top)
    ref_gate = (picked / picked.sum(-1, keepdim=True)).to(torch.bfloat16)
    assert_bytes_equal(layer["top"], ref_top.cpu())
    assert_bytes_equal(layer["gate"], ref_gate.cpu())
    # and against the CPU oracle: its sigmoid is the CPU's (not CUDA's expf),
    # so a pick may flip where two biased scores are within an ulp
    top, gate = O.route(layer["logits"], layer["bias"], k, tie_order="cuda")
    same_tok = (top == layer["top"]).all(-1)
    assert same_tok.float().mean().item() >= 1 - 1e-4
    d = (gate[same_tok].view(torch.int16).int() - layer["gate"][same_tok].view(torch.int16).int()).abs()
    assert d.max().item() <= 1 and (d != 0).float().mean().item() < 1e-3


def test_dispatch_and_activation_scales(layer):
    t, c, e, k, f, skew = layer["shape"]
    order, inverse, tokens, sorted_gate, offsets, csr = O.dispatch(layer["top"], layer["gate"], e)
    for n, want in (("order", order), ("inverse", inverse), ("tokens", tokens), ("sorted_gate", sorted_gate),
                    ("offsets", offsets), ("csr", csr)):
        assert_bytes_equal(layer[n], want)
    assert_bytes_equal(layer["pcsr"], O.pad_csr(csr))
    assert_bytes_equal(layer["act_global"], O.segment_global_scales(O.row_amax(layer["x"]), csr, tokens))
    if skew:  # the calibrated Zipf skew: the top expert is picked by about 30% of the tokens
        share = (csr[1:] - csr[:-1]).max().item() / t
        assert 0.25 < share < 0.35, share


def _live_rows(layer):
    csr, pcsr = layer["csr"], layer["pcsr"]
    rows = []
    for ex in range(csr.numel() - 1):
        live = (int(csr[ex + 1] - csr[ex]) + 127) // 128 * 128
        rows.append(torch.arange(int(pcsr[ex]), int(pcsr[ex]) + live))
    return torch.cat(rows)


def test_gather_quantize_bit_exact(layer):
    t, c, e, k, f, _ = layer["shape"]
    rp = O.padded_rows(t * k, e)
    oq, osf = O.quantize_activations(layer["x"], layer["csr"], layer["pcsr"], rp, layer["act_global"],
                                     row_indices=layer["tokens"])
    rows = _live_rows(layer)
    assert_bytes_equal(layer["aq"][rows], oq[rows])
    kb = c // 16
    assert_bytes_equal(O.unswizzle_scales(layer["asf"], rp, kb)[rows], O.unswizzle_scales(osf, rp, kb)[rows])


def test_gate_up_gemm_with_swiglu_on_sampled_rows(layer):
    """K = C (3072 at config 2): the fused rescale + SwiGLU output against the
    exact dequantised product of the same FP4 operands."""
    t, c, e, k, f, _ = layer["shape"]
    rows = sample_rows(layer["pcsr"], layer["csr"], 24, seed=5)
    experts = O.expert_of_rows(layer["pcsr"], rows)
    a = dequant_rows_sample(layer["aq"], layer["asf"], rows, c)
    st = layer["state"]
    gu = gemm_rows_oracle(a, experts, st["gate_up_q"], st["gate_up_sf"], 2 * f, c)
    want = torch.empty(rows.numel(), f, dtype=torch.bfloat16)
    for ex in experts.unique().tolist():
        sel = (experts == ex).nonzero().flatten()
        h, _ = O.rescale_swiglu_maximum(gu[sel], torch.tensor([0, sel.numel()]), layer["act_global"][ex:ex + 1],
                                        st["gate_up_global"][ex:ex + 1])
        want[sel] = h
    got = layer["hidden"][rows]
    assert ulp_mismatch(got, want) < 1e-2
    assert O.rel_l2(got, want) < 2e-3


def test_hidden_scales_and_quantize_bit_exact(layer):
    t, c, e, k, f, _ = layer["shape"]
    csr, pcsr = layer["csr"], layer["pcsr"]
    hid = layer["hidden"].float().abs()
    for ex in range(e):
        n = int(csr[ex + 1] - csr[ex])
        m = hid[int(pcsr[ex]): int(pcsr[ex]) + n].max().item() if n else 0.0
        assert layer["hamax"][ex].view(torch.float32).item() == m, ex
    hg = O.global_scale_from_amax(layer["hamax"].view(torch.float32).to(torch.bfloat16))
    rp = layer["hidden"].shape[0]
    oq, osf = O.quantize_activations(layer["hidden"], pcsr, pcsr, rp, hg)
    rows = _live_rows(layer)
    assert_bytes_equal(layer["hq"][rows], oq[rows])
    kb = f // 16
    assert_bytes_equal(O.unswizzle_scales(layer["hsf"], rp, kb)[rows], O.unswizzle_scales(osf, rp, kb)[rows])


def test_down_gemm_on_sampled_rows_and_rescale_epilogue(layer):
    """K = F (1536 at config 2): plain product against the exact dequantised
    product; the fused rescale epilogue equals bf16(plain * bf16(g_h * g_w))."""
    t, c, e, k, f, _ = layer["shape"]
    rows = sample_rows(layer["pcsr"], layer["csr"], 24, seed=6)
    experts = O.expert_of_rows(layer["pcsr"], rows)
    st = layer["state"]
    a = dequant_rows_sample(layer["hq"], layer["hsf"], rows, f)
    want = gemm_rows_oracle(a, experts, st["down_q"], st["down_sf"], c, f)
    got = layer["raw"][rows]
    assert ulp_mismatch(got, want) < 1e-2
    assert O.rel_l2(got, want) < 2e-3
    hg = O.global_scale_from_amax(layer["hamax"].view(torch.float32).to(torch.bfloat16))
    ex_all = O.expert_of_rows(layer["pcsr"], torch.arange(layer["raw"].shape[0]))
    live = _live_rows(layer)
    mult = O.bf16_round(hg[ex_all[live]] * st["down_global"][ex_all[live]]).unsqueeze(1)
    assert_bytes_equal(layer["rows"][live], (layer["raw"][live].float() * mult).to(torch.bfloat16))


def test_combine_bit_exact(layer):
    st = layer["state"]
    hg = O.global_scale_from_amax(layer["hamax"].view(torch.float32).to(torch.bfloat16))
    want = O.rescale_combine(layer["raw"], layer["inverse"], layer["top"], layer["gate"], layer["csr"], layer["pcsr"],
                             hg, st["down_global"], SCALING)
    assert_bytes_equal(layer["out_stage"], want)


def test_layer_output_vs_oracle_chain(layer):
    """The whole routed bank on the GPU's routing against the oracle's
    dequantised chain (its own quantizations, float64 GEMMs, combine)."""
    t = layer["shape"][0]
    want = O.routed_forward(layer["x"], layer["top"], layer["gate"], layer["state"], SCALING, t)
    err = O.rel_l2(layer["out_fused"], want)
    assert err <= 1e-2, err
