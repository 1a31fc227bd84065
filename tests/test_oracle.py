"""The CPU oracle against the reference's own outputs (golden fixtures) and
known-answer vectors. No GPU."""

from __future__ import annotations

import pytest
import torch
from conftest import assert_bytes_equal, golden, routing_inputs, sha

from oracle import nvfp4_moe_oracle as O


@pytest.mark.parametrize("name", ["cfg1_e8_k2", "e64_k4_bias", "e128_k8_bias", "e32_k2"])
def test_routing_matches_reference_cpu(name):
    case = golden()["routing"][name]
    x, w, bias = routing_inputs(case["seed"], case["tokens"], case["dim"], case["experts"], case["bias_scale"])
    assert sha(x) == case["x_sha"] and sha(w) == case["w_sha"] and sha(bias) == case["bias_sha"]
    logits = O.router_logits(x, w)
    assert_bytes_equal(logits, case["logits"])
    top_idx, gate = O.route(logits, bias, case["top_k"], tie_order="torch")
    assert_bytes_equal(top_idx, case["top_idx"])
    assert_bytes_equal(gate, case["gate"])
    # The CUDA tie/sum order emulation picks the same set and slots on
    # tie-free data; the gate may differ by the sum order only.
    top_c, gate_c = O.route(logits, bias, case["top_k"], tie_order="cuda")
    assert_bytes_equal(top_c, case["top_idx"])
    ulps = (gate_c.view(torch.int16).int() - case["gate"].view(torch.int16).int()).abs()
    assert ulps.max() <= 1


@pytest.mark.parametrize("name", ["cfg1_e8_k2", "e64_k4_bias", "e128_k8_bias", "e32_k2", "concentrated"])
def test_dispatch_matches_reference_cpu(name):
    d = golden()["dispatch"][name]
    if name == "concentrated":
        top_idx, gate, e = d["top_idx"], d["gate"], 16
    else:
        r = golden()["routing"][name]
        top_idx, gate, e = r["top_idx"], r["gate"], r["experts"]
    order, inverse, tokens, sorted_gate, offsets, csr = O.dispatch(top_idx, gate, e)
    assert_bytes_equal(order, d["order"])
    assert_bytes_equal(inverse, d["inverse"])
    assert_bytes_equal(tokens, d["tokens"])
    assert_bytes_equal(sorted_gate, d["sorted_gate"])
    assert_bytes_equal(offsets, d["offsets"])


@pytest.mark.parametrize("name", ["gather", "plain", "all_zero", "trailing"])
def test_global_scales_match_reference_cpu(name):
    s = golden()["scales"][name]
    amax = O.row_amax(s["x"])
    got = O.segment_global_scales(amax, s["csr"], s.get("tokens"))
    assert_bytes_equal(got, s["result"])


@pytest.mark.parametrize("k", [2, 4, 8])
def test_combine_order_matches_reference_cpu(k):
    c = golden()["combine"][f"k{k}"]
    t = c["rows"].shape[0] // k
    rows, inverse, scale = c["rows"], c["inverse"], c["scale"]
    accs = [torch.zeros(t, rows.shape[1]) for _ in range(4)]
    for s in range(k):
        r = inverse.view(t, k)[:, s]
        accs[s % 4] = accs[s % 4] + rows[r].float() * scale[inverse].view(t, k)[:, s : s + 1]
    got = ((accs[0] + accs[1]) + accs[2]) + accs[3]
    assert_bytes_equal(got, c["result"])


def test_e2m1_known_answers():
    # Ties to even on the E2M1 grid, saturation, and the sign bit.
    x = torch.tensor([0.0, -0.0, 0.25, 0.2501, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.01, 7.0, -0.1, -6.0, 1e9])
    want = torch.tensor([0, 8, 0, 1, 2, 2, 4, 4, 6, 6, 7, 7, 8, 15, 7], dtype=torch.uint8)
    assert torch.equal(O.e2m1_codes(x), want)
    assert torch.equal(O.e2m1_values(want[:12]), torch.tensor(
        [0.0, -0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0]))


def test_swizzle_layout_known_answers():
    # praxis/kernels/nvfp4.py:114-119 for a 256-row, 8-scale matrix.
    kb = 8
    assert O.sf_offset(torch.tensor(0), torch.tensor(0), kb) == 0
    assert O.sf_offset(torch.tensor(1), torch.tensor(0), kb) == 16
    assert O.sf_offset(torch.tensor(32), torch.tensor(0), kb) == 4
    assert O.sf_offset(torch.tensor(0), torch.tensor(3), kb) == 3
    assert O.sf_offset(torch.tensor(0), torch.tensor(4), kb) == 512
    assert O.sf_offset(torch.tensor(128), torch.tensor(0), kb) == 1024
    s = torch.randint(0, 255, (200, kb), dtype=torch.uint8)
    sw = O.swizzle_scales(s)
    assert sw.shape == (256, kb)
    assert torch.equal(O.unswizzle_scales(sw, 200, kb), s)


def qat_weight_reference(weight):
    """tests/test_nvfp4.py:486-507 (the QAT training rounding) with torchao's
    E2M1 conversion replaced by the oracle's: global amax*(1/2688),
    block_amax*(1/6)/global, x*((1/global)/block_scale), clamp, E2M1 RNE."""
    n, k = weight.shape
    gs = weight.abs().amax().clamp_min(1e-12).float() * torch.tensor(1.0 / 2688.0)
    blocks = weight.float().reshape(n, k // 16, 16)
    bsc = ((blocks.abs().amax(-1) * torch.tensor(1.0 / 6.0)) / gs).clamp(2.0**-6, 448.0).to(torch.float8_e4m3fn)
    rc = (1.0 / gs) / bsc.float()
    scaled = (blocks * rc.unsqueeze(-1)).clamp(-6.0, 6.0).reshape(n, k)
    return O.e2m1_codes(scaled), bsc, gs


@pytest.mark.parametrize("seed", [9, 10, 14, 28, 30, 34])
def test_packing_rounds_like_the_qat_recipe(seed):
    # tests/test_nvfp4.py:527-533: seeds that round differently under true
    # division by 2688 and 6.
    g = torch.Generator().manual_seed(seed)
    weight = (torch.randn(128, 256, generator=g) * 0.02).to(torch.bfloat16)
    q, sf, gs = O.pack_matrix(weight)
    codes = O.unpack_nibbles(q)
    scales = O.unswizzle_scales(sf, 128, 16)
    ref_codes, ref_scales, ref_g = qat_weight_reference(weight)
    assert torch.equal(codes, ref_codes)
    assert torch.equal(scales, ref_scales.view(torch.uint8))
    assert gs.item() == ref_g.item()


def test_topk_cuda_tie_order_is_a_permutation_of_the_top_set():
    g = torch.Generator().manual_seed(5)
    biased = torch.randint(0, 4, (300, 64), generator=g).float() / 4  # tie-heavy
    for k in (1, 2, 3, 4, 6, 8):
        idx = O.topk_cuda_order(biased, k)
        vals = biased.gather(1, idx)
        assert (vals[:, :-1] >= vals[:, 1:]).all()  # sorted descending
        want = biased.topk(k, dim=-1).values
        assert torch.equal(vals, want)


def test_nvfp4_chain_is_close_to_bf16_reference_layer():
    """The NVFP4 chain on the reference's bf16 layer weights stays near the
    reference's bf16 output. Sanity only: E2M1 with 16-element scales has a
    relative RMS error near 10% per quantized operand, and the chain quantizes
    four operands across two GEMMs (measured here: 0.20)."""
    lay = golden()["layer"]["bf16_t64"]
    t, c, e, k, f = lay["shape"]
    g = torch.Generator().manual_seed(lay["seed"])
    shapes = {"router.weight": (e, c), "routed.gate_up_weight": (e, c, 2 * f),
              "routed.down_weight": (e, f, c), "shared.gate_up": (c, 2 * f), "shared.down": (f, c)}
    params = {}
    for name in lay["param_order"]:
        params[name] = (torch.randn(shapes[name], generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    assert sha(x) == lay["x_sha"]
    for name, v in params.items():
        assert sha(v) == lay["state_sha"][name]
    bank = O.pack_routed_experts(params["routed.gate_up_weight"], params["routed.down_weight"])
    y, _, _ = O.moe_forward(x, params["router.weight"], torch.zeros(e), bank, k, 2.5, t,
                            shared=lay["shared"])
    assert O.rel_l2(y, lay["y"]) < 0.3


def test_softmax_exponential_is_within_two_ulp():
    """The routing kernel's softmax exponential (restated op by op here) is an
    explicit Cody-Waite + Taylor evaluation: within 2 ulp of e^x on the range
    a softmax uses, exactly 1 at 0, 0 below -87."""
    g = torch.Generator().manual_seed(0)
    x = torch.cat([-torch.rand(1_000_000, generator=g, dtype=torch.float64) * 87,
                   -torch.rand(200_000, generator=g, dtype=torch.float64) * 0.5,
                   torch.tensor([-0.0, -1e-30, -0.34657, -0.34658, -86.999, -87.0])]).float()
    got = O.exp_softmax(x).double()
    ref = torch.exp(x.double())
    ulp = torch.nextafter(ref.float(), torch.tensor(float("inf"))).double() - ref.float().double()
    assert ((got - ref).abs() / ulp).max().item() < 2.0
    assert O.exp_softmax(torch.tensor([0.0])).item() == 1.0
    assert O.exp_softmax(torch.tensor([-87.5, -1e30])).tolist() == [0.0, 0.0]
    assert O.exp_softmax(torch.tensor([float("nan")])).isnan().all()


def test_softmax_rows_sum_order_and_accuracy():
    g = torch.Generator().manual_seed(1)
    for e in (8, 32, 64, 100, 256):
        logits = torch.randn(300, e, generator=g) * 4
        got = O.softmax_rows(logits)
        ref = torch.softmax(logits.double(), -1)
        # float32 softmax: the rounding of l - max (|l - max| up to ~30 here)
        # carries into e^x, as in torch's own float32 softmax
        f32 = torch.softmax(logits, -1).double()
        err, err_torch = ((got.double() - ref).abs() / ref).max().item(), ((f32 - ref).abs() / ref).max().item()
        assert err < 4e-6 and err < 4 * err_torch + 1e-6, (e, err, err_torch)


def test_tail_norm_restatement_close_to_float64():
    """The oracle's tail (eager reduction order) against float64 arithmetic:
    the residual add is exact up to its bf16 rounding and the normalised rows
    agree within one bf16 ulp."""
    g = torch.Generator().manual_seed(5)
    for n in (512, 3072, 1020):
        x = torch.randn(40, n, generator=g).to(torch.bfloat16)
        y = torch.randn(40, n, generator=g).to(torch.bfloat16)
        w1 = 1 + torch.randn(n, generator=g) * 0.1
        xo, h = O.tail_add_norm_scale(y, x, w1, 1e-6, 0.5)
        assert torch.equal(xo, (x.float() + y.float()).to(torch.bfloat16))
        ss = O.rms_sum_of_squares(xo).double()
        ref = (xo.double() ** 2).sum(-1)
        assert ((ss - ref).abs() / ref).max().item() < 1e-5
        r = (ref / n + 1e-6).rsqrt().unsqueeze(1)
        want = ((w1.double() * (r * xo.double())).to(torch.bfloat16).double() * 0.5).to(torch.bfloat16)
        d = (h.view(torch.int16).int() - want.view(torch.int16).int()).abs()
        assert d.max().item() <= 1


def test_modulation_row_map():
    """The compact modulation row map (praxis/kernels/norm_triton.py:417-431)
    against its definition written out row by row."""
    rf, rc, nreg, pw, wd, ph = geom = (26, 8, 2, 2, 3, 2)
    got = O.mod_row_map(60, geom).tolist()
    want = []
    for row in range(60):
        b, t = divmod(row, rf)
        if t < nreg:
            want.append(b * rc + t)
            continue
        u = t - nreg
        j, u = u % pw, u // pw   # innermost index j < PW
        x, u = u % wd, u // wd   # then x < WD
        i, fy = u % ph, u // ph  # then i < PH; the rest is (f, y)
        want.append(b * rc + nreg + fy * wd + x)
    assert got == want
    assert O.mod_row_map(5).tolist() == [0, 1, 2, 3, 4]


def test_modulation_fused_and_unfused_agree():
    """bf16 operands make the modulation product exact in fp32, so the fused
    (FMA) and unfused forms give the same bits (the oracle has one form)."""
    g = torch.Generator().manual_seed(8)
    xo = torch.randn(64, 256, generator=g).to(torch.bfloat16)
    mod = (torch.randn(64, 512, generator=g) * 0.3).to(torch.bfloat16)
    sc1 = (mod[:, 256:].float() + 1).to(torch.bfloat16).float()
    prod = xo.float() * sc1
    assert torch.equal(prod.double(), xo.double() * sc1.double())
    out = O.tail_modulate(xo, mod, torch.arange(64))
    assert torch.equal(out, (prod + mod[:, :256].float()).to(torch.bfloat16))


def test_dispatch_passes_one_input_is_the_dispatch():
    """dispatch_passes with one input is the single-input dispatch, and for a
    pair its order is that of the concatenated input (a stable sort by
    expert puts pass 0's rows first inside every expert), only the segment
    offsets split per pass."""
    g = torch.Generator().manual_seed(4)
    top = torch.randint(0, 16, (300, 4), generator=g)
    gate = torch.rand(300, 4, generator=g).to(torch.bfloat16)
    o1, i1, t1, sg1, off1, csr1 = O.dispatch(top, gate, 16)
    o, i, t, sg, seg, off = O.dispatch_passes(top, gate, 16, (300,))
    assert torch.equal(o, o1) and torch.equal(i, i1) and torch.equal(t, t1) and torch.equal(sg, sg1)
    assert torch.equal(seg, csr1) and torch.equal(off, off1)
    o2, i2, t2, sg2, seg2, off2 = O.dispatch_passes(top, gate, 16, (120, 180))
    assert torch.equal(o2, o1) and torch.equal(i2, i1) and torch.equal(off2, off1)
    assert seg2.numel() == 33 and torch.equal(seg2[::2], csr1)
    pass0 = torch.bincount(top[:120].reshape(-1), minlength=16)
    assert torch.equal((seg2[1::2] - seg2[:-1:2]).long(), pass0)
