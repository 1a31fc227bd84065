"""Parity of the sm_100a kernels (called through the C ABI) with the CPU
oracle and, for routing, with torch's own CUDA ops (the reference's stock
routing code path run on the same GPU).

Tolerances: integer/byte/index outputs (top-k, dispatch permutation, FP4
codes, scale bytes, tile tables) are bit-exact. GEMM outputs are compared
with the oracle's exact (float64-accumulated) products rounded like the
tensor core (float32 -> bf16); rounding-boundary flips are allowed on at most
0.5% of elements and the relative L2 error must stay below 1e-3. The layer
output bar is relative L2 <= 1e-2 against the dequantised-fp32 chain.
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


def gen(seed):
    return torch.Generator().manual_seed(seed)


def random_routing(t, e, k, seed, concentrated=False, empty=()):
    g = gen(seed)
    logits = torch.randn(t, e, generator=g)
    for x in empty:
        logits[:, x] = -1e9
    if concentrated:
        logits[: (3 * t) // 4, 1] += 50.0
    top_idx = logits.topk(k, -1).indices.contiguous()
    gate = torch.softmax(torch.randn(t, k, generator=g), -1).to(torch.bfloat16)
    return top_idx, gate


def make_bank(e, c, f, seed):
    g = gen(seed)
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(torch.bfloat16)
    return gu, down


def replicated(sf: torch.Tensor, rows: int, kb: int, group_rows: int) -> torch.Tensor:
    """The GEMM's replicated scale layout from compact swizzled scales, as
    [groups, k-blocks, halves, copies, 512] (halves = group_rows / 128)."""
    atoms = sf.reshape(rows // 128, kb // 4, 512)  # compact: [tile][k-block][atom]
    halves = group_rows // 128
    a = atoms.reshape(rows // group_rows, halves, kb // 4, 512).permute(0, 2, 1, 3)
    return a.unsqueeze(3).expand(-1, -1, -1, 4, -1).contiguous()


def ulp_mismatch(a: torch.Tensor, b: torch.Tensor):
    a = a.detach().cpu().view(torch.int16).int()
    b = b.detach().cpu().view(torch.int16).int()
    d = (a - b).abs()
    return (d != 0).float().mean().item(), d.max().item()


# ---------------------------------------------------------------------------
# Routing
# ---------------------------------------------------------------------------
def torch_cuda_routing(logits, bias, k):
    """The reference's stock routing ops (praxis/layers.py:2167-2173) on CUDA."""
    scores = torch.sigmoid(logits)
    biased = scores + bias.to(scores.dtype)
    _, top_idx = torch.topk(biased, k, dim=-1)
    picked = scores.gather(dim=-1, index=top_idx)
    gate = picked / picked.sum(dim=-1, keepdim=True)
    return top_idx, gate.to(torch.bfloat16)


@pytest.mark.parametrize("e,k", [(8, 2), (32, 2), (64, 4), (128, 8), (64, 1), (16, 3), (256, 8)])
@pytest.mark.parametrize("ties", [False, True])
def test_routing_bit_exact_vs_torch_cuda(P, e, k, ties):
    g = gen(e * 10 + k)
    t = 777
    logits = torch.randn(t, e, generator=g)
    if ties:  # tie-heavy: few distinct values, so k-th-value ties are common
        logits = (logits * 2).round() / 2
    bias = (torch.randn(e, generator=g) * 0.05) if not ties else torch.zeros(e)
    lc, bc = logits.to(DEV), bias.to(DEV)
    top, gate = P.ops.route(lc, bc, k)
    ref_top, ref_gate = torch_cuda_routing(lc, bc, k)
    assert_bytes_equal(top, ref_top)
    assert_bytes_equal(gate, ref_gate)
    # the CPU oracle's emulation of the CUDA tie order picks the same slots
    o_top, _ = O.route(logits, bias, k, tie_order="cuda")
    assert_bytes_equal(top.cpu(), o_top)


@pytest.mark.parametrize("e,k", [(8, 2), (32, 2), (64, 4), (128, 8), (256, 8), (16, 3), (100, 6)])
@pytest.mark.parametrize("ties", [False, True])
def test_softmax_routing_bit_exact_vs_oracle(P, e, k, ties):
    """Softmax gating (BASELINE config 1's router): the kernel's explicit
    exponential and warp sum order are restated by the oracle, so top-k slots
    and bf16 gates match bit for bit, ties included."""
    g = gen(e * 7 + k)
    t = 777
    logits = torch.randn(t, e, generator=g) * 3
    if ties:
        logits = (logits * 2).round() / 2
    bias = None if ties else torch.randn(e, generator=g) * 0.01
    top, gate = P.ops.route(logits.to(DEV), None if bias is None else bias.to(DEV), k, activation="softmax")
    o_top, o_gate = O.route(logits, bias, k, activation="softmax", tie_order="cuda")
    assert_bytes_equal(top.cpu(), o_top)
    assert_bytes_equal(gate.cpu(), o_gate)
    # against torch.softmax (CUDA expf, another sum order): the picks agree
    # wherever the k-th and (k+1)-th scores are more than a few ulp apart
    ref = torch.softmax(logits.to(DEV), -1) + (0 if bias is None else bias.to(DEV))
    srt = ref.sort(-1, descending=True).values
    clear = (srt[:, k - 1] - srt[:, k]) > 1e-6 * srt[:, k - 1].abs()
    rt = ref.topk(k, -1).indices.sort(-1).values
    assert torch.equal(top.sort(-1).values[clear], rt[clear])


@pytest.mark.parametrize("splits_dtype", [torch.bfloat16, torch.float32])
def test_router_logits_and_row_amax(P, splits_dtype):
    g = gen(4)
    t, c, e = 300, 512, 64
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    w = (torch.randn(e, c, generator=g) * 0.02).to(splits_dtype)
    terms = P.ops.split_router_weight(w.to(DEV))
    logits, amax = P.ops.router_logits(x.to(DEV), terms)
    ref = x.double() @ w.double().t()
    err = (logits.cpu().double() - ref).abs().max().item()
    assert err < 2e-5 * ref.abs().max().item()
    assert_bytes_equal(amax.cpu(), O.row_amax(x))


# ---------------------------------------------------------------------------
# Dispatch
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("t,e,k,mode", [
    (256, 8, 2, "plain"), (1000, 64, 4, "plain"), (1000, 64, 4, "concentrated"),
    (33, 16, 2, "empty"), (1, 8, 2, "plain"), (4099, 128, 8, "plain"), (20000, 64, 4, "plain"),
    # 4,096 routed rows = 32 segments: the single-CTA dispatch; one token
    # more takes the three-pass launches
    (1024, 64, 4, "concentrated"), (1025, 64, 4, "plain"), (100, 256, 8, "empty"),
])
def test_dispatch_bit_exact(P, t, e, k, mode):
    top, gate = random_routing(t, e, k, seed=t + e, concentrated=mode == "concentrated",
                               empty=(0, 3, e - 1) if mode == "empty" else ())
    g = gen(9)
    x = (torch.randn(t, 128, generator=g) * 3).to(torch.bfloat16)
    amax = O.row_amax(x)
    r = P.ops.dispatch(top.to(DEV), gate.to(DEV), e, amax.to(DEV))
    order, inverse, tokens, sorted_gate, offsets, csr = O.dispatch(top, gate, e)
    assert_bytes_equal(r.order.cpu(), order)
    assert_bytes_equal(r.inverse.cpu(), inverse)
    assert_bytes_equal(r.tokens.cpu(), tokens)
    assert_bytes_equal(r.tokens32.cpu(), tokens.to(torch.int32))
    assert_bytes_equal(r.sorted_gate.cpu(), sorted_gate)
    assert_bytes_equal(r.offsets.cpu(), offsets)
    assert_bytes_equal(r.csr.cpu(), csr)
    assert_bytes_equal(r.pcsr.cpu(), O.pad_csr(csr))
    assert_bytes_equal(r.act_global.cpu(), O.segment_global_scales(amax, csr, tokens))
    counts = torch.bincount(top.flatten(), minlength=e)
    n, npairs = r.num_tiles.cpu().tolist()
    assert n == int(((counts + 127) // 128).sum())
    assert npairs == int(((counts + 255) // 256).sum())
    max_tiles = O.padded_rows(t * k, e) // 128
    tiles = r.tiles[:n].cpu()
    pairs = r.tiles[max_tiles: max_tiles + npairs].cpu()
    pcsr = O.pad_csr(csr)
    i = j2 = 0
    for ex in range(e):
        cnt = int(counts[ex])
        for j in range((cnt + 127) // 128):
            assert tiles[i].tolist() == [ex, int(pcsr[ex]) + 128 * j, min(128, cnt - 128 * j), 0]
            i += 1
        live = (cnt + 127) // 128 * 128
        for j in range((cnt + 255) // 256):
            assert pairs[j2].tolist() == [ex, int(pcsr[ex]) + 256 * j, min(256, cnt - 256 * j),
                                          min(256, live - 256 * j)]
            j2 += 1


# ---------------------------------------------------------------------------
# Quantization and packing
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("t,c,e,k", [(256, 512, 8, 2), (300, 3072, 16, 8), (50, 256, 8, 2)])
@pytest.mark.parametrize("layout", ["compact", "replicated"])
def test_quantize_gather_bit_exact(P, t, c, e, k, layout):
    top, gate = random_routing(t, e, k, seed=c)
    g = gen(c + 1)
    x = (torch.randn(t, c, generator=g) * 1.5).to(torch.bfloat16)
    x[0, :16] = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 6.0, -6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 100.0,
                              -100.0, 0.5]).to(torch.bfloat16)
    # values near the bf16 maximum (the experts' global scale follows them)
    x[1, 16:32] = torch.tensor([3e38, -3e38, 1.0, -2.0, 3.0, 0.0, -0.0, 7.0, 1e30, -1e30, 0.1, 0.2, 0.3, -0.4,
                                5.5, 6.5]).to(torch.bfloat16)
    xd = x.to(DEV)
    amax = P.ops.row_amax(xd)
    r = P.ops.dispatch(top.to(DEV), gate.to(DEV), e, amax)
    sf_layout = P.capi.SF_REPLICATED if layout == "replicated" else P.capi.SF_COMPACT
    q, sf = P.ops.quantize_gather(xd, r, r.act_global, sf_layout=sf_layout)
    _, _, tokens, _, offsets, csr = O.dispatch(top, gate, e)
    pcsr = O.pad_csr(csr)
    rp = O.padded_rows(t * k, e)
    ag = O.segment_global_scales(O.row_amax(x), csr, tokens)
    oq, osf = O.quantize_activations(x, csr, pcsr, rp, ag, row_indices=tokens)
    # compare the rows the GPU writes: routed rows + padding rows of live tiles
    counts = torch.bincount(top.flatten(), minlength=e)
    rows = []
    for ex in range(e):
        live = (int(counts[ex]) + 127) // 128 * 128
        rows.extend(range(int(pcsr[ex]), int(pcsr[ex]) + live))
    rows = torch.tensor(rows, dtype=torch.int64)
    assert_bytes_equal(q.cpu()[rows], oq[rows])
    kb = c // 16
    if layout == "replicated":
        live = torch.unique(rows // 128)
        got = sf.cpu().view(rp // 128, kb // 4, 1, 4, 512)[live]
        assert_bytes_equal(got, replicated(osf, rp, kb, 128)[live])
        return
    got = O.unswizzle_scales(sf.cpu(), rp, kb)[rows]
    want = O.unswizzle_scales(osf, rp, kb)[rows]
    assert_bytes_equal(got, want)


@pytest.mark.parametrize("rows,kdim,group", [(128, 256, 128), (768, 512, 128), (512, 3072, 256), (256, 64, 256)])
def test_replicate_scales_layout(P, rows, kdim, group):
    sf = torch.randint(0, 127, (rows, kdim // 16), dtype=torch.uint8, generator=gen(rows + kdim))
    got = P.ops.replicate_scales(sf.to(DEV), group)
    assert_bytes_equal(got.cpu().view(-1), replicated(sf, rows, kdim // 16, group).view(-1))


@pytest.mark.parametrize("e,kdim,n", [(2, 256, 128), (4, 512, 256), (3, 3072, 384)])
def test_pack_weights_bit_exact(P, e, kdim, n):
    g = gen(e * n)
    w = (torch.randn(e, kdim, n, generator=g) * 0.02).to(torch.bfloat16)
    q, sf, gl = P.ops.pack_weights(w.to(DEV))
    for ex in range(e):
        oq, osf, og = O.pack_matrix(w[ex].t().contiguous())
        assert_bytes_equal(q[ex].cpu(), oq)
        assert_bytes_equal(sf[ex].cpu(), osf)
        assert gl[ex].item() == og.item()


def test_interleave_gate_up_layout(P):
    e, c, f = 2, 256, 256
    gu, down = make_bank(e, c, f, 5)
    bank = O.pack_routed_experts(gu, down)
    q, sf = P.ops.interleave_gate_up(bank["gate_up_q"].to(DEV), bank["gate_up_sf"].to(DEV))
    for ex in range(e):
        rows = []
        for r in range(2 * f):
            blk, w = divmod(r, 64)
            h = (blk & ~3) | ((blk & 1) << 1) | ((blk & 3) >> 1)  # blocks 1, 2 of each four swapped
            rows.append(32 * h + w if w < 32 else f + 32 * h + w - 32)
        rows = torch.tensor(rows)
        assert_bytes_equal(q[ex].cpu(), bank["gate_up_q"][ex][rows])
        got = O.unswizzle_scales(sf[ex].cpu(), 2 * f, c // 16)
        want = O.unswizzle_scales(bank["gate_up_sf"][ex], 2 * f, c // 16)[rows]
        assert_bytes_equal(got, want)


# ---------------------------------------------------------------------------
# SwiGLU element arithmetic (fused GEMM epilogue == conversion-unit version)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("mult", [1.0, 0.3])
def test_swiglu_alu_arithmetic_equals_ieee_on_every_bf16_gate(P, mult):
    """The fused epilogue computes two columns at a time with paired fp32
    instructions and divides with a refined reciprocal; it must give the bits
    of the scalar IEEE-division form for every bf16 gate value in either
    column of a pair (NaN payloads aside)."""
    rows, hidden = 65536, 128
    g = gen(11)
    raw = torch.empty(rows, 2 * hidden, dtype=torch.bfloat16)
    raw[:, 2:hidden] = torch.randn(rows, hidden - 2, generator=g).to(torch.bfloat16) * 4
    patterns = torch.arange(rows, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)  # all 2^16 patterns
    raw[:, 0] = patterns
    raw[:, 1] = patterns.roll(12345)
    raw[:, hidden:] = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    raw = raw.to(DEV)
    pcsr = torch.tensor([0, rows], dtype=torch.int32, device=DEV)
    ag = torch.tensor([1.0], device=DEV)
    wg = torch.tensor([mult], device=DEV)
    h_alu, m_alu = P.ops.rescale_swiglu(raw, pcsr, ag, wg, alu=True)
    h_ref, m_ref = P.ops.rescale_swiglu(raw, pcsr, ag, wg, alu=False)
    a, b = h_alu.float(), h_ref.float()
    same = (a.view(torch.int32) == b.view(torch.int32)) | (a.isnan() & b.isnan())
    assert bool(same.all()), int((~same).sum())
    finite = raw.float().isfinite().all(dim=1)
    assert torch.equal(m_alu[finite], m_ref[finite])


def test_rescale_swiglu_close_to_oracle(P):
    rows, hidden, e = 384, 256, 3
    g = gen(12)
    raw = (torch.randn(rows, 2 * hidden, generator=g) * 50).to(torch.bfloat16)
    pcsr = torch.tensor([0, 128, 128, 384], dtype=torch.int32)
    ag = torch.rand(e, generator=g) * 1e-3
    wg = torch.rand(e, generator=g) * 1e-4
    h, m = P.ops.rescale_swiglu(raw.to(DEV), pcsr.to(DEV), ag.to(DEV), wg.to(DEV))
    want_h, want_m = O.rescale_swiglu_maximum(raw, pcsr, ag, wg)
    # Triton's ex2.approx sigmoid (GPU) vs torch.sigmoid (oracle): rare
    # one-ulp flips of the bf16 silu
    frac, _ = ulp_mismatch(h.cpu(), want_h)
    assert frac < 1e-2 and O.rel_l2(h.cpu(), want_h) < 1e-3
    assert O.rel_l2(m.cpu(), want_m) < 1e-2


# ---------------------------------------------------------------------------
# Grouped GEMM (tcgen05)
# ---------------------------------------------------------------------------
def _gemm_case(P, t, e, k, c, f, seed, mode="plain"):
    top, gate = random_routing(t, e, k, seed=seed, concentrated=mode == "concentrated",
                               empty=(1,) if mode == "empty" else ())
    g = gen(seed + 1)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    gu, down = make_bank(e, c, f, seed + 2)
    bank = O.pack_routed_experts(gu, down)
    xd = x.to(DEV)
    r = P.ops.dispatch(top.to(DEV), gate.to(DEV), e, P.ops.row_amax(xd))
    aq, asf = P.ops.quantize_gather(xd, r, r.act_global)
    return top, gate, x, bank, r, aq, asf


@pytest.fixture(params=["pair_replicated", "pair", "single"])
def gemm_variant(request, monkeypatch):
    """The CTA-pair (M=256, N=256) kernel with replicated or compact scales
    and the 1-CTA (M=128, N=128) kernel."""
    monkeypatch.setenv("PRAXIS_B200_GEMM", "single" if request.param == "single" else "pair")
    return request.param


def gemm_scales(P, variant, asf, bsf):
    """(a_sf, b_sf, sf_layout) for the variant: replicated copies of the
    compact scales for "pair_replicated"."""
    if variant != "pair_replicated":
        return asf, bsf, P.capi.SF_COMPACT
    return P.ops.replicate_scales(asf, 128), P.ops.replicate_scales(bsf, 256), P.capi.SF_REPLICATED


@pytest.mark.parametrize("t,e,k,c,f,mode", [
    (256, 8, 2, 512, 1024, "plain"), (200, 4, 2, 256, 384, "empty"), (700, 8, 2, 384, 256, "concentrated"),
    (1500, 8, 2, 256, 128, "concentrated"),
])
def test_grouped_gemm_plain_vs_dequantised_oracle(P, gemm_variant, t, e, k, c, f, mode):
    top, gate, x, bank, r, aq, asf = _gemm_case(P, t, e, k, c, f, seed=t + c, mode=mode)
    bq, bsf = bank["down_q"].to(DEV), bank["down_sf"].to(DEV)  # N = C, K = F
    # use gate_up (N = 2F, K = C) as a plain GEMM
    bq, bsf = bank["gate_up_q"].to(DEV), bank["gate_up_sf"].to(DEV)
    a_sf, b_sf, layout = gemm_scales(P, gemm_variant, asf, bsf)
    out = P.ops.grouped_gemm(aq, a_sf, bq, b_sf, r, epilogue=P.capi.EPI_PLAIN, sf_layout=layout)
    csr = r.csr.cpu()
    pcsr = r.pcsr.cpu()
    want = O.grouped_gemm(aq.cpu(), asf.cpu(), bank["gate_up_q"], bank["gate_up_sf"], pcsr, c, 2 * f)
    counts = (csr[1:] - csr[:-1]).tolist()
    rows = torch.cat([torch.arange(int(pcsr[ex]), int(pcsr[ex]) + counts[ex]) for ex in range(e)])
    got = out.cpu()[rows]
    ref = want[rows]
    frac, _ = ulp_mismatch(got, ref)
    assert frac < 5e-3
    assert O.rel_l2(got, ref) < 1e-3


def test_gemm_swiglu_and_rescale_epilogues(P, gemm_variant):
    t, e, k, c, f = 256, 8, 2, 512, 1024
    top, gate, x, bank, r, aq, asf = _gemm_case(P, t, e, k, c, f, seed=17)
    gq, gsf = P.ops.interleave_gate_up(bank["gate_up_q"].to(DEV), bank["gate_up_sf"].to(DEV))
    amax = torch.zeros(e, dtype=torch.int32, device=DEV)
    a_sf, g_sf, layout = gemm_scales(P, gemm_variant, asf, gsf)
    hidden = P.ops.grouped_gemm(aq, a_sf, gq, g_sf, r, epilogue=P.capi.EPI_SWIGLU, act_global=r.act_global,
                                w_global=bank["gate_up_global"].to(DEV), amax_out=amax, sf_layout=layout)
    pcsr, csr = r.pcsr.cpu(), r.csr.cpu()
    gu = O.grouped_gemm(aq.cpu(), asf.cpu(), bank["gate_up_q"], bank["gate_up_sf"], pcsr, c, 2 * f)
    want_h, rowmax = O.rescale_swiglu_maximum(gu, pcsr, r.act_global.cpu(), bank["gate_up_global"])
    counts = (csr[1:] - csr[:-1]).tolist()
    rows = torch.cat([torch.arange(int(pcsr[ex]), int(pcsr[ex]) + counts[ex]) for ex in range(e)])
    frac, _ = ulp_mismatch(hidden.cpu()[rows], want_h[rows])
    assert frac < 1e-2
    assert O.rel_l2(hidden.cpu()[rows], want_h[rows]) < 2e-3
    # per-expert max |hidden| == max over the expert's rows of the GPU hidden
    gh = hidden.cpu().float().abs()
    for ex in range(e):
        seg = gh[int(pcsr[ex]): int(pcsr[ex]) + counts[ex]]
        m = seg.max().item() if counts[ex] else 0.0
        assert amax[ex].view(torch.float32).item() == m
    # rescale epilogue on the down projection
    hq, hsf = P.ops.quantize_rows(hidden, r, amax_bits=amax)
    h_sf, d_sf, layout = gemm_scales(P, gemm_variant, hsf, bank["down_sf"].to(DEV))
    if layout == P.capi.SF_REPLICATED:
        # the row quantizer's own replicated output must match
        _, h_sf2 = P.ops.quantize_rows(hidden, r, amax_bits=amax, sf_layout=layout)
        live = torch.unique(torch.cat([torch.arange(int(pcsr[ex]), int(pcsr[ex]) + counts[ex]) for ex in range(e)])
                            // 128)
        rp = hidden.shape[0]
        assert_bytes_equal(h_sf2.cpu().view(rp // 128, -1)[live], h_sf.cpu().view(rp // 128, -1)[live])
    rows_out = P.ops.grouped_gemm(hq, h_sf, bank["down_q"].to(DEV), d_sf, r, epilogue=P.capi.EPI_RESCALE,
                                  act_amax=amax, w_global=bank["down_global"].to(DEV), sf_layout=layout)
    hg = O.global_scale_from_amax(amax.cpu().view(torch.float32).to(torch.bfloat16))
    raw = O.grouped_gemm(hq.cpu(), hsf.cpu(), bank["down_q"], bank["down_sf"], pcsr, f, c)
    expert = O.expert_of_rows(pcsr, torch.arange(raw.shape[0]))
    mult = O.bf16_round(hg[expert] * bank["down_global"][expert]).unsqueeze(1)
    want_rows = (raw.float() * mult).to(torch.bfloat16)
    frac, _ = ulp_mismatch(rows_out.cpu()[rows], want_rows[rows])
    assert frac < 5e-3


# ---------------------------------------------------------------------------
# The layer
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("t,c,e,k,f,chunk,shared", [
    (256, 512, 8, 2, 1024, 256, True),      # config-1 shape
    (256, 512, 8, 2, 1024, 100, False),     # several dispatch chunks
    (64, 256, 32, 2, 512, 64, True),
    (130, 256, 64, 4, 256, 130, False),
    (1, 256, 8, 1, 128, 1, True),
    (96, 384, 8, 2, 256, 96, False),        # C % 256 != 0: compact weight scales
])
def test_bank_forward_matches_oracle(P, t, c, e, k, f, chunk, shared):
    top, gate = random_routing(t, e, k, seed=t * k + e)
    g = gen(t + c)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    sh = (torch.randn(t, c, generator=g) * 0.1).to(torch.bfloat16) if shared else None
    gu, down = make_bank(e, c, f, seed=e + f)
    obank = O.pack_routed_experts(gu, down)
    bank = P.B200NVFP4RoutedExperts.from_packed({kk: v.clone() for kk, v in obank.items()}).to(DEV)
    if shared:
        got = bank.routed_forward_with_shared(x.to(DEV), top.to(DEV), gate.to(DEV), scaling=2.5, chunk_size=chunk,
                                              shared=sh.to(DEV))
    else:
        got = bank.routed_forward(x.to(DEV), top.to(DEV), gate.to(DEV), scaling=2.5, chunk_size=chunk)
    want = O.routed_forward(x, top, gate, obank, 2.5, chunk, shared=sh)
    err = O.rel_l2(got.cpu(), want)
    assert err <= 1e-2, err
    assert P.capi.device_error(torch.cuda.current_device()) == 0


def test_module_with_router_matches_oracle(P):
    t, c, e, k, f = 256, 512, 8, 2, 1024
    g = gen(31)
    gu, down = make_bank(e, c, f, seed=32)
    mod = P.B200MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=t, shared_expert=False).to(DEV)
    with torch.no_grad():
        mod.router.weight.copy_((torch.randn(e, c, generator=g) * 0.02).to(DEV))
    mod.set_routed_weights(gu.to(DEV), down.to(DEV))
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    y = mod(x.to(DEV))
    obank = O.pack_routed_experts(gu, down)
    logits = x.float() @ mod.router.weight.detach().cpu().float().t()
    top, gate = O.route(logits, torch.zeros(e), k)
    want = O.routed_forward(x, top, gate, obank, 2.5, t)
    assert O.rel_l2(y.cpu(), want) <= 1e-2


def test_cuda_graph_replay_matches_eager(P):
    t, c, e, k, f = 512, 1024, 32, 2, 2048
    gu, down = make_bank(e, c, f, seed=41)
    bank = P.pack_routed_experts(gu.to(DEV), down.to(DEV), keep_on_device=True)
    bank.prepare()
    g = gen(42)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16).to(DEV)
    top, gate = random_routing(t, e, k, seed=43)
    top, gate = top.to(DEV), gate.to(DEV)
    eager = bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t)
    graph.replay()
    torch.cuda.synchronize()
    assert_bytes_equal(out, eager)
    # new routing and activations in the same buffers
    x2 = torch.randn(t, c, generator=g).to(torch.bfloat16)
    top2, gate2 = random_routing(t, e, k, seed=44, concentrated=True)
    x.copy_(x2.to(DEV))
    top.copy_(top2.to(DEV))
    gate.copy_(gate2.to(DEV))
    graph.replay()
    torch.cuda.synchronize()
    assert_bytes_equal(out, bank.routed_forward(x, top, gate, scaling=2.5, chunk_size=t))
    del graph


def test_host_pipeline_matches_direct_calls(P):
    t, c, e, k, f = 256, 512, 8, 2, 1024
    gu, down = make_bank(e, c, f, seed=51)
    bank = P.pack_routed_experts(gu.to(DEV), down.to(DEV), keep_on_device=True)
    bank.prepare()
    kw = bank.kernel_weights()
    top, gate = random_routing(t, e, k, seed=52)
    top, gate = top.to(DEV), gate.to(DEV)

    def layer(xin, yout):
        P.ops.moe_forward(xin, top, gate, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q,
                          kw.down_sf, bank.down_global, 2.5, out=yout, gate_up_sf_layout=kw.gate_up_sf_layout,
                          down_sf_layout=kw.down_sf_layout)

    g = gen(53)
    host_in = [torch.randn(t, c, generator=g).to(torch.bfloat16).pin_memory() for _ in range(5)]
    host_out = [torch.empty(t, c, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    pipe = P.pipeline.HostPipeline(layer, (t, c), (t, c), torch.bfloat16, torch.device(DEV))
    pipe.run(host_in, host_out)
    torch.cuda.synchronize()
    for hi, ho in zip(host_in, host_out):
        want = torch.empty(t, c, dtype=torch.bfloat16, device=DEV)
        layer(hi.to(DEV), want)
        assert torch.equal(ho.view(torch.int16), want.cpu().view(torch.int16))


def _midpoint_globals(bs: float, experts: int, seed: int) -> torch.Tensor:
    """Per-expert global scales that put bs / g within a few ulps of an e4m3
    rounding midpoint (each expert its own midpoint and offset)."""
    vals = O.e4m3_values(torch.arange(0x08, 0x7F, dtype=torch.uint8)).double()
    mids = (vals[:-1] + vals[1:]) / 2
    g = torch.Generator().manual_seed(seed)
    pick = mids[torch.randint(0, mids.numel(), (experts,), generator=g)]
    g0 = (bs / pick).float()
    step = torch.randint(-6, 7, (experts,), generator=g, dtype=torch.int32)
    return (g0.view(torch.int32) + step).view(torch.float32)


@pytest.mark.parametrize("t,c,e,k", [(512, 1024, 16, 4), (200, 3072, 64, 8)])
def test_quantize_scales_at_e4m3_midpoints(P, t, c, e, k):
    """Gather-quantize and row-quantize with global scales that put the block
    scales next to e4m3 rounding midpoints: the kernels' division-free scale
    path must take the division there (codes and scale bytes bit-exact)."""
    top, gate = random_routing(t, e, k, seed=t + c)
    g = gen(c + 7)
    x = (torch.randn(t, c, generator=g) * 0.3).to(torch.bfloat16)
    x[:, ::16] = 1.5  # every 16-block's max |v| = 1.5
    bs = float(torch.tensor(1.5, dtype=torch.float32) * torch.tensor(1.0 / 6.0, dtype=torch.float32))
    glob = _midpoint_globals(bs, e, seed=c)
    xd = x.to(DEV)
    r = P.ops.dispatch(top.to(DEV), gate.to(DEV), e)
    q, sf = P.ops.quantize_gather(xd, r, glob.to(DEV))
    _, _, tokens, _, _, csr = O.dispatch(top, gate, e)
    pcsr = O.pad_csr(csr)
    rp = O.padded_rows(t * k, e)
    oq, osf = O.quantize_activations(x, csr, pcsr, rp, glob, row_indices=tokens)
    counts = torch.bincount(top.flatten(), minlength=e)
    rows = torch.cat([torch.arange(int(pcsr[ex]), int(pcsr[ex]) + int(counts[ex])) for ex in range(e)])
    assert_bytes_equal(q.cpu()[rows], oq[rows])
    kb = c // 16
    assert_bytes_equal(O.unswizzle_scales(sf.cpu(), rp, kb)[rows], O.unswizzle_scales(osf, rp, kb)[rows])
    # the row quantizer on the gathered rows (one global per expert group)
    gathered = torch.zeros(rp, c, dtype=torch.bfloat16)
    gathered[rows] = x[tokens]
    hq, hsf = P.ops.quantize_rows(gathered.to(DEV), r, glob.to(DEV))
    assert_bytes_equal(hq.cpu()[rows], oq[rows])
    assert_bytes_equal(O.unswizzle_scales(hsf.cpu(), rp, kb)[rows], O.unswizzle_scales(osf, rp, kb)[rows])
