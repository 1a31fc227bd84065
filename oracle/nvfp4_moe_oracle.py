"""CPU restatement of Praxis-1's routed-expert NVFP4 MoE hot path.

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA
path: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it. The product path never calls it and has no CPU
fallback.

Every function restates one step of the reference (runwayml/praxis-1-oss) and
cites the file:line it follows. All arithmetic is torch on the CPU, one
IEEE-rounded op at a time, so nothing is fused or contracted:

* routing            praxis/layers.py:1647-1653 (== :2167-2173)
* dispatch           praxis/layers.py:1330-1346, praxis/quantization/nvfp4.py:705-708
* CSR padding        praxis/kernels/nvfp4.py:37-41
* global scales      praxis/kernels/nvfp4_moe.py:15-57, praxis/kernels/nvfp4.py:154-194
* NVFP4 quantize     praxis/kernels/nvfp4.py:44-124
* weight packing     praxis/quantization/nvfp4.py:67-146
* grouped GEMM       praxis/kernels/nvfp4.py:355-419 (FlashInfer, alpha = 1): restated
                     from the operands' definition: exact dequantised products,
                     float64 accumulation, then float32 -> bfloat16
* rescale + SwiGLU   praxis/kernels/nvfp4_moe.py:102-133
* rescale + combine  praxis/kernels/nvfp4_moe.py:206-269
* chunk loop         praxis/quantization/nvfp4.py:616-747

Parity pins: ``tests/golden/make_golden.py`` runs the reference's own CPU
code (routing, dispatch, global scales, combine order) and the fixtures it
writes are checked against this module by ``tests/test_oracle.py``. The E2M1
rounding and the swizzled scale layout are pinned by known-answer vectors
taken from the reference's tests; the packing recipe of torchao (absent from
this image, pinned version torchao==0.17.0 in the reference's pyproject) is
restated from its published definition (round-to-nearest-even onto the E2M1
grid, two codes per byte with the even element in the low nibble).
"""

from __future__ import annotations

import math

import torch

# Magnitudes of the eight E2M1 codes 0..7 (sign in bit 3).
FP4_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
ALIGN = 128  # SM100 per-expert row alignment, praxis/quantization/nvfp4.py:671
_F32 = torch.float32
_BF16 = torch.bfloat16


def f32(value: float) -> torch.Tensor:
    """A Python float rounded to float32, as Triton and torch fold constants."""
    return torch.tensor(value, dtype=_F32)


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    """float32 -> bfloat16 (RNE) -> float32."""
    return x.to(_BF16).to(_F32)


# ---------------------------------------------------------------------------
# Element formats
# ---------------------------------------------------------------------------
def e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    """float32 -> E2M1 code (uint8 0..15), round to nearest even, saturating.

    Restates ``cvt.rn.satfinite.e2m1x2.f32`` (praxis/kernels/nvfp4.py:92-103)
    and torchao's ``f32_to_f4_unpacked`` (praxis/quantization/nvfp4.py:96):
    the decision points are the midpoints of the grid 0, .5, 1, 1.5, 2, 3, 4, 6;
    a tie goes to the code with an even mantissa bit (0.25 -> 0, 0.75 -> 1,
    1.25 -> 1, 1.75 -> 2, 2.5 -> 2, 3.5 -> 4, 5 -> 4). The sign bit of the
    input (including -0.0 and negatives that round to zero) becomes bit 3.
    """
    x = x.to(_F32)
    a = x.abs()
    code = (
        (a > 0.25).to(torch.uint8)
        + (a >= 0.75).to(torch.uint8)
        + (a > 1.25).to(torch.uint8)
        + (a >= 1.75).to(torch.uint8)
        + (a > 2.5).to(torch.uint8)
        + (a >= 3.5).to(torch.uint8)
        + (a > 5.0).to(torch.uint8)
    )
    sign = (x.view(torch.int32) < 0).to(torch.uint8) << 3
    return code | sign


def e2m1_values(codes: torch.Tensor) -> torch.Tensor:
    """E2M1 codes -> float32 values (exact)."""
    mag = torch.tensor(FP4_MAGNITUDES, dtype=_F32)[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """(..., K) codes -> (..., K/2) bytes; the even element is the low nibble
    (``pack_uint4``, tests/test_nvfp4.py:513)."""
    c = codes.reshape(*codes.shape[:-1], codes.shape[-1] // 2, 2)
    return (c[..., 0] | (c[..., 1] << 4)).to(torch.uint8)


def unpack_nibbles(q: torch.Tensor) -> torch.Tensor:
    return torch.stack([q & 0xF, q >> 4], -1).reshape(*q.shape[:-1], q.shape[-1] * 2)


def e4m3_bytes(x: torch.Tensor) -> torch.Tensor:
    """float32 -> float8_e4m3fn bytes (RNE), as ``.to(tl.float8e4nv)``."""
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_values(b: torch.Tensor) -> torch.Tensor:
    return b.view(torch.float8_e4m3fn).to(_F32)


# ---------------------------------------------------------------------------
# Swizzled scale-factor layout (128 x 4 atoms of 512 bytes)
# ---------------------------------------------------------------------------
def sf_offset(row: torch.Tensor, col: torch.Tensor, kb: int) -> torch.Tensor:
    """Byte offset of scale (row, col) for ``kb`` scales per row.

    praxis/kernels/nvfp4.py:114-119: ((l//128)*(K/64) + j//4)*512
    + (l%32)*16 + ((l%128)//32)*4 + j%4.
    """
    return (
        ((row // 128) * (kb // 4) + col // 4) * 512
        + (row % 32) * 16
        + ((row % 128) // 32) * 4
        + col % 4
    )


def swizzle_scales(scales: torch.Tensor) -> torch.Tensor:
    """(n, kb) uint8 -> (ceil(n/128)*128, kb) uint8 in the blocked layout
    (torchao ``to_blocked`` as used at praxis/quantization/nvfp4.py:97-99)."""
    n, kb = scales.shape
    npad = (n + 127) // 128 * 128
    out = torch.zeros(npad * kb, dtype=torch.uint8)
    rows = torch.arange(n).unsqueeze(1).expand(n, kb)
    cols = torch.arange(kb).unsqueeze(0).expand(n, kb)
    out[sf_offset(rows, cols, kb).reshape(-1)] = scales.reshape(-1)
    return out.reshape(npad, kb)


def unswizzle_scales(sf: torch.Tensor, n: int, kb: int) -> torch.Tensor:
    flat = sf.reshape(-1)
    rows = torch.arange(n).unsqueeze(1).expand(n, kb)
    cols = torch.arange(kb).unsqueeze(0).expand(n, kb)
    return flat[sf_offset(rows, cols, kb)]


# ---------------------------------------------------------------------------
# Quantization recipe
# ---------------------------------------------------------------------------
def global_scale_from_amax(amax_bf16: torch.Tensor) -> torch.Tensor:
    """f32(bf16(max(amax, 1e-12))) * f32(1/2688).

    praxis/kernels/nvfp4_moe.py:55-57 (activations) and
    praxis/quantization/nvfp4.py:86 (weights: clamp_min on the bf16 amax).
    """
    clamped = torch.clamp_min(amax_bf16.to(_F32), 1e-12).to(_BF16).to(_F32)
    return clamped * f32(1.0 / 2688.0)


def quantize_blocks(values: torch.Tensor, g: torch.Tensor):
    """Rows of float32 values, one global scale per row -> (codes, scale bytes).

    praxis/kernels/nvfp4.py:76-103 == praxis/quantization/nvfp4.py:88-96:
    bs = max|v| * f32(1/6); sf = e4m3(clamp(bs / g, 2^-6, 448));
    rc = (1 / g) / sf; n = clamp(v * rc, -6, 6); NaN -> signed zero; e2m1 RNE.
    """
    n, k = values.shape
    blocks = values.to(_F32).reshape(n, k // 16, 16)
    g = g.to(_F32).reshape(n, 1)
    bs = blocks.abs().amax(-1) * f32(1.0 / 6.0)
    sfv = torch.clamp(bs / g, 2.0**-6, 448.0)
    sf = e4m3_bytes(sfv)
    rc = (f32(1.0) / g) / e4m3_values(sf)
    norm = torch.clamp(blocks * rc.unsqueeze(-1), -6.0, 6.0)
    signed_zero = (norm.view(torch.int32) & -0x80000000).view(_F32)
    norm = torch.where(norm != norm, signed_zero, norm)
    return e2m1_codes(norm.reshape(n, k)), sf


def pack_matrix(weight: torch.Tensor):
    """One bf16 [out, in] matrix -> (q, swizzled sf, global).

    praxis/quantization/nvfp4.py:67-101 (``_pack_matrix_cpu``).
    """
    n, k = weight.shape
    g = global_scale_from_amax(weight.abs().amax().to(_BF16))
    codes, sf = quantize_blocks(weight.to(_F32), g.expand(n))
    return pack_nibbles(codes), swizzle_scales(sf), g.reshape(())


def pack_routed_experts(gate_up_weight: torch.Tensor, down_weight: torch.Tensor):
    """Expert-first bf16 banks [E,C,2H] / [E,H,C] -> the packed buffers.

    praxis/quantization/nvfp4.py:104-146: each expert matrix is transposed
    (row = output feature) before packing; gate rows 0..H-1, up rows H..2H-1.
    """
    e, c, h2 = gate_up_weight.shape
    h = h2 // 2
    state = {}
    for name, weight, n, k in (
        ("gate_up", gate_up_weight, 2 * h, c),
        ("down", down_weight, c, h),
    ):
        qs, sfs, gs = [], [], []
        for expert in range(e):
            q, sf, g = pack_matrix(weight[expert].t().contiguous())
            qs.append(q)
            sfs.append(sf)
            gs.append(g)
        state[name + "_q"] = torch.stack(qs)
        state[name + "_sf"] = torch.stack(sfs)
        state[name + "_global"] = torch.stack(gs).to(_F32)
    state["_unit_alpha"] = torch.ones(e, dtype=_F32)
    return state


def dequant_matrix(q: torch.Tensor, sf: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Packed rows -> float32 values without the global scale (exact)."""
    codes = unpack_nibbles(q.reshape(n, k // 2))
    scales = e4m3_values(unswizzle_scales(sf, n, k // 16))
    return e2m1_values(codes) * scales.repeat_interleave(16, -1)


# ---------------------------------------------------------------------------
# Routing
# ---------------------------------------------------------------------------
def _ordered_key(v: torch.Tensor) -> torch.Tensor:
    """float32 -> int64 whose integer order is the float order (-0 < +0)."""
    b = v.view(torch.int32).to(torch.int64)
    return torch.where(b >= 0, b, b ^ 0x7FFFFFFF)


def bitonic32_slots(k: int):
    """Where ATen's 32-wide bitonic key/value sort (16 threads, 2 items each,
    invalid entries sort last, comparator ``a > b``; SortUtils.cuh as
    described at praxis/kernels/router_fused.py:21-26) moves ``k`` valid
    entries. Returns a list of compare-exchange steps (ia, ib, dir) on the
    valid registers and the register that ends in each output slot."""
    where = {i: i for i in range(k)}  # position -> register
    steps = []

    def exchange(pa, pb, direction):
        va, vb = pa in where, pb in where
        if va and vb:
            steps.append((where[pa], where[pb], direction))
        elif va and direction:  # B invalid: swap flag is true
            where[pb] = where.pop(pa)
        elif vb and not direction:  # A invalid: swap flag is false
            where[pa] = where.pop(pb)

    size = 2
    while size < 32:
        stride = size // 2
        while stride > 0:
            for tid in range(16):
                pos = 2 * tid - (tid & (stride - 1))
                exchange(pos, pos + stride, (tid & (size // 2)) != 0)
            stride //= 2
        size *= 2
    stride = 16
    while stride > 0:
        for tid in range(16):
            pos = 2 * tid - (tid & (stride - 1))
            exchange(pos, pos + stride, False)
        stride //= 2
    return steps, [where[i] for i in range(k)]


def topk_cuda_order(biased: torch.Tensor, k: int) -> torch.Tensor:
    """``torch.topk(biased, k, -1).indices`` in the slot order of ATen's CUDA
    kernel, ties included (praxis/kernels/router_fused.py:21-26, :125-155):
    the set is the k largest (ties at the k-th value: lowest index wins);
    the elements above the k-th value in index order, then those equal to it
    in index order, go through the 32-wide bitonic sort."""
    t, e = biased.shape
    idx = torch.arange(e, dtype=torch.int64)
    keys = (_ordered_key(biased) << 32) | (e - 1 - idx)
    top = keys.topk(k, dim=-1).values
    sel = (e - 1) - (top & 0xFFFFFFFF)
    hi = top >> 32
    tie = hi == hi[:, k - 1 : k]
    gather = sel.gather(1, (tie.to(torch.int64) * e + sel).argsort(dim=-1))
    vals = biased.gather(1, gather)
    steps, out = bitonic32_slots(k)
    v = [vals[:, i].clone() for i in range(k)]
    r = [gather[:, i].clone() for i in range(k)]
    for a, b, direction in steps:
        gt = v[a] > v[b]
        sw = gt if direction else ~gt
        v[a], v[b] = torch.where(sw, v[b], v[a]), torch.where(sw, v[a], v[b])
        r[a], r[b] = torch.where(sw, r[b], r[a]), torch.where(sw, r[a], r[b])
    return torch.stack([r[out[i]] for i in range(k)], dim=1)


def gate_sum(picked: torch.Tensor) -> torch.Tensor:
    """``picked.sum(-1)`` in ATen's CUDA reduction order for a narrow row:
    w = last_pow2(k) lanes, lane t adds elements t, t+w, ... in order, then a
    shuffle-down tree with offsets w/2 .. 1. For k = 8 this is
    ((p0+p4)+(p2+p6))+((p1+p5)+(p3+p7)) (praxis/kernels/router_fused.py:158-162)."""
    k = picked.shape[1]
    w = 1 << (k.bit_length() - 1)
    lanes = []
    for t in range(w):
        acc = picked[:, t]
        for j in range(t + w, k, w):
            acc = acc + picked[:, j]
        lanes.append(acc)
    off = w // 2
    while off > 0:
        lanes = [lanes[i] + lanes[i + off] if i + off < w else lanes[i] for i in range(w)]
        off //= 2
    return lanes[0]


def exp_softmax(x: torch.Tensor) -> torch.Tensor:
    """e^x (x <= 0) of the softmax router, defined op by op so that the CUDA
    kernel and this restatement give the same bits: Cody and Waite's range
    reduction (W. J. Cody, W. Waite, "Software Manual for the Elementary
    Functions", 1980), x = n ln2 + r with n = rint(x log2 e) and ln2 = C1 + C2,
    then e^r by its degree-7 Taylor polynomial in Horner form, then 2^n; each
    step one float32 multiply or add rounded to nearest. x < -87 -> 0."""
    x = x.to(_F32)
    c = lambda h: torch.tensor(float.fromhex(h), dtype=_F32)  # noqa: E731
    n = torch.round(x * c("0x1.715476p+0"))  # half to even, as rint
    r = x + (-n) * c("0x1.63p-1")
    r = r + (-n) * c("-0x1.bd0106p-13")
    q = c("0x1.a01a02p-13").expand_as(r)
    for h in ("0x1.6c16c2p-10", "0x1.111112p-7", "0x1.555556p-5", "0x1.555556p-3", "0x1.0p-1", "0x1.0p+0",
              "0x1.0p+0"):
        q = q * r + c(h)
    scale = ((n.clamp(-126, 127).to(torch.int32) + 127) << 23).view(_F32)
    out = q * scale
    out = torch.where(x < -87.0, torch.zeros_like(out), out)
    return torch.where(x != x, x, out)


def softmax_rows(logits: torch.Tensor) -> torch.Tensor:
    """Softmax over the experts in the routing kernel's order (one warp per
    token, expert e on lane e % 32): p = exp_softmax(l - max); lane l sums
    its experts l, l + 32, ... in that order, a butterfly over lane distances
    16, 8, 4, 2, 1 adds the 32 lane sums; score = p / sum (IEEE division)."""
    logits = logits.to(_F32)
    t, e = logits.shape
    p = exp_softmax(logits - logits.amax(-1, keepdim=True))
    lanes = torch.zeros(t, 32, dtype=_F32)
    for i in range((e + 31) // 32):
        chunk = p[:, 32 * i: 32 * (i + 1)]
        lanes[:, : chunk.shape[1]] = lanes[:, : chunk.shape[1]] + chunk
    lane = torch.arange(32)
    for o in (16, 8, 4, 2, 1):
        lanes = lanes + lanes[:, lane ^ o]
    return p / lanes[:, :1]


def route(
    logits: torch.Tensor,
    bias: torch.Tensor | None,
    k: int,
    activation: str = "sigmoid",
    tie_order: str = "cuda",
):
    """Stock routing: praxis/layers.py:1647-1653 (sigmoid, the reference's
    only router). ``activation="softmax"`` is this build's extension
    (BASELINE config 1's softmax router): ``softmax_rows`` (an explicit
    exponential and sum order, see there), then the same bias / top-k /
    renormalisation.

    ``tie_order="cuda"`` emulates torch.topk's CUDA slot order and ATen's CUDA
    sum order; ``"torch"`` calls the torch ops of the reference on the CPU.
    """
    logits = logits.to(_F32)
    if activation == "sigmoid":
        scores = torch.sigmoid(logits)
    elif activation == "softmax":
        scores = softmax_rows(logits) if tie_order == "cuda" else torch.softmax(logits, dim=-1)
    else:
        raise ValueError(activation)
    biased = scores if bias is None else scores + bias.to(_F32)
    if tie_order == "torch":
        top_idx = torch.topk(biased, k, dim=-1).indices
        picked = scores.gather(-1, top_idx)
        total = picked.sum(dim=-1, keepdim=True)
    else:
        top_idx = topk_cuda_order(biased, k)
        picked = scores.gather(-1, top_idx)
        total = gate_sum(picked).unsqueeze(-1)
    gate = (picked / total).to(_BF16)
    return top_idx, gate


def router_logits(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """praxis/layers.py:1104-1122: float32 x @ float32 W^T (K order of the
    CPU BLAS; the GPU's order differs within float32 rounding)."""
    return torch.nn.functional.linear(x.to(_F32), weight.to(_F32))


# ---------------------------------------------------------------------------
# Dispatch
# ---------------------------------------------------------------------------
def dispatch(top_idx: torch.Tensor, gate: torch.Tensor, num_experts: int):
    """praxis/layers.py:1330-1346 + praxis/quantization/nvfp4.py:705-708.

    Returns order, inverse, tokens, sorted_gate (int64/int64/int64/bf16),
    offsets (int32 end offsets) and csr (int32, E+1)."""
    t, k = top_idx.shape
    experts = top_idx.reshape(-1)
    _, order = experts.sort(stable=True)
    tokens = torch.arange(t).repeat_interleave(k)[order]
    counts = torch.bincount(experts, minlength=num_experts)
    offsets = counts.cumsum(0).to(torch.int32)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel())
    csr = torch.nn.functional.pad(offsets, (1, 0))
    return order, inverse, tokens, gate.reshape(-1)[order], offsets, csr


def dispatch_passes(top_idx: torch.Tensor, gate: torch.Tensor, num_experts: int, rows):
    """The dispatch metadata of lockstep inputs ``rows = (T0, T1)`` (or one
    input, ``(T,)``): ``dispatch_ref`` of praxis/kernels/router_fused.py:
    820-852. Key of slot (t, s) = top_idx[t, s] * P + pass(t); a stable sort
    of the keys gives order and inverse; seg_csr [P*E + 1] counts per key;
    offsets = seg_csr[P::P] (per-expert end offsets); tokens = order // k.
    Returns order, inverse, tokens, sorted_gate, seg_csr, offsets."""
    rows = tuple(int(r) for r in rows)
    npass = len(rows)
    t, k = top_idx.shape
    pas = torch.zeros(t, dtype=torch.int64)
    if npass == 2:
        pas[rows[0]:] = 1
    keys = (top_idx * npass + pas[:, None]).reshape(-1)
    _, order = keys.sort(stable=True)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel())
    counts = torch.bincount(keys, minlength=npass * num_experts)
    seg_csr = torch.nn.functional.pad(counts.cumsum(0).to(torch.int32), (1, 0))
    return order, inverse, order // k, gate.reshape(-1)[order], seg_csr, seg_csr[npass::npass].contiguous()


def pad_csr(csr: torch.Tensor, align: int = ALIGN) -> torch.Tensor:
    """praxis/kernels/nvfp4.py:37-41: ((csr[i] + (align-1)*i) // align) * align."""
    i = torch.arange(csr.numel(), dtype=torch.int64)
    return ((csr.to(torch.int64) + (align - 1) * i) // align * align).to(torch.int32)


def padded_rows(rows: int, experts: int, align: int = ALIGN) -> int:
    """praxis/kernels/nvfp4.py:213."""
    return (rows + (align - 1) * experts) // align * align


def expert_of_rows(csr: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """``_expert`` (praxis/kernels/nvfp4.py:24-34): the expert whose CSR
    segment holds the row; rows past the end belong to the last expert."""
    e = csr.numel() - 1
    return torch.bucketize(rows.to(torch.int64), csr[1:].to(torch.int64), right=True).clamp_max(e - 1)


# ---------------------------------------------------------------------------
# Global scales
# ---------------------------------------------------------------------------
def row_amax(x: torch.Tensor) -> torch.Tensor:
    """praxis/kernels/nvfp4_moe.py:15-21: bf16(max |x[row]|)."""
    return x.to(_F32).abs().amax(-1).to(_BF16)


def segment_global_scales(row_maximum: torch.Tensor, csr: torch.Tensor, rows_map=None):
    """praxis/kernels/nvfp4_moe.py:24-57: per-expert max of bf16 row maxima
    (rows past the last CSR end count for the last expert), then the QAT
    global-scale formula."""
    e = csr.numel() - 1
    values = row_maximum if rows_map is None else row_maximum[rows_map]
    nrows = values.numel()
    expert = expert_of_rows(csr, torch.arange(nrows))
    group = torch.zeros(e, dtype=_F32)
    group.scatter_reduce_(0, expert, values.to(_F32), "amax")
    return global_scale_from_amax(group.to(_BF16))


# ---------------------------------------------------------------------------
# Activation quantization (padded, expert-grouped rows)
# ---------------------------------------------------------------------------
def quantize_activations(x, csr, pcsr, nrows_padded, g, row_indices=None, pad_fill_all=False):
    """praxis/kernels/nvfp4.py:44-124 and :197-254 (alignment 128,
    ``grouped_scales=False``): row r of expert e (gathered through
    ``row_indices`` when given) goes to padded row pcsr[e] + r - csr[e].
    Rows not written stay zero, as the reference allocates zeros
    (:227-231). With ``row_indices`` None every padded row is a source row
    (the hidden quantize, where csr == pcsr)."""
    k = x.shape[1]
    m = x.shape[0] if row_indices is None else row_indices.numel()
    q = torch.zeros(nrows_padded, k // 2, dtype=torch.uint8)
    sf = torch.zeros(nrows_padded * (k // 16), dtype=torch.uint8)
    if m == 0:
        return q, sf.reshape(nrows_padded, k // 16)
    rows = torch.arange(m)
    expert = expert_of_rows(csr, rows)
    dest = pcsr.to(torch.int64)[expert] + rows - csr.to(torch.int64)[expert]
    src = x if row_indices is None else x[row_indices]
    codes, scales = quantize_blocks(src.to(_F32), g[expert])
    q[dest] = pack_nibbles(codes)
    kb = k // 16
    cols = torch.arange(kb).unsqueeze(0).expand(m, kb)
    sf[sf_offset(dest.unsqueeze(1).expand(m, kb), cols, kb).reshape(-1)] = scales.reshape(-1)
    return q, sf.reshape(nrows_padded, k // 16)


def dequant_rows(q: torch.Tensor, sf: torch.Tensor, k: int) -> torch.Tensor:
    n = q.shape[0]
    return dequant_matrix(q, sf, n, k)


# ---------------------------------------------------------------------------
# Grouped GEMM with dequantised operands
# ---------------------------------------------------------------------------
def grouped_gemm(a_q, a_sf, b_q, b_sf, pcsr, k: int, n: int) -> torch.Tensor:
    """``grouped_nvfp4_mm`` (praxis/kernels/nvfp4.py:355-419; FlashInfer
    block-scaled contiguous grouped GEMM, alpha = 1, 128-row expert tiles):
    out[r, :] = bf16(f32(sum_k dq(a[r,k]) * dq(b[e(r), :, k]))) with exact
    products accumulated in float64."""
    rows = a_q.shape[0]
    a = dequant_rows(a_q, a_sf, k).to(torch.float64)
    out = torch.zeros(rows, n, dtype=_BF16)
    e = b_q.shape[0]
    bounds = pcsr.tolist()
    for expert in range(e):
        lo, hi = bounds[expert], bounds[expert + 1]
        if expert == e - 1:
            hi = rows
        if hi <= lo:
            continue
        w = dequant_matrix(b_q[expert], b_sf[expert], n, k).to(torch.float64)
        out[lo:hi] = (a[lo:hi] @ w.t()).to(_F32).to(_BF16)
    return out


def grouped_gemm_rows(a_q, a_sf, b_q, b_sf, experts_of_rows, k: int, n: int) -> torch.Tensor:
    """The same computation for an arbitrary list of rows (one expert id per
    row): lets large-shape tests check a sample of rows."""
    a = dequant_rows(a_q, a_sf, k).to(torch.float64)
    out = torch.empty(a_q.shape[0], n, dtype=_BF16)
    for expert in experts_of_rows.unique().tolist():
        sel = (experts_of_rows == expert).nonzero().flatten()
        w = dequant_matrix(b_q[expert], b_sf[expert], n, k).to(torch.float64)
        out[sel] = (a[sel] @ w.t()).to(_F32).to(_BF16)
    return out


# ---------------------------------------------------------------------------
# Epilogues
# ---------------------------------------------------------------------------
def rescale_swiglu_maximum(gu: torch.Tensor, pcsr: torch.Tensor, ag, wg):
    """praxis/kernels/nvfp4_moe.py:102-133: m = bf16(g_a*g_w);
    gate = bf16(gu_gate*m); up = bf16(gu_up*m);
    h = bf16(bf16(gate*sigmoid(gate)) * up); row max |h| as bf16."""
    rows, h2 = gu.shape
    h = h2 // 2
    expert = expert_of_rows(pcsr, torch.arange(rows))
    m = bf16_round(ag[expert] * wg[expert]).unsqueeze(1)
    gate = bf16_round(gu[:, :h].to(_F32) * m)
    up = bf16_round(gu[:, h:].to(_F32) * m)
    silu = bf16_round(gate * torch.sigmoid(gate))
    hidden = (silu * up).to(_BF16)
    return hidden, hidden.to(_F32).abs().amax(-1).to(_BF16)


def rescale_combine(raw, inverse, top_idx, gate, csr, pcsr, hg, wg, scaling, shared=None):
    """praxis/kernels/nvfp4_moe.py:206-269: per token and slot
    v = bf16(raw[src] * bf16(g_h*g_w)); acc[s % 4] += v * (gate * scaling);
    y = bf16(((a0 + a1) + a2) + a3); y = bf16(y + shared)."""
    t, k = top_idx.shape
    c = raw.shape[1]
    accs = [torch.zeros(t, c, dtype=_F32) for _ in range(4)]
    sc = f32(float(scaling))
    for s in range(k):
        i = inverse.reshape(t, k)[:, s]
        e = top_idx[:, s]
        src = pcsr.to(torch.int64)[e] + i - csr.to(torch.int64)[e]
        mult = bf16_round(hg[e] * wg[e]).unsqueeze(1)
        v = bf16_round(raw[src].to(_F32) * mult)
        scale = (gate[:, s].to(_F32) * sc).unsqueeze(1)
        accs[s % 4] = accs[s % 4] + v * scale
    y = (((accs[0] + accs[1]) + accs[2]) + accs[3]).to(_BF16)
    if shared is not None:
        y = (y.to(_F32) + shared.to(_F32)).to(_BF16)
    return y


def rms_sum_of_squares(xo: torch.Tensor) -> torch.Tensor:
    """Per row, sum of f32(xo)^2 in the order of torch's vectorized RMSNorm
    kernel that the reference's fused norms reproduce
    (praxis/kernels/norm_triton.py:11-22, praxis/kernels/moe_tail_triton.py:
    160-190): 128 threads t = 32 w + l, thread t adds the squares of the four
    elements of float4 vectors t, t + 128, ... in order; a shuffle-down tree
    (16, 8, 4, 2, 1) per warp; then (w0 + w2) + (w1 + w3). Missing elements
    (rows not a multiple of 512 wide) add +0.0."""
    t, n = xo.shape
    ni = (n + 511) // 512
    v = torch.zeros(t, ni * 512, dtype=_F32)
    v[:, :n] = xo.to(_F32)
    v = v.reshape(t, ni, 4, 32, 4)
    acc = torch.zeros(t, 4, 32, dtype=_F32)
    for i in range(ni):
        for e in range(4):
            q = v[:, i, :, :, e]
            acc = acc + q * q
    for off in (16, 8, 4, 2, 1):
        acc = acc[..., :off] + acc[..., off:2 * off]
    w = acc[..., 0]
    return (w[:, 0] + w[:, 2]) + (w[:, 1] + w[:, 3])


def mod_row_map(rows: int, geom=None) -> torch.Tensor:
    """The modulation row of token rows 0..rows-1
    (praxis/kernels/norm_triton.py:417-431): geom = (RF, RC, NREG, PW, WD,
    PH) of a compact modulation, None for one row per token."""
    r = torch.arange(rows, dtype=torch.int64)
    if geom is None:
        return r
    rf, rc, nreg, pw, wd, ph = (int(v) for v in geom)
    b = r // rf
    t = r - b * rf
    q = (t - nreg).clamp(min=0) // pw
    return b * rc + torch.where(t < nreg, t, nreg + ((q // wd) // ph) * wd + q % wd)


def tail_residual_add(y: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """``x + y`` in bf16 (praxis/kernels/moe_tail_triton.py:401-428)."""
    return (x.to(_F32) + y.to(_F32)).to(_BF16)


def tail_modulate(xo: torch.Tensor, mod: torch.Tensor, mrow: torch.Tensor) -> torch.Tensor:
    """The modulation of praxis/kernels/moe_tail_triton.py:257-266 on the
    new residual: bf16(xo * bf16(scale + 1) + shift), mod rows [R, 2C] =
    (shift | scale). With bf16 operands the product is exact in fp32, so the
    fused and the unfused forms round alike."""
    n = xo.shape[1]
    m = mod[mrow].to(_F32)
    sh, sc = m[:, :n], m[:, n:]
    sc1 = (sc + f32(1.0)).to(_BF16).to(_F32)
    return (xo.to(_F32) * sc1 + sh).to(_BF16)


def tail_add_norm_scale(y: torch.Tensor, x: torch.Tensor, w1: torch.Tensor, eps: float, s: float,
                        mod: torch.Tensor | None = None, geom=None, row0: int = 0):
    """The MoE tail fused into the next block's residual add + RMSNorm
    (praxis/kernels/moe_tail_triton.py:108-190, the ``add_norm_scale``
    contract of praxis/kernels/norm_triton.py:1-32): xo = bf16(x + y);
    with ``mod`` the modulation of :func:`tail_modulate` (rows mapped by
    :func:`mod_row_map` from token row + ``row0``, moe_tail_triton.py:
    196-307); r = rsqrt(ss / N + eps) (IEEE division; here the correctly
    rounded reciprocal square root, where the GPU's hardware estimate may
    differ by an ulp); h = bf16(bf16(w1 * (r * xo)) * s), w1 = 1 + weight in
    fp32."""
    n = x.shape[1]
    xo = tail_residual_add(y, x)
    if mod is not None:
        xo = tail_modulate(xo, mod, mod_row_map(row0 + x.shape[0], geom)[row0:])
    ss = rms_sum_of_squares(xo)
    v = ss / f32(float(n)) + f32(float(eps))
    r = v.to(torch.float64).rsqrt().to(_F32).unsqueeze(1)
    o = (w1.to(_F32).unsqueeze(0) * (r * xo.to(_F32))).to(_BF16)
    h = (o.to(_F32) * f32(float(s))).to(_BF16)
    return xo, h


# ---------------------------------------------------------------------------
# The routed bank forward
# ---------------------------------------------------------------------------
def expert_outputs(x, tokens, offsets, bank, trace=None, hidden_global=None):
    """``_expert_outputs(raw_output=True)`` on SM100
    (praxis/quantization/nvfp4.py:291-388): returns raw, csr, pcsr, g_h.
    ``hidden_global``: a calibrated FC1 output scale (the
    ``set_fused_swiglu_scale`` path, :327-339): the hidden rows are
    quantized at this frozen global for every expert, which the combine's
    rescale then uses."""
    e = bank["gate_up_q"].shape[0]
    c = x.shape[1]
    f = bank["down_q"].shape[2] * 2
    csr = torch.nn.functional.pad(offsets, (1, 0))
    m = tokens.numel()
    pcsr = pad_csr(csr)
    prows = padded_rows(m, e)
    ag = segment_global_scales(row_amax(x), csr, tokens)
    aq, asf = quantize_activations(x, csr, pcsr, prows, ag, row_indices=tokens)
    gu = grouped_gemm(aq, asf, bank["gate_up_q"], bank["gate_up_sf"], pcsr, c, 2 * f)
    hidden, rowmax = rescale_swiglu_maximum(gu, pcsr, ag, bank["gate_up_global"])
    if hidden_global is None:
        hg = segment_global_scales(rowmax, pcsr)
    else:
        hg = torch.full((e,), float(hidden_global), dtype=_F32)
    hq, hsf = quantize_activations(hidden, pcsr, pcsr, prows, hg)
    raw = grouped_gemm(hq, hsf, bank["down_q"], bank["down_sf"], pcsr, f, c)
    if trace is not None:
        trace.update(dict(csr=csr, pcsr=pcsr, ag=ag, aq=aq, asf=asf, gu=gu,
                          hidden=hidden, hg=hg, hq=hq, hsf=hsf, raw=raw))
    return raw, csr, pcsr, hg


def routed_forward(x, top_idx, gate, bank, scaling, chunk_size, shared=None, trace=None, hidden_global=None):
    """``NVFP4RoutedExperts._routed_forward`` on SM100
    (praxis/quantization/nvfp4.py:616-747): per dispatch chunk, dispatch,
    expert outputs and the fused rescale + combine (+ shared);
    ``hidden_global`` as in :func:`expert_outputs`."""
    e = bank["gate_up_q"].shape[0]
    out = torch.empty_like(x)
    for start in range(0, x.shape[0], chunk_size):
        end = min(start + chunk_size, x.shape[0])
        order, inverse, tokens, _sg, offsets, _csr = dispatch(top_idx[start:end], gate[start:end], e)
        raw, csr, pcsr, hg = expert_outputs(x[start:end], tokens, offsets, bank, trace, hidden_global)
        out[start:end] = rescale_combine(
            raw, inverse, top_idx[start:end], gate[start:end], csr, pcsr, hg,
            bank["down_global"], scaling, None if shared is None else shared[start:end],
        )
    return out


def moe_forward(x, router_weight, expert_bias, bank, top_k, scaling, chunk_size,
                activation="sigmoid", shared=None):
    """Router + routed bank (the MoE module's routed path,
    praxis/layers.py:2134-2199 with the NVFP4 bank)."""
    logits = router_logits(x, router_weight)
    top_idx, gate = route(logits, expert_bias, top_k, activation)
    return routed_forward(x, top_idx, gate, bank, scaling, chunk_size, shared), top_idx, gate


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.to(torch.float64)
    b = b.to(torch.float64)
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def flops_per_layer(tokens: int, top_k: int, c: int, f: int) -> float:
    """Algorithmic GEMM FLOPs, padding excluded: 6 * R * C * F."""
    return 6.0 * tokens * top_k * c * f


__all__ = [name for name in dir() if not name.startswith("_")] + ["math"]
