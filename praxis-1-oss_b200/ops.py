"""Torch-facing functions over the C ABI (one per reference kernel function).

Each function checks its tensors (``ValueError`` before any launch, like
praxis/quantization/nvfp4.py:631-675), allocates its outputs with the torch
caching allocator, and enqueues the CUDA library's kernels on the current
stream of the tensors' device. No host synchronisation, so every op can be
captured in a CUDA graph. There is no CPU path: the library must be built
and a sm_100 GPU present.
"""

from __future__ import annotations

import ctypes as C
from typing import NamedTuple

import torch
from torch import Tensor

from . import capi

BF16 = torch.bfloat16


def _p(t: Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dev(t: Tensor) -> int:
    if t.device.type != "cuda":
        raise ValueError("praxis_b200 ops need CUDA tensors")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _stream(t: Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need(t: Tensor, name: str, dtype, ndim: int | None = None, device=None) -> None:
    if not isinstance(t, Tensor) or t.dtype != dtype or not t.is_contiguous() or t.device.type != "cuda":
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name}: expected {ndim} dims, got {t.ndim}")
    if device is not None and t.device != device:
        raise ValueError(f"{name}: tensors must share a device")


def padded_rows(routed_rows: int, experts: int) -> int:
    """praxis/kernels/nvfp4.py:213 with alignment 128."""
    return (routed_rows + 127 * experts) // 128 * 128


class Routing(NamedTuple):
    """``praxis.kernels.router_fused.Routing`` (router_fused.py:58-68) plus the
    grouped-GEMM metadata of this library (csr, pcsr, tiles, globals)."""

    top_idx: Tensor
    gate: Tensor
    order: Tensor
    inverse: Tensor
    sorted_gate: Tensor
    tokens: Tensor
    tokens32: Tensor
    seg_csr: Tensor
    offsets: Tensor
    rows: tuple
    csr: Tensor
    pcsr: Tensor
    tiles: Tensor
    num_tiles: Tensor
    act_global: Tensor | None
    act_amax: Tensor | None


def split_router_weight(weight: Tensor) -> Tensor:
    """[E, C] router weight -> [S, E, C] bf16 terms whose sum is the weight:
    S = 1 for bf16, S = 3 (hi, mid, lo) for fp32 (exact decomposition)."""
    if weight.dtype == BF16:
        return weight.contiguous().unsqueeze(0)
    w = weight.to(torch.float32)
    hi = w.to(BF16)
    r1 = w - hi.float()
    mid = r1.to(BF16)
    lo = (r1 - mid.float()).to(BF16)
    return torch.stack([hi, mid, lo]).contiguous()


def router_logits(x: Tensor, weight_terms: Tensor) -> tuple[Tensor, Tensor]:
    """fp32 logits x @ W^T (praxis/layers.py:1104-1122) and bf16 row max |x|
    (praxis/kernels/nvfp4_moe.py:15-21) in one pass."""
    _need(x, "x", BF16, 2)
    _need(weight_terms, "router weight", BF16, 3, x.device)
    t, c = x.shape
    s, e, c2 = weight_terms.shape
    if c2 != c:
        raise ValueError("router weight / activation width mismatch")
    logits = torch.empty(t, e, dtype=torch.float32, device=x.device)
    amax = torch.empty(t, dtype=BF16, device=x.device)
    capi.check(capi.load().praxis_b200_router_logits(
        _p(x), _p(weight_terms), s, t, c, e, _p(logits), _p(amax), _dev(x), _stream(x)))
    return logits, amax


def route(logits: Tensor, bias: Tensor | None, top_k: int, activation: str = "sigmoid") -> tuple[Tensor, Tensor]:
    """Gating + top-k + renormalised bf16 gates (praxis/layers.py:1647-1653)."""
    _need(logits, "logits", torch.float32, 2)
    if bias is not None:
        _need(bias, "expert bias", torch.float32, 1, logits.device)
    t, e = logits.shape
    act = {"sigmoid": capi.SIGMOID, "softmax": capi.SOFTMAX}[activation]
    top_idx = torch.empty(t, top_k, dtype=torch.int64, device=logits.device)
    gate = torch.empty(t, top_k, dtype=BF16, device=logits.device)
    capi.check(capi.load().praxis_b200_route(
        _p(logits), _p(bias), t, e, top_k, act, _p(top_idx), _p(gate), _dev(logits), _stream(logits)))
    return top_idx, gate


def row_amax(x: Tensor) -> Tensor:
    _need(x, "x", BF16, 2)
    out = torch.empty(x.shape[0], dtype=BF16, device=x.device)
    capi.check(capi.load().praxis_b200_row_amax(_p(x), x.shape[0], x.shape[1], _p(out), _dev(x), _stream(x)))
    return out


def _passes(rows, t: int) -> tuple[int, int]:
    """(passes, tokens of pass 0) of the reference's ``rows`` tuple: one input
    (``(T,)`` or None) or a lockstep pair ``(T0, T1)``."""
    if rows is None:
        return 1, 0
    rows = tuple(int(r) for r in rows)
    if len(rows) not in (1, 2) or sum(rows) != t or min(rows) < 0:
        raise ValueError(f"rows {rows}: one or two inputs whose tokens add up to {t}")
    return (2, rows[0]) if len(rows) == 2 else (1, 0)


def dispatch(top_idx: Tensor, gate: Tensor, num_experts: int, amax: Tensor | None = None,
             full: bool = True, rows: tuple | None = None) -> Routing:
    """``_dispatch_rows`` + inverse + padded CSR + tile table (+ activation
    global scales from ``amax``) on the device. ``rows = (T0, T1)``: the
    tokens are a lockstep pair (praxis/kernels/router_fused.py:820-852, P =
    2); csr / pcsr / tiles / globals are then per (expert, input) group
    2 e + s, ``seg_csr`` is the reference's and ``offsets`` its per-expert
    end offsets."""
    _need(top_idx, "top_idx", torch.int64, 2)
    _need(gate, "gate", BF16, 2, top_idx.device)
    if gate.shape != top_idx.shape:
        raise ValueError("gate / top_idx shape mismatch")
    t, k = top_idx.shape
    npass, t0 = _passes(rows, t)
    dev = top_idx.device
    r = t * k
    e = num_experts
    g = e * npass
    max_tiles = padded_rows(r, g) // 128
    lib = capi.load()
    ws = torch.empty(int(lib.praxis_b200_dispatch_passes_workspace_size(t, k, e, npass)), dtype=torch.uint8,
                     device=dev)
    i64 = dict(dtype=torch.int64, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    order = torch.empty(r, **i64) if full else None
    inverse = torch.empty(r, **i64)
    tokens = torch.empty(r, **i64) if full else None
    tokens32 = torch.empty(r, **i32) if full else None
    sorted_gate = torch.empty(r, dtype=BF16, device=dev) if full else None
    offsets = torch.empty(g, **i32)
    csr = torch.empty(g + 1, **i32)
    pcsr = torch.empty(g + 1, **i32)
    tiles = torch.empty(2 * max(max_tiles, 1), 4, **i32)  # 128-row tiles, then 256-row pairs
    num_tiles = torch.empty(2, **i32)
    act_global = act_amax = None
    if amax is not None:
        _need(amax, "row amax", BF16, 1, dev)
        act_global = torch.empty(g, dtype=torch.float32, device=dev)
        act_amax = torch.empty(g, dtype=torch.int32, device=dev)
    capi.check(lib.praxis_b200_dispatch_passes(
        _p(top_idx), _p(gate), _p(amax), t, k, e, npass, t0, _p(ws), ws.numel(), _p(order), _p(inverse),
        _p(tokens), _p(tokens32), _p(sorted_gate), _p(offsets), _p(csr), _p(pcsr), _p(tiles), max_tiles,
        _p(num_tiles), _p(act_global), _p(act_amax), _dev(top_idx), _stream(top_idx)))
    rows_t = (t,) if npass == 1 else (t0, t - t0)
    return Routing(top_idx, gate, order, inverse, sorted_gate, tokens, tokens32, csr,
                   offsets if npass == 1 else offsets[1::2], rows_t, csr, pcsr, tiles, num_tiles, act_global,
                   act_amax)


def dispatch_noalloc(top_idx: Tensor, gate: Tensor, num_experts: int, amax: Tensor | None = None, *,
                     order: Tensor, inverse: Tensor, tokens: Tensor, tokens32: Tensor, sorted_gate: Tensor,
                     offsets: Tensor, csr: Tensor, pcsr: Tensor, tiles: Tensor, num_tiles: Tensor,
                     act_global: Tensor | None = None, act_amax: Tensor | None = None) -> None:
    """:func:`dispatch` into caller-owned output tensors through
    ``praxis_b200_dispatch_noalloc``: no workspace, nothing allocated."""
    _need(top_idx, "top_idx", torch.int64, 2)
    _need(gate, "gate", BF16, 2, top_idx.device)
    if gate.shape != top_idx.shape:
        raise ValueError("gate / top_idx shape mismatch")
    t, k = top_idx.shape
    _check_dispatch_outputs(t, k, num_experts, top_idx.device, amax, order=order, inverse=inverse, tokens=tokens,
                            tokens32=tokens32, sorted_gate=sorted_gate, offsets=offsets, csr=csr, pcsr=pcsr,
                            tiles=tiles, num_tiles=num_tiles, act_global=act_global, act_amax=act_amax)
    max_tiles = tiles.shape[0] // 2
    capi.check(capi.load().praxis_b200_dispatch_noalloc(
        _p(top_idx), _p(gate), _p(amax), t, k, num_experts, _p(order), _p(inverse), _p(tokens), _p(tokens32),
        _p(sorted_gate), _p(offsets), _p(csr), _p(pcsr), _p(tiles), max_tiles, _p(num_tiles), _p(act_global),
        _p(act_amax), _dev(top_idx), _stream(top_idx)))


def _check_dispatch_outputs(t: int, k: int, e: int, device, amax: Tensor | None, *, order: Tensor, inverse: Tensor,
                            tokens: Tensor, tokens32: Tensor, sorted_gate: Tensor, offsets: Tensor, csr: Tensor,
                            pcsr: Tensor, tiles: Tensor, num_tiles: Tensor, act_global: Tensor | None,
                            act_amax: Tensor | None) -> None:
    """Caller-owned dispatch outputs: dtype, contiguity, device and size of
    every buffer the kernels write, checked before any launch (an undersized
    or mistyped buffer would be written out of bounds on the device)."""
    r = t * k
    if e < 1:
        raise ValueError("num_experts must be positive")

    def need(ten, name, dtype, numel):
        if not isinstance(ten, Tensor) or ten.dtype != dtype or not ten.is_contiguous() or ten.device != device:
            raise ValueError(f"{name}: expected a contiguous {dtype} tensor on {device}")
        if ten.numel() < numel:
            raise ValueError(f"{name}: needs at least {numel} elements, got {ten.numel()}")

    for name, ten, dtype, numel in (
        ("order", order, torch.int64, r), ("inverse", inverse, torch.int64, r), ("tokens", tokens, torch.int64, r),
        ("tokens32", tokens32, torch.int32, r), ("sorted_gate", sorted_gate, BF16, r),
        ("offsets", offsets, torch.int32, e), ("csr", csr, torch.int32, e + 1), ("pcsr", pcsr, torch.int32, e + 1),
        ("num_tiles", num_tiles, torch.int32, 2),
    ):
        need(ten, name, dtype, numel)
    need(tiles, "tiles", torch.int32, 0)
    want_tiles = max(padded_rows(r, e) // 128, 1)
    if tiles.ndim != 2 or tiles.shape[1] != 4 or tiles.shape[0] % 2 or tiles.shape[0] // 2 < want_tiles:
        raise ValueError(f"tiles: expected int32 [2 * max_tiles, 4] with max_tiles >= {want_tiles}")
    if amax is not None:
        need(amax, "row amax", BF16, t)
    if act_global is not None:
        need(act_global, "act_global", torch.float32, e)
    if act_amax is not None:
        need(act_amax, "act_amax", torch.int32, e)


def route_dispatch(logits: Tensor, bias: Tensor, rows: tuple, top_k: int = 8,
                   activation: str = "sigmoid") -> Routing:
    """``router_fused.route_dispatch`` (praxis/kernels/router_fused.py:738)
    for one input (``rows = (T,)``) or a lockstep pair (``rows = (T0, T1)``,
    the reference's P = 2), any E <= 256 and k <= 8."""
    _passes(rows, logits.shape[0])
    top_idx, gate = route(logits, bias, top_k, activation)
    return dispatch(top_idx, gate, logits.shape[1], rows=rows)


def _sf_buffer(rows: int, kdim: int, sf_layout: int, device) -> Tensor:
    """Scale buffer: [rows, K/16] compact, or the flat replicated layout."""
    if sf_layout == capi.SF_COMPACT:
        return torch.empty(rows, kdim // 16, dtype=torch.uint8, device=device)
    if sf_layout == capi.SF_REPLICATED:
        return torch.empty(4 * rows * (kdim // 16), dtype=torch.uint8, device=device)
    raise ValueError(f"unknown scale layout {sf_layout}")


def quantize_gather(x: Tensor, routing: Routing, act_global: Tensor, *,
                    sf_layout: int = capi.SF_COMPACT) -> tuple[Tensor, Tensor]:
    """``quantize_activations(x, csr, row_indices=tokens, alignment=128,
    grouped_scales=False)`` (praxis/kernels/nvfp4.py:197-254) into the
    padded layout; padding rows of partly filled tiles are zero. With
    ``sf_layout=SF_REPLICATED`` the scales come in the GEMM's replicated
    layout (flat, 4x the compact size)."""
    _need(x, "x", BF16, 2)
    t, c = x.shape
    k = routing.top_idx.shape[1]
    e = routing.csr.numel() - 1
    rp = padded_rows(t * k, e)
    q = torch.empty(rp, c // 2, dtype=torch.uint8, device=x.device)
    sf = _sf_buffer(rp, c, sf_layout, x.device)
    capi.check(capi.load().praxis_b200_quantize_gather(
        _p(x), t, c, _p(routing.top_idx), _p(routing.inverse), _p(routing.csr), _p(routing.pcsr), _p(act_global),
        None, k, e, _p(routing.tiles), _p(routing.num_tiles), rp // 128, _p(q), _p(sf), sf_layout, _dev(x),
        _stream(x)))
    return q, sf


def quantize_rows(x: Tensor, routing: Routing, globals_: Tensor | None = None,
                  amax_bits: Tensor | None = None, *, sf_layout: int = capi.SF_COMPACT) -> tuple[Tensor, Tensor]:
    """Quantize every row of the routed tiles of a padded [Rp, K] tensor."""
    _need(x, "x", BF16, 2)
    rp, kdim = x.shape
    q = torch.empty(rp, kdim // 2, dtype=torch.uint8, device=x.device)
    sf = _sf_buffer(rp, kdim, sf_layout, x.device)
    capi.check(capi.load().praxis_b200_quantize_rows(
        _p(x), kdim, _p(routing.tiles), _p(routing.num_tiles), rp // 128, _p(globals_), _p(amax_bits), _p(q),
        _p(sf), sf_layout, _dev(x), _stream(x)))
    return q, sf


def grouped_gemm(a_q: Tensor, a_sf: Tensor, b_q: Tensor, b_sf: Tensor, routing: Routing, *,
                 epilogue: int = capi.EPI_PLAIN, act_global: Tensor | None = None,
                 act_amax: Tensor | None = None, w_global: Tensor | None = None,
                 amax_out: Tensor | None = None, sf_layout: int = capi.SF_COMPACT) -> Tensor:
    """``grouped_nvfp4_mm`` (praxis/kernels/nvfp4.py:355-419) on tcgen05 with
    an optional fused epilogue (see include/praxis_b200_moe.h). With
    ``sf_layout=SF_REPLICATED`` a_sf is replicated in 128-row groups and b_sf
    in 256-row groups (:func:`replicate_scales`)."""
    rp = a_q.shape[0]
    kdim = a_q.shape[1] * 2
    e, n = b_q.shape[0], b_q.shape[1]
    if b_q.shape[2] * 2 != kdim:
        raise ValueError("A / B reduction width mismatch")
    cols = n // 2 if epilogue == capi.EPI_SWIGLU else n
    out = torch.empty(rp, cols, dtype=BF16, device=a_q.device)
    capi.check(capi.load().praxis_b200_grouped_gemm(
        _p(a_q), _p(a_sf), _p(b_q), _p(b_sf), _p(routing.tiles), _p(routing.num_tiles), rp // 128, rp, n, kdim, e,
        epilogue, _p(out), _p(act_global), _p(act_amax), _p(w_global), _p(amax_out), sf_layout, _dev(a_q),
        _stream(a_q)))
    return out


def grouped_gemm_swiglu_fp4(a_q: Tensor, a_sf: Tensor, b_q: Tensor, b_sf: Tensor, routing: Routing, *,
                            act_global: Tensor, w_global: Tensor, hidden_global: float) -> tuple[Tensor, Tensor]:
    """The gate/up GEMM with SwiGLU and FP4 hidden output at the calibrated
    global ``hidden_global`` (``gate_up_fp4``, praxis/kernels/nvfp4_swiglu.py:
    40-74): returns (q [Rp, F/2], sf [Rp, F/16] compact), the bytes that
    :func:`quantize_rows` gives for the EPI_SWIGLU hidden rows at that
    global. ``b_q`` / ``b_sf`` in the interleaved gate/up layout."""
    _need(a_q, "a_q", torch.uint8, 2)
    rp = a_q.shape[0]
    e, n, _ = b_q.shape
    k = a_q.shape[1] * 2
    f = n // 2
    q = torch.empty(rp, f // 2, dtype=torch.uint8, device=a_q.device)
    sf = torch.empty(rp, f // 16, dtype=torch.uint8, device=a_q.device)
    capi.check(capi.load().praxis_b200_gemm_swiglu_fp4(
        _p(a_q), _p(a_sf), _p(b_q), _p(b_sf), _p(routing.tiles), _p(routing.num_tiles), rp // 128,
        rp, n, k, e, _p(act_global), None, _p(w_global), float(hidden_global), _p(q), _p(sf), _dev(a_q),
        _stream(a_q)))
    return q, sf


def replicate_scales(sf: Tensor, group_rows: int) -> Tensor:
    """Compact swizzled scales [..., rows, K/16] -> the GEMM's replicated
    layout (flat uint8, 4x the size); ``group_rows`` 128 for activation
    rows, 256 for weight rows (all experts' rows taken as one stack)."""
    _need(sf, "sf", torch.uint8)
    kdim = sf.shape[-1] * 16
    rows = sf.numel() // sf.shape[-1]
    out = torch.empty(4 * sf.numel(), dtype=torch.uint8, device=sf.device)
    capi.check(capi.load().praxis_b200_replicate_scales(
        _p(sf), rows, kdim, group_rows, _p(out), _dev(sf), _stream(sf)))
    return out


def rescale_swiglu(raw: Tensor, pcsr: Tensor, act_global: Tensor, w_global: Tensor, *, alu: bool = True
                   ) -> tuple[Tensor, Tensor]:
    """``rescale_swiglu_maximum`` (praxis/kernels/nvfp4_moe.py:136-158) on the
    padded gate/up GEMM output; ``alu`` picks the fused epilogue's arithmetic."""
    _need(raw, "raw", BF16, 2)
    rows, h2 = raw.shape
    out = torch.empty(rows, h2 // 2, dtype=BF16, device=raw.device)
    rowmax = torch.empty(rows, dtype=BF16, device=raw.device)
    capi.check(capi.load().praxis_b200_rescale_swiglu(
        _p(raw), rows, h2 // 2, _p(pcsr), pcsr.numel() - 1, _p(act_global), _p(w_global), _p(out), _p(rowmax),
        int(alu), _dev(raw), _stream(raw)))
    return out, rowmax


def combine(rows: Tensor, routing: Routing, scaling: float, *, h_global: Tensor | None = None,
            h_amax: Tensor | None = None, w_global: Tensor | None = None, rows_rescaled: bool = False,
            shared: Tensor | None = None) -> Tensor:
    """``rescale_combine`` (praxis/kernels/nvfp4_moe.py:206-311)."""
    t, k = routing.top_idx.shape
    c = rows.shape[1]
    e = routing.csr.numel() - 1
    out = torch.empty(t, c, dtype=BF16, device=rows.device)
    if shared is not None:
        _need(shared, "shared", BF16, 2, rows.device)
    capi.check(capi.load().praxis_b200_combine(
        _p(rows), c, _p(routing.inverse), _p(routing.top_idx), _p(routing.gate), _p(routing.csr),
        _p(routing.pcsr), _p(h_global), _p(h_amax), _p(w_global), int(rows_rescaled), float(scaling), _p(shared),
        _p(out), t, k, e, _dev(rows), _stream(rows)))
    return out


class Tail(NamedTuple):
    """What follows the MoE output in the reference's MOE_TAIL_NORM path
    (praxis/layers.py:429-441, praxis/kernels/moe_tail_triton.py:329-445):
    the residual add of ``residual``; with ``norm_weight`` (fp32 ``1 +
    weight`` of the next block's zero-centred RMSNorm, its ``eps``) the norm
    of the new residual times ``norm_scale``; with ``mod`` ([R, 2C] bf16,
    shift then scale, row map ``mod_geom`` = (RF, RC, NREG, PW, WD, PH) of
    ``CompactMod`` or None for one row per token, applied to the token's row
    + ``mod_row0``) the modulation between the two, fused (``mod_fma``) or
    rounded product first."""

    residual: Tensor
    norm_weight: Tensor | None = None
    eps: float = 1e-6
    norm_scale: float = 1.0
    mod: Tensor | None = None
    mod_fma: bool = True
    mod_geom: tuple | None = None
    mod_row0: int = 0

    def chunk(self, start: int, end: int) -> "Tail":
        """The tail of token rows start..end-1 (the modulation rows keep
        their global row map)."""
        return self._replace(residual=self.residual[start:end], mod_row0=self.mod_row0 + start)


def _tail_struct(tail: Tail, t: int, c: int, device, outs: tuple | None = None
                 ) -> tuple[capi.TailArgs, Tensor, Tensor | None]:
    """Validates ``tail`` for [t, c] outputs on ``device`` and allocates them
    (or checks ``outs`` = (new residual, normed rows or None))."""
    _need(tail.residual, "residual", BF16, 2, device)
    if tuple(tail.residual.shape) != (t, c):
        raise ValueError("the residual does not match the MoE output shape")
    if tail.norm_weight is not None:
        _need(tail.norm_weight, "norm weight", torch.float32, 1, device)
        if tail.norm_weight.numel() != c:
            raise ValueError("the norm weight does not match the hidden size")
    if tail.mod is not None:
        if tail.norm_weight is None:
            raise ValueError("the modulation needs the norm")
        _need(tail.mod, "mod", BF16, 2, device)
        if tail.mod.shape[1] != 2 * c:
            raise ValueError("modulation rows must be [R, 2C] (shift | scale)")
        geom = (1, 1, 0, 1, 1, 1) if tail.mod_geom is None else tuple(int(v) for v in tail.mod_geom)
        need_rows = _mod_rows_needed(t + int(tail.mod_row0), geom)
        if tail.mod.shape[0] < need_rows:
            raise ValueError(f"modulation has {tail.mod.shape[0]} rows, the token rows map to {need_rows}")
    else:
        geom = (1, 1, 0, 1, 1, 1)
    if outs is None:
        residual_out = torch.empty_like(tail.residual)
        normed = None if tail.norm_weight is None else torch.empty_like(tail.residual)
    else:
        residual_out, normed = outs
        for ten, name in ((residual_out, "residual_out"), (normed, "normed_out")):
            if ten is None and (name == "residual_out" or tail.norm_weight is not None):
                raise ValueError(f"{name} is missing")
            if ten is not None:
                _need(ten, name, BF16, 2, device)
                if tuple(ten.shape) != (t, c) or not ten.is_contiguous():
                    raise ValueError(f"{name} must be a contiguous [{t}, {c}] tensor")
    st = capi.TailArgs(
        residual=tail.residual.data_ptr(), residual_out=residual_out.data_ptr(),
        norm_weight=_p(tail.norm_weight), normed_out=_p(normed), eps=float(tail.eps),
        norm_scale=float(tail.norm_scale), mod=_p(tail.mod), mod_fma=int(bool(tail.mod_fma)),
        mod_geom=(capi.I64 * 6)(*geom), mod_row0=int(tail.mod_row0))
    return st, residual_out, normed


def _mod_rows_needed(t: int, geom: tuple) -> int:
    """1 + the largest modulation row the token rows 0..t-1 map to
    (praxis/kernels/norm_triton.py:417-431)."""
    rf, rc, nreg, pw, wd, ph = geom
    if min(rf, rc, pw, wd, ph) <= 0 or nreg < 0:
        raise ValueError(f"bad modulation geometry {geom}")
    if t == 0:
        return 0
    row = torch.arange(t, dtype=torch.int64)
    b = row // rf
    tt = row - b * rf
    q = (tt - nreg).clamp(min=0) // pw
    col = torch.where(tt < nreg, tt, nreg + (q // wd) // ph * wd + q % wd)
    return int((b * rc + col).max()) + 1


def combine_tail(rows: Tensor, routing: Routing, scaling: float, tail: Tail, *, shared: Tensor | None = None,
                 h_global: Tensor | None = None, h_amax: Tensor | None = None, w_global: Tensor | None = None,
                 rows_rescaled: bool = False) -> tuple[Tensor, Tensor | None]:
    """The combine of :func:`combine` (with ``shared``) fused into ``tail``
    (MOE_TAIL_NORM: ``tail_add_norm_scale``, ``tail_add_mod_norm_scale`` or
    ``tail_residual_add`` of praxis/kernels/moe_tail_triton.py:329-445):
    returns ``(new residual, normed rows or None)`` with the eager bits."""
    t, k = routing.top_idx.shape
    c = rows.shape[1]
    e = routing.csr.numel() - 1
    if shared is not None:
        _need(shared, "shared", BF16, 2, rows.device)
    st, residual_out, normed = _tail_struct(tail, t, c, rows.device)
    capi.check(capi.load().praxis_b200_combine_tail(
        _p(rows), c, _p(routing.inverse), _p(routing.top_idx), _p(routing.gate), _p(routing.csr), _p(routing.pcsr),
        _p(h_global), _p(h_amax), _p(w_global), int(rows_rescaled), float(scaling), _p(shared), C.byref(st), t, k,
        e, _dev(rows), _stream(rows)))
    return residual_out, normed


def pack_weights(w: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Expert-first bf16 bank [E, K, N] -> (q [E,N,K/2], sf [E,N,K/16],
    global [E]) on the GPU, the bytes of praxis/quantization/nvfp4.py:67-146."""
    _need(w, "weights", BF16, 3)
    e, kdim, n = w.shape
    q = torch.empty(e, n, kdim // 2, dtype=torch.uint8, device=w.device)
    sf = torch.empty(e, n, kdim // 16, dtype=torch.uint8, device=w.device)
    g = torch.empty(e, dtype=torch.float32, device=w.device)
    scratch = torch.empty(e, dtype=torch.int32, device=w.device)
    capi.check(capi.load().praxis_b200_pack_weights(
        _p(w), e, kdim, n, _p(q), _p(sf), _p(g), _p(scratch), _dev(w), _stream(w)))
    return q, sf, g


def interleave_gate_up(q: Tensor, sf: Tensor) -> tuple[Tensor, Tensor]:
    """The fused-SwiGLU GEMM layout of gate_up q/sf (64-row gate/up blocks)."""
    _need(q, "gate_up_q", torch.uint8, 3)
    _need(sf, "gate_up_sf", torch.uint8, 3, q.device)
    e, n2, c2 = q.shape
    qo = torch.empty_like(q)
    so = torch.empty_like(sf)
    capi.check(capi.load().praxis_b200_interleave_gate_up(
        _p(q), _p(sf), e, n2 // 2, c2 * 2, _p(qo), _p(so), _dev(q), _stream(q)))
    return qo, so


def expert_forward(q: Tensor, sf: Tensor, counts: Tensor, starts: Tensor, act_global: Tensor,
                   gate_up_q: Tensor, gate_up_sf: Tensor, gate_up_global: Tensor, down_q: Tensor,
                   down_sf: Tensor, down_global: Tensor, *, gate_up_sf_layout: int, down_sf_layout: int,
                   sm_limit: int = 0, out_ptr: int | None = None) -> Tensor | None:
    """The expert-rank half of an expert-parallel layer
    (``praxis_b200_expert_forward``): received NVFP4 rows in padded segments
    (segment v = source * E_local + local expert, ``counts[v]`` rows from
    ``starts[v]``) -> rescaled bf16 down-projection rows in the same layout.
    With ``out_ptr`` (a 16-byte aligned device address of ``rows`` x C bf16,
    e.g. in a peer's mapped buffer) the down GEMM writes the rows there and
    nothing is returned."""
    _need(q, "q", torch.uint8, 2)
    rows, c_half = q.shape
    c = c_half * 2
    f = down_q.shape[2] * 2
    e_local = down_q.shape[0]
    segments = counts.numel()
    _need(counts, "counts", torch.int32, 1, q.device)
    _need(starts, "starts", torch.int32, 1, q.device)
    _need(act_global, "act_global", torch.float32, 1, q.device)
    if starts.numel() != segments + 1 or act_global.numel() != segments:
        raise ValueError("starts / act_global do not match the segment count")
    out = torch.empty(rows, c, dtype=BF16, device=q.device) if out_ptr is None else None
    lib = capi.load()
    ws_size = int(lib.praxis_b200_expert_workspace_size(rows, segments, c, f))
    ws = torch.empty(max(ws_size, 1), dtype=torch.uint8, device=q.device)
    args = capi.ExpertArgs(
        q=q.data_ptr(), sf=sf.data_ptr(), rows=rows, counts=counts.data_ptr(), starts=starts.data_ptr(),
        act_global=act_global.data_ptr(), segments=segments, gate_up_q=gate_up_q.data_ptr(),
        gate_up_sf=gate_up_sf.data_ptr(), gate_up_global=gate_up_global.data_ptr(), down_q=down_q.data_ptr(),
        down_sf=down_sf.data_ptr(), down_global=down_global.data_ptr(), gate_up_sf_layout=int(gate_up_sf_layout),
        down_sf_layout=int(down_sf_layout),
        dim=c, hidden=f, experts=e_local, sm_limit=int(sm_limit),
        rows_out=out.data_ptr() if out is not None else int(out_ptr), workspace=ws.data_ptr(),
        workspace_size=ws.numel(), device=_dev(q), stream=torch.cuda.current_stream(q.device).cuda_stream,
    )
    capi.check(lib.praxis_b200_expert_forward(C.byref(args)))
    return out


def expert_hidden(q: Tensor, sf: Tensor, counts: Tensor, starts: Tensor, act_global: Tensor,
                  gate_up_q: Tensor, gate_up_sf: Tensor, gate_up_global: Tensor, *, hidden: int,
                  gate_up_sf_layout: int, sm_limit: int = 0, out: tuple | None = None
                  ) -> tuple[Tensor, Tensor, Tensor]:
    """The gate/up half of the expert rank (``praxis_b200_expert_forward`` in
    hidden-output mode): received NVFP4 rows in padded segments -> the FP4
    hidden rows [rows, F/2], their compact scales [rows, F/16] and each
    segment's max |hidden| (fp32 bits, int32 [segments]), quantized with one
    global per segment, as the single-GPU path quantizes each (chunk,
    expert). ``out``: (hq, hsf, hamax) views to write into (e.g. a peer's
    mapped buffer); else they are allocated."""
    _need(q, "q", torch.uint8, 2)
    rows, c_half = q.shape
    c = c_half * 2
    f = int(hidden)
    e_local = gate_up_global.numel()
    segments = counts.numel()
    _need(counts, "counts", torch.int32, 1, q.device)
    _need(starts, "starts", torch.int32, 1, q.device)
    _need(act_global, "act_global", torch.float32, 1, q.device)
    if starts.numel() != segments + 1 or act_global.numel() != segments:
        raise ValueError("starts / act_global do not match the segment count")
    if out is None:
        out = (torch.empty(rows, f // 2, dtype=torch.uint8, device=q.device),
               torch.empty(rows, f // 16, dtype=torch.uint8, device=q.device),
               torch.empty(segments, dtype=torch.int32, device=q.device))
    hq, hsf, hamax = out
    for ten, name, shape in ((hq, "hq", (rows, f // 2)), (hsf, "hsf", (rows, f // 16)), (hamax, "hamax", (segments,))):
        if tuple(ten.shape) != shape or not ten.is_contiguous() or ten.device != q.device:
            raise ValueError(f"{name}: expected a contiguous {shape} tensor on {q.device}")
    lib = capi.load()
    ws_size = int(lib.praxis_b200_expert_workspace_size(rows, segments, c, f))
    ws = torch.empty(max(ws_size, 1), dtype=torch.uint8, device=q.device)
    args = capi.ExpertArgs(
        q=q.data_ptr(), sf=sf.data_ptr(), rows=rows, counts=counts.data_ptr(), starts=starts.data_ptr(),
        act_global=act_global.data_ptr(), segments=segments, gate_up_q=gate_up_q.data_ptr(),
        gate_up_sf=gate_up_sf.data_ptr(), gate_up_global=gate_up_global.data_ptr(),
        gate_up_sf_layout=int(gate_up_sf_layout), down_sf_layout=capi.SF_COMPACT, dim=c, hidden=f,
        experts=e_local, sm_limit=int(sm_limit), workspace=ws.data_ptr(), workspace_size=ws.numel(),
        device=_dev(q), stream=torch.cuda.current_stream(q.device).cuda_stream, hidden_q=hq.data_ptr(),
        hidden_sf=hsf.data_ptr(), hidden_amax=hamax.data_ptr())
    capi.check(lib.praxis_b200_expert_forward(C.byref(args)))
    return hq, hsf, hamax


def _layout_of(sf: Tensor, q: Tensor, name: str) -> int:
    """Scale layout told by size: compact = q bytes / 8, replicated = q bytes / 2."""
    if sf.numel() * 8 == q.numel():
        return capi.SF_COMPACT
    if sf.numel() * 2 == q.numel():
        return capi.SF_REPLICATED
    raise ValueError(f"{name} size matches neither scale layout")


def moe_forward(x: Tensor, top_idx: Tensor | None, gate: Tensor | None, gate_up_q: Tensor, gate_up_sf: Tensor,
                gate_up_global: Tensor, down_q: Tensor, down_sf: Tensor, down_global: Tensor, scaling: float,
                shared: Tensor | None = None, *, router_terms: Tensor | None = None,
                router_bias: Tensor | None = None, top_k: int | None = None, activation: str = "sigmoid",
                out: Tensor | None = None, gate_up_sf_layout: int | None = None,
                down_sf_layout: int | None = None, tail: Tail | None = None, tail_out: tuple | None = None,
                rows: tuple | None = None, fc1_output_scale: float | None = None):
    """One dispatch chunk through ``praxis_b200_moe_forward``. With
    ``router_terms`` the router runs too and (out, top_idx, gate) is returned.
    ``gate_up_q/sf`` are in the interleaved kernel layout; the weight scales
    are compact or replicated (``*_sf_layout``, else told by their size).
    With ``tail`` the combine is fused into what follows the layer
    (:func:`combine_tail`) and ``(new residual, normed rows or None)`` takes
    the place of ``out`` (written into ``tail_out`` when given).
    ``rows = (T0, T1)``: x holds a lockstep pair of inputs back to back (the
    reference's forward_pair); one pass of the expert GEMMs serves both and
    every output row has the bits of its input run alone.
    ``fc1_output_scale``: the calibrated FC1 output scale (the gate/up GEMM
    writes FP4 hidden rows at this frozen global, praxis/quantization/
    nvfp4.py:327-339); None: dynamic hidden globals."""
    _need(x, "x", BF16, 2)
    t, c = x.shape
    e, c_half_f, _ = down_q.shape
    f = down_q.shape[2] * 2
    dev = x.device
    if router_terms is not None:
        k = int(top_k)
        top_idx = torch.empty(t, k, dtype=torch.int64, device=dev)
        gate = torch.empty(t, k, dtype=BF16, device=dev)
    else:
        k = top_idx.shape[1]
    st = None
    if tail is not None:
        st, residual_out, normed = _tail_struct(tail, t, c, dev, tail_out)
        out = None
    elif out is None:
        out = torch.empty_like(x)
    if gate_up_sf_layout is None:
        gate_up_sf_layout = _layout_of(gate_up_sf, gate_up_q, "gate_up_sf")
    if down_sf_layout is None:
        down_sf_layout = _layout_of(down_sf, down_q, "down_sf")
    npass, t0 = _passes(rows, t)
    lib = capi.load()
    ws_size = int(lib.praxis_b200_moe_workspace_size(t, k, e, c, f, int(router_terms is not None), npass))
    ws = torch.empty(ws_size, dtype=torch.uint8, device=dev)
    args = capi.MoeArgs(
        x=x.data_ptr(), router_weight=None if router_terms is None else router_terms.data_ptr(),
        router_splits=0 if router_terms is None else router_terms.shape[0],
        activation={"sigmoid": capi.SIGMOID, "softmax": capi.SOFTMAX}[activation],
        router_bias=None if router_bias is None else router_bias.data_ptr(),
        top_idx=top_idx.data_ptr(), gate=gate.data_ptr(),
        shared=None if shared is None else shared.data_ptr(), out=_p(out),
        gate_up_q=gate_up_q.data_ptr(), gate_up_sf=gate_up_sf.data_ptr(), gate_up_global=gate_up_global.data_ptr(),
        down_q=down_q.data_ptr(), down_sf=down_sf.data_ptr(), down_global=down_global.data_ptr(),
        gate_up_sf_layout=int(gate_up_sf_layout), down_sf_layout=int(down_sf_layout), tokens=t, dim=c, hidden=f, experts=e, top_k=k, scaling=float(scaling),
        workspace=ws.data_ptr(), workspace_size=ws_size, device=_dev(x),
        stream=torch.cuda.current_stream(dev).cuda_stream,
        tail=None if st is None else C.addressof(st), passes=npass, pass0_tokens=t0,
        fc1_output_scale=0.0 if fc1_output_scale is None else float(fc1_output_scale),
    )
    capi.check(lib.praxis_b200_moe_forward(C.byref(args)))
    res = (out,) if tail is None else (residual_out, normed)
    if router_terms is not None:
        res = res + (top_idx, gate)
    return res if len(res) > 1 else out
