"""Drop-in routed NVFP4 bank for B200.

``B200NVFP4RoutedExperts`` holds the reference's packed buffers (same names,
shapes, dtypes and validation as praxis/quantization/nvfp4.py:149-227) and
implements the routed-bank protocol that ``MoEFeedForward._routed_tail``
calls (praxis/layers.py:2230-2270):

    routed_forward(x, top_idx, gate, *, scaling, chunk_size, dispatch=None)
    routed_forward_with_shared(x, top_idx, gate, *, scaling, chunk_size, shared, dispatch=None)
    routed_forward_pair(xs, top_idxs, gates, *, scaling, ...)   (praxis/layers.py:1803-1806)

so ``layer.routed = B200NVFP4RoutedExperts.from_packed(layer.routed.state_dict())``
swaps the reference's FlashInfer/Triton kernels for this library's sm_100a
kernels. The forward runs entirely on the GPU through the C ABI; there is no
CPU path.
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from typing import NamedTuple

import torch
from torch import Tensor, nn

from . import capi, ops

PACKING_RECIPE = "qat-reciprocal-v1"
_BUFFER_NAMES = frozenset(
    ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf", "down_global", "_unit_alpha")
)


class KernelWeights(NamedTuple):
    """Device copies in the kernels' layouts (built by ``prepare()``)."""

    gate_up_q: Tensor       # rows interleaved in 64-row blocks (32 gate, 32 up)
    gate_up_sf: Tensor      # same row order, compact (reference) scale layout
    down_sf: Tensor         # the bank's own compact scales of down_q
    gate_up_sf_layout: int  # capi.SF_COMPACT
    down_sf_layout: int     # capi.SF_COMPACT


def _validate(state: Mapping[str, Tensor], require_cpu: bool = True) -> tuple[int, int, int]:
    """praxis/quantization/nvfp4.py:163-213 (``require_cpu``: the reference's
    rule that reconstruction starts from CPU buffers; this library's own
    packers build banks from device buffers)."""
    if not isinstance(state, Mapping) or set(state) != _BUFFER_NAMES:
        raise ValueError("Unexpected NVFP4 packed buffer keys")
    if any(
        not isinstance(v, Tensor)
        or (require_cpu and v.device.type != "cpu")
        or v.layout != torch.strided
        or not v.is_contiguous()
        or v.requires_grad
        for v in state.values()
    ):
        raise ValueError("Reconstruction requires contiguous detached CPU buffers" if require_cpu else
                         "Reconstruction requires contiguous detached buffers")
    gu = state["gate_up_q"]
    if gu.ndim != 3:
        raise ValueError("Expected grouped gate/up packed matrix")
    e, n, k2 = gu.shape
    c, h = k2 * 2, n // 2
    if e <= 0 or c <= 0 or h <= 0 or n % 2 or c % 128 or h % 128:
        raise ValueError("Invalid grouped NVFP4 dimensions")
    expected = {
        "gate_up_q": ((e, 2 * h, c // 2), torch.uint8),
        "gate_up_sf": ((e, 2 * h, c // 16), torch.uint8),
        "gate_up_global": ((e,), torch.float32),
        "down_q": ((e, c, h // 2), torch.uint8),
        "down_sf": ((e, c, h // 16), torch.uint8),
        "down_global": ((e,), torch.float32),
        "_unit_alpha": ((e,), torch.float32),
    }
    for name, (shape, dtype) in expected.items():
        value = state[name]
        if tuple(value.shape) != shape or value.dtype != dtype:
            raise ValueError(f"Invalid NVFP4 buffer shape/dtype: {name}")
        if name.endswith("_global"):
            if not torch.isfinite(value).all().item() or not (value > 0).all().item():
                raise ValueError(f"Invalid positive global scales: {name}")
        if name.endswith("_sf"):
            decoded = value.view(torch.float8_e4m3fn).float()
            if not torch.isfinite(decoded).all().item() or (decoded < 0).any().item():
                raise ValueError(f"Invalid E4M3 block scales: {name}")
    if not torch.equal(state["_unit_alpha"].cpu(), torch.ones(e, dtype=torch.float32)):
        raise ValueError("NVFP4 GEMM alpha must be one")
    return e, c, h


class B200NVFP4RoutedExperts(nn.Module):
    """Packed NVFP4 routed experts executed by the sm_100a kernels.

    Device moves are supported; dtype casts, training and gradients are not
    (praxis/quantization/nvfp4.py:229-290). The fused SwiGLU GEMM reads the
    gate/up weight in 64-row gate/up blocks: that copy is built on the device
    by ``prepare()`` (called by the first forward; call it before capturing a
    CUDA graph) and is not part of the state dict.
    """

    format = "nvfp4"
    backend = "b200_sm100a_tcgen05_nvfp4"
    # The routing kernels here build their own dispatch metadata (tile tables,
    # padded offsets, global scales) in the same launch sequence as the
    # experts, so a ``router_fused.Routing`` from the caller is not needed and
    # ``MoEFeedForward._routed_tail`` (praxis/layers.py:2245-2250) passes none.
    ACCEPTS_DISPATCH = False

    def __init__(self, state: Mapping[str, Tensor], *, _device_state: bool = False) -> None:
        super().__init__()
        e, c, h = _validate(state, require_cpu=not _device_state)
        self.num_experts, self.in_features, self.hidden_features = e, c, h
        for name in sorted(_BUFFER_NAMES):
            self.register_buffer(name, state[name].detach())
        self._kernel: KernelWeights | None = None
        self._fc1_fp4_scale: float | None = None
        super().train(False)

    @classmethod
    def from_packed(cls, state: Mapping[str, Tensor]) -> B200NVFP4RoutedExperts:
        """The reference's reconstruction (praxis/quantization/nvfp4.py:149-227):
        contiguous detached CPU buffers; move the bank with ``.to(device)``."""
        return cls(state)

    @classmethod
    def from_device_state(cls, state: Mapping[str, Tensor]) -> B200NVFP4RoutedExperts:
        """The same validation for buffers already on a device (this library's
        GPU packer and the expert-parallel shards), without a host copy."""
        return cls(state, _device_state=True)

    def train(self, mode: bool = True) -> B200NVFP4RoutedExperts:
        if mode:
            raise RuntimeError("NVFP4 routed experts support inference only")
        super().train(False)
        return self

    def _apply(self, fn, recurse: bool = True) -> B200NVFP4RoutedExperts:
        moved = {name: fn(value) for name, value in self._buffers.items()}
        for name, value in self._buffers.items():
            other = moved[name]
            if other.dtype != value.dtype or other.shape != value.shape:
                raise TypeError("NVFP4 buffers support device moves, not dtype/shape casts")
        self._buffers.update(moved)
        self._kernel = None
        return self

    def _load_from_state_dict(self, *args, **kwargs):
        self._kernel = None
        self._fc1_fp4_scale = None
        super()._load_from_state_dict(*args, **kwargs)

    def set_fused_swiglu_scale(self, scale: float | None) -> None:
        """Set a calibrated FC1 output scale, or go back to dynamic hidden
        scales with None (praxis/quantization/nvfp4.py:235-260, the same
        checks): the gate/up GEMM then writes FP4 hidden rows at this frozen
        global, which is also the down GEMM's activation global. This changes
        output bits (by design: the reference's calibrated path does too).
        The scale is runtime state, not a checkpoint buffer; loading a state
        dict clears it."""
        if scale is not None and (
            isinstance(scale, bool)
            or not isinstance(scale, float | int)
            or not math.isfinite(scale)
            or scale <= 0
        ):
            raise ValueError("FC1 output scale must be finite and positive")
        self._fc1_fp4_scale = None if scale is None else float(scale)

    def prepare(self) -> None:
        """Build the kernel-layout gate/up weights on the buffers' device:
        rows interleaved for the fused SwiGLU epilogue (their scales follow
        the rows, still in the reference's compact layout; the down GEMM reads
        the bank's own buffers). The packed buffers stay in the reference's
        row order."""
        if self.gate_up_q.device.type != "cuda":
            raise RuntimeError("prepare() needs the bank on a CUDA device")
        gu_q, gu_sf = ops.interleave_gate_up(self.gate_up_q, self.gate_up_sf)
        self._kernel = KernelWeights(gu_q, gu_sf, self.down_sf, capi.SF_COMPACT, capi.SF_COMPACT)

    def kernel_weights(self) -> KernelWeights:
        """The kernel-layout weights (prepare() on first use)."""
        if self._kernel is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Call prepare() on the NVFP4 bank before CUDA Graph capture")
            self.prepare()
        return self._kernel

    # -- the routed-bank protocol -------------------------------------------
    def routed_forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float, chunk_size: int,
                       dispatch=None) -> Tensor:
        """The scaled routed sum with the bf16 output boundary."""
        return self._routed_forward(x, top_idx, gate, scaling=scaling, chunk_size=chunk_size)

    def routed_forward_with_shared(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float,
                                   chunk_size: int, shared: Tensor, dispatch=None) -> Tensor:
        """Adds the shared expert after rounding the routed sum to bf16
        (praxis/quantization/nvfp4.py:505-544, same fallback rule)."""
        if (
            shared.shape != x.shape
            or shared.dtype != x.dtype
            or shared.device != x.device
            or not shared.is_contiguous()
            or (torch.is_grad_enabled() and shared.requires_grad)
        ):
            return self.routed_forward(x, top_idx, gate, scaling=scaling, chunk_size=chunk_size) + shared
        return self._routed_forward(x, top_idx, gate, scaling=scaling, chunk_size=chunk_size, shared=shared)

    def routed_forward_pair(self, xs, top_idxs, gates, *, scaling: float, shared=None, tail: ops.Tail | None = None,
                            dispatch=None) -> list:
        """``[self.routed_forward(x, i, g, scaling=scaling, chunk_size=len(x)) for ...]``
        of two inputs (the guided and unguided passes of a CFG pair) in one
        paired dispatch, each input one dispatch chunk
        (praxis/quantization/nvfp4.py:467-488, the paired dispatch of
        praxis/kernels/nvfp4_pair.py:1-20): the rows of expert e are grouped
        per input, each group with its own activation and hidden global
        scales, so every output has the bits of its input run alone, while
        the expert GEMMs run once over both inputs' rows. ``shared``: the two
        shared-expert outputs, added after rounding as by
        ``routed_forward_with_shared``. ``tail``: the fused tail over both
        inputs' rows back to back (:func:`routed_forward_tail`); the result
        is then ``[(new residual, normed or None)]`` per input. ``dispatch``
        is accepted for the reference's signature and not needed (the
        dispatch runs inside the fused call). Inputs that sit back to back
        in one buffer are used in place; others are copied together."""
        del dispatch
        xs, top_idxs, gates = list(xs), list(top_idxs), list(gates)
        if not (len(xs) == len(top_idxs) == len(gates) == 2):
            raise ValueError("routed_forward_pair takes two inputs")
        t0, t1 = xs[0].shape[0], xs[1].shape[0]
        for x, i, g in zip(xs, top_idxs, gates, strict=True):
            self._check(x, i, g, scaling, max(1, x.shape[0]))
        if top_idxs[0].shape[1] != top_idxs[1].shape[1] or xs[0].device != xs[1].device:
            raise ValueError("the two inputs must share top-k and device")
        x = _adjacent(xs)
        top_idx = _adjacent(top_idxs)
        gate = _adjacent(gates)
        self._check(x, top_idx, gate, scaling, max(1, t0 + t1))
        sh = None
        if shared is not None:
            shared = list(shared)
            if len(shared) != 2 or any(s.shape != xi.shape or s.dtype != xi.dtype or s.device != xi.device
                                       for s, xi in zip(shared, xs, strict=True)):
                raise ValueError("Expected two BF16 shared-expert outputs shaped like the inputs")
            sh = _adjacent(shared)
        kw = self.kernel_weights()
        common = dict(gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout, rows=(t0, t1),
                      fc1_output_scale=self._fc1_fp4_scale)
        if tail is not None:
            xo, h = ops.moe_forward(
                x, top_idx, gate, kw.gate_up_q, kw.gate_up_sf, self.gate_up_global, self.down_q, kw.down_sf,
                self.down_global, float(scaling), sh, tail=tail, **common)
            return [(xo[:t0], None if h is None else h[:t0]), (xo[t0:], None if h is None else h[t0:])]
        out = ops.moe_forward(
            x, top_idx, gate, kw.gate_up_q, kw.gate_up_sf, self.gate_up_global, self.down_q, kw.down_sf,
            self.down_global, float(scaling), sh, **common)
        return [out[:t0], out[t0:]]

    def forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float, chunk_size: int) -> Tensor:
        return self.routed_forward(x, top_idx, gate, scaling=scaling, chunk_size=chunk_size)

    def _check(self, x, top_idx, gate, scaling, chunk_size) -> None:
        """praxis/quantization/nvfp4.py:630-682, the same errors."""
        if self.training or (torch.is_grad_enabled() and (x.requires_grad or gate.requires_grad)):
            raise RuntimeError("NVFP4 routed experts support inference only")
        if (
            x.ndim != 2
            or x.shape[1] != self.in_features
            or x.dtype != torch.bfloat16
            or not x.is_contiguous()
            or x.device.type != "cuda"
        ):
            raise ValueError("Expected contiguous CUDA BF16 routed activations")
        if (
            top_idx.ndim != 2
            or top_idx.shape[0] != x.shape[0]
            or not 1 <= top_idx.shape[1] <= min(8, self.num_experts)
            or top_idx.dtype != torch.int64
            or top_idx.device != x.device
            or not top_idx.is_contiguous()
        ):
            raise ValueError("Expected contiguous CUDA int64 expert indices, top-k <= 8")
        if gate.shape != top_idx.shape or gate.dtype != torch.bfloat16 or gate.device != x.device or not gate.is_contiguous():
            raise ValueError("Expected contiguous CUDA BF16 gate weights")
        if any(value.device != x.device for value in self.buffers()):
            raise ValueError("Packed expert buffers and inputs must share a device")
        if type(chunk_size) is not int or chunk_size <= 0:
            raise ValueError("NVFP4 inference requires a positive dispatch chunk size")
        if isinstance(scaling, bool) or not isinstance(scaling, float | int) or not math.isfinite(scaling):
            raise ValueError("Routed scaling must be finite")
        top_k = top_idx.shape[1]
        # the reference's bound (praxis/quantization/nvfp4.py:677-682), kept so
        # that the same calls are rejected; the kernels here index with 64 bits
        if (min(chunk_size, x.shape[0]) * top_k + 127 * self.num_experts) * max(
            self.in_features, 2 * self.hidden_features
        ) >= 2**31:
            raise ValueError("Routed chunk exceeds NVFP4 kernel indexing bounds")

    def _routed_forward(self, x: Tensor, top_idx: Tensor, gate: Tensor, *, scaling: float, chunk_size: int,
                        shared: Tensor | None = None) -> Tensor:
        """The dispatch-chunk loop of praxis/quantization/nvfp4.py:683-747;
        each chunk is one praxis_b200_moe_forward call."""
        self._check(x, top_idx, gate, scaling, chunk_size)
        kw = self.kernel_weights()
        out = torch.empty_like(x)
        for start in range(0, x.shape[0], chunk_size):
            end = min(start + chunk_size, x.shape[0])
            ops.moe_forward(
                x[start:end], top_idx[start:end], gate[start:end], kw.gate_up_q, kw.gate_up_sf, self.gate_up_global,
                self.down_q, kw.down_sf, self.down_global, float(scaling),
                None if shared is None else shared[start:end], out=out[start:end],
                gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout,
                fc1_output_scale=self._fc1_fp4_scale,
            )
        return out


def _adjacent(parts: list) -> Tensor:
    """The rows of ``parts`` (contiguous 2-D tensors of one width) back to
    back: a view when they already sit so in one buffer (the reference's
    PAIR_BUFFER writes the paired inputs into adjacent slices), else a copy."""
    a, b = parts
    if (
        a.is_contiguous() and b.is_contiguous() and a.dtype == b.dtype and a.shape[1:] == b.shape[1:]
        and a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr()
        and b.data_ptr() == a.data_ptr() + a.numel() * a.element_size()
    ):
        return torch.as_strided(a, (a.shape[0] + b.shape[0],) + tuple(a.shape[1:]), a.stride())
    return torch.cat([a, b])


def routed_forward_tail(bank: B200NVFP4RoutedExperts, x: Tensor, top_idx: Tensor, gate: Tensor, *,
                        scaling: float, chunk_size: int, tail: ops.Tail, shared: Tensor | None = None
                        ) -> tuple[Tensor, Tensor | None]:
    """``routed_forward_with_shared`` whose output goes straight into what
    follows the layer (the reference's MOE_TAIL_NORM, praxis/layers.py:429-441,
    praxis/kernels/moe_tail_triton.py:329-445): the residual add of
    ``tail.residual``, then, when ``tail.norm_weight`` is set, the next block's
    RMSNorm (with its modulation when ``tail.mod`` is set). Returns ``(new
    residual, normed rows or None)`` with the eager bits; the routed output
    itself is never stored. Each dispatch chunk fuses its own rows."""
    bank._check(x, top_idx, gate, scaling, chunk_size)
    r = tail.residual
    if r.shape != x.shape or r.dtype != torch.bfloat16 or not r.is_contiguous() or r.device != x.device:
        raise ValueError("Expected a contiguous BF16 residual shaped like the routed activations")
    if shared is not None and (shared.shape != x.shape or shared.dtype != x.dtype or not shared.is_contiguous()):
        raise ValueError("Expected a contiguous BF16 shared-expert output shaped like the activations")
    kw = bank.kernel_weights()
    residual_out = torch.empty_like(x)
    normed = None if tail.norm_weight is None else torch.empty_like(x)
    for start in range(0, x.shape[0], chunk_size):
        end = min(start + chunk_size, x.shape[0])
        ops.moe_forward(
            x[start:end], top_idx[start:end], gate[start:end], kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global,
            bank.down_q, kw.down_sf, bank.down_global, float(scaling), None if shared is None else shared[start:end],
            gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout, tail=tail.chunk(start, end),
            tail_out=(residual_out[start:end], None if normed is None else normed[start:end]),
            fc1_output_scale=bank._fc1_fp4_scale)
    return residual_out, normed


def pack_routed_experts(gate_up_weight: Tensor, down_weight: Tensor, *, keep_on_device: bool = False
                        ) -> B200NVFP4RoutedExperts:
    """Packs expert-first bf16 banks [E,C,2H] / [E,H,C] on the GPU with the
    reference recipe (praxis/quantization/nvfp4.py:104-146, same bytes).
    CPU banks are copied to the current CUDA device for packing; the packed
    buffers come back to the CPU (as the reference returns them) unless
    ``keep_on_device``."""
    for weight in (gate_up_weight, down_weight):
        if (
            not isinstance(weight, Tensor)
            or weight.ndim != 3
            or weight.dtype != torch.bfloat16
            or weight.layout != torch.strided
            or weight.device.type == "meta"
        ):
            raise ValueError("Packing requires real BF16 expert-first banks")
    e, c, doubled = gate_up_weight.shape
    h = doubled // 2
    if e <= 0 or c <= 0 or h <= 0 or doubled % 2 or c % 128 or h % 128 or tuple(down_weight.shape) != (e, h, c):
        raise ValueError("Inconsistent routed banks; C and H must be multiples of 128")
    if not torch.cuda.is_available():
        raise RuntimeError("B200 NVFP4 packing runs on the GPU")
    dev = gate_up_weight.device if gate_up_weight.device.type == "cuda" else torch.device("cuda")
    state = {}
    with torch.no_grad():
        for name, weight in (("gate_up", gate_up_weight), ("down", down_weight)):
            q, sf, g = ops.pack_weights(weight.to(dev).contiguous())
            state[name + "_q"], state[name + "_sf"], state[name + "_global"] = q, sf, g
        state["_unit_alpha"] = torch.ones(e, dtype=torch.float32, device=dev)
    if not keep_on_device:
        return B200NVFP4RoutedExperts.from_packed({k: v.cpu() for k, v in state.items()})
    return B200NVFP4RoutedExperts.from_device_state(state)
