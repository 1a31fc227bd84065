"""CUDA graphs of the MoE layer's inference calls.

The capture contract of the reference's ``CudaGraphPool`` /
``enable_nvfp4_moe_cuda_graphs`` (praxis/cuda_graphs.py:66-243, :245-283):
a wrapped call is captured lazily, once per input signature (shapes,
strides, dtypes, devices and the plain values among the arguments), after
``warmup`` eager runs on the capture stream; each capture is checked byte
for byte against an eager run of the same inputs; replays copy the inputs
into the graph's own buffers and return fresh copies of its outputs;
``freeze()`` turns an unseen signature into an error; past ``max_graphs``
signatures a stage runs eagerly (counted in ``stats()``). Inference only,
one stream, no concurrent calls.

The layer's kernels take every buffer from the caller (workspaces included)
and synchronize nothing, so a whole ``B200MoEFeedForward.forward`` (router,
dispatch, quantize, GEMMs, combine, shared expert) captures into one graph;
the bank's kernel-layout weights must exist before capture
(``B200NVFP4RoutedExperts.prepare``, which the validating eager run of the
first capture performs).
"""

from __future__ import annotations

import contextlib
import logging
import threading
from collections.abc import Iterator

import torch
from torch import Tensor, nn

logger = logging.getLogger(__name__)

_PLAIN = (str, int, float, bool, type(None))


def _flatten(value, tensors: list) -> object:
    """The structure of ``value`` with its tensors replaced by their index in
    ``tensors`` (appended in traversal order)."""
    if isinstance(value, Tensor):
        tensors.append(value)
        return ("t", len(tensors) - 1)
    if isinstance(value, dict):
        return ("d", tuple((k, _flatten(v, tensors)) for k, v in value.items()))
    if isinstance(value, list | tuple):
        return ("l" if isinstance(value, list) else "u", tuple(_flatten(v, tensors) for v in value))
    if isinstance(value, _PLAIN):
        return ("v", value)
    raise TypeError(f"a CUDA graph boundary cannot hold {type(value).__name__}")


def _rebuild(structure, tensors: list):
    kind, payload = structure
    if kind == "t":
        return tensors[payload]
    if kind == "d":
        return {k: _rebuild(v, tensors) for k, v in payload}
    if kind in ("l", "u"):
        items = [_rebuild(v, tensors) for v in payload]
        return items if kind == "l" else tuple(items)
    return payload


def _key(structure, tensors: list) -> tuple:
    described = tuple((tuple(t.shape), tuple(t.stride()), t.dtype, t.device) for t in tensors)
    return (structure, described, torch.is_inference_mode_enabled(), torch.is_autocast_enabled("cuda"))


def _same_bytes(a: Tensor, b: Tensor) -> bool:
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    return torch.equal(a.contiguous().reshape(-1).view(torch.uint8), b.contiguous().reshape(-1).view(torch.uint8))


class _Entry:
    __slots__ = ("graph", "inputs", "structure", "outputs", "out_structure")

    def __init__(self, graph, inputs, structure, outputs, out_structure):
        self.graph, self.inputs, self.structure = graph, inputs, structure
        self.outputs, self.out_structure = outputs, out_structure


class CudaGraphPool:
    """Graph cache of one pipeline's wrapped calls on one device and stream
    (``praxis.cuda_graphs.CudaGraphPool``'s contract, see the module doc)."""

    def __init__(self, device, *, warmup: int = 3, max_graphs: int = 8, validate: bool = True) -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("CUDA Graphs require a CUDA device")
        if warmup < 1 or max_graphs < 1:
            raise ValueError("warmup and max_graphs must be positive")
        self.device = device if device.index is not None else torch.device("cuda", torch.cuda.current_device())
        self.warmup, self.max_graphs, self.validate = warmup, max_graphs, validate
        self.frozen = False
        self.bypass = False
        self._pool = None
        self._capture_stream = None
        self._stream = None
        self._lock = threading.Lock()
        self._stages: dict[str, dict] = {}
        self._wrapped: list[tuple[object, str, object]] = []

    @contextlib.contextmanager
    def eager(self) -> Iterator[None]:
        """Run wrapped calls eagerly (no capture) inside the block."""
        before, self.bypass = self.bypass, True
        try:
            yield
        finally:
            self.bypass = before

    def freeze(self) -> None:
        """Reject signatures not captured so far (after the warm-up phase)."""
        self.frozen = True

    def stats(self) -> dict:
        return {name: dict(s["counts"]) for name, s in self._stages.items()}

    def release(self) -> None:
        """Restore the wrapped methods and drop every graph."""
        for owner, attr, original in reversed(self._wrapped):
            if attr in getattr(owner, "__dict__", {}):
                delattr(owner, attr)  # a method of the class shows through again
            if getattr(owner, attr) != original:
                setattr(owner, attr, original)
        self._wrapped.clear()
        self._stages.clear()

    def wrap(self, owner, attr: str, name: str) -> None:
        """Route ``owner.attr`` through this pool under the stage ``name``."""
        if name in self._stages:
            raise ValueError(f"stage {name!r} is already wrapped")
        original = getattr(owner, attr)
        stage = {"cache": {}, "counts": {"captures": 0, "replays": 0, "validated": 0, "eager": 0}}
        self._stages[name] = stage

        def call(*args, **kwargs):
            if self.bypass:
                return original(*args, **kwargs)
            return self._call(name, stage, original, args, kwargs)

        call.__wrapped__ = original
        setattr(owner, attr, call)
        self._wrapped.append((owner, attr, original))

    # ------------------------------------------------------------------
    def _call(self, name, stage, original, args, kwargs):
        if torch.is_grad_enabled():
            raise RuntimeError("CUDA Graph inference requires no_grad/inference_mode")
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("CUDA Graph pipeline does not support concurrent calls")
        try:
            with torch.cuda.device(self.device):
                stream = torch.cuda.current_stream()
                if self._stream is None:
                    self._stream = stream.cuda_stream
                elif stream.cuda_stream != self._stream:
                    raise RuntimeError("CUDA Graph pipeline must run on one CUDA stream")
                tensors: list[Tensor] = []
                structure = _flatten((args, kwargs), tensors)
                if any(not t.is_cuda or t.device != self.device for t in tensors):
                    raise ValueError("CUDA Graph inputs must be CUDA tensors on the pipeline's device")
                key = _key(structure, tensors)
                entry = stage["cache"].get(key)
                if entry is None:
                    if self.frozen:
                        raise RuntimeError(f"Unwarmed CUDA Graph shape in {name}")
                    if len(stage["cache"]) >= self.max_graphs:
                        if stage["counts"]["eager"] == 0:
                            logger.warning("%s holds %d CUDA Graph shapes; new shapes run eagerly", name,
                                           self.max_graphs)
                        stage["counts"]["eager"] += 1
                        return original(*args, **kwargs)
                    entry = self._capture(name, stage, original, structure, tensors, stream)
                    stage["cache"][key] = entry
                for dst, src in zip(entry.inputs, tensors, strict=True):
                    dst.copy_(src)
                entry.graph.replay()
                stage["counts"]["replays"] += 1
                return _rebuild(entry.out_structure, [t.clone() for t in entry.outputs])
        finally:
            self._lock.release()

    def _capture(self, name, stage, original, structure, tensors, stream) -> _Entry:
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
            self._capture_stream = torch.cuda.Stream(self.device)
        static = [t.detach().clone() for t in tensors]
        s_args, s_kwargs = _rebuild(structure, static)
        expected = None
        if self.validate:
            expected_tensors: list[Tensor] = []
            _flatten(original(*s_args, **s_kwargs), expected_tensors)
            expected = [t.clone() for t in expected_tensors]
        side = self._capture_stream
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                original(*s_args, **s_kwargs)
        stream.wait_stream(side)
        torch.cuda.synchronize(self.device)
        torch.cuda.empty_cache()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._pool, stream=side):
            out = original(*s_args, **s_kwargs)
        outputs: list[Tensor] = []
        out_structure = _flatten(out, outputs)
        stage["counts"]["captures"] += 1
        if self.validate:
            graph.replay()
            if len(outputs) != len(expected) or not all(
                    _same_bytes(a, b) for a, b in zip(outputs, expected, strict=True)):
                raise RuntimeError(f"CUDA Graph changed output bits in {name}")
            stage["counts"]["validated"] += 1
        logger.info("captured %s specialization %d", name, len(stage["cache"]) + 1)
        return _Entry(graph, static, structure, outputs, out_structure)


def enable_moe_cuda_graphs(modules, device=None, *, warmup: int = 3, max_graphs: int = 8,
                           validate: bool = True) -> CudaGraphPool:
    """``enable_nvfp4_moe_cuda_graphs`` (praxis/cuda_graphs.py:245-283) for a
    set of MoE layers: every module whose routed bank is this library's (a
    ``B200MoEFeedForward``, or a reference ``MoEFeedForward`` whose
    ``routed`` was swapped for ``B200NVFP4RoutedExperts``) gets its
    ``forward`` captured per input shape, with the routing, dispatch,
    quantization, GEMMs and combine inside one graph. ``modules``: a module
    (its MoE submodules are found by name) or an iterable of (name, module).
    Frozen eval modules only; their banks are prepared here."""
    from .bank import B200NVFP4RoutedExperts

    if isinstance(modules, nn.Module):
        found = [(n, m) for n, m in modules.named_modules()
                 if isinstance(getattr(m, "routed", None), B200NVFP4RoutedExperts)]
    else:
        found = list(modules)
    if not found:
        raise ValueError("no MoE layer with a B200 NVFP4 routed bank")
    for _, m in found:
        if m.training or any(p.requires_grad for p in m.parameters()):
            raise ValueError("MoE CUDA Graphs require frozen eval MoEs")
    if device is None:
        device = found[0][1].routed.gate_up_q.device
    device = torch.device(device)
    if device.type != "cuda" or torch.cuda.get_device_capability(device) != (10, 0):
        raise ValueError("MoE CUDA Graphs require an SM100 CUDA device")
    pool = CudaGraphPool(device, warmup=warmup, max_graphs=max_graphs, validate=validate)
    for name, m in found:
        m.routed.prepare()
        pool.wrap(m, "forward", name or type(m).__name__)
    return pool
