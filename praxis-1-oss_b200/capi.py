"""ctypes binding of include/praxis_b200_moe.h.

This is the reference-side stub a Python caller binds: plain pointers,
sizes, a device ordinal and a ``cudaStream_t``. ``load()`` raises when the
library is missing or cannot be loaded; nothing falls back to another path.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from . import build as _build

_LOCK = threading.Lock()
_LIB: C.CDLL | None = None

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
SZ = C.c_size_t

ABI_VERSION = 4  # PRAXIS_B200_ABI_VERSION of include/praxis_b200_moe.h

OK, EINVAL, ECUDA, EUNSUPPORTED = 0, 1, 2, 3
SIGMOID, SOFTMAX = 0, 1
EPI_PLAIN, EPI_SWIGLU, EPI_RESCALE = 0, 1, 2
SF_COMPACT, SF_REPLICATED = 0, 1


class MoeArgs(C.Structure):
    """``praxis_b200_moe_args``."""

    _fields_ = [
        ("x", P),
        ("router_weight", P),
        ("router_splits", I32),
        ("activation", I32),
        ("router_bias", P),
        ("top_idx", P),
        ("gate", P),
        ("shared", P),
        ("out", P),
        ("gate_up_q", P),
        ("gate_up_sf", P),
        ("gate_up_global", P),
        ("down_q", P),
        ("down_sf", P),
        ("down_global", P),
        ("gate_up_sf_layout", I32),
        ("down_sf_layout", I32),
        ("tokens", I64),
        ("dim", I32),
        ("hidden", I32),
        ("experts", I32),
        ("top_k", I32),
        ("scaling", F32),
        ("workspace", P),
        ("workspace_size", SZ),
        ("device", C.c_int),
        ("stream", P),
        ("tail", P),
        ("passes", I32),
        ("pass0_tokens", I64),
        ("fc1_output_scale", F32),
    ]


class TailArgs(C.Structure):
    """``praxis_b200_tail``."""

    _fields_ = [
        ("residual", P),
        ("residual_out", P),
        ("norm_weight", P),
        ("normed_out", P),
        ("eps", F32),
        ("norm_scale", F32),
        ("mod", P),
        ("mod_fma", I32),
        ("mod_geom", I64 * 6),
        ("mod_row0", I64),
    ]


class ExpertArgs(C.Structure):
    """``praxis_b200_expert_args``."""

    _fields_ = [
        ("q", P),
        ("sf", P),
        ("rows", I64),
        ("counts", P),
        ("starts", P),
        ("act_global", P),
        ("segments", I32),
        ("gate_up_q", P),
        ("gate_up_sf", P),
        ("gate_up_global", P),
        ("down_q", P),
        ("down_sf", P),
        ("down_global", P),
        ("gate_up_sf_layout", I32),
        ("down_sf_layout", I32),
        ("dim", I32),
        ("hidden", I32),
        ("experts", I32),
        ("sm_limit", I32),
        ("rows_out", P),
        ("workspace", P),
        ("workspace_size", SZ),
        ("device", C.c_int),
        ("stream", P),
        ("hidden_q", P),
        ("hidden_sf", P),
        ("hidden_amax", P),
    ]


# name -> (restype, argtypes); the order and types follow the header.
SIGNATURES: dict[str, tuple] = {
    "praxis_b200_abi_version": (C.c_int, []),
    "praxis_b200_last_error": (C.c_char_p, []),
    "praxis_b200_device_check": (C.c_int, [C.c_int]),
    "praxis_b200_device_error": (C.c_int, [C.c_int, C.POINTER(C.c_uint32)]),
    "praxis_b200_padded_rows": (I64, [I64, I32]),
    "praxis_b200_router_logits": (C.c_int, [P, P, I32, I64, I32, I32, P, P, C.c_int, P]),
    "praxis_b200_route": (C.c_int, [P, P, I64, I32, I32, I32, P, P, C.c_int, P]),
    "praxis_b200_row_amax": (C.c_int, [P, I64, I32, P, C.c_int, P]),
    "praxis_b200_dispatch_workspace_size": (SZ, [I64, I32, I32]),
    "praxis_b200_dispatch_passes_workspace_size": (SZ, [I64, I32, I32, I32]),
    "praxis_b200_dispatch_passes": (
        C.c_int,
        [P, P, P, I64, I32, I32, I32, I64, P, SZ, P, P, P, P, P, P, P, P, P, I32, P, P, P, C.c_int, P],
    ),
    "praxis_b200_dispatch": (
        C.c_int,
        [P, P, P, I64, I32, I32, P, SZ, P, P, P, P, P, P, P, P, P, I32, P, P, P, C.c_int, P],
    ),
    "praxis_b200_quantize_gather": (
        C.c_int,
        [P, I64, I32, P, P, P, P, P, P, I32, I32, P, P, I32, P, P, I32, C.c_int, P],
    ),
    "praxis_b200_quantize_rows": (C.c_int, [P, I32, P, P, I32, P, P, P, P, I32, C.c_int, P]),
    "praxis_b200_grouped_gemm": (
        C.c_int,
        [P, P, P, P, P, P, I32, I64, I32, I32, I32, I32, P, P, P, P, P, I32, C.c_int, P],
    ),
    "praxis_b200_replicate_scales": (C.c_int, [P, I64, I32, I32, P, C.c_int, P]),
    "praxis_b200_gemm_swiglu_fp4": (
        C.c_int,
        [P, P, P, P, P, P, I32, I64, I32, I32, I32, P, P, P, F32, P, P, C.c_int, P],
    ),
    "praxis_b200_rescale_swiglu": (C.c_int, [P, I64, I32, P, I32, P, P, P, P, I32, C.c_int, P]),
    "praxis_b200_combine": (
        C.c_int,
        [P, I32, P, P, P, P, P, P, P, P, I32, F32, P, P, I64, I32, I32, C.c_int, P],
    ),
    "praxis_b200_combine_tail": (
        C.c_int,
        [P, I32, P, P, P, P, P, P, P, P, I32, F32, P, C.POINTER(TailArgs), I64, I32, I32, C.c_int, P],
    ),
    "praxis_b200_pack_weights": (C.c_int, [P, I32, I32, I32, P, P, P, P, C.c_int, P]),
    "praxis_b200_interleave_gate_up": (C.c_int, [P, P, I32, I32, I32, P, P, C.c_int, P]),
    "praxis_b200_moe_workspace_size": (SZ, [I64, I32, I32, I32, I32, I32, I32]),
    "praxis_b200_moe_forward": (C.c_int, [C.POINTER(MoeArgs)]),
    "praxis_b200_expert_workspace_size": (SZ, [I64, I32, I32, I32]),
    "praxis_b200_expert_forward": (C.c_int, [C.POINTER(ExpertArgs)]),
    "praxis_b200_dispatch_noalloc": (
        C.c_int,
        [P, P, P, I64, I32, I32, P, P, P, P, P, P, P, P, P, I32, P, P, P, C.c_int, P],
    ),
    "praxis_b200_ipc_alloc": (C.c_int, [C.c_size_t, C.c_int, C.POINTER(C.c_void_p)]),
    "praxis_b200_ipc_free": (C.c_int, [P, C.c_int]),
    "praxis_b200_ipc_handle": (C.c_int, [P, C.c_int, P]),
    "praxis_b200_ipc_open": (C.c_int, [P, C.c_int, C.POINTER(C.c_void_p)]),
    "praxis_b200_ipc_close": (C.c_int, [P, C.c_int]),
    "praxis_b200_copy_async": (C.c_int, [P, P, C.c_size_t, C.c_int, P]),
    "praxis_b200_wait_value": (C.c_int, [P, I32, I64, C.c_int, P]),
    "praxis_b200_sm_copy": (C.c_int, [P, P, C.c_size_t, C.c_int, C.c_int, P]),
}

IPC_HANDLE_BYTES = 64


class PraxisB200Error(RuntimeError):
    """A non-zero status from the C library."""


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = False) -> C.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not path.exists():
            if not build_if_missing:
                raise PraxisB200Error(
                    f"{path} is missing: build it first (python {Path(_build.__file__).name} or "
                    "__graft_entry__.build())"
                )
            _build.build()
        lib = C.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.praxis_b200_abi_version() != ABI_VERSION:
            raise PraxisB200Error("ABI version mismatch")
        _LIB = lib
        return lib


def check(status: int) -> None:
    if status != OK:
        msg = load().praxis_b200_last_error().decode(errors="replace")
        if status == EINVAL:
            raise ValueError(msg)
        raise PraxisB200Error(f"praxis_b200 status {status}: {msg}")


def device_error(device: int) -> int:
    """Read (and clear) the device error word; synchronizes the device."""
    code = C.c_uint32(0)
    check(load().praxis_b200_device_error(device, C.byref(code)))
    return int(code.value)
