"""B200-native routed-expert NVFP4 MoE hot path of Praxis-1.

Import with ``importlib.import_module("praxis-1-oss_b200")`` (the directory
name is not an identifier); the module also registers itself as
``praxis_b200`` in ``sys.modules``.

Layers:
    capi    ctypes binding of include/praxis_b200_moe.h (the C ABI)
    ops     torch-facing functions, one per reference kernel function
    bank    B200NVFP4RoutedExperts, the drop-in routed bank
    moe     B200MoEFeedForward, the MoE module
    expert_parallel  the bank sharded over GPUs with an all-to-all exchange
    pipeline  host-resident batches with copies overlapped with compute
    torch_ops  the entry points as torch operators (torch.ops.praxis_b200.*)
    graphs  CUDA-graph capture of the MoE layers (the CudaGraphPool contract)
    build   nvcc build of libpraxis_b200_moe.so (sm_100a)
"""

from __future__ import annotations

import sys

from . import build, capi, expert_parallel, graphs, ops, pipeline, torch_ops  # noqa: F401
from .bank import B200NVFP4RoutedExperts, pack_routed_experts, routed_forward_tail  # noqa: F401
from .moe import B200MoEFeedForward  # noqa: F401

sys.modules.setdefault("praxis_b200", sys.modules[__name__])

__all__ = ["B200NVFP4RoutedExperts", "B200MoEFeedForward", "pack_routed_experts", "routed_forward_tail",
           "build", "capi", "ops", "expert_parallel", "graphs", "pipeline", "torch_ops"]
