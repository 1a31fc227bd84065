"""CUDA-graph capture of the MoE layer under the reference's capture
contract (``CudaGraphPool`` / ``enable_nvfp4_moe_cuda_graphs``,
praxis/cuda_graphs.py:66-283): lazy capture per input shape with a byte
check against eager, replays equal to eager runs, freeze and max_graphs,
one stream, inference only. Also the reference's own ``CudaGraphPool``
(from the offline install under baseline/_ref, when present) capturing this
library's module.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from conftest import assert_bytes_equal, pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    p = pkg()
    p.capi.load()
    return p


def config5_module(P, seed=5):
    """BASELINE config 5's layer (C=1024, E=32, k=2, F=2048) with a shared
    expert, bf16, frozen."""
    c, f, e, k = 1024, 2048, 32, 2
    g = torch.Generator().manual_seed(seed)
    mod = P.B200MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=4096).to(DEV)
    with torch.no_grad():
        mod.router.weight.copy_((torch.randn(e, c, generator=g) * 0.05).to(DEV))
        mod.shared.gate_up.copy_((torch.randn(c, 2 * f, generator=g) * 0.02).to(DEV))
        mod.shared.down.copy_((torch.randn(f, c, generator=g) * 0.02).to(DEV))
    mod = mod.to(torch.bfloat16).eval()
    gu = (torch.randn(e, c, 2 * f, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=g) * 0.02).to(torch.bfloat16)
    mod.set_routed_weights(gu.to(DEV), down.to(DEV))
    for prm in mod.parameters():
        prm.requires_grad_(False)
    return mod


def inputs(t, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(t, 1024, generator=g).to(torch.bfloat16).to(DEV)


def test_pool_captures_validates_and_replays(P):
    mod = config5_module(P)
    x0, x1, x2 = inputs(512, 1), inputs(512, 2), inputs(384, 3)
    with torch.no_grad():
        eager = [mod(x).clone() for x in (x0, x1, x2)]
    pool = P.graphs.enable_moe_cuda_graphs(mod, warmup=2, max_graphs=2)
    with torch.no_grad():
        assert_bytes_equal(mod(x0), eager[0])  # capture (validated against eager) + replay
        assert_bytes_equal(mod(x1), eager[1])  # replay with new data
        assert_bytes_equal(mod(x0), eager[0])
        assert_bytes_equal(mod(x2), eager[2])  # a second shape: second capture
        name = next(iter(pool.stats()))
        st = pool.stats()[name]
        assert st["captures"] == 2 and st["validated"] == 2 and st["replays"] == 4 and st["eager"] == 0
        x3 = inputs(256, 4)
        want3 = None
        with pool.eager():
            want3 = mod(x3).clone()
        assert pool.stats()[name]["captures"] == 2
        assert_bytes_equal(mod(x3), want3)  # past max_graphs: eager
        assert pool.stats()[name]["eager"] == 1
        pool.freeze()
        with pytest.raises(RuntimeError):
            mod(inputs(128, 5))
        with pytest.raises(RuntimeError):  # one stream per pipeline
            with torch.cuda.stream(torch.cuda.Stream()):
                mod(x0)
    with pytest.raises(RuntimeError):  # inference only
        mod(x0)
    pool.release()
    with torch.no_grad():
        assert_bytes_equal(mod(x1), eager[1])
    assert "forward" not in mod.__dict__


def test_graph_replay_with_router_rows(P):
    """The reference block's call (``self.ffn(normed, router_rows=rows)``)
    through the pool: keyword arguments are part of the signature."""
    mod = config5_module(P, seed=6)
    x = inputs(512, 7).reshape(2, 256, 1024)
    with torch.no_grad():
        want = mod(x, router_rows=(0, 256, 256)).clone()
        pool = P.graphs.enable_moe_cuda_graphs(mod, warmup=1)
        assert_bytes_equal(mod(x, router_rows=(0, 256, 256)), want)
        assert_bytes_equal(mod(x, router_rows=(0, 256, 256)), want)
    name = next(iter(pool.stats()))
    assert pool.stats()[name]["captures"] == 1
    pool.release()


def test_reference_pool_captures_this_module(P):
    """The reference's own CudaGraphPool (praxis/cuda_graphs.py:66-243)
    wrapping this library's module: its capture check (bytes against eager)
    passes and its replays equal eager runs."""
    if not (REF / "praxis" / "cuda_graphs.py").is_file():
        pytest.skip("the reference install (baseline/_ref) is absent")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    try:
        from praxis.cuda_graphs import CudaGraphPool
    except Exception as exc:  # a reference dependency is missing
        pytest.skip(f"reference cuda_graphs not importable: {type(exc).__name__}: {exc}")
    mod = config5_module(P, seed=8)
    mod.routed.prepare()
    x0, x1 = inputs(512, 9), inputs(512, 10)
    with torch.no_grad():
        want0, want1 = mod(x0).clone(), mod(x1).clone()
        pool = CudaGraphPool(DEV, warmup=2, max_graphs=4, validate=True)
        pool.wrap(mod, "forward", "moe")
        assert_bytes_equal(mod(x0), want0)
        assert_bytes_equal(mod(x1), want1)
    st = pool.stats()["moe"]
    assert st["captures"] == 1 and st["validated"] == 1 and st["replays"] == 2
