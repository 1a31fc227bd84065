"""Host-side checks that need no GPU: argument validation of the
expert-parallel helpers and the bench's algorithmic-byte bookkeeping."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest
from conftest import pkg

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("bench_module", mod)
    spec.loader.exec_module(mod)
    return mod


def test_peer_exchange_rejects_a_bad_sm_copy_fraction():
    P = pkg()
    for frac in (-0.1, 1.5):
        with pytest.raises(ValueError):
            P.expert_parallel.PeerExchange(None, "cpu", sm_copy_fraction=frac)


def test_gate_up_algorithmic_bytes_match_the_config_2_budget():
    b = _bench()
    t, k, c, f, e = 16384, 4, 3072, 1536, 64
    got = b.gemm1_bytes(t, k, c, f, e)
    weights = e * 2 * f * c // 2 + e * 2 * f * c // 16
    rows = t * k * c // 2 + t * k * c // 16 + t * k * f * 2
    assert got == weights + rows == 654_311_424
    # the measured DRAM traffic of one launch moves every byte about once:
    # within the padding rows (at most 127 per expert) of the activations
    traffic = b.GEMM1_TRAFFIC[("2", t)]
    padding = e * 127 * (c // 2 + c // 16)
    assert got * 0.95 < traffic < got + padding


def test_bench_configs_cover_the_baseline_shapes():
    b = _bench()
    for name in ("1", "2", "3", "4", "5", "ckpt"):
        cfg = b.CONFIGS[name]
        assert cfg["dim"] % 64 == 0 and cfg["hidden"] % 128 == 0 and cfg["top_k"] <= cfg["experts"]


def _noalloc_outputs(t, k, e, **override):
    import torch

    r = t * k
    mt = max(pkg().ops.padded_rows(r, e) // 128, 1)
    out = dict(order=torch.empty(r, dtype=torch.int64), inverse=torch.empty(r, dtype=torch.int64),
               tokens=torch.empty(r, dtype=torch.int64), tokens32=torch.empty(r, dtype=torch.int32),
               sorted_gate=torch.empty(r, dtype=torch.bfloat16), offsets=torch.empty(e, dtype=torch.int32),
               csr=torch.empty(e + 1, dtype=torch.int32), pcsr=torch.empty(e + 1, dtype=torch.int32),
               tiles=torch.empty(2 * mt, 4, dtype=torch.int32), num_tiles=torch.empty(2, dtype=torch.int32),
               act_global=torch.empty(e), act_amax=torch.empty(e, dtype=torch.int32))
    out.update(override)
    return out


@pytest.mark.parametrize("bad", [
    ("order", "short"), ("inverse", "dtype"), ("tokens32", "dtype"), ("sorted_gate", "short"), ("offsets", "short"),
    ("csr", "short"), ("pcsr", "dtype"), ("num_tiles", "short"), ("tiles", "short"), ("tiles", "cols"),
    ("act_global", "dtype"), ("act_amax", "short"), ("order", "strided"),
])
def test_noalloc_dispatch_outputs_are_checked_before_launch(bad):
    """Every caller-owned output of the no-allocation dispatch is checked for
    dtype, layout and size on the host; the check needs no GPU."""
    import torch

    t, k, e = 300, 4, 16
    ops = pkg().ops
    good = _noalloc_outputs(t, k, e)
    ops._check_dispatch_outputs(t, k, e, torch.device("cpu"), None, **good)  # accepted as is
    name, kind = bad
    ref = good[name]
    if kind == "short":
        ten = ref.reshape(-1)[:-1] if ref.ndim == 1 else ref[:-2]
    elif kind == "dtype":
        ten = ref.to(torch.float64 if ref.dtype != torch.float64 else torch.int32)
    elif kind == "cols":
        ten = torch.empty(ref.shape[0], 3, dtype=torch.int32)
    else:
        ten = torch.empty(2 * ref.numel(), dtype=ref.dtype)[::2]
    with pytest.raises(ValueError, match=name):
        ops._check_dispatch_outputs(t, k, e, torch.device("cpu"), None, **dict(good, **{name: ten}))
    # the public op refuses host tensors before it gets that far
    with pytest.raises(ValueError):
        ops.dispatch_noalloc(torch.zeros(t, k, dtype=torch.int64), torch.zeros(t, k, dtype=torch.bfloat16), e,
                             **good)


def test_fused_swiglu_scale_contract():
    """``set_fused_swiglu_scale`` (praxis/quantization/nvfp4.py:235-260): the
    reference's checks, None goes back to dynamic scales, and loading a
    state dict clears the runtime scale (it is not a checkpoint buffer)."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    g = torch.Generator().manual_seed(3)
    gu = (torch.randn(2, 128, 256, generator=g) * 0.02).to(torch.bfloat16)
    down = (torch.randn(2, 128, 128, generator=g) * 0.02).to(torch.bfloat16)
    state = O.pack_routed_experts(gu, down)
    bank = pkg().B200NVFP4RoutedExperts.from_packed({k: v.clone() for k, v in state.items()})
    for bad in (0.0, -1.0, float("inf"), float("nan"), True, "1"):
        with pytest.raises(ValueError):
            bank.set_fused_swiglu_scale(bad)
    bank.set_fused_swiglu_scale(2)
    assert bank._fc1_fp4_scale == 2.0
    assert "_fc1_fp4_scale" not in bank.state_dict()
    bank.load_state_dict({k: v.clone() for k, v in state.items()})
    assert bank._fc1_fp4_scale is None
    bank.set_fused_swiglu_scale(0.5)
    bank.set_fused_swiglu_scale(None)
    assert bank._fc1_fp4_scale is None


def test_graph_pool_argument_checks():
    """The capture pool's constructor rules (praxis/cuda_graphs.py:82-91)
    and its boundary types, without a GPU."""
    graphs = pkg().graphs
    with pytest.raises(ValueError):
        graphs.CudaGraphPool("cpu")
    with pytest.raises(ValueError):
        graphs.CudaGraphPool("cuda:0", warmup=0)
    with pytest.raises(ValueError):
        graphs.CudaGraphPool("cuda:0", max_graphs=0)
    tensors = []
    with pytest.raises(TypeError):
        graphs._flatten((object(),), tensors)
    import torch

    s = graphs._flatten(((torch.zeros(2), [1, torch.ones(3)]), {"k": None}), tensors)
    assert len(tensors) == 2
    rebuilt = graphs._rebuild(s, tensors)
    assert rebuilt[0][1][0] == 1 and rebuilt[1]["k"] is None and rebuilt[0][0] is tensors[0]


def test_clock_sampler_keeps_the_timed_window():
    """The bench's clock record: samples inside the timed window only (idle
    time before and after does not count), the nearest sample of each GPU
    when the window is shorter than the sampling loop, and the throttle
    reasons seen in it."""
    import datetime

    b = _bench()
    cs = b.ClockSampler([0, 1])

    def line(t, gpu, mhz, cap="Not Active"):
        ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return f"{ts}, {gpu}, {mhz}, 1965, 500.0, Not Active, Not Active, Not Active, {cap}"

    t0 = 1_800_000_000.0
    cs.t0, cs.t1 = t0, t0 + 0.05
    cs.lines = [line(t0 - 0.3, 0, 345), line(t0 + 0.02, 0, 1965), line(t0 + 0.02, 1, 1900, "Active"),
                line(t0 + 0.4, 1, 345)]
    s = cs.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == (1965 + 1900) / 2 and s["reasons"] == ["sw_power_cap"]
    cs.t1 = t0 + 0.005  # shorter than the loop: nearest sample per GPU
    cs.lines = [line(t0 - 0.3, 0, 345), line(t0 + 0.015, 0, 1965), line(t0 + 0.012, 1, 1965)]
    s = cs.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1965 and s["gpus"] == ["0", "1"]
    cs.lines = []
    assert cs.summary()["reasons"] == ["unavailable"]
