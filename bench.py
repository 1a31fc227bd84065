"""Benchmark of one routed-expert NVFP4 MoE layer forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2]

One step = one MoE layer forward of the configured shape: router logits
(tensor cores) + sigmoid/top-k/renorm, dispatch, NVFP4 gather-quantize,
gate/up grouped GEMM with fused SwiGLU, hidden quantize, down grouped GEMM
with fused rescale, weighted combine. Metric: routed-expert tokens/s per MoE
layer (whole job: tokens of all ranks / max-over-ranks step time).

Inputs are synthetic and seeded (x ~ N(0,1) bf16, expert weights ~ N(0,0.02)
packed to NVFP4 on the GPU, router weight ~ N(0, 1/C) so the logits are
~N(0,1)); x (100 MB) plus the packed weights (510 MB) exceed the 126 MB L2,
so no L2 flush is needed between steps.

N > 1 (torchrun): every rank runs the full layer on its own tokens (expert
weights replicated): weak scaling, no data-path collective.

--impl reference: the CPU port of the reference path (the oracle's NVFP4
chain with weights dequantised once, float32 GEMMs, all host threads) on a
bounded sample of tokens of the same layer; rank 0 only.
"""

from __future__ import annotations

import argparse
import contextlib
import importlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: tokens, dim, experts, top_k, hidden, skew
    "1": dict(tokens=256, dim=512, experts=8, top_k=2, hidden=1024, skew=False),
    "2": dict(tokens=16384, dim=3072, experts=64, top_k=4, hidden=1536, skew=False),
    "3": dict(tokens=16384, dim=3072, experts=64, top_k=4, hidden=1536, skew=True),
    # expert parallel over N GPUs: tokens per rank (weak scaling)
    "4": dict(tokens=65536, dim=3072, experts=64, top_k=4, hidden=1536, skew=False),
    "5": dict(tokens=512, dim=1024, experts=32, top_k=2, hidden=2048, skew=False),
    "ckpt": dict(tokens=16384, dim=3072, experts=128, top_k=8, hidden=1280, skew=False),
}
METRIC = "routed-expert tokens/sec per MoE layer"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one gate/up GEMM
# launch, from one single-pass ncu capture of the full-size bench workload:
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#       --clock-control none -k regex:gemm_nvfp4_pair -s 5 -c 5 python bench.py --steps 2 --warmup 3
# (read 616,229,120 + write 194,864,384 at config 2, 16384 tokens).
GEMM1_TRAFFIC = {("2", 16384): 616229120 + 194864384}


def gemm1_bytes(t, k, c, f, e):
    """Algorithmic bytes of the gate/up GEMM: every expert's packed weights and
    compact ue4m3 scales once, the routed rows' packed activations and compact
    scales once, and the bf16 hidden rows written once (padding rows excluded)."""
    rows = t * k
    return e * 2 * f * c // 2 + e * 2 * f * c // 16 + rows * c // 2 + rows * c // 16 + rows * f * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default=None, choices=sorted(CONFIGS),
                    help="default: 2 on one GPU, 4 (expert parallel) on several")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--ep-chunks", type=int, default=None,
                    help="expert groups per source in the expert-parallel exchange (N > 1)")
    ap.add_argument("--copy-streams", type=int, default=4, help="copy streams of the peer exchange (N > 1)")
    ap.add_argument("--sm-copy-fraction", type=float, default=0.0,
                    help="share of the peer exchange's bytes moved by a copy kernel on 16 SMs (N > 1)")
    ap.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel row exchange (N > 1): copy engines into IPC-mapped peer buffers, or NCCL")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override the config's token count (small profiling cases)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_inputs(cfg, seed, device):
    import torch

    t, c, e, k, f = cfg["tokens"], cfg["dim"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    router = torch.randn(e, c, generator=g) * (1.0 / c) ** 0.5
    bias = torch.zeros(e)
    if cfg["skew"]:
        # Zipf(s=1.2) expert popularity through the routing bias
        ranks = torch.randperm(e, generator=torch.Generator().manual_seed(0)).float() + 1
        bias = -1.2 * torch.log(ranks) * 0.08
    gw = torch.Generator(device=device).manual_seed(seed + 1)
    gu = (torch.randn(e, c, 2 * f, generator=gw, device=device) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=gw, device=device) * 0.02).to(torch.bfloat16)
    return x, router, bias, gu, down


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region (index
    None: every GPU of the node from one process)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", *(["-i", str(self.index)] if self.index is not None else []),
                 f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        else:
            self.lines = []

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_port_forward(prep, x, router, bias, cfg):
    """The oracle's NVFP4 chain with dequantised fp32 weights (CPU port)."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    e, k, c, f = cfg["experts"], cfg["top_k"], cfg["dim"], cfg["hidden"]
    logits = O.router_logits(x, router)
    top, gate = O.route(logits, bias, k)
    order, inverse, tokens, _sg, offsets, csr = O.dispatch(top, gate, e)
    pcsr = O.pad_csr(csr)
    m = tokens.numel()
    prows = O.padded_rows(m, e)
    ag = O.segment_global_scales(O.row_amax(x), csr, tokens)
    aq, asf = O.quantize_activations(x, csr, pcsr, prows, ag, row_indices=tokens)
    a = O.dequant_rows(aq, asf, c)
    gu = torch.zeros(prows, 2 * f, dtype=torch.bfloat16)
    b = pcsr.tolist()
    for ex in range(e):
        if b[ex + 1] > b[ex]:
            gu[b[ex]:b[ex + 1]] = (a[b[ex]:b[ex + 1]] @ prep["gu"][ex].t()).to(torch.bfloat16)
    hidden, rowmax = O.rescale_swiglu_maximum(gu, pcsr, ag, prep["gug"])
    hg = O.segment_global_scales(rowmax, pcsr)
    hq, hsf = O.quantize_activations(hidden, pcsr, pcsr, prows, hg)
    h = O.dequant_rows(hq, hsf, f)
    raw = torch.zeros(prows, c, dtype=torch.bfloat16)
    for ex in range(e):
        if b[ex + 1] > b[ex]:
            raw[b[ex]:b[ex + 1]] = (h[b[ex]:b[ex + 1]] @ prep["dn"][ex].t()).to(torch.bfloat16)
    return O.rescale_combine(raw, inverse, top, gate, csr, pcsr, hg, prep["dng"], 2.5)


def cpu_baseline(cfg, budget_s=12.0, sample_tokens=None):
    """Time the CPU port on a bounded token sample of the layer; tokens/s."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    c, e, f = cfg["dim"], cfg["experts"], cfg["hidden"]
    t = sample_tokens or min(cfg["tokens"], 1024)
    sub = dict(cfg, tokens=t)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    router = torch.randn(e, c, generator=g) * (1.0 / c) ** 0.5
    bias = torch.zeros(e)
    # packed weights -> dequantised once (load-time work, not timed)
    gw = torch.Generator().manual_seed(8)
    prep = {"gu": [], "dn": [], "gug": torch.empty(e), "dng": torch.empty(e)}
    for ex in range(e):
        w1 = (torch.randn(2 * f, c, generator=gw) * 0.02).to(torch.bfloat16)
        q, sf, gg = O.pack_matrix(w1)
        prep["gu"].append(O.dequant_matrix(q, sf, 2 * f, c))
        prep["gug"][ex] = gg
        w2 = (torch.randn(c, f, generator=gw) * 0.02).to(torch.bfloat16)
        q, sf, gg = O.pack_matrix(w2)
        prep["dn"].append(O.dequant_matrix(q, sf, c, f))
        prep["dng"][ex] = gg
    times = []
    start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        cpu_port_forward(prep, x, router, bias, sub)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget_s or len(times) >= 5:
            break
    med = statistics.median(times)
    return {"value": t / med, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{t} tokens of the layer (C={c}, E={e}, k={cfg['top_k']}, F={f}), median of {len(times)} "
                      f"forwards, weights dequantised once outside the timing"}


def run_reference(args, cfg):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cb = cpu_baseline(cfg, budget_s=max(5.0, 2.0 * args.steps))
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"config {args.config}", **cfg}, "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(args, cfg):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module("praxis-1-oss_b200")
    pkg.capi.load()
    peaks = {}
    pfile = ROOT / "MEASURED_PEAKS.json"
    if pfile.exists():
        peaks = json.loads(pfile.read_text())

    t, c, e, k, f = cfg["tokens"], cfg["dim"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    x_cpu, router, bias, gu, down = make_inputs(cfg, 1000 + rank, dev)
    mod = pkg.B200MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=t, shared_expert=False).to(dev)
    with torch.no_grad():
        mod.router.weight.copy_(router.to(dev))
        mod.expert_bias.copy_(bias.to(dev))
    mod.set_routed_weights(gu, down)
    del gu, down
    bank = mod.routed
    bank.prepare()
    terms = mod.router_terms()
    kw = bank.kernel_weights()
    x = x_cpu.to(dev)
    out = torch.empty_like(x)
    ops = pkg.ops

    def layer(xin, yout):
        return ops.moe_forward(xin, None, None, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q,
                               kw.down_sf, bank.down_global, 2.5, router_terms=terms, router_bias=mod.expert_bias,
                               top_k=k, out=yout, gate_up_sf_layout=kw.gate_up_sf_layout,
                               down_sf_layout=kw.down_sf_layout)

    def step():
        return layer(x, out)

    # correctness guard of the measured path: routing and output vs the
    # stage-by-stage ops path (same kernels, separate launches)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream(dev)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    value = t * world / (ms / 1e3)

    latency = None
    if args.config == "5":
        latency = graph_latency(step, dev, calls=max(20, args.steps * 5))

    # per-stage timing (same kernels launched stage by stage, events on the
    # launching stream) for the roofline of the dominant kernel
    stages = time_stages(pkg, x, terms, mod, bank, kw, cfg, reps=max(3, min(args.steps, 10)))
    gemm1_ms = stages["gemm1_swiglu"]
    flops1 = 2.0 * t * k * c * 2 * f
    bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
    fp4_peak = 4.0 * bf16_peak
    traffic = GEMM1_TRAFFIC.get((args.config, t))
    roofline = {"bound": "tensor", "kernel": "gemm_nvfp4_pair_kernel<EPI_SWIGLU> (gate/up)",
                "achieved": flops1 / (gemm1_ms / 1e3) / 1e12, "peak": fp4_peak, "unit": "TFLOP/s",
                "frac": flops1 / (gemm1_ms / 1e3) / 1e12 / fp4_peak,
                "traffic": traffic, "traffic_unit": "bytes per launch (ncu dram read + write)" if traffic else None,
                "algorithmic_bytes": gemm1_bytes(t, k, c, f, e),
                "peak_note": ("dense FP4 peak = 4 x measured cuBLAS bf16 burst "
                              f"({bf16_peak} TFLOP/s, MEASURED_PEAKS.json); nominal dense FP4 9000 TFLOP/s")}
    layer_flops = 6.0 * t * k * c * f
    e2e = None
    if not args.no_e2e:
        e2e = time_e2e(pkg, layer, x_cpu, out, args, dev, t, world)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, ue4m3 block16 scales, fp32 accumulate), bf16 I/O",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) expert weights packed to NVFP4)",
        "config": {"workload": f"BASELINE config {args.config}: one MoE layer forward incl. router", "tokens": t,
                   "dim": c, "experts": e, "top_k": k, "expert_hidden": f, "router": "sigmoid+renorm",
                   "parallelism": "replicas" if world > 1 else "single-gpu",
                   "l2": "inputs + packed weights (610 MB) exceed the 126 MB L2; no flush"},
        "layer_tflops": layer_flops / (ms / 1e3) / 1e12,
        "stages_ms": stages,
        "roofline": roofline,
        "graph_latency": latency,
        "clocks": clk.summary(),
        # router 2, dispatch 3, quantize 2 + scale replication 1, GEMM 2, combine 1
        "gpu_launches": 11 * args.steps,
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_expert_parallel(args, cfg):
    """N > 1: the layer expert-parallel over the N GPUs of one node (config 4:
    each rank routes its own tokens; experts sharded 64/N per rank; NVFP4 rows
    and scales out, bf16 rows back; by default on the copy engines into
    IPC-mapped peer buffers, ``--transport nccl`` for NCCL transfers)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    pkg = importlib.import_module("praxis-1-oss_b200")
    pkg.capi.load()
    ops = pkg.ops
    peaks = {}
    pfile = ROOT / "MEASURED_PEAKS.json"
    if pfile.exists():
        peaks = json.loads(pfile.read_text())
    t, c, e, k, f = cfg["tokens"], cfg["dim"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    if e % world:
        raise SystemExit(f"{e} experts do not shard over {world} ranks")
    el = e // world
    # tokens seeded per rank; the same weights on every rank (the full bank is
    # generated from one seed, each rank packs its own experts)
    x_cpu, router, bias, _gu, _dn = make_inputs(dict(cfg, experts=0), 1000 + rank, dev)
    gw = torch.Generator(device=dev).manual_seed(7)
    gu = (torch.randn(e, c, 2 * f, generator=gw, device=dev) * 0.02).to(torch.bfloat16)[rank * el:(rank + 1) * el]
    down = (torch.randn(e, f, c, generator=gw, device=dev) * 0.02).to(torch.bfloat16)[rank * el:(rank + 1) * el]
    bank = pkg.pack_routed_experts(gu.contiguous(), down.contiguous(), keep_on_device=True)
    del gu, down
    bank.prepare()
    ep = pkg.expert_parallel.ExpertParallelRoutedExperts(bank, e, transport=args.transport, chunks=args.ep_chunks,
                                                         copy_streams=args.copy_streams,
                                                         sm_copy_fraction=args.sm_copy_fraction)
    grouter = torch.Generator().manual_seed(11)
    router = (torch.randn(e, c, generator=grouter) * (1.0 / c) ** 0.5).to(dev)
    terms = ops.split_router_weight(router)
    bias = torch.zeros(e, device=dev)
    x = x_cpu.to(dev)

    def step(inp=None):
        xin = x if inp is None else inp
        logits, _amax = ops.router_logits(xin, terms)
        top, gate = ops.route(logits, bias, k)
        return ep.routed_forward(xin, top, gate, scaling=2.5)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one sampler process for the node (rank 0), not one per rank
    clk = ClockSampler(None) if rank == 0 else None
    with clk if clk is not None else contextlib.nullcontext():
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    tt = torch.tensor([ms], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    value = t * world / (ms / 1e3)

    # expert-rank compute of one exchange, timed alone (both GEMMs and the
    # hidden quantize on the rows this rank received)
    be = ep._backend
    routing = be.route_rows(x, *ops.route(ops.router_logits(x, terms)[0], bias, k), e)
    q, sf = be.quantize(x, routing)
    pc = routing.pcsr.cpu().long()
    rows_here = int(pc[-1])
    cnt = (routing.csr[1:] - routing.csr[:-1]).to(torch.int32)
    starts = routing.pcsr[:-1].to(torch.int32)
    # (every expert's rows of this rank's tokens through the local weights:
    # the same FLOPs as the rank's share of the layer)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    be.experts(q[:rows_here], sf[:rows_here], cnt, torch.cat([starts, routing.pcsr[-1:]]).to(torch.int32),
               routing.act_global, 0, el)
    torch.cuda.synchronize()
    evs[0].record(stream)
    be.experts(q[:rows_here], sf[:rows_here], cnt, torch.cat([starts, routing.pcsr[-1:]]).to(torch.int32),
               routing.act_global, 0, el)
    evs[1].record(stream)
    torch.cuda.synchronize()
    exp_ms = evs[0].elapsed_time(evs[1])
    flops = 6.0 * t * k * c * f
    fp4_peak = 4.0 * float(peaks.get("bf16_tflops", 1590.0))
    roofline = {"bound": "tensor", "kernel": "expert_forward (gate/up GEMM + SwiGLU, hidden quantize, down GEMM)",
                "achieved": flops / (exp_ms / 1e3) / 1e12, "peak": fp4_peak, "unit": "TFLOP/s",
                "frac": flops / (exp_ms / 1e3) / 1e12 / fp4_peak, "traffic": None,
                "peak_note": "4 x measured cuBLAS bf16 burst (MEASURED_PEAKS.json); rows of this rank's own tokens "
                             "through its local experts' weights, one launch sequence"}
    e2e = None
    if not args.no_e2e:
        torch.cuda.synchronize()
        dist.barrier()
        out = torch.empty(t, c, dtype=torch.bfloat16, device=dev)
        e2e = time_e2e(pkg, lambda xin, yout: yout.copy_(step(xin)), x_cpu, out, args, dev, t, world)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, ue4m3 block16 scales, fp32 accumulate), bf16 I/O",
        "data": "synthetic (seeded N(0,1) activations per rank, N(0,0.02) expert weights packed to NVFP4)",
        "config": {"workload": f"BASELINE config {args.config}: expert-parallel MoE layer forward incl. router",
                   "tokens_per_rank": t, "dim": c, "experts": e, "experts_per_rank": el, "top_k": k,
                   "expert_hidden": f, "router": "sigmoid+renorm", "parallelism": f"ep{world}",
                   "exchange": ("copy engines into IPC-mapped peer buffers" if args.transport == "peer" else
                                "NCCL point-to-point") + ": FP4 rows + UE4M3 scales out, bf16 rows back",
                   "l2": "per-rank inputs and weights exceed the 126 MB L2; no flush"},
        "layer_tflops": flops * world / (ms / 1e3) / 1e12,
        "roofline": roofline,
        "clocks": clk.summary() if clk is not None else None,
        # router 2, row max 1, dispatch 3, quantize 1, and per expert-forward call (one per source rank):
        # tiles 1, scale replication 1, GEMM 2, hidden quantize 1; combine 1 (NCCL's own kernels not counted)
        "gpu_launches": (8 + 5 * world) * args.steps,
        "e2e": e2e,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    ep.close()
    dist.barrier()
    dist.destroy_process_group()


def graph_latency(step, dev, calls=50, euler_steps=10):
    """the layer forward captured in a CUDA graph and
    replayed as the 10 steps of a flow-matching Euler loop; per-call (one
    replay) latency p50/p90 from CUDA events around each replay."""
    import torch

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    stream = torch.cuda.current_stream(dev)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(calls):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(euler_steps + 1)]
        evs[0].record(stream)
        for i in range(euler_steps):
            graph.replay()
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        times += [evs[i].elapsed_time(evs[i + 1]) for i in range(euler_steps)]
    times.sort()
    del graph
    return {"p50_ms": times[len(times) // 2], "p90_ms": times[(len(times) * 9) // 10], "calls": len(times),
            "euler_steps_per_loop": euler_steps, "capture": "whole layer incl. router in one CUDA graph"}


def time_stages(pkg, x, terms, mod, bank, kw, cfg, reps=5):
    import torch

    ops, capi = pkg.ops, pkg.capi
    k = cfg["top_k"]
    names = ["router_logits", "route", "dispatch", "quantize_gather", "gemm1_swiglu", "quantize_hidden",
             "gemm2_rescale", "combine"]
    acc = {n: 0.0 for n in names}
    stream = torch.cuda.current_stream(x.device)
    for rep in range(reps + 1):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        # a spin of ~2 ms ahead of the stages lets the host enqueue all of
        # them first, so the event gaps hold device time only (no launch gaps)
        torch.cuda._sleep(4_000_000)
        evs[0].record(stream)
        logits, amax = ops.router_logits(x, terms)
        evs[1].record(stream)
        top, gate = ops.route(logits, mod.expert_bias, k)
        evs[2].record(stream)
        r = ops.dispatch(top, gate, cfg["experts"], amax, full=False)
        evs[3].record(stream)
        aq, asf = ops.quantize_gather(x, r, r.act_global)
        if kw.gate_up_sf_layout == capi.SF_REPLICATED:
            asf = ops.replicate_scales(asf, 128)
        evs[4].record(stream)
        hamax = torch.zeros(cfg["experts"], dtype=torch.int32, device=x.device)
        e_g0 = torch.cuda.Event(enable_timing=True)
        e_g0.record(stream)
        hidden = ops.grouped_gemm(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, epilogue=capi.EPI_SWIGLU,
                                  act_global=r.act_global, w_global=bank.gate_up_global, amax_out=hamax,
                                  sf_layout=kw.gate_up_sf_layout)
        evs[5].record(stream)
        hq, hsf = ops.quantize_rows(hidden, r, amax_bits=hamax)
        if kw.down_sf_layout == capi.SF_REPLICATED:
            hsf = ops.replicate_scales(hsf, 128)
        evs[6].record(stream)
        rows = ops.grouped_gemm(hq, hsf, bank.down_q, kw.down_sf, r, epilogue=capi.EPI_RESCALE, act_amax=hamax,
                                w_global=bank.down_global, sf_layout=kw.down_sf_layout)
        evs[7].record(stream)
        ops.combine(rows, r, 2.5, rows_rescaled=True)
        evs[8].record(stream)
        torch.cuda.synchronize()
        if rep == 0:
            continue
        for i, n in enumerate(names):
            if n == "gemm1_swiglu":
                acc[n] += e_g0.elapsed_time(evs[5])
            else:
                acc[n] += evs[i].elapsed_time(evs[i + 1])
    return {n: v / reps for n, v in acc.items()}


def time_e2e(pkg, layer, x_cpu, out, args, dev, t, world):
    """Same metric through the public API with host buffers: every step
    copies its input from pinned host memory and reads the whole output back
    (praxis_b200.pipeline.HostPipeline: the copies of neighbouring steps
    overlap the compute on their own streams)."""
    import torch

    host_in = x_cpu.pin_memory()
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    pipe = pkg.pipeline.HostPipeline(layer, x_cpu.shape, out.shape, out.dtype, dev)
    pipe.run([host_in] * 2, [host_out] * 2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(pipe.copy_in)
    pipe.run([host_in] * args.steps, [host_out] * args.steps)
    e1.record(pipe.copy_out)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        import torch.distributed as dist

        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    return {"value": t * world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "h2d_bytes_per_step": host_in.numel() * 2 * world, "d2h_bytes_per_step": host_out.numel() * 2 * world}


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.config is None:
        args.config = "4" if dist_env()[1] > 1 else "2"
    cfg = dict(CONFIGS[args.config])
    if args.tokens is not None:
        cfg["tokens"] = args.tokens
    if args.impl == "reference":
        run_reference(args, cfg)
    elif dist_env()[1] > 1:
        run_expert_parallel(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
