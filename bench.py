"""Benchmark of one routed-expert NVFP4 MoE layer forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2]

One step = one MoE layer forward of the configured shape: router logits
(tensor cores) + sigmoid/top-k/renorm, dispatch, NVFP4 gather-quantize,
gate/up grouped GEMM with fused SwiGLU, hidden quantize, down grouped GEMM
with fused rescale, weighted combine. Metric: routed-expert tokens/s per MoE
layer (whole job: tokens of all ranks / max-over-ranks step time).

Inputs are synthetic and seeded (x ~ N(0,1) bf16, expert weights ~ N(0,0.02)
packed to NVFP4 on the GPU, router weight ~ N(0, 1/C) so the logits are
~N(0,1)); no public dataset stands behind the BASELINE configs.

N = 1 runs BASELINE config 2 (16,384 tokens) and, as extra keys of the same
line, config 3 (Zipf-skewed routing with its per-expert histogram), config 5
(CUDA-graph latency over 10 Euler steps) and config 4's per-rank shape
(65,536 tokens) on one GPU, the like-for-like base of the scaling run.
N > 1 (torchrun) runs config 4: the layer expert-parallel over the N GPUs of
one node, 65,536 tokens per rank (weak scaling), each rank's output checked
bit for bit against the single-GPU bank on the same tokens.

The CPU leg (``cpu_baseline`` at N = 1, and ``--impl reference``) times the
CPU port of the reference path (the oracle's NVFP4 chain with weights
dequantised once, float32 GEMMs) on the same full batch with all host
threads, plus a one-thread figure on a token sample; at N = 1 it also checks
the GPU output against that chain (``parity``).
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
# Zipf(s=1.2) expert popularity of config 3 enters through the routing bias
# (the reference's expert_bias: it changes which experts are picked, not their
# gates); this strength makes the most popular expert be picked by about 30%
# of the tokens (calibrated on N(0,1) logits, 16,384 tokens, top-4).
ZIPF_S = 1.2
ZIPF_BETA = 0.052


def zipf_selection_bias(experts: int, beta: float = ZIPF_BETA, seed: int = 0):
    """float32 expert bias beta * log p_e with p_e proportional to rank^-1.2
    over a fixed random permutation of the expert ids (seed 0)."""
    import torch

    perm = torch.randperm(experts, generator=torch.Generator().manual_seed(seed))
    rank = torch.empty(experts)
    rank[perm] = torch.arange(1, experts + 1, dtype=torch.float32)
    logp = -ZIPF_S * torch.log(rank)
    return beta * (logp - torch.logsumexp(logp, 0))

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one gate/up GEMM
# launch at the full config-2 workload, from a capture of those two metrics
# alone (one pass, as ncu reported for the same metrics on a 2,048-token case):
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none
#       -k regex:gemm_nvfp4_pair_kernel -c 1
#       python bench.py --steps 1 --warmup 1 --no-e2e --no-cpu-baseline --no-extra
# (read 462,110,976 + write 193,003,520 at config 2, 16384 tokens; compact scales).
GEMM1_TRAFFIC = {("2", 16384): 462110976 + 193003520}


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
    ap.add_argument("--no-extra", action="store_true", help="skip the extra config keys of the default line")
    ap.add_argument("--flashinfer", action="store_true",
                    help="also time FlashInfer's block-scaled grouped GEMM (the kernel the reference calls) on the "
                         "same operands (N = 1)")
    ap.add_argument("--router-fused", action="store_true",
                    help="also time the reference's own router_fused.route_dispatch (CuTe DSL, E=128/top-8) from the "
                         "offline reference install under baseline/_ref against this library's routing (N = 1)")
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
    x, router, bias = make_host_inputs(cfg, seed)
    gw = torch.Generator(device=device).manual_seed(seed + 1)
    gu = (torch.randn(e, c, 2 * f, generator=gw, device=device) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=gw, device=device) * 0.02).to(torch.bfloat16)
    return x, router, bias, gu, down


def _smi_ids(ordinals) -> list[str]:
    """nvidia-smi ids of CUDA device ordinals (through CUDA_VISIBLE_DEVICES)."""
    vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return [vis[i] if i < len(vis) else str(i) for i in ordinals]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of the GPUs in use (CUDA
    ordinals ``ordinals``) during the timed region: a 20 ms sampling loop
    started before the region; the summary keeps the samples whose own
    timestamps fall inside the region (the nearest one per GPU when the
    region is shorter than the loop)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, ordinals):
        self.ids = _smi_ids(ordinals)
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = 0.0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(self.ids), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.4)  # the loop is running before the region starts
        except OSError:
            self.proc = None
        self.t0 = time.time()
        return self

    def __exit__(self, *exc):
        self.t1 = time.time()
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        import datetime

        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        samples = []  # (time, gpu, sm MHz, max MHz, reasons)
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((ts, parts[1], float(parts[2]), float(parts[3]),
                                {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))
            except (ValueError, IndexError):
                continue
        inside = [x for x in samples if self.t0 - 0.01 <= x[0] <= self.t1 + 0.01]
        if not inside:  # region shorter than the loop: the nearest sample of each GPU
            best = {}
            for x in samples:
                d = min(abs(x[0] - self.t0), abs(x[0] - self.t1))
                if x[1] not in best or d < best[x[1]][0]:
                    best[x[1]] = (d, x)
            inside = [v[1] for v in best.values()]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        reasons = set().union(*(x[4] for x in inside))
        return {"sm_mhz": statistics.median(x[2] for x in inside), "sm_max_mhz": max(x[3] for x in inside),
                "reasons": sorted(reasons), "samples": len(inside), "gpus": sorted({x[1] for x in inside})}


def cpu_port_forward(prep, x, router, bias, cfg, routing=None):
    """The oracle's NVFP4 chain with dequantised fp32 weights (CPU port of the
    reference path): router, routing, dispatch, activation quantize, gate/up
    GEMM, rescale + SwiGLU, hidden quantize, down GEMM, rescale + combine.
    ``routing`` = (top_idx, gate) replaces the port's own router."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    e, k, c, f = cfg["experts"], cfg["top_k"], cfg["dim"], cfg["hidden"]
    if routing is None:
        logits = O.router_logits(x, router)
        top, gate = O.route(logits, bias, k)
    else:
        top, gate = routing
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


def port_weights(state, cfg):
    """Packed bank buffers (CPU) -> the port's fp32 dequantised matrices and
    global scales (load-time work, not timed)."""
    from oracle import nvfp4_moe_oracle as O

    c, f = cfg["dim"], cfg["hidden"]
    n = state["gate_up_q"].shape[0]
    return {"gu": [O.dequant_matrix(state["gate_up_q"][ex], state["gate_up_sf"][ex], 2 * f, c) for ex in range(n)],
            "dn": [O.dequant_matrix(state["down_q"][ex], state["down_sf"][ex], c, f) for ex in range(n)],
            "gug": state["gate_up_global"].float(), "dng": state["down_global"].float()}


def port_weights_synthetic(cfg, distinct=8):
    """The port's weights without a GPU: ``distinct`` experts' bf16 weights
    ~ N(0, 0.02) packed with the oracle's recipe, expert e using those of
    e % distinct (the CPU work per expert does not depend on the values)."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    e, c, f = cfg["experts"], cfg["dim"], cfg["hidden"]
    g = torch.Generator().manual_seed(8)
    base = {"gu": [], "dn": [], "gug": [], "dng": []}
    for _ in range(min(distinct, e)):
        for key, (n, k) in (("gu", (2 * f, c)), ("dn", (c, f))):
            w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
            q, sf, gg = O.pack_matrix(w)
            base[key].append(O.dequant_matrix(q, sf, n, k))
            base[key + "g"].append(float(gg))
    d = len(base["gu"])
    return {"gu": [base["gu"][ex % d] for ex in range(e)], "dn": [base["dn"][ex % d] for ex in range(e)],
            "gug": torch.tensor([base["gug"][ex % d] for ex in range(e)]),
            "dng": torch.tensor([base["dng"][ex % d] for ex in range(e)])}


def time_port(prep, x, router, bias, cfg, threads, budget_s, max_runs, min_runs=1):
    """Median seconds per forward of the CPU port on ``threads`` threads,
    and the last output."""
    import torch

    torch.set_num_threads(threads)
    times, out = [], None
    start = time.perf_counter()
    while len(times) < max_runs:
        t0 = time.perf_counter()
        out = cpu_port_forward(prep, x, router, bias, cfg)
        times.append(time.perf_counter() - t0)
        if len(times) >= min_runs and time.perf_counter() - start > budget_s:
            break
    return statistics.median(times), len(times), out


def cpu_baseline(cfg, prep, x, router, bias, budget_s=30.0, max_runs=3, single_thread_tokens=2048):
    """The CPU port on the full batch with every host thread, plus one thread
    on the first ``single_thread_tokens`` tokens; tokens/s."""
    import torch

    threads = os.cpu_count() or 1
    t = x.shape[0]
    med, runs, out = time_port(prep, x, router, bias, cfg, threads, budget_s, max_runs)
    sub = min(t, single_thread_tokens)
    med1, runs1, _ = time_port(prep, x[:sub].contiguous(), router, bias, dict(cfg, tokens=sub), 1, 10.0, 2)
    torch.set_num_threads(threads)
    return {"value": t / med, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"the full batch: {t} tokens (C={cfg['dim']}, E={cfg['experts']}, k={cfg['top_k']}, "
                      f"F={cfg['hidden']}), median of {runs} forwards incl. the router, weights dequantised once "
                      f"outside the timing",
            "single_thread": {"value": sub / med1, "unit": "tokens/s", "cores": 1,
                              "sample": f"first {sub} tokens of the batch, median of {runs1} forwards"}}, out


def workload_config(cfg, name, world):
    """The ``config`` object of a bench line (shared by both arms so that the
    driver sees the same workload)."""
    t = cfg["tokens"]
    in_bytes = t * cfg["dim"] * 2
    weights = cfg["experts"] * 3 * cfg["hidden"] * cfg["dim"] * (1 / 2 + 1 / 16)
    fits = in_bytes + weights < 126e6
    return {"workload": f"BASELINE config {name}: one MoE layer forward incl. router" +
                        (" (expert parallel)" if world > 1 else ""),
            "tokens" if world == 1 else "tokens_per_rank": t, "dim": cfg["dim"], "experts": cfg["experts"],
            "top_k": cfg["top_k"], "expert_hidden": cfg["hidden"],
            "router": "sigmoid+renorm" + (", Zipf(1.2) selection bias" if cfg["skew"] else ""),
            "parallelism": f"ep{world}" if world > 1 else "single-gpu",
            "l2": (f"activations + packed weights ({(in_bytes + weights) / 1e6:.0f} MB) fit in the 126 MB L2 "
                   "(steady-state serving: weights stay resident)") if fits else
                  (f"activations + packed weights ({(in_bytes + weights) / 1e6:.0f} MB) exceed the 126 MB L2; "
                   "no flush")}


def run_reference(args, cfg):
    """``--impl reference``: the CPU port of the reference path on the box's
    host cores, on the same workload as the GPU arm; rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    c, e = cfg["dim"], cfg["experts"]
    x, router, bias = make_host_inputs(cfg, 1000)
    prep = port_weights_synthetic(cfg)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(min(args.warmup, 1)):
        cpu_port_forward(prep, x, router, bias, cfg)
    med, runs, _ = time_port(prep, x, router, bias, cfg, threads, budget_s=120.0, max_runs=args.steps,
                             min_runs=min(args.steps, 3))
    value = cfg["tokens"] / med
    sample = (f"the full batch of {cfg['tokens']} tokens per forward, median of {runs} of the {args.steps} "
              f"requested forwards (capped at ~2 min of CPU time), 1 warm-up forward")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, fp32 accumulate)",
            "data": "synthetic", "config": workload_config(cfg, args.config, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def make_host_inputs(cfg, seed):
    """x, router weight and routing bias of a config on the host (the seeds
    of make_inputs)."""
    import torch

    t, c, e = cfg["tokens"], cfg["dim"], cfg["experts"]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(t, c, generator=g).to(torch.bfloat16)
    router = torch.randn(e, c, generator=g) * (1.0 / c) ** 0.5
    bias = zipf_selection_bias(e) if cfg["skew"] else torch.zeros(e)
    return x, router, bias


def build_layer(pkg, cfg, seed, dev):
    """A B200MoEFeedForward of the config with seeded weights; returns the
    module, its bank, kernel weights, router terms, host inputs and the
    layer call (x, out) -> (out, top_idx, gate) through the public op."""
    import torch

    t, c, e, k, f = cfg["tokens"], cfg["dim"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    x_cpu, router, bias, gu, down = make_inputs(cfg, seed, dev)
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
    ops = pkg.ops

    def layer(xin, yout):
        return ops.moe_forward(xin, None, None, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q,
                               kw.down_sf, bank.down_global, 2.5, router_terms=terms, router_bias=mod.expert_bias,
                               top_k=k, out=yout, gate_up_sf_layout=kw.gate_up_sf_layout,
                               down_sf_layout=kw.down_sf_layout)

    return dict(mod=mod, bank=bank, kw=kw, terms=terms, x_cpu=x_cpu, router=router, bias=bias, layer=layer)


def time_steps(step, dev, steps, warmup):
    """ms per step: CUDA events on the launching stream around ``steps``
    back-to-back steps after ``warmup`` untimed ones."""
    import torch

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / steps


def gpu_parity(pkg, L, x, cfg):
    """The measured path (one fused praxis_b200_moe_forward with the router)
    against the same kernels launched stage by stage through the ops: routing
    and output bit for bit (GPU only; the oracle check is in the CPU leg)."""
    import torch

    ops, capi = pkg.ops, pkg.capi
    bank, kw, mod = L["bank"], L["kw"], L["mod"]
    e, k = cfg["experts"], cfg["top_k"]
    out_f, top_f, gate_f = L["layer"](x, torch.empty_like(x))
    logits, amax = ops.router_logits(x, L["terms"])
    top, gate = ops.route(logits, mod.expert_bias, k)
    r = ops.dispatch(top, gate, e, amax, full=False)
    aq, asf = ops.quantize_gather(x, r, r.act_global)
    hamax = torch.zeros(e, dtype=torch.int32, device=x.device)
    a_sf = ops.replicate_scales(asf, 128) if kw.gate_up_sf_layout == capi.SF_REPLICATED else asf
    hidden = ops.grouped_gemm(aq, a_sf, kw.gate_up_q, kw.gate_up_sf, r,
                              epilogue=capi.EPI_SWIGLU, act_global=r.act_global, w_global=bank.gate_up_global,
                              amax_out=hamax, sf_layout=kw.gate_up_sf_layout)
    hq, hsf = ops.quantize_rows(hidden, r, amax_bits=hamax)
    rows = ops.grouped_gemm(hq, hsf, bank.down_q, kw.down_sf, r, epilogue=capi.EPI_RESCALE, act_amax=hamax,
                            w_global=bank.down_global, sf_layout=kw.down_sf_layout)
    out_s = ops.combine(rows, r, 2.5, rows_rescaled=True)
    # the reference's stock routing ops (praxis/layers.py:2167-2173) by torch on this GPU
    scores = torch.sigmoid(logits)
    ref_top = torch.topk(scores + mod.expert_bias, k, dim=-1).indices
    picked = scores.gather(-1, ref_top)
    ref_gate = (picked / picked.sum(-1, keepdim=True)).to(torch.bfloat16)
    torch.cuda.synchronize()
    same = lambda a, b: bool(torch.equal(a.view(torch.uint8), b.view(torch.uint8)))  # noqa: E731
    err = capi.device_error(x.device.index or 0)
    res = {"fused_vs_stage_ops_bit_exact": same(out_f, out_s) and same(top_f, top) and same(gate_f, gate),
           "routing_bit_exact_vs_torch_stock_ops": same(top, ref_top) and same(gate, ref_gate),
           "device_error_word": err}
    counts = torch.bincount(top.flatten(), minlength=e).cpu()
    return res, dict(logits=logits.cpu(), top=top.cpu(), gate=gate.cpu(), out=out_f.cpu()), counts


def run_b200(args, cfg):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module("praxis-1-oss_b200")
    pkg.capi.load()
    peaks = {}
    pfile = ROOT / "MEASURED_PEAKS.json"
    if pfile.exists():
        peaks = json.loads(pfile.read_text())

    t, c, e, k, f = cfg["tokens"], cfg["dim"], cfg["experts"], cfg["top_k"], cfg["hidden"]
    L = build_layer(pkg, cfg, 1000, dev)
    x = L["x_cpu"].to(dev)
    out = torch.empty_like(x)
    parity, gpu_res, counts = gpu_parity(pkg, L, x, cfg)

    def step():
        return L["layer"](x, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler([dev.index]) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    value = t / (ms / 1e3)

    # per-stage timing (same kernels launched stage by stage, events on the
    # launching stream) for the roofline of the dominant kernel
    stages = time_stages(pkg, x, L["terms"], L["mod"], L["bank"], L["kw"], cfg, reps=max(3, min(args.steps, 10)))
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
    gemm2_ms = stages["gemm2_rescale"]
    roofline["down_gemm"] = {"kernel": "gemm_nvfp4_pair_kernel<EPI_RESCALE> (down)",
                             "achieved": 2.0 * t * k * f * c / (gemm2_ms / 1e3) / 1e12,
                             "frac": 2.0 * t * k * f * c / (gemm2_ms / 1e3) / 1e12 / fp4_peak}
    layer_flops = 6.0 * t * k * c * f
    e2e = None
    if not args.no_e2e:
        e2e = time_e2e(pkg, L["layer"], L["x_cpu"], out, args, dev, t, 1)

    extra = {}
    if args.config == "2" and not args.no_extra:
        extra = extra_configs(pkg, L, args, dev)
    if args.flashinfer:
        extra["flashinfer_gemm"] = flashinfer_gemm(pkg, L, x, cfg, stages)
    if args.router_fused:
        extra["router_fused_reference"] = router_fused_head_to_head(pkg, dev)

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e2m1, ue4m3 block16 scales, fp32 accumulate), bf16 I/O",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) expert weights packed to NVFP4)",
        "config": workload_config(cfg, args.config, 1),
        "layer_tflops": layer_flops / (ms / 1e3) / 1e12,
        "stages_ms": stages,
        "read_floor": read_floor(x, reps=max(3, min(args.steps, 10))),
        "roofline": roofline,
        "expert_rows": {"max": int(counts.max()), "min": int(counts.min()), "top_expert_token_share": float(
            counts.max()) / t},
        "clocks": clk.summary(),
        # router 2, dispatch 3, quantize 1 (+ scale replication 1 for replicated weight scales), GEMM 2,
        # hidden quantize 1, combine 1
        "gpu_launches": (10 + int(L["kw"].gate_up_sf_layout == pkg.capi.SF_REPLICATED)) * args.steps,
        "e2e": e2e,
        "parity": parity,
        **extra,
    }
    if args.config == "5":
        line["graph_latency"] = graph_latency(step, dev, calls=max(20, args.steps * 5))
    if not args.no_cpu_baseline:
        line["cpu_baseline"], port_out = cpu_leg_with_parity(L, cfg, gpu_res)
        parity.update(port_out)
    parity["ok"] = bool(parity["fused_vs_stage_ops_bit_exact"] and parity["device_error_word"] == 0 and
                        parity["routing_bit_exact_vs_torch_stock_ops"] and
                        parity.get("topk_agreement_oracle_on_gpu_logits", 1.0) >= 0.9999 and
                        parity.get("gate_max_bf16_ulp_vs_oracle", 0) <= 1 and
                        parity.get("out_rel_l2_vs_port", 0.0) <= 1e-2)
    print(json.dumps(line), flush=True)


def flashinfer_gemm(pkg, L, x, cfg, stages):
    """FlashInfer's block-scaled contiguous grouped GEMM, the kernel the
    reference's grouped_nvfp4_mm calls on SM100 (praxis/kernels/nvfp4.py:
    355-419), timed on this layer's own FP4 operands with the reference's
    call: 128-row tiles, cluster 1x1, the tile table of the padded CSR, unit
    alpha, and the identity row mapping with unit scales (the reference pins
    flashinfer 0.6.18, whose use_fused_finalize=False returns the plain GEMM;
    the installed version always finalizes, here with atomic adds into a
    zeroed output). Against this library's gate/up (SwiGLU fused) and down
    (rescale fused) GEMMs; the reference runs its SwiGLU and rescale as
    separate passes."""
    import torch

    try:
        import flashinfer
        from flashinfer.fused_moe.cute_dsl.blockscaled_contiguous_grouped_gemm_finalize_fusion import (
            blockscaled_contiguous_grouped_gemm_finalize_fusion_nvfp4 as fi,
        )
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"flashinfer not importable: {type(exc).__name__}: {exc}"[:200]}
    ops, capi = pkg.ops, pkg.capi
    bank, kw = L["bank"], L["kw"]
    e, k, c, f = cfg["experts"], cfg["top_k"], cfg["dim"], cfg["hidden"]
    t = x.shape[0]
    dev = x.device
    logits, amax = ops.router_logits(x, L["terms"])
    top, gate = ops.route(logits, L["mod"].expert_bias, k)
    r = ops.dispatch(top, gate, e, amax, full=False)
    aq, asf = ops.quantize_gather(x, r, r.act_global)
    hamax = torch.zeros(e, dtype=torch.int32, device=dev)
    hidden = ops.grouped_gemm(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, epilogue=capi.EPI_SWIGLU,
                              act_global=r.act_global, w_global=bank.gate_up_global, amax_out=hamax,
                              sf_layout=kw.gate_up_sf_layout)
    hq, hsf = ops.quantize_rows(hidden, r, amax_bits=hamax)
    rp = aq.shape[0]
    tiles = rp // 128
    pc = r.pcsr.long()
    expert = torch.bucketize(torch.arange(tiles, device=dev) * 128, pc[1:], right=True).clamp_max(e - 1)
    limit = pc[1:][expert].to(torch.int32)
    expert = expert.to(torch.int32)
    # the reference's operand shapes exactly (its 128-row tile table must match the padded layout)
    assert int(limit.max()) <= rp and tuple(asf.shape) == (rp, c // 16) and tuple(hsf.shape) == (rp, f // 16)
    ntiles = torch.tensor([tiles], dtype=torch.int32, device=dev)
    ident = torch.arange(rp, dtype=torch.int32, device=dev)
    ones = torch.ones(rp, 1, dtype=torch.float32, device=dev)
    alpha = torch.ones(e, dtype=torch.float32, device=dev)
    res = {"version": getattr(flashinfer, "__version__", "?"), "tile": [128, 128], "cluster": [1, 1]}
    flops = {"gate_up": 2.0 * t * k * c * 2 * f, "down": 2.0 * t * k * f * c}
    for name, a_, as_, b_, bs_, n_ in (("gate_up", aq, asf, bank.gate_up_q, bank.gate_up_sf, 2 * f),
                                       ("down", hq, hsf, bank.down_q, bank.down_sf, c)):
        out = torch.zeros(rp, n_, dtype=torch.bfloat16, device=dev)

        def call():
            fi(a_, b_, as_, bs_, alpha, expert, ntiles, limit, ident, ones, out, mma_tiler_mn=(128, 128),
               cluster_shape_mn=(1, 1), enable_pdl=False)

        try:
            for _ in range(3):
                call()
            ms = time_steps(call, dev, 20, 0)
        except Exception as exc:  # noqa: BLE001
            res[name] = {"failed": f"{type(exc).__name__}: {exc}"[:200]}
            continue
        ours = stages["gemm1_swiglu" if name == "gate_up" else "gemm2_rescale"]
        res[name] = {"flashinfer_ms": ms, "flashinfer_tflops": flops[name] / (ms / 1e3) / 1e12, "b200_ms": ours,
                     "speedup": ms / ours}
    return res


def router_fused_head_to_head(pkg, dev, tokens=16384, dim=3072, experts=128, top_k=8):
    """The reference's sm_100 routing path at its own shape (E=128, top-8):
    the stock fp32 router GEMM (``F.linear(x.float(), W.float())``,
    praxis/layers.py:1104-1122) and ``router_fused.route_dispatch``
    (praxis/kernels/router_fused.py:738-804, CuTe DSL) from the offline
    reference install, against this library's logits kernel and its route +
    dispatch kernels; P = 1 and the CFG pair P = 2. Also the bitwise
    agreement of the two routings on the reference's logits."""
    import sys

    import torch
    import torch.nn.functional as F

    ref = ROOT / "baseline" / "_ref"
    if not (ref / "praxis" / "kernels" / "router_fused.py").is_file():
        return {"unavailable": "the reference install (baseline/_ref) is absent"}
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        import cutlass.cute  # noqa: F401
        from praxis.kernels import router_fused as rf
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"router_fused not importable: {type(exc).__name__}: {exc}"[:200]}
    try:  # the kernel imports more of the DSL when it is first compiled
        rf.route_dispatch(torch.zeros(64, experts, device=dev), torch.zeros(experts, device=dev), (64,))
    except ImportError as exc:
        return {"unavailable": f"router_fused does not build with this image's CUTLASS DSL: {exc}"[:200]}
    ops = pkg.ops
    g = torch.Generator(device=dev).manual_seed(77)
    x = torch.randn(tokens, dim, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(experts, dim, generator=g, device=dev) * 0.02)
    bias = (torch.randn(experts, generator=g, device=dev) * 0.05).float()
    terms = ops.split_router_weight(w)
    res = {"workload": f"T={tokens}, C={dim}, E={experts}, top-{top_k}", "reps": 20}
    try:
        for name, rows in (("single", (tokens,)), ("pair", (tokens // 2, tokens - tokens // 2))):
            logits = F.linear(x.float(), w.float())
            ref_ms = time_steps(lambda: rf.route_dispatch(logits, bias, rows), dev, 20, 3)
            ours_ms = time_steps(lambda: ops.route_dispatch(logits, bias, rows, top_k=top_k), dev, 20, 3)
            a, b = rf.route_dispatch(logits, bias, rows), ops.route_dispatch(logits, bias, rows, top_k=top_k)
            same = all(torch.equal(getattr(a, n), getattr(b, n)) for n in
                       ("top_idx", "gate", "order", "inverse", "sorted_gate", "tokens", "tokens32", "seg_csr"))
            same = same and torch.equal(a.offsets, b.offsets.contiguous())
            res[name] = {"route_dispatch_reference_ms": ref_ms, "route_dispatch_b200_ms": ours_ms,
                         "speedup": ref_ms / ours_ms, "bit_exact": bool(same)}
        sgemm_ms = time_steps(lambda: F.linear(x.float(), w.float()), dev, 20, 3)
        logits_ms = time_steps(lambda: ops.router_logits(x, terms), dev, 20, 3)
        res["router_logits"] = {"reference_fp32_gemm_ms": sgemm_ms, "b200_ms": logits_ms,
                                "speedup": sgemm_ms / logits_ms}
        res["total_speedup"] = (sgemm_ms + res["single"]["route_dispatch_reference_ms"]) / (
            logits_ms + res["single"]["route_dispatch_b200_ms"])
    except Exception as exc:  # noqa: BLE001
        res["failed"] = f"{type(exc).__name__}: {exc}"[:300]
    return res


def cpu_leg_with_parity(L, cfg, gpu_res):
    """The CPU baseline on the GPU arm's own packed weights and inputs, and
    the parity of the GPU results with it: routing on the GPU's logits
    (bit for bit) and the layer output (relative L2, bar 1e-2)."""
    import torch

    from oracle import nvfp4_moe_oracle as O

    bank = L["bank"]
    state = {n: getattr(bank, n).cpu() for n in ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf",
                                                 "down_global")}
    prep = port_weights(state, cfg)
    cb, port_out = cpu_baseline(cfg, prep, L["x_cpu"], L["router"], L["bias"])
    top, gate = O.route(gpu_res["logits"], L["bias"], cfg["top_k"], tie_order="cuda")
    port_top = O.route(O.router_logits(L["x_cpu"], L["router"]), L["bias"], cfg["top_k"])[0]
    gd = (gate.view(torch.int16).int() - gpu_res["gate"].view(torch.int16).int()).abs()
    res = {"topk_agreement_oracle_on_gpu_logits": float((top == gpu_res["top"]).all(-1).float().mean()),
           "gate_max_bf16_ulp_vs_oracle": int(gd.max()),
           "topk_agreement_port_router": float((port_top == gpu_res["top"]).all(-1).float().mean()),
           "out_rel_l2_vs_port": O.rel_l2(gpu_res["out"], port_out),
           "bar": ("routing bit-exact against torch's stock routing ops on the GPU; against the CPU oracle (CPU "
                   "sigmoid) >= 99.99% of tokens and gates within 1 bf16 ulp; output relative L2 <= 1e-2 against "
                   "the CPU port (dequantised fp32 chain, its own router)")}
    return cb, res


def extra_configs(pkg, L, args, dev):
    """Extra keys of the default line: config 3 (same weights, Zipf-skewed
    routing bias), config 4's per-rank shape on one GPU, config 5 (own
    weights, CUDA-graph latency)."""
    import torch

    out = {}
    steps, warm = max(5, args.steps // 2), 3
    mod, cfg2 = L["mod"], CONFIGS["2"]
    # config 3: the same layer with the calibrated Zipf(1.2) selection bias
    cfg3 = CONFIGS["3"]
    x3, _r, bias3 = make_host_inputs(cfg3, 1003)
    xd3, y3 = x3.to(dev), torch.empty(x3.shape, dtype=torch.bfloat16, device=dev)
    keep = mod.expert_bias.clone()
    with torch.no_grad():
        mod.expert_bias.copy_(bias3.to(dev))
    ms3 = time_steps(lambda: L["layer"](xd3, y3), dev, steps, warm)
    _, top3, _ = L["layer"](xd3, y3)
    cnt = torch.bincount(top3.flatten(), minlength=cfg3["experts"]).cpu()
    with torch.no_grad():
        mod.expert_bias.copy_(keep)
    out["config3"] = {"workload": "BASELINE config 3: config 2 shapes, Zipf(1.2) expert popularity through the "
                                  f"routing bias (strength {ZIPF_BETA})",
                      "ms_per_step": ms3, "value": cfg3["tokens"] / (ms3 / 1e3), "unit": "tokens/s",
                      "top_expert_token_share": float(cnt.max()) / cfg3["tokens"],
                      "expert_rows_sorted": sorted(cnt.tolist(), reverse=True), "steps": steps}
    # config 4's per-rank load on one GPU (65,536 tokens, the same weights)
    cfg4 = CONFIGS["4"]
    x4, _r, _b = make_host_inputs(cfg4, 1000)
    xd4, y4 = x4.to(dev), torch.empty(x4.shape, dtype=torch.bfloat16, device=dev)
    ms4 = time_steps(lambda: L["layer"](xd4, y4), dev, steps, warm)
    out["config4_single_gpu"] = {"workload": "config 4's per-rank shape (65,536 tokens) on one GPU: the "
                                             "like-for-like base of the expert-parallel scaling run",
                                 "ms_per_step": ms4, "value": cfg4["tokens"] / (ms4 / 1e3), "unit": "tokens/s",
                                 "steps": steps}
    del xd4, y4
    # config 5: its own layer, whole forward in one CUDA graph, 10 Euler steps
    cfg5 = CONFIGS["5"]
    L5 = build_layer(pkg, cfg5, 1005, dev)
    x5 = L5["x_cpu"].to(dev)
    y5 = torch.empty_like(x5)
    lat = graph_latency(lambda: L5["layer"](x5, y5), dev, calls=max(20, args.steps * 2))
    out["config5_graph_latency"] = dict(lat, workload="BASELINE config 5: T=512, C=1024, E=32, k=2, F=2048")
    del L5, x5, y5
    out["tail_fusion"] = tail_fusion(pkg, L, dev, steps)
    out["fc1_fp4"] = fc1_fp4(pkg, L, dev, steps)
    out["checkpoint_pair"] = checkpoint_pair(pkg, dev, steps)
    return out


def tail_fusion(pkg, L, dev, steps):
    """Config 2 with the MoE tail fused into the next block's residual add +
    RMSNorm (praxis.layers.MOE_TAIL_NORM, praxis/kernels/moe_tail_triton.py:
    329-352) against the layer followed by the reference's eager residual add
    and norm (praxis/layers.py:214-224); the two must give the same bits."""
    import torch
    import torch.nn.functional as F

    x = L["x_cpu"].to(dev)
    t, c = x.shape
    g = torch.Generator(device=dev).manual_seed(5)
    resid = torch.randn(t, c, generator=g, device=dev).to(torch.bfloat16)
    w1 = (1 + torch.randn(c, generator=g, device=dev) * 0.1).float()
    s_bf16 = torch.tensor(0.75, dtype=torch.bfloat16, device=dev)
    y = torch.empty_like(x)
    tail = pkg.ops.Tail(resid, w1, 1e-6, 0.75)
    bank, kw, mod = L["bank"], L["kw"], L["mod"]

    def fused():
        return pkg.ops.moe_forward(x, None, None, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q,
                                   kw.down_sf, bank.down_global, 2.5, router_terms=L["terms"],
                                   router_bias=mod.expert_bias, top_k=mod.top_k, tail=tail,
                                   gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout)

    def unfused():
        L["layer"](x, y)
        xo = resid + y
        return xo, F.rms_norm(xo.float(), (c,), weight=w1, eps=1e-6).to(torch.bfloat16) * s_bf16

    xo_f, h_f, _, _ = fused()
    xo_u, h_u = unfused()
    same = bool(torch.equal(xo_f, xo_u) and torch.equal(h_f, h_u))
    ms_f = time_steps(fused, dev, steps, 3)
    ms_u = time_steps(unfused, dev, steps, 3)
    return {"workload": "config 2 + the next block's residual add and RMSNorm (C=3072)",
            "fused_ms": ms_f, "unfused_eager_ms": ms_u, "saved_ms": ms_u - ms_f, "bit_exact": same,
            "steps": steps}


def fc1_fp4(pkg, L, dev, steps):
    """Config 2 with a calibrated FC1 output scale (set_fused_swiglu_scale,
    praxis/quantization/nvfp4.py:235-260, :327-339): the gate/up GEMM writes
    FP4 hidden rows at a frozen global, so the bf16 hidden rows and the hidden
    quantize pass go away. The scale follows the reference's calibration rule
    (2 x max |hidden| / 2688, here of this batch); the output changes bits by
    design, reported as its relative L2 distance to the dynamic path."""
    import torch

    ops = pkg.ops
    x = L["x_cpu"].to(dev)
    bank, kw, mod = L["bank"], L["kw"], L["mod"]
    e = mod.num_experts
    logits, amax = ops.router_logits(x, L["terms"])
    top, gate = ops.route(logits, mod.expert_bias, mod.top_k)
    r = ops.dispatch(top, gate, e, amax, full=False)
    aq, asf = ops.quantize_gather(x, r, r.act_global)
    hamax = torch.zeros(e, dtype=torch.int32, device=dev)
    ops.grouped_gemm(aq, asf, kw.gate_up_q, kw.gate_up_sf, r, epilogue=pkg.capi.EPI_SWIGLU, act_global=r.act_global,
                     w_global=bank.gate_up_global, amax_out=hamax)
    g = float(2.0 * hamax.view(torch.float32).max() / 2688.0)
    del aq, asf, r
    y = torch.empty_like(x)
    y_dyn = torch.empty_like(x)
    L["layer"](x, y_dyn)

    def calibrated():
        return ops.moe_forward(x, None, None, kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q,
                               kw.down_sf, bank.down_global, 2.5, router_terms=L["terms"],
                               router_bias=mod.expert_bias, top_k=mod.top_k, out=y,
                               gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout,
                               fc1_output_scale=g)

    calibrated()
    a, b = y.double(), y_dyn.double()
    rel = float((a - b).norm() / b.norm())
    ms = time_steps(calibrated, dev, steps, 3)
    return {"workload": "config 2 with a calibrated FC1 output scale (FP4 hidden rows from the gate/up epilogue)",
            "hidden_global": g, "ms_per_step": ms, "value": x.shape[0] / (ms / 1e3), "unit": "tokens/s",
            "rel_l2_vs_dynamic_scales": rel, "steps": steps}


def checkpoint_pair(pkg, dev, steps):
    """The released checkpoint's MoE shape (E=128, top-8, C=3072, F=1280) as
    a classifier-free-guidance pair of two 8,192-token inputs: one routed
    pass for both (forward_pair, praxis/layers.py:1779-1853) against one
    forward per input (what the reference runs on B200: its NVFP4 pair path
    is SM 11.0 only); the pair must give each input's bits."""
    import torch

    ck = CONFIGS["ckpt"]
    Lc = build_layer(pkg, ck, 1006, dev)
    x = Lc["x_cpu"].to(dev)
    t = x.shape[0]
    t0 = t // 2
    bank, kw, mod = Lc["bank"], Lc["kw"], Lc["mod"]
    args = (kw.gate_up_q, kw.gate_up_sf, bank.gate_up_global, bank.down_q, kw.down_sf, bank.down_global, 2.5)
    kwargs = dict(router_terms=Lc["terms"], router_bias=mod.expert_bias, top_k=ck["top_k"],
                  gate_up_sf_layout=kw.gate_up_sf_layout, down_sf_layout=kw.down_sf_layout)

    def pair():
        return pkg.ops.moe_forward(x, None, None, *args, rows=(t0, t - t0), **kwargs)

    def separate():
        return [pkg.ops.moe_forward(x[a:b], None, None, *args, **kwargs) for a, b in ((0, t0), (t0, t))]

    yp = pair()[0]
    ys = separate()
    same = bool(torch.equal(yp[:t0], ys[0][0]) and torch.equal(yp[t0:], ys[1][0]))
    ms_p = time_steps(pair, dev, steps, 3)
    ms_s = time_steps(separate, dev, steps, 3)
    return {"workload": f"checkpoint shape E=128, top-8, C=3072, F=1280; CFG pair of 2 x {t0} tokens",
            "pair_ms": ms_p, "separate_ms": ms_s, "speedup": ms_s / ms_p, "bit_exact_vs_separate": same,
            "value": t / (ms_p / 1e3), "unit": "tokens/s", "steps": steps}


def run_expert_parallel(args, cfg):
    """N > 1: the layer expert-parallel over the N GPUs of one node (config 4:
    each rank routes its own tokens; gate/up experts sharded 64/N per rank,
    down weights on every rank; NVFP4 rows and scales out, FP4 hidden rows and
    scales back, the down GEMM and the combine on the source rank; by default
    on the copy engines into IPC-mapped peer buffers, ``--transport nccl``
    for NCCL transfers)."""
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
    gu = (torch.randn(e, c, 2 * f, generator=gw, device=dev) * 0.02).to(torch.bfloat16)
    down = (torch.randn(e, f, c, generator=gw, device=dev) * 0.02).to(torch.bfloat16)
    # the whole bank on every rank, for the parity check against one GPU; the
    # expert-parallel layer keeps this rank's shard of the same bytes
    full = pkg.pack_routed_experts(gu, down, keep_on_device=True)
    del gu, down
    names = ("gate_up_q", "gate_up_sf", "gate_up_global", "down_q", "down_sf", "down_global", "_unit_alpha")
    shard = pkg.expert_parallel.shard_packed_state({n: getattr(full, n) for n in names}, rank, world)
    bank = pkg.B200NVFP4RoutedExperts.from_device_state(shard)
    bank.prepare()
    ep = pkg.expert_parallel.ExpertParallelRoutedExperts(bank, e, transport=args.transport, chunks=args.ep_chunks,
                                                         copy_streams=args.copy_streams,
                                                         sm_copy_fraction=args.sm_copy_fraction,
                                                         down_full=(full.down_q, full.down_sf, full.down_global))
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

    # parity: this rank's expert-parallel output against the single-GPU bank
    # on the same tokens and routing, bit for bit (every rank checks its own;
    # the result is all-reduced so rank 0 reports whether all ranks agree)
    logits0, _ = ops.router_logits(x, terms)
    top0, gate0 = ops.route(logits0, bias, k)
    got = ep.routed_forward(x, top0, gate0, scaling=2.5)
    want = full.routed_forward(x, top0, gate0, scaling=2.5, chunk_size=t)
    torch.cuda.synchronize()
    ok = torch.tensor([int(torch.equal(got.view(torch.int16), want.view(torch.int16))),
                       int(pkg.capi.device_error(dev.index) == 0)], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    ep_parity = {"bit_exact_vs_single_gpu_all_ranks": bool(ok[0].item()), "device_error_free": bool(ok[1].item()),
                 "check": "each rank's output vs the single-GPU bank on its tokens (all 64 experts on one GPU)"}
    del got, want, full
    torch.cuda.empty_cache()

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one sampler process for the node (rank 0), not one per rank; it starts
    # (and waits for its first samples) before the barrier, so no rank's
    # timed region holds rank 0's start-up
    clk = ClockSampler(range(world)) if rank == 0 else None
    with clk if clk is not None else contextlib.nullcontext():
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        if clk is not None:
            clk.t0 = time.time()
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
    # bytes this rank's tokens move over NVLink per step: FP4 rows + scales of
    # whole padded tiles to the other ranks' experts, FP4 hidden rows +
    # scales back (and the experts' hidden maxima); by symmetry each
    # direction of a rank's links carries about this much
    blocks = (pc[el::el] - pc[:-1:el]).tolist()
    off = sum(b for d, b in enumerate(blocks) if d != rank)
    # whether every pair of this node's ranks has direct peer access (NVLink
    # P2P); without it the copy engines stage through host memory
    peer = torch.tensor([int(all(torch.cuda.can_device_access_peer(local, j)
                                 for j in range(torch.cuda.device_count()) if j != local))], device=dev)
    dist.all_reduce(peer, op=dist.ReduceOp.MIN)
    peer_ok = bool(peer.item())
    xbytes = torch.tensor([float(off * (c // 2 + c // 16 + f // 2 + f // 16) + 4 * e)], device=dev)
    dist.all_reduce(xbytes, op=dist.ReduceOp.MAX)
    exchange = {"bytes_per_rank_per_step": float(xbytes.item()),
                "gbs_per_rank": float(xbytes.item()) / (ms / 1e3) / 1e9,
                "nvlink_peer_copy_gbs_measured": 770.0,
                "transport": ("copy engines into IPC-mapped peer buffers" if args.transport == "peer" else
                              "NCCL point-to-point") + ": FP4 rows + UE4M3 scales out, FP4 hidden rows + scales "
                             "back, the down GEMM on the source rank",
                "experts_per_rank": el, "sm_copy_fraction": args.sm_copy_fraction,
                "peer_access_all_pairs": peer_ok}
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
        "config": workload_config(cfg, args.config, world),
        "exchange": exchange,
        "ep_parity": ep_parity,
        "layer_tflops": flops * world / (ms / 1e3) / 1e12,
        "roofline": roofline,
        "clocks": clk.summary() if clk is not None else None,
        # router 2, row max 1, dispatch 3, quantize 1; per expert-hidden call (two for the rank's own rows
        # and `chunks` per other source on the peer transport, one and `chunks` on NCCL): tiles 1, gate/up
        # GEMM 1, hidden quantize 1 (+ scale replication 1 for replicated weight scales); the down GEMM 1 and
        # the combine 1 (NCCL's own kernels and the copy engines' copies not counted)
        "gpu_launches": (9 + (3 + int(bank.kernel_weights().gate_up_sf_layout == pkg.capi.SF_REPLICATED))
                         * ((2 if ep.transport == "peer" else 1)
                            + (ep.chunks or (2 if ep.transport == "peer" else 1)) * (world - 1))) * args.steps,
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
    # the same replays with L2 flushed before each one (a 256 MB write outside
    # the events): the cold-cache latency of a layer whose weights were evicted
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    cold = []
    for _ in range(max(10, calls)):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        cold.append(e0.elapsed_time(e1))
    cold.sort()
    del graph, flush
    return {"p50_ms": times[len(times) // 2], "p90_ms": times[(len(times) * 9) // 10], "calls": len(times),
            "euler_steps_per_loop": euler_steps, "capture": "whole layer incl. router in one CUDA graph",
            "l2": "back-to-back replays of the Euler loop reuse the weights (113 MB, L2-resident)",
            "p50_ms_l2_flushed": cold[len(cold) // 2], "p90_ms_l2_flushed": cold[(len(cold) * 9) // 10]}


def read_floor(x, reps=5):
    """A plain read of the layer input (torch's amax reduction, one launch)
    timed like the stages (L2 flushed by a 256 MB write first, CUDA events
    around the launch): what a single launch that only streams these bytes
    reaches, the context for the HBM kernels' fractions of the copy peak."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    total = 0.0
    for rep in range(reps + 1):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(1_000_000)
        e0.record(stream)
        torch.amax(x)
        e1.record(stream)
        torch.cuda.synchronize()
        if rep:
            total += e0.elapsed_time(e1)
    ms = total / reps
    nbytes = x.numel() * x.element_size()
    return {"what": "torch.amax over the layer input (bf16), L2 flushed, CUDA events around the launch",
            "bytes": nbytes, "ms": ms, "gbs": nbytes / (ms / 1e3) / 1e9}


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
    if world > 1:  # every rank starts its timed steps together
        import torch.distributed as dist

        dist.barrier()
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
