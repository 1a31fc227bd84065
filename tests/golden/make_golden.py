"""Generate the golden fixtures of ``tests/golden/*.pt`` from the reference.

Run in a container that holds the reference checkout (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/praxis-1-oss

It imports the reference's own CPU code and records what it computes on
seeded inputs. Inputs are regenerated from their seeds by the tests, so the
fixtures hold the seeds, a SHA-256 of the generated input bytes, and the
reference's outputs:

* routing   ``MoEFeedForward._route`` (praxis/layers.py:1632-1655): sigmoid
            router in float32, expert bias, torch.topk, renormalised gates;
* dispatch  ``_dispatch_rows`` (praxis/layers.py:1330-1346) and the inverse
            permutation (praxis/quantization/nvfp4.py:705-708);
* scales    ``expert_global_scales`` (praxis/kernels/nvfp4.py:154-194, its
            CPU branch) on the reference test's counts with empty experts;
* combine   ``_sum_rows_of_tokens`` (praxis/layers.py:1349-1364);
* layer     the bf16 ``MoEFeedForward.forward`` on the CPU (a small shape;
            parameters regenerated from the seed in ``named_parameters``
            order), a loose sanity target for the NVFP4 path.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def routing_inputs(seed: int, tokens: int, dim: int, experts: int, bias_scale: float):
    """Seeded router inputs (the tests rebuild them with this same function)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, dim, generator=g).to(torch.bfloat16)
    w = (torch.randn(experts, dim, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.randn(experts, generator=g) * bias_scale
    return x, w, bias


ROUTING_CASES = [
    # name, seed, tokens, dim, experts, top_k, bias_scale
    ("cfg1_e8_k2", 0, 256, 512, 8, 2, 0.0),
    ("e64_k4_bias", 1, 192, 256, 64, 4, 0.05),
    ("e128_k8_bias", 2, 96, 256, 128, 8, 0.05),
    ("e32_k2", 3, 128, 256, 32, 2, 0.0),
]


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    os.environ.setdefault("PRAXIS_NVTX", "0")
    from praxis import layers
    from praxis.kernels.nvfp4 import expert_global_scales
    from praxis.layers import MoEFeedForward, _dispatch_rows, _sum_rows_of_tokens

    torch.set_num_threads(1)
    out: dict = {"routing": {}, "dispatch": {}, "scales": {}, "combine": {}, "layer": {}}
    for name, seed, tokens, dim, experts, k, bias_scale in ROUTING_CASES:
        x, w, bias = routing_inputs(seed, tokens, dim, experts, bias_scale)
        moe = MoEFeedForward(dim, 128, experts, k, 2.5, dispatch_chunk_size=tokens)
        with torch.no_grad():
            moe.router.weight.copy_(w.float())
            moe.expert_bias.copy_(bias)
            logits = layers._router_logits(moe.router.weight, x)
            top_idx, gate = moe._route(x)
        order, tok, sorted_gate, offsets = _dispatch_rows(top_idx, gate, experts)
        inverse = torch.empty_like(order)
        inverse[order] = torch.arange(order.numel())
        out["routing"][name] = dict(
            seed=seed, tokens=tokens, dim=dim, experts=experts, top_k=k,
            bias_scale=bias_scale, x_sha=sha(x), w_sha=sha(w), bias_sha=sha(bias),
            logits=logits, top_idx=top_idx, gate=gate,
        )
        out["dispatch"][name] = dict(
            order=order, tokens=tok, sorted_gate=sorted_gate, offsets=offsets,
            inverse=inverse,
        )

    # Concentrated routing (tests/test_moe_dispatch.py:37-54 style): most
    # rows on one expert, one expert empty.
    g = torch.Generator().manual_seed(7)
    top = torch.randint(0, 16, (200, 4), generator=g)
    top[:150, 0] = 5
    top[top == 9] = 10
    gate = torch.rand(200, 4, generator=g).to(torch.bfloat16)
    order, tok, sorted_gate, offsets = _dispatch_rows(top, gate, 16)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel())
    out["dispatch"]["concentrated"] = dict(
        top_idx=top, gate=gate, order=order, tokens=tok, sorted_gate=sorted_gate,
        offsets=offsets, inverse=inverse,
    )

    # Global activation scales (tests/test_nvfp4.py:566-632 inputs).
    g = torch.Generator().manual_seed(0)
    counts = torch.tensor([0, 5, 3, 0, 9, 1, 4, 0])
    offsets = counts.cumsum(0).to(torch.int32)
    csr = torch.nn.functional.pad(offsets, (1, 0))
    rows_total = int(counts.sum())
    x = (torch.randn(rows_total, 256, generator=g) * 30).to(torch.bfloat16)
    tokens = torch.randint(0, rows_total, (rows_total,), generator=g)
    out["scales"]["gather"] = dict(
        x=x, csr=csr, tokens=tokens, result=expert_global_scales(x, csr, tokens)
    )
    out["scales"]["plain"] = dict(x=x, csr=csr, result=expert_global_scales(x, csr, None))
    rows = torch.zeros(3, 128, dtype=torch.bfloat16)
    csr0 = torch.tensor([0, 0, 2, 3], dtype=torch.int32)
    out["scales"]["all_zero"] = dict(x=rows, csr=csr0, result=expert_global_scales(rows, csr0))
    rows = torch.tensor([2, 4, 8, 16, 32, 64], dtype=torch.bfloat16)[:, None].expand(-1, 128).contiguous()
    csr1 = torch.tensor([0, 1, 2, 2], dtype=torch.int32)
    out["scales"]["trailing"] = dict(x=rows, csr=csr1, result=expert_global_scales(rows, csr1))

    # Combine order (tests/test_nvfp4.py:888-904 / test_moe_chunked.py:17-33).
    for k in (2, 4, 8):
        g = torch.Generator().manual_seed(100 + k)
        t = 9
        vals = torch.randn(t * k, 160, generator=g).to(torch.bfloat16)
        inverse = torch.randperm(t * k, generator=g)
        scale = torch.randn(t * k, generator=g).to(torch.bfloat16).float() * 2.5
        out["combine"][f"k{k}"] = dict(
            rows=vals, inverse=inverse, scale=scale,
            result=_sum_rows_of_tokens(vals, inverse.view(t, k), scale[inverse].view(t, k)),
        )

    # The bf16 reference layer on the config-1 shape (sanity only).
    g = torch.Generator().manual_seed(11)
    t, c, e, k, f = 64, 256, 8, 2, 256
    moe = MoEFeedForward(c, f, e, k, 2.5, dispatch_chunk_size=t)
    with torch.no_grad():
        for p in moe.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)
        moe = moe.to(torch.bfloat16)
        x = torch.randn(t, c, generator=g).to(torch.bfloat16)
        y = moe(x)
        y_shared = moe.shared(x)
    out["layer"]["bf16_t64"] = dict(
        seed=11, shape=(t, c, e, k, f),
        param_order=[n for n, _ in moe.named_parameters()],
        state_sha={n: sha(v) for n, v in moe.state_dict().items()},
        x_sha=sha(x), y=y, shared=y_shared, top_k=k, scaling=2.5,
    )
    torch.save(out, HERE / "reference_cpu.pt")
    print("wrote", HERE / "reference_cpu.pt", (HERE / "reference_cpu.pt").stat().st_size, "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PRAXIS_REFERENCE", "."))
