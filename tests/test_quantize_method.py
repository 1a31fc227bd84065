"""The quantize kernels' division-free scale path, emulated on the CPU with
IEEE float32 arithmetic (numpy) and checked against the recipe's two
divisions (praxis/kernels/nvfp4.py:44-124: sf = e4m3(clamp(div_rn(bs, g),
2^-6, 448)), rc = div_rn(div_rn(1, g), sf)) on random and adversarial
inputs: every e4m3 rounding midpoint of the normal range approached to
within a few ulps from both sides, global scales across the range the
recipe produces, and the clamp bounds.

The kernel (csrc/quantize.cu, quantize16_fast): q = bs * inv_g, the exact
division only when q's 20 dropped bits are within 16 ulps of 0x80000;
rc = 2^(7 - E) * div_rn(inv_g, 1 + m/8) through the exponent bits.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import nvfp4_moe_oracle as O

F32 = np.float32
SIXTH = F32(1.0) / F32(6.0)


def e4m3_byte(q: np.ndarray) -> np.ndarray:
    c = np.clip(q, F32(0.015625), F32(448.0)).astype(F32)
    return O.e4m3_bytes(torch.from_numpy(c)).numpy().astype(np.uint32)


def e4m3_value(b: np.ndarray) -> np.ndarray:
    return O.e4m3_values(torch.from_numpy(b.astype(np.uint8))).numpy().astype(F32)


def reference(bs, g):
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        sf = e4m3_byte((bs / g).astype(F32))
        rc = ((F32(1.0) / g).astype(F32) / e4m3_value(sf)).astype(F32)
    return sf, rc


def fast(bs, g):
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        inv_g = (F32(1.0) / g).astype(F32)
        q = (bs * inv_g).astype(F32)
        dropped = q.view(np.uint32) & np.uint32(0xFFFFF)
        near = (dropped - np.uint32(0x80000 - 16)).astype(np.uint32) <= np.uint32(32)
        q = np.where(near, (bs / g).astype(F32), q)
        sf = e4m3_byte(q)
        m = (sf & 7).astype(F32)
        r8 = (inv_g / (F32(1.0) + F32(0.125) * m)).astype(F32)
        e = (sf >> 3).astype(np.int64) - 7
        rc = (r8.view(np.uint32).astype(np.int64) - e * (1 << 23)).astype(np.uint32).view(F32)
    return sf, rc, near


def globals_from(amax_bf16: np.ndarray) -> np.ndarray:
    return O.global_scale_from_amax(torch.from_numpy(amax_bf16).to(torch.bfloat16)).numpy().astype(F32)


def bs_from(amax: np.ndarray) -> np.ndarray:
    a = torch.from_numpy(amax.astype(F32)).to(torch.bfloat16).float().numpy()
    return (a * SIXTH).astype(F32)


def check(bs, g):
    sf_r, rc_r = reference(bs, g)
    sf_f, rc_f, near = fast(bs, g)
    bad = np.nonzero((sf_r != sf_f) | (rc_r.view(np.uint32) != rc_f.view(np.uint32)))[0]
    assert bad.size == 0, (bs[bad[:5]], g[bad[:5]], sf_r[bad[:5]], sf_f[bad[:5]])
    return near


def test_random_blocks_and_global_scales():
    rng = np.random.default_rng(0)
    n = 400_000
    g = globals_from(np.exp(rng.uniform(np.log(1e-6), np.log(3e4), n)).astype(F32))
    amax = np.exp(rng.uniform(np.log(1e-8), np.log(6e4), n)).astype(F32)
    bs = bs_from(amax)
    near = check(bs, g)
    # the exact division is rare: bf16 block maxima over bf16-derived global
    # scales land near a midpoint for about 0.5 % of the blocks
    assert near.mean() < 1e-2


def test_every_e4m3_midpoint_from_both_sides():
    """For every pair of neighbouring normal e4m3 values (and the clamp
    bounds), global scales that put bs / g within +-40 ulps of their
    midpoint, for several bs."""
    vals = e4m3_value(np.arange(0x08, 0x7F, dtype=np.uint32))
    mids = ((vals[:-1].astype(np.float64) + vals[1:]) / 2).astype(F32)
    targets = np.concatenate([mids, vals, [F32(0.015625), F32(448.0), F32(0.0155), F32(450.0)]]).astype(F32)
    rng = np.random.default_rng(1)
    bs = bs_from(np.exp(rng.uniform(np.log(1e-3), np.log(1e3), 64)).astype(F32))
    gs, bss = [], []
    for b in bs:
        g0 = (np.float64(b) / targets.astype(np.float64)).astype(F32)
        for k in range(-40, 41):
            gs.append((g0.view(np.uint32).astype(np.int64) + k).astype(np.uint32).view(F32))
            bss.append(np.full(g0.shape, b, dtype=F32))
    g = np.concatenate(gs)
    bsa = np.concatenate(bss)
    ok = np.isfinite(g) & (g > 0)
    near = check(bsa[ok], g[ok])
    assert near.any()  # the division path was exercised


def test_extremes_of_the_global_scale_range():
    """The smallest and largest global scales the recipe produces (amax
    clamped at 1e-12, bf16 max), with block maxima across the range, the
    reciprocal's exponent arithmetic stays exact (no subnormal result)."""
    g = globals_from(np.array([1e-12, 1e-10, 3.3895314e38, 1e30, 1.0], dtype=F32))
    amax = np.exp(np.linspace(np.log(1e-30), np.log(3e38), 2000)).astype(F32)
    bs = bs_from(amax)
    gg = np.repeat(g, bs.size)
    bb = np.tile(bs, g.size)
    keep = np.isfinite(bb)
    check(bb[keep], gg[keep])
