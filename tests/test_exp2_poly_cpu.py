"""The FMA-pipe exponential ex2_poly2 (selectssm_b200/csrc/common.cuh) in exact
fp32 arithmetic: constants read from the source, each step rounded like the
kernel rounds it, relative error against float64 over the clamped range."""

import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "selectssm_b200", "csrc", "common.cuh")


def constants():
    text = open(SRC).read()
    c = {k: np.float32(float(v)) for k, v in re.findall(r"(kExp2P\d) = ([0-9.e+-]+)f", text)}
    magic = np.float32(float(re.search(r"kRoundMagic = ([0-9.e+-]+)f", text).group(1)))
    return [c[f"kExp2P{i}"] for i in range(6)], magic


def ex2_poly(x):
    (p0, p1, p2, p3, p4, p5), magic = constants()
    x = np.clip(x.astype(np.float32), np.float32(-126), np.float32(126))
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)

    def fma(a, b, c):  # fp32 fused multiply-add: one rounding of the exact result
        return (a.astype(np.float64) * b.astype(np.float64) + np.float64(c)).astype(np.float32)

    p = fma(np.full_like(f, p5), f, p4)
    for c in (p3, p2, p1, p0):
        p = fma(p, f, c)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_over_range():
    x = np.concatenate([np.linspace(-126, 126, 2_000_001, dtype=np.float32),
                        np.linspace(-0.6, 0.6, 200_001, dtype=np.float32)])
    got = ex2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / ref - 1)) < 3e-7


def test_clamped_ends_are_finite():
    got = ex2_poly(np.array([-1e4, -200.0, 200.0, 1e4], dtype=np.float32))
    assert np.all(np.isfinite(got)) and got[0] > 0 and got[-1] > 1e37
