"""Generates the golden fixtures in tests/golden/ from the NumPy oracle.

The reference (JAX/Flax) cannot run on this image, so these fixtures freeze the
oracle's float64 outputs on seeded inputs; tests check the oracle against them
(regression pin) and the CUDA path against the same inputs.  Cases:

  raw_scan.npz      raw scan forward (chunked selector, default chunk rule) and the
                    custom-VJP gradients, batch=2, L=64, D=32, N=16
  fused_rev.npz     fused op (softplus, bias, D skip, silu gate) with
                    reverse=True, complement=True, forward + all gradients
  selective_ssm.npz SelectiveSSM forward (config-1 layout at L=64: d_inner=128,
                    K=4, dt_rank=4, log-uniform dt init)

Run: python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import selectssm_oracle as O  # noqa: E402


def raw_scan():
    inp = O.make_scan_inputs(2, 64, 32, 16, seed=0)
    dt = O.softplus(inp["delta"])
    y = O.ssm_chunked_scan(inp["u"], inp["A"], inp["B"], inp["C"], dt)
    dx, dA, dB, dC, ddt = O.ssm_scan_backward(inp["u"], inp["A"], inp["B"], inp["C"], dt, inp["dout"])
    return dict(x=inp["u"], A=inp["A"], B=inp["B"], C=inp["C"], dt=dt, dy=inp["dout"], y=y, dx=dx, dA=dA,
                dB=dB, dC=dC, ddt=ddt)


def fused_rev():
    inp = O.make_scan_inputs(2, 48, 32, 16, seed=1)
    bias = np.random.default_rng(101).uniform(-0.5, 0.5, 32)
    kw = dict(D=inp["D"], z=inp["z"], delta_bias=bias, delta_softplus=True, reverse=True, complement=True)
    out = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    g = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)
    res = dict(u=inp["u"], delta=inp["delta"], A=inp["A"], B=inp["B"], C=inp["C"], D=inp["D"], z=inp["z"],
               bias=bias, dout=inp["dout"], out=out)
    res.update({k: v for k, v in g.items() if v is not None})
    return res


def selective_ssm():
    D, L = 128, 64
    params = O.make_selective_ssm_params(D, 16, dt_rank=4, conv_size=4, seed=0, log_uniform_dt=True)
    x = np.random.default_rng(0).standard_normal((2, L, D))
    y = O.selective_ssm_fwd(params, x)
    yr = O.selective_ssm_fwd(params, x, reverse=True, complement=True)
    flat = {"x": x, "y": y, "y_rev_comp": yr}
    flat["shift_conv_kernel"] = params["shift_conv"]["kernel"]
    flat["A_log"] = params["A_log"]
    flat["BC_kernel"], flat["BC_bias"] = params["BC"]["kernel"], params["BC"]["bias"]
    flat["D"] = params["D"]
    flat["dt_kernel"], flat["dt_bias"] = params["dt"]["kernel"], params["dt"]["bias"]
    flat["dt_proj_kernel"], flat["dt_proj_bias"] = params["dt_proj"]["kernel"], params["dt_proj"]["bias"]
    return flat


def main():
    for name, fn in (("raw_scan", raw_scan), ("fused_rev", fused_rev), ("selective_ssm", selective_ssm)):
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **fn())
        print("wrote", name)


if __name__ == "__main__":
    main()
