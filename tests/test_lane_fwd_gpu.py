"""Parity of the one-lane-per-channel forward (ssm_fwd_lane_kernel) with the oracle.

The library runs that kernel for single-direction, forward-frame calls with
softplus(dt) whose length is whole 16-step chunks, whose channels fill whole
128-channel tiles and whose batch x channels is at least 65536 (enough channels
to fill the GPU one lane each).  Every case below meets those conditions, so its
forward (the output and the checkpoints the backward restarts from) comes from
that kernel.  Channels are independent given B and C, so the full-size run is
compared with the oracle on a complement-closed channel subset.

Tolerances: max|got-ref|/max|ref| <= 1e-4 for fp32 I/O, 2e-2 for bf16 I/O.
"""

import numpy as np
import pytest
import torch

from oracle import selectssm_oracle as O

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def rel(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


def npy(t):
    return t.detach().double().cpu().numpy()


def gen(Bsz, L, D, dtype, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)

    def n(*s):
        return torch.randn(*s, generator=g, device=dev)
    t = {"u": n(Bsz, L, D), "z": n(Bsz, L, D), "delta": n(Bsz, L, D) - 4.0, "dout": n(Bsz, L, D),
         "A": -(1.0 + 15.0 * torch.rand(D, 16, generator=g, device=dev)), "B": n(Bsz, L, 16), "C": n(Bsz, L, 16),
         "D": 1.0 + 0.1 * n(D), "bias": 0.1 * n(D)}
    for k in ("u", "z", "delta", "dout", "B", "C"):
        t[k] = t[k].to(dtype)
    return t


def channels(D, k=4):
    return torch.cat([torch.arange(k), torch.arange(D // 2 - k, D // 2 + k), torch.arange(D - k, D)])


@pytest.mark.parametrize("dtype,gate,skip,bias", [
    (torch.float32, "silu", True, True),
    (torch.float32, None, False, False),
    (torch.float32, "gelu", True, False),
    (torch.float32, "relu", False, True),
    (torch.float32, "none", True, True),
    (torch.bfloat16, "silu", True, True),
])
def test_lane_forward_backward_vs_oracle(cuda, dtype, gate, skip, bias):
    import selectssm_b200 as S
    Bsz, L, D = 64, 48, 1024
    assert Bsz * D >= 65536 and L % 16 == 0 and D % 128 == 0
    t = gen(Bsz, L, D, dtype, 11, cuda)
    keys = ["u", "delta", "A", "B", "C"] + (["z"] if gate else []) + (["D"] if skip else []) + \
        (["bias"] if bias else [])
    leaves = {k: t[k].detach().clone().requires_grad_() for k in keys}
    out = S.selective_scan(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], D=leaves.get("D"),
                           z=leaves.get("z"), delta_bias=leaves.get("bias"), delta_softplus=True,
                           gate_act=gate or "silu")
    out.backward(t["dout"])
    torch.cuda.synchronize()
    idx = channels(D).to(cuda)
    a = {k: npy(t[k].index_select(-1, idx) if t[k].dim() == 3 and k not in ("B", "C") else
                (t[k].index_select(0, idx) if k in ("A", "D", "bias") else t[k])) for k in t}
    kw = dict(D=a["D"] if skip else None, z=a["z"] if gate else None, delta_bias=a["bias"] if bias else None,
              delta_softplus=True, gate_act=gate or "silu")
    ref = O.selective_scan_fwd(a["u"], a["delta"], a["A"], a["B"], a["C"], **kw)
    g = O.selective_scan_bwd(a["u"], a["delta"], a["A"], a["B"], a["C"], a["dout"], **kw)
    tol = TOL[dtype]
    assert rel(npy(out.index_select(-1, idx)), ref) < tol, "out"
    pairs = [("du", "u"), ("ddelta", "delta"), ("dA", "A")] + ([("dz", "z")] if gate else []) + \
        ([("dD", "D")] if skip else []) + ([("ddelta_bias", "bias")] if bias else [])
    for name, k in pairs:
        got = leaves[k].grad.index_select(-1 if k in ("u", "delta", "z") else 0, idx)
        assert rel(npy(got), g[name]) < tol, name


def test_lane_forward_matches_small_batch_kernel(cuda):
    """The lane kernel's output on a batch equals the per-row runs of the
    quad-per-channel kernel (a single row is below the lane threshold)."""
    import selectssm_b200 as S
    Bsz, L, D = 64, 64, 1024
    t = gen(Bsz, L, D, torch.float32, 3, cuda)
    with torch.no_grad():
        full = S.selective_scan(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"],
                                delta_bias=t["bias"], delta_softplus=True)
        for b in (0, 17, 63):
            one = S.selective_scan(t["u"][b:b + 1], t["delta"][b:b + 1], t["A"], t["B"][b:b + 1], t["C"][b:b + 1],
                                   D=t["D"], z=t["z"][b:b + 1], delta_bias=t["bias"], delta_softplus=True)
            err = float((full[b:b + 1] - one).abs().max() / one.abs().max())
            assert err < 1e-5, (b, err)
