"""Seeded sweep of irregular shapes and flag combinations through the fused
op, forward and backward, against the NumPy oracle: channel counts that are
not multiples of the CTA tiles, lengths that are not multiples of the 16-step
stage or the 8-step checkpoint, long enough sequences to be cut into
segments, every dtype combination, reverse / complement / aligned skip and
every gate."""

import numpy as np
import pytest
import torch

from oracle import selectssm_oracle as O

pytestmark = pytest.mark.gpu

F32, BF16 = torch.float32, torch.bfloat16
ACTS = ["silu", "gelu", "relu", "none", None]


def cases(n=24, seed=2024):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        bf16_act = bool(rng.integers(2))
        dim = int(rng.choice([8, 24, 40, 136, 200, 264])) if not bf16_act else int(rng.choice([8, 24, 40, 136, 264]))
        out.append(dict(batch=int(rng.integers(1, 4)), L=int(rng.choice([1, 7, 9, 17, 33, 250, 777, 1300])),
                        dim=dim, act_dtype=BF16 if bf16_act else F32, bc_dtype=BF16 if rng.integers(2) else F32,
                        reverse=bool(rng.integers(2)), complement=bool(rng.integers(2)),
                        aligned=bool(rng.integers(3) == 0), gate=ACTS[int(rng.integers(len(ACTS)))],
                        has_D=bool(rng.integers(4)), has_bias=bool(rng.integers(2)), softplus=bool(rng.integers(4)),
                        seed=i))
    return out


def to_np(t):
    return t.detach().double().cpu().numpy()


def rel(a, b):
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.parametrize("c", cases(), ids=lambda c: "b{batch}_L{L}_d{dim}".format(**c))
def test_sweep(cuda, c):
    import selectssm_b200 as S
    inp = O.make_scan_inputs(c["batch"], c["L"], c["dim"], 16, seed=100 + c["seed"])
    inp["bias"] = np.random.default_rng(c["seed"]).uniform(-0.5, 0.5, c["dim"])
    if not c["softplus"]:  # keep dt = delta + bias positive without the softplus (a decaying recurrence)
        inp["delta"] = np.abs(inp["delta"]) * 0.05
        inp["bias"] = np.abs(inp["bias"]) * 0.1
    for keys, dt in ((("u", "z", "delta", "dout"), c["act_dtype"]), (("B", "C"), c["bc_dtype"])):
        if dt == BF16:
            for k in keys:
                inp[k] = to_np(torch.from_numpy(inp[k]).to(BF16))
    comp = c["complement"] and c["reverse"]
    kw = dict(D=inp["D"] if c["has_D"] else None, z=inp["z"] if c["gate"] else None,
              delta_bias=inp["bias"] if c["has_bias"] else None, delta_softplus=c["softplus"],
              reverse=c["reverse"], complement=comp, gate_act=c["gate"] or "silu", aligned_skip=c["aligned"])
    ref_out = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    ref = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)

    def t(k, dt=F32):
        return torch.from_numpy(np.ascontiguousarray(inp[k])).to(device=cuda, dtype=dt).requires_grad_()

    u, delta, z = t("u", c["act_dtype"]), t("delta", c["act_dtype"]), t("z", c["act_dtype"])
    Bm, Cm = t("B", c["bc_dtype"]), t("C", c["bc_dtype"])
    A, Dv, bias = t("A"), t("D"), t("bias")
    out = S.selective_scan(u, delta, A, Bm, Cm, D=Dv if c["has_D"] else None, z=z if c["gate"] else None,
                           delta_bias=bias if c["has_bias"] else None, delta_softplus=c["softplus"],
                           reverse=c["reverse"], complement=comp, gate_act=c["gate"] or "silu",
                           aligned_skip=c["aligned"])
    tol = 2e-2 if BF16 in (c["act_dtype"], c["bc_dtype"]) else 1e-4
    assert rel(to_np(out), ref_out) < tol, "out"
    out.backward(torch.from_numpy(np.ascontiguousarray(inp["dout"])).to(device=cuda, dtype=c["act_dtype"]))
    pairs = [("du", u), ("ddelta", delta), ("dA", A), ("dB", Bm), ("dC", Cm)]
    if c["has_D"]:
        pairs.append(("dD", Dv))
    if c["has_bias"]:
        pairs.append(("ddelta_bias", bias))
    if c["gate"]:
        pairs.append(("dz", z))
    for name, x in pairs:
        assert rel(to_np(x.grad), ref[name]) < tol, name
