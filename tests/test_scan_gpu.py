"""Parity of the CUDA scan path (through the C ABI) with the NumPy oracle.

Tolerance (the reference's stated bar): per output tensor,
max|got - ref| / max|ref| <= 1e-4 for float32 inputs and <= 2e-2 for bfloat16
inputs with float32 state.  The oracle runs in float64 on the same inputs (for
bf16 runs, on the bf16-rounded inputs).
"""

import numpy as np
import pytest
import torch

from oracle import selectssm_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def relerr(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


def to_t(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def to_np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def make(batch, L, D, seed, dtype, bias=True):
    inp = O.make_scan_inputs(batch, L, D, 16, seed=seed)
    if bias:
        inp["bias"] = np.random.default_rng(seed + 100).uniform(-0.5, 0.5, D)
    if dtype == torch.bfloat16:  # oracle sees the rounded activations
        for k in ("u", "z", "delta", "B", "C", "dout"):
            inp[k] = to_np(torch.from_numpy(inp[k]).to(torch.bfloat16))
    return inp


SHAPES = [(2, 64, 64), (1, 37, 32), (2, 16, 40), (1, 1, 8), (3, 100, 96), (1, 300, 24)]


@pytest.mark.parametrize("shape", SHAPES)
def test_raw_scan_forward_matches_selectors(cuda, shape):
    """ssm_chunked_scan / ssm_recursive_scan / ssm_scan drop-ins vs the oracle."""
    import selectssm_b200 as S
    Bsz, L, D = shape
    inp = make(Bsz, L, D, 1, torch.float32)
    dt = O.softplus(inp["delta"])
    ref = O.ssm_scan_sequential(inp["u"], inp["A"], inp["B"], inp["C"], dt)
    args = [to_t(inp["u"], cuda), to_t(inp["A"], cuda), to_t(inp["B"], cuda), to_t(inp["C"], cuda),
            to_t(dt, cuda)]
    y1 = S.ssm_chunked_scan(*args, chunk_size=1)
    y2 = S.ssm_recursive_scan(*args)
    y3 = S.ssm_scan(*args)
    for y in (y1, y2, y3):
        assert relerr(to_np(y), ref) < 1e-4


@pytest.mark.parametrize("shape", SHAPES)
def test_raw_scan_backward_matches_custom_vjp(cuda, shape):
    """Gradients of ssm_scan vs the restated custom VJP (ssmrecscan.py:111-181)."""
    import selectssm_b200 as S
    Bsz, L, D = shape
    inp = make(Bsz, L, D, 2, torch.float32)
    dt = O.softplus(inp["delta"])
    ref = O.ssm_scan_backward(inp["u"], inp["A"], inp["B"], inp["C"], dt, inp["dout"])
    ts = [to_t(a, cuda).requires_grad_() for a in (inp["u"], inp["A"], inp["B"], inp["C"], dt)]
    y = S.ssm_scan(*ts)
    y.backward(to_t(inp["dout"], cuda))
    for name, t, r in zip(["dx", "dA", "dB", "dC", "dDelta"], ts, ref):
        assert relerr(to_np(t.grad), r) < 1e-4, name


FUSED_CASES = [
    # (reverse, complement, aligned_skip, gate)
    (False, False, False, "silu"),
    (True, False, False, "silu"),
    (True, True, False, "silu"),
    (True, True, True, "gelu"),
    (False, False, False, "relu"),
    (True, True, False, None),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", FUSED_CASES)
def test_fused_forward_backward(cuda, case, dtype):
    import selectssm_b200 as S
    rev, comp, aligned, gate = case
    Bsz, L, D = 2, 83, 64
    inp = make(Bsz, L, D, 3, dtype)
    kw = dict(D=inp["D"], z=inp["z"] if gate else None, delta_bias=inp["bias"], delta_softplus=True,
              reverse=rev, complement=comp, gate_act=gate or "silu", aligned_skip=aligned)
    ref_out = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    ref = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)
    u = to_t(inp["u"], cuda, dtype).requires_grad_()
    delta = to_t(inp["delta"], cuda, dtype).requires_grad_()
    A = to_t(inp["A"], cuda).requires_grad_()
    Bm = to_t(inp["B"], cuda, dtype).requires_grad_()
    Cm = to_t(inp["C"], cuda, dtype).requires_grad_()
    Dv = to_t(inp["D"], cuda).requires_grad_()
    bias = to_t(inp["bias"], cuda).requires_grad_()
    z = to_t(inp["z"], cuda, dtype).requires_grad_() if gate else None
    out = S.selective_scan(u, delta, A, Bm, Cm, D=Dv, z=z, delta_bias=bias, delta_softplus=True, reverse=rev,
                           complement=comp, gate_act=gate or "silu", aligned_skip=aligned)
    tol = TOL[dtype]
    assert relerr(to_np(out), ref_out) < tol
    out.backward(to_t(inp["dout"], cuda, dtype))
    pairs = [("du", u), ("ddelta", delta), ("dA", A), ("dB", Bm), ("dC", Cm), ("dD", Dv), ("ddelta_bias", bias)]
    if gate:
        pairs.append(("dz", z))
    for name, t in pairs:
        assert relerr(to_np(t.grad), ref[name]) < tol, name


@pytest.mark.parametrize("rev,comp", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("act", ["silu", "gelu", "relu", None])
def test_conv1d_act(cuda, rev, comp, act):
    import selectssm_b200 as S
    Bsz, L, D, K = 2, 301, 48, 4
    rng = np.random.default_rng(5)
    x = rng.standard_normal((Bsz, L, D))
    w = rng.standard_normal((K, D)) * 0.5
    du = rng.standard_normal((Bsz, L, D))
    ref_u = O.conv1d_act_fwd(x, w, act, rev, comp)
    ref_dx, ref_dw = O.conv1d_act_bwd(x, w, du, act, rev, comp)
    xt = to_t(x, cuda).requires_grad_()
    wt = to_t(w[:, None, :], cuda).requires_grad_()
    u = S.conv1d_act(xt, wt, act, rev, comp)
    assert relerr(to_np(u), ref_u) < 1e-5
    u.backward(to_t(du, cuda))
    assert relerr(to_np(xt.grad), ref_dx) < 1e-5
    assert relerr(to_np(wt.grad)[:, 0, :], ref_dw) < 1e-5


@pytest.mark.parametrize("complement", [False, True])
def test_bidir_single_launch(cuda, complement):
    """Both directions in one launch == two single-direction calls, incl. tied z."""
    import selectssm_b200 as S
    Bsz, L, D = 2, 70, 32
    f = make(Bsz, L, D, 7, torch.float32)
    r = make(Bsz, L, D, 8, torch.float32)
    z = f["z"]

    def leaves(d):
        return [to_t(d[k], cuda).requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "bias")]

    lf, lr = leaves(f), leaves(r)
    zt = to_t(z, cuda).requires_grad_()
    out = S.selective_scan_bidir(*lf, zt, *lr, zt, complement=complement)
    dout = np.random.default_rng(9).standard_normal((Bsz, L, 2 * D))
    out.backward(to_t(dout, cuda))
    kwf = dict(D=f["D"], z=z, delta_bias=f["bias"], delta_softplus=True)
    kwr = dict(D=r["D"], z=z, delta_bias=r["bias"], delta_softplus=True, reverse=True, complement=complement)
    ref_f = O.selective_scan_fwd(f["u"], f["delta"], f["A"], f["B"], f["C"], **kwf)
    ref_r = O.selective_scan_fwd(r["u"], r["delta"], r["A"], r["B"], r["C"], **kwr)
    assert relerr(to_np(out[..., :D]), ref_f) < 1e-4
    assert relerr(to_np(out[..., D:]), ref_r) < 1e-4
    gf = O.selective_scan_bwd(f["u"], f["delta"], f["A"], f["B"], f["C"], dout[..., :D], **kwf)
    gr = O.selective_scan_bwd(r["u"], r["delta"], r["A"], r["B"], r["C"], dout[..., D:], **kwr)
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"]
    for name, t in zip(names, lf):
        assert relerr(to_np(t.grad), gf[name]) < 1e-4, name
    for name, t in zip(names, lr):
        assert relerr(to_np(t.grad), gr[name]) < 1e-4, name
    assert relerr(to_np(zt.grad), gf["dz"] + gr["dz"]) < 1e-4


@pytest.mark.parametrize("act_dtype,bc_dtype,gate", [(torch.float32, torch.bfloat16, "none"),
                                                      (torch.bfloat16, torch.float32, "silu"),
                                                      (torch.float32, torch.float32, "none")])
def test_mixed_bc_dtype_and_identity_gate(cuda, act_dtype, bc_dtype, gate):
    """B / C in a different dtype than the activations, and the identity gate
    (y * z); the oracle sees the same rounded inputs."""
    import selectssm_b200 as S
    Bsz, L, D = 2, 77, 48
    inp = make(Bsz, L, D, 11, torch.float32)
    for dt_, keys in ((act_dtype, ("u", "z", "delta", "dout")), (bc_dtype, ("B", "C"))):
        if dt_ == torch.bfloat16:
            for k in keys:
                inp[k] = to_np(torch.from_numpy(inp[k]).to(torch.bfloat16))
    kw = dict(D=inp["D"], z=inp["z"], delta_bias=inp["bias"], delta_softplus=True, gate_act=gate)
    ref_out = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    ref = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)
    ts = {k: to_t(inp[k], cuda, act_dtype).requires_grad_() for k in ("u", "delta", "z")}
    ts.update({k: to_t(inp[k], cuda, bc_dtype).requires_grad_() for k in ("B", "C")})
    ts.update({k: to_t(inp[k], cuda).requires_grad_() for k in ("A", "D", "bias")})
    out = S.selective_scan(ts["u"], ts["delta"], ts["A"], ts["B"], ts["C"], D=ts["D"], z=ts["z"],
                           delta_bias=ts["bias"], delta_softplus=True, gate_act=gate)
    tol = 2e-2 if torch.bfloat16 in (act_dtype, bc_dtype) else 1e-4
    assert relerr(to_np(out), ref_out) < tol
    out.backward(to_t(inp["dout"], cuda, act_dtype))
    for name, k in (("du", "u"), ("ddelta", "delta"), ("dz", "z"), ("dA", "A"), ("dB", "B"), ("dC", "C"),
                    ("dD", "D"), ("ddelta_bias", "bias")):
        assert ts[k].grad.dtype == ts[k].dtype
        assert relerr(to_np(ts[k].grad), ref[name]) < tol, name


def test_bidir_gate_on_one_direction(cuda):
    """Forward direction gated by z, reverse direction ungated: the backward
    runs one launch per gate and must still match the oracle."""
    import selectssm_b200 as S
    Bsz, L, D = 1, 90, 32
    f = make(Bsz, L, D, 21, torch.float32)
    r = make(Bsz, L, D, 22, torch.float32)

    def leaves(d):
        return [to_t(d[k], cuda).requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "bias")]

    lf, lr = leaves(f), leaves(r)
    zt = to_t(f["z"], cuda).requires_grad_()
    out = S.selective_scan_bidir(*lf, zt, *lr, None, complement=True)
    dout = np.random.default_rng(23).standard_normal((Bsz, L, 2 * D))
    out.backward(to_t(dout, cuda))
    kwf = dict(D=f["D"], z=f["z"], delta_bias=f["bias"], delta_softplus=True)
    kwr = dict(D=r["D"], z=None, delta_bias=r["bias"], delta_softplus=True, reverse=True, complement=True)
    assert relerr(to_np(out[..., :D]), O.selective_scan_fwd(f["u"], f["delta"], f["A"], f["B"], f["C"], **kwf)) < 1e-4
    assert relerr(to_np(out[..., D:]), O.selective_scan_fwd(r["u"], r["delta"], r["A"], r["B"], r["C"], **kwr)) < 1e-4
    gf = O.selective_scan_bwd(f["u"], f["delta"], f["A"], f["B"], f["C"], dout[..., :D], **kwf)
    gr = O.selective_scan_bwd(r["u"], r["delta"], r["A"], r["B"], r["C"], dout[..., D:], **kwr)
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias"]
    for name, t in zip(names, lf):
        assert relerr(to_np(t.grad), gf[name]) < 1e-4, name
    for name, t in zip(names, lr):
        assert relerr(to_np(t.grad), gr[name]) < 1e-4, name
    assert relerr(to_np(zt.grad), gf["dz"]) < 1e-4


def test_empty_inputs(cuda):
    import selectssm_b200 as S
    for shape in [(0, 16, 32), (2, 0, 32)]:
        u = torch.zeros(shape, device=cuda, requires_grad=True)
        A = -torch.ones(32, 16, device=cuda, requires_grad=True)
        Bm = torch.zeros(shape[0], shape[1], 16, device=cuda, requires_grad=True)
        y = S.selective_scan(u, u, A, Bm, Bm)
        assert y.shape == shape
        y.sum().backward()
        assert A.grad is None or bool(torch.all(A.grad == 0))


def test_long_sequence_states_roundtrip(cuda):
    """Forward at a length well past the 16-step chunk: last outputs still match,
    so the carried state is exact across hundreds of chunks."""
    import selectssm_b200 as S
    Bsz, L, D = 1, 4096, 32
    inp = make(Bsz, L, D, 11, torch.float32)
    dt = O.softplus(inp["delta"])
    ref = O.ssm_scan_sequential(inp["u"], inp["A"], inp["B"], inp["C"], dt)
    y = S.ssm_chunked_scan(to_t(inp["u"], cuda), to_t(inp["A"], cuda), to_t(inp["B"], cuda), to_t(inp["C"], cuda),
                           to_t(dt, cuda))
    assert relerr(to_np(y), ref) < 1e-4


@pytest.mark.parametrize("rev,comp", [(False, False), (True, True)])
def test_segmented_long_sequence_fwd_bwd(cuda, rev, comp):
    """Few channels and a long sequence: the kernels cut the sequence into
    concurrent segments joined by carried states / adjoints."""
    import selectssm_b200 as S
    Bsz, L, D = 1, 1100, 64
    inp = make(Bsz, L, D, 21, torch.float32)
    kw = dict(D=inp["D"], z=inp["z"], delta_bias=inp["bias"], delta_softplus=True, reverse=rev, complement=comp)
    ref_out = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    ref = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)
    t = {k: to_t(inp[k], cuda).requires_grad_() for k in ("u", "delta", "A", "B", "C", "D", "bias", "z")}
    out = S.selective_scan(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_bias=t["bias"],
                           delta_softplus=True, reverse=rev, complement=comp)
    assert relerr(to_np(out), ref_out) < 1e-4
    out.backward(to_t(inp["dout"], cuda))
    for name, key in (("du", "u"), ("ddelta", "delta"), ("dA", "A"), ("dB", "B"), ("dC", "C"), ("dD", "D"),
                      ("ddelta_bias", "bias"), ("dz", "z")):
        assert relerr(to_np(t[key].grad), ref[name]) < 1e-4, name
