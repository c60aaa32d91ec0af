"""The NumPy oracle against itself, finite differences and the golden fixtures (CPU)."""

import os

import numpy as np
import pytest

from oracle import selectssm_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-300)


def test_chunk_size_rule():
    # selectssm.py:50-51 on the benchmark lengths
    assert O.default_chunk_size(1024) == 32
    assert O.default_chunk_size(131072) == 256
    assert O.default_chunk_size(2048) == 32
    assert O.default_chunk_size(4096) == 64
    assert O.default_chunk_size(1) == 1
    assert O.default_chunk_size(37) == 1  # prime length: chunks of one step
    assert O.largest_factor_up_to(10, 1) == 1


def test_chunked_valueerrors():
    with pytest.raises(ValueError):
        O.check_chunked_args(64, 30, None, 4)      # K does not divide D
    with pytest.raises(ValueError):
        O.check_chunked_args(64, 32, 7, 1)         # chunk does not divide L


@pytest.mark.parametrize("shape", [(2, 24, 8), (1, 37, 4), (3, 16, 6)])
def test_selectors_agree(shape):
    B, L, D = shape
    inp = O.make_scan_inputs(B, L, D, 16, seed=3)
    dt = O.softplus(inp["delta"] + 2)
    y0 = O.ssm_scan_sequential(inp["u"], inp["A"], inp["B"], inp["C"], dt)
    ys = [O.ssm_chunked_scan(inp["u"], inp["A"], inp["B"], inp["C"], dt),
          O.ssm_recursive_scan(inp["u"], inp["A"], inp["B"], inp["C"], dt),
          O.ssm_recursive_scan(inp["u"], inp["A"], inp["B"], inp["C"], dt, 3, 2)]
    if D % 2 == 0 and L % 4 == 0:
        ys.append(O.ssm_chunked_scan(inp["u"], inp["A"], inp["B"], inp["C"], dt, chunk_size=4, n_channel_groups=2))
    for y in ys:
        assert rel(y, y0) < 1e-12


def test_custom_vjp_vs_finite_differences():
    inp = O.make_scan_inputs(1, 12, 3, 16, seed=4)
    dt = O.softplus(inp["delta"] + 2)
    args = [inp["u"], inp["A"], inp["B"], inp["C"], dt]
    dy = inp["dout"]
    g = O.ssm_scan_backward(*args, dy)

    def loss(*a):
        return (O.ssm_scan_sequential(*a) * dy).sum()

    rng = np.random.default_rng(0)
    for i in range(5):
        a = args[i]
        for _ in range(6):
            idx = tuple(rng.integers(0, s) for s in a.shape)
            ap = [x.copy() for x in args]
            am = [x.copy() for x in args]
            ap[i][idx] += 1e-6
            am[i][idx] -= 1e-6
            num = (loss(*ap) - loss(*am)) / 2e-6
            assert abs(num - g[i][idx]) <= 1e-6 * max(1.0, abs(num))


def test_custom_vjp_recursion_levels_agree():
    inp = O.make_scan_inputs(2, 32, 4, 16, seed=5)
    dt = O.softplus(inp["delta"])
    a = O.ssm_scan_backward(inp["u"], inp["A"], inp["B"], inp["C"], dt, inp["dout"])
    b = O.ssm_scan_backward(inp["u"], inp["A"], inp["B"], inp["C"], dt, inp["dout"], min_recursion_length=100)
    c = O.ssm_scan_backward(inp["u"], inp["A"], inp["B"], inp["C"], dt, inp["dout"], 4, 4)
    for x, y, z in zip(a, b, c):
        assert rel(x, y) < 1e-12 and rel(x, z) < 1e-12


def test_golden_raw_scan():
    g = np.load(os.path.join(GOLD, "raw_scan.npz"))
    y = O.ssm_chunked_scan(g["x"], g["A"], g["B"], g["C"], g["dt"])
    assert rel(y, g["y"]) < 1e-12
    grads = O.ssm_scan_backward(g["x"], g["A"], g["B"], g["C"], g["dt"], g["dy"])
    for name, v in zip(["dx", "dA", "dB", "dC", "ddt"], grads):
        assert rel(v, g[name]) < 1e-12, name


def test_golden_fused_reverse_complement():
    g = np.load(os.path.join(GOLD, "fused_rev.npz"))
    kw = dict(D=g["D"], z=g["z"], delta_bias=g["bias"], delta_softplus=True, reverse=True, complement=True)
    out = O.selective_scan_fwd(g["u"], g["delta"], g["A"], g["B"], g["C"], **kw)
    assert rel(out, g["out"]) < 1e-12
    r = O.selective_scan_bwd(g["u"], g["delta"], g["A"], g["B"], g["C"], g["dout"], **kw)
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias", "dz"):
        assert rel(r[k], g[k]) < 1e-12, k


def test_golden_selective_ssm():
    g = np.load(os.path.join(GOLD, "selective_ssm.npz"))
    params = {"shift_conv": {"kernel": g["shift_conv_kernel"]}, "A_log": g["A_log"],
              "BC": {"kernel": g["BC_kernel"], "bias": g["BC_bias"]}, "D": g["D"],
              "dt": {"kernel": g["dt_kernel"], "bias": g["dt_bias"]},
              "dt_proj": {"kernel": g["dt_proj_kernel"], "bias": g["dt_proj_bias"]}}
    assert rel(O.selective_ssm_fwd(params, g["x"]), g["y"]) < 1e-12
    assert rel(O.selective_ssm_fwd(params, g["x"], reverse=True, complement=True), g["y_rev_comp"]) < 1e-12
    # the three selectors agree on the module too
    for scan in ("recursive", "sequential"):
        assert rel(O.selective_ssm_fwd(params, g["x"], scan=scan), g["y"]) < 1e-12


def test_reverse_skip_frame_quirk():
    """selectssm.py:230-238: the reverse SSM adds the flipped-frame u unflipped, so
    out[l] = y_scan[L-1-l] + u_flip[l] * D, which differs from flipping the skip."""
    inp = O.make_scan_inputs(1, 10, 4, 16, seed=6)
    kw = dict(D=inp["D"], delta_softplus=True, reverse=True)
    a = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], **kw)
    b = O.selective_scan_fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], aligned_skip=True, **kw)
    dt = O.softplus(inp["delta"])
    ys = O.ssm_scan_sequential(inp["u"], inp["A"], inp["B"], inp["C"], dt)
    assert rel(a, ys[:, ::-1] + inp["u"] * inp["D"]) < 1e-12
    assert rel(b, (ys + inp["u"] * inp["D"])[:, ::-1]) < 1e-12
    assert rel(a, b) > 1e-3


def test_carry_helpers_match_sequential():
    """The chunked final-state and adjoint-carry helpers equal the per-step
    recurrences (forward_scan_fn / backward_scan_fn, ssmrecscan.py:90-100)."""
    inp = O.make_scan_inputs(2, 200, 5, 16, seed=7)
    dt = O.softplus(inp["delta"])
    y, hs = O.ssm_scan_sequential(inp["u"], inp["A"], inp["B"], inp["C"], dt, return_states=True)
    h = O.ssm_scan_final_state(inp["u"], inp["A"], inp["B"], inp["C"], dt, chunk=64)
    assert np.abs(h - hs[:, -1]).max() <= 1e-12 * np.abs(hs[:, -1]).max()
    fa = np.zeros((2, 5, 16))
    alpha = np.exp(inp["A"][None, None] * dt[..., None])
    cdy = inp["dout"][..., None] * inp["C"][:, :, None, :]
    for t in range(199, -1, -1):
        fa = (fa + cdy[:, t]) * alpha[:, t]
    got = O.ssm_scan_adjoint_carry(inp["A"], inp["C"], dt, inp["dout"], chunk=48)
    assert np.abs(got - fa).max() <= 1e-12 * np.abs(fa).max()


@pytest.mark.parametrize("reverse,complement", [(False, False), (True, True)])
def test_window_with_carries_matches_whole_sequence(reverse, complement):
    """A window [t0, t1) of the scan frame, run with the state carried into it
    and the adjoint carried in from its right, reproduces the whole-sequence
    outputs and per-step gradients on the window (the leaf carries of
    ssm_scan_backward_recursive, ssmrecscan.py:111)."""
    L, t0, t1 = 96, 40, 72
    inp = O.make_scan_inputs(2, L, 6, 16, seed=3)
    kw = dict(D=inp["D"], z=inp["z"], delta_softplus=True, reverse=reverse, complement=complement)
    args = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"])
    out = O.selective_scan_fwd(*args, **kw)
    g = O.selective_scan_bwd(*args, inp["dout"], **kw)
    flip = (lambda a: a[:, ::-1, ::-1] if complement else a[:, ::-1]) if reverse else (lambda a: a)
    # window carries from the scan-frame data (output-frame tensors flipped into the scan frame)
    dt = O.softplus(inp["delta"])
    dys = flip(inp["dout"] * O.activation(inp["z"], "silu"))
    h0 = O.ssm_scan_final_state(inp["u"][:, :t0], inp["A"], inp["B"][:, :t0], inp["C"][:, :t0], dt[:, :t0])
    fa = O.ssm_scan_adjoint_carry(inp["A"], inp["C"][:, t1:], dt[:, t1:], dys[:, t1:])
    win = lambda a: a[:, t0:t1]
    if reverse:
        # the reverse direction's window is a window of its scan frame: check the raw scan
        # there, driven by the scan-frame upstream gradient
        wkw = dict(D=None, z=None, delta_softplus=True)
        gw = O.selective_scan_bwd(win(inp["u"]), win(inp["delta"]), inp["A"], win(inp["B"]), win(inp["C"]),
                                  win(dys), h0=h0, fa_right=fa, **wkw)
        gf = O.selective_scan_bwd(*args, dys, **wkw)
        for k in ("du", "ddelta", "dB", "dC"):
            assert np.abs(gw[k] - win(gf[k])).max() <= 1e-10 * np.abs(gf[k]).max(), k
        return
    ow = O.selective_scan_fwd(win(inp["u"]), win(inp["delta"]), inp["A"], win(inp["B"]), win(inp["C"]),
                              D=inp["D"], z=win(inp["z"]), delta_softplus=True, h0=h0)
    assert np.abs(ow - win(out)).max() <= 1e-10 * np.abs(out).max()
    gw = O.selective_scan_bwd(win(inp["u"]), win(inp["delta"]), inp["A"], win(inp["B"]), win(inp["C"]),
                              win(inp["dout"]), D=inp["D"], z=win(inp["z"]), delta_softplus=True, h0=h0,
                              fa_right=fa)
    for k in ("du", "ddelta", "dz", "dB", "dC"):
        assert np.abs(gw[k] - win(g[k])).max() <= 1e-10 * np.abs(g[k]).max(), k
