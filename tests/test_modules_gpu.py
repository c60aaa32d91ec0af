"""SelectiveSSM / BidirectionalMamba on the CUDA path.

The first two classes re-run the reference's own tests (tests/test_selectssm.py
:18-85: output shapes for the three scan selectors and the bidirectional
variants, finite and non-zero gradients).  The rest compare module outputs with
the NumPy oracle on the same parameters, and module parameter gradients with
float64 central differences of the oracle forward.
"""

import os

import numpy as np
import pytest
import torch

from oracle import selectssm_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return np.abs(a - b).max() / np.abs(b).max()


def npy(t):
    return t.detach().double().cpu().numpy()


def _tree(module):
    def cv(v):
        return {k: cv(x) for k, x in v.items()} if isinstance(v, dict) else npy(v)
    return cv(module.flax_params())


class TestSelectiveSSMShapes:  # tests/test_selectssm.py:18-38
    @pytest.mark.parametrize("kw", [{}, {"recursive_scan": True}, {"custom_vjp_scan": True}])
    def test_forward_shape(self, cuda, kw):
        from selectssm_b200 import SelectiveSSM
        model = SelectiveSSM(64, hidden_features=16, **kw).to(cuda)
        x = torch.randn(2, 32, 64, device=cuda)
        assert model(x).shape == x.shape


class TestBidirectionalMambaShapes:  # tests/test_selectssm.py:41-85
    @pytest.mark.parametrize("kw", [{}, {"complement": True, "tie_in_proj": True, "tie_gate": True},
                                    {"concatenate_fwd_rev": True}, {"concatenate_fwd_rev": False}])
    def test_forward_shape(self, cuda, kw):
        from selectssm_b200 import BidirectionalMamba
        model = BidirectionalMamba(64, hidden_features=16, expansion_factor=2.0, **kw).to(cuda)
        x = torch.randn(2, 32, 64, device=cuda)
        assert model(x).shape == x.shape

    def test_gradient_flow(self, cuda):
        from selectssm_b200 import BidirectionalMamba
        model = BidirectionalMamba(32, hidden_features=16, expansion_factor=2.0).to(cuda)
        x = torch.randn(2, 16, 32, device=cuda)
        (model(x) ** 2).sum().backward()
        grads = [p.grad for p in model.parameters()]
        assert all(g is not None and torch.isfinite(g).all() for g in grads)
        assert any(g.abs().max() > 0 for g in grads)


@pytest.mark.parametrize("reverse,complement", [(False, False), (True, False), (True, True)])
def test_selective_ssm_matches_oracle_golden_params(cuda, reverse, complement):
    from selectssm_b200 import SelectiveSSM
    g = np.load(os.path.join(GOLD, "selective_ssm.npz"))
    model = SelectiveSSM(128, reverse=reverse, complement=complement, hidden_features=16, dt_rank=4,
                         shift_conv_size=4).to(cuda)
    tree = {"shift_conv": {"kernel": g["shift_conv_kernel"]}, "A_log": g["A_log"],
            "BC": {"kernel": g["BC_kernel"], "bias": g["BC_bias"]}, "D": g["D"],
            "dt": {"kernel": g["dt_kernel"], "bias": g["dt_bias"]},
            "dt_proj": {"kernel": g["dt_proj_kernel"], "bias": g["dt_proj_bias"]}}
    model.load_flax_params(tree)
    y = model(torch.tensor(g["x"], dtype=torch.float32, device=cuda))
    ref = O.selective_ssm_fwd(tree, g["x"], reverse=reverse, complement=complement)
    if not reverse:
        assert rel(npy(y), g["y"]) < 1e-4
    assert rel(npy(y), ref) < 1e-4


@pytest.mark.parametrize("kw", [dict(complement=True, tie_in_proj=True, tie_gate=True, concatenate_fwd_rev=True),
                                dict(complement=False, concatenate_fwd_rev=False),
                                dict(complement=True, tie_in_proj=False, tie_gate=True, concatenate_fwd_rev=True,
                                     activation="gelu")])
def test_bidirectional_mamba_matches_oracle(cuda, kw):
    from selectssm_b200 import BidirectionalMamba
    torch.manual_seed(0)
    model = BidirectionalMamba(32, hidden_features=16, expansion_factor=2.0,
                               ssm_args={"shift_conv_size": 4}, **kw).to(cuda)
    with torch.no_grad():
        for p in model.parameters():  # non-trivial norm scales and biases
            p.add_(0.05 * torch.randn_like(p))
    x = torch.randn(2, 80, 32, device=cuda)
    y = model(x)
    params = {"RMSNorm_0": {"scale": npy(model.RMSNorm_0.scale)},
              "in_proj": {"kernel": npy(model.in_proj.kernel), "bias": npy(model.in_proj.bias)},
              "out_proj": {"kernel": npy(model.out_proj.kernel), "bias": npy(model.out_proj.bias)},
              "ssm_fwd": _tree(model.ssm_fwd), "ssm_rev": _tree(model.ssm_rev)}
    ref = O.bidirectional_mamba_fwd(params, npy(x), activation_name=kw.get("activation", "silu"),
                                    **{k: v for k, v in kw.items() if k != "activation"})
    assert rel(npy(y), ref) < 1e-4


@pytest.mark.parametrize("reverse,complement", [(False, False), (True, True)])
def test_selective_ssm_param_grads_vs_finite_differences(cuda, reverse, complement):
    """d(sum(w * y))/d(param) through the CUDA backward vs fp64 central
    differences of the oracle forward, on a sample of entries of every parameter."""
    from selectssm_b200 import SelectiveSSM
    torch.manual_seed(1)
    D, L = 32, 40
    model = SelectiveSSM(D, reverse=reverse, complement=complement, hidden_features=16,
                         shift_conv_size=4).to(cuda)
    x = torch.randn(2, L, D, device=cuda)
    w = torch.randn(2, L, D, device=cuda)
    (model(x) * w).sum().backward()
    tree = _tree(model)
    xn, wn = npy(x), npy(w)
    grads = {"shift_conv": {"kernel": model.shift_conv.kernel.grad}, "A_log": model.A_log.grad,
             "BC": {"kernel": model.BC.kernel.grad, "bias": model.BC.bias.grad}, "D": model.D.grad,
             "dt": {"kernel": model.dt.kernel.grad, "bias": model.dt.bias.grad},
             "dt_proj": {"kernel": model.dt_proj.kernel.grad, "bias": model.dt_proj.bias.grad}}
    rng = np.random.default_rng(0)

    def loss(t):
        return (O.selective_ssm_fwd(t, xn, reverse=reverse, complement=complement) * wn).sum()

    def leaves(t, prefix=()):
        for k, v in t.items():
            if isinstance(v, dict):
                yield from leaves(v, prefix + (k,))
            else:
                yield prefix + (k,), v

    for path, arr in leaves(tree):
        g = grads
        for k in path:
            g = g[k]
        g = npy(g)
        scale = np.abs(g).max() + 1e-12
        for _ in range(3):
            idx = tuple(rng.integers(0, s) for s in arr.shape)
            eps = 1e-6 * max(1.0, abs(arr[idx]))

            def perturbed(d):
                t = {k: (dict(v) if isinstance(v, dict) else v) for k, v in tree.items()}
                node = t
                for k in path[:-1]:
                    node = node[k]
                a2 = arr.copy()
                a2[idx] += d
                node[path[-1]] = a2
                return t

            num = (loss(perturbed(eps)) - loss(perturbed(-eps))) / (2 * eps)
            assert abs(num - g[idx]) <= 2e-4 * scale + 1e-6, (path, idx, num, g[idx])
