"""RMSNorm + residual-base kernel (ssm_rmsnorm_fwd / _bwd) against a plain
PyTorch fp32 reference of flax.linen.RMSNorm (selectssm.py:306-313) and the
residual add of selectssm.py:345-352."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def ref_norm(x, scale, bias, eps=1e-6):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * scale
    return y, xf + bias


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("dim", [32, 64, 200, 256, 512, 768, 1024])
def test_rmsnorm_residual_matches_torch(cuda, dtype, tol, dim):
    from selectssm_b200 import rmsnorm_residual
    torch.manual_seed(dim)
    rows = 1000
    x = torch.randn(2, rows // 2, dim, device=cuda).to(dtype).requires_grad_()
    scale = (1 + 0.1 * torch.randn(dim, device=cuda)).requires_grad_()
    bias = (0.1 * torch.randn(dim, device=cuda)).requires_grad_()
    y, base = rmsnorm_residual(x, scale, bias)
    xr = x.detach().float().requires_grad_()
    sr, br = scale.detach().clone().requires_grad_(), bias.detach().clone().requires_grad_()
    yr, baser = ref_norm(xr, sr, br)

    def rel(a, b):
        return float((a.detach().float() - b.detach()).abs().max() / b.detach().abs().max())

    assert rel(y, yr) < tol and rel(base, baser) < tol
    gy, gb = torch.randn_like(yr), torch.randn_like(yr)
    (y.float() * gy + base.float() * gb).sum().backward()
    (yr * gy + baser * gb).sum().backward()
    assert rel(x.grad, xr.grad) < tol
    assert rel(scale.grad, sr.grad) < tol
    assert rel(bias.grad, br.grad) < tol


def test_rmsnorm_many_rows_deterministic(cuda):
    """More rows than the backward grid (rows stride over CTAs); two runs give
    bit-identical gradients."""
    from selectssm_b200 import rmsnorm_residual
    torch.manual_seed(0)
    x = torch.randn(4, 8192, 256, device=cuda).requires_grad_()
    scale = torch.ones(256, device=cuda).requires_grad_()
    grads = []
    for _ in range(2):
        x.grad = scale.grad = None
        y, base = rmsnorm_residual(x, scale, None)
        (y * 1.5 + base).sum().backward()
        grads.append((x.grad.clone(), scale.grad.clone()))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])
    xr = x.detach().requires_grad_()
    sr = scale.detach().clone().requires_grad_()
    yr, _ = ref_norm(xr, sr, torch.zeros(256, device=cuda))
    (yr * 1.5 + xr).sum().backward()
    assert float((grads[0][1] - sr.grad).abs().max() / sr.grad.abs().max()) < 1e-5


def test_dense_onto_is_residual_plus_projection(cuda):
    from selectssm_b200 import dense_onto
    base = torch.randn(3, 40, 64, device=cuda)
    h = torch.randn(3, 40, 128, device=cuda)
    w = torch.randn(128, 64, device=cuda)
    torch.testing.assert_close(dense_onto(base, h, w), base + h @ w, rtol=1e-4, atol=1e-4)
