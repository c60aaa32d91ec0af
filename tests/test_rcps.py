"""RCPS wrappers (src/selectssm/rcps.py).  The CPU tests re-run the reference's
tests/test_selectssm.py:88-135 on the PyTorch mirror (shapes, RC equivariance
with a Dense inner module); the GPU test checks equivariance and the batch-
stacked single inner call with BidirectionalMamba on the CUDA path."""

import pytest
import torch

from selectssm_b200.modules import _Dense
from selectssm_b200.rcps import RCPSEmbedding, RCPSLMHead, RCPSNorm, RCPSWrapper, rc_conjugate


def test_wrapper_shape():  # tests/test_selectssm.py:89-94
    torch.manual_seed(0)
    model = RCPSWrapper(_Dense(32, 32))
    x = torch.randn(2, 16, 64)
    assert model(x).shape == x.shape


def test_equivariance():  # tests/test_selectssm.py:96-107
    torch.manual_seed(0)
    model = RCPSWrapper(_Dense(32, 32))
    x = torch.randn(1, 16, 64)
    y1 = rc_conjugate(model(x))
    y2 = model(rc_conjugate(x))
    assert torch.allclose(y1, y2, atol=1e-5)


def test_norm_shape_and_equivariance():  # tests/test_selectssm.py:109-114
    torch.manual_seed(0)
    model = RCPSNorm(32)
    with torch.no_grad():
        model.norm.scale.uniform_(0.5, 1.5)
    x = torch.randn(2, 16, 64)
    assert model(x).shape == x.shape
    assert torch.allclose(rc_conjugate(model(x)), model(rc_conjugate(x)), atol=1e-5)


def test_embedding_shape_and_strands():  # tests/test_selectssm.py:116-123
    cmap = [3, 2, 1, 0]
    model = RCPSEmbedding(vocab_size=4, d_model=16, complement_map=cmap)
    tokens = torch.tensor([[0, 1, 2, 3]])
    y = model(tokens)
    assert y.shape == (1, 4, 32)
    # the reverse complement of the sequence swaps the two strands (conjugated)
    rc_tokens = torch.flip(torch.tensor(cmap)[tokens], dims=(-1,))
    y_rc = model(rc_tokens)
    assert torch.allclose(y_rc, rc_conjugate(y))


def test_lm_head_shape():  # tests/test_selectssm.py:125-131
    model = RCPSLMHead(16, vocab_size=4, complement_map=[3, 2, 1, 0])
    x = torch.randn(1, 8, 32)
    assert model(x).shape == (1, 8, 4)


@pytest.mark.gpu
def test_wrapper_around_bidirectional_mamba(cuda):
    from selectssm_b200 import BidirectionalMamba
    torch.manual_seed(3)
    inner = BidirectionalMamba(32, hidden_features=16, expansion_factor=2.0, complement=True, tie_in_proj=True,
                               tie_gate=True, ssm_args={"shift_conv_size": 4}).to(cuda)
    model = RCPSWrapper(inner)
    x = torch.randn(2, 96, 64, device=cuda)
    y = model(x)
    # one stacked inner call == the reference's two calls
    ref = torch.cat([inner(x[..., :32]), rc_conjugate(inner(rc_conjugate(x[..., 32:])))], dim=-1)
    scale = ref.abs().max()
    assert ((y - ref).abs().max() / scale) < 1e-5
    # RC equivariance
    assert ((rc_conjugate(y) - model(rc_conjugate(x))).abs().max() / scale) < 1e-4
    (y ** 2).sum().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in inner.parameters())


@pytest.mark.gpu
def test_wrapper_around_selective_ssm_reads_antisense_in_place(cuda, monkeypatch):
    """A forward SelectiveSSM inner module runs the antisense strand through the
    kernels' reversed, complemented read: no flipped copy is made, and the
    result equals the reference's rc(inner(rc(x))) (rcps.py:42-72)."""
    import selectssm_b200.rcps as R
    from selectssm_b200 import SelectiveSSM
    torch.manual_seed(5)
    inner = SelectiveSSM(48, hidden_features=16, shift_conv_size=4).to(cuda)
    with torch.no_grad():
        inner.D.uniform_(0.5, 1.5)  # a non-trivial skip, so its frame matters
    model = RCPSWrapper(inner)
    x = torch.randn(2, 200, 96, device=cuda)
    ref = torch.cat([inner(x[..., :48]), rc_conjugate(inner(rc_conjugate(x[..., 48:])))], dim=-1)

    def no_flip(t):
        raise AssertionError("the antisense strand was flipped in memory")

    monkeypatch.setattr(R, "rc_conjugate", no_flip)
    y = model(x)
    monkeypatch.undo()
    scale = ref.abs().max()
    assert ((y - ref).abs().max() / scale) < 1e-5
    assert ((rc_conjugate(y) - model(rc_conjugate(x))).abs().max() / scale) < 1e-4
    (y ** 2).sum().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in inner.parameters())
