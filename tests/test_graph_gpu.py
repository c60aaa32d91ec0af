"""The fused op inside a captured CUDA graph: a forward + backward captured
once and replayed gives the eager results (the host side launches only
kernels and stream-ordered work, so small, launch-bound shapes can be
replayed without per-call host overhead)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_capture_and_replay_fwd_bwd(cuda):
    import selectssm_b200 as S
    torch.manual_seed(0)
    Bsz, L, D = 2, 1024, 128  # config 1's scan shape (latency bound)
    f32 = dict(device=cuda, dtype=torch.float32)
    u, delta, z, dout = (torch.randn(Bsz, L, D, **f32) for _ in range(4))
    delta -= 4.0
    A = -(1.0 + 15.0 * torch.rand(D, 16, **f32))
    Bm, Cm = torch.randn(Bsz, L, 16, **f32), torch.randn(Bsz, L, 16, **f32)
    Dv = torch.ones(D, **f32)
    leaves = [t.clone().requires_grad_() for t in (u, delta, A, Bm, Cm, Dv, z)]

    def step():
        for t in leaves:
            t.grad = None
        uu, dd, AA, BB, CC, DD, zz = leaves
        out = S.selective_scan(uu, dd, AA, BB, CC, D=DD, z=zz, delta_softplus=True)
        out.backward(dout)
        return out

    ref_out = step().detach().clone()
    ref_grads = [t.grad.clone() for t in leaves]

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    for t in leaves:
        t.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    for t, g in zip(leaves, ref_grads):
        assert torch.allclose(t.grad, g, rtol=0, atol=1e-6 * float(g.abs().max()))
