"""Device-side failure path without a GPU fault: a bounded wait that cannot
complete reports SSM_ERR_TIMEOUT through the status word and the context stays
usable for the next call."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    import selectssm_b200 as S
    from selectssm_b200 import _lib
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    st = lib.ssm_selftest_wait_timeout(ctypes.c_void_p(status.data_ptr()), 1 << 12,
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.SSM_OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.SSM_ERR_TIMEOUT
    # the context is intact: a normal scan still runs and gives finite output
    u = torch.randn(1, 64, 32, device=cuda)
    out = S.selective_scan(u, u - 4.0, -torch.rand(32, 16, device=cuda) - 0.5, torch.randn(1, 64, 16, device=cuda),
                           torch.randn(1, 64, 16, device=cuda), delta_softplus=True)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_lookback_wait_reports_timeout_and_context_survives(cuda):
    """The backward's decoupled lookback: with the CTAs of the last segment
    left out, the segment before it waits for a flag nothing sets; every wait
    gives up after its poll limit, the kernel reports SSM_ERR_TIMEOUT and the
    next (normal) backward on the same shape is exact again."""
    import numpy as np
    import selectssm_b200 as S
    from oracle import selectssm_oracle as O
    from selectssm_b200 import _lib
    from selectssm_b200.ops import _Prepared, _stream, _workspace, ctypes_byref
    lib = _lib.load()
    Bsz, L, D = 1, 2048, 128  # one chain: the backward cuts it into segments
    inp = O.make_scan_inputs(Bsz, L, D, 16, seed=3)
    t = {k: torch.tensor(v, dtype=torch.float32, device=cuda) for k, v in inp.items()}
    pr = _Prepared(t["u"], t["delta"], t["A"], t["B"], t["C"], t["D"], t["z"], None, True, False, False, "silu",
                   False)
    out = torch.empty(pr.shape, device=cuda)
    states = pr.new_states()
    p = pr.params(out=out, out_stride=D, states=states)
    ws_f = _workspace(p, cuda, kind="fwd")
    assert lib.ssm_fwd(ctypes_byref(p), _stream()) == _lib.SSM_OK
    p = pr.params(states=states)
    grads = pr.grads(p, t["dout"], D)  # keep the gradient buffers alive while the kernels write them
    ws_b = _workspace(p, cuda, kind="bwd")
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    p.status = status.data_ptr()
    assert lib.ssm_selftest_lookback_timeout(ctypes_byref(p), 2000, _stream()) == _lib.SSM_OK
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.SSM_ERR_TIMEOUT
    del ws_f, ws_b, grads
    # the context is intact and the lookback path is exact on the next call
    ts = {k: v.clone().requires_grad_() for k, v in t.items()}
    y = S.selective_scan(ts["u"], ts["delta"], ts["A"], ts["B"], ts["C"], D=ts["D"], z=ts["z"], delta_softplus=True)
    y.backward(ts["dout"])
    torch.cuda.synchronize()
    kw = dict(D=inp["D"], z=inp["z"], delta_softplus=True)
    ref = O.selective_scan_bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["dout"], **kw)
    for name, key in (("du", "u"), ("ddelta", "delta"), ("dA", "A"), ("dB", "B"), ("dC", "C")):
        got = ts[key].grad.double().cpu().numpy()
        assert np.abs(got - ref[name]).max() / np.abs(ref[name]).max() < 1e-4, name
