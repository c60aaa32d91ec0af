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
