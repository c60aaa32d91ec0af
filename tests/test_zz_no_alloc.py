"""ssm_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such callers (a framework that owns every device allocation, or a hot path
where allocating is not allowed) get the same gradients as ssm_bwd, with the
scratch taken from a fixed per-GPU array inside the library.  This file is
named to be collected last, so a run that stops at the first failure has run
every other test before it.
"""

import ctypes

import numpy as np
import pytest
import torch

from selectssm_b200 import _lib


def relerr(got, ref):
    got = got.detach().double().cpu().numpy()
    ref = ref.detach().double().cpu().numpy()
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


def test_noalloc_rejects_oversized_scratch():
    """Sizes whose scratch exceeds the fixed array fail with a clear status,
    before any pointer is touched."""
    lib = _lib.load()
    p = _lib.SSMParams()
    p.batch, p.seqlen, p.dim, p.dstate = 4096, 64, 4096, 16  # 4096*4096*72 bytes > 8 MiB
    assert lib.ssm_workspace_bytes(ctypes.byref(p)) > _lib.NOALLOC_SCRATCH_BYTES
    assert lib.ssm_bwd_noalloc(ctypes.byref(p), None) == _lib.SSM_ERR_WORKSPACE


@pytest.mark.gpu
@pytest.mark.parametrize("bc_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_ssm_bwd_twice(cuda, bc_dtype):
    """Two consecutive ssm_bwd_noalloc calls give ssm_bwd's gradients (1e-4)."""
    from selectssm_b200.ops import _Prepared, _workspace

    torch.manual_seed(0)
    Bsz, L, D = 2, 200, 64
    f32 = dict(device=cuda, dtype=torch.float32)
    u, z = torch.randn(Bsz, L, D, **f32), torch.randn(Bsz, L, D, **f32)
    delta = torch.randn(Bsz, L, D, **f32) - 4
    A = -torch.empty(D, 16, **f32).uniform_(1, 16)
    Bm = torch.randn(Bsz, L, 16, **f32).to(bc_dtype)
    Cm = torch.randn(Bsz, L, 16, **f32).to(bc_dtype)
    Dv, bias = 1 + 0.1 * torch.randn(D, **f32), 0.1 * torch.randn(D, **f32)
    dout = torch.randn(Bsz, L, D, **f32)
    pr = _Prepared(u, delta, A, Bm, Cm, Dv, z, bias, True, True, True, "silu", False)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.empty(Bsz, L, D, **f32)
    states = pr.new_states()
    p = pr.params(out=out, out_stride=D, states=states)
    fws = _workspace(p, cuda)  # the forward keeps its ordinary workspace
    assert lib.ssm_fwd(ctypes.byref(p), stream) == _lib.SSM_OK
    torch.cuda.synchronize()
    del fws

    ref_p = pr.params(states=states)
    ref = pr.grads(ref_p, dout, D)
    ws = _workspace(ref_p, cuda)
    assert lib.ssm_bwd(ctypes.byref(ref_p), stream) == _lib.SSM_OK
    torch.cuda.synchronize()
    del ws

    for _ in range(2):
        q = pr.params(states=states)
        got = pr.grads(q, dout, D)
        q.workspace, q.workspace_bytes = None, 0
        st = lib.ssm_bwd_noalloc(ctypes.byref(q), stream)
        assert st == _lib.SSM_OK, lib.ssm_last_error()
        torch.cuda.synchronize()
        for name, r in ref.items():
            if r is not None:
                assert relerr(got[name], r) < 1e-4, name
