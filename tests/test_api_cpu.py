"""Host-side checks that need no GPU: the C ABI library, argument validation,
parameter layouts of the modules."""

import ctypes
import os
import re
import subprocess

import pytest
import torch

from selectssm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "selectssm_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"SSM_API\s+[\w\s\*]+?\b(ssm_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert names and set(names) == set(_lib.EXPORTED_SYMBOLS)
    for n in names:
        assert hasattr(lib, n), n
    assert b"sm_100a" in lib.ssm_version()


def test_struct_layout_matches_header(tmp_path):
    """ctypes mirrors of ssm_params_t / ssm_conv_params_t match the C compiler's layout."""
    src = tmp_path / "lay.c"
    fields = [f[0] for f in _lib.SSMParams._fields_]
    cfields = [f[0] for f in _lib.SSMConvParams._fields_]
    body = "\n".join(f'printf("p {f} %zu\\n", offsetof(ssm_params_t, {f}));' for f in fields)
    body += "\n" + "\n".join(f'printf("c {f} %zu\\n", offsetof(ssm_conv_params_t, {f}));' for f in cfields)
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "selectssm_b200.h"\nint main(){\n'
                   + body + '\nprintf("s %zu %zu\\n", sizeof(ssm_params_t), sizeof(ssm_conv_params_t));}\n')
    exe = tmp_path / "lay"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    for line in out:
        parts = line.split()
        if not parts:
            continue
        if parts[0] == "s":
            assert int(parts[1]) == ctypes.sizeof(_lib.SSMParams)
            assert int(parts[2]) == ctypes.sizeof(_lib.SSMConvParams)
        else:
            cls = _lib.SSMParams if parts[0] == "p" else _lib.SSMConvParams
            assert getattr(cls, parts[1]).offset == int(parts[2]), parts[1]


def test_validation_without_gpu():
    lib = _lib.load()
    p = _lib.SSMParams()
    p.batch, p.seqlen, p.dim, p.dstate = 2, 16, 32, 8            # dstate must be 16
    assert lib.ssm_fwd(ctypes.byref(p), None) == _lib.SSM_ERR_SHAPE
    p.dstate, p.dtype = 16, 7
    assert lib.ssm_fwd(ctypes.byref(p), None) == _lib.SSM_ERR_DTYPE
    p.dtype, p.dim = _lib.SSM_F32, 30                             # 30 * 4 bytes is not 16-aligned
    assert lib.ssm_fwd(ctypes.byref(p), None) == _lib.SSM_ERR_ALIGN
    p.dim = 32
    assert lib.ssm_fwd(ctypes.byref(p), None) == _lib.SSM_ERR_NULL
    assert lib.ssm_workspace_bytes(ctypes.byref(p)) > 0
    assert lib.ssm_strerror(_lib.SSM_ERR_SHAPE)


def test_reference_valueerrors_and_chunk_rule():
    """selectssm.py:47-48, :53-54 raise before any device work."""
    from selectssm_b200 import largest_factor_up_to, ssm_chunked_scan
    x = torch.zeros(1, 64, 30)
    A = torch.zeros(30, 16)
    Bm = torch.zeros(1, 64, 16)
    with pytest.raises(ValueError, match="n_channel_groups"):
        ssm_chunked_scan(x, A, Bm, Bm, x, n_channel_groups=4)
    with pytest.raises(ValueError, match="chunk_size"):
        ssm_chunked_scan(x, A, Bm, Bm, x, chunk_size=7)
    assert largest_factor_up_to(45, 2048) == 32
    with pytest.raises(ValueError, match="CUDA"):
        ssm_chunked_scan(x, A, Bm, Bm, x)


def test_module_parameters_use_flax_names_and_layouts():
    from selectssm_b200 import BidirectionalMamba, SelectiveSSM
    m = SelectiveSSM(64, shift_conv_size=4)
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes == {"A_log": (64, 16), "D": (64,), "shift_conv.kernel": (4, 1, 64), "BC.kernel": (64, 32),
                      "BC.bias": (32,), "dt.kernel": (64, 4), "dt.bias": (4,), "dt_proj.kernel": (4, 64),
                      "dt_proj.bias": (64,)}
    assert torch.allclose(m.A_log[0], torch.log(torch.arange(1, 17.0)))       # selectssm.py:190
    b = BidirectionalMamba(64, 16, 2.0, complement=True, tie_in_proj=True, tie_gate=True)
    assert tuple(b.in_proj.kernel.shape) == (64, 2 * 128)                       # tied: 1 x + 1 z
    assert tuple(b.out_proj.kernel.shape) == (256, 64)
    with pytest.raises(Exception, match="Unknown activation"):
        BidirectionalMamba(64, 16, 2.0, activation="tanh")
    with pytest.raises(ValueError, match="chunk_size"):
        SelectiveSSM(64, chunk_size=7)(torch.zeros(1, 32, 64))


def test_workspace_covers_widened_bc_and_bidirectional_segments():
    """bf16 B/C need room for their float32 copies (2 x B*L*16*4 bytes) on top
    of the fp32 case's scratch, and one parameter set's size already covers a
    bidirectional launch (its segment count may differ)."""
    lib = _lib.load()

    def ws(bc, B=2, L=131072, D=512):
        p = _lib.SSMParams()
        p.batch, p.seqlen, p.dim, p.dstate = B, L, D, 16
        p.dtype, p.bc_dtype = _lib.SSM_BF16, bc
        return lib.ssm_workspace_bytes(ctypes.byref(p))

    f32, b16 = ws(_lib.SSM_F32), ws(_lib.SSM_BF16)
    assert f32 > 0 and b16 >= f32 + 2 * 2 * 131072 * 16 * 4


def test_multicast_backward_validates_arguments_without_gpu():
    lib = _lib.load()
    p = _lib.SSMParams()
    p.batch, p.seqlen, p.dim, p.dstate = 2, 16, 32, 16
    assert lib.ssm_bwd_bc_multicast(ctypes.byref(p), None, None) == _lib.SSM_ERR_NULL
    assert lib.ssm_bwd_bc_multicast(ctypes.byref(p), 0x1008, None) == _lib.SSM_ERR_ALIGN
    p.dstate = 8
    assert lib.ssm_bwd_bc_multicast(ctypes.byref(p), 0x1000, None) == _lib.SSM_ERR_SHAPE
