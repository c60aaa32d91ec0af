"""ctypes binding of the C ABI declared in include/selectssm_b200.h.

The shared library is built in-tree (``selectssm_b200/libselectssm_b200.so``).
There is no fallback path: if the library is missing or fails to load, every
op raises :class:`SSMLibraryError`.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libselectssm_b200.so")

# status codes (enum ssm_status)
SSM_OK = 0
SSM_ERR_SHAPE = 1
SSM_ERR_DTYPE = 2
SSM_ERR_LAUNCH = 3
SSM_ERR_TIMEOUT = 4
SSM_ERR_NULL = 5
SSM_ERR_ALIGN = 6
SSM_ERR_WORKSPACE = 7

SSM_F32 = 0
SSM_BF16 = 1

SSM_DELTA_SOFTPLUS = 1 << 0
SSM_REVERSE = 1 << 1
SSM_COMPLEMENT = 1 << 2
SSM_ALIGNED_SKIP = 1 << 3

ACT_CODES = {None: 0, "none": 0, "silu": 1, "gelu": 2, "relu": 3}

SSM_CHUNK = 8
NOALLOC_SCRATCH_BYTES = 8 << 20
DSTATE = 16

# Every symbol include/selectssm_b200.h declares.
EXPORTED_SYMBOLS = (
    "ssm_workspace_bytes", "ssm_states_elems", "ssm_fwd", "ssm_bwd", "ssm_fwd_bidir", "ssm_bwd_bidir",
    "ssm_conv1d_workspace_bytes", "ssm_conv1d_act_fwd", "ssm_conv1d_act_bwd", "ssm_strerror", "ssm_last_error",
    "ssm_version", "ssm_bwd_noalloc", "ssm_launch_count",
    "ssm_rmsnorm_workspace_bytes", "ssm_rmsnorm_fwd", "ssm_rmsnorm_bwd", "ssm_selftest_wait_timeout",
    "ssm_bwd_bc_multicast", "ssm_bwd_workspace_bytes", "ssm_fwd_workspace_bytes",
    "ssm_selftest_lookback_timeout",
)


class SSMLibraryError(RuntimeError):
    """The native library is missing or a call into it failed."""


class SSMParams(ctypes.Structure):
    """Mirror of ``ssm_params_t``."""

    _fields_ = [
        ("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("dim", ctypes.c_int32), ("dstate", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("bc_dtype", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("gate_act", ctypes.c_int32),
        ("z_stride", ctypes.c_int64), ("out_stride", ctypes.c_int64), ("bc_stride", ctypes.c_int64),
        ("u", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("A", ctypes.c_void_p), ("Bm", ctypes.c_void_p),
        ("Cm", ctypes.c_void_p), ("D", ctypes.c_void_p), ("delta_bias", ctypes.c_void_p), ("z", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("states", ctypes.c_void_p),
        ("dout", ctypes.c_void_p), ("du", ctypes.c_void_p), ("ddelta", ctypes.c_void_p), ("dA", ctypes.c_void_p),
        ("dB", ctypes.c_void_p), ("dC", ctypes.c_void_p), ("dD", ctypes.c_void_p), ("ddelta_bias", ctypes.c_void_p),
        ("dz", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
    ]


class SSMConvParams(ctypes.Structure):
    """Mirror of ``ssm_conv_params_t``."""

    _fields_ = [
        ("batch", ctypes.c_int32), ("seqlen", ctypes.c_int32), ("dim", ctypes.c_int32), ("width", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("flags", ctypes.c_int32), ("act", ctypes.c_int32),
        ("x_stride", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("u", ctypes.c_void_p), ("du", ctypes.c_void_p),
        ("dx", ctypes.c_void_p), ("dw", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class SSMNormParams(ctypes.Structure):
    """Mirror of ``ssm_norm_params_t``."""

    _fields_ = [
        ("rows", ctypes.c_int64), ("dim", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("x", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("y", ctypes.c_void_p), ("rstd", ctypes.c_void_p),
        ("res_bias", ctypes.c_void_p), ("res_base", ctypes.c_void_p), ("dy", ctypes.c_void_p),
        ("dres", ctypes.c_void_p), ("dx", ctypes.c_void_p), ("dscale", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library with typed signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise SSMLibraryError(
            f"native library not found at {p}; build it with `python -m selectssm_b200.build` "
            "(there is no non-CUDA fallback)")
    try:
        lib = ctypes.CDLL(p)
    except OSError as e:  # pragma: no cover - environment specific
        raise SSMLibraryError(f"failed to load {p}: {e}") from e
    P = ctypes.POINTER(SSMParams)
    CP = ctypes.POINTER(SSMConvParams)
    NP = ctypes.POINTER(SSMNormParams)
    sigs = {
        "ssm_workspace_bytes": (ctypes.c_size_t, [P]),
        "ssm_states_elems": (ctypes.c_size_t, [P]),
        "ssm_bwd_workspace_bytes": (ctypes.c_size_t, [P, ctypes.c_int]),
        "ssm_fwd_workspace_bytes": (ctypes.c_size_t, [P]),
        "ssm_fwd": (ctypes.c_int, [P, ctypes.c_void_p]),
        "ssm_bwd": (ctypes.c_int, [P, ctypes.c_void_p]),
        "ssm_fwd_bidir": (ctypes.c_int, [P, P, ctypes.c_void_p]),
        "ssm_bwd_bidir": (ctypes.c_int, [P, P, ctypes.c_void_p]),
        "ssm_conv1d_workspace_bytes": (ctypes.c_size_t, [CP]),
        "ssm_conv1d_act_fwd": (ctypes.c_int, [CP, ctypes.c_void_p]),
        "ssm_conv1d_act_bwd": (ctypes.c_int, [CP, ctypes.c_void_p]),
        "ssm_rmsnorm_workspace_bytes": (ctypes.c_size_t, [NP]),
        "ssm_rmsnorm_fwd": (ctypes.c_int, [NP, ctypes.c_void_p]),
        "ssm_rmsnorm_bwd": (ctypes.c_int, [NP, ctypes.c_void_p]),
        "ssm_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
        "ssm_selftest_lookback_timeout": (ctypes.c_int, [ctypes.POINTER(SSMParams), ctypes.c_uint32, ctypes.c_void_p]),
        "ssm_strerror": (ctypes.c_char_p, [ctypes.c_int]),
        "ssm_last_error": (ctypes.c_char_p, []),
        "ssm_version": (ctypes.c_char_p, []),
        "ssm_launch_count": (ctypes.c_ulonglong, []),
        "ssm_bwd_noalloc": (ctypes.c_int, [P, ctypes.c_void_p]),
        "ssm_bwd_bc_multicast": (ctypes.c_int, [P, ctypes.c_void_p, ctypes.c_void_p]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def strerror(status: int) -> str:
    return load().ssm_strerror(status).decode()


def check(status: int, what: str) -> None:
    """Raise the reference's error type for a failed call: ValueError for shapes
    it rejects (selectssm.py:47-48, :53-54), SSMLibraryError otherwise."""
    if status == SSM_OK:
        return
    msg = f"{what}: {strerror(status)} (status {status})"
    if status == SSM_ERR_LAUNCH:
        msg += f" [{load().ssm_last_error().decode()}]"
    if status in (SSM_ERR_SHAPE, SSM_ERR_ALIGN, SSM_ERR_DTYPE):
        raise ValueError(msg)
    raise SSMLibraryError(msg)
