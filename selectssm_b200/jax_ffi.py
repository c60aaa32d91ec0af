"""JAX bindings of the scan kernels through jax.ffi custom calls.

UNVERIFIED: JAX and jaxlib are not installed where this package is developed
and tested, so nothing here has run.  It is the binding a JAX user of the
reference would take: the reference's scan functions with their signatures
and ValueErrors, backed by the same C ABI the PyTorch host uses.

* ``ssm_chunked_scan(x, Acoeff, Bcoeff, Ccoeff, dt, chunk_size=None,
  n_channel_groups=1)``                       src/selectssm/selectssm.py:37-109
* ``ssm_recursive_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, ...)``
                                              src/selectssm/ssmrecscan.py:36-77
* ``ssm_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, ...)``  (custom VJP)
                                              src/selectssm/ssmrecscan.py:80-183
* ``selective_scan(...)``: the fused op (softplus(delta + bias), D skip,
  reverse / complement, gate), as SelectiveSSM + BidirectionalMamba use it.

A reference model switches to the kernels by rebinding its module-level
functions, e.g. ``selectssm.selectssm.ssm_chunked_scan = jax_ffi.ssm_chunked_scan``.

Setup in a JAX environment: ``build_handlers()`` once (compiles
``csrc/jax_ffi_handlers.cc`` against ``jax.ffi.include_dir()``), then
``register()`` before tracing.  JAX is imported lazily, so importing this
module without JAX works (and does nothing).  Nothing here imports PyTorch.
"""

from __future__ import annotations

import ctypes
import functools
import os
import subprocess

from . import _lib
from ._checks import check_chunked as _check_chunked, largest_factor_up_to  # noqa: F401  (same ValueErrors)

HERE = os.path.dirname(os.path.abspath(__file__))
HANDLER_SRC = os.path.join(HERE, "csrc", "jax_ffi_handlers.cc")
HANDLER_LIB = os.path.join(HERE, "libselectssm_b200_jax.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
TARGETS = ("selectssm_scan_fwd", "selectssm_scan_bwd")
_registered = False


def build_handlers() -> str:
    """Compile the XLA FFI handlers (needs jaxlib's FFI headers and nvcc)."""
    import jax.ffi
    cmd = ["nvcc", "-x", "cu", "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC",
           f"-I{jax.ffi.include_dir()}", f"-I{INCLUDE}", HANDLER_SRC, "-o", HANDLER_LIB,
           f"-L{HERE}", "-lselectssm_b200", f"-Xlinker=-rpath,{HERE}"]
    subprocess.run(cmd, check=True)
    return HANDLER_LIB


def register() -> None:
    """Register the handlers as CUDA custom-call targets (once per process)."""
    global _registered
    if _registered:
        return
    import jax.ffi
    _lib.load()  # the kernels' library, loaded first so the handler's dependency resolves
    lib = ctypes.cdll.LoadLibrary(HANDLER_LIB)
    for name in TARGETS:
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(lib, name)), platform="CUDA")
    _registered = True


def _code(dtype) -> int:
    import jax.numpy as jnp
    if dtype == jnp.float32:
        return _lib.SSM_F32
    if dtype == jnp.bfloat16:
        return _lib.SSM_BF16
    raise ValueError(f"unsupported dtype {dtype}; the kernels take float32 or bfloat16")


def _sizes(x, B, flags, gate):
    """(workspace bytes, states shape) from shapes alone (no device pointers)."""
    p = _lib.SSMParams()
    p.batch, p.seqlen, p.dim, p.dstate = x.shape[0], x.shape[1], x.shape[2], B.shape[2]
    p.dtype, p.bc_dtype, p.flags, p.gate_act = _code(x.dtype), _code(B.dtype), flags, gate
    lib = _lib.load()
    ws = max(int(lib.ssm_workspace_bytes(ctypes.byref(p))), 256)
    states = (x.shape[0], -(-x.shape[1] // _lib.SSM_CHUNK), x.shape[2], B.shape[2])
    return ws, states


@functools.lru_cache(maxsize=None)
def _make_op(flags: int, gate: int):
    import jax
    import jax.numpy as jnp
    import numpy as np

    attrs = dict(flags=np.int32(flags), gate_act=np.int32(gate))

    def call_fwd(x, delta, A, B, C, D, bias, z):
        ws, st = _sizes(x, B, flags, gate)
        out, states, _ = jax.ffi.ffi_call(
            TARGETS[0],
            (jax.ShapeDtypeStruct(x.shape, x.dtype), jax.ShapeDtypeStruct(st, jnp.float32),
             jax.ShapeDtypeStruct((ws,), jnp.uint8)))(x, delta, A, B, C, D, bias, z, **attrs)
        return out, states

    @jax.custom_vjp
    def op(x, delta, A, B, C, D, bias, z):
        return call_fwd(x, delta, A, B, C, D, bias, z)[0]

    def fwd(x, delta, A, B, C, D, bias, z):
        out, states = call_fwd(x, delta, A, B, C, D, bias, z)
        return out, (x, delta, A, B, C, D, bias, z, states)

    def bwd(res, dout):
        x, delta, A, B, C, D, bias, z, states = res
        ws, _ = _sizes(x, B, flags, gate)
        shapes = (jax.ShapeDtypeStruct(x.shape, x.dtype), jax.ShapeDtypeStruct(delta.shape, delta.dtype),
                  jax.ShapeDtypeStruct(A.shape, jnp.float32), jax.ShapeDtypeStruct(B.shape, B.dtype),
                  jax.ShapeDtypeStruct(C.shape, C.dtype), jax.ShapeDtypeStruct(D.shape, jnp.float32),
                  jax.ShapeDtypeStruct(bias.shape, jnp.float32), jax.ShapeDtypeStruct(z.shape, z.dtype),
                  jax.ShapeDtypeStruct((ws,), jnp.uint8))
        grads = jax.ffi.ffi_call(TARGETS[1], shapes)(x, delta, A, B, C, D, bias, z, states,
                                                     dout.astype(x.dtype), **attrs)
        return tuple(grads[:8])

    op.defvjp(fwd, bwd)
    return op


def selective_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, reverse=False,
                   complement=False, gate_act="silu", aligned_skip=False):
    """The fused op: (unflip(scan(u, softplus?(delta + bias))) + skip) * act(z)."""
    import jax.numpy as jnp
    register()
    f32 = jnp.float32
    flags = ((_lib.SSM_DELTA_SOFTPLUS if delta_softplus else 0) | (_lib.SSM_REVERSE if reverse else 0)
             | (_lib.SSM_COMPLEMENT if (reverse and complement) else 0)
             | (_lib.SSM_ALIGNED_SKIP if aligned_skip else 0))
    gate = _lib.ACT_CODES[gate_act] if z is not None else 0
    empty = jnp.zeros((0,), f32)
    op = _make_op(flags, gate)
    return op(u, delta, A.astype(f32), B, C, empty if D is None else D.astype(f32),
              empty if delta_bias is None else delta_bias.astype(f32),
              jnp.zeros((0,), u.dtype) if z is None else z)


def ssm_chunked_scan(x, Acoeff, Bcoeff, Ccoeff, dt, chunk_size: int = None, n_channel_groups: int = 1):
    """selectssm.py:37-109 (same ValueErrors); the chunking arguments are memory knobs."""
    _check_chunked(x.shape[1], x.shape[2], chunk_size, n_channel_groups)
    return selective_scan(x, dt, Acoeff, Bcoeff, Ccoeff)


def ssm_recursive_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, min_recursion_length: int = 2, recursive_split: int = 2):
    """ssmrecscan.py:36-77."""
    return selective_scan(x, Delta, Acoeff, Bcoeff, Ccoeff)


def ssm_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, min_recursion_length: int = 2, recursive_split: int = 2):
    """ssmrecscan.py:80-183 (custom VJP; the backward is the kernel's)."""
    return selective_scan(x, Delta, Acoeff, Bcoeff, Ccoeff)
