"""The jax.ffi binding without JAX: the module imports (JAX is loaded lazily),
the handler source calls only functions the C header declares, and the
registered target names are the handler symbols.  Running it needs JAX
(absent here), so that part is skipped."""

import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_module_imports_without_jax():
    from selectssm_b200 import jax_ffi
    assert jax_ffi.TARGETS == ("selectssm_scan_fwd", "selectssm_scan_bwd")


def test_handler_source_matches_header_and_targets():
    from selectssm_b200 import jax_ffi
    src = open(jax_ffi.HANDLER_SRC).read()
    header = open(os.path.join(ROOT, "include", "selectssm_b200.h")).read()
    declared = set(re.findall(r"SSM_API\s+[\w\s\*]+?\b(ssm_\w+)\s*\(", header))
    called = set(re.findall(r"\b(ssm_\w+)\s*\(", src))
    assert called and called <= declared, called - declared
    defined = set(re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\(\s*(\w+)", src))
    assert defined == set(jax_ffi.TARGETS)


def test_jax_path_when_available():
    pytest.importorskip("jax")
    from selectssm_b200 import jax_ffi  # noqa: F401  (exercised only where JAX exists)


def test_jax_binding_imports_without_torch():
    """The JAX host path needs no PyTorch: importing the binding in a process
    where ``import torch`` fails still works, and keeps the reference's
    ValueErrors (selectssm.py:47-48, :53-54)."""
    import subprocess
    import sys
    code = (
        "import sys; sys.modules['torch'] = None\n"
        "from selectssm_b200 import jax_ffi\n"
        "assert jax_ffi.largest_factor_up_to(64, 1024) == 64\n"
        "try:\n"
        "    jax_ffi._check_chunked(1000, 8, 64, 1)\n"
        "except ValueError:\n"
        "    pass\n"
        "else:\n"
        "    raise SystemExit('no ValueError')\n"
        "assert 'torch' not in [m for m in sys.modules if sys.modules[m] is not None]\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr
