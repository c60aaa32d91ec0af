"""selectssm_b200: the selectssm selective-scan hot path on B200 (sm_100a).

Public names follow the reference package (src/selectssm/__init__.py:1-2):
``ssm_chunked_scan``, ``ssm_recursive_scan``, ``ssm_scan``, ``SelectiveSSM``,
``BidirectionalMamba``; plus the fused op ``selective_scan`` and the
conv preamble ``conv1d_act``.

The PyTorch host layer (ops, modules, rcps) is imported on first use of one of
its names, so the JAX binding (``selectssm_b200.jax_ffi``) and the C-ABI loader
(``selectssm_b200._lib``) import without PyTorch.
"""

from ._checks import largest_factor_up_to  # noqa: F401

__version__ = "0.1.0"

_LAZY = {
    "conv1d_act": "ops", "dense_onto": "ops", "rmsnorm_residual": "ops", "selective_scan": "ops",
    "selective_scan_bidir": "ops", "ssm_chunked_scan": "ops", "ssm_recursive_scan": "ops", "ssm_scan": "ops",
    "BidirectionalMamba": "modules", "SelectiveSSM": "modules",
    "RCPSEmbedding": "rcps", "RCPSLMHead": "rcps", "RCPSNorm": "rcps", "RCPSWrapper": "rcps",
    "rc_conjugate": "rcps",
}
__all__ = sorted(_LAZY) + ["largest_factor_up_to"]


def __getattr__(name):
    mod = _LAZY.get(name)
    if mod is None:
        raise AttributeError(f"module 'selectssm_b200' has no attribute {name!r}")
    import importlib
    value = getattr(importlib.import_module(f".{mod}", __name__), name)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(_LAZY))
