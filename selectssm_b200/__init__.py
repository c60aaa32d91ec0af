"""selectssm_b200: the selectssm selective-scan hot path on B200 (sm_100a).

Public names follow the reference package (src/selectssm/__init__.py:1-2):
``ssm_chunked_scan``, ``ssm_recursive_scan``, ``ssm_scan``, ``SelectiveSSM``,
``BidirectionalMamba``; plus the fused op ``selective_scan`` and the
conv preamble ``conv1d_act``.
"""

from .ops import (  # noqa: F401
    conv1d_act,
    dense_onto,
    largest_factor_up_to,
    rmsnorm_residual,
    selective_scan,
    selective_scan_bidir,
    ssm_chunked_scan,
    ssm_recursive_scan,
    ssm_scan,
)

__version__ = "0.1.0"
from .modules import BidirectionalMamba, SelectiveSSM  # noqa: F401,E402
from .rcps import RCPSEmbedding, RCPSLMHead, RCPSNorm, RCPSWrapper, rc_conjugate  # noqa: F401,E402
