"""B200-native (sm_100a) selective-scan hot path of MotifMamba.

Public API (same signatures as the reference's ``mamba_ssm`` / ``causal_conv1d``):
``selective_scan_fn``, ``mamba_inner_fn``, ``causal_conv1d_fn``, ``causal_conv1d_update``,
``selective_state_update``; the raw extension API is ``motif_ssm.selective_scan_cuda``
(``fwd`` / ``bwd``).  ``motif_ssm.shims.install()`` registers the reference's module names.
Importing this package loads ``libmotif_ssm.so`` and raises if it is missing.
"""
from ._lib import CHUNK_LEN, MAX_DSTATE, VERSION, MotifSsmError  # noqa: F401
from . import selective_scan_cuda  # noqa: F401
from .causal_conv1d import causal_conv1d_fn, causal_conv1d_update  # noqa: F401
from .selective_scan_interface import mamba_inner_fn, selective_scan_fn  # noqa: F401
from .selective_state_update import selective_state_update  # noqa: F401
