"""csn_b200 -- B200-native (sm_100a) rotor-scan hot path of Clifford Space Networks.

Public ops live in :mod:`csn_b200.ops`; the reference-compatible module API lives in
the sibling packages ``python`` and ``csn`` (same import paths as the reference).
"""
from . import algebra  # noqa: F401  (pure numpy, no CUDA needed)

__version__ = "0.1.0"


def __getattr__(name):
    # ops import torch lazily so that `import csn_b200` stays cheap for the build step
    if name in ("rotor_scan", "fused_rotor_scan", "cayley"):
        import importlib
        return getattr(importlib.import_module(".ops", __name__), name)
    raise AttributeError(name)
