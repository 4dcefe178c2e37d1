"""Clifford Space Network toolkit -- scan and rotor API (drop-in for csn_toolkit/csn).

Exports the scan and rotor names of csn_toolkit/csn/__init__.py.  The toolkit's vision
detector, losses and transformer LM (csn.vision, csn.loss, csn.transformer) are callers
of the scan, not part of it, and are not provided by this package.
"""
from csn.scan import CliffordScanFunction, parallel_rotor_scan, rotor_binary_op, surrogate_spike
from csn.rotors import (cayley_rotor_4x4, cayley_rotor_8x8, cayley_rotor_16x16, schulz_inverse_4x4,
                        schulz_inverse_16x16)

__version__ = "1.0.0"

__all__ = [
    "CliffordScanFunction", "parallel_rotor_scan", "rotor_binary_op", "surrogate_spike",
    "cayley_rotor_4x4", "cayley_rotor_8x8", "cayley_rotor_16x16", "schulz_inverse_4x4",
    "schulz_inverse_16x16",
]
