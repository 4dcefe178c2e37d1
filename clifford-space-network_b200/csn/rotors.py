"""Toolkit rotor API, drop-in for csn_toolkit/csn/rotors.py.

The toolkit's Cayley convention is Q = (I - Omega)(I + Omega)^{-1}
(csn_toolkit/csn/rotors.py:54-115), the transpose of the python/ convention; this
module keeps it: cayley_rotor_*(Omega) = exact_cayley(-Omega) = exact_cayley(Omega)^T.
``use_schulz`` is accepted and ignored: every rotor is exact (the reference's fixed
Schulz iteration count does not converge at block magnitudes).

schulz_inverse_* keep the reference's semantics -- a fixed number of Newton-Schulz
steps X <- X (2I - A X) from X_0 = A^T / |A|_F^2 (csn_toolkit/csn/rotors.py:20-51);
they are helpers outside the scan path and run as batched PyTorch matmuls.
"""
import torch

from csn_b200 import ops


def _schulz(A: torch.Tensor, max_iters: int) -> torch.Tensor:
    D = A.shape[-1]
    I = torch.eye(D, dtype=A.dtype, device=A.device).expand_as(A)
    norm_est = torch.norm(A, p="fro", dim=(-2, -1), keepdim=True).clamp(min=1e-6)
    X = A.transpose(-1, -2) / (norm_est ** 2)
    for _ in range(max_iters):
        X = torch.matmul(X, 2.0 * I - torch.matmul(A, X))
    return X


def schulz_inverse_4x4(A: torch.Tensor, max_iters: int = 5) -> torch.Tensor:
    return _schulz(A, max_iters)


def schulz_inverse_16x16(A: torch.Tensor, max_iters: int = 6) -> torch.Tensor:
    return _schulz(A, max_iters)


def cayley_rotor_4x4(Omega: torch.Tensor, use_schulz: bool = True) -> torch.Tensor:
    return ops.cayley(-Omega)


def cayley_rotor_8x8(Omega: torch.Tensor, use_schulz: bool = True) -> torch.Tensor:
    return ops.cayley(-Omega)


def cayley_rotor_16x16(Omega: torch.Tensor, use_schulz: bool = True) -> torch.Tensor:
    return ops.cayley(-Omega)
