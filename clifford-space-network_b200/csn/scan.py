"""Toolkit scan API, drop-in for csn_toolkit/csn/scan.py.

One backend: the CUDA library.  ``backend`` ("auto" / "cuda" / "triton" / "pytorch")
and ``force_tree`` are accepted for signature compatibility and select the same
kernels; the result is the reference's trajectory in every case.  The toolkit default
is the one-sided ("spinor bundle") recurrence X_t = M_t X_{t-1} + C_t
(csn_toolkit/csn/scan.py:96-102); is_spinor_bundle=False gives the two-sided one.
"""
import math
from typing import Literal, Tuple

import torch

from csn_b200 import ops


class CliffordScanFunction(torch.autograd.Function):
    """One-sided sequential scan with the analytic reverse-time adjoint
    (csn_toolkit/csn/scan.py:16-72), on the CUDA kernels."""

    @staticmethod
    def forward(ctx, M: torch.Tensor, C: torch.Tensor) -> torch.Tensor:
        return ops.ScanFunction.forward(ctx, M, C, None, False)

    @staticmethod
    def backward(ctx, grad_X: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        dM, dC, _, _ = ops.ScanFunction.backward(ctx, grad_X)
        return dM, dC


def rotor_binary_op(M_right: torch.Tensor, C_right: torch.Tensor, M_left: torch.Tensor,
                    C_left: torch.Tensor, is_spinor_bundle: bool = True):
    """(M_r, C_r) o (M_l, C_l) (csn_toolkit/csn/scan.py:75-93)."""
    M_new = torch.matmul(M_right, M_left)
    if is_spinor_bundle:
        C_new = torch.matmul(M_right, C_left) + C_right
    else:
        C_new = torch.matmul(torch.matmul(M_right, C_left), M_right.transpose(-1, -2)) + C_right
    return M_new, C_new


def parallel_rotor_scan(M: torch.Tensor, C: torch.Tensor, is_spinor_bundle: bool = True,
                        force_tree: bool = False,
                        backend: Literal["auto", "cuda", "triton", "pytorch"] = "auto") -> torch.Tensor:
    """M, C: [B, T, N, D, D] -> X [B, T, N, D, D] (csn_toolkit/csn/scan.py:96-151)."""
    if backend not in ("auto", "cuda", "triton", "pytorch"):
        raise ValueError(f"unknown backend {backend!r}")
    return ops.rotor_scan(M, C, two_sided=not is_spinor_bundle)


def _parallel_tree_scan(M: torch.Tensor, C: torch.Tensor, is_spinor_bundle: bool = True) -> torch.Tensor:
    """Same trajectory as the reference's padded log-depth tree (csn_toolkit/csn/scan.py:154-187)."""
    return ops.rotor_scan(M, C, two_sided=not is_spinor_bundle)


class SurrogateSpike(torch.autograd.Function):
    """Heaviside forward, alpha / (2 (1 + (pi/2 alpha x)^2)) surrogate backward
    (csn_toolkit/csn/scan.py:190-203)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, alpha: float = 2.0) -> torch.Tensor:
        ctx.save_for_backward(x)
        ctx.alpha = alpha
        return (x > 0.0).float()

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, = ctx.saved_tensors
        a = ctx.alpha
        return grad_output * (a / (2.0 * (1.0 + (math.pi / 2.0 * a * x).pow(2)))), None


surrogate_spike = SurrogateSpike.apply
