"""Associative rotor scan, drop-in for python/clifford_scan.py.

    X_t = M_t X_{t-1} M_t^T + C_t   (default, two-sided)     X_0 = C_0
    X_t = M_t X_{t-1} + C_t         (is_spinor_bundle=True)

``parallel_rotor_scan`` has the reference signature (python/clifford_scan.py:41) and
returns the same trajectory, computed by the chunked CUDA scan (work-efficient,
O(T) instead of the reference's O(T log T) Hillis-Steele tree with padding).
"""
import torch

from csn_b200 import ops


def rotor_binary_op(M_b: torch.Tensor, C_b: torch.Tensor, M_a: torch.Tensor, C_a: torch.Tensor,
                    is_spinor_bundle: bool = False):
    """Compose two scan elements, (M_b, C_b) o (M_a, C_a) = (M_b M_a, M_b C_a M_b^T + C_b)
    (one-sided: M_b C_a + C_b).  Same as python/clifford_scan.py:19-38."""
    M_new = torch.matmul(M_b, M_a)
    if is_spinor_bundle:
        C_new = torch.matmul(M_b, C_a) + C_b
    else:
        C_new = torch.matmul(torch.matmul(M_b, C_a), M_b.transpose(-1, -2)) + C_b
    return M_new, C_new


def parallel_rotor_scan(M: torch.Tensor, C: torch.Tensor, is_spinor_bundle: bool = False) -> torch.Tensor:
    """M, C: [B, T, N, D, D] (D in 4, 8, 16) -> X: [B, T, N, D, D]."""
    return ops.rotor_scan(M, C, two_sided=not is_spinor_bundle)


class SurrogateSpikeFunction(torch.autograd.Function):
    """Heaviside forward, fast-sigmoid surrogate backward 1 / (1 + beta |x|)^2
    (python/clifford_scan.py:92-111)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, beta: float = 10.0):
        ctx.save_for_backward(x)
        ctx.beta = beta
        return (x >= 0.0).float()

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, = ctx.saved_tensors
        surrogate_grad = 1.0 / (1.0 + ctx.beta * torch.abs(x)) ** 2
        return grad_output * surrogate_grad, None


def surrogate_spike(x: torch.Tensor, threshold: float = 0.5, beta: float = 10.0) -> torch.Tensor:
    return SurrogateSpikeFunction.apply(x - threshold, beta)
