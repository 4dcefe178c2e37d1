"""Fused CUDA scan entry points, drop-in for csn_toolkit/csn/cuda/__init__.py.

``fused_cuda_clifford_scan(M[S,T,4,4], C)`` is the one-sided D = 4 scan with its
reverse-time adjoint (csn_toolkit/csn/cuda/__init__.py:54-92).  The reference JIT-
compiles csn_fast_scan_cuda on first use; here the prebuilt libcsn_b200.so is loaded.
There is no silent fallback: load failures raise.
"""
import torch
from torch.autograd import Function

from csn_b200 import _lib, ops


def load_cuda_scan_extension():
    """Return the loaded library handle (csn_toolkit/csn/cuda/__init__.py:16-51)."""
    return _lib.load()


class FusedCudaCliffordScanFunction(Function):
    @staticmethod
    def forward(ctx, M: torch.Tensor, C: torch.Tensor):
        S, T = M.shape[:2]
        X = ops.ScanFunction.forward(ctx, M.reshape(S, T, 1, 4, 4), C.reshape(S, T, 1, 4, 4), None, False)
        return X.view(S, T, 4, 4)

    @staticmethod
    def backward(ctx, grad_X: torch.Tensor):
        S, T = grad_X.shape[:2]
        dM, dC, _, _ = ops.ScanFunction.backward(ctx, grad_X.reshape(S, T, 1, 4, 4))
        return dM.view(S, T, 4, 4), dC.view(S, T, 4, 4)


def fused_cuda_clifford_scan(M: torch.Tensor, C: torch.Tensor) -> torch.Tensor:
    """M, C: [S, T, 4, 4] -> X [S, T, 4, 4], X_t = M_t X_{t-1} + C_t, X_0 = C_0."""
    if M.dim() != 4 or M.shape[-2:] != (4, 4) or C.shape != M.shape:
        raise ValueError("fused_cuda_clifford_scan expects M, C of shape [S, T, 4, 4]")
    return FusedCudaCliffordScanFunction.apply(M, C)


def is_fused_cuda_available() -> bool:
    """True when the library loads and a CUDA device is present."""
    try:
        _lib.load()
    except (RuntimeError, OSError):
        return False
    return torch.cuda.is_available()
