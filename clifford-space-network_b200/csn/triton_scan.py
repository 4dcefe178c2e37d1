"""Compatibility module for csn_toolkit/csn/triton_scan.py.

This build has no Triton path (sm_100a CUDA only).  The names are kept so callers that
import them still work: ``triton_clifford_scan`` runs the same one-sided D = 4 scan on
the CUDA library and ``is_triton_available`` reports whether that library is usable.
"""
import torch

from csn.cuda import fused_cuda_clifford_scan, is_fused_cuda_available


def is_triton_available() -> bool:
    return is_fused_cuda_available()


def triton_clifford_scan(M: torch.Tensor, C: torch.Tensor) -> torch.Tensor:
    return fused_cuda_clifford_scan(M, C)
