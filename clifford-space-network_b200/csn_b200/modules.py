"""nn.Module front ends of the block kernels, parameter-compatible with torch.nn."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


class LayerNorm(nn.LayerNorm):
    """nn.LayerNorm (same parameters, state_dict keys and eps) computed by the CUDA LayerNorm
    kernels (csn_layer_norm_fwd / _bwd) for one normalised axis of C % 4 == 0, C <= 1024
    features with affine weight and bias; other shapes go to F.layer_norm."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        C = x.shape[-1]
        if (len(self.normalized_shape) == 1 and self.weight is not None and self.bias is not None
                and ops.layer_norm_supported(C)):
            return ops.layer_norm(x, self.weight, self.bias, self.eps)
        return F.layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)
