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


def causal_conv_input(ln: nn.LayerNorm, conv: nn.Conv1d, x: torch.Tensor) -> torch.Tensor:
    """x_conv = silu(conv(ln(x).transpose(1, 2))[:, :, :T].transpose(1, 2)) of the blocks
    (python/clifford_cl6.py:140-142), as the fused CUDA kernels when the layers have the blocks'
    form (affine LayerNorm over C; depthwise, bias, stride 1, dilation 1, left padding K - 1
    conv) and the sizes fit them; otherwise the same chain of library layers."""
    T = x.shape[1]
    C = x.shape[-1]
    K = conv.kernel_size[0]
    if (x.dim() == 3 and len(ln.normalized_shape) == 1 and ln.weight is not None and ln.bias is not None
            and conv.groups == C == conv.in_channels == conv.out_channels and conv.bias is not None
            and conv.stride == (1,) and conv.dilation == (1,) and conv.padding == (K - 1,)
            and conv.padding_mode == "zeros" and ops.ln_conv_silu_supported(C, K)):
        return ops.ln_conv_silu(x, ln.weight, ln.bias, ln.eps, conv.weight, conv.bias)
    return F.silu(conv(ln(x).transpose(1, 2))[:, :, :T].transpose(1, 2))


def generator_inputs(x: torch.Tensor, biv_proj: nn.Linear, gamma_proj: nn.Linear, time_proj: nn.Linear,
                     omega_scale: torch.Tensor, dt_base: float):
    """(biv [..., N*K], gamma [..., N], dt [..., HT]) of the blocks' projections
    (python/clifford_cl6.py:144-155: biv_proj(x) * omega_scale, softplus(gamma_proj(x)),
    softplus(time_head.proj(x)) * dt_base) as ONE GEMM over the concatenated weights and the
    CUDA projection epilogue; the parameters stay the three nn.Linear layers'."""
    N = gamma_proj.out_features
    HT = time_proj.out_features
    K = biv_proj.out_features // N
    W = torch.cat([biv_proj.weight, gamma_proj.weight, time_proj.weight], 0)
    b = torch.cat([biv_proj.bias, gamma_proj.bias, time_proj.bias], 0)
    raw = ops.linear(x, W, b)
    return ops.projection_epilogue(raw, omega_scale, dt_base, N, K, HT)
