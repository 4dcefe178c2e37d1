"""Clifford-LTC / TENN cell, drop-in for python/clifford_layer.py.

Same parameters (W_rec, W_in, gamma_bias, bivector_bias), same forward signature and
return value (next, next).  The step runs as a CUDA kernel (csn_cell_fwd / _bwd);
bivector_bias is kept for state_dict compatibility and, as in the reference
(python/clifford_layer.py:71-115), does not enter the computation.
"""
import math
from typing import Tuple

import torch
import torch.nn as nn

from csn_b200 import ops


class CliffordTENNCell(nn.Module):
    def __init__(self, num_neurons: int = 32, in_dim: int = 8, algebra_dim: int = 16):
        super().__init__()
        if algebra_dim != 16:
            raise ValueError("CliffordTENNCell is defined for Cl(4,0) ~ M_4(R): algebra_dim=16")
        self.num_neurons = num_neurons
        self.in_dim = in_dim
        self.algebra_dim = algebra_dim
        self.W_rec = nn.Parameter(torch.randn(num_neurons, num_neurons, algebra_dim)
                                  * (0.05 / math.sqrt(num_neurons)))
        self.W_in = nn.Parameter(torch.randn(num_neurons, in_dim, algebra_dim) * (0.1 / math.sqrt(in_dim)))
        self.gamma_bias = nn.Parameter(torch.zeros(num_neurons))
        self.bivector_bias = nn.Parameter(torch.zeros(num_neurons, 6))

    def init_state(self, batch_size: int, device: torch.device) -> torch.Tensor:
        return torch.zeros(batch_size, self.num_neurons, self.algebra_dim, device=device)

    def forward(self, x_t: torch.Tensor, prev_state: torch.Tensor, dt: float = 0.02
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        nxt = ops.cell_step(x_t, prev_state, self.W_rec, self.W_in, self.gamma_bias, dt)
        return nxt, nxt
