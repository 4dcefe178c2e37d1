"""Cl(4,0) block and the shared heads, drop-in for python/clifford_model.py.

RiemannianGeodesicHead and GeometricGatedLinearUnit are plain PyTorch modules with the
reference's parameters (python/clifford_model.py:24-75).  CliffordTENNBlock builds the
reference's symmetric rational rotor Q = (I + Om)(I - Om) / (1 + |Om|^2/8)
(python/clifford_model.py:165-180) in PyTorch and runs the scan on the CUDA library; its
spike is the CUDA state-spike kernel, its inter-neuron mixing is folded into out_proj's weight
and its LayerNorms run the CUDA LayerNorm kernels, as in the Cl(6) block.
"""
import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from csn_b200 import ops
from csn_b200.modules import LayerNorm, causal_conv_input
from python.clifford_scan import parallel_rotor_scan, surrogate_spike  # noqa: F401 (re-export)


class RiemannianGeodesicHead(nn.Module):
    def __init__(self, vocab_size: int, d_model: int, init_scale: float = 16.0):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.prototypes = nn.Parameter(torch.randn(vocab_size, d_model) / math.sqrt(d_model))
        self.scale = nn.Parameter(torch.tensor(float(init_scale)))
        self.bias = nn.Parameter(torch.zeros(vocab_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        norm_x = F.normalize(x, p=2, dim=-1)
        norm_proto = F.normalize(self.prototypes, p=2, dim=-1)
        return self.scale * torch.matmul(norm_x, norm_proto.t()) + self.bias


class GeometricGatedLinearUnit(nn.Module):
    def __init__(self, d_model: int, d_ffn: Optional[int] = None):
        super().__init__()
        if d_ffn is None:
            d_ffn = int(2 * d_model)
        self.w_gate = nn.Linear(d_model, d_ffn, bias=False)
        self.w_up = nn.Linear(d_model, d_ffn, bias=False)
        self.w_down = nn.Linear(d_ffn, d_model, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # w_gate and w_up as one GEMM, silu(g) * u as one CUDA kernel each way
        gu = ops.linear(x, torch.cat([self.w_gate.weight, self.w_up.weight], 0))
        return ops.linear(ops.silu_gate(gu), self.w_down.weight)


class CliffordTENNBlock(nn.Module):
    def __init__(self, d_model: int, num_neurons: int = 16, kernel_size: int = 4,
                 spike_threshold: float = 0.1, spike_beta: float = 10.0):
        super().__init__()
        self.d_model = d_model
        self.num_neurons = num_neurons
        self.spike_threshold = spike_threshold
        self.spike_beta = spike_beta
        self.ln_1 = LayerNorm(d_model)
        self.conv1d = nn.Conv1d(d_model, d_model, kernel_size=kernel_size, padding=kernel_size - 1,
                                groups=d_model)
        self.in_proj = nn.Linear(d_model, num_neurons * 16)
        self.gamma_proj = nn.Linear(d_model, num_neurons)
        self.biv_proj = nn.Linear(d_model, num_neurons * 6)
        self.omega_scale = nn.Parameter(torch.ones(num_neurons, 1) * 10.0)
        self.W_mix = nn.Parameter(torch.randn(num_neurons, num_neurons) * (1.0 / math.sqrt(num_neurons)))
        self.out_proj = nn.Linear(num_neurons * 16, d_model)
        self.ln_2 = LayerNorm(d_model)
        self.gglu = GeometricGatedLinearUnit(d_model, d_ffn=2 * d_model)
        u, v = torch.triu_indices(4, 4, offset=1)
        self.register_buffer("_triu_u", u, persistent=False)
        self.register_buffer("_triu_v", v, persistent=False)

    def forward(self, x: torch.Tensor, dt: float = 0.05) -> Tuple[torch.Tensor, torch.Tensor]:
        B, T, _ = x.shape
        residual = x
        x_conv = causal_conv_input(self.ln_1, self.conv1d, x)      # ln_1 -> causal conv -> SiLU, fused
        S = self.in_proj(x_conv).view(B, T, self.num_neurons, 4, 4)
        gamma = F.softplus(self.gamma_proj(x_conv))
        decay = torch.sigmoid(-gamma * dt).unsqueeze(-1).unsqueeze(-1)
        biv = self.biv_proj(x_conv).view(B, T, self.num_neurons, 6) * self.omega_scale
        skew = torch.zeros(B, T, self.num_neurons, 4, 4, device=x.device, dtype=x.dtype)
        skew[..., self._triu_u, self._triu_v] = biv
        skew[..., self._triu_v, self._triu_u] = -biv
        Omega = skew * (0.5 * dt)
        eye = torch.eye(4, device=x.device, dtype=x.dtype)
        denom = 1.0 + 0.25 * (0.5 * torch.sum(Omega ** 2, dim=(-1, -2), keepdim=True))
        Q = torch.matmul(eye + Omega, eye - Omega) / denom
        X_all = parallel_rotor_scan(torch.sqrt(decay) * Q, (1.0 - decay) * S)
        X_spiked = ops.state_spike(X_all, self.spike_threshold, self.spike_beta)
        N = self.num_neurons
        # mixing folded into out_proj: W[o, j*16 + rc] = sum_i W_out[o, i*16 + rc] W_mix[i, j]
        W = torch.einsum("oir,ij->ojr", self.out_proj.weight.view(self.d_model, N, 16), self.W_mix)
        h = residual + F.linear(X_spiked.reshape(B, T, N * 16), W.reshape(self.d_model, N * 16), self.out_proj.bias)
        return h + self.gglu(self.ln_2(h)), Omega


class CliffordTENNForCausalLM(nn.Module):
    def __init__(self, vocab_size: int, d_model: int = 64, num_layers: int = 2, num_neurons: int = 16,
                 kernel_size: int = 4, spike_threshold: float = 0.1, lambda_kin: float = 0.02,
                 lambda_smooth: float = 0.01):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.num_layers = num_layers
        self.lambda_kin = lambda_kin
        self.lambda_smooth = lambda_smooth
        self.tok_emb = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([CliffordTENNBlock(d_model, num_neurons, kernel_size, spike_threshold)
                                     for _ in range(num_layers)])
        self.ln_f = LayerNorm(d_model)
        self.head = RiemannianGeodesicHead(vocab_size=vocab_size, d_model=d_model)

    def forward(self, idx: torch.Tensor, dt: float = 0.05, targets: Optional[torch.Tensor] = None):
        B, T = idx.shape
        x = self.tok_emb(idx)
        e_kin = 0.0
        e_smooth = 0.0
        for block in self.blocks:
            x, Omega = block(x, dt=dt)
            e_kin = e_kin + (Omega ** 2).mean()
            if T > 1:
                e_smooth = e_smooth + ((Omega[:, 1:] - Omega[:, :-1]) ** 2).mean()
        logits = self.head(self.ln_f(x))
        loss, action = None, 0.0
        if targets is not None:
            ce = F.cross_entropy(logits.view(-1, self.vocab_size), targets.view(-1))
            pen = self.lambda_kin * e_kin + self.lambda_smooth * e_smooth
            loss = ce + pen
            action = float(pen)
        return logits, loss, action
