"""Cl(8,0) ~ M_16(R) block, drop-in for python/clifford_cl8.py.

Deviation from the reference, on purpose: ``use_schulz`` is accepted but every rotor
is the EXACT Cayley transform.  The reference's 5-step Schulz iteration
(python/clifford_cl8.py:47-62) has not converged at the block's magnitudes (12.7 %
off the exact rotor, |Q^T Q - I| = 0.24), which would break the rotor-norm contract
|R R~ - 1| <= 1e-5.  With use_schulz=False the reference and this module agree.
"""
import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from csn_b200 import ops
from csn_b200.modules import LayerNorm, causal_conv_input, generator_inputs
from python.clifford_cl6 import AdaptiveTimeHead, generator_action, read_diagnostics, skew_from_generators
from python.clifford_model import GeometricGatedLinearUnit, RiemannianGeodesicHead
from python.clifford_scan import parallel_rotor_scan, surrogate_spike  # noqa: F401 (re-export)


def cayley_rotor_16x16(Omega: torch.Tensor, use_schulz: bool = True) -> torch.Tensor:
    """Exact Q = (I - Omega)^{-1} (I + Omega) for skew 16 x 16 Omega (use_schulz ignored)."""
    return ops.cayley(Omega)


def cayley_rotor_4x4(Omega: torch.Tensor, use_schulz: bool = True) -> torch.Tensor:
    """Exact Q = (I - Omega)^{-1} (I + Omega) for skew 4 x 4 Omega (use_schulz ignored)."""
    return ops.cayley(Omega)


class CliffordCL8Block(nn.Module):
    def __init__(self, d_model: int, num_neurons: int = 2, kernel_size: int = 4, dt_base: float = 0.05,
                 spike_threshold: float = 0.1, spike_beta: float = 10.0, use_schulz: bool = True,
                 is_spinor_bundle: bool = False):
        super().__init__()
        self.d_model = d_model
        self.num_neurons = num_neurons
        self.dt_base = dt_base
        self.spike_threshold = spike_threshold
        self.spike_beta = spike_beta
        self.use_schulz = use_schulz
        self.is_spinor_bundle = is_spinor_bundle
        self.num_biv = 120
        self.ln_1 = LayerNorm(d_model)
        self.conv1d = nn.Conv1d(d_model, d_model, kernel_size=kernel_size, padding=kernel_size - 1,
                                groups=d_model)
        self.time_head = AdaptiveTimeHead(d_model, dt_base=dt_base)
        self.in_proj = nn.Linear(d_model, num_neurons * 256)
        self.gamma_proj = nn.Linear(d_model, num_neurons)
        self.biv_proj = nn.Linear(d_model, num_neurons * self.num_biv)
        self.omega_scale = nn.Parameter(torch.ones(num_neurons, 1) * 10.0)
        self.W_mix = nn.Parameter(torch.randn(num_neurons, num_neurons) / math.sqrt(num_neurons))
        self.out_proj = nn.Linear(num_neurons * 256, d_model)
        self.ln_2 = LayerNorm(d_model)
        self.gglu = GeometricGatedLinearUnit(d_model, d_ffn=2 * d_model)
        u, v = torch.triu_indices(16, 16, offset=1)
        self.register_buffer("triu_u", u, persistent=False)
        self.register_buffer("triu_v", v, persistent=False)

    def mixed_out_weight(self) -> torch.Tensor:
        """out_proj's weight with the inter-neuron mixing folded in (python/clifford_cl8.py:189-193):
        W[o, j*256 + rc] = sum_i W_out[o, i*256 + rc] W_mix[i, j]."""
        N = self.num_neurons
        W = self.out_proj.weight.view(self.d_model, N, 256)
        return torch.einsum("oir,ij->ojr", W, self.W_mix).reshape(self.d_model, N * 256)

    def forward_core(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """forward() without Omega: (out, biv [B, T, N, 120] scaled generators, dt [B, T])."""
        B, T, _ = x.shape
        N = self.num_neurons
        residual = x
        x_conv = causal_conv_input(self.ln_1, self.conv1d, x)      # ln_1 -> causal conv -> SiLU, fused
        S = ops.linear(x_conv, self.in_proj.weight, self.in_proj.bias).view(B, T, N, 16, 16)
        biv, gamma, dt = generator_inputs(x_conv, self.biv_proj, self.gamma_proj, self.time_head.proj,
                                          self.omega_scale, self.time_head.dt_base)
        biv, dt = biv.view(B, T, N, self.num_biv), dt.view(B, T)
        X_all = ops.fused_rotor_scan(biv, dt, gamma, S, two_sided=not self.is_spinor_bundle)
        X_spiked = ops.state_spike(X_all, self.spike_threshold, self.spike_beta)
        h = residual + ops.linear(X_spiked.view(B, T, N * 256), self.mixed_out_weight(), self.out_proj.bias)
        out = h + self.gglu(self.ln_2(h))
        return out, biv, dt

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        out, biv, dt = self.forward_core(x)
        Omega = skew_from_generators(biv, 16, self.triu_u, self.triu_v) * (0.5 * dt)[..., None, None, None]
        return out, Omega, dt


class CliffordCL8ForCausalLM(nn.Module):
    def __init__(self, vocab_size: int, d_model: int = 48, num_layers: int = 2, num_neurons: int = 2,
                 dt_base: float = 0.05, kernel_size: int = 4, spike_threshold: float = 0.1,
                 lambda_kin: float = 0.01, lambda_smooth: float = 0.005, lambda_time: float = 0.01,
                 use_schulz: bool = True, is_spinor_bundle: bool = False):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.num_layers = num_layers
        self.dt_base = dt_base
        self.lambda_kin = lambda_kin
        self.lambda_smooth = lambda_smooth
        self.lambda_time = lambda_time
        self.use_schulz = use_schulz
        self.is_spinor_bundle = is_spinor_bundle
        self.tok_emb = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([
            CliffordCL8Block(d_model=d_model, num_neurons=num_neurons, kernel_size=kernel_size,
                             dt_base=dt_base, spike_threshold=spike_threshold, use_schulz=use_schulz,
                             is_spinor_bundle=is_spinor_bundle)
            for _ in range(num_layers)])
        self.ln_f = LayerNorm(d_model)
        self.head = RiemannianGeodesicHead(vocab_size=vocab_size, d_model=d_model)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None):
        B, T = idx.shape
        x = self.tok_emb(idx)
        e_kin = 0.0
        e_smooth = 0.0
        t_loss = 0.0
        dts = []
        for block in self.blocks:
            x, biv, dt_t = block.forward_core(x)
            dts.append(dt_t)
            kin, smooth = generator_action(biv, dt_t, 16)
            e_kin = e_kin + kin
            if T > 1:
                e_smooth = e_smooth + smooth
                t_loss = t_loss + (((dt_t[:, 1:] - dt_t[:, :-1]) / self.dt_base) ** 2).mean()
        logits = self.head(self.ln_f(x))
        stacked = torch.stack(dts)
        named = {"mean_dt": stacked.mean(), "min_dt": stacked.min(), "max_dt": stacked.max()}
        loss = None
        if targets is not None:
            ce = F.cross_entropy(logits.view(-1, self.vocab_size), targets.view(-1))
            action = self.lambda_kin * e_kin + self.lambda_smooth * e_smooth
            time_pen = self.lambda_time * t_loss
            loss = ce + action + time_pen
            named.update(ce_loss=ce, action_loss=action, time_loss=time_pen)
        diagnostics: Dict[str, float] = read_diagnostics(named)
        return logits, loss, diagnostics
