"""Multi-head Cl(6,0) block and LM, drop-in for python/clifford_multihead.py.

Same parameters (state_dict keys and shapes), inputs and outputs as the reference's
MultiHeadAdaptiveTime, MultiHeadCliffordCL6Block and MultiHeadCliffordLM
(python/clifford_multihead.py:28-304).  The scan section (:137-173) -- skew generators,
Omega, exact Cayley rotors, per-head decay, the fold of heads into the batch, M/C and the scan
over [B*H, T, Nh] -- runs as ONE fused CUDA op (csn_b200.ops.fused_rotor_scan_heads) that reads
the [B, T, H, Nh, ...] projections in place with one dt per head: nothing is folded, unfolded
or transposed, and M, C and Q are never materialised.  The spike is one CUDA kernel each way,
the per-head mixing is folded into out_proj's weight and the LayerNorms run the CUDA kernels,
as in the Cl(6) block.  Omega is still returned by forward(); the LM takes its action
regulariser from the generator coefficients instead.
"""
import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from csn_b200 import ops
from csn_b200.modules import LayerNorm, causal_conv_input, generator_inputs
from python.clifford_cl6 import (cayley_rotor_8x8, generator_action, read_diagnostics,  # noqa: F401
                                 skew_from_generators)
from python.clifford_model import GeometricGatedLinearUnit, RiemannianGeodesicHead
from python.clifford_scan import parallel_rotor_scan, surrogate_spike  # noqa: F401 (re-export)


class MultiHeadAdaptiveTime(nn.Module):
    """Per-head dt_t^(h) = softplus(W^(h) x_t + b^(h)) * dt_base, initialised at dt_base
    (python/clifford_multihead.py:28-53).  Returns [B, T, H]."""

    def __init__(self, d_model: int, num_heads: int, dt_base: float = 0.05):
        super().__init__()
        self.num_heads = num_heads
        self.dt_base = dt_base
        self.proj = nn.Linear(d_model, num_heads)
        nn.init.zeros_(self.proj.weight)
        nn.init.constant_(self.proj.bias, math.log(math.e - 1.0))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.softplus(self.proj(x)) * self.dt_base


class MultiHeadCliffordCL6Block(nn.Module):
    def __init__(self, d_model: int, num_heads: int = 3, num_neurons_per_head: int = 2,
                 kernel_size: int = 4, dt_base: float = 0.05, spike_threshold: float = 0.1,
                 spike_beta: float = 10.0):
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.num_neurons_per_head = num_neurons_per_head
        self.total_neurons = num_heads * num_neurons_per_head
        self.dt_base = dt_base
        self.spike_threshold = spike_threshold
        self.spike_beta = spike_beta
        self.ln_1 = LayerNorm(d_model)
        self.conv1d = nn.Conv1d(d_model, d_model, kernel_size=kernel_size, padding=kernel_size - 1,
                                groups=d_model)
        self.time_head = MultiHeadAdaptiveTime(d_model, num_heads=num_heads, dt_base=dt_base)
        self.in_proj = nn.Linear(d_model, self.total_neurons * 64)
        self.gamma_proj = nn.Linear(d_model, self.total_neurons)
        self.biv_proj = nn.Linear(d_model, self.total_neurons * 28)
        self.omega_scale = nn.Parameter(torch.ones(num_heads, num_neurons_per_head, 1) * 10.0)
        self.W_mix = nn.Parameter(torch.randn(num_heads, num_neurons_per_head, num_neurons_per_head)
                                  / math.sqrt(num_neurons_per_head))
        self.out_proj = nn.Linear(self.total_neurons * 64, d_model)
        self.ln_2 = LayerNorm(d_model)
        self.gglu = GeometricGatedLinearUnit(d_model, d_ffn=2 * d_model)
        self.register_buffer("triu_u", torch.triu_indices(8, 8, offset=1)[0], persistent=False)
        self.register_buffer("triu_v", torch.triu_indices(8, 8, offset=1)[1], persistent=False)

    def mixed_out_weight(self) -> torch.Tensor:
        """out_proj's weight with the block-diagonal head mixing folded in
        (python/clifford_multihead.py:184-191): W[o, (h, n, rc)] = sum_m W_out[o, (h, m, rc)] W_mix[h, m, n]."""
        H, Nh = self.num_heads, self.num_neurons_per_head
        W = self.out_proj.weight.view(self.d_model, H, Nh, 64)
        return torch.einsum("ohmr,hmn->ohnr", W, self.W_mix).reshape(self.d_model, H * Nh * 64)

    def forward_core(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """forward() without Omega: (out, biv [B, T, H, Nh, 28] scaled generators, dt [B, T, H])."""
        B, T, _ = x.shape
        H, Nh = self.num_heads, self.num_neurons_per_head
        residual = x
        x_conv = causal_conv_input(self.ln_1, self.conv1d, x)      # ln_1 -> causal conv -> SiLU, fused
        S = ops.linear(x_conv, self.in_proj.weight, self.in_proj.bias).view(B, T, H, Nh, 8, 8)
        biv, gamma, dt = generator_inputs(x_conv, self.biv_proj, self.gamma_proj, self.time_head.proj,
                                          self.omega_scale, self.time_head.dt_base)       # dt [B, T, H]
        biv, gamma = biv.view(B, T, H, Nh, 28), gamma.view(B, T, H, Nh)
        # lines 137-173 fused: per-head dt, heads read in place, X [B, T, H, Nh, 8, 8]
        X = ops.fused_rotor_scan_heads(biv, dt, gamma, S)
        X = ops.state_spike(X, self.spike_threshold, self.spike_beta)
        h = residual + ops.linear(X.view(B, T, self.total_neurons * 64), self.mixed_out_weight(), self.out_proj.bias)
        out = h + self.gglu(self.ln_2(h))
        return out, biv, dt

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """x [B, T, d_model] -> (out [B, T, d_model], Omega [B, T, H, Nh, 8, 8], dt [B, T, H])."""
        out, biv, dt = self.forward_core(x)
        Omega = skew_from_generators(biv, 8, self.triu_u, self.triu_v) * (0.5 * dt[..., None, None, None])
        return out, Omega, dt


class MultiHeadCliffordLM(nn.Module):
    """Embedding, MultiHeadCliffordCL6Block stack, final LayerNorm and geodesic head, with the
    reference's action / smoothness / time regularisers and per-head dt diagnostics
    (python/clifford_multihead.py:197-304)."""

    def __init__(self, vocab_size: int, d_model: int = 48, num_layers: int = 2, num_heads: int = 3,
                 num_neurons_per_head: int = 2, dt_base: float = 0.05, kernel_size: int = 4,
                 spike_threshold: float = 0.1, lambda_kin: float = 0.01, lambda_smooth: float = 0.005,
                 lambda_time: float = 0.01):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.num_neurons_per_head = num_neurons_per_head
        self.dt_base = dt_base
        self.lambda_kin = lambda_kin
        self.lambda_smooth = lambda_smooth
        self.lambda_time = lambda_time
        self.tok_emb = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([
            MultiHeadCliffordCL6Block(d_model=d_model, num_heads=num_heads,
                                      num_neurons_per_head=num_neurons_per_head, kernel_size=kernel_size,
                                      dt_base=dt_base, spike_threshold=spike_threshold)
            for _ in range(num_layers)])
        self.ln_f = LayerNorm(d_model)
        self.head = RiemannianGeodesicHead(vocab_size=vocab_size, d_model=d_model)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor], Dict[str, float]]:
        B, T = idx.shape
        x = self.tok_emb(idx)
        e_kin = e_smooth = t_smooth = 0.0
        dts = []
        for block in self.blocks:
            x, biv, dt = block.forward_core(x)
            dts.append(dt)
            kin, smooth = generator_action(biv, dt, 8)
            e_kin = e_kin + kin
            e_smooth = e_smooth + smooth
            if T > 1:
                t_smooth = t_smooth + (((dt[:, 1:] - dt[:, :-1]) / self.dt_base) ** 2).mean()
            else:
                t_smooth = t_smooth + torch.tensor(0.0, device=idx.device)
        logits = self.head(self.ln_f(x))
        stacked = torch.stack(dts)  # [L, B, T, H]
        named = {}
        for h in range(self.num_heads):
            d = stacked[..., h]
            named[f"head_{h}_mean_dt"] = d.mean()
            named[f"head_{h}_min_dt"] = d.min()
            named[f"head_{h}_max_dt"] = d.max()
        loss = None
        if targets is not None:
            ce = F.cross_entropy(logits.view(-1, self.vocab_size), targets.view(-1))
            action = self.lambda_kin * e_kin + self.lambda_smooth * e_smooth
            time_pen = self.lambda_time * t_smooth
            loss = ce + action + time_pen
            named.update(ce_loss=ce, action_loss=action, time_loss=time_pen)
        diagnostics: Dict[str, float] = read_diagnostics(named)
        return logits, loss, diagnostics
