"""Cl(6,0) ~ M_8(R) block with adaptive dt, drop-in for python/clifford_cl6.py.

``CliffordCL6Block.forward`` keeps the reference's parameters, inputs and outputs
(python/clifford_cl6.py:71-186) with the block's producer/consumer chain fused:
  * lines 150-171 -- skew generator, Omega, exact Cayley rotor, decay, M/C construction and the
    scan -- are ONE fused CUDA op (csn_b200.ops.fused_rotor_scan): M and C are never materialised;
  * the event spike of lines 174-176 is one CUDA kernel each way (ops.state_spike);
  * the inter-neuron mixing of line 179 is linear, so it is folded into out_proj's weight
    (W_out (W_mix (x) I_64), a [d_model, N*64] matrix built per call): X_mixed is never formed;
  * ln_1 -> causal depthwise conv -> SiLU (lines 140-142) is one CUDA kernel each way
    (csn_b200.modules.causal_conv_input), and ln_2 runs the CUDA LayerNorm kernels;
  * the generator, decay and time projections (lines 144-155) are one GEMM whose output
    the CUDA projection epilogue turns into the scan's inputs (omega_scale, softplus, dt_base);
    bias gradients are deterministic CUDA column sums (csn_b200.ops.linear).
Omega is still returned by forward(); CliffordCL6ForCausalLM takes its action regulariser from
the generator coefficients instead (sum Omega^2 = 2 sum (0.5 dt biv)^2), so it never forms Omega.
"""
import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from csn_b200 import graphs, ops
from csn_b200.modules import LayerNorm, causal_conv_input, generator_inputs
from python.clifford_model import GeometricGatedLinearUnit, RiemannianGeodesicHead
from python.clifford_scan import parallel_rotor_scan, surrogate_spike  # noqa: F401 (re-export)


class AdaptiveTimeHead(nn.Module):
    """dt_t = softplus(W x_t + b) * dt_base, initialised at dt_base (python/clifford_cl6.py:27-54)."""

    def __init__(self, d_model: int, dt_base: float = 0.05):
        super().__init__()
        self.dt_base = dt_base
        self.proj = nn.Linear(d_model, 1)
        nn.init.zeros_(self.proj.weight)
        nn.init.constant_(self.proj.bias, math.log(math.e - 1.0))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = F.softplus(self.proj(x)) * self.dt_base
        return dt.unsqueeze(-1).unsqueeze(-1)  # [B, T, 1, 1, 1]


def cayley_rotor_8x8(Omega: torch.Tensor) -> torch.Tensor:
    """Exact Q = (I - Omega)^{-1} (I + Omega) for skew 8 x 8 Omega (python/clifford_cl6.py:57-68)."""
    return ops.cayley(Omega)


def generator_action(biv: torch.Tensor, dt: torch.Tensor, D: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(Omega^2).mean() and ((Omega[:, 1:] - Omega[:, :-1])^2).mean() of the LMs' least-action
    regulariser (python/clifford_cl6.py:257-262, clifford_cl8.py, clifford_multihead.py) from the
    K generator coefficients, without forming Omega = skew(biv) * 0.5 dt: each coefficient
    w = 0.5 dt biv sits at (u, v) and, negated, at (v, u) of a D x D matrix with a zero diagonal,
    so a mean over Omega's D^2 entries is (2 K / D^2) times the mean over w.  One CUDA kernel
    each way (ops.generator_action).  biv [B, T, ..., K]; dt [B, T] or [B, T, H] (per head).
    The smoothness term is 0 for T = 1."""
    return ops.generator_action(biv, dt, D)


def read_diagnostics(named: Dict[str, torch.Tensor]) -> Dict[str, float]:
    """{name: float} of scalar tensors with one device -> host read for all of them.  Inside
    csn_b200.graphs.deferred_diagnostics() (a captured training step) the scalars stay on the
    device, unread: {name: 0-d tensor}."""
    if graphs.diagnostics_deferred():
        return {k: v.detach().float().reshape(()) if torch.is_tensor(v) else float(v) for k, v in named.items()}
    vals = torch.stack([torch.as_tensor(v).detach().float().reshape(()).to(next(iter(named.values())).device)
                        for v in named.values()]).tolist()
    return dict(zip(named.keys(), vals))


def skew_from_generators(biv: torch.Tensor, D: int, triu_u: torch.Tensor, triu_v: torch.Tensor):
    skew = torch.zeros(*biv.shape[:-1], D, D, device=biv.device, dtype=biv.dtype)
    skew[..., triu_u, triu_v] = biv
    skew[..., triu_v, triu_u] = -biv
    return skew


class CliffordCL6Block(nn.Module):
    def __init__(self, d_model: int, num_neurons: int = 6, kernel_size: int = 4, dt_base: float = 0.05,
                 spike_threshold: float = 0.1, spike_beta: float = 10.0):
        super().__init__()
        self.d_model = d_model
        self.num_neurons = num_neurons
        self.dt_base = dt_base
        self.spike_threshold = spike_threshold
        self.spike_beta = spike_beta
        self.ln_1 = LayerNorm(d_model)
        self.conv1d = nn.Conv1d(d_model, d_model, kernel_size=kernel_size, padding=kernel_size - 1,
                                groups=d_model)
        self.time_head = AdaptiveTimeHead(d_model, dt_base=dt_base)
        self.in_proj = nn.Linear(d_model, num_neurons * 64)
        self.gamma_proj = nn.Linear(d_model, num_neurons)
        self.biv_proj = nn.Linear(d_model, num_neurons * 28)
        self.omega_scale = nn.Parameter(torch.ones(num_neurons, 1) * 10.0)
        self.W_mix = nn.Parameter(torch.randn(num_neurons, num_neurons) / math.sqrt(num_neurons))
        self.out_proj = nn.Linear(num_neurons * 64, d_model)
        self.ln_2 = LayerNorm(d_model)
        self.gglu = GeometricGatedLinearUnit(d_model, d_ffn=2 * d_model)
        self.register_buffer("triu_u", torch.triu_indices(8, 8, offset=1)[0], persistent=False)
        self.register_buffer("triu_v", torch.triu_indices(8, 8, offset=1)[1], persistent=False)

    def mixed_out_weight(self) -> torch.Tensor:
        """out_proj's weight with the mixing folded in: out_proj(mix(X)) = X W^T + b with
        W[o, j*64 + rc] = sum_i W_out[o, i*64 + rc] W_mix[i, j] (python/clifford_cl6.py:179-184)."""
        N = self.num_neurons
        W = self.out_proj.weight.view(self.d_model, N, 64)
        return torch.einsum("oir,ij->ojr", W, self.W_mix).reshape(self.d_model, N * 64)

    def forward_core(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """forward() without Omega: (out [B, T, d_model], biv [B, T, N, 28] (the scaled generator
        coefficients, Omega = skew(biv) * 0.5 dt), dt [B, T])."""
        B, T, _ = x.shape
        N = self.num_neurons
        residual = x
        x_conv = causal_conv_input(self.ln_1, self.conv1d, x)      # ln_1 -> causal conv -> SiLU, fused
        S = ops.linear(x_conv, self.in_proj.weight, self.in_proj.bias).view(B, T, N, 8, 8)
        # lines 144-155: generator, decay and time projections as one GEMM + CUDA epilogue
        biv, gamma, dt = generator_inputs(x_conv, self.biv_proj, self.gamma_proj, self.time_head.proj,
                                          self.omega_scale, self.time_head.dt_base)
        biv, dt = biv.view(B, T, N, 28), dt.view(B, T)
        X_all = ops.fused_rotor_scan(biv, dt, gamma, S)               # lines 150-171 fused
        X_spiked = ops.state_spike(X_all, self.spike_threshold, self.spike_beta)
        h = residual + ops.linear(X_spiked.view(B, T, N * 64), self.mixed_out_weight(), self.out_proj.bias)
        out = h + self.gglu(self.ln_2(h))
        return out, biv, dt

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        out, biv, dt = self.forward_core(x)
        Omega = skew_from_generators(biv, 8, self.triu_u, self.triu_v) * (0.5 * dt)[..., None, None, None]
        return out, Omega, dt

    # ------------------------------------------------ O(1)-state generation (extension)
    def init_state(self, batch_size: int, device=None):
        """Zero decoding state: (causal-conv window [B, d_model, k-1], rotor state [B, N, 8, 8]).

        The reference has no step API (its generation re-runs the prefix,
        tests/profile_performance.py:58-66); step() advances this state one token at O(1)
        cost and produces the same outputs as forward() on the whole prefix."""
        device = device if device is not None else self.in_proj.weight.device
        k = self.conv1d.kernel_size[0]
        return (torch.zeros(batch_size, self.d_model, k - 1, device=device),
                torch.zeros(batch_size, self.num_neurons, 8, 8, device=device))

    @torch.no_grad()
    def step(self, x_t: torch.Tensor, state):
        """One token: x_t [B, d_model] -> (out [B, d_model], new state).  The rotor state is
        updated in place by the CUDA step kernel (csn_rotor_step)."""
        conv_buf, X = state
        B = x_t.shape[0]
        N = self.num_neurons
        window = torch.cat([conv_buf, self.ln_1(x_t).unsqueeze(-1)], dim=-1)       # oldest first
        xc = F.silu((window * self.conv1d.weight[:, 0, :]).sum(-1) + self.conv1d.bias)
        dt = F.softplus(self.time_head.proj(xc)) * self.time_head.dt_base          # [B, 1]
        S = self.in_proj(xc).view(B, N, 8, 8)
        gamma = F.softplus(self.gamma_proj(xc))
        biv = self.biv_proj(xc).view(B, N, 28) * self.omega_scale
        ops.rotor_step(biv, dt.view(B), gamma, S, X)
        energy = torch.norm(X, dim=(-1, -2), keepdim=True)
        X_spiked = X * surrogate_spike(energy, threshold=self.spike_threshold, beta=self.spike_beta)
        feat = torch.einsum("ij,bjrc->birc", self.W_mix, X_spiked).reshape(B, N * 64)
        h = x_t + self.out_proj(feat)
        out = h + self.gglu(self.ln_2(h))
        return out, (window[:, :, 1:].contiguous(), X)


class CliffordCL6ForCausalLM(nn.Module):
    def __init__(self, vocab_size: int, d_model: int = 48, num_layers: int = 2, num_neurons: int = 6,
                 dt_base: float = 0.05, kernel_size: int = 4, spike_threshold: float = 0.1,
                 lambda_kin: float = 0.01, lambda_smooth: float = 0.005, lambda_time: float = 0.01):
        super().__init__()
        self.vocab_size = vocab_size
        self.d_model = d_model
        self.num_layers = num_layers
        self.dt_base = dt_base
        self.lambda_kin = lambda_kin
        self.lambda_smooth = lambda_smooth
        self.lambda_time = lambda_time
        self.tok_emb = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([
            CliffordCL6Block(d_model=d_model, num_neurons=num_neurons, kernel_size=kernel_size,
                             dt_base=dt_base, spike_threshold=spike_threshold)
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
            kin, smooth = generator_action(biv, dt_t, 8)
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
