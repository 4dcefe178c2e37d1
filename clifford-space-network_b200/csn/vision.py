"""Spatial rotor blocks, drop-in for CliffordSpatialRotorBlockCl4 / CliffordSpatialRotorBlockCl8
of csn_toolkit/csn/vision.py:56-167.

Same parameters and buffers (state_dict-compatible: in_proj, biv_proj, metric_proj, gamma_log,
lambda_sw, out_proj, norm, triu_u, triu_v) and the same forward: 1x1 / 3x3 convolutions give
the per-pixel step size, injection and generators; Omega = (skew(gens) + tanh(lambda) J_sw)
* ds / 2 clamped to [-3, 3] and the decay sigmoid(-softplus(gamma) ds), both in one CUDA
kernel from the convolutions' NCHW outputs (csn_b200.ops.spatial_generators; the skew uses the
row-major triu order of the triu_u / triu_v buffers); M = decay Q with the toolkit Cayley
rotor; then the 2D bidirectional one-sided scan, here csn_b200.spatial.spatial_scan_2d --
four scans on views of one buffer with the reverse-time mode instead of the reference's
permute / contiguous copies and flips.  Rotors are exact whatever ``use_schulz`` says
(the toolkit Cayley of this package).  The detector parts of that file (stem, FPN, heads,
EMA) are callers of these blocks and are not part of this package.
"""
import torch
import torch.nn as nn

from csn.rotors import cayley_rotor_4x4, cayley_rotor_16x16
from csn_b200 import ops
from csn_b200.spatial import spatial_scan_2d


class _SpatialRotorBlock(nn.Module):
    D = 4
    K = 6

    def __init__(self, in_channels: int, num_neurons: int, use_schulz: bool = True):
        super().__init__()
        D, K = self.D, self.K
        self.in_channels = in_channels
        self.num_neurons = num_neurons
        self.use_schulz = use_schulz
        self.in_proj = nn.Conv2d(in_channels, num_neurons * D * D, kernel_size=1, bias=False)
        self.biv_proj = nn.Conv2d(in_channels, num_neurons * K, kernel_size=1, bias=False)
        self.metric_proj = nn.Conv2d(in_channels, num_neurons, kernel_size=3, padding=1, bias=False)
        self.gamma_log = nn.Parameter(torch.zeros(num_neurons))
        self.lambda_sw = nn.Parameter(torch.tensor(0.1))
        self.out_proj = nn.Conv2d(num_neurons * D * D, in_channels, kernel_size=1, bias=False)
        self.norm = nn.BatchNorm2d(in_channels)
        self.act = nn.SiLU(inplace=True)
        iu = torch.triu_indices(D, D, offset=1)
        self.register_buffer("triu_u", iu[0])
        self.register_buffer("triu_v", iu[1])

    def _cayley(self, Omega):
        raise NotImplementedError

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, _, H, W = x.shape
        N, D = self.num_neurons, self.D
        # softplus step size, triu skew scatter, tanh-gated antisymmetric injection, scale,
        # clamp, decay and the pixel-major layout: one CUDA kernel each way
        Omega, C_inj, decay = ops.spatial_generators(self.in_proj(x), self.biv_proj(x), self.metric_proj(x),
                                                     self.lambda_sw, self.gamma_log, D)
        Q = self._cayley(Omega)
        psi = spatial_scan_2d(decay[..., None, None] * Q, C_inj, H, W, two_sided=False)
        out = psi.reshape(B, H, W, N * D * D).permute(0, 3, 1, 2)
        return self.act(self.norm(x + self.out_proj(out)))


class CliffordSpatialRotorBlockCl4(_SpatialRotorBlock):
    """2D bidirectional spatial scan with Spin(4) rotors (4 x 4, 6 generators)."""
    D, K = 4, 6

    def __init__(self, in_channels: int, num_neurons: int = 2, use_schulz: bool = True):
        super().__init__(in_channels, num_neurons, use_schulz)

    def _cayley(self, Omega):
        return cayley_rotor_4x4(Omega, use_schulz=self.use_schulz)


class CliffordSpatialRotorBlockCl8(_SpatialRotorBlock):
    """2D bidirectional spatial scan with Spin(8) rotors in the 16 x 16 representation
    (120 generators)."""
    D, K = 16, 120

    def __init__(self, in_channels: int, num_neurons: int = 1, use_schulz: bool = True):
        super().__init__(in_channels, num_neurons, use_schulz)

    def _cayley(self, Omega):
        return cayley_rotor_16x16(Omega, use_schulz=self.use_schulz)
