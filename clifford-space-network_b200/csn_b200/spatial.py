"""2D bidirectional spatial scan: the scan section of the reference's spatial rotor blocks
(csn_toolkit/csn/vision.py:97-107 for Cl(4), :154-164 for Cl(8)).

Pixels (b, h, w) of an H x W map carry N channels of D x D matrices, laid out
[B, H*W, N, D, D] (row-major over h, w).  The reference averages a left-to-right and a
right-to-left one-sided scan along every row, then does the same along every column of
that result:

    psi_h = (scan(M_h, C_h) + flip(scan(flip(M_h), flip(C_h)))) / 2        rows    [B*H, W, N]
    psi_v = (scan(M_v, C_v) + flip(scan(flip(M_v), flip(C_v)))) / 2        columns [B*W, H, N]

and builds M_v, C_v = psi_h and the output with permute + contiguous copies and the
reversed scans with flips.  Here each of the four scans runs on a VIEW of one
[B, H*W, N, D, D] buffer: a row scan is the layout [B*H, W, N] (time = w), a column scan is
the layout [B, H, W*N] (time = h, the column index folded into the channel axis), and a
right-to-left or bottom-to-top scan is the plain scan's reverse-time mode.  No tensor is
permuted or flipped.
"""
from __future__ import annotations

from . import ops


def bidirectional_scan(M, C, two_sided: bool = False):
    """(forward scan + reverse-time scan) / 2 along the time axis of [B, T, N, D, D]."""
    fwd = ops.rotor_scan(M, C, two_sided=two_sided)
    bwd = ops.rotor_scan(M, C, two_sided=two_sided, reverse=True)
    return 0.5 * (fwd + bwd)


def spatial_scan_2d(M, C, H: int, W: int, two_sided: bool = False):
    """Row-then-column bidirectional scan of M, C [B, H*W, N, D, D]; returns [B, H*W, N, D, D]
    in the same pixel order (the reference's `out` before its channel reshape)."""
    if M.dim() != 5 or C.shape != M.shape:
        raise ValueError(f"spatial_scan_2d expects M, C of shape [B, H*W, N, D, D], got "
                         f"{tuple(M.shape)}, {tuple(C.shape)}")
    B, L, N, D, _ = M.shape
    if L != H * W:
        raise ValueError(f"spatial_scan_2d: {L} pixels is not H * W = {H} * {W}")
    M = M.contiguous()
    psi_h = bidirectional_scan(M.reshape(B * H, W, N, D, D), C.contiguous().reshape(B * H, W, N, D, D),
                               two_sided)
    psi_v = bidirectional_scan(M.reshape(B, H, W * N, D, D), psi_h.reshape(B, H, W * N, D, D), two_sided)
    return psi_v.reshape(B, L, N, D, D)
