"""PyTorch front end of the CUDA rotor-scan library (autograd + shape handling).

Every op runs on the current CUDA stream through the C ABI (``_lib``).  Inputs
must be CUDA tensors; there is no CPU path and no silent fallback.  Computation
is float32: float64/float16/bfloat16 inputs are computed in float32 and the
result is returned in the input dtype.

Ops (reference functions they replace, paths relative to the reference root):

* :func:`rotor_scan`        -- python/clifford_scan.py:41 parallel_rotor_scan (two-sided),
                               csn_toolkit/csn/scan.py:16-72 CliffordScanFunction (one-sided)
* :func:`fused_rotor_scan`  -- python/clifford_cl6.py:150-171 / python/clifford_cl8.py:160-179
                               (Cayley rotor + decay + scan in one pass)
* :func:`fused_rotor_scan_heads` -- python/clifford_multihead.py:137-170 (per-head dt, heads
                               read in place instead of folded into the batch)
* :func:`cayley`            -- python/clifford_cl6.py:57, python/clifford_cl8.py:29,65
* :func:`cell_step`         -- python/clifford_layer.py:50-115 CliffordTENNCell.forward
* :func:`ga3_rotor_scan`    -- Cl(3,0) blade-basis form of the two-sided scan
                               (layout include/clifford_configs.cuh:38-51)
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

__all__ = ["rotor_scan", "fused_rotor_scan", "fused_rotor_scan_heads", "cayley", "cell_step", "ga3_rotor_scan",
           "rotor_step", "RotorStepGraph", "state_spike", "layer_norm", "ln_conv_silu",
           "generator_action", "linear", "projection_epilogue", "silu_gate", "column_sum", "BASIS"]

BASIS = {"triu": 0, "ga": 1}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("csn_b200 ops need CUDA tensors: the library has no CPU path")


def _f32(t):
    """Contiguous float32 copy (or the tensor itself when it already is one), 16-byte aligned."""
    if t is None:
        return None
    t = t.detach()
    if t.dtype != torch.float32:
        t = t.float()
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _workspace(nbytes, device):
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


# --------------------------------------------------------------------- plain scan
SCAN_TWO_SIDED, SCAN_REVERSE = 1, 2  # csn_scan_* flags


def _scan_flags(two_sided, reverse=False):
    return (SCAN_TWO_SIDED if two_sided else 0) | (SCAN_REVERSE if reverse else 0)


def _scan_fwd(M, C, h0, two_sided, reverse=False):
    B, T, N, D, _ = M.shape
    X = torch.empty_like(C)
    ws_bytes = _lib.load().csn_scan_workspace_bytes(B, T, N, D)
    ws = _workspace(ws_bytes, M.device)
    _lib.call("csn_scan_fwd", _ptr(M), _ptr(C), _ptr(h0), _ptr(X), B, T, N, D,
              _scan_flags(two_sided, reverse), _ptr(ws), ws_bytes, _stream(M.device))
    return X


def _scan_bwd(M, X, dX, h0, two_sided, need_dh0, reverse=False):
    B, T, N, D, _ = M.shape
    dM = torch.empty_like(M)
    dC = torch.empty_like(M)
    dh0 = torch.empty_like(h0) if (need_dh0 and h0 is not None) else None
    ws_bytes = _lib.load().csn_scan_workspace_bytes(B, T, N, D)
    ws = _workspace(ws_bytes, M.device)
    _lib.call("csn_scan_bwd", _ptr(M), _ptr(X), _ptr(dX), _ptr(h0), _ptr(dM), _ptr(dC), _ptr(dh0),
              B, T, N, D, _scan_flags(two_sided, reverse), _ptr(ws), ws_bytes, _stream(M.device))
    return dM, dC, dh0


class ScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, M, C, h0, two_sided, reverse=False):
        _require_cuda(M, C, h0)
        Mf, Cf, hf = _f32(M), _f32(C), _f32(h0)
        X = _scan_fwd(Mf, Cf, hf, two_sided, reverse)
        ctx.save_for_backward(Mf, X, hf)
        ctx.two_sided, ctx.reverse = two_sided, reverse
        ctx.dtypes = (M.dtype, C.dtype, None if h0 is None else h0.dtype)
        return X.to(C.dtype)

    @staticmethod
    def backward(ctx, dX):
        Mf, X, hf = ctx.saved_tensors
        need_dh0 = len(ctx.needs_input_grad) > 2 and ctx.needs_input_grad[2]
        dM, dC, dh0 = _scan_bwd(Mf, X, _f32(dX), hf, ctx.two_sided, need_dh0, ctx.reverse)
        dM = dM.to(ctx.dtypes[0])
        dC = dC.to(ctx.dtypes[1])
        if dh0 is not None:
            dh0 = dh0.to(ctx.dtypes[2])
        return dM, dC, dh0, None, None


def rotor_scan(M, C, two_sided: bool = True, h0=None, reverse: bool = False):
    """Inclusive scan X_t = M_t X_{t-1} M_t^T + C_t (two-sided) or M_t X_{t-1} + C_t.

    M, C: [B, T, N, D, D] with D in {4, 8, 16}; h0: optional [B, N, D, D] (X_{-1}).
    reverse=True scans from t = T-1 down to 0 (X_t = M_t X_{t+1} (M_t^T) + C_t, h0 = X_T):
    the flipped scan, without flipping any tensor.
    """
    if M.dim() != 5 or C.shape != M.shape or M.shape[-1] != M.shape[-2]:
        raise ValueError(f"rotor_scan expects M, C of shape [B, T, N, D, D], got {tuple(M.shape)}, "
                         f"{tuple(C.shape)}")
    return ScanFunction.apply(M, C, h0, bool(two_sided), bool(reverse))


# ---------------------------------------------------------------- fused rotor scan
def _rotor_dims(s):
    """(B, T, H, Nh, D) of S: [B, T, N, D, D] is one dt per step (H = 0), [B, T, H, Nh, D, D]
    one dt per head."""
    if s.dim() == 6:
        B, T, H, Nh, D, _ = s.shape
        return B, T, H, Nh, D
    B, T, N, D, _ = s.shape
    return B, T, 0, N, D


def _rotor_ws_bytes(s):
    B, T, H, Nh, D = _rotor_dims(s)
    return _lib.load().csn_rotor_scan_workspace_bytes(B, T, max(H, 1) * Nh, D)


def _rotor_fwd(g, d, ga, s, hf, basis, two_sided, Mc=None, ws=None):
    """Raw fused forward on float32 contiguous CUDA tensors -> X.  S is [B, T, N, D, D] (dt
    [B, T]) or the multi-head layout [B, T, H, Nh, D, D] (dt [B, T, H]).  With Mc (the shape
    of S, D = 16 only) every step's rotor M_t is stored there for the backward.  `ws`: a
    workspace of csn_rotor_scan_workspace_bytes to use (and keep for a reusing backward)."""
    B, T, H, Nh, D = _rotor_dims(s)
    X = torch.empty_like(s)
    ws_bytes = _rotor_ws_bytes(s)
    if ws is None:
        ws = _workspace(ws_bytes, s.device)
    if H:
        _lib.call("csn_rotor_scan_heads_fwd", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
                  _ptr(Mc), B, T, H, Nh, D, basis, int(two_sided), _ptr(ws), ws_bytes, _stream(s.device))
        return X
    if Mc is not None:
        _lib.call("csn_rotor_scan_fwd_cached", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
                  _ptr(Mc), B, T, Nh, D, basis, int(two_sided), _ptr(ws), ws_bytes, _stream(s.device))
        return X
    _lib.call("csn_rotor_scan_fwd", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
              B, T, Nh, D, basis, int(two_sided), _ptr(ws), ws_bytes, _stream(s.device))
    return X


def _rotor_bwd(g, d, ga, s, hf, X, dXf, basis, two_sided, need_dh0, Mc=None, fwd_ws=None):
    """Raw fused adjoint -> (dgens, ddt, dgamma or None, dS, dh0 or None); Mc = the rotors
    stored by the forward (D = 16) or None to rebuild them; fwd_ws = the forward's workspace,
    whose chunk rotor products the backward then reuses."""
    B, T, H, Nh, D = _rotor_dims(s)
    dg = torch.empty_like(g)
    ddt = torch.empty_like(d)
    dga = torch.empty_like(ga) if ga is not None else None
    dS = torch.empty_like(s)
    dh0 = torch.empty_like(hf) if (hf is not None and need_dh0) else None
    ws_bytes = _rotor_ws_bytes(s)
    if H or (Mc is not None and fwd_ws is not None):
        # the multi-head entry point (H = 1 is the [B, T, N] layout) takes the rotor cache and
        # the forward's workspace together
        ws = fwd_ws if fwd_ws is not None else _workspace(ws_bytes, s.device)
        _lib.call("csn_rotor_scan_heads_bwd", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
                  _ptr(dXf), _ptr(Mc), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS), _ptr(dh0), B, T, max(H, 1), Nh,
                  D, basis, int(two_sided), int(fwd_ws is not None), _ptr(ws), ws_bytes, _stream(s.device))
        return dg, ddt, dga, dS, dh0
    if fwd_ws is not None and Mc is None:
        _lib.call("csn_rotor_scan_bwd_reuse", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
                  _ptr(dXf), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS), _ptr(dh0), B, T, Nh, D,
                  basis, int(two_sided), _ptr(fwd_ws), ws_bytes, _stream(s.device))
        return dg, ddt, dga, dS, dh0
    ws = _workspace(ws_bytes, s.device)
    if Mc is not None:
        _lib.call("csn_rotor_scan_bwd_cached", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
                  _ptr(dXf), _ptr(Mc), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS), _ptr(dh0), B, T, Nh, D,
                  basis, int(two_sided), _ptr(ws), ws_bytes, _stream(s.device))
        return dg, ddt, dga, dS, dh0
    _lib.call("csn_rotor_scan_bwd", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(hf), _ptr(X),
              _ptr(dXf), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS), _ptr(dh0), B, T, Nh, D,
              basis, int(two_sided), _ptr(ws), ws_bytes, _stream(s.device))
    return dg, ddt, dga, dS, dh0


class RotorScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gens, dt, gamma, S, h0, basis, two_sided):
        _require_cuda(gens, dt, gamma, S, h0)
        g, d, ga, s, hf = _f32(gens), _f32(dt), _f32(gamma), _f32(S), _f32(h0)
        # D = 16: keep the step rotors for the backward (1 KB per element, like S) instead
        # of rebuilding them there
        Mc = torch.empty_like(s) if s.shape[-1] == 16 else None
        # keep the forward's workspace, whose chunk rotor products the backward reuses
        ws = _workspace(_rotor_ws_bytes(s), s.device)
        X = _rotor_fwd(g, d, ga, s, hf, basis, two_sided, Mc, ws)
        ctx.save_for_backward(g, d, ga, s, hf, X, Mc)
        ctx.fwd_ws = ws
        ctx.basis, ctx.two_sided = basis, two_sided
        ctx.dtypes = tuple(None if t is None else t.dtype for t in (gens, dt, gamma, S, h0))
        return X.to(S.dtype)

    @staticmethod
    def backward(ctx, dX):
        g, d, ga, s, hf, X, Mc = ctx.saved_tensors
        outs = _rotor_bwd(g, d, ga, s, hf, X, _f32(dX), ctx.basis, ctx.two_sided, ctx.needs_input_grad[4], Mc,
                          ctx.fwd_ws)
        ctx.fwd_ws = None
        outs = [None if o is None else o.to(dt_) for o, dt_ in zip(outs, ctx.dtypes)]
        return outs[0], outs[1], outs[2], outs[3], outs[4], None, None


def fused_rotor_scan(gens, dt, gamma, S, basis: str = "triu", two_sided: bool = True, h0=None):
    """Cayley rotor + decay + scan in one pass (M and C are never materialised).

    gens [B, T, N, K], dt [B, T] (or [B, T, 1, 1, 1]), gamma [B, T, N] (post-softplus;
    None = undamped, M = Q and C = S), S [B, T, N, D, D].  ``basis`` "triu" is the
    reference generator layout (K = D(D-1)/2); "ga" takes GA bivector blades (Cl(3,0)
    for D = 4, Cl(8,0) for D = 16).
    """
    if S.dim() != 5:
        raise ValueError("S must be [B, T, N, D, D]")
    B, T, N, D, _ = S.shape
    dt = dt.reshape(B, T)
    if gamma is not None:
        gamma = gamma.reshape(B, T, N)
    if basis not in BASIS:
        raise ValueError(f"basis must be one of {sorted(BASIS)}")
    return RotorScanFunction.apply(gens, dt, gamma, S, h0, BASIS[basis], bool(two_sided))


def fused_rotor_scan_heads(gens, dt, gamma, S, basis: str = "triu", two_sided: bool = True, h0=None):
    """fused_rotor_scan on the multi-head layout, one dt per head (python/clifford_multihead.py:137-170).

    gens [B, T, H, Nh, K], dt [B, T, H] (or [B, T, H, 1, 1, 1]), gamma [B, T, H, Nh] (or
    [B, T, H, Nh, 1, 1]; None = undamped), S [B, T, H, Nh, D, D], h0 [B, H, Nh, D, D] ->
    X [B, T, H, Nh, D, D].  Neuron (h, i) uses dt[b, t, h]; the reference's fold of heads into
    the batch is read in place, so neither inputs nor X are transposed.
    """
    if S.dim() != 6:
        raise ValueError("S must be [B, T, H, Nh, D, D]")
    B, T, H, Nh, D, _ = S.shape
    if H < 1:
        raise ValueError("fused_rotor_scan_heads needs at least one head")
    dt = dt.reshape(B, T, H)
    if gamma is not None:
        gamma = gamma.reshape(B, T, H, Nh)
    if basis not in BASIS:
        raise ValueError(f"basis must be one of {sorted(BASIS)}")
    return RotorScanFunction.apply(gens, dt, gamma, S, h0, BASIS[basis], bool(two_sided))


# ------------------------------------------------------------------------ Cayley
def _cayley_fwd(O):
    D = O.shape[-1]
    Q = torch.empty_like(O)
    _lib.call("csn_cayley_fwd", _ptr(O), _ptr(Q), O.numel() // (D * D), D, _stream(O.device))
    return Q


def _cayley_bwd(Q, dQf):
    D = Q.shape[-1]
    dO = torch.empty_like(Q)
    _lib.call("csn_cayley_bwd", _ptr(Q), _ptr(dQf), _ptr(dO), Q.numel() // (D * D), D, _stream(Q.device))
    return dO


class CayleyFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Om):
        _require_cuda(Om)
        Q = _cayley_fwd(_f32(Om))
        ctx.save_for_backward(Q)
        ctx.dtype = Om.dtype
        return Q.to(Om.dtype)

    @staticmethod
    def backward(ctx, dQ):
        (Q,) = ctx.saved_tensors
        return _cayley_bwd(Q, _f32(dQ)).to(ctx.dtype)


def cayley(Omega):
    """Q = (I - Omega)^{-1} (I + Omega) for skew Omega[..., D, D], D in {4, 8, 16}."""
    return CayleyFunction.apply(Omega)


# ----------------------------------------------------------------- Clifford cell
def _cell_fwd(xf, pf, wr, wi, gb, dt):
    Bt, N, A = pf.shape
    if A != 16:
        raise ValueError("the Clifford cell works on 16-component (4 x 4) states")
    nxt = torch.empty_like(pf)
    _lib.call("csn_cell_fwd", _ptr(pf), _ptr(xf), _ptr(wr), _ptr(wi), _ptr(gb), float(dt),
              _ptr(nxt), Bt, N, xf.shape[1], _stream(pf.device))
    return nxt


def _cell_bwd(xf, pf, wr, wi, gb, dt, dnf):
    """-> (dx, dprev, dW_rec, dW_in, dgamma_bias)"""
    Bt, N, _ = pf.shape
    dprev, dx = torch.empty_like(pf), torch.empty_like(xf)
    dwr, dwi, dgb = torch.empty_like(wr), torch.empty_like(wi), torch.empty_like(gb)
    nbytes = _lib.load().csn_cell_workspace_bytes(Bt, N)
    ws = _workspace(nbytes, pf.device)
    _lib.call("csn_cell_bwd", _ptr(pf), _ptr(xf), _ptr(wr), _ptr(wi), _ptr(gb), float(dt),
              _ptr(dnf), _ptr(dprev), _ptr(dx), _ptr(dwr), _ptr(dwi), _ptr(dgb),
              Bt, N, xf.shape[1], _ptr(ws), nbytes, _stream(pf.device))
    return dx, dprev, dwr, dwi, dgb


class CellFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, prev, W_rec, W_in, gamma_bias, dt):
        _require_cuda(x, prev, W_rec, W_in, gamma_bias)
        xf, pf, wr, wi, gb = (_f32(t) for t in (x, prev, W_rec, W_in, gamma_bias))
        nxt = _cell_fwd(xf, pf, wr, wi, gb, dt)
        ctx.save_for_backward(xf, pf, wr, wi, gb)
        ctx.dt = float(dt)
        ctx.dtypes = (x.dtype, prev.dtype, W_rec.dtype, W_in.dtype, gamma_bias.dtype)
        return nxt.to(prev.dtype)

    @staticmethod
    def backward(ctx, dnext):
        xf, pf, wr, wi, gb = ctx.saved_tensors
        outs = _cell_bwd(xf, pf, wr, wi, gb, ctx.dt, _f32(dnext))
        outs = [o.to(d) for o, d in zip(outs, ctx.dtypes)]
        return outs[0], outs[1], outs[2], outs[3], outs[4], None


def cell_step(x, prev, W_rec, W_in, gamma_bias, dt: float = 0.02):
    """One CliffordTENNCell step: x [Bt, in_dim], prev [Bt, N, 16] -> next [Bt, N, 16]."""
    return CellFunction.apply(x, prev, W_rec, W_in, gamma_bias, dt)


# ----------------------------------------------------------- Cl(3,0) blade scan
def _ga3_fwd(g, d, xf, hf):
    B, T, N, _ = xf.shape
    h = torch.empty_like(xf)
    nbytes = _lib.load().csn_ga3_workspace_bytes(B, T, N)
    ws = _workspace(nbytes, xf.device)
    _lib.call("csn_ga3_scan_fwd", _ptr(g), _ptr(d), _ptr(xf), _ptr(hf), _ptr(h), B, T, N,
              _ptr(ws), nbytes, _stream(xf.device))
    return h


def _ga3_bwd(g, d, hf, h, dhf, need_dh0):
    """-> (dgens, ddt, dx, dh0 or None)"""
    B, T, N, _ = h.shape
    dg, ddt, dx = torch.empty_like(g), torch.empty_like(d), torch.empty_like(h)
    dh0 = torch.empty_like(hf) if (hf is not None and need_dh0) else None
    nbytes = _lib.load().csn_ga3_workspace_bytes(B, T, N)
    ws = _workspace(nbytes, h.device)
    _lib.call("csn_ga3_scan_bwd", _ptr(g), _ptr(d), _ptr(hf), _ptr(h), _ptr(dhf), _ptr(dg),
              _ptr(ddt), _ptr(dx), _ptr(dh0), B, T, N, _ptr(ws), nbytes, _stream(h.device))
    return dg, ddt, dx, dh0


class Ga3ScanFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gens, dt, x, h0):
        _require_cuda(gens, dt, x, h0)
        g, d, xf, hf = _f32(gens), _f32(dt), _f32(x), _f32(h0)
        h = _ga3_fwd(g, d, xf, hf)
        ctx.save_for_backward(g, d, hf, h)
        ctx.dtypes = tuple(None if t is None else t.dtype for t in (gens, dt, x, h0))
        return h.to(x.dtype)

    @staticmethod
    def backward(ctx, dh):
        g, d, hf, h = ctx.saved_tensors
        outs = _ga3_bwd(g, d, hf, h, _f32(dh), ctx.needs_input_grad[3])
        return tuple(None if o is None else o.to(t) for o, t in zip(outs, ctx.dtypes))


def ga3_rotor_scan(gens, dt, x, h0=None):
    """Cl(3,0) affine rotor scan h_t = R_t h_{t-1} R~_t + x_t in the blade basis.

    gens [B, T, N, 3] on (e12, e23, e31), dt [B, T], x [B, T, N, 8] on
    [1, e1, e2, e3, e12, e23, e31, e123], h0 optional [B, N, 8].
    """
    B, T, N, _ = x.shape
    return Ga3ScanFunction.apply(gens, dt.reshape(B, T), x, h0)


# ------------------------------------------------------------ O(1) generation step
def rotor_step(gens, dt, gamma, S, h, basis: str = "triu", two_sided: bool = True):
    """Advance the carried state one token, in place: h <- M h M^T + C.

    gens [B, N, K], dt [B], gamma [B, N] (None = undamped), S [B, N, D, D], h [B, N, D, D]
    (float32, contiguous, CUDA).  Inference only (no autograd).  Returns h.
    """
    _require_cuda(gens, dt, gamma, S, h)
    if h.dtype != torch.float32 or not h.is_contiguous() or h.data_ptr() % 16:
        raise ValueError("rotor_step updates h in place: h must be contiguous, aligned float32")
    B, N, D, _ = h.shape
    g, d, ga, s = _f32(gens), _f32(dt), _f32(gamma), _f32(S)
    _lib.call("csn_rotor_step", _ptr(g), _ptr(d), _ptr(ga), _ptr(s), _ptr(h), B, N, D,
              BASIS[basis], int(two_sided), _stream(h.device))
    return h


class RotorStepGraph:
    """A CUDA graph of `steps` consecutive rotor steps on static buffers.

    Fill ``gens[t], dt[t], gamma[t], S[t]`` (leading step axis) and call ``replay()``: the
    state ``h`` advances `steps` tokens with one graph launch, i.e. without a host round
    trip per token.  Capture happens once, at construction.

    ``chained`` (default): the steps are captured with csn_rotor_step_chained, so each step
    builds its rotor while the previous step finishes (valid because every step input is in
    place before replay()).  ``chained=False`` captures ordinary csn_rotor_step launches, each
    waiting for the previous step to complete, as a decode loop whose inputs are produced
    between steps must.
    """

    def __init__(self, B, N, D, steps=1, damped=True, basis="triu", two_sided=True, device="cuda",
                 chained=True):
        K = D * (D - 1) // 2 if basis == "triu" else (3 if D == 4 else 28)
        dev = torch.device(device)
        self.h = torch.zeros(B, N, D, D, device=dev)
        self.gens = torch.zeros(steps, B, N, K, device=dev)
        self.dt = torch.full((steps, B), 0.05, device=dev)
        self.gamma = torch.ones(steps, B, N, device=dev) if damped else None
        self.S = torch.zeros(steps, B, N, D, D, device=dev)
        self.steps = steps
        args = (BASIS[basis], int(two_sided))
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):  # warm-up launch outside the graph (lazy module load)
            rotor_step(self.gens[0], self.dt[0], None if self.gamma is None else self.gamma[0],
                       self.S[0], self.h, basis, two_sided)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.h.zero_()
        self.graph = torch.cuda.CUDAGraph()
        # the step inputs are filled before replay() and no kernel in the graph writes them,
        # so the steps may chain: each builds its rotor while the previous one finishes
        entry = "csn_rotor_step_chained" if chained else "csn_rotor_step"
        with torch.cuda.graph(self.graph, stream=s):
            for t in range(steps):
                _lib.call(entry, _ptr(self.gens[t]), _ptr(self.dt[t]),
                          _ptr(None if self.gamma is None else self.gamma[t]), _ptr(self.S[t]),
                          _ptr(self.h), B, N, D, *args, ctypes.c_void_p(s.cuda_stream))

    def replay(self):
        self.graph.replay()
        return self.h


# ------------------------------------------------------------ block kernels
class StateSpikeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, threshold, beta):
        _require_cuda(X)
        x = _f32(X)
        D = x.shape[-1]
        Xs = torch.empty_like(x)
        _lib.call("csn_spike_fwd", _ptr(x), _ptr(Xs), x.numel() // (D * D), D, float(threshold),
                  _stream(x.device))
        ctx.save_for_backward(x)
        ctx.threshold, ctx.beta, ctx.dtype = float(threshold), float(beta), X.dtype
        return Xs.to(X.dtype)

    @staticmethod
    def backward(ctx, dXs):
        (x,) = ctx.saved_tensors
        g = _f32(dXs)
        D = x.shape[-1]
        dX = torch.empty_like(x)
        _lib.call("csn_spike_bwd", _ptr(x), _ptr(g), _ptr(dX), x.numel() // (D * D), D, ctx.threshold, ctx.beta,
                  _stream(x.device))
        return dX.to(ctx.dtype), None, None


def state_spike(X, threshold: float = 0.5, beta: float = 10.0):
    """X * surrogate_spike(||X||_F, threshold, beta) over the last two (D x D) axes, as one CUDA
    kernel each way (python/clifford_scan.py:90-116 applied as in python/clifford_cl6.py:174-176).
    D in {4, 8, 16}."""
    if X.dim() < 2 or X.shape[-1] != X.shape[-2] or X.shape[-1] not in (4, 8, 16):
        raise ValueError(f"state_spike expects [..., D, D] with D in (4, 8, 16), got {tuple(X.shape)}")
    return StateSpikeFunction.apply(X, threshold, beta)


class LayerNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        _require_cuda(x, weight, bias)
        C = x.shape[-1]
        xf, w, b = _f32(x), _f32(weight), _f32(bias)
        R = xf.numel() // C
        y = torch.empty_like(xf)
        mean = torch.empty(R, device=xf.device)
        rstd = torch.empty(R, device=xf.device)
        _lib.call("csn_layer_norm_fwd", _ptr(xf), _ptr(w), _ptr(b), _ptr(y), _ptr(mean), _ptr(rstd), R, C,
                  float(eps), _stream(xf.device))
        ctx.save_for_backward(xf, w, mean, rstd)
        ctx.dtypes = (x.dtype, weight.dtype, bias.dtype)
        return y.to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        xf, w, mean, rstd = ctx.saved_tensors
        C = xf.shape[-1]
        R = xf.numel() // C
        g = _f32(dy)
        dx = torch.empty_like(xf)
        dw = torch.empty_like(w) if ctx.needs_input_grad[1] else None
        db = torch.empty_like(w) if ctx.needs_input_grad[2] else None
        nb = _lib.load().csn_layer_norm_bwd_workspace_bytes(R, C)
        ws = _workspace(max(nb, 16), xf.device)
        _lib.call("csn_layer_norm_bwd", _ptr(g), _ptr(xf), _ptr(mean), _ptr(rstd), _ptr(w), _ptr(dx), _ptr(dw),
                  _ptr(db), R, C, _ptr(ws), nb, _stream(xf.device))
        out = (dx.to(ctx.dtypes[0]), None if dw is None else dw.to(ctx.dtypes[1]),
               None if db is None else db.to(ctx.dtypes[2]), None)
        return out


LAYER_NORM_MAX_C = 1024


def layer_norm_supported(C: int) -> bool:
    """Feature counts the CUDA LayerNorm handles (C % 4 == 0, C <= 1024)."""
    return 0 < C <= LAYER_NORM_MAX_C and C % 4 == 0


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """F.layer_norm(x, (C,), weight, bias, eps) over the last axis as one CUDA kernel each way
    (the blocks' nn.LayerNorm, python/clifford_cl6.py:94,121,229); layer_norm_supported(C) only."""
    C = x.shape[-1]
    if not layer_norm_supported(C) or weight is None or bias is None:
        raise ValueError(f"layer_norm: needs affine weight and bias and C % 4 == 0, C <= {LAYER_NORM_MAX_C}")
    return LayerNormFunction.apply(x, weight, bias, eps)


class LnConvSiluFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, ln_w, ln_b, eps, conv_w, conv_b):
        _require_cuda(x, ln_w, ln_b, conv_w, conv_b)
        B, T, C = x.shape
        K = conv_w.shape[-1]
        xf, lw, lb, cw, cb = _f32(x), _f32(ln_w), _f32(ln_b), _f32(conv_w), _f32(conv_b)
        y = torch.empty_like(xf)
        mean = torch.empty(B * T, device=xf.device)
        rstd = torch.empty(B * T, device=xf.device)
        _lib.call("csn_ln_conv_silu_fwd", _ptr(xf), _ptr(lw), _ptr(lb), _ptr(cw), _ptr(cb), _ptr(y), _ptr(mean),
                  _ptr(rstd), B, T, C, K, float(eps), _stream(xf.device))
        ctx.save_for_backward(xf, lw, lb, cw, cb, mean, rstd)
        ctx.dtypes = (x.dtype, ln_w.dtype, ln_b.dtype, conv_w.dtype, conv_b.dtype)
        return y.to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        xf, lw, lb, cw, cb, mean, rstd = ctx.saved_tensors
        B, T, C = xf.shape
        K = cw.shape[-1]
        g = _f32(dy)
        dx = torch.empty_like(xf)
        need = ctx.needs_input_grad
        dlw = torch.empty_like(lw) if need[1] else None
        dlb = torch.empty_like(lb) if need[2] else None
        dcw = torch.empty_like(cw) if need[4] else None
        dcb = torch.empty_like(cb) if need[5] else None
        nb = _lib.load().csn_ln_conv_silu_bwd_workspace_bytes(B, T, C, K)
        ws = _workspace(max(nb, 16), xf.device)
        _lib.call("csn_ln_conv_silu_bwd", _ptr(g), _ptr(xf), _ptr(mean), _ptr(rstd), _ptr(lw), _ptr(lb), _ptr(cw),
                  _ptr(cb), _ptr(dx), _ptr(dlw), _ptr(dlb), _ptr(dcw), _ptr(dcb), B, T, C, K, _ptr(ws), nb,
                  _stream(xf.device))
        outs = (dx, dlw, dlb, None, dcw, dcb)
        dts = (ctx.dtypes[0], ctx.dtypes[1], ctx.dtypes[2], None, ctx.dtypes[3], ctx.dtypes[4])
        return tuple(None if o is None else o.to(d) for o, d in zip(outs, dts))


def ln_conv_silu_supported(C: int, K: int) -> bool:
    """Shapes the fused ln -> causal conv -> SiLU kernels handle (C % 4 == 0, C <= 256, K <= 4)."""
    return 0 < C <= 256 and C % 4 == 0 and 1 <= K <= 4


def ln_conv_silu(x, ln_weight, ln_bias, eps, conv_weight, conv_bias):
    """silu(causal_depthwise_conv1d(layer_norm(x))) over x [B, T, C] as one CUDA kernel each way:
    the blocks' python/clifford_cl6.py:140-142 (LayerNorm(C, eps), Conv1d(C, C, K, padding=K-1,
    groups=C) keeping the first T outputs, SiLU).  conv_weight [C, 1, K]."""
    B, T, C = x.shape
    K = conv_weight.shape[-1]
    if not ln_conv_silu_supported(C, K) or tuple(conv_weight.shape) != (C, 1, K) or conv_bias is None:
        raise ValueError("ln_conv_silu: needs C % 4 == 0, C <= 256, K <= 4, a [C, 1, K] depthwise weight and a bias")
    return LnConvSiluFunction.apply(x, ln_weight, ln_bias, eps, conv_weight, conv_bias)


class GeneratorActionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, biv, dt, D):
        _require_cuda(biv, dt)
        B, T = biv.shape[:2]
        H = dt.shape[2] if dt.dim() == 3 else 1
        bf, df = _f32(biv), _f32(dt)
        R = math.prod(biv.shape[2:])
        K = biv.shape[-1]
        ratio = 2.0 * K / float(D * D)
        ck = ratio / max(1, B * T * R)
        cs = ratio / max(1, B * (T - 1) * R) if T > 1 else 0.0
        out = torch.empty(2, device=bf.device)
        nb = _lib.load().csn_generator_action_workspace_bytes(B, T)
        ws = _workspace(max(nb, 16), bf.device)
        _lib.call("csn_generator_action_fwd", _ptr(bf), _ptr(df), B, T, R, H, ck, cs, _ptr(out), _ptr(ws), nb,
                  _stream(bf.device))
        ctx.save_for_backward(bf, df)
        ctx.meta = (B, T, R, H, ck, cs, biv.dtype, dt.dtype)
        return out[0].to(biv.dtype), out[1].to(biv.dtype)

    @staticmethod
    def backward(ctx, g_kin, g_smooth):
        bf, df = ctx.saved_tensors
        B, T, R, H, ck, cs, bdt, ddt_type = ctx.meta
        gk = None if g_kin is None else _f32(g_kin.reshape(1))
        gs = None if g_smooth is None else _f32(g_smooth.reshape(1))
        dbiv = torch.empty_like(bf) if ctx.needs_input_grad[0] else None
        ddt = torch.empty_like(df) if ctx.needs_input_grad[1] else None
        _lib.call("csn_generator_action_bwd", _ptr(bf), _ptr(df), _ptr(gk), _ptr(gs), B, T, R, H, ck, cs, _ptr(dbiv),
                  _ptr(ddt), _stream(bf.device))
        return (None if dbiv is None else dbiv.to(bdt), None if ddt is None else ddt.to(ddt_type), None)


def generator_action(biv, dt, D: int):
    """(Omega^2).mean() and ((Omega[:, 1:] - Omega[:, :-1])^2).mean() for Omega = skew(biv) * 0.5 dt
    (D x D, K = biv.shape[-1] generators) without forming Omega -- the LMs' least-action terms
    (python/clifford_cl6.py:257-262) as one CUDA kernel each way.  biv [B, T, ..., K]; dt [B, T]
    (one dt per step) or [B, T, H] (one per head: biv [B, T, H, ..., K])."""
    if biv.dim() < 3 or dt.shape[:2] != biv.shape[:2] or dt.dim() > 3:
        raise ValueError("generator_action: biv [B, T, ..., K] and dt [B, T] or [B, T, H]")
    return GeneratorActionFunction.apply(biv, dt, int(D))


def column_sum(x2d):
    """Deterministic column sums of a float32 [R, C] CUDA matrix (csn_column_sum)."""
    _require_cuda(x2d)
    xf = _f32(x2d)
    R, C = xf.shape
    out = torch.empty(C, device=xf.device)
    nb = _lib.load().csn_column_sum_workspace_bytes(R, C)
    ws = _workspace(max(nb, 16), xf.device)
    _lib.call("csn_column_sum", _ptr(xf), R, C, _ptr(out), _ptr(ws), nb, _stream(xf.device))
    return out


WGRAD_SPLIT = 32


def _weight_grad(d2, x2):
    """dW = d2^T x2 over R rows.  For the LM's R = B*T (tens of thousands of rows) and narrow
    W, one GEMM has too few output tiles to fill the GPU; the sum over rows is split into
    WGRAD_SPLIT batched GEMMs whose partial products are then added (deterministic; measured
    1.7x faster on [65536, 512] x [65536, 128])."""
    R = d2.shape[0]
    s = WGRAD_SPLIT
    if R % s == 0 and R >= s * 1024:
        return torch.bmm(d2.reshape(s, R // s, d2.shape[1]).transpose(1, 2),
                         x2.reshape(s, R // s, x2.shape[1])).sum(0)
    return d2.t() @ x2


class LinearFunction(torch.autograd.Function):
    """y = x W^T + b with cuBLAS GEMMs both ways (the weight gradient split over rows) and the
    bias gradient by csn_column_sum."""

    @staticmethod
    def forward(ctx, x, W, b):
        _require_cuda(x, W, b)
        x2 = x.reshape(-1, x.shape[-1])
        y = torch.addmm(b, x2, W.t()) if b is not None else x2 @ W.t()
        ctx.save_for_backward(x2, W)
        ctx.has_b = b is not None
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], W.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, W = ctx.saved_tensors
        d2 = dy.reshape(-1, dy.shape[-1])
        dx = (d2 @ W).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        dW = _weight_grad(d2, x2) if ctx.needs_input_grad[1] else None
        db = column_sum(d2).to(dy.dtype) if (ctx.has_b and ctx.needs_input_grad[2]) else None
        return dx, dW, db


def linear(x, W, b=None):
    """F.linear(x, W, b) whose bias gradient is a deterministic CUDA column sum."""
    return LinearFunction.apply(x, W, b)


class ProjectionEpilogueFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, raw, scale, dt_base, N, K, HT):
        _require_cuda(raw, scale)
        rf, sf = _f32(raw), _f32(scale)
        lead = raw.shape[:-1]
        R = rf.numel() // rf.shape[-1]
        biv = torch.empty(*lead, N * K, device=rf.device)
        gamma = torch.empty(*lead, N, device=rf.device)
        dt = torch.empty(*lead, HT, device=rf.device)
        _lib.call("csn_projection_epilogue_fwd", _ptr(rf), R, N, K, HT, _ptr(sf), float(dt_base), _ptr(biv),
                  _ptr(gamma), _ptr(dt), _stream(rf.device))
        ctx.save_for_backward(rf, sf)
        ctx.meta = (float(dt_base), N, K, HT, raw.dtype, scale.dtype)
        return biv, gamma, dt

    @staticmethod
    def backward(ctx, dbiv, dgamma, ddt):
        rf, sf = ctx.saved_tensors
        dt_base, N, K, HT, rdt, sdt = ctx.meta
        R = rf.numel() // rf.shape[-1]
        draw = torch.empty_like(rf)
        part = torch.empty(R, N, device=rf.device)
        _lib.call("csn_projection_epilogue_bwd", _ptr(rf), R, N, K, HT, _ptr(sf), dt_base,
                  _ptr(None if dbiv is None else _f32(dbiv)), _ptr(None if dgamma is None else _f32(dgamma)),
                  _ptr(None if ddt is None else _f32(ddt)), _ptr(draw), _ptr(part), _stream(rf.device))
        dscale = column_sum(part).to(sdt) if ctx.needs_input_grad[1] else None
        return draw.to(rdt), dscale, None, None, None, None


def projection_epilogue(raw, omega_scale, dt_base: float, N: int, K: int, HT: int):
    """(biv [..., N*K], gamma [..., N], dt [..., HT]) from the fused projection output raw
    [..., N*K + N + HT]: biv = raw * omega_scale[n], gamma = softplus, dt = softplus * dt_base
    (python/clifford_cl6.py:144-155), one CUDA kernel each way."""
    if raw.shape[-1] != N * K + N + HT or omega_scale.numel() != N:
        raise ValueError("projection_epilogue: raw must have N*K + N + HT columns and omega_scale N entries")
    return ProjectionEpilogueFunction.apply(raw, omega_scale.reshape(N), dt_base, N, K, HT)


class SiluGateFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        _require_cuda(gu)
        gf = _f32(gu)
        F2 = gf.shape[-1]
        R = gf.numel() // F2
        y = torch.empty(*gf.shape[:-1], F2 // 2, device=gf.device)
        _lib.call("csn_silu_gate_fwd", _ptr(gf), R, F2 // 2, _ptr(y), _stream(gf.device))
        ctx.save_for_backward(gf)
        ctx.dtype = gu.dtype
        return y.to(gu.dtype)

    @staticmethod
    def backward(ctx, dy):
        (gf,) = ctx.saved_tensors
        F2 = gf.shape[-1]
        R = gf.numel() // F2
        dgu = torch.empty_like(gf)
        _lib.call("csn_silu_gate_bwd", _ptr(gf), _ptr(_f32(dy)), R, F2 // 2, _ptr(dgu), _stream(gf.device))
        return dgu.to(ctx.dtype)


def silu_gate(gu):
    """silu(g) * u for gu = [g | u] on the last axis (GeometricGatedLinearUnit's gate,
    python/clifford_model.py:42-43), one CUDA kernel each way."""
    if gu.shape[-1] % 2:
        raise ValueError("silu_gate: the last axis must hold [g | u]")
    return SiluGateFunction.apply(gu)


class SpatialGeneratorsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, in_proj, biv_proj, metric, lambda_sw, gamma_log, D: int):
        _require_cuda(in_proj, biv_proj, metric, lambda_sw, gamma_log)
        B, NDD, H, W = in_proj.shape
        N = NDD // (D * D)
        cf, bf, mf = _f32(in_proj), _f32(biv_proj), _f32(metric)
        lf, gf = _f32(lambda_sw).reshape(1), _f32(gamma_log).reshape(N)
        omega = torch.empty(B, H * W, N, D, D, device=cf.device, dtype=torch.float32)
        c = torch.empty_like(omega)
        decay = torch.empty(B, H * W, N, device=cf.device, dtype=torch.float32)
        _lib.call("csn_spatial_generators_fwd", _ptr(cf), _ptr(bf), _ptr(mf), _ptr(lf), _ptr(gf), _ptr(omega),
                  _ptr(c), _ptr(decay), B, H * W, N, D, _stream(cf.device))
        ctx.save_for_backward(cf, bf, mf, lf, gf)
        ctx.D, ctx.dtypes = D, (in_proj.dtype, biv_proj.dtype, metric.dtype, lambda_sw.dtype, gamma_log.dtype)
        ctx.shapes = (lambda_sw.shape, gamma_log.shape)
        return omega, c, decay

    @staticmethod
    def backward(ctx, d_omega, d_c, d_decay):
        cf, bf, mf, lf, gf = ctx.saved_tensors
        D = ctx.D
        B, NDD, H, W = cf.shape
        N, HW = NDD // (D * D), H * W
        zeros = lambda shape: torch.zeros(shape, device=cf.device, dtype=torch.float32)
        dom = _f32(d_omega) if d_omega is not None else zeros((B, HW, N, D, D))
        dc = _f32(d_c) if d_c is not None else zeros((B, HW, N, D, D))
        ddec = _f32(d_decay) if d_decay is not None else zeros((B, HW, N))
        dcraw, dbraw, dmraw = torch.empty_like(cf), torch.empty_like(bf), torch.empty_like(mf)
        P = _lib.load().csn_spatial_generators_partials(B, HW, D)
        dlam = torch.zeros(P, device=cf.device, dtype=torch.float32)
        dgam = torch.zeros(P, N, device=cf.device, dtype=torch.float32)
        _lib.call("csn_spatial_generators_bwd", _ptr(cf), _ptr(bf), _ptr(mf), _ptr(lf), _ptr(gf), _ptr(dom),
                  _ptr(dc), _ptr(ddec), _ptr(dcraw), _ptr(dbraw), _ptr(dmraw), _ptr(dlam), _ptr(dgam),
                  B, HW, N, D, _stream(cf.device))
        t = ctx.dtypes
        return (dcraw.to(t[0]), dbraw.to(t[1]), dmraw.to(t[2]), dlam.sum().reshape(ctx.shapes[0]).to(t[3]),
                dgam.sum(0).reshape(ctx.shapes[1]).to(t[4]), None)


def spatial_generators(in_proj, biv_proj, metric, lambda_sw, gamma_log, D: int):
    """(Omega, C, decay) of the spatial rotor blocks from their NCHW convolution outputs
    (csn_toolkit/csn/vision.py:79-94, :136-151): ds = softplus(metric), Omega = clamp((skew(biv)
    + tanh(lambda) (C - C^T) / 2) ds / 2, -3, 3), decay = sigmoid(-softplus(gamma_log) ds).
    in_proj [B, N*D*D, H, W], biv_proj [B, N*K, H, W], metric [B, N, H, W] -> Omega, C
    [B, H*W, N, D, D] and decay [B, H*W, N], pixel-major; one CUDA kernel each way."""
    B, NDD, H, W = in_proj.shape
    K = D * (D - 1) // 2
    if NDD % (D * D) or biv_proj.shape != (B, NDD // (D * D) * K, H, W) or metric.shape != (B, NDD // (D * D), H, W):
        raise ValueError("spatial_generators: in_proj [B, N*D*D, H, W], biv_proj [B, N*K, H, W], "
                         "metric [B, N, H, W] expected")
    if lambda_sw.numel() != 1 or gamma_log.numel() != NDD // (D * D):
        raise ValueError("spatial_generators: lambda_sw has 1 value and gamma_log N")
    return SpatialGeneratorsFunction.apply(in_proj, biv_proj, metric, lambda_sw, gamma_log, D)


# torch.ops.csn.* registrations (needs the helpers above; imported last on purpose)
from . import library  # noqa: E402,F401
