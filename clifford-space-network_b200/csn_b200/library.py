"""PyTorch operator registrations: ``torch.ops.csn.*``.

The same CUDA entry points as ``csn_b200.ops``, registered with ``torch.library`` so that
they are first-class operators: they have a schema, a fake (shape-only) implementation for
tracing on meta / fake tensors, and autograd through the matching ``*_bwd`` operator.
Every operator computes in float32 on CUDA tensors and returns float32.

    scan_fwd(M, C, h0?, two_sided, reverse) -> X            scan_bwd(...) -> (dM, dC, dh0)
    fused_rotor_scan_fwd(gens, dt, gamma?, S, h0?, basis, two_sided) -> X
    fused_rotor_scan_bwd(...) -> (dgens, ddt, dgamma, dS, dh0)
    cayley_fwd(Omega) -> Q                                   cayley_bwd(Q, dQ) -> dOmega
    cell_fwd(x, prev, W_rec, W_in, gamma_bias, dt) -> next   cell_bwd(...) -> 5 gradients
    ga3_scan_fwd(gens, dt, x, h0?) -> h                      ga3_scan_bwd(...) -> 4 gradients
    rotor_step(gens, dt, gamma?, S, h!, basis, two_sided)    (updates h in place)

Optional gradients that do not exist (no h0, undamped) come back as empty tensors.
The sequence-parallel scan takes a process group and stays a Python entry point
(csn_b200.sequence_parallel.sequence_parallel_rotor_scan).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import ops
from .ops import _f32, _require_cuda

_EMPTY = lambda ref: ref.new_empty((0,), dtype=torch.float32)


def _f(t):
    return None if t is None else _f32(t)


def _like(t):
    return torch.empty(t.shape, dtype=torch.float32, device=t.device)


# ------------------------------------------------------------------ plain scan
@torch.library.custom_op("csn::scan_fwd", mutates_args=())
def scan_fwd(M: Tensor, C: Tensor, h0: Optional[Tensor], two_sided: bool, reverse: bool) -> Tensor:
    _require_cuda(M, C, h0)
    return ops._scan_fwd(_f(M), _f(C), _f(h0), two_sided, reverse)


@scan_fwd.register_fake
def _(M, C, h0, two_sided, reverse):
    return _like(C)


@torch.library.custom_op("csn::scan_bwd", mutates_args=())
def scan_bwd(M: Tensor, X: Tensor, dX: Tensor, h0: Optional[Tensor], two_sided: bool,
             reverse: bool) -> Tuple[Tensor, Tensor, Tensor]:
    _require_cuda(M, X, dX, h0)
    dM, dC, dh0 = ops._scan_bwd(_f(M), _f(X), _f(dX), _f(h0), two_sided, h0 is not None, reverse)
    return dM, dC, (dh0 if dh0 is not None else _EMPTY(M))


@scan_bwd.register_fake
def _(M, X, dX, h0, two_sided, reverse):
    return _like(M), _like(M), (_like(h0) if h0 is not None else M.new_empty((0,), dtype=torch.float32))


def _scan_setup(ctx, inputs, output):
    M, C, h0, two_sided, reverse = inputs
    ctx.save_for_backward(M, output, h0)
    ctx.two_sided, ctx.reverse, ctx.has_h0 = two_sided, reverse, h0 is not None


def _scan_backward(ctx, dX):
    M, X, h0 = ctx.saved_tensors
    dM, dC, dh0 = torch.ops.csn.scan_bwd(M, X, dX, h0, ctx.two_sided, ctx.reverse)
    return dM, dC, (dh0 if ctx.has_h0 else None), None, None


scan_fwd.register_autograd(_scan_backward, setup_context=_scan_setup)


# ------------------------------------------------------------ fused rotor scan
@torch.library.custom_op("csn::fused_rotor_scan_fwd", mutates_args=())
def fused_rotor_scan_fwd(gens: Tensor, dt: Tensor, gamma: Optional[Tensor], S: Tensor,
                         h0: Optional[Tensor], basis: int, two_sided: bool) -> Tensor:
    _require_cuda(gens, dt, gamma, S, h0)
    return ops._rotor_fwd(_f(gens), _f(dt), _f(gamma), _f(S), _f(h0), basis, two_sided)


@fused_rotor_scan_fwd.register_fake
def _(gens, dt, gamma, S, h0, basis, two_sided):
    return _like(S)


@torch.library.custom_op("csn::fused_rotor_scan_bwd", mutates_args=())
def fused_rotor_scan_bwd(gens: Tensor, dt: Tensor, gamma: Optional[Tensor], S: Tensor,
                         h0: Optional[Tensor], X: Tensor, dX: Tensor, basis: int,
                         two_sided: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    _require_cuda(gens, dt, gamma, S, h0, X, dX)
    dg, ddt, dga, dS, dh0 = ops._rotor_bwd(_f(gens), _f(dt), _f(gamma), _f(S), _f(h0), _f(X), _f(dX),
                                           basis, two_sided, h0 is not None)
    return dg, ddt, (dga if dga is not None else _EMPTY(S)), dS, (dh0 if dh0 is not None else _EMPTY(S))


@fused_rotor_scan_bwd.register_fake
def _(gens, dt, gamma, S, h0, X, dX, basis, two_sided):
    e = S.new_empty((0,), dtype=torch.float32)
    return (_like(gens), _like(dt), _like(gamma) if gamma is not None else e, _like(S),
            _like(h0) if h0 is not None else e)


def _rotor_setup(ctx, inputs, output):
    gens, dt, gamma, S, h0, basis, two_sided = inputs
    ctx.save_for_backward(gens, dt, gamma, S, h0, output)
    ctx.basis, ctx.two_sided = basis, two_sided
    ctx.has = (gamma is not None, h0 is not None)


def _rotor_backward(ctx, dX):
    gens, dt, gamma, S, h0, X = ctx.saved_tensors
    dg, ddt, dga, dS, dh0 = torch.ops.csn.fused_rotor_scan_bwd(gens, dt, gamma, S, h0, X, dX,
                                                                ctx.basis, ctx.two_sided)
    return dg, ddt, (dga if ctx.has[0] else None), dS, (dh0 if ctx.has[1] else None), None, None


fused_rotor_scan_fwd.register_autograd(_rotor_backward, setup_context=_rotor_setup)


# ----------------------------------------------------------------------- Cayley
@torch.library.custom_op("csn::cayley_fwd", mutates_args=())
def cayley_fwd(Omega: Tensor) -> Tensor:
    _require_cuda(Omega)
    return ops._cayley_fwd(_f(Omega))


@cayley_fwd.register_fake
def _(Omega):
    return _like(Omega)


@torch.library.custom_op("csn::cayley_bwd", mutates_args=())
def cayley_bwd(Q: Tensor, dQ: Tensor) -> Tensor:
    _require_cuda(Q, dQ)
    return ops._cayley_bwd(_f(Q), _f(dQ))


@cayley_bwd.register_fake
def _(Q, dQ):
    return _like(Q)


def _cayley_setup(ctx, inputs, output):
    ctx.save_for_backward(output)


def _cayley_backward(ctx, dQ):
    (Q,) = ctx.saved_tensors
    return torch.ops.csn.cayley_bwd(Q, dQ)


cayley_fwd.register_autograd(_cayley_backward, setup_context=_cayley_setup)


# ------------------------------------------------------------------------- cell
@torch.library.custom_op("csn::cell_fwd", mutates_args=())
def cell_fwd(x: Tensor, prev: Tensor, W_rec: Tensor, W_in: Tensor, gamma_bias: Tensor,
             dt: float) -> Tensor:
    _require_cuda(x, prev, W_rec, W_in, gamma_bias)
    return ops._cell_fwd(_f(x), _f(prev), _f(W_rec), _f(W_in), _f(gamma_bias), dt)


@cell_fwd.register_fake
def _(x, prev, W_rec, W_in, gamma_bias, dt):
    return _like(prev)


@torch.library.custom_op("csn::cell_bwd", mutates_args=())
def cell_bwd(x: Tensor, prev: Tensor, W_rec: Tensor, W_in: Tensor, gamma_bias: Tensor, dt: float,
             dnext: Tensor) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    _require_cuda(x, prev, W_rec, W_in, gamma_bias, dnext)
    return ops._cell_bwd(_f(x), _f(prev), _f(W_rec), _f(W_in), _f(gamma_bias), dt, _f(dnext))


@cell_bwd.register_fake
def _(x, prev, W_rec, W_in, gamma_bias, dt, dnext):
    return _like(x), _like(prev), _like(W_rec), _like(W_in), _like(gamma_bias)


def _cell_setup(ctx, inputs, output):
    x, prev, W_rec, W_in, gamma_bias, dt = inputs
    ctx.save_for_backward(x, prev, W_rec, W_in, gamma_bias)
    ctx.dt = dt


def _cell_backward(ctx, dnext):
    x, prev, W_rec, W_in, gamma_bias = ctx.saved_tensors
    return (*torch.ops.csn.cell_bwd(x, prev, W_rec, W_in, gamma_bias, ctx.dt, dnext), None)


cell_fwd.register_autograd(_cell_backward, setup_context=_cell_setup)


# --------------------------------------------------------- Cl(3,0) blade scan
@torch.library.custom_op("csn::ga3_scan_fwd", mutates_args=())
def ga3_scan_fwd(gens: Tensor, dt: Tensor, x: Tensor, h0: Optional[Tensor]) -> Tensor:
    _require_cuda(gens, dt, x, h0)
    return ops._ga3_fwd(_f(gens), _f(dt), _f(x), _f(h0))


@ga3_scan_fwd.register_fake
def _(gens, dt, x, h0):
    return _like(x)


@torch.library.custom_op("csn::ga3_scan_bwd", mutates_args=())
def ga3_scan_bwd(gens: Tensor, dt: Tensor, h0: Optional[Tensor], h: Tensor,
                 dh: Tensor) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    _require_cuda(gens, dt, h0, h, dh)
    dg, ddt, dx, dh0 = ops._ga3_bwd(_f(gens), _f(dt), _f(h0), _f(h), _f(dh), h0 is not None)
    return dg, ddt, dx, (dh0 if dh0 is not None else _EMPTY(h))


@ga3_scan_bwd.register_fake
def _(gens, dt, h0, h, dh):
    return _like(gens), _like(dt), _like(h), (_like(h0) if h0 is not None
                                              else h.new_empty((0,), dtype=torch.float32))


def _ga3_setup(ctx, inputs, output):
    gens, dt, x, h0 = inputs
    ctx.save_for_backward(gens, dt, h0, output)
    ctx.has_h0 = h0 is not None


def _ga3_backward(ctx, dh):
    gens, dt, h0, h = ctx.saved_tensors
    dg, ddt, dx, dh0 = torch.ops.csn.ga3_scan_bwd(gens, dt, h0, h, dh)
    return dg, ddt, dx, (dh0 if ctx.has_h0 else None)


ga3_scan_fwd.register_autograd(_ga3_backward, setup_context=_ga3_setup)


# -------------------------------------------------------- O(1) generation step
@torch.library.custom_op("csn::rotor_step", mutates_args=("h",))
def rotor_step(gens: Tensor, dt: Tensor, gamma: Optional[Tensor], S: Tensor, h: Tensor, basis: int,
               two_sided: bool) -> None:
    ops.rotor_step(gens, dt, gamma, S, h, basis={v: k for k, v in ops.BASIS.items()}[basis],
                   two_sided=two_sided)


@rotor_step.register_fake
def _(gens, dt, gamma, S, h, basis, two_sided):
    return None


# ------------------------------------------------------- sequence-parallel scan
def _resolve_group(group_name: str):
    """The process group registered under `group_name` ("" = the default group)."""
    if not group_name:
        return None
    import torch.distributed.distributed_c10d as c10d
    return c10d._resolve_process_group(group_name)


def _basis_name(basis: int) -> str:
    return {v: k for k, v in ops.BASIS.items()}[basis]


@torch.library.custom_op("csn::sp_scan", mutates_args=())
def sp_scan(gens: Tensor, dt: Tensor, gamma: Optional[Tensor], S: Tensor, group_name: str, basis: int,
            two_sided: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """Sequence-parallel fused rotor scan of this rank's time shard over the group named
    `group_name` (csn_b200.sequence_parallel): returns (X, h_in, Ps) -- the shard's trajectory,
    its carry-in (zeros on the first rank) and the gathered shard products [ranks, B, N, D, D],
    the last two kept for the backward.  Every rank of the group calls it with its shard."""
    from .sequence_parallel import sp_forward
    B, T, N, D, _ = S.shape
    g, d, ga, sf = _f(gens), _f(dt).reshape(B, T), _f(gamma), _f(S)
    X, h_in, Ps = sp_forward(g, d, None if ga is None else ga.reshape(B, T, N), sf, _resolve_group(group_name),
                             None, _basis_name(basis), two_sided)
    h = h_in if h_in is not None else torch.zeros(B, N, D, D, device=S.device)
    return X, h, torch.stack(Ps)


@sp_scan.register_fake
def _(gens, dt, gamma, S, group_name, basis, two_sided):
    import torch.distributed as dist
    ws = dist.get_world_size(_resolve_group(group_name)) if dist.is_initialized() else 1
    B, T, N, D, _ = S.shape
    return (torch.empty_like(S, dtype=torch.float32), S.new_empty((B, N, D, D), dtype=torch.float32),
            S.new_empty((ws, B, N, D, D), dtype=torch.float32))


@torch.library.custom_op("csn::sp_scan_bwd", mutates_args=())
def sp_scan_bwd(gens: Tensor, dt: Tensor, gamma: Optional[Tensor], S: Tensor, X: Tensor, dX: Tensor,
                h_in: Tensor, Ps: Tensor, group_name: str, basis: int,
                two_sided: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """Adjoint of csn::sp_scan on this rank's shard: (dgens, ddt, dgamma or [0], dS)."""
    from .sequence_parallel import sp_backward
    B, T, N, D, _ = S.shape
    ga = _f(gamma)
    dg, ddt, dga, dS = sp_backward(_f(gens), _f(dt).reshape(B, T), None if ga is None else ga.reshape(B, T, N),
                                   _f(S), _f(X), _f(dX), _f(h_in), list(_f(Ps).unbind(0)),
                                   _resolve_group(group_name), None, _basis_name(basis), two_sided)
    return (dg, ddt.reshape(dt.shape), dga.reshape(gamma.shape) if dga is not None else dS.new_empty((0,)), dS)


@sp_scan_bwd.register_fake
def _(gens, dt, gamma, S, X, dX, h_in, Ps, group_name, basis, two_sided):
    return (torch.empty_like(gens, dtype=torch.float32), torch.empty_like(dt, dtype=torch.float32),
            torch.empty_like(gamma, dtype=torch.float32) if gamma is not None else S.new_empty((0,)),
            torch.empty_like(S, dtype=torch.float32))


def _sp_setup(ctx, inputs, output):
    gens, dt, gamma, S, group_name, basis, two_sided = inputs
    X, h, Ps = output
    ctx.save_for_backward(gens, dt, gamma, S, X, h, Ps)
    ctx.args = (group_name, basis, two_sided)


def _sp_backward(ctx, dX, dh, dPs):
    gens, dt, gamma, S, X, h, Ps = ctx.saved_tensors
    dg, ddt, dga, dS = torch.ops.csn.sp_scan_bwd(gens, dt, gamma, S, X, dX, h, Ps, *ctx.args)
    return dg, ddt, (dga if gamma is not None else None), dS, None, None, None


sp_scan.register_autograd(_sp_backward, setup_context=_sp_setup)
