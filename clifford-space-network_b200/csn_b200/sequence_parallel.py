"""Sequence-parallel rotor scan: one long sequence split over the ranks of a process group.

Rank g holds time steps [g*T, (g+1)*T) of every (batch, channel) sequence.  The scan is
associative, so each shard is summarised by its aggregate and only those summaries
cross GPUs (one all-gather of B*N pairs of D x D matrices per pass):

forward
  1. (P_g, c_g) = shard aggregate: P = M_last ... M_first, c = shard scanned from zero
  2. all-gather (P, c)
  3. carry-in h_g = scan of (P_r, c_r), r < g            (plain scan kernel, X_0 = c_0)
  4. resume the shard from h_g: carry + apply passes over the chunk aggregates of step 1
backward (mirror image in reverse time)
  1. c'_g = gradient leaving the shard at its first step with zero gradient from the right
  2. all-gather c'
  3. H_g = reverse scan of (P_r^T, c'_r), r > g           (gradient entering from the right)
  4. resume the local adjoint with h0 = h_g and H_g entering after the last step

The cross-shard compositions run on the same CUDA kernels as everything else.

Per direction the ranks make ONE collective and no host synchronisation: the shard
summaries are packed into one buffer together with a finiteness flag of this rank's
summaries, and all-gathered.  The gathered flags are reduced on the device and copied to
pinned host memory asynchronously; the next sequence-parallel call (or ``check()``) reads
that copy, long finished by then, and raises ``ShardMismatchError`` on every rank alike when
a carry was not finite.  The layout (shapes, flags) is validated once: the first call with a
given layout all-gathers a small header first, with a host check, so that a rank with a
mismatched shard is reported on every rank instead of deadlocking the collective; later
calls with a layout that every rank has validated skip it (ranks that keep calling with
the same shapes make the same decision).  A rank that changes its shapes alone after that
first call runs into the process group's timeout instead.

The kernel calls go through a backend object (``CudaBackend`` here); tests substitute a
CPU backend to exercise the exchange logic with the gloo backend.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .ops import BASIS, _f32, _ptr, _require_cuda, _stream, _workspace


class ShardMismatchError(RuntimeError):
    """Ranks disagree on the shard layout, or a gathered carry is not finite."""


class CudaBackend:
    """Shard primitives on the CUDA library (float32, current stream).

    The aggregate calls return their workspace: it holds the chunk aggregates that the
    matching resume call (``rotor_fwd`` / ``rotor_bwd`` with ``ws``) reuses, so each
    shard's inputs are reduced once per direction."""

    @staticmethod
    def _agg_ws(B, T, N, D, device):
        n = _lib.load().csn_rotor_scan_aggregate_workspace_bytes(B, T, N, D)
        return torch.empty(n, dtype=torch.uint8, device=device)

    def fwd_aggregate(self, gens, dt, gamma, S, basis, two_sided):
        B, T, N, D, _ = S.shape
        P = torch.empty(B, N, D, D, device=S.device)
        c = torch.empty_like(P)
        ws = self._agg_ws(B, T, N, D, S.device)
        _lib.call("csn_rotor_scan_aggregate", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(S), _ptr(P), _ptr(c),
                  B, T, N, D, BASIS[basis], int(two_sided), _ptr(ws), ws.numel(), _stream(S.device))
        return P, c, ws

    def bwd_aggregate(self, gens, dt, gamma, dX, basis, two_sided):
        B, T, N, D, _ = dX.shape
        c = torch.empty(B, N, D, D, device=dX.device)
        ws = self._agg_ws(B, T, N, D, dX.device)
        _lib.call("csn_rotor_scan_bwd_aggregate", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(dX), _ptr(c),
                  B, T, N, D, BASIS[basis], int(two_sided), _ptr(ws), ws.numel(), _stream(dX.device))
        return c, ws

    def scan_mc(self, M, C, two_sided):
        from .ops import _scan_fwd
        return _scan_fwd(_f32(M), _f32(C), None, two_sided)

    def rotor_fwd(self, gens, dt, gamma, S, h0, basis, two_sided, ws=None):
        B, T, N, D, _ = S.shape
        X = torch.empty_like(S)
        if ws is not None:
            _lib.call("csn_rotor_scan_fwd_resume", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(S), _ptr(h0),
                      _ptr(X), B, T, N, D, BASIS[basis], int(two_sided), _ptr(ws), ws.numel(),
                      _stream(S.device))
            return X
        n = _lib.load().csn_rotor_scan_workspace_bytes(B, T, N, D)
        w = _workspace(n, S.device)
        _lib.call("csn_rotor_scan_fwd", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(S), _ptr(h0), _ptr(X),
                  B, T, N, D, BASIS[basis], int(two_sided), _ptr(w), n, _stream(S.device))
        return X

    def rotor_bwd(self, gens, dt, gamma, S, h0, X, dX, basis, two_sided, dh_right=None, ws=None):
        B, T, N, D, _ = S.shape
        dg, ddt, dS = torch.empty_like(gens), torch.empty_like(dt), torch.empty_like(S)
        dga = torch.empty_like(gamma) if gamma is not None else None
        if ws is not None:
            _lib.call("csn_rotor_scan_bwd_resume", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(S), _ptr(h0),
                      _ptr(X), _ptr(dX), _ptr(dh_right), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS),
                      _ptr(None), B, T, N, D, BASIS[basis], int(two_sided), _ptr(ws), ws.numel(),
                      _stream(S.device))
            return dg, ddt, dga, dS
        if dh_right is not None:
            dX = dX.clone()
            dX[:, -1] += dh_right
        n = _lib.load().csn_rotor_scan_workspace_bytes(B, T, N, D)
        w = _workspace(n, S.device)
        _lib.call("csn_rotor_scan_bwd", _ptr(gens), _ptr(dt), _ptr(gamma), _ptr(S), _ptr(h0), _ptr(X),
                  _ptr(dX), _ptr(dg), _ptr(ddt), _ptr(dga), _ptr(dS), _ptr(None), B, T, N, D,
                  BASIS[basis], int(two_sided), _ptr(w), n, _stream(S.device))
        return dg, ddt, dga, dS


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _check_header(local: torch.Tensor, group, what: str):
    """All-gather a small int64 header; raise the same error on every rank on mismatch.
    One collective and one host synchronisation; it runs before any collective whose sizes
    depend on the shard, so a mismatched rank cannot leave the others waiting."""
    ws, _ = _world(group)
    hdr = local.new_empty((ws * local.shape[0],))
    dist.all_gather_into_tensor(hdr, local.contiguous(), group=group)
    hdr = hdr.view(ws, -1)
    bad = (hdr != hdr[:1]).any(dim=1)
    if bool(bad.any()):
        r = int(bad.nonzero()[0])
        raise ShardMismatchError(f"{what}: rank {r} shard header {hdr[r].tolist()} != rank 0 {hdr[0].tolist()}")


# layouts every rank of a group has validated: (group key, direction, header) -> True
_VALIDATED: dict = {}


def _group_key(group):
    return "default" if group is None else id(group)


def _validate_layout_once(header: tuple, group, direction: str, device, what: str):
    """The header exchange of `_check_header`, made only the first time this rank uses this
    layout on this group."""
    key = (_group_key(group), direction, header)
    if key in _VALIDATED:
        return
    _check_header(torch.tensor(header, dtype=torch.int64, device=device), group, what)
    _VALIDATED[key] = True


class _PendingCheck:
    """Finiteness of the last exchange: a device flag copied asynchronously to pinned host
    memory, read at the next call or by check()."""

    def __init__(self):
        self.item = None  # (host tensor [2], event or None, what)

    def set(self, bad_any, first_bad, what):
        flags = torch.stack([bad_any.to(torch.int64), first_bad.to(torch.int64)])
        if flags.is_cuda:
            host = torch.empty(2, dtype=torch.int64, pin_memory=True)
            host.copy_(flags, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(flags.device))
        else:
            host, ev = flags.clone(), None
        self.item = (host, ev, what)

    def raise_if_bad(self):
        if self.item is None:
            return
        host, ev, what = self.item
        self.item = None
        if ev is not None:
            ev.synchronize()  # recorded one exchange ago: normally long complete
        if int(host[0]):
            raise ShardMismatchError(f"{what}: carry from rank {int(host[1])} is not finite")


_PENDING = _PendingCheck()


def check() -> None:
    """Raise ShardMismatchError if the last exchange gathered a non-finite carry (every rank
    reaches the same verdict).  Calls of sp_forward / sp_backward do this themselves for the
    exchange before them."""
    _PENDING.raise_if_bad()


def _gather_packed(parts, group, what: str):
    """All-gather the shard summaries of every rank and this rank's finiteness flag in ONE
    collective (one packed buffer), with no host synchronisation; returns one [ws, ...]
    tensor per part.  The verdict on finiteness is left in _PENDING."""
    ws, _ = _world(group)
    shapes = [tuple(p.shape) for p in parts]
    flat = [p.reshape(-1) for p in parts]
    ok = torch.stack([torch.isfinite(f).all() for f in flat]).all().to(flat[0].dtype).reshape(1)
    local = torch.cat(flat + [ok])
    out = local.new_empty((ws * local.numel(),))
    dist.all_gather_into_tensor(out, local, group=group)  # rank-major concatenation
    out = out.view(ws, -1)
    bad = out[:, -1] == 0
    _PENDING.set(bad.any(), torch.argmax(bad.to(torch.int32)), what)
    res, o = [], 0
    for shp in shapes:
        n = 1
        for d in shp:
            n *= d
        res.append(out[:, o:o + n].reshape((ws,) + shp))
        o += n
    return res


def sp_forward(gens, dt, gamma, S, group=None, backend=None, basis="triu", two_sided=True):
    """Forward of the sequence-parallel scan on this rank's shard.

    Returns (X_local, h_in, Ps): the shard trajectory, the carry-in (None on rank 0) and the
    gathered shard products (kept for the backward pass)."""
    backend = backend or CudaBackend()
    _PENDING.raise_if_bad()
    ws, g = _world(group)
    B, T, N, D, _ = S.shape
    dev = S.device
    flags = int(gamma is not None) * 1 + int(two_sided) * 2 + (BASIS[basis] << 2)
    _validate_layout_once((B, T, N, D, gens.shape[-1], flags), group, "fwd", dev, "sequence-parallel forward")
    P, c, ws_fwd = backend.fwd_aggregate(gens, dt, gamma, S, basis, two_sided)
    Pall, call = _gather_packed([P, c], group, "sequence-parallel forward")  # [ws, B, N, D, D]
    Ps = list(Pall.unbind(0))
    h_in = None
    if g > 0:
        Mseq = Pall[:g].transpose(0, 1).contiguous()  # [B, g, N, D, D]
        Cseq = call[:g].transpose(0, 1).contiguous()
        h_in = backend.scan_mc(Mseq, Cseq, two_sided)[:, -1].contiguous()
    X = backend.rotor_fwd(gens, dt, gamma, S, h_in, basis, two_sided, ws=ws_fwd)
    return X, h_in, Ps


def sp_backward(gens, dt, gamma, S, X, dX, h_in, Ps, group=None, backend=None, basis="triu",
                two_sided=True):
    """Backward of the sequence-parallel scan: (dgens, ddt, dgamma, dS) of this shard."""
    backend = backend or CudaBackend()
    _PENDING.raise_if_bad()
    ws, g = _world(group)
    B, T, N, D, _ = S.shape
    _validate_layout_once((B, T, N, D, int(dX.shape == S.shape)), group, "bwd", S.device,
                          "sequence-parallel backward")
    cb, ws_bwd = backend.bwd_aggregate(gens, dt, gamma, dX, basis, two_sided)
    (cball,) = _gather_packed([cb], group, "sequence-parallel backward")
    cbs = list(cball.unbind(0))
    H = None
    if g < ws - 1:
        later = list(range(ws - 1, g, -1))         # r = G-1 .. g+1
        Mseq = torch.stack([Ps[r].transpose(-1, -2) for r in later], dim=1)
        Cseq = torch.stack([cbs[r] for r in later], dim=1)
        H = backend.scan_mc(Mseq, Cseq, two_sided)[:, -1].contiguous()
    return backend.rotor_bwd(gens, dt, gamma, S, h_in, X, dX, basis, two_sided, dh_right=H, ws=ws_bwd)


class SequenceParallelRotorScan(torch.autograd.Function):
    """Autograd wrapper: every rank calls it with its own time shard (same B, N, D, K)."""

    @staticmethod
    def forward(ctx, gens, dt, gamma, S, group, basis, two_sided):
        _require_cuda(gens, dt, gamma, S)
        g, d, ga, s = _f32(gens), _f32(dt), _f32(gamma), _f32(S)
        X, h_in, Ps = sp_forward(g, d, ga, s, group, None, basis, two_sided)
        ctx.save_for_backward(g, d, ga, s, X, h_in, *Ps)
        ctx.group, ctx.basis, ctx.two_sided = group, basis, two_sided
        return X

    @staticmethod
    def backward(ctx, dX):
        g, d, ga, s, X, h_in, *Ps = ctx.saved_tensors
        dg, ddt, dga, dS = sp_backward(g, d, ga, s, X, _f32(dX), h_in, list(Ps), ctx.group, None,
                                       ctx.basis, ctx.two_sided)
        return dg, ddt, dga, dS, None, None, None


def sequence_parallel_rotor_scan(gens, dt, gamma, S, group=None, basis="triu", two_sided=True):
    """Rotor scan of a sequence whose time axis is sharded over the ranks of `group`.

    Each rank passes its own shard ([B, T_local, N, ...]); ranks must be ordered by time.
    """
    B, T, N = S.shape[:3]
    return SequenceParallelRotorScan.apply(gens, dt.reshape(B, T), None if gamma is None else
                                           gamma.reshape(B, T, N), S, group, basis, bool(two_sided))
