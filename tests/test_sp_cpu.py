"""Sequence-parallel exchange logic on CPU ranks (gloo), with the float64 oracle standing
in for the CUDA shard primitives.  Each rank owns a time shard; the sharded forward and
backward must equal the single-process scan of the whole sequence.  Failures are made on
the host: a rank with a mismatched shard, a non-finite carry, and a rank that never joins."""
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


class OracleBackend:
    """CPU float64 stand-in for csn_b200.sequence_parallel.CudaBackend."""

    def __init__(self, basis_matrix, poison=False):
        from oracle import oracle as orc
        self.orc, self.E, self.poison = orc, basis_matrix, poison

    @staticmethod
    def _n(t):
        return None if t is None else t.detach().double().numpy()

    def fwd_aggregate(self, gens, dt, gamma, S, basis, two_sided):
        o, n = self.orc, self._n
        M, _ = o.rotor_build(n(gens), n(dt), n(gamma), n(S), self.E)
        B, T, N, D, _ = M.shape
        P = np.broadcast_to(np.eye(D), (B, N, D, D)).copy()
        for t in range(T):
            P = M[:, t] @ P
        c = o.rotor_scan_fwd(n(gens), n(dt), n(gamma), n(S), self.E, two_sided=two_sided)[:, -1]
        if self.poison:
            c = c * np.nan
        return torch.from_numpy(P), torch.from_numpy(np.ascontiguousarray(c)), None

    def bwd_aggregate(self, gens, dt, gamma, dX, basis, two_sided):
        o, n = self.orc, self._n
        B, T, N, D, _ = dX.shape
        S = np.zeros((B, T, N, D, D))
        X = o.rotor_scan_fwd(n(gens), n(dt), n(gamma), S, self.E, h0=np.zeros((B, N, D, D)),
                             two_sided=two_sided)
        *_, dh0 = o.rotor_scan_bwd(n(gens), n(dt), n(gamma), S, self.E, X, n(dX),
                                   h0=np.zeros((B, N, D, D)), two_sided=two_sided)
        return torch.from_numpy(dh0), None

    def scan_mc(self, M, C, two_sided):
        return torch.from_numpy(self.orc.scan_fwd(self._n(M), self._n(C), two_sided=two_sided))

    def rotor_fwd(self, gens, dt, gamma, S, h0, basis, two_sided, ws=None):
        n = self._n
        return torch.from_numpy(self.orc.rotor_scan_fwd(n(gens), n(dt), n(gamma), n(S), self.E, h0=n(h0),
                                                        two_sided=two_sided))

    def rotor_bwd(self, gens, dt, gamma, S, h0, X, dX, basis, two_sided, dh_right=None, ws=None):
        n = self._n
        if dh_right is not None:
            dX = dX.clone()
            dX[:, -1] += dh_right
        h0n = n(h0) if h0 is not None else np.zeros((S.shape[0], S.shape[2], S.shape[3], S.shape[4]))
        dg, ddt, dga, dS, _ = self.orc.rotor_scan_bwd(n(gens), n(dt), n(gamma), n(S), self.E, n(X), n(dX),
                                                      h0=h0n, two_sided=two_sided)
        t = torch.from_numpy
        return t(dg), t(ddt), None if dga is None else t(dga), t(dS)


def make_problem(B, T, N, D, damped, seed=0):
    from csn_b200 import algebra
    rng = np.random.default_rng(seed)
    E = algebra.triu_basis(D)
    gens = rng.standard_normal((B, T, N, E.shape[0])) * 3.0
    dt = rng.uniform(0.01, 0.1, (B, T))
    gamma = np.log1p(np.exp(rng.standard_normal((B, T, N)))) if damped else None
    S = rng.standard_normal((B, T, N, D, D))
    dX = rng.standard_normal((B, T, N, D, D))
    return E, gens, dt, gamma, S, dX


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, scenario, q, shape, damped, two_sided):
    try:
        for p in (str(REPO / "clifford-space-network_b200"), str(REPO)):
            if p not in sys.path:
                sys.path.insert(0, p)
        from datetime import timedelta
        from csn_b200 import sequence_parallel as sp
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=6))
        B, T, N, D = shape
        E, gens, dt, gamma, S, dX = make_problem(B, T, N, D, damped)
        Tl = T // ws
        sl = slice(rank * Tl, (rank + 1) * Tl)
        t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a[:, sl]))
        lg, ldt, lga, lS, ldX = t(gens), t(dt), t(gamma), t(S), t(dX)
        be = OracleBackend(E, poison=(scenario == "nan" and rank == 1))
        if scenario == "mismatch" and rank == 1:
            lS = lS[:, :-1].contiguous()
            lg, ldt = lg[:, :-1].contiguous(), ldt[:, :-1].contiguous()
            if lga is not None:
                lga = lga[:, :-1].contiguous()
        if scenario == "dropped" and rank == 1:
            q.put((rank, "left"))
            return  # never joins the collective
        X, h_in, Ps = sp.sp_forward(lg, ldt, lga, lS, None, be, "triu", two_sided)
        dg, ddt, dga, dS = sp.sp_backward(lg, ldt, lga, lS, X, ldX, h_in, Ps, None, be, "triu", two_sided)
        q.put((rank, "ok", X.numpy(), dg.numpy(), ddt.numpy(), None if dga is None else dga.numpy(),
               dS.numpy()))
    except Exception as e:  # report the failure to the parent
        q.put((rank, "error", type(e).__name__, str(e), traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run_ranks(ws, scenario, shape=(2, 24, 2, 4), damped=True, two_sided=True):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, scenario, q, shape, damped, two_sided))
             for r in range(ws)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(ws):
        item = q.get(timeout=120)
        out[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("ws", [2, 3])
@pytest.mark.parametrize("damped,two_sided", [(True, True), (False, True), (True, False)])
def test_sharded_scan_equals_single_process(oracle, ws, damped, two_sided):
    shape = (2, 24, 2, 4)
    out = run_ranks(ws, "ok", shape, damped, two_sided)
    assert all(v[0] == "ok" for v in out.values()), {k: v[:3] for k, v in out.items()}
    B, T, N, D = shape
    E, gens, dt, gamma, S, dX = make_problem(B, T, N, D, damped)
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E, two_sided=two_sided)
    dg, ddt, dga, dS, _ = oracle.rotor_scan_bwd(gens, dt, gamma, S, E, Xr, dX, two_sided=two_sided)
    cat = lambda i: np.concatenate([out[r][i] for r in range(ws)], axis=1)
    assert np.max(np.abs(cat(1) - Xr)) < 1e-9
    assert np.max(np.abs(cat(2) - dg)) < 1e-9
    assert np.max(np.abs(cat(3) - ddt)) < 1e-9
    assert np.max(np.abs(cat(5) - dS)) < 1e-9
    if damped:
        assert np.max(np.abs(cat(4) - dga)) < 1e-9


def test_mismatched_shard_is_reported_on_every_rank():
    out = run_ranks(2, "mismatch")
    for r in (0, 1):
        assert out[r][0] == "error" and out[r][1] == "ShardMismatchError", out[r][:3]


def test_non_finite_carry_is_reported_on_every_rank():
    out = run_ranks(2, "nan")
    for r in (0, 1):
        assert out[r][0] == "error" and out[r][1] == "ShardMismatchError", out[r][:3]
        assert "not finite" in out[r][2]


def test_dropped_rank_ends_the_collective_with_an_error():
    out = run_ranks(2, "dropped")
    assert out[1][0] == "left"
    assert out[0][0] == "error", out[0][:3]
