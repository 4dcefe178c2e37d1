"""GPU parity at the benchmarked shapes and launch plans, through the C ABI entry points
that bench.py times, against the float64 oracle.

The other parity tests use a handful of sequences.  The chunk plan, however, is sized from
B * N to fill the 148 SMs, so the bench's shapes run chunkings that small shapes never
reach.  Each test here launches the full benchmark problem on the GPU, then checks a seeded
subset of whole batches (every channel of the chosen batch rows, so the per-batch dt
gradient, a sum over channels, is checkable too) at full sequence length against the
oracle run on that subset.  Sequences are independent, so a subset is an exact check of
the sequences in it.

Tolerances (reference metric max|a - ref| / max|ref|,
csn_toolkit/examples/benchmark_cuda_kernels.py:60-62): forward <= 1e-4; gradients <= 1e-3
at L = 2048 (the reference's gradient bound) and <= 1e-4 at L = 8192 (the fp32-over-8192
contract of the rotor scan).  The Cl(3) run is 65536 steps long: its first 8192 steps are
held to 1e-4 and the whole length to the bounds stated in that test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def rel(a, ref):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(a - ref)) / den)


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def lib():
    from csn_b200 import _build, _lib
    _build.build()
    assert torch.cuda.is_available()
    return _lib


def _subset(t, rows):
    return t[rows].double().cpu().numpy()


# --------------------------------------------------------------- Cl(6) LM scan, B32 L2048 C8
CL6_MAGNITUDES = {
    # the bench workload's inputs (bench.py Cl6LM)
    "bench": dict(gscale=1.0, dt=(0.04, 0.06), gam=0.5),
    # generator and dt ranges of the Cl(6) configurations of the reference's benchmark set
    "cfg": dict(gscale=0.1, dt=(0.01, 0.1), gam=1.0),
}


@pytest.mark.parametrize("mag", sorted(CL6_MAGNITUDES))
def test_cl6_lm_shape_fwd_and_reusing_bwd_match_oracle(lib, oracle, mag):
    """B32 L2048 N8 D8 two-sided damped through csn_rotor_scan_fwd + csn_rotor_scan_bwd_reuse
    on one workspace (the bench's calls), checked on 4 whole batch rows (32 sequences)."""
    from csn_b200 import algebra
    m = CL6_MAGNITUDES[mag]
    B, T, N, D, K = 32, 2048, 8, 8, 28
    g = torch.Generator(device="cpu").manual_seed(2048)
    gens = torch.randn(B, T, N, K, generator=g) * m["gscale"]
    lo, hi = m["dt"]
    dt = torch.rand(B, T, generator=g) * (hi - lo) + lo
    gamma = torch.nn.functional.softplus(torch.randn(B, T, N, generator=g) * m["gam"])
    S = torch.randn(B, T, N, D, D, generator=g)
    dX = torch.randn(B, T, N, D, D, generator=g)
    gens, dt, gamma, S, dX = (t.to(DEV) for t in (gens, dt, gamma, S, dX))
    X, dS = torch.empty_like(S), torch.empty_like(S)
    dgens, ddt, dgamma = torch.empty_like(gens), torch.empty_like(dt), torch.empty_like(gamma)
    nb = lib.load().csn_rotor_scan_workspace_bytes(B, T, N, D)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    st = _stream()
    lib.call("csn_rotor_scan_fwd", _p(gens), _p(dt), _p(gamma), _p(S), None, _p(X), B, T, N, D, 0, 1,
             _p(ws), nb, st)
    lib.call("csn_rotor_scan_bwd_reuse", _p(gens), _p(dt), _p(gamma), _p(S), None, _p(X), _p(dX),
             _p(dgens), _p(ddt), _p(dgamma), _p(dS), None, B, T, N, D, 0, 1, _p(ws), nb, st)
    torch.cuda.synchronize()
    rows = np.random.default_rng(5).choice(B, 4, replace=False)
    E = algebra.triu_basis(D)
    a = {k: _subset(v, rows) for k, v in dict(gens=gens, dt=dt, gamma=gamma, S=S, dX=dX).items()}
    Xr = oracle.rotor_scan_fwd(a["gens"], a["dt"], a["gamma"], a["S"], E)
    dg, ddt_r, dgam, dS_r, _ = oracle.rotor_scan_bwd(a["gens"], a["dt"], a["gamma"], a["S"], E, Xr, a["dX"])
    assert rel(X[rows], Xr) < 1e-4
    assert rel(dS[rows], dS_r) < 1e-3
    assert rel(dgens[rows], dg) < 1e-3
    assert rel(ddt[rows], ddt_r) < 1e-3
    assert rel(dgamma[rows], dgam) < 1e-3
    assert torch.isfinite(X).all() and torch.isfinite(dgens).all()


# ------------------------------------------------------- Cl(8) scan, B16 L8192 C32, GA basis
def test_cl8_shape_cached_rotor_path_matches_oracle(lib, oracle):
    """B16 L8192 C32 D16 with the 28 GA bivector-blade generators, undamped two-sided, through
    csn_rotor_scan_fwd_cached + csn_rotor_scan_heads_bwd (cached rotors, reused chunk
    products: the bench's calls), checked on one whole batch row (32 sequences, L = 8192)."""
    from csn_b200 import algebra
    B, T, N, D, K = 16, 8192, 32, 16, 28
    g = torch.Generator(device=DEV).manual_seed(8192)
    gens = torch.randn(B, T, N, K, generator=g, device=DEV) * 0.05
    dt = torch.rand(B, T, generator=g, device=DEV) * 0.045 + 0.005
    S = torch.randn(B, T, N, D, D, generator=g, device=DEV)
    dX = torch.randn(B, T, N, D, D, generator=g, device=DEV)
    X, dS, Mc = torch.empty_like(S), torch.empty_like(S), torch.empty_like(S)
    dgens, ddt = torch.empty_like(gens), torch.empty_like(dt)
    nb = lib.load().csn_rotor_scan_workspace_bytes(B, T, N, D)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    st = _stream()
    lib.call("csn_rotor_scan_fwd_cached", _p(gens), _p(dt), None, _p(S), None, _p(X), _p(Mc), B, T, N, D,
             1, 1, _p(ws), nb, st)
    lib.call("csn_rotor_scan_heads_bwd", _p(gens), _p(dt), None, _p(S), None, _p(X), _p(dX), _p(Mc),
             _p(dgens), _p(ddt), None, _p(dS), None, B, T, 1, N, D, 1, 1, 1, _p(ws), nb, st)
    torch.cuda.synchronize()
    del Mc
    rows = np.array([11])
    E = algebra.bivector_basis(algebra.CL8)
    a = {k: _subset(v, rows) for k, v in dict(gens=gens, dt=dt, S=S, dX=dX).items()}
    Xr = oracle.rotor_scan_fwd(a["gens"], a["dt"], None, a["S"], E)
    dg, ddt_r, _, dS_r, _ = oracle.rotor_scan_bwd(a["gens"], a["dt"], None, a["S"], E, Xr, a["dX"])
    assert rel(X[rows], Xr) < 1e-4
    assert rel(dS[rows], dS_r) < 1e-4
    assert rel(dgens[rows], dg) < 1e-4
    assert rel(ddt[rows], ddt_r) < 1e-4


# --------------------------------------------------- Cl(3) scan at bandwidth scale, B64 L65536 C16
def test_cl3_bandwidth_shape_matches_oracle(lib, oracle):
    """B64 L65536 C16 Cl(3,0) blade-basis scan through csn_ga3_scan_fwd/bwd (the bench's
    calls), checked on 2 whole batch rows (32 sequences).  The first 8192 steps of the
    forward are held to the 1e-4 contract.  Over all 65536 steps the fp32 recurrence keeps
    drifting from the float64 one (the states grow like sqrt(t) with unit-variance
    injections); the whole-length bounds are 1e-4 forward and 1e-3 for the gradients."""
    B, T, N = 64, 65536, 16
    g = torch.Generator(device=DEV).manual_seed(65536)
    gens = torch.randn(B, T, N, 3, generator=g, device=DEV) * 0.1
    dt = torch.rand(B, T, generator=g, device=DEV) * 0.09 + 0.01
    x = torch.randn(B, T, N, 8, generator=g, device=DEV)
    dh = torch.randn(B, T, N, 8, generator=g, device=DEV)
    h, dx = torch.empty_like(x), torch.empty_like(x)
    dgens, ddt = torch.empty_like(gens), torch.empty_like(dt)
    nb = lib.load().csn_ga3_workspace_bytes(B, T, N)
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    st = _stream()
    lib.call("csn_ga3_scan_fwd", _p(gens), _p(dt), _p(x), None, _p(h), B, T, N, _p(ws), nb, st)
    lib.call("csn_ga3_scan_bwd", _p(gens), _p(dt), None, _p(h), _p(dh), _p(dgens), _p(ddt), _p(dx), None,
             B, T, N, _p(ws), nb, st)
    torch.cuda.synchronize()
    rows = np.array([3, 40])
    a = {k: _subset(v, rows) for k, v in dict(gens=gens, dt=dt, x=x, dh=dh).items()}
    hr = oracle.ga3_scan_fwd(a["gens"], a["dt"], a["x"])
    dg, ddt_r, dx_r, _ = oracle.ga3_scan_bwd(a["gens"], a["dt"], hr, a["dh"])
    assert rel(h[rows][:, :8192], hr[:, :8192]) < 1e-4
    assert rel(h[rows], hr) < 1e-4
    assert rel(dx[rows], dx_r) < 1e-3
    assert rel(dgens[rows], dg) < 1e-3
    assert rel(ddt[rows], ddt_r) < 1e-3
