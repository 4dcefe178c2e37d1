"""GPU parity of the CUDA scans (through the C ABI) against the float64 oracle and
the reference's golden vectors.

Tolerances (reference metric max|a - ref| / max|ref|,
csn_toolkit/examples/benchmark_cuda_kernels.py:60-62):
  forward outputs  <= 1e-4   (BASELINE: fp32 over L = 8192 vs the fp64 oracle)
  gradients        <= 1e-3   (the reference's own gradient tolerance, same file :75-77)
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
BWD_TOL = 1e-3
DEV = "cuda:0"


def rel(a, ref):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(a - ref)) / den) if den > 0 else float(np.max(np.abs(a - ref)))


def cuda(a, grad=False):
    t = torch.as_tensor(np.asarray(a), dtype=torch.float32, device=DEV)
    return t.requires_grad_(grad)


def transitions(rng, B, T, N, D):
    A = rng.standard_normal((B, T, N, D, D)) * 0.4
    skew = 0.5 * (A - np.swapaxes(A, -1, -2))
    eye = np.eye(D)
    Q = np.linalg.solve(eye - skew, eye + skew)
    return rng.uniform(0.6, 1.0, (B, T, N, 1, 1)) * Q + 0.05 * rng.standard_normal((B, T, N, D, D))


@pytest.fixture(scope="module")
def ops():
    from csn_b200 import _build, ops as o
    _build.build()
    assert torch.cuda.is_available()
    return o


# ----------------------------------------------------------------- plain scan
SHAPES = [(2, 37, 3), (1, 1, 2), (1, 300, 2), (3, 129, 5)]


@pytest.mark.parametrize("D", [4, 8, 16])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_h0", [False, True], ids=["zero", "h0"])
def test_scan_matches_oracle(ops, oracle, D, two, shape, with_h0):
    rng = np.random.default_rng(hash((D, two, shape, with_h0)) % 2**32)
    B, T, N = shape
    M = transitions(rng, B, T, N, D)
    C = rng.standard_normal((B, T, N, D, D))
    W = rng.standard_normal((B, T, N, D, D))
    h0 = rng.standard_normal((B, N, D, D)) if with_h0 else None
    Xr = oracle.scan_fwd(M, C, h0=h0, two_sided=two)
    dMr, dCr, dh0r = oracle.scan_bwd(M, Xr, W, h0=h0, two_sided=two)

    Mt, Ct = cuda(M, True), cuda(C, True)
    ht = cuda(h0, True) if with_h0 else None
    X = ops.rotor_scan(Mt, Ct, two_sided=two, h0=ht)
    assert rel(X, Xr) < FWD_TOL
    (X * cuda(W)).sum().backward()
    assert rel(Ct.grad, dCr) < BWD_TOL
    assert rel(Mt.grad, dMr) < BWD_TOL
    if with_h0:
        assert rel(ht.grad, dh0r) < BWD_TOL


@pytest.mark.parametrize("name", ["two_d4_T37", "two_d8_T23", "two_d16_T19", "one_d4_T37",
                                  "one_d8_T23", "one_d16_T19", "two_d8_T1", "one_d4_T1"])
def test_scan_matches_reference_golden(ops, golden, name):
    g = golden(f"scan_{name}")
    two = name.startswith("two")
    M, C = cuda(g["M"], True), cuda(g["C"], True)
    X = ops.rotor_scan(M, C, two_sided=two)
    assert rel(X, g["X"]) < FWD_TOL
    (X * cuda(g["W"])).sum().backward()
    assert rel(C.grad, g["dC"]) < BWD_TOL
    ref_dM = g["dM"] if g["dM"].shape == tuple(M.shape) else np.zeros(M.shape)
    assert rel(M.grad, ref_dM) < BWD_TOL


# ------------------------------------------------------------------ Cayley
@pytest.mark.parametrize("D", [4, 8, 16])
def test_cayley_matches_reference_golden(ops, golden, D):
    g = golden(f"cayley_d{D}")
    Om = cuda(g["Om"], True)
    Q = ops.cayley(Om)
    assert rel(Q, g["Q"]) < FWD_TOL
    eye = torch.eye(D, device=DEV)
    assert (Q.transpose(-1, -2) @ Q - eye).abs().max().item() < 1e-5  # |R R~ - 1| <= 1e-5
    (Q * cuda(g["W"])).sum().backward()
    assert rel(Om.grad, g["dOm"]) < BWD_TOL


# -------------------------------------------------------------- fused rotor scan
ROTOR_GOLDEN = ["rotor_d8_damped", "rotor_d8_undamped", "rotor_d4_damped", "rotor_d16_damped",
                "rotor_d16_spinor", "rotor_cl8ga_undamped", "rotor_cl8ga_damped"]


@pytest.mark.parametrize("case", ROTOR_GOLDEN)
def test_fused_rotor_scan_matches_reference_golden(ops, golden, case):
    g = golden(case)
    basis = "ga" if "cl8ga" in case else "triu"
    gens, dt, S = cuda(g["gens"], True), cuda(g["dt"], True), cuda(g["S"], True)
    gamma = cuda(g["gamma"], True) if "gamma" in g else None
    X = ops.fused_rotor_scan(gens, dt, gamma, S, basis=basis, two_sided=not bool(g["spinor"]))
    assert rel(X, g["X"]) < FWD_TOL
    (X * cuda(g["W"])).sum().backward()
    assert rel(S.grad, g["dS"]) < BWD_TOL
    assert rel(gens.grad, g["dgens"]) < BWD_TOL
    assert rel(dt.grad, g["ddt"]) < BWD_TOL
    if gamma is not None:
        assert rel(gamma.grad, g["dgamma"]) < BWD_TOL


def _rotor_case(rng, B, T, N, D, basis, damped, gscale=1.0):
    from csn_b200 import algebra
    if basis == "triu":
        E = algebra.triu_basis(D)
    else:
        E = algebra.bivector_basis(algebra.CL3 if D == 4 else algebra.CL8)
    K = E.shape[0]
    gens = rng.standard_normal((B, T, N, K)) * gscale
    dt = rng.uniform(0.01, 0.1, (B, T))
    gamma = np.log1p(np.exp(rng.standard_normal((B, T, N)))) if damped else None
    S = rng.standard_normal((B, T, N, D, D))
    return E, gens, dt, gamma, S


@pytest.mark.parametrize("D,basis", [(4, "triu"), (4, "ga"), (8, "triu"), (16, "triu"), (16, "ga")])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_fused_rotor_scan_matches_oracle(ops, oracle, D, basis, damped, two):
    rng = np.random.default_rng(hash((D, basis, damped, two)) % 2**32)
    B, T, N = (2, 150, 3) if D < 16 else (1, 70, 2)
    E, gens, dt, gamma, S = _rotor_case(rng, B, T, N, D, basis, damped, gscale=8.0)
    h0 = rng.standard_normal((B, N, D, D))
    W = rng.standard_normal((B, T, N, D, D))
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E, h0=h0, two_sided=two)
    dg, ddt, dgam, dS, dh0 = oracle.rotor_scan_bwd(gens, dt, gamma, S, E, Xr, W, h0=h0, two_sided=two)
    tg, tdt, tS, th0 = cuda(gens, True), cuda(dt, True), cuda(S, True), cuda(h0, True)
    tgam = cuda(gamma, True) if damped else None
    X = ops.fused_rotor_scan(tg, tdt, tgam, tS, basis=basis, two_sided=two, h0=th0)
    assert rel(X, Xr) < FWD_TOL
    (X * cuda(W)).sum().backward()
    assert rel(tS.grad, dS) < BWD_TOL
    assert rel(tg.grad, dg) < BWD_TOL
    assert rel(tdt.grad, ddt) < BWD_TOL
    assert rel(th0.grad, dh0) < BWD_TOL
    if damped:
        assert rel(tgam.grad, dgam) < BWD_TOL


@pytest.mark.parametrize("basis", ["triu", "ga"])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_d16_cayley_over_generator_norms(ops, oracle, basis, damped, two):
    """D = 16 Cayley inverse (Gauss-Jordan on the fragment) at generator norms from tiny to
    large: every (step, channel) generator is scaled to a target |h Omega|_F cycling through
    0.02 / 0.07 / 2.0 inside every chunk of the forward and backward passes."""
    rng = np.random.default_rng(11 + 2 * (basis == "ga") + 4 * damped + 8 * two)
    B, T, N = 1, 96, 2
    E, gens, dt, gamma, S = _rotor_case(rng, B, T, N, 16, basis, damped, gscale=1.0)
    fro = lambda t, n: np.linalg.norm(0.5 * dt[0, t] * np.einsum("k,kij->ij", gens[0, t, n], E))
    target = np.array([0.02, 0.07, 2.0])
    for t in range(T):
        for n in range(N):
            gens[0, t, n] *= target[(t + n) % 3] / fro(t, n)
    got = np.array([[fro(t, n) for n in range(N)] for t in range(T)])
    assert np.allclose(got, target[(np.arange(T)[:, None] + np.arange(N)[None, :]) % 3], rtol=1e-6)
    W = rng.standard_normal((B, T, N, 16, 16))
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E, two_sided=two)
    dg, ddt, dgam, dS, _ = oracle.rotor_scan_bwd(gens, dt, gamma, S, E, Xr, W, two_sided=two)
    tg, tdt, tS = cuda(gens, True), cuda(dt, True), cuda(S, True)
    tgam = cuda(gamma, True) if damped else None
    X = ops.fused_rotor_scan(tg, tdt, tgam, tS, basis=basis, two_sided=two)
    assert rel(X, Xr) < FWD_TOL
    (X * cuda(W)).sum().backward()
    assert rel(tS.grad, dS) < BWD_TOL
    assert rel(tg.grad, dg) < BWD_TOL
    assert rel(tdt.grad, ddt) < BWD_TOL
    if damped:
        assert rel(tgam.grad, dgam) < BWD_TOL


def test_fused_matches_materialised_transitions(ops, oracle):
    """The fused kernel equals Cayley + decay + plain scan run separately."""
    rng = np.random.default_rng(7)
    E, gens, dt, gamma, S = _rotor_case(rng, 2, 64, 3, 8, "triu", True, gscale=5.0)
    M, C = oracle.rotor_build(gens, dt, gamma, S, E)
    X1 = ops.rotor_scan(cuda(M), cuda(C))
    X2 = ops.fused_rotor_scan(cuda(gens), cuda(dt), cuda(gamma), cuda(S))
    assert (X1 - X2).abs().max().item() / X1.abs().max().item() < 1e-5


# --------------------------------------------------------- long sequences (L = 8192)
@pytest.mark.parametrize("D,shape", [(8, (1, 8192, 2)), (16, (1, 8192, 1)), (4, (2, 8192, 2))])
def test_long_sequence_tolerance_L8192(ops, oracle, D, shape):
    """BASELINE tolerance: max-rel <= 1e-4 at fp32 over L = 8192 against fp64."""
    rng = np.random.default_rng(D)
    B, T, N = shape
    E, gens, dt, gamma, S = _rotor_case(rng, B, T, N, D, "triu", True, gscale=1.0)
    W = rng.standard_normal((B, T, N, D, D))
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E)
    dg, ddt, dgam, dS, _ = oracle.rotor_scan_bwd(gens, dt, gamma, S, E, Xr, W)
    tg, tdt, tgam, tS = cuda(gens, True), cuda(dt, True), cuda(gamma, True), cuda(S, True)
    X = ops.fused_rotor_scan(tg, tdt, tgam, tS)
    assert rel(X, Xr) < FWD_TOL
    (X * cuda(W)).sum().backward()
    for got, ref in ((tS.grad, dS), (tg.grad, dg), (tdt.grad, ddt), (tgam.grad, dgam)):
        assert rel(got, ref) < FWD_TOL


def test_undamped_orthogonal_scan_preserves_norm_L8192(ops):
    """Undamped two-sided scan with zero injection after t = 0 is a pure rotation:
    |X_t|_F stays |C_0|_F (orthogonal Cayley rotors), a size-independent invariant."""
    B, T, N, D = 2, 8192, 4, 8
    g = torch.Generator(device="cpu").manual_seed(0)
    gens = torch.randn(B, T, N, 28, generator=g).to(DEV)
    dt = torch.rand(B, T, generator=g).mul(0.09).add(0.01).to(DEV)
    S = torch.zeros(B, T, N, D, D, device=DEV)
    S[:, 0] = torch.randn(B, N, D, D, generator=g).to(DEV)
    X = ops.fused_rotor_scan(gens, dt, None, S)
    n0 = S[:, 0].flatten(2).norm(dim=-1)
    nT = X[:, -1].flatten(2).norm(dim=-1)
    assert ((nT - n0).abs() / n0).max().item() < 1e-4


@pytest.mark.parametrize("basis", ["triu", "ga"])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
@pytest.mark.parametrize("T", [6, 150])  # one chunk (apply stores the rotors) / many chunks
def test_d16_rotor_cache_matches_uncached_entry_points(ops, basis, damped, two, T):
    """csn_rotor_scan_{fwd,bwd}_cached (rotors stored once, reused by the other passes) give
    the results of the entry points that rebuild every rotor, and store M_t = sqrt(a) Q."""
    from csn_b200 import _lib
    rng = np.random.default_rng(31 + T + 2 * damped + 4 * two + 8 * (basis == "ga"))
    B, N = 2, 3
    from csn_b200 import algebra
    E = algebra.triu_basis(16) if basis == "triu" else algebra.bivector_basis(algebra.CL8)
    gens = cuda(rng.standard_normal((B, T, N, E.shape[0])) * np.where(rng.random((B, T, N, 1)) < 0.5, 0.05, 2.0))
    dt, S, dX = cuda(rng.uniform(0.01, 0.1, (B, T))), cuda(rng.standard_normal((B, T, N, 16, 16))), cuda(rng.standard_normal((B, T, N, 16, 16)))
    gamma = cuda(np.log1p(np.exp(rng.standard_normal((B, T, N))))) if damped else None
    h0 = cuda(rng.standard_normal((B, N, 16, 16)))
    bi = ops.BASIS[basis]
    X0 = ops._rotor_fwd(gens, dt, gamma, S, h0, bi, two)
    Mc = torch.empty_like(S)
    X1 = ops._rotor_fwd(gens, dt, gamma, S, h0, bi, two, Mc)
    assert rel(X1, X0.cpu().numpy()) < 1e-5
    # the stored rotors are the transitions of the plain scan
    C = S if gamma is None else S * (1.0 - torch.sigmoid(-gamma * dt[..., None]))[..., None, None]
    Xm = ops.rotor_scan(Mc, C, two_sided=two, h0=h0)
    assert rel(Xm, X0.cpu().numpy()) < 1e-4
    g0 = ops._rotor_bwd(gens, dt, gamma, S, h0, X0, dX, bi, two, True)
    g1 = ops._rotor_bwd(gens, dt, gamma, S, h0, X1, dX, bi, two, True, Mc)
    for a_, b_ in zip(g1, g0):
        if b_ is not None:
            assert rel(a_, b_.cpu().numpy()) < 1e-5
    # cached rotors together with the forward's chunk products (the autograd op's path)
    ws = torch.zeros(_lib.load().csn_rotor_scan_workspace_bytes(B, T, N, 16), dtype=torch.uint8, device=DEV)
    Mc2 = torch.empty_like(S)
    X2 = ops._rotor_fwd(gens, dt, gamma, S, h0, bi, two, Mc2, ws)
    g2 = ops._rotor_bwd(gens, dt, gamma, S, h0, X2, dX, bi, two, True, Mc2, ws)
    for a_, b_ in zip(g2, g0):
        if b_ is not None:
            assert rel(a_, b_.cpu().numpy()) < 1e-5
    with pytest.raises(_lib.CsnError, match="UNSUPPORTED"):
        s8 = cuda(rng.standard_normal((1, 4, 1, 8, 8)))
        ops._rotor_fwd(cuda(rng.standard_normal((1, 4, 1, 28))), cuda(np.full((1, 4), 0.05)), None, s8,
                       None, 0, True, torch.empty_like(s8))


def _heads_case(rng, B, T, H, Nh, D, basis, damped):
    E, gens, _, gamma, S = _rotor_case(rng, B, T, H * Nh, D, basis, damped, gscale=8.0)
    gens = gens.reshape(B, T, H, Nh, -1)
    gamma = gamma.reshape(B, T, H, Nh) if damped else None
    dt = rng.uniform(0.01, 0.1, (B, T, H))
    return E, gens, dt, gamma, S.reshape(B, T, H, Nh, D, D)


@pytest.mark.parametrize("D,basis", [(4, "triu"), (8, "triu"), (16, "ga")])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_heads_layout_matches_oracle_on_folded_heads(ops, oracle, D, basis, damped, two):
    """fused_rotor_scan_heads (one dt per head, [B, T, H, Nh, ...] read in place) against the
    oracle on the reference's fold of heads into the batch, [B*H, T, Nh]
    (python/clifford_multihead.py:157-170)."""
    rng = np.random.default_rng(hash(("heads", D, basis, damped, two)) % 2**32)
    B, T, H, Nh = (2, 150, 3, 2) if D < 16 else (1, 70, 2, 2)
    E, gens, dt, gamma, S = _heads_case(rng, B, T, H, Nh, D, basis, damped)
    h0 = rng.standard_normal((B, H, Nh, D, D))
    W = rng.standard_normal((B, T, H, Nh, D, D))

    def fold(a):
        return np.swapaxes(a, 1, 2).reshape(B * H, T, *a.shape[3:])

    def unfold(a):
        return np.swapaxes(a.reshape(B, H, T, *a.shape[2:]), 1, 2)

    h0f = h0.reshape(B * H, Nh, D, D)
    gf = fold(gamma) if damped else None
    Xr = oracle.rotor_scan_fwd(fold(gens), fold(dt), gf, fold(S), E, h0=h0f, two_sided=two)
    dg, ddt, dgam, dS, dh0 = oracle.rotor_scan_bwd(fold(gens), fold(dt), gf, fold(S), E, Xr, fold(W),
                                                   h0=h0f, two_sided=two)
    tg, tdt, tS, th0 = cuda(gens, True), cuda(dt, True), cuda(S, True), cuda(h0, True)
    tga = cuda(gamma, True) if damped else None
    X = ops.fused_rotor_scan_heads(tg, tdt, tga, tS, basis=basis, two_sided=two, h0=th0)
    assert X.shape == (B, T, H, Nh, D, D)
    assert rel(X, unfold(Xr)) < FWD_TOL
    (X * cuda(W)).sum().backward()
    assert rel(tg.grad, unfold(dg)) < BWD_TOL
    assert rel(tdt.grad, unfold(ddt)) < BWD_TOL
    assert rel(tS.grad, unfold(dS)) < BWD_TOL
    assert rel(th0.grad, dh0.reshape(B, H, Nh, D, D)) < BWD_TOL
    if damped:
        assert rel(tga.grad, unfold(dgam)) < BWD_TOL


@pytest.mark.parametrize("D,basis", [(4, "triu"), (8, "triu"), (16, "triu")])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_heads_layout_is_bit_identical_to_folded_entry_points(ops, D, basis, damped, two):
    """The multi-head entry points run the same per-sequence arithmetic, chunking and ddt
    summation order as the plain ones on the folded copies, so every output is bit-identical
    (forward, reusing backward for D = 4, 8, cached rotors for D = 16)."""
    rng = np.random.default_rng(hash(("heads-bits", D, damped, two)) % 2**32)
    B, T, H, Nh = (2, 300, 3, 2) if D < 16 else (1, 120, 2, 2)
    E, gens, dt, gamma, S = _heads_case(rng, B, T, H, Nh, D, basis, damped)
    g, d, s = cuda(gens), cuda(dt), cuda(S)
    ga = cuda(gamma) if damped else None
    h0 = cuda(rng.standard_normal((B, H, Nh, D, D)))
    dX = cuda(rng.standard_normal((B, T, H, Nh, D, D)))
    bi = ops.BASIS[basis]

    def fold(t):
        return None if t is None else t.transpose(1, 2).reshape(B * H, T, *t.shape[3:]).contiguous()

    def unfold(t):
        return None if t is None else t.reshape(B, H, T, *t.shape[2:]).transpose(1, 2)

    def state(Mc_like):
        if D == 16:
            return torch.empty_like(Mc_like), None
        return None, torch.zeros(ops._rotor_ws_bytes(Mc_like), dtype=torch.uint8, device=DEV)

    Mc_h, ws_h = state(s)
    Mc_f, ws_f = state(fold(s))
    Xh = ops._rotor_fwd(g, d, ga, s, h0, bi, two, Mc_h, ws_h)
    Xf = ops._rotor_fwd(fold(g), fold(d), fold(ga), fold(s), h0.reshape(B * H, Nh, D, D), bi, two, Mc_f, ws_f)
    assert torch.equal(Xh, unfold(Xf))
    if D == 16:
        assert torch.equal(Mc_h, unfold(Mc_f))
    gh = ops._rotor_bwd(g, d, ga, s, h0, Xh, dX, bi, two, True, Mc_h, ws_h)
    gf = ops._rotor_bwd(fold(g), fold(d), fold(ga), fold(s), h0.reshape(B * H, Nh, D, D), Xf, fold(dX), bi, two,
                        True, Mc_f, ws_f)
    names = ("dgens", "ddt", "dgamma", "dS")
    for name, a_, b_ in zip(names, gh[:4], gf[:4]):
        if b_ is not None:
            assert torch.equal(a_, unfold(b_)), name
    assert torch.equal(gh[4], gf[4].reshape(B, H, Nh, D, D))


def test_heads_layout_without_neurons_zeroes_ddt(ops):
    """Nh = 0: nothing to scan, and ddt [B, T, H] (the gradient of an unused dt) is zero."""
    from csn_b200 import _lib
    B, T, H, D = 2, 5, 3, 8
    g = torch.zeros(B, T, H, 0, 28, device=DEV)
    d = torch.full((B, T, H), 0.05, device=DEV)
    s = torch.zeros(B, T, H, 0, D, D, device=DEV)
    X = ops._rotor_fwd(g, d, None, s, None, 0, True)
    assert X.shape == s.shape
    ddt = torch.full_like(d, 7.0)
    _lib.call("csn_rotor_scan_heads_bwd", ops._ptr(g), ops._ptr(d), None, ops._ptr(s), None, ops._ptr(X),
              ops._ptr(X), None, ops._ptr(g), ops._ptr(ddt), None, ops._ptr(s), None, B, T, H, 0, D, 0, 1, 0,
              None, 0, ops._stream(d.device))
    torch.cuda.synchronize()
    assert torch.count_nonzero(ddt) == 0


@pytest.mark.parametrize("D,basis", [(4, "triu"), (8, "triu"), (16, "ga")])
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_backward_reusing_forward_workspace_matches(ops, D, basis, damped, two):
    """csn_rotor_scan_bwd_reuse on the forward's workspace (chunk rotor products taken from
    it) equals csn_rotor_scan_bwd on a fresh workspace."""
    from csn_b200 import _lib
    rng = np.random.default_rng(57 + D + 2 * damped + 4 * two)
    B, T, N = (2, 300, 3) if D < 16 else (1, 120, 2)
    E, gens, dt, gamma, S = _rotor_case(rng, B, T, N, D, basis, damped, gscale=2.0)
    g, d, s = cuda(gens), cuda(dt), cuda(S)
    ga = cuda(gamma) if damped else None
    h0, dX = cuda(rng.standard_normal((B, N, D, D))), cuda(rng.standard_normal((B, T, N, D, D)))
    bi = ops.BASIS[basis]
    ws = torch.zeros(_lib.load().csn_rotor_scan_workspace_bytes(B, T, N, D), dtype=torch.uint8, device=DEV)
    X = ops._rotor_fwd(g, d, ga, s, h0, bi, two, None, ws)
    ref = ops._rotor_bwd(g, d, ga, s, h0, X, dX, bi, two, True)
    for _ in range(2):  # the reused products survive a backward (aggP is only read)
        got = ops._rotor_bwd(g, d, ga, s, h0, X, dX, bi, two, True, None, ws)
        for a_, b_ in zip(got, ref):
            if b_ is not None:
                assert rel(a_, b_.cpu().numpy()) < 1e-5
