"""O(1)-state generation (config 4): stepping the recurrence one token at a time equals
the full scan, and the Cl(6) block's step() equals its forward() on the whole prefix."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, ref):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else a
    ref = ref.detach().double().cpu().numpy() if torch.is_tensor(ref) else ref
    return float(np.max(np.abs(a - ref)) / np.max(np.abs(ref)))


@pytest.fixture(scope="module")
def ops():
    from csn_b200 import _build, ops as o
    _build.build()
    return o


@pytest.mark.parametrize("D,basis,damped", [(8, "triu", True), (8, "triu", False), (4, "ga", False),
                                            (16, "triu", True)])
def test_stepping_equals_scan_and_oracle(ops, oracle, D, basis, damped):
    """256 streams x 8 channels (config 4 shape) for D = 8; fewer steps for the others."""
    from csn_b200 import algebra
    B, N, T = (256, 8, 2048) if D == 8 else (8, 2, 300)
    E = algebra.triu_basis(D) if basis == "triu" else algebra.bivector_basis(algebra.CL3)
    rng = np.random.default_rng(D + damped)
    gens = rng.standard_normal((B, T, N, E.shape[0])) * 0.1 * (10 if D == 4 else 1)
    dt = rng.uniform(0.01, 0.1, (B, T))
    gamma = np.log1p(np.exp(rng.standard_normal((B, T, N)))) if damped else None
    S = rng.standard_normal((B, T, N, D, D))
    tg = torch.tensor(gens, dtype=torch.float32, device=DEV)
    tdt = torch.tensor(dt, dtype=torch.float32, device=DEV)
    tga = torch.tensor(gamma, dtype=torch.float32, device=DEV) if damped else None
    tS = torch.tensor(S, dtype=torch.float32, device=DEV)
    h = torch.zeros(B, N, D, D, device=DEV)
    traj = []
    for t in range(T):
        ops.rotor_step(tg[:, t].contiguous(), tdt[:, t].contiguous(),
                       None if tga is None else tga[:, t].contiguous(), tS[:, t].contiguous(), h, basis)
        if t % 97 == 0 or t == T - 1:
            traj.append((t, h.clone()))
    X = ops.fused_rotor_scan(tg, tdt, tga, tS, basis=basis)
    for t, ht in traj:
        assert rel(ht, X[:, t]) < 1e-4
    if D == 8:  # oracle on a slice of the streams (sequences are independent)
        Xr = oracle.rotor_scan_fwd(gens[:16], dt[:16], None if gamma is None else gamma[:16], S[:16], E)
        assert rel(traj[-1][1][:16], Xr[:, -1]) < 1e-4


@pytest.mark.parametrize("B,N", [(1, 1), (3, 5), (7, 3), (33, 9)])  # partial 8-lane groups / CTAs
@pytest.mark.parametrize("damped", [True, False], ids=["damped", "undamped"])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
def test_d8_step_ragged_state_counts_match_oracle_and_scan(ops, oracle, B, N, damped, two):
    """The D = 8 step kernel runs 16 states per CTA, 8 lanes per state: state counts that
    leave part of a warp or a CTA idle, from a random initial state, against one oracle step
    and against the scan's T = 1 path with the same h0 (no state outside [B, N] written)."""
    from csn_b200 import algebra
    D = 8
    E = algebra.triu_basis(D)
    rng = np.random.default_rng(100 * B + N + 2 * damped + two)
    gens = rng.standard_normal((B, 1, N, 28)) * 0.3
    dt = rng.uniform(0.01, 0.1, (B, 1))
    gamma = np.log1p(np.exp(rng.standard_normal((B, 1, N)))) if damped else None
    S = rng.standard_normal((B, 1, N, D, D))
    h0 = rng.standard_normal((B, N, D, D))
    t = lambda a: torch.tensor(a, dtype=torch.float32, device=DEV)
    # the state sits inside a larger buffer: the guard entries after it must stay untouched
    buf = torch.full((B * N * D * D + 64,), 7.0, device=DEV)
    h = buf[:B * N * D * D].view(B, N, D, D)
    h.copy_(t(h0))
    ops.rotor_step(t(gens[:, 0]), t(dt[:, 0]), None if gamma is None else t(gamma[:, 0]), t(S[:, 0]), h,
                   two_sided=two)
    assert torch.all(buf[B * N * D * D:] == 7.0)
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E, h0=h0, two_sided=two)[:, 0]
    assert rel(h, Xr) < 1e-5
    X = ops.fused_rotor_scan(t(gens), t(dt), None if gamma is None else t(gamma), t(S), h0=t(h0),
                             two_sided=two)
    assert rel(h, X[:, 0]) < 1e-6


@pytest.mark.parametrize("D", [4, 8, 16])
@pytest.mark.parametrize("chained", [True, False])
def test_step_graph_matches_step_loop(ops, chained, D):
    """A captured chain of steps (chained: each step's rotor built while the previous step
    runs, the state read after it completes; for D = 4 and 16 the chained entry point launches
    as the plain one) equals the same steps launched one by one."""
    B, N, steps = (256, 8, 64) if D == 8 else (16, 4, 16)
    K = D * (D - 1) // 2
    g = ops.RotorStepGraph(B, N, D, steps=steps, damped=True, chained=chained)
    gen = torch.Generator(device="cpu").manual_seed(0)
    g.gens.copy_(torch.randn(steps, B, N, K, generator=gen) * 0.1)
    g.dt.copy_(torch.rand(steps, B, generator=gen) * 0.09 + 0.01)
    g.gamma.copy_(torch.rand(steps, B, N, generator=gen))
    g.S.copy_(torch.randn(steps, B, N, D, D, generator=gen))
    g.h.zero_()
    hg = g.replay().clone()
    h = torch.zeros(B, N, D, D, device=DEV)
    for t in range(steps):
        ops.rotor_step(g.gens[t], g.dt[t], g.gamma[t], g.S[t], h)
    assert torch.equal(hg, h)


def test_cl6_block_step_equals_forward(ops):
    from python.clifford_cl6 import CliffordCL6Block
    torch.manual_seed(0)
    blk = CliffordCL6Block(32, num_neurons=4).to(DEV).eval()
    with torch.no_grad():
        blk.time_head.proj.weight.normal_(0, 0.1)
    x = torch.randn(3, 40, 32, device=DEV)
    with torch.no_grad():
        out_full, _, _ = blk(x)
        state = blk.init_state(3)
        outs = []
        for t in range(40):
            o, state = blk.step(x[:, t], state)
            outs.append(o)
    assert rel(torch.stack(outs, 1), out_full) < 1e-4
