"""The bounded device-side waits of the bulk-copy kernels (mbarrier waits with a poll limit).

A wait that gives up sets a status bit instead of hanging the GPU.  The self-test entry point
arms a barrier phase that no copy completes, so its wait must give up; the status must then
read CSN_STATUS_WAIT_TIMEOUT, clear on reset, and the context must stay usable: a scan through
the bulk-copy kernels afterwards runs, matches the oracle and leaves the status at 0."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def lib():
    from csn_b200 import _build, _lib
    _build.build()
    assert torch.cuda.is_available()
    return _lib


def test_wait_that_never_completes_reports_a_timeout_and_the_context_stays_usable(lib, oracle):
    from csn_b200 import algebra, ops
    torch.cuda.synchronize()
    lib.device_status(reset=True)
    lib.call("csn_selftest_bounded_wait", 2000, None)
    assert lib.device_status(reset=True) == 1  # CSN_STATUS_WAIT_TIMEOUT
    assert lib.device_status(reset=False) == 0
    rng = np.random.default_rng(3)
    B, T, N, D = 2, 300, 3, 8
    E = algebra.triu_basis(D)
    gens = rng.standard_normal((B, T, N, 28)) * 3.0
    dt = rng.uniform(0.01, 0.1, (B, T))
    gamma = np.log1p(np.exp(rng.standard_normal((B, T, N))))
    S = rng.standard_normal((B, T, N, D, D))
    W = rng.standard_normal((B, T, N, D, D))
    t = lambda a: torch.tensor(a, dtype=torch.float32, device=DEV, requires_grad=True)
    tg, tdt, tga, tS = t(gens), t(dt), t(gamma), t(S)
    X = ops.fused_rotor_scan(tg, tdt, tga, tS)
    (X * torch.tensor(W, dtype=torch.float32, device=DEV)).sum().backward()
    Xr = oracle.rotor_scan_fwd(gens, dt, gamma, S, E)
    dg, *_ = oracle.rotor_scan_bwd(gens, dt, gamma, S, E, Xr, W)
    assert oracle.max_rel(tg.grad.double().cpu().numpy(), dg) < 1e-3
    assert lib.device_status(reset=True) == 0
