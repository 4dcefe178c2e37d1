"""torch.ops.csn.* on the GPU: same values and gradients as csn_b200.ops, and the
registrations pass torch.library.opcheck (schema, fake implementation, autograd)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def mods():
    from csn_b200 import _build, ops
    _build.build()
    return ops, torch.ops.csn


def _t(rng, *shape, scale=1.0, grad=True):
    return torch.tensor(rng.standard_normal(shape) * scale, dtype=torch.float32, device=DEV,
                        requires_grad=grad)


def _grads(out, W, inputs):
    return torch.autograd.grad((out * W).sum(), [i for i in inputs if i is not None])


def test_scan_and_rotor_ops_match_the_autograd_functions(mods):
    ops, csn = mods
    rng = np.random.default_rng(0)
    B, T, N, D = 2, 33, 3, 8
    M = (0.3 * _t(rng, B, T, N, D, D, grad=False)).requires_grad_(True)
    C, h0 = _t(rng, B, T, N, D, D), _t(rng, B, N, D, D)
    W = _t(rng, B, T, N, D, D, grad=False)
    for rev in (False, True):
        a = ops.rotor_scan(M, C, True, h0, reverse=rev)
        b = csn.scan_fwd(M, C, h0, True, rev)
        assert torch.equal(a, b)
        for ga, gb in zip(_grads(a, W, [M, C, h0]), _grads(b, W, [M, C, h0])):
            assert torch.equal(ga, gb)
    gens, dt = _t(rng, B, T, N, 28), torch.rand(B, T, device=DEV).mul(0.09).add(0.01).requires_grad_(True)
    gamma, S = torch.rand(B, T, N, device=DEV).requires_grad_(True), _t(rng, B, T, N, D, D)
    a = ops.fused_rotor_scan(gens, dt, gamma, S, h0=h0)
    b = csn.fused_rotor_scan_fwd(gens, dt, gamma, S, h0, 0, True)
    assert torch.equal(a, b)
    # the op's backward reuses the chunk rotor products of its forward (products formed as M P);
    # the functional operator rebuilds them (P M): equal up to fp32 rounding
    for ga, gb in zip(_grads(a, W, [gens, dt, gamma, S, h0]), _grads(b, W, [gens, dt, gamma, S, h0])):
        assert ((ga - gb).abs().max() / gb.abs().max()).item() < 1e-5


def test_cayley_cell_ga3_ops_match(mods):
    ops, csn = mods
    rng = np.random.default_rng(1)
    A = _t(rng, 5, 16, 16, scale=0.3, grad=False)
    Om = (A - A.transpose(-1, -2)).requires_grad_(True)
    W = _t(rng, 5, 16, 16, grad=False)
    a, b = ops.cayley(Om), csn.cayley_fwd(Om)
    assert torch.equal(a, b)
    assert torch.equal(_grads(a, W, [Om])[0], _grads(b, W, [Om])[0])
    x, prev = _t(rng, 4, 3), _t(rng, 4, 5, 16)
    Wr, Wi, gb = _t(rng, 5, 5, 16, scale=0.3), _t(rng, 5, 3, 16, scale=0.3), _t(rng, 5)
    a, b = ops.cell_step(x, prev, Wr, Wi, gb, 0.05), csn.cell_fwd(x, prev, Wr, Wi, gb, 0.05)
    assert torch.equal(a, b)
    Wc = _t(rng, 4, 5, 16, grad=False)
    for ga, gb_ in zip(_grads(a, Wc, [x, prev, Wr, Wi, gb]), _grads(b, Wc, [x, prev, Wr, Wi, gb])):
        assert torch.equal(ga, gb_)
    g3, d3, x3 = _t(rng, 2, 40, 3, 3, scale=0.2), torch.rand(2, 40, device=DEV).requires_grad_(True), _t(rng, 2, 40, 3, 8)
    a, b = ops.ga3_rotor_scan(g3, d3, x3), csn.ga3_scan_fwd(g3, d3, x3, None)
    assert torch.equal(a, b)


def test_rotor_step_op_updates_in_place(mods):
    ops, csn = mods
    rng = np.random.default_rng(2)
    B, N, D = 3, 2, 8
    gens, dt = _t(rng, B, N, 28, grad=False), torch.full((B,), 0.05, device=DEV)
    S, h = _t(rng, B, N, D, D, grad=False), _t(rng, B, N, D, D, grad=False)
    h2 = h.clone()
    ops.rotor_step(gens, dt, None, S, h)
    csn.rotor_step(gens, dt, None, S, h2, 0, True)
    assert torch.equal(h, h2)


@pytest.mark.parametrize("case", ["scan", "rotor", "cayley", "ga3"])
def test_opcheck(mods, case):
    _, csn = mods
    rng = np.random.default_rng(3)
    if case == "scan":
        args = ((0.3 * _t(rng, 1, 9, 2, 4, 4, grad=False)).requires_grad_(True), _t(rng, 1, 9, 2, 4, 4),
                None, False, True)
        op = csn.scan_fwd
    elif case == "rotor":
        args = (_t(rng, 1, 9, 2, 28), torch.rand(1, 9, device=DEV).requires_grad_(True), None,
                _t(rng, 1, 9, 2, 8, 8), None, 0, True)
        op = csn.fused_rotor_scan_fwd
    elif case == "cayley":
        A = _t(rng, 3, 8, 8, scale=0.3, grad=False)
        args = ((A - A.transpose(-1, -2)).requires_grad_(True),)
        op = csn.cayley_fwd
    else:
        args = (_t(rng, 1, 9, 2, 3, scale=0.2), torch.rand(1, 9, device=DEV).requires_grad_(True),
                _t(rng, 1, 9, 2, 8), None)
        op = csn.ga3_scan_fwd
    torch.library.opcheck(op, args, test_utils=("test_schema", "test_autograd_registration",
                                                 "test_faketensor"))
