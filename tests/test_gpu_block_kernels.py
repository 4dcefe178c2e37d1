"""GPU parity of the block kernels around the scan (through the C ABI) against the PyTorch
formulation of the reference:

* state spike: torch.norm over the D x D state + the reference's SurrogateSpikeFunction
  (python/clifford_scan.py:90-116), forward and gradient, float64 torch reference;
* LayerNorm: F.layer_norm forward and gradients (input, weight, bias), float64 torch reference.

Tolerances (max|a - ref| / max|ref|): 1e-5 forward, 1e-4 gradients (fp32 kernels).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, ref):
    a, ref = a.detach().double().cpu(), ref.detach().double().cpu()
    den = ref.abs().max().item()
    err = (a - ref).abs().max().item()
    return err / den if den > 0 else err


@pytest.fixture(scope="module")
def ops():
    from csn_b200 import _build, ops as o
    _build.build()
    return o


def reference_spike(X, thr, beta):
    from python.clifford_scan import SurrogateSpikeFunction
    energy = torch.norm(X, dim=(-1, -2), keepdim=True)
    return X * SurrogateSpikeFunction.apply(energy - thr, beta)


@pytest.mark.parametrize("D", [4, 8, 16])
@pytest.mark.parametrize("n", [1, 7, 33, 1000])
def test_state_spike_matches_reference(ops, D, n):
    rng = np.random.default_rng(D * 1000 + n)
    # energies spread around the threshold; a few all-zero states (norm gradient 0 there)
    X = rng.standard_normal((n, D, D)) * rng.uniform(0.0, 2.0 / D, (n, 1, 1))
    X[::5] = 0.0
    W = rng.standard_normal((n, D, D))
    thr, beta = 0.1 * D / 4, 10.0
    x64 = torch.tensor(X, dtype=torch.float64, device=DEV, requires_grad=True)
    ref = reference_spike(x64, thr, beta)
    (ref * torch.tensor(W, dtype=torch.float64, device=DEV)).sum().backward()
    # keep states whose energy is more than 1e-5 from the threshold (an fp32 energy within
    # rounding of it may fall on the other side)
    e = np.sqrt((X ** 2).sum((-1, -2)))
    keep = torch.tensor(np.abs(e - thr) > 1e-5, device=DEV)
    x = torch.tensor(X, dtype=torch.float32, device=DEV, requires_grad=True)
    got = ops.state_spike(x, thr, beta)
    (got * torch.tensor(W, dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(got[keep], ref[keep]) < 1e-5
    assert rel(x.grad[keep], x64.grad[keep]) < 1e-4
    assert torch.count_nonzero(got[::5]) == 0 and torch.count_nonzero(x.grad[::5]) == 0


def test_state_spike_batched_shape_and_dtype(ops):
    X = torch.randn(2, 3, 5, 8, 8, device=DEV, dtype=torch.float64) * 0.05
    Y = ops.state_spike(X, 0.1, 10.0)
    assert Y.shape == X.shape and Y.dtype == torch.float64
    with pytest.raises(ValueError):
        ops.state_spike(torch.zeros(3, 8, 4, device=DEV))


@pytest.mark.parametrize("C", [4, 48, 128, 256, 640, 1024])
@pytest.mark.parametrize("R", [1, 37, 5000])
def test_layer_norm_matches_torch(ops, C, R):
    rng = np.random.default_rng(C * 7 + R)
    x = rng.standard_normal((R, C)) * 3.0 + 1.5
    w = rng.standard_normal(C)
    b = rng.standard_normal(C)
    dy = rng.standard_normal((R, C))
    t64 = [torch.tensor(a, dtype=torch.float64, device=DEV, requires_grad=True) for a in (x, w, b)]
    ref = torch.nn.functional.layer_norm(t64[0], (C,), t64[1], t64[2], 1e-5)
    (ref * torch.tensor(dy, dtype=torch.float64, device=DEV)).sum().backward()
    t32 = [torch.tensor(a, dtype=torch.float32, device=DEV, requires_grad=True) for a in (x, w, b)]
    got = ops.layer_norm(t32[0], t32[1], t32[2], 1e-5)
    (got * torch.tensor(dy, dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(got, ref) < 1e-5
    for a, r in zip(t32, t64):
        assert rel(a.grad, r.grad) < 1e-4


def test_layer_norm_module_keeps_nn_layernorm_state(ops):
    from csn_b200.modules import LayerNorm
    m = LayerNorm(96).to(DEV)
    ref = torch.nn.LayerNorm(96).to(DEV)
    assert set(m.state_dict()) == set(ref.state_dict())
    with torch.no_grad():
        m.weight.normal_()
        m.bias.normal_()
    ref.load_state_dict(m.state_dict())
    x = torch.randn(4, 9, 96, device=DEV)
    assert rel(m(x), ref(x)) < 1e-5
    odd = LayerNorm(6).to(DEV)  # C % 4 != 0: F.layer_norm
    assert odd(torch.randn(2, 6, device=DEV)).shape == (2, 6)


def test_layer_norm_rejects_unsupported_sizes(ops):
    from csn_b200 import _lib
    with pytest.raises(ValueError):
        ops.layer_norm(torch.zeros(2, 6, device=DEV), torch.ones(6, device=DEV), torch.zeros(6, device=DEV))
    with pytest.raises(_lib.CsnError, match="UNSUPPORTED"):
        x = torch.zeros(2, 2048, device=DEV)
        _lib.call("csn_layer_norm_fwd", ops._ptr(x), ops._ptr(x), ops._ptr(x), ops._ptr(x), ops._ptr(x),
                  ops._ptr(x), 2, 2048, 1e-5, ops._stream(x.device))


def reference_conv_input(x, lw, lb, cw, cb, eps):
    T = x.shape[1]
    ln = torch.nn.functional.layer_norm(x, (x.shape[-1],), lw, lb, eps)
    u = torch.nn.functional.conv1d(ln.transpose(1, 2), cw, cb, padding=cw.shape[-1] - 1, groups=x.shape[-1])
    return torch.nn.functional.silu(u[:, :, :T].transpose(1, 2))


@pytest.mark.parametrize("C", [4, 48, 128, 256])
@pytest.mark.parametrize("K", [1, 2, 3, 4])
@pytest.mark.parametrize("BT", [(1, 1), (2, 3), (3, 100), (2, 2048)], ids=lambda s: f"B{s[0]}T{s[1]}")
def test_ln_conv_silu_matches_torch_chain(ops, C, K, BT):
    """ln -> causal depthwise conv (left padding K - 1, first T outputs) -> SiLU of the blocks
    (python/clifford_cl6.py:140-142): output and the gradients of x, both LayerNorm parameters
    and both conv parameters, against the float64 torch chain."""
    B, T = BT
    rng = np.random.default_rng(C * 100 + K * 10 + T)
    arrs = [rng.standard_normal((B, T, C)) * 2.0 + 0.5, rng.standard_normal(C), rng.standard_normal(C),
            rng.standard_normal((C, 1, K)) * 0.5, rng.standard_normal(C) * 0.3]
    dy = rng.standard_normal((B, T, C))
    t64 = [torch.tensor(a, dtype=torch.float64, device=DEV, requires_grad=True) for a in arrs]
    ref = reference_conv_input(*t64, 1e-5)
    (ref * torch.tensor(dy, dtype=torch.float64, device=DEV)).sum().backward()
    t32 = [torch.tensor(a, dtype=torch.float32, device=DEV, requires_grad=True) for a in arrs]
    got = ops.ln_conv_silu(t32[0], t32[1], t32[2], 1e-5, t32[3], t32[4])
    (got * torch.tensor(dy, dtype=torch.float32, device=DEV)).sum().backward()
    assert got.shape == (B, T, C)
    assert rel(got, ref) < 1e-5
    for name, a, r in zip(("x", "ln_w", "ln_b", "conv_w", "conv_b"), t32, t64):
        assert rel(a.grad, r.grad) < 1e-4, name


def test_causal_conv_input_module_path(ops):
    """The blocks' helper takes the fused kernels for the block layers and the library chain for
    layers outside the kernels' range, with the same result."""
    from csn_b200.modules import LayerNorm, causal_conv_input
    torch.manual_seed(0)
    for C, K in ((64, 4), (6, 4), (320, 4), (64, 5)):
        ln = LayerNorm(C).to(DEV)
        conv = torch.nn.Conv1d(C, C, K, padding=K - 1, groups=C).to(DEV)
        x = torch.randn(2, 17, C, device=DEV)
        ref = reference_conv_input(x.double(), ln.weight.double(), ln.bias.double(), conv.weight.double(),
                                   conv.bias.double(), ln.eps)
        assert rel(causal_conv_input(ln, conv, x), ref) < 1e-5


def reference_action(biv, dt, D):
    """The reference's terms on the explicit Omega (python/clifford_cl6.py:257-262)."""
    from python.clifford_cl6 import skew_from_generators
    u, v = torch.triu_indices(D, D, offset=1, device=biv.device)
    dtb = dt.reshape(*dt.shape, *([1] * (biv.dim() - dt.dim())))
    Omega = skew_from_generators(biv, D, u, v) * (0.5 * dtb)[..., None]
    kin = (Omega ** 2).mean()
    smooth = ((Omega[:, 1:] - Omega[:, :-1]) ** 2).mean() if biv.shape[1] > 1 else torch.zeros((), device=biv.device,
                                                                                                 dtype=biv.dtype)
    return kin, smooth


@pytest.mark.parametrize("case", ["cl6", "cl8", "heads", "T1", "cl6_long"])
def test_generator_action_matches_omega_form(ops, case):
    rng = np.random.default_rng(len(case) * 31 + ord(case[-1]))
    if case == "cl6":
        biv, dt, D = rng.standard_normal((3, 17, 8, 28)) * 5, rng.uniform(0.02, 0.08, (3, 17)), 8
    elif case == "cl6_long":
        biv, dt, D = rng.standard_normal((4, 2048, 8, 28)) * 5, rng.uniform(0.02, 0.08, (4, 2048)), 8
    elif case == "cl8":
        biv, dt, D = rng.standard_normal((2, 9, 2, 120)) * 5, rng.uniform(0.02, 0.08, (2, 9)), 16
    elif case == "heads":
        biv, dt, D = rng.standard_normal((2, 11, 3, 2, 28)) * 5, rng.uniform(0.02, 0.08, (2, 11, 3)), 8
    else:
        biv, dt, D = rng.standard_normal((2, 1, 4, 28)) * 5, rng.uniform(0.02, 0.08, (2, 1)), 8
    wk, ws = 0.7, -1.3
    b64 = torch.tensor(biv, dtype=torch.float64, device=DEV, requires_grad=True)
    d64 = torch.tensor(dt, dtype=torch.float64, device=DEV, requires_grad=True)
    rk, rs = reference_action(b64, d64, D)
    (wk * rk + ws * rs).backward()
    b32 = torch.tensor(biv, dtype=torch.float32, device=DEV, requires_grad=True)
    d32 = torch.tensor(dt, dtype=torch.float32, device=DEV, requires_grad=True)
    gk, gs = ops.generator_action(b32, d32, D)
    (wk * gk + ws * gs).backward()
    assert abs(gk.item() - rk.item()) <= 1e-5 * abs(rk.item())
    assert abs(gs.item() - rs.item()) <= 1e-5 * max(abs(rs.item()), 1e-30)
    assert rel(b32.grad, b64.grad) < 1e-5
    assert rel(d32.grad, d64.grad) < 1e-5
    # only one of the two terms in the loss
    b32.grad = None
    d32.grad = None
    ops.generator_action(b32, d32, D)[0].backward()
    b64.grad = None
    d64.grad = None
    reference_action(b64, d64, D)[0].backward()
    assert rel(b32.grad, b64.grad) < 1e-5 and rel(d32.grad, d64.grad) < 1e-5


@pytest.mark.parametrize("N,K,HT", [(8, 28, 1), (2, 120, 1), (6, 28, 3)])
def test_projection_epilogue_matches_torch(ops, N, K, HT):
    """biv * omega_scale, softplus(gamma), softplus(time) * dt_base on the fused projection output
    (python/clifford_cl6.py:144-155), forward and gradients, including raw values above
    softplus's threshold of 20."""
    rng = np.random.default_rng(N * 7 + K + HT)
    R = 333
    raw = rng.standard_normal((3, R, N * K + N + HT)) * 4.0
    raw[0, :5] = 25.0
    scale = rng.standard_normal((N, 1)) * 3.0
    gb, gg, gd = (rng.standard_normal(s) for s in ((3, R, N * K), (3, R, N), (3, R, HT)))
    F = torch.nn.functional
    r64 = torch.tensor(raw, dtype=torch.float64, device=DEV, requires_grad=True)
    s64 = torch.tensor(scale, dtype=torch.float64, device=DEV, requires_grad=True)
    biv = (r64[..., :N * K].reshape(3, R, N, K) * s64).reshape(3, R, N * K)
    gam = F.softplus(r64[..., N * K:N * K + N])
    dt = F.softplus(r64[..., N * K + N:]) * 0.05
    loss = sum((a * torch.tensor(g, dtype=torch.float64, device=DEV)).sum() for a, g in ((biv, gb), (gam, gg), (dt, gd)))
    loss.backward()
    r32 = torch.tensor(raw, dtype=torch.float32, device=DEV, requires_grad=True)
    s32 = torch.tensor(scale, dtype=torch.float32, device=DEV, requires_grad=True)
    ob, og, od = ops.projection_epilogue(r32, s32, 0.05, N, K, HT)
    loss32 = sum((a * torch.tensor(g, dtype=torch.float32, device=DEV)).sum() for a, g in ((ob, gb), (og, gg), (od, gd)))
    loss32.backward()
    for a, r in ((ob, biv), (og, gam), (od, dt)):
        assert rel(a, r) < 1e-6
    assert rel(r32.grad, r64.grad) < 1e-5
    assert rel(s32.grad, s64.grad) < 1e-5


@pytest.mark.parametrize("R,C", [(1, 1), (7, 3), (65536, 224), (1000, 512)])
def test_column_sum_is_deterministic_and_exact(ops, R, C):
    rng = np.random.default_rng(R + C)
    x = rng.standard_normal((R, C))
    got = ops.column_sum(torch.tensor(x, dtype=torch.float32, device=DEV))
    assert rel(got, torch.tensor(x.sum(0))) < 1e-5
    assert torch.equal(got, ops.column_sum(torch.tensor(x, dtype=torch.float32, device=DEV)))


def test_linear_matches_torch_linear(ops):
    torch.manual_seed(0)
    x = torch.randn(4, 50, 128, device=DEV, dtype=torch.float64)
    W = torch.randn(233, 128, device=DEV, dtype=torch.float64)
    b = torch.randn(233, device=DEV, dtype=torch.float64)
    dy = torch.randn(4, 50, 233, device=DEV, dtype=torch.float64)
    ts = [t.clone().requires_grad_(True) for t in (x, W, b)]
    (torch.nn.functional.linear(*ts) * dy).sum().backward()
    us = [t.float().clone().requires_grad_(True) for t in (x, W, b)]
    y = ops.linear(*us)
    (y * dy.float()).sum().backward()
    assert rel(y, torch.nn.functional.linear(x, W, b)) < 1e-5
    for a, r in zip(us, ts):
        assert rel(a.grad, r.grad) < 1e-5


@pytest.mark.parametrize("F_", [1, 256, 100])
def test_silu_gate_matches_torch(ops, F_):
    rng = np.random.default_rng(F_)
    gu = rng.standard_normal((3, 77, 2 * F_)) * 3
    dy = rng.standard_normal((3, 77, F_))
    g64 = torch.tensor(gu, dtype=torch.float64, device=DEV, requires_grad=True)
    ref = torch.nn.functional.silu(g64[..., :F_]) * g64[..., F_:]
    (ref * torch.tensor(dy, dtype=torch.float64, device=DEV)).sum().backward()
    g32 = torch.tensor(gu, dtype=torch.float32, device=DEV, requires_grad=True)
    got = ops.silu_gate(g32)
    (got * torch.tensor(dy, dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(got, ref) < 1e-6
    assert rel(g32.grad, g64.grad) < 1e-5
