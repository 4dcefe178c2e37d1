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
