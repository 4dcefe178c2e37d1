"""Reverse-time plain scan and the 2D bidirectional spatial scan on the GPU.

* reverse=True equals flip(scan(flip(M), flip(C))) of the float64 oracle, forward and
  adjoint (the flipped scan of csn_toolkit/csn/vision.py:97-107).
* spatial_scan_2d equals the reference's flip / permute composition (vision.py:97-107),
  restated below in float64 PyTorch with a sequential one-sided scan, values and gradients.
* The drop-in CliffordSpatialRotorBlockCl4 / Cl8 reproduce the reference blocks' golden
  fixtures (tests/golden/spatial_cl*.npz, made by the reference modules in float64).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
FWD_TOL, BWD_TOL = 1e-4, 1e-3


def rel(a, ref):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a, dtype=np.float64)
    ref = ref.detach().double().cpu().numpy() if torch.is_tensor(ref) else np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(a - ref)) / den) if den > 0 else float(np.max(np.abs(a - ref)))


def transitions(rng, shape, D):
    A = rng.standard_normal((*shape, D, D)) * 0.4
    skew = 0.5 * (A - np.swapaxes(A, -1, -2))
    Q = np.linalg.solve(np.eye(D) - skew, np.eye(D) + skew)
    return rng.uniform(0.6, 1.0, (*shape, 1, 1)) * Q + 0.05 * rng.standard_normal((*shape, D, D))


@pytest.fixture(scope="module")
def ops():
    from csn_b200 import _build, ops as o
    _build.build()
    return o


@pytest.mark.parametrize("D", [4, 8, 16])
@pytest.mark.parametrize("two", [True, False], ids=["two", "one"])
@pytest.mark.parametrize("with_h0", [False, True], ids=["zero", "h0"])
def test_reverse_scan_matches_flipped_oracle(ops, oracle, D, two, with_h0):
    rng = np.random.default_rng(100 + D + 7 * two + 3 * with_h0)
    B, T, N = (2, 67, 3) if D < 16 else (1, 41, 2)
    M = transitions(rng, (B, T, N), D)
    C = rng.standard_normal((B, T, N, D, D))
    W = rng.standard_normal((B, T, N, D, D))
    h0 = rng.standard_normal((B, N, D, D)) if with_h0 else None
    f = lambda a: np.ascontiguousarray(a[:, ::-1])
    Xr = f(oracle.scan_fwd(f(M), f(C), h0=h0, two_sided=two))
    dMr, dCr, dh0r = oracle.scan_bwd(f(M), f(Xr), f(W), h0=h0, two_sided=two)
    tM = torch.tensor(M, dtype=torch.float32, device=DEV, requires_grad=True)
    tC = torch.tensor(C, dtype=torch.float32, device=DEV, requires_grad=True)
    th = torch.tensor(h0, dtype=torch.float32, device=DEV, requires_grad=True) if with_h0 else None
    X = ops.rotor_scan(tM, tC, two_sided=two, h0=th, reverse=True)
    assert rel(X, Xr) < FWD_TOL
    (X * torch.tensor(W, dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(tC.grad, f(dCr)) < BWD_TOL
    assert rel(tM.grad, f(dMr)) < BWD_TOL
    if with_h0:
        assert rel(th.grad, dh0r) < BWD_TOL


def _ref_scan64(M, C):
    """One-sided sequential scan X_t = M_t X_{t-1} + C_t over dim 1 (float64, autograd)."""
    out, X = [], torch.zeros_like(C[:, 0])
    for t in range(M.shape[1]):
        X = M[:, t] @ X + C[:, t]
        out.append(X)
    return torch.stack(out, 1)


def _ref_spatial64(M, C, H, W):
    """The reference's row / column bidirectional composition with flips and permutes."""
    B, L, N, D, _ = M.shape
    Mh, Ch = M.view(B * H, W, N, D, D), C.view(B * H, W, N, D, D)
    psi_h = (_ref_scan64(Mh, Ch) + _ref_scan64(Mh.flip(1), Ch.flip(1)).flip(1)) * 0.5
    perm = lambda a: a.view(B, H, W, N, D, D).permute(0, 2, 1, 3, 4, 5).reshape(B * W, H, N, D, D)
    Mv, Cv = perm(M), perm(psi_h)
    psi_v = (_ref_scan64(Mv, Cv) + _ref_scan64(Mv.flip(1), Cv.flip(1)).flip(1)) * 0.5
    return psi_v.view(B, W, H, N, D, D).permute(0, 2, 1, 3, 4, 5).reshape(B, L, N, D, D)


@pytest.mark.parametrize("D,shape", [(4, (2, 5, 7, 3)), (8, (1, 6, 4, 2)), (16, (1, 3, 5, 1))])
def test_spatial_scan_2d_matches_flip_permute_composition(D, shape):
    from csn_b200.spatial import spatial_scan_2d
    B, H, W, N = shape
    rng = np.random.default_rng(D)
    M = torch.tensor(transitions(rng, (B, H * W, N), D))
    C = torch.tensor(rng.standard_normal((B, H * W, N, D, D)))
    G = torch.tensor(rng.standard_normal((B, H * W, N, D, D)))
    M64, C64 = M.clone().requires_grad_(True), C.clone().requires_grad_(True)
    ref = _ref_spatial64(M64, C64, H, W)
    (ref * G).sum().backward()
    tM = M.float().to(DEV).requires_grad_(True)
    tC = C.float().to(DEV).requires_grad_(True)
    out = spatial_scan_2d(tM, tC, H, W)
    assert rel(out, ref) < FWD_TOL
    (out * G.float().to(DEV)).sum().backward()
    assert rel(tM.grad, M64.grad) < BWD_TOL
    assert rel(tC.grad, C64.grad) < BWD_TOL


@pytest.mark.parametrize("name,cls", [("spatial_cl4", "CliffordSpatialRotorBlockCl4"),
                                      ("spatial_cl8", "CliffordSpatialRotorBlockCl8")])
def test_spatial_block_matches_reference_golden(golden, name, cls, monkeypatch):
    import csn.vision as vision
    # the blocks' convolutions are cuDNN's; keep them in full fp32 (cuDNN defaults to TF32)
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    g = golden(name)
    sd = {k[len("param."):]: torch.tensor(v) for k, v in g.items() if k.startswith("param.")}
    B, C, H, W = g["x"].shape
    N = sd["gamma_log"].shape[0]
    blk = getattr(vision, cls)(C, num_neurons=N, use_schulz=False)
    blk.load_state_dict(sd)
    blk = blk.float().to(DEV).eval()
    x = torch.tensor(g["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    out = blk(x)
    assert rel(out, g["out"]) < FWD_TOL
    (out * torch.tensor(g["W"], dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(x.grad, g["dx"]) < BWD_TOL
    for k, p in blk.named_parameters():
        assert rel(p.grad, g[f"grad.{k}"]) < BWD_TOL, k


def _generator_chain64(craw, braw, mraw, lam, gam, D):
    """The spatial blocks' torch chain between the convolutions and the Cayley rotor
    (csn_toolkit/csn/vision.py:79-94), float64 on the CPU."""
    import torch.nn.functional as F
    B, _, H, W = craw.shape
    N, K = gam.shape[0], D * (D - 1) // 2
    pix = lambda t, *shape: t.permute(0, 2, 3, 1).reshape(B, H * W, *shape)
    ds = pix(F.softplus(mraw), N)
    C = pix(craw, N, D, D)
    biv = pix(braw, N, K)
    iu = torch.triu_indices(D, D, 1)
    skew = biv.new_zeros(B, H * W, N, D, D)
    skew[..., iu[0], iu[1]] = biv
    skew[..., iu[1], iu[0]] = -biv
    J = 0.5 * (C - C.transpose(-1, -2))
    Omega = ((skew + torch.tanh(lam) * J) * (0.5 * ds[..., None, None])).clamp(min=-3.0, max=3.0)
    decay = torch.sigmoid(-F.softplus(gam).view(1, 1, N) * ds)
    return Omega, C, decay


@pytest.mark.parametrize("D,N,shape", [(4, 2, (2, 5, 7)), (4, 2, (2, 9, 9)), (4, 3, (1, 16, 16)), (8, 1, (2, 3, 11)),
                                       (16, 1, (2, 6, 5)), (16, 2, (1, 4, 9))])
def test_spatial_generators_match_torch_chain(ops, D, N, shape):
    """Fused generator chain vs the torch chain in float64: Omega (clamped entries included),
    pixel-major C, decay and every input gradient, on pixel counts that leave a partial tile."""
    B, H, W = shape
    K = D * (D - 1) // 2
    g = torch.Generator().manual_seed(D * 100 + N)
    ins = [torch.randn(B, N * D * D, H, W, generator=g, dtype=torch.float64) * 3,
           torch.randn(B, N * K, H, W, generator=g, dtype=torch.float64) * 3,
           torch.randn(B, N, H, W, generator=g, dtype=torch.float64),
           torch.tensor(0.3, dtype=torch.float64), torch.randn(N, generator=g, dtype=torch.float64)]
    ref_in = [t.clone().requires_grad_(True) for t in ins]
    outs64 = _generator_chain64(*ref_in, D)
    assert (outs64[0].abs() == 3.0).any()  # the clamp is exercised
    grads = [torch.randn(o.shape, generator=g, dtype=torch.float64) for o in outs64]
    sum((o * w).sum() for o, w in zip(outs64, grads)).backward()
    gpu_in = [t.float().to(DEV).requires_grad_(True) for t in ins]
    outs = ops.spatial_generators(*gpu_in, D)
    for o, r in zip(outs, outs64):
        assert o.shape == r.shape
        assert rel(o, r) < 1e-5
    sum((o * w.float().to(DEV)).sum() for o, w in zip(outs, grads)).backward()
    for name, t, r in zip(("in_proj", "biv_proj", "metric", "lambda_sw", "gamma_log"), gpu_in, ref_in):
        assert rel(t.grad, r.grad) < 1e-4, name
