"""GPU parity of the reference-compatible modules (python.*, csn.*) against the
reference's own float64 outputs (tests/golden) and the oracle.  Ports of the
reference's hot-path tests are marked with the file they follow."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, ref):
    a = a.detach().double().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(a - ref)) / den) if den > 0 else float(np.max(np.abs(a - ref)))


def load_block(ctor, g):
    blk = ctor().to(DEV)
    sd = {k[len("param."):]: torch.as_tensor(v, dtype=torch.float32) for k, v in g.items()
          if k.startswith("param.")}
    blk.load_state_dict(sd)
    return blk


@pytest.mark.parametrize("name", ["cl6_block", "cl8_block"])
def test_block_forward_backward_matches_reference(golden, name):
    from python.clifford_cl6 import CliffordCL6Block
    from python.clifford_cl8 import CliffordCL8Block
    g = golden(name)
    ctor = (lambda: CliffordCL6Block(32, num_neurons=4)) if name == "cl6_block" else \
        (lambda: CliffordCL8Block(32, num_neurons=2, use_schulz=False))
    blk = load_block(ctor, g)
    x = torch.tensor(g["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    out, Omega, dt = blk(x)
    assert rel(out, g["out"]) < 1e-4
    assert rel(Omega, g["Omega"]) < 1e-4 and rel(dt, g["dt"]) < 1e-5
    (out * torch.tensor(g["W"], dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(x.grad, g["dx"]) < 1e-3
    for k, p in blk.named_parameters():
        assert rel(p.grad, g["grad." + k]) < 1e-3, k


def test_multihead_block_matches_reference(golden):
    """python/clifford_multihead.py:56-194: per-head dt, head-folded fused scan."""
    from python.clifford_multihead import MultiHeadCliffordCL6Block
    g = golden("multihead_block")
    blk = load_block(lambda: MultiHeadCliffordCL6Block(16, num_heads=2, num_neurons_per_head=2), g)
    x = torch.tensor(g["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    out, Omega, dt = blk(x)
    assert rel(out, g["out"]) < 1e-4
    assert rel(Omega, g["Omega"]) < 1e-4 and rel(dt, g["dt"]) < 1e-5
    (out * torch.tensor(g["W"], dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(x.grad, g["dx"]) < 1e-3
    for k, p in blk.named_parameters():
        assert rel(p.grad, g["grad." + k]) < 1e-3, k


def test_multihead_lm_matches_reference(golden):
    """python/clifford_multihead.py:197-304: logits, loss with the action / time penalties,
    every parameter gradient."""
    from python.clifford_multihead import MultiHeadCliffordLM
    g = golden("multihead_lm")
    lm = load_block(lambda: MultiHeadCliffordLM(vocab_size=11, d_model=16, num_layers=2, num_heads=2), g)
    idx = torch.as_tensor(g["idx"], device=DEV)
    logits, loss, diag = lm(idx, torch.as_tensor(g["targets"], device=DEV))
    assert rel(logits, g["logits"]) < 1e-4
    assert abs(loss.item() - float(g["loss"])) / abs(float(g["loss"])) < 1e-5
    assert set(diag) >= {"head_0_mean_dt", "head_1_max_dt", "ce_loss", "action_loss", "time_loss"}
    loss.backward()
    for k, p in lm.named_parameters():
        assert rel(p.grad, g["grad." + k]) < 1e-3, k


@pytest.mark.parametrize("case", ["cell_a", "cell_b"])
def test_cell_matches_reference(golden, case):
    from python.clifford_layer import CliffordTENNCell
    g = golden(case)
    N, in_dim = g["W_in"].shape[:2]
    cell = CliffordTENNCell(num_neurons=N, in_dim=in_dim).to(DEV)
    with torch.no_grad():
        for k in ("W_rec", "W_in", "gamma_bias"):
            getattr(cell, k).copy_(torch.as_tensor(g[k]))
    x = torch.tensor(g["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    prev = torch.tensor(g["prev"], dtype=torch.float32, device=DEV, requires_grad=True)
    out, nxt = cell(x, prev, dt=float(g["dt"]))
    assert out is nxt
    assert rel(out, g["out"]) < 1e-4
    (out * torch.tensor(g["W"], dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(x.grad, g["dx"]) < 1e-3 and rel(prev.grad, g["dprev"]) < 1e-3
    assert rel(cell.W_rec.grad, g["dW_rec"]) < 1e-3 and rel(cell.W_in.grad, g["dW_in"]) < 1e-3
    assert rel(cell.gamma_bias.grad, g["dgamma_bias"]) < 1e-3


@pytest.mark.parametrize("Bt,N,in_dim,dt", [(64, 32, 8, 0.02), (3, 64, 5, 0.5), (1, 1, 1, 0.1)])
def test_cell_matches_oracle_at_scale(oracle, Bt, N, in_dim, dt):
    from python.clifford_layer import CliffordTENNCell
    torch.manual_seed(Bt + N)
    cell = CliffordTENNCell(num_neurons=N, in_dim=in_dim)
    with torch.no_grad():
        cell.W_rec.mul_(20.0)
        cell.gamma_bias.normal_()
    x = torch.randn(Bt, in_dim)
    prev = torch.randn(Bt, N, 16)
    ref = oracle.cell_fwd(prev.numpy(), x.numpy(), cell.W_rec.detach().numpy(), cell.W_in.detach().numpy(),
                          cell.gamma_bias.detach().numpy(), dt)
    cell = cell.to(DEV)
    out, _ = cell(x.to(DEV), prev.to(DEV), dt=dt)
    assert rel(out, ref) < 1e-4


def test_csn_rotors_keep_the_toolkit_transposed_convention(golden):
    from csn.rotors import cayley_rotor_8x8, cayley_rotor_16x16
    for D, fn in ((8, cayley_rotor_8x8), (16, cayley_rotor_16x16)):
        g = golden(f"cayley_d{D}")
        Q = fn(torch.tensor(g["Om"], dtype=torch.float32, device=DEV), use_schulz=False)
        assert rel(Q, g["Q_csn_transposed"]) < 1e-4


def test_scan_equivalence_port():
    """tests/test_scan_equivalence.py:15-56 -- tree vs sequential, D = 4, B4 T32 N8, seeded."""
    from python.clifford_scan import parallel_rotor_scan
    torch.manual_seed(0)
    B, T, N = 4, 32, 8
    skew = torch.randn(B, T, N, 4, 4, device=DEV)
    skew = 0.5 * (skew - skew.transpose(-1, -2))
    eye = torch.eye(4, device=DEV).view(1, 1, 1, 4, 4)
    Q = torch.matmul(eye + skew, eye - skew) / (1.0 + 0.25 * (skew ** 2).sum(dim=(-1, -2), keepdim=True))
    decay = torch.sigmoid(torch.randn(B, T, N, 1, 1, device=DEV))
    M = torch.sqrt(decay) * Q
    C = (1.0 - decay) * torch.randn(B, T, N, 4, 4, device=DEV)
    seq = []
    x = torch.zeros(B, N, 4, 4, device=DEV)
    for t in range(T):
        x = M[:, t] @ x @ M[:, t].transpose(-1, -2) + C[:, t]
        seq.append(x)
    assert (torch.stack(seq, 1) - parallel_rotor_scan(M, C)).abs().max().item() < 1e-4


def test_adaptive_dt_port():
    """tests/test_adaptive_dt.py:20-84 -- dt initialisation, rotor orthogonality under
    adaptive dt, gradient flow into the time head, 2-layer LM forward/backward."""
    from python.clifford_cl6 import AdaptiveTimeHead, CliffordCL6Block, CliffordCL6ForCausalLM, cayley_rotor_8x8
    torch.manual_seed(0)
    head = AdaptiveTimeHead(48, dt_base=0.05).to(DEV)
    dt = head(torch.randn(4, 32, 48, device=DEV))
    assert (dt > 0).all() and (dt - 0.05).abs().max().item() < 1e-3
    block = CliffordCL6Block(48, num_neurons=4, dt_base=0.05).to(DEV)
    out, Omega, dt = block(torch.randn(4, 32, 48, device=DEV))
    Q = cayley_rotor_8x8(Omega)
    eye = torch.eye(8, device=DEV)
    assert (Q.transpose(-1, -2) @ Q - eye).abs().max().item() < 1e-5
    x = torch.randn(2, 16, 48, device=DEV, requires_grad=True)
    out, Omega, dt = block(x)
    (out.sum() + (dt ** 2).sum()).backward()
    assert torch.isfinite(block.time_head.proj.weight.grad).all()
    assert torch.isfinite(block.time_head.proj.bias.grad).all()
    model = CliffordCL6ForCausalLM(vocab_size=65, d_model=48, num_layers=2, num_neurons=6).to(DEV)
    idx = torch.randint(0, 65, (4, 64), device=DEV)
    logits, loss, diags = model(idx, targets=torch.randint(0, 65, (4, 64), device=DEV))
    assert logits.shape == (4, 64, 65) and torch.isfinite(loss)
    loss.backward()
    for name, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name


def test_optimized_cl8_port():
    """tests/test_optimized_cl8.py:46-91 -- one-sided scan vs sequential (D16 T32), and
    finite gradients through a 2-layer Cl(8) LM with the spinor-bundle scan."""
    from python.clifford_cl8 import CliffordCL8ForCausalLM
    from python.clifford_scan import parallel_rotor_scan
    torch.manual_seed(0)
    M = torch.randn(4, 32, 1, 16, 16, device=DEV) * 0.1
    C = torch.randn(4, 32, 1, 16, 16, device=DEV)
    psi = torch.zeros(4, 1, 16, 16, device=DEV)
    seq = []
    for t in range(32):
        psi = M[:, t] @ psi + C[:, t]
        seq.append(psi)
    seq = torch.stack(seq, 1)
    X = parallel_rotor_scan(M, C, is_spinor_bundle=True)
    assert (torch.norm(seq - X) / torch.norm(seq)).item() < 1e-5
    model = CliffordCL8ForCausalLM(vocab_size=65, d_model=32, num_layers=2, num_neurons=1,
                                   use_schulz=True, is_spinor_bundle=True).to(DEV)
    x = torch.randint(0, 65, (4, 32), device=DEV)
    logits, loss, _ = model(x, targets=torch.randint(0, 65, (4, 32), device=DEV))
    loss.backward()
    for name, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name


def test_fused_cuda_d4_port(oracle):
    """csn_toolkit/examples/benchmark_cuda_kernels.py:30-77 -- the fused D = 4 one-sided
    CUDA scan vs the sequential reference, seed 42, S = 160 sequences, T = 80, rel 1e-4
    forward and 1e-3 gradients."""
    import csn.scan as cs
    from csn.cuda import fused_cuda_clifford_scan, is_fused_cuda_available
    assert is_fused_cuda_available()
    torch.manual_seed(42)
    B, T, N, D = 2, 80, 1, 4
    M = (0.5 * torch.randn(B, T, N, D, D, device=DEV)).requires_grad_(True)
    C = torch.randn(B, T, N, D, D, device=DEV).requires_grad_(True)
    X = cs.parallel_rotor_scan(M, C, backend="cuda")
    (X ** 2).sum().backward()
    Xr = oracle.scan_fwd(M.detach().double().cpu().numpy(), C.detach().double().cpu().numpy(), two_sided=False)
    dMr, dCr, _ = oracle.scan_bwd(M.detach().double().cpu().numpy(), Xr, 2 * Xr, two_sided=False)
    assert rel(X, Xr) < 1e-4
    assert rel(M.grad, dMr) < 1e-3 and rel(C.grad, dCr) < 1e-3
    # the [S, T, 4, 4] entry point gives the same trajectory
    Xf = fused_cuda_clifford_scan(M.detach().permute(0, 2, 1, 3, 4).reshape(B * N, T, 4, 4),
                                  C.detach().permute(0, 2, 1, 3, 4).reshape(B * N, T, 4, 4))
    assert rel(Xf.view(B, N, T, 4, 4).permute(0, 2, 1, 3, 4), Xr) < 1e-4


LM_CTORS = {
    "cl6_lm": ("python.clifford_cl6", "CliffordCL6ForCausalLM", dict(vocab_size=11, d_model=16, num_layers=2,
                                                                    num_neurons=2)),
    "cl8_lm": ("python.clifford_cl8", "CliffordCL8ForCausalLM", dict(vocab_size=11, d_model=16, num_layers=1,
                                                                    num_neurons=1, use_schulz=False)),
    "tenn_lm": ("python.clifford_model", "CliffordTENNForCausalLM", dict(vocab_size=11, d_model=16, num_layers=2,
                                                                         num_neurons=2)),
}


@pytest.mark.parametrize("name", sorted(LM_CTORS))
def test_lm_matches_reference(golden, name):
    """Whole LMs on the fused block path (python/clifford_cl6.py:189-297, clifford_cl8.py:199-298,
    clifford_model.py:207-295): logits, the loss with its least-action (and time) penalties, and
    every parameter gradient against the reference's float64 run."""
    import importlib
    mod, cls, kw = LM_CTORS[name]
    ctor = getattr(importlib.import_module(mod), cls)
    g = golden(name)
    lm = load_block(lambda: ctor(**kw), g)
    idx = torch.as_tensor(g["idx"], device=DEV)
    logits, loss, _ = lm(idx, targets=torch.as_tensor(g["targets"], device=DEV))
    assert rel(logits, g["logits"]) < 1e-4
    assert abs(loss.item() - float(g["loss"])) / abs(float(g["loss"])) < 1e-5
    loss.backward()
    for k, p in lm.named_parameters():
        assert rel(p.grad, g["grad." + k]) < 1e-3, k


def test_tenn_block_matches_reference(golden):
    """python/clifford_model.py:78-205 CliffordTENNBlock: output, Omega and every gradient."""
    from python.clifford_model import CliffordTENNBlock
    g = golden("tenn_block")
    blk = load_block(lambda: CliffordTENNBlock(16, num_neurons=2), g)
    x = torch.tensor(g["x"], dtype=torch.float32, device=DEV, requires_grad=True)
    out, Omega = blk(x, dt=0.07)
    assert rel(out, g["out"]) < 1e-4 and rel(Omega, g["Omega"]) < 1e-5
    (out * torch.tensor(g["W"], dtype=torch.float32, device=DEV)).sum().backward()
    assert rel(x.grad, g["dx"]) < 1e-3
    for k, p in blk.named_parameters():
        assert rel(p.grad, g["grad." + k]) < 1e-3, k
