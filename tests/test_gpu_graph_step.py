"""A captured training step (csn_b200.graphs.TrainStepGraph) equals the same steps run
eagerly: loss, diagnostics and every parameter after several steps on changing inputs."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def rel(a, ref):
    den = ref.abs().max().clamp_min(1e-30)
    return float((a - ref).abs().max() / den)


@pytest.mark.parametrize("lm", ["cl6", "cl8", "multihead"])
def test_graphed_train_step_equals_eager_steps(lm):
    from csn_b200 import graphs
    from python.clifford_cl6 import CliffordCL6ForCausalLM
    from python.clifford_cl8 import CliffordCL8ForCausalLM
    from python.clifford_multihead import MultiHeadCliffordLM
    torch.manual_seed(0)
    ctor = {"cl6": lambda: CliffordCL6ForCausalLM(65, d_model=32, num_layers=2, num_neurons=2),
            "cl8": lambda: CliffordCL8ForCausalLM(65, d_model=32, num_layers=2, num_neurons=2),
            "multihead": lambda: MultiHeadCliffordLM(65, d_model=24, num_layers=2, num_heads=2,
                                                              num_neurons_per_head=2)}[lm]
    eager = ctor().to(DEV)
    graphed = copy.deepcopy(eager)
    opt_e = torch.optim.AdamW(eager.parameters(), lr=1e-2, capturable=True)
    opt_g = torch.optim.AdamW(graphed.parameters(), lr=1e-2, capturable=True)
    gen = torch.Generator(device="cpu").manual_seed(1)
    batches = [(torch.randint(0, 65, (2, 48), generator=gen).to(DEV),
                torch.randint(0, 65, (2, 48), generator=gen).to(DEV)) for _ in range(4)]
    warmup = 2
    step = graphs.TrainStepGraph(graphed, opt_g, batches[0], warmup=warmup)  # runs warmup real steps

    def eager_step(i, t):
        opt_e.zero_grad(set_to_none=True)
        _, loss, diag = eager(i, t)
        loss.backward()
        opt_e.step()
        return loss.detach(), diag

    for _ in range(warmup):
        eager_step(*batches[0])
    for i, t in batches[1:]:
        loss_e, diag_e = eager_step(i, t)
        _, loss_g, diag_g = step(i, t)
        assert rel(loss_g.detach(), loss_e) < 1e-5
        got = graphs.read(diag_g)
        assert set(got) == set(diag_e)
        for k, v in diag_e.items():
            assert abs(got[k] - v) <= 1e-5 * max(1.0, abs(v)), k
    torch.cuda.synchronize()
    for (n, pe), pg in zip(eager.named_parameters(), graphed.parameters()):
        assert rel(pg.detach(), pe.detach()) < 1e-5, n


def test_graphed_forward_backward_without_optimizer_equals_eager():
    """TrainStepGraph without an optimizer (the spatial blocks' fwd + bwd): outputs, parameter
    gradients and input-map gradients of a replay equal one eager step."""
    from csn_b200 import graphs
    from csn.vision import CliffordSpatialRotorBlockCl4, CliffordSpatialRotorBlockCl8
    torch.manual_seed(0)

    class Blocks(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = torch.nn.ModuleList([CliffordSpatialRotorBlockCl4(16, num_neurons=2, use_schulz=False),
                                               CliffordSpatialRotorBlockCl8(32, num_neurons=1, use_schulz=False)])
            self.w = [torch.randn(2, 16, 8, 8, device=DEV), torch.randn(2, 32, 6, 6, device=DEV)]

        def forward(self, *xs):
            outs = [blk(x) for blk, x in zip(self.blocks, xs)]
            return outs, sum((y * w).sum() for y, w in zip(outs, self.w))

    eager = Blocks().to(DEV)
    graphed = copy.deepcopy(eager)
    xs = [torch.randn(2, 16, 8, 8, device=DEV), torch.randn(2, 32, 6, 6, device=DEV)]
    step = graphs.TrainStepGraph(graphed, None, xs, warmup=2, inputs_require_grad=True)
    new = [torch.randn_like(x) for x in xs]
    outs_g, _ = step(*new)
    xe = [x.clone().requires_grad_(True) for x in new]
    outs_e, loss = eager(*xe)
    loss.backward()
    torch.cuda.synchronize()
    for a, b in zip(outs_g, outs_e):
        assert rel(a.detach(), b.detach()) < 1e-5
    for a, b in zip(step.inputs, xe):
        assert rel(a.grad, b.grad) < 1e-5
    for (n, pe), pg in zip(eager.named_parameters(), graphed.parameters()):
        assert rel(pg.grad, pe.grad) < 1e-5, n
