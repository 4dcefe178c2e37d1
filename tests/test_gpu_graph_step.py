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
