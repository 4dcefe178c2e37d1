"""Host logic of csn_b200.graphs (no GPU): the deferred-diagnostics switch, the one-copy
diagnostics read and TrainStepGraph's argument checks."""
import pytest
import torch


def test_deferred_diagnostics_is_scoped_and_nests():
    from csn_b200 import graphs
    assert not graphs.diagnostics_deferred()
    with graphs.deferred_diagnostics():
        assert graphs.diagnostics_deferred()
        with graphs.deferred_diagnostics():
            assert graphs.diagnostics_deferred()
        assert graphs.diagnostics_deferred()
    assert not graphs.diagnostics_deferred()
    with pytest.raises(RuntimeError):
        with graphs.deferred_diagnostics():
            raise RuntimeError("inside")
    assert not graphs.diagnostics_deferred()


def test_read_diagnostics_defers_inside_a_captured_step():
    from csn_b200 import graphs
    from python.clifford_cl6 import read_diagnostics
    named = {"mean_dt": torch.tensor(0.05), "ce_loss": torch.tensor([4.25]), "time_loss": 0.0}
    eager = read_diagnostics(named)
    assert eager == {"mean_dt": pytest.approx(0.05), "ce_loss": 4.25, "time_loss": 0.0}
    with graphs.deferred_diagnostics():
        deferred = read_diagnostics(named)
    assert torch.is_tensor(deferred["mean_dt"]) and deferred["mean_dt"].shape == ()
    assert deferred["time_loss"] == 0.0
    assert list(deferred) == list(named)
    assert graphs.read(deferred) == eager


def test_train_step_graph_checks_its_arguments():
    from csn_b200 import graphs
    model = torch.nn.Linear(4, 4)
    with pytest.raises(ValueError, match="capturable"):
        graphs.TrainStepGraph(model, torch.optim.AdamW(model.parameters()), [torch.zeros(2, 4)])
    with pytest.raises(ValueError, match="CUDA"):
        graphs.TrainStepGraph(model, torch.optim.AdamW(model.parameters(), capturable=True), [torch.zeros(2, 4)])
