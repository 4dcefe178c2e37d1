"""CPU checks of the reference-compatible module API: names, signatures and
state_dict keys match the reference (paths relative to the reference root)."""
import inspect

import numpy as np
import pytest
import torch


def params(fn):
    return list(inspect.signature(fn).parameters)


def test_scan_signatures_match_reference():
    import csn.scan as cs
    import python.clifford_scan as ps
    # python/clifford_scan.py:19, :41
    assert params(ps.parallel_rotor_scan) == ["M", "C", "is_spinor_bundle"]
    assert inspect.signature(ps.parallel_rotor_scan).parameters["is_spinor_bundle"].default is False
    assert params(ps.rotor_binary_op) == ["M_b", "C_b", "M_a", "C_a", "is_spinor_bundle"]
    # csn_toolkit/csn/scan.py:96-102 (toolkit default is the one-sided scan)
    assert params(cs.parallel_rotor_scan) == ["M", "C", "is_spinor_bundle", "force_tree", "backend"]
    assert inspect.signature(cs.parallel_rotor_scan).parameters["is_spinor_bundle"].default is True
    assert params(cs.rotor_binary_op) == ["M_right", "C_right", "M_left", "C_left", "is_spinor_bundle"]


def test_rotor_and_cell_signatures_match_reference():
    from python import clifford_cl6, clifford_cl8, clifford_layer
    from csn import rotors
    assert params(clifford_cl6.cayley_rotor_8x8) == ["Omega"]
    assert params(clifford_cl8.cayley_rotor_16x16) == ["Omega", "use_schulz"]
    assert params(clifford_cl8.cayley_rotor_4x4) == ["Omega", "use_schulz"]
    for fn in (rotors.cayley_rotor_4x4, rotors.cayley_rotor_8x8, rotors.cayley_rotor_16x16):
        assert params(fn) == ["Omega", "use_schulz"]
    assert params(clifford_layer.CliffordTENNCell.forward) == ["self", "x_t", "prev_state", "dt"]
    assert params(clifford_layer.CliffordTENNCell.__init__) == ["self", "num_neurons", "in_dim",
                                                                 "algebra_dim"]


@pytest.mark.parametrize("name,ctor", [
    ("cl6_block", lambda: __import__("python.clifford_cl6", fromlist=["x"]).CliffordCL6Block(32, num_neurons=4)),
    ("cl8_block", lambda: __import__("python.clifford_cl8", fromlist=["x"]).CliffordCL8Block(32, num_neurons=2)),
])
def test_block_state_dict_matches_reference(golden, name, ctor):
    g = golden(name)
    ref_keys = {k[len("param."):]: v.shape for k, v in g.items() if k.startswith("param.")}
    blk = ctor()
    mine = {k: tuple(v.shape) for k, v in blk.state_dict().items()}
    assert mine == {k: tuple(s) for k, s in ref_keys.items()}
    blk.load_state_dict({k: torch.as_tensor(g["param." + k]) for k in ref_keys})


@pytest.mark.parametrize("name,cls,kw", [("spatial_cl4", "CliffordSpatialRotorBlockCl4", dict(num_neurons=2)),
                                         ("spatial_cl8", "CliffordSpatialRotorBlockCl8", dict(num_neurons=1))])
def test_spatial_block_state_dict_matches_reference(golden, name, cls, kw):
    import csn.vision as vision
    g = golden(name)
    ref_keys = {k[len("param."):]: tuple(v.shape) for k, v in g.items() if k.startswith("param.")}
    blk = getattr(vision, cls)(g["x"].shape[1], **kw)
    assert {k: tuple(v.shape) for k, v in blk.state_dict().items()} == ref_keys
    blk.load_state_dict({k: torch.as_tensor(g["param." + k]) for k in ref_keys})
    # csn_toolkit/csn/vision.py:58, :115
    assert params(type(blk).__init__) == ["self", "in_channels", "num_neurons", "use_schulz"]


@pytest.mark.parametrize("name,ctor", [
    ("multihead_block", lambda: __import__("python.clifford_multihead", fromlist=["x"]).MultiHeadCliffordCL6Block(
        16, num_heads=2, num_neurons_per_head=2)),
    ("multihead_lm", lambda: __import__("python.clifford_multihead", fromlist=["x"]).MultiHeadCliffordLM(
        vocab_size=11, d_model=16, num_layers=2, num_heads=2)),
])
def test_multihead_state_dict_matches_reference(golden, name, ctor):
    g = golden(name)
    ref_keys = {k[len("param."):]: tuple(v.shape) for k, v in g.items() if k.startswith("param.")}
    m = ctor()
    assert {k: tuple(v.shape) for k, v in m.state_dict().items()} == ref_keys
    m.load_state_dict({k: torch.as_tensor(g["param." + k]) for k in ref_keys})
    from python import clifford_multihead as mh
    # python/clifford_multihead.py:62-71, :206-219
    assert params(mh.MultiHeadCliffordCL6Block.__init__) == [
        "self", "d_model", "num_heads", "num_neurons_per_head", "kernel_size", "dt_base", "spike_threshold",
        "spike_beta"]
    assert params(mh.MultiHeadCliffordLM.forward) == ["self", "idx", "targets"]


def test_cell_parameters_match_reference():
    from python.clifford_layer import CliffordTENNCell
    cell = CliffordTENNCell(num_neurons=5, in_dim=4)
    assert {k: tuple(v.shape) for k, v in cell.state_dict().items()} == {
        "W_rec": (5, 5, 16), "W_in": (5, 4, 16), "gamma_bias": (5,), "bivector_bias": (5, 6)}


def test_rotor_binary_op_composes_like_the_reference():
    from python.clifford_scan import rotor_binary_op
    rng = np.random.default_rng(0)
    Mb, Cb, Ma, Ca = (torch.tensor(rng.standard_normal((2, 4, 4))) for _ in range(4))
    M, C = rotor_binary_op(Mb, Cb, Ma, Ca)
    assert torch.allclose(M, Mb @ Ma) and torch.allclose(C, Mb @ Ca @ Mb.transpose(-1, -2) + Cb)


def test_dropin_modules_refuse_cpu_tensors():
    from python.clifford_scan import parallel_rotor_scan
    M = torch.zeros(1, 3, 1, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        parallel_rotor_scan(M, M)


@pytest.mark.parametrize("name,mod,cls,kw", [
    ("cl6_lm", "python.clifford_cl6", "CliffordCL6ForCausalLM", dict(vocab_size=11, d_model=16, num_layers=2,
                                                                    num_neurons=2)),
    ("cl8_lm", "python.clifford_cl8", "CliffordCL8ForCausalLM", dict(vocab_size=11, d_model=16, num_layers=1,
                                                                    num_neurons=1, use_schulz=False)),
    ("tenn_lm", "python.clifford_model", "CliffordTENNForCausalLM", dict(vocab_size=11, d_model=16, num_layers=2,
                                                                         num_neurons=2)),
    ("tenn_block", "python.clifford_model", "CliffordTENNBlock", dict(d_model=16, num_neurons=2)),
])
def test_lm_state_dict_matches_reference(golden, name, mod, cls, kw):
    """Checkpoint compatibility of the whole LMs and the TENN block: the reference's state_dict
    keys and shapes load unchanged."""
    import importlib
    g = golden(name)
    ref_keys = {k[len("param."):]: tuple(v.shape) for k, v in g.items() if k.startswith("param.")}
    m = getattr(importlib.import_module(mod), cls)(**kw)
    assert {k: tuple(v.shape) for k, v in m.state_dict().items()} == ref_keys
    m.load_state_dict({k: torch.as_tensor(g["param." + k]) for k in ref_keys})
