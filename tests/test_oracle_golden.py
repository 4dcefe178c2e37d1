"""Pin the float64 C oracle to the reference's own outputs.

The fixtures in tests/golden/ were produced by running the reference in float64
(tests/golden/make_golden.py).  The oracle must agree to ~1e-10: it is the same
arithmetic, only evaluated sequentially in C.
"""
import numpy as np
import pytest

TOL = 1e-10


def rel(a, b):
    den = np.max(np.abs(b)) if np.size(b) else 0.0
    return float(np.max(np.abs(np.asarray(a) - b)) / den) if den > 0 else float(np.max(np.abs(a - b), initial=0))


SCAN_CASES = [f"{d}_T{t}" for d, t in (("d4", 37), ("d8", 23), ("d16", 19))] + \
    [f"d{d}_T1" for d in (4, 8, 16)]


@pytest.mark.parametrize("case", SCAN_CASES)
def test_two_sided_scan_matches_reference_tree(golden, oracle, case):
    g = golden(f"scan_two_{case}")
    X = oracle.scan_fwd(g["M"], g["C"], two_sided=True)
    assert rel(X, g["X"]) < TOL
    dM, dC, _ = oracle.scan_bwd(g["M"], X, g["W"], two_sided=True)
    assert rel(dC, g["dC"]) < TOL
    ref_dM = g["dM"] if g["dM"].shape == dM.shape else np.zeros_like(dM)
    assert rel(dM, ref_dM) < TOL


@pytest.mark.parametrize("case", SCAN_CASES)
def test_one_sided_scan_matches_reference(golden, oracle, case):
    g = golden(f"scan_one_{case}")
    X = oracle.scan_fwd(g["M"], g["C"], two_sided=False)
    assert rel(X, g["X"]) < TOL and rel(X, g["X_tree"]) < TOL
    dM, dC, _ = oracle.scan_bwd(g["M"], X, g["W"], two_sided=False)
    assert rel(dC, g["dC"]) < TOL and rel(dC, g["dC_tree"]) < TOL
    assert rel(dM, g["dM"]) < TOL and rel(dM, g["dM_tree"]) < TOL


@pytest.mark.parametrize("D", [4, 8, 16])
def test_cayley_matches_reference_solve(golden, oracle, D):
    g = golden(f"cayley_d{D}")
    Q = oracle.cayley(g["Om"])
    assert rel(Q, g["Q"]) < TOL
    # csn_toolkit/csn/rotors.py uses the transposed convention
    assert rel(np.swapaxes(Q, -1, -2), g["Q_csn_transposed"]) < 1e-9
    eye = np.eye(D)
    assert np.max(np.abs(np.swapaxes(Q, -1, -2) @ Q - eye)) < 1e-12


ROTOR_CASES = ["rotor_d8_damped", "rotor_d8_undamped", "rotor_d4_damped", "rotor_d16_damped",
               "rotor_d16_spinor", "rotor_cl8ga_undamped", "rotor_cl8ga_damped"]


@pytest.mark.parametrize("case", ROTOR_CASES)
def test_rotor_scan_matches_reference_block_section(golden, oracle, case):
    g = golden(case)
    gamma = g.get("gamma")
    two = not bool(g["spinor"])
    X = oracle.rotor_scan_fwd(g["gens"], g["dt"], gamma, g["S"], g["basis"], two_sided=two)
    assert rel(X, g["X"]) < TOL
    dgens, ddt, dgamma, dS, _ = oracle.rotor_scan_bwd(g["gens"], g["dt"], gamma, g["S"], g["basis"],
                                                      X, g["W"], two_sided=two)
    assert rel(dgens, g["dgens"]) < 1e-9
    assert rel(ddt, g["ddt"]) < 1e-9
    assert rel(dS, g["dS"]) < TOL
    if gamma is not None:
        assert rel(dgamma, g["dgamma"]) < 1e-9


def test_rotor_build_matches_materialised_transitions(golden, oracle):
    g = golden("rotor_d8_damped")
    M, C = oracle.rotor_build(g["gens"], g["dt"], g["gamma"], g["S"], g["basis"])
    X = oracle.scan_fwd(M, C, two_sided=True)
    assert rel(X, g["X"]) < TOL


@pytest.mark.parametrize("case", ["ga3_config1", "ga3_large"])
def test_ga3_scan_matches_reference_via_real_rep(golden, oracle, case):
    g = golden(case)
    h = oracle.ga3_scan_fwd(g["gens"], g["dt"], g["x"])
    assert rel(h, g["h"]) < TOL
    dgens, ddt, dx, _ = oracle.ga3_scan_bwd(g["gens"], g["dt"], h, g["W"])
    assert rel(dx, g["dx"]) < TOL
    assert rel(dgens, g["dgens"]) < 1e-9
    assert rel(ddt, g["ddt"]) < 1e-9


@pytest.mark.parametrize("case", ["cell_a", "cell_b"])
def test_cell_forward_matches_reference(golden, oracle, case):
    g = golden(case)
    out = oracle.cell_fwd(g["prev"], g["x"], g["W_rec"], g["W_in"], g["gamma_bias"], float(g["dt"]))
    assert rel(out, g["out"]) < TOL


def test_ga_product_rule_matches_generated_tables(oracle):
    from csn_b200 import algebra
    rng = np.random.default_rng(0)
    for alg in (algebra.CL3, algebra.CL4):
        a = rng.standard_normal((5, alg.size))
        b = rng.standard_normal((5, alg.size))
        ref = alg.mul(a, b)
        got = oracle.ga_product(alg.masks, alg.orient, a, b)
        assert rel(got, ref) < 1e-13
