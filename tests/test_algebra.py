"""Generated blade tables and real representations (pure CPU)."""
import numpy as np
import pytest

from csn_b200 import algebra as A


@pytest.mark.parametrize("alg", [A.CL3, A.CL8], ids=["cl3", "cl8"])
def test_real_rep_is_a_homomorphism_with_transpose_reversion(alg):
    rng = np.random.default_rng(1)
    rep = A.real_rep(alg)
    D = rep.shape[-1]
    vec = rep[alg.blades_of_grade(1)]
    for i in range(alg.n):
        assert np.allclose(vec[i], vec[i].T) and np.allclose(vec[i] @ vec[i], np.eye(D))
        for j in range(i + 1, alg.n):
            assert np.allclose(vec[i] @ vec[j], -vec[j] @ vec[i])
    a, b = rng.standard_normal(alg.size), rng.standard_normal(alg.size)
    lhs = A.blades_to_matrix(alg, alg.mul(a, b))
    rhs = A.blades_to_matrix(alg, a) @ A.blades_to_matrix(alg, b)
    assert np.max(np.abs(lhs - rhs)) < 1e-10
    assert np.allclose(A.blades_to_matrix(alg, alg.reverse(a)), A.blades_to_matrix(alg, a).T)
    assert np.allclose(A.matrix_to_blades(alg, A.blades_to_matrix(alg, a)), a)


def test_bivectors_map_to_skew_signed_permutations():
    for alg in (A.CL3, A.CL8):
        for E in A.bivector_basis(alg):
            assert np.allclose(E, -E.T)
            assert np.all(np.sum(np.abs(E), axis=1) == 1)


def test_cl3_layout_matches_reference_order():
    assert A.CL3.names == ["1", "e1", "e2", "e3", "e12", "e23", "e31", "e123"]
    # e31 = e3 e1 = -e1 e3
    e1 = np.eye(8)[1]; e3 = np.eye(8)[3]
    assert np.allclose(A.CL3.mul(e3, e1), np.eye(8)[6])


def test_cl3_sandwich_table_matches_product(tmp_path):
    text = A.emit_header(tmp_path / "t.h")
    rng = np.random.default_rng(2)
    r = rng.standard_normal(4)
    r /= np.linalg.norm(r)
    R = np.zeros(8); R[[0, 4, 5, 6]] = r
    L = np.zeros((8, 8))
    for line in text.splitlines():
        if line.strip().startswith("L.m["):
            lhs, rhs = line.strip().rstrip(";").split(" = ")
            i, j = [int(x) for x in lhs[4:-1].split("][")]
            expr = rhs.replace("f", "")
            L[i, j] = eval(expr, {"r0": r[0], "r1": r[1], "r2": r[2], "r3": r[3]})
    h = rng.standard_normal(8)
    ref = A.CL3.mul(A.CL3.mul(R, h), A.CL3.reverse(R))
    assert np.allclose(L @ h, ref)


def test_generated_header_is_up_to_date(tmp_path):
    from pathlib import Path
    committed = (Path(A.__file__).resolve().parent.parent / "csrc" / "ga_tables.h").read_text()
    fresh = A.emit_header(tmp_path / "ga_tables.h")
    assert committed == fresh
