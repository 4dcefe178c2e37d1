"""torch.ops.csn.* registrations, checked on CPU: every operator exists with its schema and
its fake implementation gives the right shapes on meta tensors (no kernel runs)."""
import pytest
import torch


@pytest.fixture(scope="module")
def csn_ops():
    import csn_b200.ops  # noqa: F401  (registers the operators)
    return torch.ops.csn


NAMES = ["scan_fwd", "scan_bwd", "fused_rotor_scan_fwd", "fused_rotor_scan_bwd", "cayley_fwd",
         "cayley_bwd", "cell_fwd", "cell_bwd", "ga3_scan_fwd", "ga3_scan_bwd", "rotor_step", "sp_scan",
         "sp_scan_bwd"]


@pytest.mark.parametrize("name", NAMES)
def test_operator_is_registered(csn_ops, name):
    op = getattr(csn_ops, name)
    assert op.default._schema.name == f"csn::{name}"


def test_fake_shapes_on_meta(csn_ops):
    m = lambda *s: torch.empty(*s, device="meta")
    B, T, N, D, K = 2, 5, 3, 8, 28
    M, C = m(B, T, N, D, D), m(B, T, N, D, D)
    assert csn_ops.scan_fwd(M, C, None, True, False).shape == (B, T, N, D, D)
    dM, dC, dh0 = csn_ops.scan_bwd(M, C, C, m(B, N, D, D), True, True)
    assert dM.shape == M.shape and dC.shape == M.shape and dh0.shape == (B, N, D, D)
    X = csn_ops.fused_rotor_scan_fwd(m(B, T, N, K), m(B, T), None, M, None, 0, True)
    assert X.shape == M.shape
    g = csn_ops.fused_rotor_scan_bwd(m(B, T, N, K), m(B, T), m(B, T, N), M, None, X, X, 0, True)
    assert [tuple(t.shape) for t in g] == [(B, T, N, K), (B, T), (B, T, N), (B, T, N, D, D), (0,)]
    assert csn_ops.cayley_fwd(m(7, 16, 16)).shape == (7, 16, 16)
    assert csn_ops.cell_fwd(m(4, 3), m(4, 5, 16), m(5, 5, 16), m(5, 3, 16), m(5), 0.02).shape == (4, 5, 16)
    assert csn_ops.ga3_scan_fwd(m(B, T, N, 3), m(B, T), m(B, T, N, 8), None).shape == (B, T, N, 8)
    X, h, Ps = csn_ops.sp_scan(m(B, T, N, K), m(B, T), None, M, "", 0, True)  # no process group: 1 rank
    assert X.shape == M.shape and h.shape == (B, N, D, D) and Ps.shape == (1, B, N, D, D)
    g = csn_ops.sp_scan_bwd(m(B, T, N, K), m(B, T), None, M, X, X, h, Ps, "", 0, True)
    assert [tuple(t.shape) for t in g] == [(B, T, N, K), (B, T), (0,), (B, T, N, D, D)]


def test_schema_arguments_follow_the_ops_api(csn_ops):
    args = [a.name for a in csn_ops.fused_rotor_scan_fwd.default._schema.arguments]
    assert args == ["gens", "dt", "gamma", "S", "h0", "basis", "two_sided"]
    args = [a.name for a in csn_ops.scan_fwd.default._schema.arguments]
    assert args == ["M", "C", "h0", "two_sided", "reverse"]


def test_sp_scan_schema(csn_ops):
    args = [a.name for a in csn_ops.sp_scan.default._schema.arguments]
    assert args == ["gens", "dt", "gamma", "S", "group_name", "basis", "two_sided"]
