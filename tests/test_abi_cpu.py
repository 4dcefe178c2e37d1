"""CPU-only checks of the C ABI: the library loads, exports every symbol that
include/csn_b200.h declares, and rejects invalid arguments before touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parent.parent / "include" / "csn_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(csn_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from csn_b200 import _build, _lib
    _build.build()
    return _lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "csn_scan_fwd" in syms and "csn_rotor_scan_bwd" in syms and len(syms) >= 10


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in csn_b200.h but not exported"


def test_binding_covers_every_declared_symbol():
    from csn_b200 import _lib
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_string(lib):
    assert b"sm_100a" in lib.csn_version()


def test_invalid_arguments_are_rejected_without_a_gpu(lib):
    null = ctypes.c_void_p(0)
    rc = lib.csn_scan_fwd(null, null, null, null, -1, 4, 2, 8, 1, null, 0, null)
    assert rc == 1 and b"negative" in lib.csn_last_error()
    rc = lib.csn_scan_fwd(null, null, null, null, 1, 4, 2, 7, 1, null, 0, null)
    assert rc == 1
    rc = lib.csn_scan_fwd(null, null, null, null, 1, 4, 2, 8, 1, null, 0, null)
    assert rc == 1 and b"required" in lib.csn_last_error()
    rc = lib.csn_rotor_scan_fwd(null, null, null, null, null, null, 1, 4, 2, 8, 1, 1, null, 0, null)
    assert rc == 2  # GA basis is not defined for D = 8
    rc = lib.csn_cayley_fwd(null, null, 4, 5, null)
    assert rc == 1
    # empty problems are a no-op
    assert lib.csn_scan_fwd(null, null, null, null, 0, 4, 2, 8, 1, null, 0, null) == 0


def test_spatial_generator_arguments_are_checked_without_a_gpu(lib):
    null = ctypes.c_void_p(0)
    fwd = lambda B, HW, N, D: lib.csn_spatial_generators_fwd(null, null, null, null, null, null, null, null,
                                                             B, HW, N, D, null)
    bwd = lambda B, HW, N, D: lib.csn_spatial_generators_bwd(*([null] * 13), B, HW, N, D, null)
    assert fwd(2, 64, 1, 5) == 2 and b"4, 8 or 16" in lib.csn_last_error()
    assert bwd(-1, 64, 1, 4) == 1
    assert fwd(2, 64, 1, 16) == 1 and b"missing pointer" in lib.csn_last_error()
    assert bwd(2, 64, 2, 8) == 1 and b"missing pointer" in lib.csn_last_error()
    assert bwd(1, 64, 6, 16) == 2 and b"shared memory" in lib.csn_last_error()  # 6 neurons of 16 x 16
    assert fwd(0, 64, 1, 4) == 0 and bwd(2, 0, 1, 16) == 0  # empty problems are a no-op
    # one partial row per CTA: 64 / 32 / 16 pixels per CTA for D = 4 / 8 / 16
    assert lib.csn_spatial_generators_partials(16, 6400, 4) == 1600
    assert lib.csn_spatial_generators_partials(16, 1600, 16) == 1600
    assert lib.csn_spatial_generators_partials(2, 33, 8) == 4
    assert lib.csn_spatial_generators_partials(2, 33, 5) == 0


def test_workspace_query_is_pure(lib):
    n1 = lib.csn_scan_workspace_bytes(32, 2048, 8, 8)
    n2 = lib.csn_rotor_scan_workspace_bytes(32, 2048, 8, 8)
    assert n2 > n1 > 0
    assert lib.csn_scan_workspace_bytes(-1, 4, 4, 8) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    from csn_b200 import ops
    M = torch.zeros(1, 4, 1, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rotor_scan(M, M)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.cayley(M)
