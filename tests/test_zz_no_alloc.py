"""The no-allocation entry point csn_rotor_scan_fwd_noalloc, called through the C ABI.

Some hosts cannot let a library allocate device memory: they reserve the whole GPU
for their own pool, or forbid allocation once their serving loop is running.  For
them the library offers a forward rotor scan whose scratch lives in a static device
array.  This test checks that entry point against the ordinary, workspace-taking
csn_rotor_scan_fwd for every matrix size (D = 4, 8, 16), on calls in a row with
different inputs and shapes (a call must not be disturbed by what the one before it
left in the shared scratch).  Both entry points run the same chunk plan and kernels, so
their outputs are compared bit for bit.  A problem too large for the static scratch
must be refused with a clear error.

The file name sorts last so that a run stopping at the first failure has already run
every other test; it is also self-contained, so it passes run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _case(seed, B, T, N, D):
    g = torch.Generator(device="cpu").manual_seed(seed)
    K = D * (D - 1) // 2
    gens = torch.randn(B, T, N, K, generator=g) * 4.0
    dt = torch.rand(B, T, generator=g) * 0.09 + 0.01
    gamma = torch.nn.functional.softplus(torch.randn(B, T, N, generator=g))
    S = torch.randn(B, T, N, D, D, generator=g)
    return [t.to(DEV).contiguous() for t in (gens, dt, gamma, S)]


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from csn_b200 import _build, _lib
    _build.build()
    return _lib.load()


def _run_both(lib, seed, B, T, N, D):
    gens, dt, gamma, S = _case(seed, B, T, N, D)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    X_ref = torch.empty_like(S)
    nbytes = lib.csn_rotor_scan_workspace_bytes(B, T, N, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.csn_rotor_scan_fwd(_p(gens), _p(dt), _p(gamma), _p(S), _p(None), _p(X_ref),
                                B, T, N, D, 0, 1, _p(ws), nbytes, stream)
    assert rc == 0, lib.csn_last_error()
    X = torch.full_like(S, float("nan"))
    rc = lib.csn_rotor_scan_fwd_noalloc(_p(gens), _p(dt), _p(gamma), _p(S), _p(None), _p(X),
                                        B, T, N, D, 0, 1, stream)
    assert rc == 0, lib.csn_last_error()
    torch.cuda.synchronize()
    return X, X_ref


# (seed, (B, T, N, D)): every case runs several chunks per sequence; consecutive cases
# differ in shape and seed, so stale scratch from the call before would show up
CASES = ((11, (4, 777, 8, 8)), (12, (3, 1500, 5, 8)), (13, (4, 2000, 8, 4)), (14, (2, 500, 3, 16)),
         (15, (3, 911, 2, 4)), (16, (1, 300, 5, 16)))


def test_noalloc_is_bit_identical_to_workspace_entry_point_on_calls_in_a_row(lib):
    for seed, shape in CASES:
        B, T, N, D = shape
        assert 256 < lib.csn_scan_workspace_bytes(B, T, N, D) <= (32 << 20)  # chunked, fits
        X, X_ref = _run_both(lib, seed, *shape)
        assert torch.isfinite(X).all()
        assert torch.equal(X, X_ref), f"no-alloc differs from the workspace entry point at {shape}"


def test_noalloc_refuses_problems_above_its_static_scratch(lib):
    # 32000 sequences of 2000 steps: the plan splits each into 2 chunks, and the chunk
    # aggregates and carries of 64000 chunks need ~49 MB of scratch
    B, T, N, D = 4000, 2000, 8, 8
    assert lib.csn_scan_workspace_bytes(B, T, N, D) > (32 << 20)
    null = ctypes.c_void_p(0)
    dummy = torch.empty(4, device=DEV)
    rc = lib.csn_rotor_scan_fwd_noalloc(_p(dummy), _p(dummy), null, _p(dummy), null, _p(dummy),
                                        B, T, N, D, 0, 1, null)
    assert rc == 1
    assert b"32 MiB" in lib.csn_last_error()
