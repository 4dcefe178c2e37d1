"""Float64 CPU oracle for the rotor-scan hot path -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker (and the timed CPU baseline in bench.py).  It
wraps ``csn_oracle.c`` (built into ``oracle/_build/liboracle_csn.so``) with
numpy.  Only ``tests/``, ``__graft_entry__.smoke()`` and bench.py's CPU legs may
import it; the CUDA product path never does.

Every function restates one reference routine (paths relative to the reference
project root):

=====================  ============================================================
function               reference
=====================  ============================================================
scan_fwd / scan_bwd    python/clifford_scan.py:19-85 (two-sided),
                       csn_toolkit/csn/scan.py:16-72 (one-sided, analytic adjoint)
cayley                 python/clifford_cl6.py:57-68, python/clifford_cl8.py:29-45
rotor_build            python/clifford_cl6.py:150-168
rotor_scan_fwd / _bwd  python/clifford_cl6.py:150-171 + autograd
ga_product             include/clifford_algebra.cuh:60-74, :167-189
ga3_scan_fwd / _bwd    Cl(3,0) blade layout include/clifford_configs.cuh:38-51
cell_fwd               python/clifford_layer.py:50-115
=====================  ============================================================

Parity is pinned by ``tests/test_oracle_golden.py`` against fixtures that
``tests/golden/make_golden.py`` produced by running the reference itself in
float64.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle_csn.so"
_lib = None

_D = ctypes.POINTER(ctypes.c_double)
_I = ctypes.POINTER(ctypes.c_int)
_L = ctypes.c_long


def build() -> Path:
    """Compile the C oracle with the committed Makefile (idempotent)."""
    src = _HERE / "csn_oracle.c"
    if _LIB_PATH.exists() and _LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return _LIB_PATH
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    sig = {
        "orc_scan_fwd": [_D, _D, _D, _D, _L, _L, _L, ctypes.c_int, ctypes.c_int],
        "orc_scan_bwd": [_D, _D, _D, _D, _D, _D, _D, _L, _L, _L, ctypes.c_int, ctypes.c_int],
        "orc_cayley": [_D, _D, _L, ctypes.c_int],
        "orc_rotor_build": [_D, _D, _D, _D, _D, ctypes.c_int, _D, _D, _L, _L, _L, ctypes.c_int],
        "orc_rotor_scan_fwd": [_D, _D, _D, _D, _D, ctypes.c_int, _D, _D, _L, _L, _L,
                               ctypes.c_int, ctypes.c_int],
        "orc_rotor_scan_bwd": [_D, _D, _D, _D, _D, ctypes.c_int, _D, _D, _D, _D, _D, _D, _D,
                               _D, _L, _L, _L, ctypes.c_int, ctypes.c_int],
        "orc_ga_product": [_I, _I, ctypes.c_int, _D, _D, _D, _L],
        "orc_ga3_scan_fwd": [_D, _D, _D, _D, _D, _L, _L, _L],
        "orc_ga3_scan_bwd": [_D, _D, _D, _D, _D, _D, _D, _D, _D, _L, _L, _L],
        "orc_cell_fwd": [_D, _D, _D, _D, _D, ctypes.c_double, _D, _L, _L, _L],
        "orc_set_threads": [ctypes.c_int],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    _lib = lib
    return lib


def set_threads(n: int) -> int:
    """Number of OpenMP threads the oracle uses from now on, whatever OMP_NUM_THREADS the
    process was started with (torchrun sets it to 1).  Returns the count in effect."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    return int(_load().orc_set_threads(int(n)))


def _c(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def _p(a):
    return None if a is None else a.ctypes.data_as(_D)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


# --------------------------------------------------------------------------- scans
def scan_fwd(M, C, h0=None, two_sided=True):
    """X[B,T,N,D,D] of the inclusive rotor scan (X_{-1} = h0 or 0)."""
    lib = _load()
    M, C = _c(M), _c(C)
    B, T, N, D, _ = M.shape
    h0 = None if h0 is None else _c(h0)
    X = np.empty_like(C)
    _check(lib.orc_scan_fwd(_p(M), _p(C), _p(h0), _p(X), B, T, N, D, int(two_sided)), "scan_fwd")
    return X


def scan_bwd(M, X, dX, h0=None, two_sided=True):
    """(dM, dC, dh0) of the rotor scan; dh0 is None when h0 is None."""
    lib = _load()
    M, X, dX = _c(M), _c(X), _c(dX)
    B, T, N, D, _ = M.shape
    h0 = None if h0 is None else _c(h0)
    dM, dC = np.empty_like(M), np.empty_like(M)
    dh0 = None if h0 is None else np.empty_like(h0)
    _check(lib.orc_scan_bwd(_p(M), _p(X), _p(dX), _p(h0), _p(dM), _p(dC), _p(dh0),
                            B, T, N, D, int(two_sided)), "scan_bwd")
    return dM, dC, dh0


def cayley(Om):
    """Q = (I - Om)^{-1}(I + Om) over the leading dims of Om[..., D, D]."""
    lib = _load()
    Om = _c(Om)
    D = Om.shape[-1]
    Q = np.empty_like(Om)
    _check(lib.orc_cayley(_p(Om), _p(Q), Om.size // (D * D), D), "cayley")
    return Q


# ------------------------------------------------------------------ fused rotor scan
def triu_basis(D: int) -> np.ndarray:
    """Skew basis E_k [D(D-1)/2, D, D] for the reference's generator layout:
    g_k sits at torch.triu_indices(D, D, 1)[:, k] and its negative at the mirror
    (python/clifford_cl6.py:124-125, :155-158)."""
    iu, iv = np.triu_indices(D, 1)
    E = np.zeros((len(iu), D, D))
    E[np.arange(len(iu)), iu, iv] = 1.0
    E[np.arange(len(iu)), iv, iu] = -1.0
    return E


def rotor_build(gens, dt, gamma, S, basis):
    lib = _load()
    gens, dt, S, basis = _c(gens), _c(dt), _c(S), _c(basis)
    gamma = None if gamma is None else _c(gamma)
    B, T, N, D, _ = S.shape
    K = basis.shape[0]
    M, C = np.empty_like(S), np.empty_like(S)
    _check(lib.orc_rotor_build(_p(gens), _p(dt), _p(gamma), _p(S), _p(basis), K, _p(M), _p(C),
                               B, T, N, D), "rotor_build")
    return M, C


def rotor_scan_fwd(gens, dt, gamma, S, basis, h0=None, two_sided=True):
    lib = _load()
    gens, dt, S, basis = _c(gens), _c(dt), _c(S), _c(basis)
    gamma = None if gamma is None else _c(gamma)
    h0 = None if h0 is None else _c(h0)
    B, T, N, D, _ = S.shape
    X = np.empty_like(S)
    _check(lib.orc_rotor_scan_fwd(_p(gens), _p(dt), _p(gamma), _p(S), _p(basis), basis.shape[0],
                                  _p(h0), _p(X), B, T, N, D, int(two_sided)), "rotor_scan_fwd")
    return X


def rotor_scan_bwd(gens, dt, gamma, S, basis, X, dX, h0=None, two_sided=True):
    """(dgens, ddt, dgamma, dS, dh0); dgamma None when undamped, dh0 None when h0 None."""
    lib = _load()
    gens, dt, S, basis, X, dX = _c(gens), _c(dt), _c(S), _c(basis), _c(X), _c(dX)
    gamma = None if gamma is None else _c(gamma)
    h0 = None if h0 is None else _c(h0)
    B, T, N, D, _ = S.shape
    dgens, ddt, dS = np.empty_like(gens), np.empty_like(dt), np.empty_like(S)
    dgamma = None if gamma is None else np.empty_like(gamma)
    dh0 = None if h0 is None else np.empty_like(h0)
    _check(lib.orc_rotor_scan_bwd(_p(gens), _p(dt), _p(gamma), _p(S), _p(basis), basis.shape[0],
                                  _p(h0), _p(X), _p(dX), _p(dgens), _p(ddt), _p(dgamma), _p(dS),
                                  _p(dh0), B, T, N, D, int(two_sided)), "rotor_scan_bwd")
    return dgens, ddt, dgamma, dS, dh0


# ------------------------------------------------------------------ geometric algebra
def ga_product(masks, orient, a, b):
    lib = _load()
    masks = np.ascontiguousarray(masks, dtype=np.int32)
    orient = np.ascontiguousarray(orient, dtype=np.int32)
    a, b = _c(a), _c(b)
    nbl = masks.shape[0]
    out = np.empty_like(a)
    _check(lib.orc_ga_product(masks.ctypes.data_as(_I), orient.ctypes.data_as(_I), nbl, _p(a),
                              _p(b), _p(out), a.size // nbl), "ga_product")
    return out


def ga3_scan_fwd(gens, dt, x, h0=None):
    lib = _load()
    gens, dt, x = _c(gens), _c(dt), _c(x)
    h0 = None if h0 is None else _c(h0)
    B, T, N, _ = x.shape
    h = np.empty_like(x)
    _check(lib.orc_ga3_scan_fwd(_p(gens), _p(dt), _p(x), _p(h0), _p(h), B, T, N), "ga3_scan_fwd")
    return h


def ga3_scan_bwd(gens, dt, h, dh, h0=None):
    """(dgens, ddt, dx, dh0)."""
    lib = _load()
    gens, dt, h, dh = _c(gens), _c(dt), _c(h), _c(dh)
    h0 = None if h0 is None else _c(h0)
    B, T, N, _ = h.shape
    dgens, ddt, dx = np.empty_like(gens), np.empty_like(dt), np.empty_like(h)
    dh0 = None if h0 is None else np.empty_like(h0)
    _check(lib.orc_ga3_scan_bwd(_p(gens), _p(dt), _p(h0), _p(h), _p(dh), _p(dgens), _p(ddt),
                                _p(dx), _p(dh0), B, T, N), "ga3_scan_bwd")
    return dgens, ddt, dx, dh0


# ------------------------------------------------------------------------ cell
def cell_fwd(prev, x, W_rec, W_in, gamma_bias, dt):
    lib = _load()
    prev, x, W_rec, W_in, gamma_bias = _c(prev), _c(x), _c(W_rec), _c(W_in), _c(gamma_bias)
    Bt, N, _ = prev.shape
    in_dim = x.shape[1]
    out = np.empty_like(prev)
    _check(lib.orc_cell_fwd(_p(prev), _p(x), _p(W_rec), _p(W_in), _p(gamma_bias), float(dt),
                            _p(out), Bt, N, in_dim), "cell_fwd")
    return out


def max_rel(a, ref) -> float:
    """Reference metric max|a - ref| / max|ref|
    (csn_toolkit/examples/benchmark_cuda_kernels.py:60-62)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    num = float(np.max(np.abs(a - ref))) if ref.size else 0.0
    return num / den if den > 0 else num
