"""ctypes binding of the C ABI declared in include/csn_b200.h.

The library is loaded from the package directory (``libcsn_b200.so``, built in-tree
by ``csn_b200._build``).  There is no fallback: if the library is missing or CUDA
is unavailable, every entry point raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcsn_b200.so"

_lock = threading.Lock()
_lib = None

_f = ctypes.c_void_p  # device pointers
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t

# name -> argtypes, restype (int status unless stated)
SIGNATURES = {
    "csn_version": ([], ctypes.c_char_p),
    "csn_last_error": ([], ctypes.c_char_p),
    "csn_scan_workspace_bytes": ([_i64, _i64, _i64, _int], _sz),
    "csn_scan_fwd": ([_f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _f, _sz, _f], _int),
    "csn_scan_bwd": ([_f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _f, _sz, _f], _int),
    "csn_rotor_scan_workspace_bytes": ([_i64, _i64, _i64, _int], _sz),
    "csn_rotor_scan_fwd": ([_f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int, _f, _sz, _f],
                           _int),
    "csn_rotor_scan_bwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int,
                            _int, _int, _f, _sz, _f], _int),
    "csn_rotor_scan_bwd_reuse": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int,
                                  _int, _int, _f, _sz, _f], _int),
    "csn_rotor_scan_fwd_cached": ([_f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int, _f,
                                   _sz, _f], _int),
    "csn_rotor_scan_bwd_cached": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64,
                                   _i64, _int, _int, _int, _f, _sz, _f], _int),
    "csn_rotor_scan_heads_fwd": ([_f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _i64, _int, _int, _int,
                                  _f, _sz, _f], _int),
    "csn_rotor_scan_heads_bwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64,
                                  _i64, _int, _int, _int, _int, _f, _sz, _f], _int),
    "csn_rotor_scan_fwd_noalloc": ([_f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int,
                                    _f], _int),
    "csn_rotor_scan_aggregate_workspace_bytes": ([_i64, _i64, _i64, _int], _sz),
    "csn_rotor_scan_aggregate": ([_f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int, _f,
                                  _sz, _f], _int),
    "csn_rotor_scan_bwd_aggregate": ([_f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int, _f,
                                      _sz, _f], _int),
    "csn_rotor_scan_fwd_resume": ([_f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _int, _int, _f,
                                   _sz, _f], _int),
    "csn_rotor_scan_bwd_resume": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64,
                                   _i64, _int, _int, _int, _f, _sz, _f], _int),
    "csn_rotor_step": ([_f, _f, _f, _f, _f, _i64, _i64, _int, _int, _int, _f], _int),
    "csn_rotor_step_chained": ([_f, _f, _f, _f, _f, _i64, _i64, _int, _int, _int, _f], _int),
    "csn_cayley_fwd": ([_f, _f, _i64, _int, _f], _int),
    "csn_cayley_bwd": ([_f, _f, _f, _i64, _int, _f], _int),
    "csn_ga3_workspace_bytes": ([_i64, _i64, _i64], _sz),
    "csn_ga3_scan_fwd": ([_f, _f, _f, _f, _f, _i64, _i64, _i64, _f, _sz, _f], _int),
    "csn_ga3_scan_bwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _f, _sz, _f], _int),
    "csn_cell_fwd": ([_f, _f, _f, _f, _f, ctypes.c_float, _f, _i64, _i64, _i64, _f], _int),
    "csn_cell_workspace_bytes": ([_i64, _i64], _sz),
    "csn_cell_bwd": ([_f, _f, _f, _f, _f, ctypes.c_float, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64,
                      _f, _sz, _f], _int),
    "csn_spike_fwd": ([_f, _f, _i64, _int, ctypes.c_float, _f], _int),
    "csn_spike_bwd": ([_f, _f, _f, _i64, _int, ctypes.c_float, ctypes.c_float, _f], _int),
    "csn_layer_norm_fwd": ([_f, _f, _f, _f, _f, _f, _i64, _int, ctypes.c_float, _f], _int),
    "csn_layer_norm_bwd_workspace_bytes": ([_i64, _int], _sz),
    "csn_layer_norm_bwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _i64, _int, _f, _sz, _f], _int),
    "csn_ln_conv_silu_fwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _int, _int, ctypes.c_float, _f], _int),
    "csn_ln_conv_silu_bwd_workspace_bytes": ([_i64, _i64, _int, _int], _sz),
    "csn_ln_conv_silu_bwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _int, _int, _f,
                              _sz, _f], _int),
    "csn_generator_action_workspace_bytes": ([_i64, _i64], _sz),
    "csn_generator_action_fwd": ([_f, _f, _i64, _i64, _int, _int, ctypes.c_float, ctypes.c_float, _f, _f, _sz, _f],
                                 _int),
    "csn_generator_action_bwd": ([_f, _f, _f, _f, _i64, _i64, _int, _int, ctypes.c_float, ctypes.c_float, _f, _f,
                                  _f], _int),
    "csn_projection_epilogue_fwd": ([_f, _i64, _int, _int, _int, _f, ctypes.c_float, _f, _f, _f, _f], _int),
    "csn_projection_epilogue_bwd": ([_f, _i64, _int, _int, _int, _f, ctypes.c_float, _f, _f, _f, _f, _f, _f],
                                    _int),
    "csn_column_sum_workspace_bytes": ([_i64, _int], _sz),
    "csn_column_sum": ([_f, _i64, _int, _f, _f, _sz, _f], _int),
    "csn_silu_gate_fwd": ([_f, _i64, _int, _f, _f], _int),
    "csn_silu_gate_bwd": ([_f, _f, _i64, _int, _f, _f], _int),
    "csn_spatial_generators_partials": ([_i64, _i64, _int], _i64),
    "csn_spatial_generators_fwd": ([_f, _f, _f, _f, _f, _f, _f, _f, _i64, _i64, _i64, _int, _f], _int),
    "csn_spatial_generators_bwd": ([_f] * 13 + [_i64, _i64, _i64, _int, _f], _int),
    "csn_timing_enable": ([_int], _int),
    "csn_timing_reset": ([], _int),
    "csn_timing_read": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                         ctypes.POINTER(ctypes.c_int64)], _int),
}

CSN_OK = 0
STATUS = {0: "CSN_OK", 1: "CSN_ERR_INVALID", 2: "CSN_ERR_UNSUPPORTED", 3: "CSN_ERR_CUDA",
          4: "CSN_ERR_TIMEOUT"}


class CsnError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)}: {msg}")
        self.code = code


def load(path: Path | None = None):
    """Load (once) and return the ctypes handle of libcsn_b200.so."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with __graft_entry__.build() or "
                "`python -m csn_b200._build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(p))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def exported_symbols() -> list:
    return list(SIGNATURES)


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise CsnError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != CSN_OK:
        msg = lib.csn_last_error().decode(errors="replace")
        raise CsnError(name, rc, msg)


def timing_enable(on: bool) -> None:
    call("csn_timing_enable", int(on))


def timing_reset() -> None:
    call("csn_timing_reset")


def timing_read(name: str | None = None):
    """(total_ms, launches) of the library kernels named `name` since the last reset."""
    tot = ctypes.c_double(0.0)
    cnt = ctypes.c_int64(0)
    call("csn_timing_read", name.encode() if name else None, ctypes.byref(tot), ctypes.byref(cnt))
    return tot.value, cnt.value


def version() -> str:
    return load().csn_version().decode()
