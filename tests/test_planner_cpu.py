"""The chunk planner of the matrix scans, read through the workspace-size queries (host code:
no GPU needed).

A scan of S = B * N sequences of T steps is cut into chunks; with more than one chunk per
sequence it runs a reduce pass, a carry and an apply pass, and its scratch holds three D x D
matrices per chunk (the aggregates and the carry), so
    csn_scan_workspace_bytes = 256                                  (one chunk)
                             = 256 + 3 * S * nchunks * D * D * 4     (several)
which gives the chunk count the planner chose.  The cases are the benchmark shapes and the
rules the kernels were tuned for: one wave of (sequence, chunk) threads for D = 8, a wave- and
tail-aware count for D = 16, and one chunk for problems too small to fill the GPU.
"""
import pytest

from csn_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def nchunks(lib, B, T, N, D):
    nbytes = lib.csn_scan_workspace_bytes(B, T, N, D)
    if nbytes <= 256:
        return 1
    per_chunk = 3 * B * N * D * D * 4
    assert (nbytes - 256) % per_chunk == 0
    return (nbytes - 256) // per_chunk


def test_tiny_problems_run_one_chunk(lib):
    # the reference's D = 4 benchmark harness (B2 T80 N1) and the 1024-element bound
    assert nchunks(lib, 2, 80, 1, 4) == 1
    assert nchunks(lib, 1, 1024, 1, 8) == 1
    assert nchunks(lib, 1, 1025, 1, 8) > 1


def test_d8_lm_shape_fills_one_wave(lib):
    # B32 L2048 C8: 256 sequences x 147 chunks of 14 steps = 37632 threads, 294 blocks of 128
    # for the 2 x 148 resident blocks
    n = nchunks(lib, 32, 2048, 8, 8)
    assert n == 147
    assert (32 * 8 * n + 127) // 128 <= 2 * 148


def test_d16_cl8_shape_runs_several_waves(lib):
    # B16 L8192 C32: a count in the measured plateau (24 - 64 chunks: 19.3 - 19.6 ms per step,
    # against 23.7 ms with 5 chunks)
    n = nchunks(lib, 16, 8192, 32, 16)
    assert 24 <= n <= 64


def test_d16_short_sequences_that_fill_the_gpu_keep_one_chunk(lib):
    # 640 sequences of 40 steps (a row scan of the 40 x 40 spatial block): the reduce pass
    # would cost more than the tail it removes
    assert nchunks(lib, 16 * 40, 40, 1, 16) == 1


def test_d4_short_sequences_that_do_not_fill_the_gpu_are_chunked(lib):
    # 2560 sequences of 80 steps (the 80 x 80 spatial block): 8-step chunks
    assert nchunks(lib, 16 * 80, 80, 2, 4) == 10
