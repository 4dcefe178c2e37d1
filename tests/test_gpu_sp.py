"""Sequence-parallel scan on the GPU.

* Shard emulation on one GPU: the CUDA shard aggregates, the cross-shard composition
  (plain scan kernel over the shard summaries) and the carried-in passes -- resumed from
  the aggregate's workspace, or rescanned in one piece -- exactly as
  csn_b200.sequence_parallel runs them per rank, equal the one-piece fused scan.
* Multi-GPU (runs when >= 2 GPUs are visible): real NCCL ranks, one shard each, through
  sequence_parallel_rotor_scan (autograd) -- forward and gradients equal the one-piece scan.
"""
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent
DEV = "cuda:0"


def rel(a, ref):
    return ((a - ref).abs().max() / ref.abs().max()).item()


def problem(B, T, N, D, damped, seed=0, device=DEV, gscale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    K = D * (D - 1) // 2
    gens = torch.randn(B, T, N, K, generator=g) * gscale
    dt = torch.rand(B, T, generator=g) * 0.09 + 0.01
    gamma = torch.nn.functional.softplus(torch.randn(B, T, N, generator=g)) if damped else None
    S = torch.randn(B, T, N, D, D, generator=g)
    dX = torch.randn(B, T, N, D, D, generator=g)
    mv = lambda t: None if t is None else t.to(device)
    return mv(gens), mv(dt), mv(gamma), mv(S), mv(dX)


@pytest.mark.parametrize("D,damped,G,Tl", [(8, False, 4, 96), (8, True, 3, 96), (4, True, 5, 96), (16, False, 2, 40),
                                            (8, True, 3, 8), (16, True, 2, 8), (4, False, 3, 8), (8, False, 2, 5)])
def test_shard_emulation_equals_full_scan(D, damped, G, Tl):
    """Tl = 8 and 5 give single-chunk shards (the resume starts the apply pass from h0 / dh_right
    directly); the others give many chunks per shard."""
    from csn_b200 import _build, ops
    from csn_b200.sequence_parallel import CudaBackend
    _build.build()
    B, N = 2, 3
    T = Tl * G
    gens, dt, gamma, S, dX = problem(B, T, N, D, damped, gscale=0.3)
    be = CudaBackend()
    sh = lambda t, g: None if t is None else t[:, g * Tl:(g + 1) * Tl].contiguous()
    aggs = [be.fwd_aggregate(sh(gens, g), sh(dt, g), sh(gamma, g), sh(S, g), "triu", True) for g in range(G)]
    Xs, h_ins = [], []
    for g in range(G):
        h_in = None
        if g > 0:
            h_in = be.scan_mc(torch.stack([a[0] for a in aggs[:g]], 1), torch.stack([a[1] for a in aggs[:g]], 1),
                              True)[:, -1].contiguous()
        h_ins.append(h_in)
        # even shards resume from the aggregate's workspace, odd shards rescan in one piece
        Xs.append(be.rotor_fwd(sh(gens, g), sh(dt, g), sh(gamma, g), sh(S, g), h_in, "triu", True,
                               ws=aggs[g][2] if g % 2 == 0 else None))
    X = torch.cat(Xs, 1)
    Xref = ops.fused_rotor_scan(gens, dt, gamma, S)
    assert rel(X, Xref) < 1e-4
    # backward
    cbs = [be.bwd_aggregate(sh(gens, g), sh(dt, g), sh(gamma, g), sh(dX, g), "triu", True) for g in range(G)]
    grads = []
    for g in range(G):
        H = None
        if g < G - 1:
            later = list(range(G - 1, g, -1))
            H = be.scan_mc(torch.stack([aggs[r][0].transpose(-1, -2) for r in later], 1),
                           torch.stack([cbs[r][0] for r in later], 1), True)[:, -1].contiguous()
        grads.append(be.rotor_bwd(sh(gens, g), sh(dt, g), sh(gamma, g), sh(S, g), h_ins[g], Xs[g],
                                  sh(dX, g), "triu", True, dh_right=H,
                                  ws=cbs[g][1] if g % 2 == 0 else None))
    tg, tdt, tS = gens.clone().requires_grad_(True), dt.clone().requires_grad_(True), S.clone().requires_grad_(True)
    tga = gamma.clone().requires_grad_(True) if damped else None
    ops.fused_rotor_scan(tg, tdt, tga, tS).backward(dX)
    assert rel(torch.cat([g_[0] for g_ in grads], 1), tg.grad) < 1e-4
    assert rel(torch.cat([g_[1] for g_ in grads], 1), tdt.grad) < 1e-4
    assert rel(torch.cat([g_[3] for g_ in grads], 1), tS.grad) < 1e-4
    if damped:
        assert rel(torch.cat([g_[2] for g_ in grads], 1), tga.grad) < 1e-4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, ws, port, q, use_op=False):
    try:
        for p in (str(REPO / "clifford-space-network_b200"), str(REPO)):
            if p not in sys.path:
                sys.path.insert(0, p)
        from datetime import timedelta
        import torch.distributed as dist
        from csn_b200 import ops
        from csn_b200.sequence_parallel import sequence_parallel_rotor_scan
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=60),
                                device_id=dev)
        B, N, D, Tl = 2, 4, 8, 512
        gens, dt, gamma, S, dX = problem(B, Tl * ws, N, D, False, device=dev, gscale=0.5)
        sl = slice(rank * Tl, (rank + 1) * Tl)
        lg = gens[:, sl].contiguous().requires_grad_(True)
        ldt = dt[:, sl].contiguous().requires_grad_(True)
        lS = S[:, sl].contiguous().requires_grad_(True)
        if use_op:  # the torch.library operator, group by name
            X = torch.ops.csn.sp_scan(lg, ldt, None, lS, dist.group.WORLD.group_name, 0, True)[0]
        else:
            X = sequence_parallel_rotor_scan(lg, ldt, None, lS)
        X.backward(dX[:, sl].contiguous())
        tg, tdt, tS = gens.clone().requires_grad_(True), dt.clone().requires_grad_(True), S.clone().requires_grad_(True)
        Xf = ops.fused_rotor_scan(tg, tdt, None, tS)
        Xf.backward(dX)
        errs = [rel(X, Xf[:, sl]), rel(lg.grad, tg.grad[:, sl]), rel(ldt.grad, tdt.grad[:, sl]),
                rel(lS.grad, tS.grad[:, sl])]
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", errs))
    except Exception as e:
        q.put((rank, "error", repr(e), traceback.format_exc()))


def _run_nccl(ws, use_op):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, ws, port, q, use_op)) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
    return res


def test_sp_scan_operator_on_one_rank():
    """torch.ops.csn.sp_scan (forward + registered autograd) on a one-rank NCCL group equals
    the fused scan."""
    for r in _run_nccl(1, True):
        assert r[1] == "ok", r
        assert max(r[2]) < 1e-4, r


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("use_op", [False, True], ids=["function", "operator"])
def test_sequence_parallel_over_nccl_ranks(use_op):
    ws = min(torch.cuda.device_count(), 4)
    for r in _run_nccl(ws, use_op):
        assert r[1] == "ok", r
        assert max(r[2]) < 1e-4, r

