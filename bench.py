#!/usr/bin/env python
"""Throughput benchmark of the fused rotor scan (forward + backward).

Workload (one "step"): the Cl(6,0) LM scan section, forward and backward, for 4 layers
at batch 32, L = 2048, 8 channels of 8 x 8 real matrices (Cl(6,0) ~ M_8(R)), 28 so(8)
generators per channel, adaptive dt per token and decay gamma per channel.  Synthetic
seeded inputs shaped like the block's projections (python/clifford_cl6.py:144-168):
gens ~ N(0, 1), dt ~ U(0.04, 0.06), gamma = softplus(N(0, 0.5^2)), S ~ N(0, 1), dX ~ N(0, 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank owns its own batch (independent sequences, no
data-path collective: weak scaling); time is the max over ranks.  ``--impl reference``
times the float64 CPU restatement of the reference algorithm (the oracle) on the host
cores instead, on a bounded sample.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "clifford-space-network_b200"))
sys.path.insert(0, str(REPO))

METRIC = "rotor-scan fwd+bwd Gelem/s (B*L*C)"
UNIT = "Gelem/s"
B, T, N, D, K_GEN, LAYERS = 32, 2048, 8, 8, 28, 4
# compulsory HBM bytes per element (float32), n = D*D, k = K_GEN, dt amortised over N
_n, _k = D * D, K_GEN
OP_BYTES = 4.0 * (5 * _n + 3 * _k + 3 + 3.0 / N)          # whole fused fwd+bwd op
KERNEL_BYTES = {                                           # per kernel, per element
    "fwd_apply": 4.0 * (_k + 2 * _n + 1 + 1.0 / N),        # gens, S, gamma, dt -> X
    "fwd_reduce": 4.0 * (_k + _n + 1 + 1.0 / N),           # gens, S, gamma, dt
    "bwd_reduce": 4.0 * (_n + _k + 1 + 1.0 / N),           # dX, gens, gamma, dt
    "bwd_apply": 4.0 * (3 * _n + 2 * _k + 2 + 2.0 / N),    # dX, X, gens, gamma, dt -> dS, dgens, dgamma, ddt
}
CONFIG = {"workload": "cl6_lm_scan_fwd_bwd", "batch": B, "seq_len": T, "channels": N,
          "matrix_dim": D, "generators": K_GEN, "layers": LAYERS, "algebra": "Cl(6,0)",
          "sided": "two", "damped": True, "l2": "inputs larger than L2 (195 MB per layer forward)"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def make_inputs(seed, device, batch=B, nlayers=LAYERS):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    layers = []
    for _ in range(nlayers):
        gens = torch.randn(batch, T, N, K_GEN, generator=g)
        dt = torch.rand(batch, T, generator=g) * 0.02 + 0.04
        gamma = torch.nn.functional.softplus(torch.randn(batch, T, N, generator=g) * 0.5)
        S = torch.randn(batch, T, N, D, D, generator=g)
        dX = torch.randn(batch, T, N, D, D, generator=g)
        layers.append({k: v.to(device) if device != "cpu" else v
                       for k, v in dict(gens=gens, dt=dt, gamma=gamma, S=S, dX=dX).items()})
    return layers


class ClockSampler:
    """SM clocks and throttle reasons sampled through NVML (read-only) every 10 ms
    during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.sm, self.mx, self.reasons = [], [], set()
        self._stop = threading.Event()
        self.thread = None
        self.err = None

    def _run(self):
        try:
            nv, h = self._nv, self._h
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            while not self._stop.is_set():
                self.sm.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                self.mx.append(mx)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
                self._stop.wait(0.01)
            nv.nvmlShutdown()
        except Exception as e:  # NVML missing: record why, never fail the bench
            self.err = repr(e)

    def __enter__(self):
        try:  # NVML initialised before the timed region starts
            import pynvml as nv
            nv.nvmlInit()
            self._nv, self._h = nv, nv.nvmlDeviceGetHandleByIndex(self.index)
        except Exception as e:
            self.err = repr(e)
            return self
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "error": self.err}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": max(self.mx),
                "reasons": sorted(self.reasons), "samples": len(self.sm)}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def run_cpu_reference(sample_batch, reps, warmup):
    """The float64 oracle (CPU restatement of the reference algorithm) on host cores."""
    import numpy as np
    from oracle import oracle as orc
    from csn_b200 import algebra
    E = algebra.triu_basis(D)
    rng = np.random.default_rng(0)
    gens = rng.standard_normal((sample_batch, T, N, K_GEN))
    dt = rng.uniform(0.04, 0.06, (sample_batch, T))
    gamma = np.log1p(np.exp(rng.standard_normal((sample_batch, T, N)) * 0.5))
    S = rng.standard_normal((sample_batch, T, N, D, D))
    dX = rng.standard_normal((sample_batch, T, N, D, D))

    def one():
        X = orc.rotor_scan_fwd(gens, dt, gamma, S, E)
        orc.rotor_scan_bwd(gens, dt, gamma, S, E, X, dX)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(reps):
        one()
    el = time.perf_counter() - t0
    elems = sample_batch * T * N * reps
    return elems / el / 1e9, el


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=B, help="per-rank batch (profiling: smaller)")
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers per step (profiling: 1)")
    args = ap.parse_args()
    bsz, nlay = args.batch, args.layers
    ELEMS_PER_LAYER = bsz * T * N
    ws, rank, local = dist_env()
    cores = os.cpu_count() or 1

    if args.impl == "reference":
        if rank != 0:
            return 0
        os.environ.setdefault("OMP_NUM_THREADS", str(cores))
        sample_batch = 8
        v, el = run_cpu_reference(sample_batch, reps=max(1, args.steps), warmup=max(0, min(args.warmup, 1)))
        line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": el / max(1, args.steps) * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic", "config": CONFIG, "impl": "reference",
                "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                 "sample": f"one layer at batch {sample_batch} of {B} (B{sample_batch} L{T} "
                                           f"C{N} D{D}) per step, float64 C oracle, OpenMP"},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    from csn_b200 import _lib, ops

    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = _lib.load()

    layers = make_inputs(1234 + rank, dev, bsz, nlay)
    basis = ops.BASIS["triu"]
    ws_bytes = lib.csn_rotor_scan_workspace_bytes(bsz, T, N, D)
    work = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    outs = [dict(X=torch.empty_like(L["S"]), dgens=torch.empty_like(L["gens"]),
                 ddt=torch.empty_like(L["dt"]), dgamma=torch.empty_like(L["gamma"]),
                 dS=torch.empty_like(L["S"])) for L in layers]
    P = ops._ptr
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)

    def step():
        for L, O in zip(layers, outs):
            _lib.call("csn_rotor_scan_fwd", P(L["gens"]), P(L["dt"]), P(L["gamma"]), P(L["S"]),
                      P(None), P(O["X"]), bsz, T, N, D, basis, 1, P(work), ws_bytes, sp)
            _lib.call("csn_rotor_scan_bwd", P(L["gens"]), P(L["dt"]), P(L["gamma"]), P(L["S"]),
                      P(None), P(O["X"]), P(L["dX"]), P(O["dgens"]), P(O["ddt"]), P(O["dgamma"]),
                      P(O["dS"]), P(None), bsz, T, N, D, basis, 1, P(work), ws_bytes, sp)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    _lib.timing_reset()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        _lib.timing_enable(True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        _lib.timing_enable(False)
    barrier()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    ms_per_step = ms / args.steps
    elems_step = ELEMS_PER_LAYER * nlay
    value = elems_step * ws / (ms_per_step * 1e-3) / 1e9

    # per-kernel device times over the timed region
    names = ["fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry", "bwd_apply",
             "reduce_channels"]
    ktimes = {n: _lib.timing_read(n) for n in names}
    launches = sum(c for _, c in ktimes.values())
    dom = max((n for n in KERNEL_BYTES), key=lambda n: ktimes[n][0])
    dom_ms = ktimes[dom][0] / max(1, ktimes[dom][1])
    hbm, peak_kind = peaks()
    achieved = KERNEL_BYTES[dom] * ELEMS_PER_LAYER / (dom_ms * 1e-3) / 1e9
    _lib.timing_reset()

    # end to end through the public op API with host buffers (pinned), copies inside
    e2e = None
    if args.e2e_steps > 0:
        host = [{k: v.cpu().pin_memory() for k, v in L.items()} for L in layers]
        h2d = sum(v.numel() * v.element_size() for Lh in host for v in Lh.values())
        d2h = sum(v.numel() * v.element_size() for O in outs for v in O.values())
        hout = [{k: torch.empty_like(v, device="cpu").pin_memory() for k, v in O.items()} for O in outs]

        def e2e_step():
            for Lh, Ho in zip(host, hout):
                gens = Lh["gens"].to(dev, non_blocking=True).requires_grad_(True)
                dt = Lh["dt"].to(dev, non_blocking=True).requires_grad_(True)
                gamma = Lh["gamma"].to(dev, non_blocking=True).requires_grad_(True)
                S = Lh["S"].to(dev, non_blocking=True).requires_grad_(True)
                dX = Lh["dX"].to(dev, non_blocking=True)
                X = ops.fused_rotor_scan(gens, dt, gamma, S)
                X.backward(dX)
                for k, src in (("X", X.detach()), ("dgens", gens.grad), ("ddt", dt.grad),
                               ("dgamma", gamma.grad), ("dS", S.grad)):
                    Ho[k].copy_(src, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            e2e_step()
        el = time.perf_counter() - t0
        if ws > 1:
            t = torch.tensor([el], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            el = t.item()
        e2e = {"value": elems_step * ws * args.e2e_steps / el / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "timing": "wall clock around K steps ending in a stream synchronize, max over ranks"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        os.environ.setdefault("OMP_NUM_THREADS", str(cores))
        v, el = run_cpu_reference(8, reps=2, warmup=0)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"B8 L{T} C{N} D{D}, one layer fwd+bwd x2, float64 C oracle (OpenMP)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": dict(CONFIG, batch=bsz, layers=nlay,
                               parallelism=f"replicas{ws}" if ws > 1 else "single"),
                "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm,
                             "unit": "GB/s", "frac": achieved / hbm, "traffic": None,
                             "peak_kind": peak_kind,
                             "bytes_per_elem": KERNEL_BYTES[dom], "avg_launch_ms": dom_ms},
                "op_roofline": {"achieved": OP_BYTES * elems_step / (ms_per_step * 1e-3) / 1e9,
                                "peak": hbm, "unit": "GB/s",
                                "frac": OP_BYTES * elems_step / (ms_per_step * 1e-3) / 1e9 / hbm,
                                "bytes_per_elem": OP_BYTES},
                "kernel_ms": {n: {"total_ms": t, "launches": c} for n, (t, c) in ktimes.items()},
                "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
