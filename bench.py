#!/usr/bin/env python
"""Throughput benchmark of the rotor-scan hot path (forward + backward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cl6_lm|cl3|cl8|gen|sp|lm_train|spatial]

Workloads (one "step" = one forward + backward pass over one batch of synthetic input,
seeded, float32, shaped like the reference's configurations):

* ``cl6_lm`` (default) -- the Cl(6,0) LM scan section of 4 layers: batch 32, L 2048,
  8 channels of 8 x 8 matrices (Cl(6,0) ~ M_8(R)), 28 so(8) generators, adaptive dt per
  token, decay gamma per channel.  Inputs shaped like the block's projections
  (python/clifford_cl6.py:144-168): gens ~ N(0,1), dt ~ U(0.04,0.06),
  gamma = softplus(N(0,0.5^2)), S ~ N(0,1), dX ~ N(0,1).
* ``cl3`` -- Cl(3,0) blade-basis scan h_t = R_t h R~_t + x_t at the bandwidth scale of
  the Cl(3) configuration: batch 64, L 65536, 16 channels, gens ~ N(0, 0.1^2) on the 3
  bivectors, dt ~ U(0.01, 0.1), x ~ N(0, 1), dh ~ N(0, 1).
* ``cl8`` -- Cl(8,0) ~ M_16(R) scan: batch 16, L 8192, 32 channels of 16 x 16 matrices,
  28 GA bivector-blade generators ~ N(0, 0.05^2) mapped through rho, dt ~ U(0.005, 0.05),
  x ~ N(0, 1), undamped.
* ``gen`` -- autoregressive O(1)-state generation, Cl(6,0), 256 streams x 8 channels:
  p50 latency of one rotor step (graph-replayed) and tokens/s.
* ``sp`` -- sequence-parallel long scan, Cl(6,0): B 8, L 2^20, C 64, time axis split over
  the torchrun ranks (strong scaling), forward + backward.
* ``lm_train`` -- one training step of the whole Cl(6,0) LM around the scan (d_model 128,
  4 blocks x 8 neurons, B32 L2048, AdamW): tokens/s, with the scan's share of the step.
* ``spatial`` -- the detector's three spatial rotor blocks (Cl(4) 80 x 80, Cl(8) 40 x 40 and
  20 x 20 feature maps of a 640 x 640 image), batch 16, forward + backward.

Without ``--workload``, a run started by torch.distributed.run (at any world size, 1
included) is the ``sp`` workload -- the long-sequence configuration that is split over
GPUs, strong scaling, with one NCCL all-gather per direction -- and a plain run is
``cl6_lm``.  The other workloads under torchrun run one replica per rank (independent
sequences, no data-path collective: weak scaling); time is the max over ranks.
``--impl reference`` times the float64 CPU restatement of the reference algorithm (the
oracle) on the host cores instead, on a bounded sample of the same workload; under torchrun
rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

import numpy as np
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


def launched_by_torchrun():
    """True when torch.distributed.run started this process (it sets these for every world
    size, 1 included)."""
    return any(k in os.environ for k in ("TORCHELASTIC_RUN_ID", "LOCAL_WORLD_SIZE", "GROUP_RANK"))


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


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


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _cpu_threads(cores):
    """Give the float64 CPU oracle every host core: set OMP_NUM_THREADS for this process
    (torchrun starts ranks with OMP_NUM_THREADS=1) and set the oracle's OpenMP thread count
    directly, which also holds when its library is already loaded.  Returns the count used."""
    os.environ["OMP_NUM_THREADS"] = str(cores)
    from oracle import oracle as orc
    return orc.set_threads(cores)


def _time_cpu(one, reps, warmup):
    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(reps):
        one()
    return time.perf_counter() - t0


# ================================================= the reference's own fp32 CPU path
# Runs in a child process whose import path holds only the reference toolkit installed in
# baseline/_ref (its `csn` package would otherwise meet this repository's drop-in `csn`).
_REF_CPU_SCRIPT = r"""
import json, sys, time
sys.path.insert(0, sys.argv[1])
import torch
from csn import rotors as rr, scan as rs
threads = int(sys.argv[2])
torch.set_num_threads(threads)
B, T, N, D = map(int, sys.argv[3:7])
dev = torch.device(sys.argv[7])
K = D * (D - 1) // 2
g = torch.Generator().manual_seed(0)
gens = torch.randn(B, T, N, K, generator=g).to(dev)
dt = (torch.rand(B, T, generator=g) * 0.02 + 0.04).to(dev)
gamma = torch.nn.functional.softplus(torch.randn(B, T, N, generator=g) * 0.5).to(dev)
S = torch.randn(B, T, N, D, D, generator=g).to(dev)
dX = torch.randn(B, T, N, D, D, generator=g).to(dev)
iu = torch.triu_indices(D, D, 1).to(dev)

def step(scan):
    gg, dd, ga, SS = (t.clone().requires_grad_(True) for t in (gens, dt, gamma, S))
    skew = torch.zeros(B, T, N, D, D, device=dev)
    skew[..., iu[0], iu[1]] = gg
    skew[..., iu[1], iu[0]] = -gg
    h = (0.5 * dd)[:, :, None, None, None]
    Q = rr.cayley_rotor_8x8(skew * h, use_schulz=False)
    a = torch.sigmoid(-ga * dd[:, :, None])[..., None, None]
    X = scan(torch.sqrt(a) * Q, (1 - a) * SS)
    X.backward(dX)

def clock():
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    return time.perf_counter()

out = {}
for name, scan in (("tree_two_sided", lambda M, C: rs._parallel_tree_scan(M, C, is_spinor_bundle=False)),
                   ("sequential_one_sided", lambda M, C: rs.CliffordScanFunction.apply(M, C))):
    step(scan)  # warm-up
    t0 = clock()
    step(scan)
    out[name] = B * T * N / (clock() - t0) / 1e9
model = ""
try:
    for line in open("/proc/cpuinfo"):
        if line.startswith("model name"):
            model = line.split(":", 1)[1].strip()
            break
except OSError:
    pass
print(json.dumps({"gelem_s": out, "threads": threads, "cpu": model}))
"""


def reference_fp32_cpu(cores, B=4, T=2048, N=8, D=8, timeout=600, device="cpu"):
    """The reference toolkit's own scan path (baseline/_ref: csn.rotors.cayley_rotor_8x8 with
    use_schulz=False, decay, then csn.scan's two-sided tree _parallel_tree_scan and the one-sided
    sequential CliffordScanFunction), fp32, forward + backward by autograd, on the Cl(6) LM
    configuration (a slice of it on the host) with all host threads, or on `device` (its torch
    code on the GPU).  On any failure: the reason."""
    import subprocess
    ref = REPO / "baseline" / "_ref"
    if not (ref / "csn" / "scan.py").exists():
        return {"unavailable": "the reference toolkit is not installed in baseline/_ref"}
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1", OMP_NUM_THREADS=str(cores), PYTHONPATH=str(ref))
    try:
        r = subprocess.run([sys.executable, "-c", _REF_CPU_SCRIPT, str(ref), str(cores), str(B), str(T), str(N),
                            str(D), device], capture_output=True, text=True, timeout=timeout, cwd=str(ref), env=env)
        if r.returncode != 0:
            return {"unavailable": (r.stderr.strip().splitlines() or ["failed"])[-1][:200]}
        d = json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as e:  # noqa: BLE001 -- a baseline that cannot run must not fail the bench
        return {"unavailable": repr(e)[:200]}
    res = {"unit": UNIT, "value_tree_two_sided": d["gelem_s"]["tree_two_sided"],
           "value_sequential_one_sided": d["gelem_s"]["sequential_one_sided"], "kind": "reference", "dtype": "f32",
           "sample": f"B{B} L{T} C{N} D{D}, Cayley + decay + scan, forward + backward (autograd), one timed "
                     f"step after one warm-up, the reference toolkit's torch code on {device}"}
    if device == "cpu":
        res.update(cores=d["threads"], cpu=d["cpu"])
    return res


# =============================================================================== workloads
class E2EPipeline:
    """End-to-end step through the public op API, pipelined over pieces of the step.

    Each piece (a layer and/or a slice of the batch) is copied host -> device on one
    stream, run forward + backward on a second, and its outputs copied device -> host on
    a third, so the PCIe transfers of neighbouring pieces (full duplex) overlap each other
    and the compute.  Device input buffers form a ring of `depth` slots; a slot is
    refilled only after the compute that read it has finished.  The op's output tensors
    stay referenced until the step's copies have reached the host (one synchronize per
    step: the step's results are then on the host), so no block is handed across
    streams to the caching allocator."""

    def __init__(self, pieces, run, dev, depth=2):
        import torch
        self.pieces, self.run, self.dev = pieces, run, dev
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream(dev) for _ in range(3))
        shapes = pieces[0][0]
        self.ring = [{k: torch.empty_like(v, device=dev) for k, v in shapes.items()} for _ in range(depth)]
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.done = [torch.cuda.Event() for _ in range(depth)]
        for ev in self.done:
            ev.record(torch.cuda.current_stream(dev))

    def step(self):
        import torch
        keep = []
        for i, (hin, hout) in enumerate(self.pieces):
            slot = i % len(self.ring)
            buf = self.ring[slot]
            with torch.cuda.stream(self.s_in):
                self.s_in.wait_event(self.done[slot])
                for k, v in hin.items():
                    buf[k].copy_(v, non_blocking=True)
                self.ready[slot].record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self.ready[slot])
                outs = self.run(buf)
                self.done[slot].record(self.s_comp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.done[slot])
                for k, v in outs.items():
                    hout[k].copy_(v, non_blocking=True)
            keep.append(outs)
        self.s_out.synchronize()
        del keep


def _batch_pieces(host_in, host_out, nslice):
    """Split pinned host dicts along the batch (outermost) axis into `nslice` pieces."""
    B = next(iter(host_in.values())).shape[0]
    step = B // nslice
    sl = lambda d, j: {k: v[j * step:(j + 1) * step] for k, v in d.items()}
    return [(sl(host_in, j), sl(host_out, j)) for j in range(nslice)]


class Cl6LM:
    """4 layers of the Cl(6,0) LM scan section, forward + backward."""
    name = "cl6_lm_scan_fwd_bwd"
    T, N, D, K = 2048, 8, 8, 28

    def __init__(self, batch=32, layers=4):
        self.B, self.layers = batch, layers
        n, k, N = self.D * self.D, self.K, self.N
        # compulsory HBM bytes per element (float32), dt amortised over the channels
        self.op_bytes = 4.0 * (5 * n + 3 * k + 3 + 3.0 / N)
        self.kernel_bytes = {
            "fwd_apply": 4.0 * (k + 2 * n + 1 + 1.0 / N),      # gens, S, gamma, dt -> X
            "fwd_reduce": 4.0 * (k + n + 1 + 1.0 / N),         # gens, S, gamma, dt
            "bwd_reduce": 4.0 * (n + k + 1 + 1.0 / N),         # dX, gens, gamma, dt
            "bwd_apply": 4.0 * (3 * n + 2 * k + 2 + 2.0 / N),  # dX, X, gens, gamma, dt -> dS, dgens, dgamma, ddt
        }
        # DRAM bytes per element of one launch measured with ncu (dram__bytes_read.sum +
        # dram__bytes_write.sum) on this workload's kernels at B32 L2048 C8: 639.6 MB for the
        # 524,288 elements of one backward apply launch (the S re-read for the decay gradient
        # is the part above the algorithmic bytes)
        self.kernel_traffic = {"bwd_apply": 639.6e6 / 524288}
        self.kernel_names = ["fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry",
                             "bwd_apply", "reduce_channels"]
        self.elems_per_step = self.B * self.T * N * layers
        self.config = {"workload": self.name, "batch": self.B, "seq_len": self.T, "channels": N,
                       "matrix_dim": self.D, "generators": k, "layers": layers, "algebra": "Cl(6,0)",
                       "sided": "two", "damped": True,
                       "l2": "inputs larger than L2 (195 MB per layer forward)"}

    def _host_inputs(self, seed, batch):
        import torch
        g = torch.Generator(device="cpu").manual_seed(seed)
        out = []
        for _ in range(self.layers):
            out.append(dict(
                gens=torch.randn(batch, self.T, self.N, self.K, generator=g),
                dt=torch.rand(batch, self.T, generator=g) * 0.02 + 0.04,
                gamma=torch.nn.functional.softplus(torch.randn(batch, self.T, self.N, generator=g) * 0.5),
                S=torch.randn(batch, self.T, self.N, self.D, self.D, generator=g),
                dX=torch.randn(batch, self.T, self.N, self.D, self.D, generator=g)))
        return out

    def setup(self, dev, rank, lib):
        import torch
        self.dev = dev
        self.inputs = [{k: v.to(dev) for k, v in L.items()} for L in self._host_inputs(1234 + rank, self.B)]
        self.outs = [dict(X=torch.empty_like(L["S"]), dgens=torch.empty_like(L["gens"]),
                          ddt=torch.empty_like(L["dt"]), dgamma=torch.empty_like(L["gamma"]),
                          dS=torch.empty_like(L["S"])) for L in self.inputs]
        self.ws_bytes = lib.csn_rotor_scan_workspace_bytes(self.B, self.T, self.N, self.D)
        self.work = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)

    def step(self, stream):
        from csn_b200 import _lib
        sp = ctypes.c_void_p(stream.cuda_stream)
        B, T, N, D = self.B, self.T, self.N, self.D
        for L, O in zip(self.inputs, self.outs):
            _lib.call("csn_rotor_scan_fwd", _p(L["gens"]), _p(L["dt"]), _p(L["gamma"]), _p(L["S"]),
                      _p(None), _p(O["X"]), B, T, N, D, 0, 1, _p(self.work), self.ws_bytes, sp)
            # the op's path: the backward reuses the chunk rotor products its forward left
            _lib.call("csn_rotor_scan_bwd_reuse", _p(L["gens"]), _p(L["dt"]), _p(L["gamma"]), _p(L["S"]),
                      _p(None), _p(O["X"]), _p(L["dX"]), _p(O["dgens"]), _p(O["ddt"]), _p(O["dgamma"]),
                      _p(O["dS"]), _p(None), B, T, N, D, 0, 1, _p(self.work), self.ws_bytes, sp)

    def e2e_setup(self):
        import torch
        self.host = [{k: v.cpu().pin_memory() for k, v in L.items()} for L in self.inputs]
        self.hout = [{k: torch.empty_like(v, device="cpu").pin_memory() for k, v in O.items()}
                     for O in self.outs]
        h2d = sum(v.numel() * v.element_size() for Lh in self.host for v in Lh.values())
        d2h = sum(v.numel() * v.element_size() for Ho in self.hout for v in Ho.values())
        # 8 batch slices per layer through a 4-deep ring: 31.1 ms per step against 33.2 with 2
        # slices and 2 slots (shorter pipeline fill and drain; both PCIe directions stay busy)
        pieces = [pc for Lh, Ho in zip(self.host, self.hout) for pc in _batch_pieces(Lh, Ho, 8)]
        self.pipe = E2EPipeline(pieces, self.e2e_run, self.dev, depth=4)
        return h2d, d2h

    @staticmethod
    def e2e_run(d):
        from csn_b200 import ops
        gens, dt, gamma, S = (d[k].detach().requires_grad_(True) for k in ("gens", "dt", "gamma", "S"))
        X = ops.fused_rotor_scan(gens, dt, gamma, S)
        X.backward(d["dX"])
        return dict(X=X.detach(), dgens=gens.grad, ddt=dt.grad, dgamma=gamma.grad, dS=S.grad)

    def e2e_step(self):
        self.pipe.step()

    def cpu_reference(self, reps, warmup, sample_batch=8):
        import numpy as np
        from csn_b200 import algebra
        from oracle import oracle as orc
        E = algebra.triu_basis(self.D)
        rng = np.random.default_rng(0)
        gens = rng.standard_normal((sample_batch, self.T, self.N, self.K))
        dt = rng.uniform(0.04, 0.06, (sample_batch, self.T))
        gamma = np.log1p(np.exp(rng.standard_normal((sample_batch, self.T, self.N)) * 0.5))
        S = rng.standard_normal((sample_batch, self.T, self.N, self.D, self.D))
        dX = rng.standard_normal((sample_batch, self.T, self.N, self.D, self.D))

        def one():
            X = orc.rotor_scan_fwd(gens, dt, gamma, S, E)
            orc.rotor_scan_bwd(gens, dt, gamma, S, E, X, dX)

        el = _time_cpu(one, reps, warmup)
        return (sample_batch * self.T * self.N * reps, el,
                f"one layer at batch {sample_batch} of {self.B} (B{sample_batch} L{self.T} C{self.N} "
                f"D{self.D}) per step, fwd+bwd, float64 C oracle, OpenMP")


class Cl3:
    """Cl(3,0) blade-basis scan at the bandwidth scale (B64 L65536 C16), fwd + bwd."""
    name = "cl3_ga_scan_fwd_bwd"
    T, N = 65536, 16

    def __init__(self, batch=64, layers=1):
        self.B = batch
        N = self.N
        # fwd reads gens (3) + x (8) + dt, writes h (8); bwd reads dh, h_{t-1}, gens, dt and
        # writes dx, dgens, ddt
        self.op_bytes = 4.0 * ((3 + 16 + 1.0 / N) + (8 + 8 + 3 + 8 + 3 + 2.0 / N))
        self.kernel_bytes = {
            "ga3_fwd_apply": 4.0 * (3 + 8 + 8 + 1.0 / N),
            "ga3_fwd_reduce": 4.0 * (3 + 8 + 1.0 / N),
            "ga3_bwd_reduce": 4.0 * (8 + 3 + 1.0 / N),
            "ga3_bwd_apply": 4.0 * (8 + 8 + 3 + 1.0 / N + 8 + 3 + 1),
        }
        # DRAM bytes per element of the backward apply, measured with ncu (dram__bytes.sum.per_second
        # x gpu__time_duration.sum) on this kernel at B4 L65536 C16: 494.0 MB for 4,194,304 elements
        self.kernel_traffic = {"ga3_bwd_apply": 494.0e6 / 4194304}
        self.kernel_names = ["ga3_fwd_reduce", "ga3_fwd_carry", "ga3_fwd_apply", "ga3_bwd_reduce",
                             "ga3_bwd_carry", "ga3_bwd_apply", "ga3_reduce_channels"]
        self.elems_per_step = self.B * self.T * N
        self.config = {"workload": self.name, "batch": self.B, "seq_len": self.T, "channels": N,
                       "multivector": 8, "rotor": 4, "algebra": "Cl(3,0)", "sided": "two",
                       "l2": "inputs larger than L2 (2.9 GB forward)"}

    def _host(self, seed, batch):
        import torch
        g = torch.Generator(device="cpu").manual_seed(seed)
        return dict(gens=torch.randn(batch, self.T, self.N, 3, generator=g) * 0.1,
                    dt=torch.rand(batch, self.T, generator=g) * 0.09 + 0.01,
                    x=torch.randn(batch, self.T, self.N, 8, generator=g),
                    dh=torch.randn(batch, self.T, self.N, 8, generator=g))

    def setup(self, dev, rank, lib):
        import torch
        self.dev = dev
        self.inp = {k: v.to(dev) for k, v in self._host(99 + rank, self.B).items()}
        self.out = dict(h=torch.empty_like(self.inp["x"]), dx=torch.empty_like(self.inp["x"]),
                        dgens=torch.empty_like(self.inp["gens"]), ddt=torch.empty_like(self.inp["dt"]))
        self.ws_bytes = lib.csn_ga3_workspace_bytes(self.B, self.T, self.N)
        self.work = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)

    def step(self, stream):
        from csn_b200 import _lib
        sp = ctypes.c_void_p(stream.cuda_stream)
        I, O = self.inp, self.out
        _lib.call("csn_ga3_scan_fwd", _p(I["gens"]), _p(I["dt"]), _p(I["x"]), _p(None), _p(O["h"]),
                  self.B, self.T, self.N, _p(self.work), self.ws_bytes, sp)
        _lib.call("csn_ga3_scan_bwd", _p(I["gens"]), _p(I["dt"]), _p(None), _p(O["h"]), _p(I["dh"]),
                  _p(O["dgens"]), _p(O["ddt"]), _p(O["dx"]), _p(None), self.B, self.T, self.N,
                  _p(self.work), self.ws_bytes, sp)

    def e2e_setup(self):
        import torch
        self.host = {k: v.cpu().pin_memory() for k, v in self.inp.items()}
        self.hout = {k: torch.empty_like(v, device="cpu").pin_memory() for k, v in self.out.items()}
        self.pipe = E2EPipeline(_batch_pieces(self.host, self.hout, 8), self.e2e_run, self.dev)
        return (sum(v.numel() * v.element_size() for v in self.host.values()),
                sum(v.numel() * v.element_size() for v in self.hout.values()))

    @staticmethod
    def e2e_run(d):
        from csn_b200 import ops
        gens, dt, x = (d[k].detach().requires_grad_(True) for k in ("gens", "dt", "x"))
        h = ops.ga3_rotor_scan(gens, dt, x)
        h.backward(d["dh"])
        return dict(h=h.detach(), dx=x.grad, dgens=gens.grad, ddt=dt.grad)

    def e2e_step(self):
        self.pipe.step()

    def cpu_reference(self, reps, warmup, sample_batch=4):
        from oracle import oracle as orc
        a = {k: v.double().numpy() for k, v in self._host(5, sample_batch).items()}

        def one():
            hh = orc.ga3_scan_fwd(a["gens"], a["dt"], a["x"])
            orc.ga3_scan_bwd(a["gens"], a["dt"], hh, a["dh"])

        el = _time_cpu(one, reps, warmup)
        return (sample_batch * self.T * self.N * reps, el,
                f"batch {sample_batch} of {self.B} (B{sample_batch} L{self.T} C{self.N}) per step, "
                f"fwd+bwd, float64 C oracle, OpenMP")


class Cl8:
    """Cl(8,0) ~ M_16(R) rotor scan (B16 L8192 C32), fwd + bwd: 28 GA bivector-blade
    generators mapped through rho, undamped (h_t = R h R~ + x_t)."""
    name = "cl8_rotor_scan_fwd_bwd"
    T, N, D, K = 8192, 32, 16, 28

    def __init__(self, batch=16, layers=1):
        self.B = batch
        n, k, N = self.D * self.D, self.K, self.N
        self.op_bytes = 4.0 * ((k + 2 * n + 1.0 / N) + (n + n + k + 1.0 / N + n + k + 1.0 / N))
        self.kernel_bytes = {
            "fwd_apply": 4.0 * (k + 2 * n + 1.0 / N),
            "fwd_reduce": 4.0 * (k + n + 1.0 / N),
            "bwd_reduce": 4.0 * (n + k + 1.0 / N),
            "bwd_apply": 4.0 * (3 * n + 2 * k + 2.0 / N + 1),
        }
        # DRAM bytes per element of the backward apply, measured with ncu (dram__bytes_read.sum +
        # dram__bytes_write.sum) at B2 L8192 C32: 1684.2 MB + 575.9 MB for 524,288 elements (the
        # cached rotor, 1 KB per element, is the part above the algorithmic bytes)
        self.kernel_traffic = {"bwd_apply": 2260.1e6 / 524288}
        self.kernel_names = ["fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry",
                             "bwd_apply", "reduce_channels"]
        self.elems_per_step = self.B * self.T * N
        self.config = {"workload": self.name, "batch": self.B, "seq_len": self.T, "channels": N,
                       "matrix_dim": self.D, "generators": k, "basis": "GA bivector blades via rho",
                       "algebra": "Cl(8,0)", "sided": "two", "damped": False,
                       "l2": "inputs larger than L2 (4.3 GB per tensor)"}

    def _host(self, seed, batch):
        import torch
        g = torch.Generator(device="cpu").manual_seed(seed)
        return dict(gens=torch.randn(batch, self.T, self.N, self.K, generator=g) * 0.05,
                    dt=torch.rand(batch, self.T, generator=g) * 0.045 + 0.005,
                    S=torch.randn(batch, self.T, self.N, self.D, self.D, generator=g),
                    dX=torch.randn(batch, self.T, self.N, self.D, self.D, generator=g))

    def setup(self, dev, rank, lib):
        import torch
        self.dev = dev
        self.inp = {k: v.to(dev) for k, v in self._host(7 + rank, self.B).items()}
        self.out = dict(X=torch.empty_like(self.inp["S"]), dS=torch.empty_like(self.inp["S"]),
                        dgens=torch.empty_like(self.inp["gens"]), ddt=torch.empty_like(self.inp["dt"]))
        self.Mc = torch.empty_like(self.inp["S"])  # rotor cache
        self.ws_bytes = lib.csn_rotor_scan_workspace_bytes(self.B, self.T, self.N, self.D)
        self.work = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)

    def step(self, stream):
        from csn_b200 import _lib
        sp = ctypes.c_void_p(stream.cuda_stream)
        I, O = self.inp, self.out
        B, T, N, D = self.B, self.T, self.N, self.D
        # the op's D = 16 path: rotors stored by the forward, reused by the backward
        _lib.call("csn_rotor_scan_fwd_cached", _p(I["gens"]), _p(I["dt"]), _p(None), _p(I["S"]), _p(None),
                  _p(O["X"]), _p(self.Mc), B, T, N, D, 1, 1, _p(self.work), self.ws_bytes, sp)
        # the op's path: the backward loads the cached rotors and reuses the chunk products the
        # forward left in the workspace (one head: the [B, T, N] layout)
        _lib.call("csn_rotor_scan_heads_bwd", _p(I["gens"]), _p(I["dt"]), _p(None), _p(I["S"]), _p(None),
                  _p(O["X"]), _p(I["dX"]), _p(self.Mc), _p(O["dgens"]), _p(O["ddt"]), _p(None), _p(O["dS"]),
                  _p(None), B, T, 1, N, D, 1, 1, 1, _p(self.work), self.ws_bytes, sp)

    def e2e_setup(self):
        import torch
        self.host = {k: v.cpu().pin_memory() for k, v in self.inp.items()}
        self.hout = {k: torch.empty_like(v, device="cpu").pin_memory() for k, v in self.out.items()}
        self.pipe = E2EPipeline(_batch_pieces(self.host, self.hout, 4), self.e2e_run, self.dev)
        return (sum(v.numel() * v.element_size() for v in self.host.values()),
                sum(v.numel() * v.element_size() for v in self.hout.values()))

    @staticmethod
    def e2e_run(d):
        from csn_b200 import ops
        gens, dt, S = (d[k].detach().requires_grad_(True) for k in ("gens", "dt", "S"))
        X = ops.fused_rotor_scan(gens, dt, None, S, basis="ga")
        X.backward(d["dX"])
        return dict(X=X.detach(), dS=S.grad, dgens=gens.grad, ddt=dt.grad)

    def e2e_step(self):
        self.pipe.step()

    def cpu_reference(self, reps, warmup, sample_batch=1):
        import numpy as np
        from csn_b200 import algebra
        from oracle import oracle as orc
        E = algebra.bivector_basis(algebra.CL8)
        h = self._host(3, sample_batch)
        a = {k: v.double().numpy()[:, :, :4] if v.dim() > 2 else v.double().numpy() for k, v in h.items()}

        def one():
            X = orc.rotor_scan_fwd(a["gens"], a["dt"], None, a["S"], E)
            orc.rotor_scan_bwd(a["gens"], a["dt"], None, a["S"], E, X, a["dX"])

        el = _time_cpu(one, reps, warmup)
        return (sample_batch * self.T * 4 * reps, el,
                f"full-L slice B{sample_batch} L{self.T} C4 (of C{self.N}) per step, fwd+bwd, "
                f"float64 C oracle, OpenMP")


WORKLOADS = {"cl6_lm": Cl6LM, "cl3": Cl3, "cl8": Cl8}


SP_KERNELS = ("agg_fwd_reduce", "agg_bwd_reduce", "agg_compose", "fwd_reduce", "fwd_carry", "fwd_apply",
              "bwd_reduce", "bwd_carry", "bwd_apply", "reduce_channels")


def run_sequence_parallel(args, ws, rank, local, cores):
    """Sequence-parallel long scan, Cl(6,0) 8 x 8, undamped: B 8, L 2^20, C 64
    (gens ~ N(0, 0.02^2), dt ~ U(0.001, 0.01), x ~ N(0, 1)), forward + backward.  The time
    axis is split over the ranks (strong scaling): each rank aggregates its shard, the
    (P, c) pairs are all-gathered over NCCL, and the shard resumes from its carry-in; the
    backward mirrors it with the gradient carries.  Channels run in slabs of min(64, 8 * ranks)
    so that every rank holds ~84 GB (inputs, trajectory, incoming and outgoing gradients);
    the slabs reuse one set of buffers."""
    B, L, C, D, K = 8, 1 << 20, 64, 8, 28
    Tl = L // ws
    cs = min(C, 8 * ws)
    nslab = C // cs
    config = {"workload": "cl6_sequence_parallel_fwd_bwd", "batch": B, "seq_len": L, "channels": C,
              "matrix_dim": D, "algebra": "Cl(6,0)", "damped": False, "ranks": ws,
              "shard_len": Tl, "channel_slab": cs, "partition": "time axis, one shard per rank",
              "exchange": "all-gather of (P, c) forward and of c' backward per slab (NCCL)",
              "l2": "inputs larger than L2"}
    elems = B * L * C
    n = D * D
    op_bytes = 4.0 * (5 * n + 3 * K + 3.0 / C)  # fwd: gens, S -> X; bwd: gens, X, dX -> dS, dgens
    if args.impl == "reference":
        if rank != 0:
            return 0
        from csn_b200 import algebra
        from oracle import oracle as orc
        cores = _cpu_threads(cores)
        E = algebra.triu_basis(D)
        rng = np.random.default_rng(0)
        Ts, Cs = 8192, min(C, max(4, cores))  # one full-length-8192 sequence per host thread
        cores = min(cores, Cs)
        gs, dts, Ss = (rng.standard_normal((1, Ts, Cs, K)) * 0.02, rng.uniform(0.001, 0.01, (1, Ts)),
                       rng.standard_normal((1, Ts, Cs, D, D)))
        dXs = rng.standard_normal((1, Ts, Cs, D, D))

        def ref_step():
            X = orc.rotor_scan_fwd(gs, dts, None, Ss, E)
            orc.rotor_scan_bwd(gs, dts, None, Ss, E, X, dXs)

        steps = max(1, args.steps)
        el = _time_cpu(ref_step, steps, 0)
        v = Ts * Cs * steps / el / 1e9
        print(json.dumps({"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
                          "warmup": 0, "ms_per_step": el / steps * 1e3, "higher_is_better": True,
                          "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                          "config": config, "impl": "reference",
                          "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                           "sample": f"B1 L{Ts} C{Cs} slice, fwd+bwd, float64 C oracle"},
                          "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    import torch
    from csn_b200 import _lib, ops
    from csn_b200 import sequence_parallel as spm
    from csn_b200.sequence_parallel import CudaBackend, sp_backward, sp_forward
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _lib.load()
    g = torch.Generator(device=dev).manual_seed(17 + rank)
    gens = torch.randn(B, Tl, cs, K, device=dev, generator=g) * 0.02
    dt = torch.rand(B, Tl, device=dev, generator=g) * 0.009 + 0.001
    S = torch.randn(B, Tl, cs, D, D, device=dev, generator=g)
    dX = torch.randn(B, Tl, cs, D, D, device=dev, generator=g)
    be = CudaBackend()

    def step():
        for _ in range(nslab):
            if ws > 1:
                X, h_in, Ps = sp_forward(gens, dt, None, S, None, be, "triu", True)
                sp_backward(gens, dt, None, S, X, dX, h_in, Ps, None, be, "triu", True)
            else:
                X = be.rotor_fwd(gens, dt, None, S, None, "triu", True)
                be.rotor_bwd(gens, dt, None, S, None, X, dX, "triu", True)
            del X

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps)
    _lib.timing_reset()
    _lib.timing_enable(True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    _lib.timing_enable(False)
    if ws > 1:
        spm.check()  # the last exchange's finiteness verdict
    kt = {k: _lib.timing_read(k) for k in SP_KERNELS}
    barrier()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    ms_step = ms / steps
    value = elems / (ms_step * 1e-3) / 1e9
    hbm, peak_kind = peaks()
    # dominant kernel's roofline: algorithmic bytes per element of each pass (undamped:
    # no gamma), elements of one launch = this rank's slab
    kbytes = {"agg_fwd_reduce": 4.0 * (K + n + 1.0 / cs), "fwd_reduce": 4.0 * (K + n + 1.0 / cs),
              "fwd_apply": 4.0 * (K + 2 * n + 1.0 / cs), "agg_bwd_reduce": 4.0 * (n + K + 1.0 / cs),
              "bwd_reduce": 4.0 * (n + K + 1.0 / cs), "bwd_apply": 4.0 * (3 * n + 2 * K + 1 + 1.0 / cs)}
    dom = max((k for k in kbytes if kt[k][1]), key=lambda k: kt[k][0])
    dom_ms = kt[dom][0] / kt[dom][1]
    dom_ach = kbytes[dom] * (B * Tl * cs) / (dom_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": dom, "achieved": dom_ach, "peak": hbm, "unit": "GB/s",
                "frac": dom_ach / hbm, "traffic": None, "peak_kind": peak_kind,
                "bytes_per_elem": kbytes[dom], "avg_launch_ms": dom_ms}
    _lib.timing_reset()
    # end to end through the public ops: every step, every slab's inputs (gens, dt, S, dX)
    # copied from pinned host memory and its outputs (X, dgens, ddt, dS) copied back.  The
    # host side is a 1 GiB pinned staging buffer per direction that the copies cycle through
    # (the bytes moved per step are those of the full tensors).
    e2e = None
    if args.e2e_steps > 0:
        stage_in = torch.randn(1 << 28).pin_memory()
        stage_out = torch.empty(1 << 28).pin_memory()

        def h2d(t):
            f = t.view(-1)
            for o in range(0, f.numel(), stage_in.numel()):
                m = min(stage_in.numel(), f.numel() - o)
                f[o:o + m].copy_(stage_in[:m], non_blocking=True)
            return t.numel() * 4

        def d2h(t):
            f = t.reshape(-1)
            for o in range(0, f.numel(), stage_out.numel()):
                m = min(stage_out.numel(), f.numel() - o)
                stage_out[:m].copy_(f[o:o + m], non_blocking=True)
            return t.numel() * 4

        def e2e_step():
            hb = db = 0
            for _ in range(nslab):
                for t in (gens, dt, S, dX):
                    hb += h2d(t)
                gd, dd, Sd = (t.detach().requires_grad_(True) for t in (gens, dt, S))
                if ws > 1:
                    X = spm.sequence_parallel_rotor_scan(gd, dd, None, Sd)
                else:
                    X = ops.fused_rotor_scan(gd, dd, None, Sd)
                X.backward(dX)
                for t in (X.detach(), gd.grad, dd.grad, Sd.grad):
                    db += d2h(t)
                del X, gd, dd, Sd
            torch.cuda.current_stream(dev).synchronize()
            return hb, db

        k_e2e = min(args.e2e_steps, 1)  # one step moves the whole problem over PCIe (~80 GB per GPU)
        barrier()
        t0 = time.perf_counter()
        for _ in range(k_e2e):
            h2d_b, d2h_b = e2e_step()
        el = time.perf_counter() - t0
        if ws > 1:
            spm.check()
            t = torch.tensor([el], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            el = t.item()
        e2e = {"value": elems * k_e2e / el / 1e9, "unit": UNIT, "h2d_bytes_per_step": h2d_b,
               "d2h_bytes_per_step": d2h_b,
               "timing": "wall clock around K steps: every slab's inputs pinned host -> device, the "
                         "sequence-parallel autograd op forward + backward, outputs -> pinned host, one "
                         "stream synchronize per step, max over ranks"}
        del stage_in, stage_out
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from csn_b200 import algebra
        from oracle import oracle as orc
        cores = _cpu_threads(cores)
        E = algebra.triu_basis(D)
        rng = np.random.default_rng(0)
        Ts, Cs = 8192, min(C, max(4, cores))
        cores = min(cores, Cs)
        a = (rng.standard_normal((1, Ts, Cs, K)) * 0.02, rng.uniform(0.001, 0.01, (1, Ts)),
             rng.standard_normal((1, Ts, Cs, D, D)))
        dXs = rng.standard_normal((1, Ts, Cs, D, D))

        def ref_step():
            Xr = orc.rotor_scan_fwd(a[0], a[1], None, a[2], E)
            orc.rotor_scan_bwd(a[0], a[1], None, a[2], E, Xr, dXs)

        cel = _time_cpu(ref_step, 2, 0)
        cpu = {"value": Ts * Cs * 2 / cel / 1e9, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"B1 L{Ts} C{Cs} slice per sample, fwd+bwd, float64 C oracle, OpenMP"}
    if rank == 0:
        ach = op_bytes * elems / ws / (ms_step * 1e-3) / 1e9
        print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT,
                          "n_gpus": ws, "steps": steps, "warmup": max(3, args.warmup),
                          "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": dict(config, parallelism=f"sequence{ws}"),
                          "roofline": roofline,
                          "op_roofline": {"achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                          "bytes_per_elem": op_bytes, "note": "per rank"},
                          "kernel_ms_per_step": {k: v[0] / steps for k, v in kt.items() if v[1]},
                          "gpu_launches": sum(v[1] for v in kt.values()),
                          "clocks": clk.summary(), "e2e": e2e, "cpu_baseline": cpu}), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_generation(args, ws, rank, local, cores):
    """Autoregressive O(1)-state generation, Cl(6,0): 256 streams x 8 channels, 8 x 8 state,
    one rotor step per token (gens ~ N(0, 0.1^2), dt ~ U(0.01, 0.1), damped).  Reports the
    p50 per-step latency of graph-replayed steps and tokens/s = streams / latency."""
    import numpy as np
    B, N, D, chunk, total = 256, 8, 8, 128, 2048
    config = {"workload": "cl6_generation_step", "streams": B, "channels": N, "matrix_dim": D,
              "steps": total, "graph_steps": chunk, "algebra": "Cl(6,0)", "damped": True}
    metric = "rotor-step p50 latency (us), 256 streams x 8 channels Cl(6,0)"
    if args.impl == "reference":
        if rank != 0:
            return 0
        from csn_b200 import algebra
        from oracle import oracle as orc
        cores = _cpu_threads(cores)
        E = algebra.triu_basis(D)
        rng = np.random.default_rng(0)
        h = np.zeros((B, N, D, D))
        lat = []
        for _ in range(max(1, args.steps)):
            g = rng.standard_normal((B, 1, N, 28)) * 0.1
            dt = rng.uniform(0.01, 0.1, (B, 1))
            gam = np.log1p(np.exp(rng.standard_normal((B, 1, N))))
            S = rng.standard_normal((B, 1, N, D, D))
            t0 = time.perf_counter()
            h = orc.rotor_scan_fwd(g, dt, gam, S, E, h0=h)[:, 0]
            lat.append((time.perf_counter() - t0) * 1e6)
        p50 = float(np.median(lat))
        print(json.dumps({"metric": metric, "value": p50, "unit": "us", "n_gpus": 1, "steps": args.steps,
                          "warmup": 0, "ms_per_step": p50 / 1e3, "higher_is_better": False,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                          "config": config, "impl": "reference", "tok_per_s": B / (p50 * 1e-6),
                          "cpu_baseline": {"value": p50, "unit": "us", "cores": cores, "kind": "port",
                                           "sample": "one step of 256 x 8 streams per sample, float64 C oracle"},
                          "e2e": {"value": p50, "unit": "us", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    import torch
    from csn_b200 import _lib, ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _lib.load()
    reps = total // chunk
    # value: steps launched as an autoregressive loop must (each waits for the previous step);
    # chained: the same graph with the next step's rotor built during the previous step, valid
    # when the step inputs are staged ahead (RotorStepGraph's default)
    lat, lat_chained = [], []
    with ClockSampler(local) as clk:
        for chained, out in ((False, lat), (True, lat_chained)):
            g = _gen_graph(B, N, D, chunk, dev, chained)
            for _ in range(max(3, args.warmup)):
                g.replay()
            torch.cuda.synchronize()
            for _ in range(max(reps, args.steps)):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                e1.synchronize()
                out.append(e0.elapsed_time(e1) * 1e3 / chunk)
    p50 = float(np.median(lat))
    # eager: one launch per step from the host (includes the host launch path)
    eager = []
    h = torch.zeros(B, N, D, D, device=dev)
    for t in range(64):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.rotor_step(g.gens[t % chunk], g.dt[t % chunk], g.gamma[t % chunk], g.S[t % chunk], h)
        e1.record()
        e1.synchronize()
        eager.append(e0.elapsed_time(e1) * 1e3)
    # end to end: pinned host inputs -> device, step, state back to host, per token
    hin = {k: v[0].cpu().pin_memory() for k, v in (("gens", g.gens), ("dt", g.dt), ("gamma", g.gamma),
                                                  ("S", g.S))}
    hout = torch.empty(B, N, D, D).pin_memory()
    e2e_lat = []
    for _ in range(32):
        t0 = time.perf_counter()
        d = {k: v.to(dev, non_blocking=True) for k, v in hin.items()}
        ops.rotor_step(d["gens"], d["dt"], d["gamma"], d["S"], h)
        hout.copy_(h, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        e2e_lat.append((time.perf_counter() - t0) * 1e6)
    h2d = sum(v.numel() * 4 for v in hin.values())
    cpu = None
    if not args.no_cpu_baseline:
        from csn_b200 import algebra
        from oracle import oracle as orc
        cores = _cpu_threads(cores)
        E = algebra.triu_basis(D)
        rng = np.random.default_rng(0)
        hh = np.zeros((B, N, D, D))
        cl = []
        for _ in range(5):
            a = (rng.standard_normal((B, 1, N, 28)) * 0.1, rng.uniform(0.01, 0.1, (B, 1)),
                 np.log1p(np.exp(rng.standard_normal((B, 1, N)))), rng.standard_normal((B, 1, N, D, D)))
            t0 = time.perf_counter()
            hh = orc.rotor_scan_fwd(*a, E, h0=hh)[:, 0]
            cl.append((time.perf_counter() - t0) * 1e6)
        cpu = {"value": float(np.median(cl)), "unit": "us", "cores": cores, "kind": "port",
               "sample": "5 steps of 256 x 8 streams, float64 C oracle"}
    print(json.dumps({
        "metric": metric, "value": p50, "unit": "us", "n_gpus": 1, "steps": len(lat) * chunk,
        "warmup": max(3, args.warmup), "ms_per_step": p50 / 1e3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
        "tok_per_s": B / (p50 * 1e-6), "p50_eager_us": float(np.median(eager)),
        "p50_chained_us": float(np.median(lat_chained)),
        "chained": "steps captured with csn_rotor_step_chained: each step's rotor is built while "
                   "the previous step runs; valid when the step inputs are staged ahead",
        "gpu_launches": (len(lat) + len(lat_chained)) * chunk, "clocks": clk.summary(),
        "e2e": {"value": float(np.median(e2e_lat)), "unit": "us", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": hout.numel() * 4,
                "timing": "wall clock per token: pinned inputs to device, step, state to host"},
        "cpu_baseline": cpu}), flush=True)
    return 0


# The reference's one published scan figure: its fused CUDA one-sided D = 4 scan, forward +
# backward, 5.34 ms per step in csn_toolkit/examples/benchmark_cuda_kernels.py:79-118
# (csn_toolkit/README.md:194, :331; hardware unspecified).
D4_PUBLISHED_MS = 5.34

# The same harness through the reference toolkit's own PyTorch path (its "sequential loop"
# arm, csn_toolkit/examples/benchmark_cuda_kernels.py:96-109), run from baseline/_ref.
_REF_D4_SCRIPT = r"""
import json, sys, time
sys.path.insert(0, sys.argv[1])
import torch
from csn.scan import parallel_rotor_scan
dev = torch.device(sys.argv[3])
torch.set_num_threads(int(sys.argv[4]))
torch.manual_seed(42)
B, T, N, D = 2, 80, 1, 4
M = (0.5 * torch.randn(B, T, N, D, D, device=dev)).contiguous().detach().requires_grad_(True)
C = torch.randn(B, T, N, D, D, device=dev).contiguous().detach().requires_grad_(True)
def one():
    M.grad = None
    C.grad = None
    loss = (parallel_rotor_scan(M, C, backend="pytorch") ** 2).sum()
    loss.backward()
def sync():
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
for _ in range(10):
    one()
sync()
n = int(sys.argv[2])
t = time.perf_counter()
for _ in range(n):
    one()
sync()
print(json.dumps({"ms": (time.perf_counter() - t) / n * 1e3}))
"""


def reference_d4_ms(runs, device, cores, timeout=900):
    """Per-step ms of the reference harness's PyTorch arm (baseline/_ref) on `device`."""
    import subprocess
    ref = REPO / "baseline" / "_ref"
    if not (ref / "csn").is_dir():
        return {"unavailable": "the reference toolkit is not installed in baseline/_ref"}
    try:
        r = subprocess.run([sys.executable, "-c", _REF_D4_SCRIPT, str(ref), str(runs), device, str(cores)],
                           capture_output=True, text=True, timeout=timeout, env=dict(os.environ, PYTHONPATH=str(ref)))
        return json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as e:  # noqa: BLE001 -- a baseline that cannot run must not fail the bench
        return {"unavailable": f"reference harness failed: {type(e).__name__}"}


def run_d4_harness(args, ws, rank, local, cores):
    """The reference's published scan benchmark (csn_toolkit/examples/benchmark_cuda_kernels.py:
    30-118) through this build's drop-in `csn.scan.parallel_rotor_scan(..., backend="cuda")`:
    M, C [B2, T80, N1, 4, 4] (M ~ 0.5 N(0, 1), seed 42), one step = forward, loss = sum(X^2),
    backward; 10 warm-up steps, then the wall-clock mean over the timed steps, as the harness
    times it (it is launch-bound at this size).  vs_baseline = value / the published 5.34 ms."""
    metric = "fused D=4 one-sided scan fwd+bwd ms/step, reference harness B2 T80 N1"
    config = {"workload": "d4_harness", "batch": 2, "seq_len": 80, "channels": 1, "matrix_dim": 4,
              "sided": "one", "harness": "csn_toolkit/examples/benchmark_cuda_kernels.py:30-118",
              "l2": "inputs far below L2 (the harness's own shape; latency-bound)"}
    runs = max(100, args.steps)
    if args.impl == "reference":
        if rank != 0:
            return 0
        cores = _cpu_threads(cores)
        r = reference_d4_ms(max(3, args.steps), "cpu", cores)
        if "ms" not in r:
            print(json.dumps({"impl": "reference", "unavailable": r.get("unavailable", "failed")}), flush=True)
            return 0
        v = r["ms"]
        print(json.dumps({"metric": metric, "value": v, "unit": "ms", "n_gpus": 1, "steps": max(3, args.steps),
                          "warmup": 10, "ms_per_step": v, "higher_is_better": False, "scaling": "weak",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                          "impl": "reference",
                          "cpu_baseline": {"value": v, "unit": "ms", "cores": cores, "kind": "reference",
                                           "sample": "the harness's PyTorch arm (parallel_rotor_scan, "
                                                     "backend='pytorch') on the host cores"},
                          "e2e": {"value": v, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return 0
    if rank != 0:
        return 0
    import torch
    from csn_b200 import _lib
    from csn.scan import parallel_rotor_scan
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _lib.load()
    torch.manual_seed(42)
    B, T, N, D = 2, 80, 1, 4
    M = (0.5 * torch.randn(B, T, N, D, D, device=dev)).contiguous().detach().requires_grad_(True)
    C = torch.randn(B, T, N, D, D, device=dev).contiguous().detach().requires_grad_(True)

    def one(m, c):
        m.grad = None
        c.grad = None
        loss = (parallel_rotor_scan(m, c, backend="cuda") ** 2).sum()
        loss.backward()
        return loss

    for _ in range(max(10, args.warmup)):
        one(M, C)
    torch.cuda.synchronize()
    _lib.timing_reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        _lib.timing_enable(True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(runs):
            one(M, C)
        e1.record()
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - t0) / runs * 1e3
        _lib.timing_enable(False)
    dev_ms = e0.elapsed_time(e1) / runs
    names = ("fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry", "bwd_apply")
    kt = {n: _lib.timing_read(n) for n in names}
    launches = sum(c for _, c in kt.values())
    _lib.timing_reset()
    # end to end: M, C from pinned host memory every step, the loss back to the host
    Mh, Ch = M.detach().cpu().pin_memory(), C.detach().cpu().pin_memory()
    e2e = []
    for _ in range(max(20, args.e2e_steps)):
        t0 = time.perf_counter()
        m = Mh.to(dev, non_blocking=True).requires_grad_(True)
        c = Ch.to(dev, non_blocking=True).requires_grad_(True)
        float(one(m, c))
        torch.cuda.synchronize()
        e2e.append((time.perf_counter() - t0) * 1e3)
    ref_gpu = reference_d4_ms(runs, f"cuda:{local}", 1)
    cpu = None
    if not args.no_cpu_baseline:
        ccores = _cpu_threads(cores)
        r = reference_d4_ms(10, "cpu", ccores)
        if "ms" in r:
            cpu = {"value": r["ms"], "unit": "ms", "cores": ccores, "kind": "reference",
                   "sample": "the harness's PyTorch arm (parallel_rotor_scan, backend='pytorch') on the "
                             "host cores, 10 steps after 10 warm-up steps"}
    print(json.dumps({
        "metric": metric, "value": wall_ms, "unit": "ms", "n_gpus": 1, "steps": runs,
        "warmup": max(10, args.warmup), "ms_per_step": wall_ms, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": wall_ms / D4_PUBLISHED_MS, "dtype": "f32", "data": "synthetic",
        "config": config, "device_ms_per_step": dev_ms,
        "kernel_ms_per_step": {n: t / runs for n, (t, c) in kt.items()},
        "published_ms": D4_PUBLISHED_MS, "reference_pytorch_gpu": ref_gpu,
        "gpu_launches": launches, "clocks": clk.summary(),
        "e2e": {"value": float(np.median(e2e)), "unit": "ms", "h2d_bytes_per_step": 2 * M.numel() * 4,
                "d2h_bytes_per_step": 4,
                "timing": "wall clock per step: M and C from pinned host memory, forward, loss, backward, "
                          "loss to the host"},
        "cpu_baseline": cpu}), flush=True)
    return 0


def run_lm_train(args, ws, rank, local, cores):
    """One training step of the Cl(6,0) LM of the Cl(6) LM config (vocab 65 uniform token ids,
    d_model 128, 4 CliffordCL6Blocks x 8 neurons, B32 L2048, AdamW lr 1e-3): embedding, blocks
    (ln_1 -> causal depthwise conv -> SiLU -> projections -> fused rotor scan -> spike -> mixed
    out_proj -> GGLU), geodesic head, cross entropy + action + time penalties, backward, optimizer
    step, diagnostics read back.  The step is captured once as a CUDA graph (TrainStepGraph) and
    replayed; tokens/s = B * L / step time (CUDA events around K replays).  The eager step time
    is reported beside it."""
    config = {"workload": "cl6_lm_train_step", "batch": args.batch or 32, "seq_len": 2048, "d_model": 128,
              "layers": args.layers or 4, "neurons": 8, "vocab": 65, "optimizer": "AdamW",
              "l2": "inputs larger than L2 (each block's S is 134 MB)"}
    metric = "Cl(6) LM training step tokens/s (fwd + bwd + AdamW)"
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference LM is PyTorch source that "
                              "is not installed where the bench runs; its scan is timed by the cl6_lm "
                              "workload"}), flush=True)
        return 0
    import torch
    from csn_b200 import _lib, graphs
    from python.clifford_cl6 import CliffordCL6ForCausalLM
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _lib.load()
    torch.manual_seed(0)
    B, T = config["batch"], config["seq_len"]
    model = CliffordCL6ForCausalLM(vocab_size=65, d_model=128, num_layers=config["layers"], num_neurons=8).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, capturable=True)
    gen = torch.Generator(device="cpu").manual_seed(0)
    idx_h = torch.randint(0, 65, (B, T), generator=gen).pin_memory()
    tgt_h = torch.randint(0, 65, (B, T), generator=gen).pin_memory()
    idx, tgt = idx_h.to(dev), tgt_h.to(dev)

    def step(i, t):
        opt.zero_grad(set_to_none=True)
        _, loss, diag = model(i, t)
        loss.backward()
        opt.step()
        return diag

    # eager steps first: the per-step launch count and kernel times of this package's kernels
    # (the same kernels run inside the captured step, where they are not timed one by one)
    for _ in range(max(3, args.warmup)):
        step(idx, tgt)
    torch.cuda.synchronize()
    _lib.timing_reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _lib.timing_enable(True)
    e0.record()
    for _ in range(args.steps):
        step(idx, tgt)
    e1.record()
    torch.cuda.synchronize()
    _lib.timing_enable(False)
    eager_ms = e0.elapsed_time(e1) / args.steps
    # the timed step: forward + backward + AdamW captured once as a CUDA graph, replayed
    g = graphs.TrainStepGraph(model, opt, [idx, tgt], warmup=3)
    for _ in range(max(3, args.warmup)):
        g(idx, tgt)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            g(idx, tgt)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # The GEMM that materialises S ([B*T, d_model] x [d_model, N*64]) once per block, timed alone:
    # building S inside the scan instead would redo this work in each of the three scan passes
    # that read S (forward reduce, forward apply, backward apply), to save S's HBM round trips.
    from csn_b200 import ops as _ops
    blk = model.blocks[0]
    xs = torch.randn(B * T, blk.d_model, device=dev)
    for _ in range(3):
        _ops.linear(xs, blk.in_proj.weight, blk.in_proj.bias)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(10):
        _ops.linear(xs, blk.in_proj.weight, blk.in_proj.bias)
    e1.record()
    torch.cuda.synchronize()
    in_proj_ms = e0.elapsed_time(e1) / 10
    s_bytes = B * T * blk.num_neurons * 64 * 4
    del xs
    names = ("fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry", "bwd_apply", "reduce_channels",
             "spike_fwd", "spike_bwd", "layer_norm_fwd", "layer_norm_bwd", "layer_norm_param_reduce",
             "ln_conv_silu_fwd", "ln_conv_silu_bwd", "ln_conv_silu_param_reduce", "generator_action_fwd",
             "generator_action_bwd", "projection_epilogue_fwd", "projection_epilogue_bwd", "column_sum",
             "silu_gate_fwd", "silu_gate_bwd")
    kt = {n: _lib.timing_read(n) for n in names}
    launches = sum(c for _, c in kt.values())  # per eager run of args.steps steps = per timed run
    _lib.timing_reset()
    # end to end: token ids from pinned host memory into the captured step's input buffers
    # every step, diagnostics (loss terms) back to host every step
    t0 = time.perf_counter()
    K = max(1, args.e2e_steps)
    for _ in range(K):
        _, _, diag = g(idx_h, tgt_h)
        graphs.read(diag)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) / K * 1e3
    print(json.dumps({
        "metric": metric, "value": B * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
        "eager_ms_per_step": eager_ms, "step": "CUDA graph of forward + backward + AdamW (capturable)",
        "scan_ms_per_step": sum(kt[n][0] for n in names[:7]) / args.steps,
        "kernel_ms": {n: {"total_ms": t, "launches": c} for n, (t, c) in kt.items()},
        "s_materialisation": {"in_proj_gemm_ms": in_proj_ms, "s_bytes_per_block": s_bytes,
                              "s_round_trips_per_block": "1 write (the GEMM) + 3 reads (scan passes)"},
        "gpu_launches": launches, "clocks": clk.summary(),
        "e2e": {"value": B * T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": 2 * B * T * 8,
                "d2h_bytes_per_step": 6 * 4, "timing": "wall clock per step: token ids pinned host -> device, "
                "train step, diagnostics to host"},
        "cpu_baseline": None}), flush=True)
    return 0


SPATIAL_BLOCKS = (("Cl4", 128, 2, 80), ("Cl8", 256, 1, 40), ("Cl8", 256, 1, 20))  # (algebra, C, N, H = W)


def _spatial_cpu(reps, warmup, cores):
    """The spatial scan section on the host cores: the four one-sided direction scans of the
    three blocks (rows left->right and right->left, then columns down and up of that result),
    forward and backward, one image, float64 C oracle (reversed scans by flipped arrays)."""
    import numpy as np
    from oracle import oracle as orc
    rng = np.random.default_rng(0)
    cases = []
    for alg, C, N, H in SPATIAL_BLOCKS:
        D = 4 if alg == "Cl4" else 16
        M = rng.uniform(0.3, 0.9, (1, H * H, N, 1, 1)) * np.eye(D) + 0.05 * rng.standard_normal((1, H * H, N, D, D))
        Cm = rng.standard_normal((1, H * H, N, D, D))
        cases.append((H, N, D, M, Cm))

    def bidir(M, C):
        f = orc.scan_fwd(M, C, two_sided=False)
        b = orc.scan_fwd(M[:, ::-1], C[:, ::-1], two_sided=False)[:, ::-1]
        orc.scan_bwd(M, f, np.ones_like(f), two_sided=False)
        orc.scan_bwd(M[:, ::-1], b[:, ::-1], np.ones_like(b), two_sided=False)
        return 0.5 * (f + b)

    def one():
        for H, N, D, M, Cm in cases:
            ph = bidir(M.reshape(H, H, N, D, D), Cm.reshape(H, H, N, D, D))
            bidir(M.reshape(1, H, H * N, D, D), ph.reshape(1, H, H * N, D, D))

    el = _time_cpu(one, reps, warmup)
    elems = sum(H * H * N for H, N, _, _, _ in cases) * reps
    return elems, el, "one image of the three blocks' scan sections (4 direction scans each), fwd+bwd, float64 C oracle"


def run_spatial(args, ws, rank, local, cores):
    """The three spatial rotor blocks of the reference detector (csn_toolkit/csn/vision.py:223-246,
    CSN-Large at 640 x 640: C3 Cl(4) 128 channels 80 x 80 with 2 neurons, C4 / C5 Cl(8) 256
    channels 40 x 40 / 20 x 20 with 1 neuron), forward + backward of each block (projections,
    Cayley, the four-direction spatial scan, out_proj, BatchNorm, SiLU) at batch 16.  Elements =
    B * H * W * N summed over the blocks; one step = one fwd + bwd of all three (parameter and
    input-map gradients), captured once as a CUDA graph and replayed; the eager step time is
    reported beside it."""
    B = args.batch or 16
    config = {"workload": "spatial_rotor_blocks_fwd_bwd", "batch": B,
              "blocks": [f"{a} C{c} N{n} {h}x{h}" for a, c, n, h in SPATIAL_BLOCKS],
              "l2": "inputs larger than L2 (the Cl(4) block's M and C are 105 MB each)"}
    metric = "spatial rotor blocks fwd+bwd Gelem/s (B*H*W*N)"
    elems = B * sum(h * h * n for _, _, n, h in SPATIAL_BLOCKS)
    if args.impl == "reference":
        if rank != 0:
            return 0
        cores = _cpu_threads(cores)
        e, el, sample = _spatial_cpu(max(1, args.steps), min(args.warmup, 1), cores)
        v = e / el / 1e9
        print(json.dumps({"metric": metric, "value": v, "unit": "Gelem/s", "n_gpus": args.gpus, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": el / max(1, args.steps) * 1e3,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                          "data": "synthetic", "config": config, "impl": "reference",
                          "cpu_baseline": {"value": v, "unit": "Gelem/s", "cores": cores, "kind": "port",
                                           "sample": sample},
                          "e2e": {"value": v, "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return 0
    import torch
    from csn_b200 import _lib, graphs
    from csn.vision import CliffordSpatialRotorBlockCl4, CliffordSpatialRotorBlockCl8
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _lib.load()
    torch.manual_seed(0)
    blocks, xs, ws_ = [], [], []
    gen = torch.Generator(device="cpu").manual_seed(0)
    for alg, C, N, H in SPATIAL_BLOCKS:
        cls = CliffordSpatialRotorBlockCl4 if alg == "Cl4" else CliffordSpatialRotorBlockCl8
        blocks.append(cls(C, num_neurons=N, use_schulz=False).to(dev))
        xs.append(torch.randn(B, C, H, H, generator=gen).to(dev))
        ws_.append(torch.randn(B, C, H, H, generator=gen).to(dev))

    class Blocks(torch.nn.Module):  # the three blocks; loss = sum over blocks of sum(y * w)
        def __init__(self):
            super().__init__()
            self.blocks = torch.nn.ModuleList(blocks)

        def forward(self, *inputs):
            outs = [blk(x) for blk, x in zip(self.blocks, inputs)]
            return outs, sum((y * w).sum() for y, w in zip(outs, ws_))

    net = Blocks()
    for x in xs:
        x.requires_grad_(True)

    def step(inputs):  # gradients of the parameters and of the input maps, not accumulated
        net.zero_grad(set_to_none=True)
        for x in inputs:
            x.grad = None
        outs, loss = net(*inputs)
        loss.backward()
        return outs

    # eager steps first: per-step launch count and kernel times of this package's kernels
    for _ in range(max(3, args.warmup)):
        step(xs)
    torch.cuda.synchronize()
    _lib.timing_reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _lib.timing_enable(True)
    e0.record()
    for _ in range(args.steps):
        step(xs)
    e1.record()
    torch.cuda.synchronize()
    _lib.timing_enable(False)
    eager_ms = e0.elapsed_time(e1) / args.steps
    # the timed step: forward + backward of the three blocks captured once as a CUDA graph
    g = graphs.TrainStepGraph(net, None, xs, warmup=3, inputs_require_grad=True)
    for _ in range(max(3, args.warmup)):
        g(*g.inputs)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            g(*g.inputs)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    names = ("fwd_reduce", "fwd_carry", "fwd_apply", "bwd_reduce", "bwd_carry", "bwd_apply", "cayley_fwd",
             "cayley_bwd", "spatial_generators_fwd", "spatial_generators_bwd")
    kt = {n: _lib.timing_read(n) for n in names}
    launches = sum(c for _, c in kt.values())
    _lib.timing_reset()
    # end to end: the three feature maps from pinned host memory, outputs back, every step
    hx = [x.detach().cpu().pin_memory() for x in xs]
    hy = [torch.empty(x.shape).pin_memory() for x in xs]
    K = max(1, args.e2e_steps)

    def e2e_step():  # the host maps into the captured step's input buffers, outputs back
        outs, _ = g(*hx)
        for h, o in zip(hy, outs):
            h.copy_(o.detach(), non_blocking=True)
        torch.cuda.synchronize()

    e2e_step()  # untimed: the first run from host buffers
    t0 = time.perf_counter()
    for _ in range(K):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) / K * 1e3
    nbytes = sum(h.numel() * 4 for h in hx)
    cpu = None
    if not args.no_cpu_baseline:
        cores = _cpu_threads(cores)
        e, el, sample = _spatial_cpu(2, 0, cores)
        cpu = {"value": e / el / 1e9, "unit": "Gelem/s", "cores": cores, "kind": "port", "sample": sample}
    print(json.dumps({
        "metric": metric, "value": elems / (ms * 1e-3) / 1e9, "unit": "Gelem/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
        "eager_ms_per_step": eager_ms, "step": "CUDA graph of the three blocks' forward + backward",
        "scan_ms_per_step": sum(kt[n][0] for n in names[:8]) / args.steps,
        "kernel_ms": {n: {"total_ms": t, "launches": c} for n, (t, c) in kt.items()},
        "gpu_launches": launches, "clocks": clk.summary(),
        "e2e": {"value": elems / (e2e_ms * 1e-3) / 1e9, "unit": "Gelem/s", "h2d_bytes_per_step": nbytes,
                "d2h_bytes_per_step": nbytes, "timing": "wall clock per step: feature maps pinned host -> device, "
                "three blocks fwd + bwd (captured step), outputs to host"},
        "cpu_baseline": cpu}), flush=True)
    return 0


# ===================================================== the other configurations, same run
def _device_inputs(wl, dev, seed):
    """wl's inputs drawn on the device (same distributions as its host inputs)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *shape: torch.randn(*shape, device=dev, generator=g)
    u = lambda *shape: torch.rand(*shape, device=dev, generator=g)
    B, T, N = wl.B, wl.T, wl.N
    if isinstance(wl, Cl8):
        return dict(gens=r(B, T, N, wl.K) * 0.05, dt=u(B, T) * 0.045 + 0.005, S=r(B, T, N, 16, 16),
                    dX=r(B, T, N, 16, 16))
    return dict(gens=r(B, T, N, 3) * 0.1, dt=u(B, T) * 0.09 + 0.01, x=r(B, T, N, 8), dh=r(B, T, N, 8))


def measure_config(wl, dev, lib, steps=10, warmup=3):
    """Device-timed value, dominant-kernel and whole-op roofline of workload wl (inputs on the
    device, no host copies); a summary of the figures the main line gives for its workload."""
    import torch
    from csn_b200 import _lib
    wl.dev = dev
    if isinstance(wl, Cl8):
        wl.inp = _device_inputs(wl, dev, 7)
        wl.out = dict(X=torch.empty_like(wl.inp["S"]), dS=torch.empty_like(wl.inp["S"]),
                      dgens=torch.empty_like(wl.inp["gens"]), ddt=torch.empty_like(wl.inp["dt"]))
        wl.Mc = torch.empty_like(wl.inp["S"])
        wl.ws_bytes = lib.csn_rotor_scan_workspace_bytes(wl.B, wl.T, wl.N, wl.D)
    else:
        wl.inp = _device_inputs(wl, dev, 99)
        wl.out = dict(h=torch.empty_like(wl.inp["x"]), dx=torch.empty_like(wl.inp["x"]),
                      dgens=torch.empty_like(wl.inp["gens"]), ddt=torch.empty_like(wl.inp["dt"]))
        wl.ws_bytes = lib.csn_ga3_workspace_bytes(wl.B, wl.T, wl.N)
    wl.work = torch.empty(wl.ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        wl.step(stream)
    torch.cuda.synchronize()
    _lib.timing_reset()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _lib.timing_enable(True)
    e0.record(stream)
    for _ in range(steps):
        wl.step(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    _lib.timing_enable(False)
    ms = e0.elapsed_time(e1) / steps
    kt = {n: _lib.timing_read(n) for n in wl.kernel_names}
    _lib.timing_reset()
    hbm, peak_kind = peaks()
    dom = max(wl.kernel_bytes, key=lambda n: kt[n][0])
    dom_ms = kt[dom][0] / max(1, kt[dom][1])
    per_launch = wl.elems_per_step * steps / max(1, kt[dom][1])
    ach = wl.kernel_bytes[dom] * per_launch / (dom_ms * 1e-3) / 1e9
    op = wl.op_bytes * wl.elems_per_step / (ms * 1e-3) / 1e9
    res = {"metric": METRIC, "value": wl.elems_per_step / (ms * 1e-3) / 1e9, "unit": UNIT,
           "ms_per_step": ms, "steps": steps, "warmup": warmup, "config": wl.config,
           "roofline": {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": hbm, "unit": "GB/s",
                        "frac": ach / hbm, "peak_kind": peak_kind, "avg_launch_ms": dom_ms,
                        "traffic": (wl.kernel_traffic[dom] * per_launch
                                    if dom in getattr(wl, "kernel_traffic", {}) else None)},
           "op_roofline": {"achieved": op, "peak": hbm, "unit": "GB/s", "frac": op / hbm,
                           "bytes_per_elem": wl.op_bytes},
           "kernel_ms_per_step": {n: t / steps for n, (t, c) in kt.items() if c},
           "gpu_launches": sum(c for _, c in kt.values())}
    del wl.inp, wl.out, wl.work
    if hasattr(wl, "Mc"):
        del wl.Mc
    torch.cuda.empty_cache()
    return res


def _gen_graph(B, N, D, chunk, dev, chained):
    """RotorStepGraph of the generation configuration with seeded inputs staged."""
    import torch
    from csn_b200 import ops
    g = ops.RotorStepGraph(B, N, D, steps=chunk, damped=True, device=dev, chained=chained)
    gen = torch.Generator(device="cpu").manual_seed(0)
    g.gens.copy_(torch.randn(chunk, B, N, 28, generator=gen) * 0.1)
    g.dt.copy_(torch.rand(chunk, B, generator=gen) * 0.09 + 0.01)
    g.gamma.copy_(torch.nn.functional.softplus(torch.randn(chunk, B, N, generator=gen)))
    g.S.copy_(torch.randn(chunk, B, N, D, D, generator=gen))
    return g


def measure_generation(dev, steps=2048, chunk=128):
    """p50 latency of one graph-replayed rotor step of the Cl(6,0) generation configuration
    (256 streams x 8 channels) and tokens/s."""
    import numpy as np
    import torch
    from csn_b200 import ops
    B, N, D = 256, 8, 8
    p = {}
    for chained in (False, True):
        g = _gen_graph(B, N, D, chunk, dev, chained)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        lat = []
        for _ in range(steps // chunk):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            lat.append(e0.elapsed_time(e1) * 1e3 / chunk)
        p[chained] = float(np.median(lat))
    p50 = p[False]
    return {"metric": "rotor-step p50 latency (us), 256 streams x 8 channels Cl(6,0)", "value": p50,
            "unit": "us", "tok_per_s": B / (p50 * 1e-6), "p50_chained_us": p[True], "steps": steps,
            "higher_is_better": False,
            "config": {"workload": "cl6_generation_step", "streams": B, "channels": N, "matrix_dim": D,
                       "graph_steps": chunk, "damped": True}}


# ==================================================================================== main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=None,
                    choices=sorted(WORKLOADS) + ["gen", "sp", "lm_train", "spatial", "d4_harness"],
                    help="default: sp when launched by torch.distributed.run (any world size), else cl6_lm")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="cl6_lm at N = 1: skip the Cl(3), Cl(8) and generation figures of the same run")
    ap.add_argument("--batch", type=int, default=None, help="per-rank batch (profiling: smaller)")
    ap.add_argument("--layers", type=int, default=None, help="layers per step (cl6_lm; profiling: 1)")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.workload is None:
        args.workload = "sp" if launched_by_torchrun() else "cl6_lm"
    cores = os.cpu_count() or 1
    if args.workload == "gen":
        return run_generation(args, ws, rank, local, cores)
    if args.workload == "sp":
        return run_sequence_parallel(args, ws, rank, local, cores)
    if args.workload == "lm_train":
        return run_lm_train(args, ws, rank, local, cores)
    if args.workload == "spatial":
        return run_spatial(args, ws, rank, local, cores)
    if args.workload == "d4_harness":
        return run_d4_harness(args, ws, rank, local, cores)
    kw = {}
    if args.batch is not None:
        kw["batch"] = args.batch
    if args.layers is not None:
        kw["layers"] = args.layers
    wl = WORKLOADS[args.workload](**kw)

    if args.impl == "reference":
        if rank != 0:
            return 0
        cores = _cpu_threads(cores)
        elems, el, sample = wl.cpu_reference(reps=max(1, args.steps), warmup=min(args.warmup, 1))
        v = elems / el / 1e9
        line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": el / max(1, args.steps) * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic", "config": wl.config, "impl": "reference",
                "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if args.workload == "cl6_lm":  # beside the port: the reference's own fp32 torch code
            line["cpu_baseline"]["reference_fp32"] = reference_fp32_cpu(cores)
        print(json.dumps(line), flush=True)
        return 0

    import torch
    from csn_b200 import _lib

    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    wl.setup(dev, rank, lib)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    for _ in range(max(3, args.warmup)):
        wl.step(stream)
    torch.cuda.synchronize()

    _lib.timing_reset()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        _lib.timing_enable(True)
        e0.record(stream)
        for _ in range(args.steps):
            wl.step(stream)
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
    value = wl.elems_per_step * ws / (ms_per_step * 1e-3) / 1e9

    # per-kernel device times over the timed region (CUDA events on the launch stream)
    ktimes = {n: _lib.timing_read(n) for n in wl.kernel_names}
    launches = sum(c for _, c in ktimes.values())
    dom = max(wl.kernel_bytes, key=lambda n: ktimes[n][0])
    dom_launches = max(1, ktimes[dom][1])
    dom_ms = ktimes[dom][0] / dom_launches
    elems_per_launch = wl.elems_per_step * args.steps / dom_launches
    hbm, peak_kind = peaks()
    achieved = wl.kernel_bytes[dom] * elems_per_launch / (dom_ms * 1e-3) / 1e9
    _lib.timing_reset()

    e2e = None
    if args.e2e_steps > 0:
        h2d, d2h = wl.e2e_setup()
        wl.e2e_step()
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            wl.e2e_step()
        torch.cuda.current_stream(dev).synchronize()
        el = time.perf_counter() - t0
        if ws > 1:
            t = torch.tensor([el], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            el = t.item()
        e2e = {"value": wl.elems_per_step * ws * args.e2e_steps / el / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "timing": "wall clock around K steps (pinned host -> device, op forward + backward, "
                         "device -> pinned host, pipelined over pieces on three streams) ending in "
                         "a stream synchronize, max over ranks"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cores = _cpu_threads(cores)
        elems, el, sample = wl.cpu_reference(reps=2, warmup=0)
        cpu = {"value": elems / el / 1e9, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
        if args.workload == "cl6_lm":
            cpu["reference_fp32"] = reference_fp32_cpu(cores)
    ref_gpu = None
    if rank == 0 and ws == 1 and args.workload == "cl6_lm" and not args.no_cpu_baseline:
        # the reference toolkit's torch code on this GPU, at this workload's shape (one layer)
        ref_gpu = reference_fp32_cpu(cores, B=wl.B, T=wl.T, N=wl.N, D=wl.D, device=f"cuda:{local}")

    # the Cl(3) bandwidth, Cl(8) and generation configurations, measured in the same run
    # (device-timed, inputs on the device) so that their figures travel with this line
    others = None
    if ws == 1 and args.workload == "cl6_lm" and not args.no_other_configs:
        del wl.inputs, wl.outs, wl.work
        if hasattr(wl, "pipe"):
            del wl.pipe, wl.host, wl.hout
        torch.cuda.empty_cache()
        others = {"cl3": measure_config(Cl3(), dev, lib), "cl8": measure_config(Cl8(), dev, lib),
                  "gen": measure_generation(dev)}

    if rank == 0:
        op_ach = wl.op_bytes * wl.elems_per_step / (ms_per_step * 1e-3) / 1e9
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": dict(wl.config, parallelism=f"replicas{ws}" if ws > 1 else "single"),
                "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm,
                             "unit": "GB/s", "frac": achieved / hbm,
                             "traffic": (wl.kernel_traffic[dom] * elems_per_launch
                                         if dom in getattr(wl, "kernel_traffic", {}) else None),
                             "peak_kind": peak_kind, "bytes_per_elem": wl.kernel_bytes[dom],
                             "avg_launch_ms": dom_ms},
                "op_roofline": {"achieved": op_ach, "peak": hbm, "unit": "GB/s", "frac": op_ach / hbm,
                                "bytes_per_elem": wl.op_bytes},
                "kernel_ms": {n: {"total_ms": t, "launches": c} for n, (t, c) in ktimes.items()},
                "gpu_launches": launches, "clocks": clk.summary(), "e2e": e2e, "cpu_baseline": cpu}
        if others is not None:
            line["other_configs"] = others
        if ref_gpu is not None:
            line["reference_fp32_gpu"] = ref_gpu
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
