#!/usr/bin/env python
"""Benchmark of the selective-scan hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1, NCCL)

Metric: selective-scan forward+backward throughput in TB/s of algorithmic
HBM bytes, on config 2 -- the Mamba-130M layer (batch 8, d_inner 1536, seqlen 2048,
d_state 16, bf16 streams, z gate, softplus).  A step is one forward and one backward over
one batch.  Multi-GPU runs are weak-scaled: every rank processes its own batch of 8 (the
batch dimension is sharded across GPUs with no data-path collective); `value` counts the
bytes of all ranks over the slowest rank's time.  Decode tokens/s (config 3) is reported as
a secondary field.

Algorithmic bytes count every input read once and every output written once
(bf16 = 2 bytes, B/C of shape (batch, 16, seqlen)):
    forward  = 4*E*2 + 2*B*N*L*2      (u, delta, z read; out written; B, C read)
    backward = 7*E*2 + 4*B*N*L*2      (u, delta, z, dout read; du, ddelta, dz written;
                                       B, C read; dB, dC written)
State checkpoints and the saved pre-gate output are implementation traffic and are not
counted.  The reference arm (--impl reference) times the reference's math on the host
CPU cores (the reference has no CPU path of its own; this is the C restatement in
oracle/, run on a bounded sample of the same workload) and, for context, the reference's
own CUDA kernels on the GPU in float32 (their only dtype).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG2 = dict(batch=8, dim=1536, seqlen=2048, dstate=16)
CFG3 = dict(batch=64, dim=5120, dstate=16, steps=1024, layers=8)
CFG5 = dict(dim=5120, seqlen=131072, dstate=16)


def scan_bytes(batch, dim, seqlen, dstate, es=2):
    E = batch * dim * seqlen
    bnl = batch * dstate * seqlen
    return 4 * E * es + 2 * bnl * es, 7 * E * es + 4 * bnl * es


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def _pure(name):
    """ssm_mamba_b200/<name>.py (workloads, weights: plain torch, no native code) loaded by path,
    without importing the ssm_mamba_b200 package, so that the reference arm, which uses these
    input generators, imports nothing of this library."""
    import importlib.util
    key = "_bench_pure_" + name
    if key not in sys.modules:
        spec = importlib.util.spec_from_file_location(key, os.path.join(ROOT, "ssm_mamba_b200", name + ".py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[key] = mod
        spec.loader.exec_module(mod)
    return sys.modules[key]


def traffic_from_profiles(name, key="traffic_bytes_per_launch"):
    """Per-launch DRAM bytes of a kernel, from a committed ncu summary (profiles/*.txt
    lines `traffic_bytes_per_launch <kernel> <bytes>`; another per-launch figure with
    `key`), or None."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".txt"):
            continue
        with open(os.path.join(d, fn)) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and parts[0] == key and parts[1] == name:
                    return float(parts[2])
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.proc = None
        self.t0 = self.t1 = None
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            ident = str(device_index)
        self.ident = ident

    def start(self):
        """Starts sampling and returns once the first sample has arrived, so that the
        sampler's own start-up (NVML initialisation, which was seen to stall a timed step
        by several ms) is over before any timing begins."""
        self.first = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.QUERY, "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.ident], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        import select
        ready, _, _ = select.select([self.proc.stdout], [], [], 10.0)
        if ready:
            self.first.append(self.proc.stdout.readline())
        time.sleep(0.2)

    def mark(self, which):
        """mark("t0") / mark("t1") bracket the timed region; only samples inside it count."""
        setattr(self, which, time.time())

    def _inside(self, stamp):
        if self.t0 is None or self.t1 is None:
            return True
        try:
            import datetime
            t = datetime.datetime.strptime(stamp.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return True
        return self.t0 - 0.05 <= t <= self.t1 + 0.05

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in (self.first + out.strip().splitlines()) if r.strip()]
        rows = [r[1:] for r in rows if len(r) >= 10 and self._inside(r[0])] or [r[1:] for r in rows if len(r) >= 10]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(n)
        loaded = sorted(sm)[len(sm) // 4:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(rows)}


def bind_host_to_gpu(local):
    """Pin this process to the CPU cores NVML reports as local to GPU `local` (a read-only
    NVML query; only this process's CPU affinity changes), so that pinned host buffers
    allocated next live on the GPU's own NUMA node.  Best effort: any failure leaves the
    affinity alone and returns None."""
    try:
        import pynvml
        import torch
        pr = torch.cuda.get_device_properties(local)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
            return sorted(cpus)
    except Exception:
        pass
    return None


def dist_setup(want_nccl=True):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1 and torch.cuda.is_available():
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl" if want_nccl else "gloo", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local, pg


def max_over_ranks(x, pg):
    import torch
    if pg is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg):
    import torch
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------------------
def host_oracle():
    """The oracle module with its OpenMP pool sized to every core this process may run on:
    a multi-rank launcher sets OMP_NUM_THREADS=1 for its ranks, and the host baselines are
    timed on all cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.set_num_threads(len(os.sched_getaffinity(0)))
    return oracle


def cpu_baseline_sample(target_s=10.0, batch=1, dim=96):
    """The oracle's float build (C + OpenMP, all host cores) on a bounded sample of the
    config-2 workload: (batch, dim) rows of the same seqlen / d_state."""
    import numpy as np
    import torch
    oracle = host_oracle()
    scan_inputs = _pure("workloads").scan_inputs
    L, N = CFG2["seqlen"], CFG2["dstate"]
    inp = scan_inputs(batch, dim, L, N, torch.bfloat16, seed=1, device="cpu", with_z=True)
    f = lambda t: t.float().numpy()  # noqa: E731
    args = [f(inp.u), f(inp.delta), f(inp.A), f(inp.B), f(inp.C)]
    kw = dict(D=f(inp.D), z=f(inp.z), delta_bias=f(inp.delta_bias), dtype=np.float32)
    reps, t_total = 0, 0.0
    while t_total < target_s and reps < 50:
        t0 = time.perf_counter()
        fw = oracle.scan_fwd(*args, **kw)
        oracle.scan_bwd(*args, f(inp.dout), fwd=fw, **kw)
        t_total += time.perf_counter() - t0
        reps += 1
    fb, bb = scan_bytes(batch, dim, L, N)
    return {"value": (fb + bb) * reps / t_total / 1e12, "unit": "TB/s", "cores": oracle.num_threads(),
            "kind": "port",
            "sample": f"oracle float32 fwd+bwd of {batch}x{dim} channel rows of config 2 (seqlen {L}, "
                      f"d_state {N}; 1/{CFG2['batch'] * CFG2['dim'] // (batch * dim)} of the batch), "
                      f"{reps} reps in {t_total:.1f} s", "seconds_per_step_full": t_total / reps *
            (CFG2["batch"] * CFG2["dim"]) / (batch * dim)}


def cpu_decode_sample(target_s=3.0):
    """Config 3 on the host: the oracle's float build of one decode step (batch 64, d_inner
    5120, d_state 16, bf16-valued inputs in float32), repeated for about `target_s`."""
    import numpy as np
    import torch
    oracle = host_oracle()
    decode_inputs = _pure("workloads").decode_inputs
    Bd, Dd, Nd = CFG3["batch"], CFG3["dim"], CFG3["dstate"]
    dec = decode_inputs(Bd, Dd, Nd, 4, torch.bfloat16, seed=2, device="cpu")
    f = lambda t: t.float().numpy()  # noqa: E731
    st = f(dec.state)
    reps, t_total = 0, 0.0
    while t_total < target_s and reps < 200:
        i = reps % 4
        t0 = time.perf_counter()
        _, st = oracle.state_update(st, f(dec.x[i]), f(dec.dt[i]), f(dec.A), f(dec.B[i]), f(dec.C[i]), D=f(dec.D),
                                    z=f(dec.z[i]), dt_bias=f(dec.dt_bias), dt_softplus=True, dtype=np.float32)
        t_total += time.perf_counter() - t0
        reps += 1
    us = t_total / reps * 1e6
    return {"us_per_step": us, "tokens_per_s": Bd / (us / 1e6), "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle float32 state update, batch {Bd} x d_inner {Dd} x d_state {Nd}, {reps} steps "
                      f"in {t_total:.1f} s (includes the oracle's input conversion)"}


def cpu_long_seq_sample(target_s=3.0, dim=48, seqlen=8192):
    """Config 5 on the host, extrapolated: the oracle's float build of fwd+bwd on `dim`
    channels of a truncated seqlen, scaled linearly to 5120 channels x 131072 tokens."""
    import numpy as np
    import torch
    oracle = host_oracle()
    scan_inputs = _pure("workloads").scan_inputs
    N = CFG5["dstate"]
    inp = scan_inputs(1, dim, seqlen, N, torch.bfloat16, seed=4, device="cpu", with_z=True)
    f = lambda t: t.float().numpy()  # noqa: E731
    a = [f(inp.u), f(inp.delta), f(inp.A), f(inp.B), f(inp.C)]
    kw = dict(D=f(inp.D), z=f(inp.z), delta_bias=f(inp.delta_bias), dtype=np.float32)
    reps, t_total = 0, 0.0
    while t_total < target_s and reps < 20:
        t0 = time.perf_counter()
        fw = oracle.scan_fwd(*a, **kw)
        oracle.scan_bwd(*a, f(inp.dout), fwd=fw, **kw)
        t_total += time.perf_counter() - t0
        reps += 1
    scale = (CFG5["dim"] * CFG5["seqlen"]) / (dim * seqlen)
    s_full = t_total / reps * scale
    fb, bb = scan_bytes(1, CFG5["dim"], CFG5["seqlen"], N)
    return {"seconds_per_step_extrapolated": s_full, "tb_s": (fb + bb) / s_full / 1e12,
            "cores": oracle.num_threads(), "kind": "port",
            "sample": f"oracle float32 fwd+bwd of 1 x {dim} channels x {seqlen} tokens, {reps} reps in "
                      f"{t_total:.1f} s, extrapolated linearly (x{scale:.0f}) to 1 x 5120 x 131072: EXTRAPOLATED"}


def run_decode(args, world, rank, local, pg, peak):
    """Config 3: 1024 decode steps in one CUDA graph, state rotated over 8 layer buffers
    (168 MB > L2) so every step reads and writes its state in HBM."""
    import torch
    from ssm_mamba_b200 import selective_state_update
    decode_inputs = _pure("workloads").decode_inputs
    dev = torch.device("cuda", local)
    Bd, Dd, Nd, S, Ly = CFG3["batch"], CFG3["dim"], CFG3["dstate"], CFG3["steps"], CFG3["layers"]
    dec = decode_inputs(Bd, Dd, Nd, S, torch.bfloat16, seed=2 + rank, device=dev)
    states = [dec.state.clone() for _ in range(Ly)]

    def loop():
        for s in range(S):
            selective_state_update(states[s % Ly], dec.x[s], dec.dt[s], dec.A, dec.B[s], dec.C[s], dec.D,
                                   dec.z[s], dec.dt_bias, dt_softplus=True)

    loop()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loop()
    for _ in range(2):
        graph.replay()
    barrier(pg)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    d0.record()
    for _ in range(reps):
        graph.replay()
    d1.record()
    torch.cuda.synchronize()
    barrier(pg)
    dec_ms = max_over_ranks(d0.elapsed_time(d1), pg) / (reps * S)
    step_bytes = 2 * Bd * Dd * Nd * 4 + 4 * Bd * Dd * 2 + Dd * Nd * 4 + 2 * Bd * Nd * 2 + 2 * Dd * 4
    del graph
    return {"metric": "decode tokens/s (one Mamba-2.8B-width layer)", "value": Bd * world / (dec_ms / 1e3),
            "unit": "tokens/s", "us_per_step": dec_ms * 1e3, "gpu_launches_per_step": 1,
            "roofline": {"bound": "hbm", "achieved": step_bytes / (dec_ms / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": step_bytes / (dec_ms / 1e3) / 1e9 / peak,
                         "bytes_per_step": step_bytes},
            "config": "batch 64, d_inner 5120, d_state 16 fp32 state, bf16 x/dt/z/B/C, 1024 steps in "
                      "one CUDA graph, state rotated over 8 layer buffers"}


def run_long_seq(args, world, rank, local, pg, peak):
    """Config 5: one sequence of 131072 tokens (batch 1, d_inner 5120, d_state 16, bf16, z
    gate), forward + backward through the public API.  One GPU scans it as segments; N GPUs
    hold N contiguous slices (each segmented further) and exchange the slice carries with one
    NCCL all_gather per direction plus an all_reduce of dA/dD/ddelta_bias (strong scaling:
    the total work is fixed)."""
    import torch
    from ssm_mamba_b200.slices import SliceGroup, plan_segments, sliced_scan
    scan_inputs = _pure("workloads").scan_inputs
    dev = torch.device("cuda", local)
    Ltot, Dm, N = (args.long_seqlen or CFG5["seqlen"]), CFG5["dim"], CFG5["dstate"]
    Lr = Ltot // world
    inp = scan_inputs(1, Dm, Lr, N, torch.bfloat16, seed=4 + rank, device=dev, with_z=True)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    S = plan_segments(1, Dm, Lr, N, sms=sms, ranks=world)
    # with the process group's store: the host-side liveness check and shape agreement of
    # every exchange go through it (no collective, no device synchronization)
    group = SliceGroup(pg.group.WORLD, store=pg.PrefixStore("ssm_long_seq", pg.distributed_c10d._get_default_store()),
                       peer_timeout=datetime.timedelta(seconds=120)) if pg is not None else SliceGroup(None)
    leaves = [t.clone().requires_grad_() for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z,
                                                   inp.delta_bias)]

    def step():
        for t in leaves:      # a training step's gradients, not an accumulation over steps
            t.grad = None
        out, _ = sliced_scan(*leaves, None, True, segments=S, group=group)
        out.backward(inp.dout)

    parity = _seqpar_parity(dev, rank, world, group, pg) if world > 1 else None
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = 3
    from ssm_mamba_b200.slices import PhaseTimer, set_phase_timer
    timer = PhaseTimer()
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    # per-phase breakdown of one more (untimed) step, queued behind the timed ones as in
    # the loop: CUDA events between the phases of the sliced scan, each the max over ranks
    set_phase_timer(timer)
    step()
    set_phase_timer(None)
    torch.cuda.synchronize()
    barrier(pg)
    ms = max_over_ranks(e0.elapsed_time(e1), pg) / steps
    ph = timer.durations_ms()
    phases = {k: max_over_ranks(ph.get(k, 0.0), pg) for k in sorted(ph)}
    barrier(pg)
    fb, bb = scan_bytes(1, Dm, Ltot, N)
    tbs = (fb + bb) / (ms / 1e3) / 1e12
    return {"metric": "long-sequence scan fwd+bwd achieved HBM TB/s", "value": tbs, "unit": "TB/s",
            "ms_per_step": ms, "steps": steps, "scaling": "strong", "segments_per_rank": S,
            "seqpar_parity": parity,
            "phase_ms": phases,
            "phase_what": "one extra step queued behind the timed ones, CUDA events between phases, max over "
                          "ranks: agree (shape agreement and liveness of the ranks through the store, on the "
                          "host), chunk_state (the chunk-state pass), exchange (carry all_gather), compose (carry "
                          "folding), scan (the per-segment scan), param_allreduce (dA/dD/ddelta_bias)",
            "elem_state_per_s": 1 * Dm * Ltot * N / (ms / 1e3),
            "frac_of_hbm_peak": tbs * 1e3 / world / peak,
            "gpu_launches_per_step": 8,
            "config": f"config 5: batch 1, d_inner {Dm}, seqlen {Ltot} ({world} slice(s) of {Lr}), d_state {N}, "
                      "bf16, z gate, softplus; sequence-parallel carries over NCCL when n_gpus > 1"}


def _seqpar_parity(dev, rank, world, group, pg):
    """Correctness of the sequence-parallel path before it is timed: the scan of one
    sequence split over the ranks (rank r holds the r-th slice, cut into 2 segments; slice
    carries over NCCL) against the unsliced scan of the whole sequence, computed on every
    rank with the same kernels (float32, batch 1, 256 channels, 8192 tokens, z gate, an
    initial state and a final-state gradient).  Forward outputs and the final state within
    rtol 1e-4 / atol 1e-5; gradients within rtol 1e-3 plus 1e-4 of their largest magnitude.
    Every rank takes the same collectives; the verdict is the worst over the ranks."""
    import torch
    from ssm_mamba_b200.slices import sliced_scan
    scan_inputs = _pure("workloads").scan_inputs
    L, Dm, N = 8192, 256, 16
    inp = scan_inputs(1, Dm, L, N, torch.float32, seed=21, device="cpu", with_z=True, with_h_init=True)
    dh = torch.randn(1, Dm, N, generator=torch.Generator().manual_seed(5))
    full = [t.to(dev) for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias, inp.h_init)]
    dout, dh = inp.dout.to(dev), dh.to(dev)
    ref = [t.clone().requires_grad_() for t in full]
    o_ref, h_ref = sliced_scan(*ref, delta_softplus=True, segments=1)
    ((o_ref * dout).sum() + (h_ref * dh).sum()).backward()
    lo, hi = rank * L // world, (rank + 1) * L // world
    sliced = (0, 1, 3, 4, 6)          # u, delta, B, C, z are split along the sequence
    loc = [(t[..., lo:hi].contiguous() if i in sliced else t).clone().requires_grad_() for i, t in enumerate(full)]
    out, hf = sliced_scan(*loc, delta_softplus=True, segments=2, group=group)
    loss = (out * dout[..., lo:hi]).sum() + ((hf * dh).sum() if rank == world - 1 else 0)
    loss.backward()

    def excess(got, want, rtol, atol, frac=0.0):
        # max over elements of |got - want| / (atol + frac*max|want| + rtol*|want|): <= 1 passes
        w = want.detach().double()
        bound = atol + frac * float(w.abs().max()) + rtol * w.abs()
        return float(((got.detach().double() - w).abs() / bound).max())

    worst = {"out": excess(out, o_ref[..., lo:hi], 1e-4, 1e-5), "h_final": excess(hf, h_ref, 1e-4, 1e-5)}
    names = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias", "h_init"]
    for i, name in enumerate(names):
        want = ref[i].grad
        if i in sliced:
            want = want[..., lo:hi]
        if name == "h_init" and rank != 0:
            want = torch.zeros_like(want)
        worst["d" + name] = excess(loc[i].grad, want, 1e-3, 1e-12, 1e-4)
    torch.cuda.synchronize()
    # worst over ranks, one all_reduce for all quantities (every rank takes it)
    keys = sorted(worst)
    vals = torch.tensor([worst[k] for k in keys], dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(vals, op=pg.ReduceOp.MAX)
    worst = {k: float(v) for k, v in zip(keys, vals.tolist())}
    ok = all(v <= 1.0 for v in worst.values())
    return {"status": "ok" if ok else "FAILED", "ranks": world,
            "worst_error_over_tolerance": worst,
            "what": f"sequence-parallel scan over {world} ranks (2 segments each) vs the unsliced scan, float32, "
                    f"1 x {Dm} x {L}, z gate, h_init, dh_last; <= 1 is within tolerance"}


EQ_SCAN = {"cfg1": (2, 64, 256, 0), "cfg2": (8, 1536, 2048, 1), "cfg5": (1, 5120, 131072, 4)}


def _time_steps(step, warmup, steps):
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _decode_graph_us(apply_fn, dev, seed=2):
    """us per decode step of an out-of-place update (the reference's semantics:
    selective_update.cpp:208-209) over 8 rotating layer states (168 MB > L2), 256 steps in
    one CUDA graph; float32 (config 3 shape)."""
    import torch
    decode_inputs = _pure("workloads").decode_inputs
    Bd, Dd, Nd, Ly = CFG3["batch"], CFG3["dim"], CFG3["dstate"], CFG3["layers"]
    S = 256
    dec = decode_inputs(Bd, Dd, Nd, S, torch.float32, seed=seed, device=dev)
    states = [dec.state.clone() for _ in range(Ly)]

    def loop():
        for s in range(S):
            _, states[s % Ly] = apply_fn(dec.x[s], dec.A, dec.B[s], dec.C[s], dec.D, dec.dt[s], dec.dt_bias,
                                         states[s % Ly])

    loop()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        loop()
    ms = _time_steps(g.replay, 2, 3)
    del g
    return ms * 1e3 / S


def run_equal_precision(dev, forward_backward, update_apply):
    """The float32 workloads the reference's kernels support (no z gate, softplus on),
    timed through a reference-shaped API: `forward_backward(inputs)` runs one forward and
    backward, `update_apply` one out-of-place decode step.  Same shapes and seeds in both
    arms of bench.py."""
    import torch
    scan_inputs = _pure("workloads").scan_inputs
    res = {}
    for name, (Bs, Dm, L, seed) in EQ_SCAN.items():
        inp = scan_inputs(Bs, Dm, L, 16, torch.float32, seed=seed, device=dev, with_z=False)
        ms = _time_steps(lambda: forward_backward(inp), 2, 3 if L > 100000 else 10)
        fb, bb = scan_bytes(Bs, Dm, L, 16, es=4)
        fb -= Bs * Dm * L * 4       # no z stream
        bb -= 2 * Bs * Dm * L * 4   # no z read, no dz written
        res[name] = {"shape": [Bs, Dm, L, 16], "ms_per_fwd_bwd": ms, "fp32_tb_s": (fb + bb) / (ms / 1e3) / 1e12}
        del inp
        torch.cuda.empty_cache()
    try:
        res["cfg3_decode"] = {"us_per_step": _decode_graph_us(update_apply, dev), "mode": "CUDA graph"}
    except Exception as e:  # noqa: BLE001 - context only
        res["cfg3_decode"] = {"error": str(e)[:200]}
    return res


def run_varlen(dev, forward_backward, dtypes=("fp32",)):
    """Variable-length rows (`length`, the reference API's padding sides): config-2 shape
    with per-row lengths drawn in [L/2, L] (seed 5), forward + backward through a
    reference-shaped call `forward_backward(inputs, length, padding)`; float32 (the
    reference kernels' only dtype) and, where given, bf16."""
    import torch
    scan_inputs = _pure("workloads").scan_inputs
    Bs, Dm, L, N = CFG2["batch"], CFG2["dim"], CFG2["seqlen"], CFG2["dstate"]
    g = torch.Generator().manual_seed(5)
    length = torch.randint(L // 2, L + 1, (Bs,), generator=g).to(dev)
    res = {"lengths": length.tolist()}
    for dn in dtypes:
        dt = torch.float32 if dn == "fp32" else torch.bfloat16
        inp = scan_inputs(Bs, Dm, L, N, dt, seed=1, device=dev, with_z=False)
        for pad in ("right", "left"):
            ms = _time_steps(lambda: forward_backward(inp, length, pad), 2, 10)
            res[f"{dn}_{pad}"] = {"ms_per_fwd_bwd": ms}
        del inp
        torch.cuda.empty_cache()
    res["config"] = (f"config-2 shape ({Bs}, {Dm}, {L}, d_state {N}), no z, softplus, per-row lengths, "
                     "padding right and left (the reference API's default)")
    return res


def _ours_varlen_fwd_bwd(inp, length, pad):
    from ssm_mamba_b200 import SelectiveScanFn
    leaves = [t.requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias)]
    out, _ = SelectiveScanFn.apply(*leaves, None, length, pad)
    out.backward(inp.dout)
    for t in leaves:
        t.grad = None


CONV = dict(batch=8, dim=1536, seqlen=2048, width=4)


def run_conv(dev, fwd_bwd, step, label):
    """Causal depthwise conv1d + SiLU in front of the scan (config-2 shape, bf16, width 4):
    forward + backward of the prefill, and one decode step of the context (batch 64,
    d_inner 5120: the config-3 width).  `fwd_bwd(x, w, b, dout)` and `step(x, state, w, b)`
    are the implementation under test."""
    import torch
    Bc, Dc, Lc, K = CONV["batch"], CONV["dim"], CONV["seqlen"], CONV["width"]
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(Bc, Dc, Lc, device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn(Bc, Dc, Lc, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randn(Dc, K, device=dev, generator=g) * 0.5
    b = torch.randn(Dc, device=dev, generator=g)
    ms = _time_steps(lambda: fwd_bwd(x, w, b, dout), 3, 50)
    E = Bc * Dc * Lc
    byts = 5 * E * 2           # forward: x in, out; backward: x, dout in, dx out
    # decode: 256 steps in one CUDA graph, the context rotating over 8 layer buffers
    Bd, Dd = CFG3["batch"], CFG3["dim"]
    S, Ly = 256, 8
    xs = torch.randn(S, Bd, Dd, device=dev, generator=g).to(torch.bfloat16)
    sts = [torch.randn(Bd, Dd, K - 1, device=dev, generator=g).to(torch.bfloat16) for _ in range(Ly)]
    wd = torch.randn(Dd, K, device=dev, generator=g) * 0.5
    bd = torch.randn(Dd, device=dev, generator=g)

    def loop():
        for i in range(S):
            step(xs[i], sts[i % Ly], wd, bd)

    loop()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loop()
    us = _time_steps(graph.replay, 2, 3) * 1e3 / S
    del graph
    return {"what": label, "prefill_fwd_bwd_ms": ms, "prefill_tb_s": byts / (ms / 1e3) / 1e12,
            "prefill_algorithmic_bytes": byts, "decode_step_us": us,
            "config": f"x ({Bc}, {Dc}, {Lc}) bf16, width {K}; decode ({Bd}, {Dd}) bf16, {S} steps in a "
                      "CUDA graph"}


LAYER = dict(batch=64, model=2560, inner=5120, state=16, rank=160, width=4)


def _layer_weights(dev, dtype, seed=11):
    """Random weights of a Mamba-2.8B-width layer (ssm_mamba_b200.weights.MambaLayerWeights)."""
    import torch
    MambaLayerWeights = _pure("weights").MambaLayerWeights
    dt_bias_init, s4d_real_A = _pure("workloads").dt_bias_init, _pure("workloads").s4d_real_A
    c = LAYER
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *sh, sc=0.02: (torch.randn(*sh, device=dev, generator=g) * sc)  # noqa: E731
    return MambaLayerWeights(
        in_proj_weight=r(2 * c["inner"], c["model"]).to(dtype), conv_weight=r(c["inner"], c["width"], sc=0.3),
        x_proj_weight=r(c["rank"] + 2 * c["state"], c["inner"]).to(dtype),
        dt_proj_weight=r(c["inner"], c["rank"], sc=0.08).to(dtype), dt_proj_bias=dt_bias_init(c["inner"], g, dev),
        A=s4d_real_A(c["inner"], c["state"], dev), D=torch.ones(c["inner"], device=dev),
        out_proj_weight=r(c["model"], c["inner"]).to(dtype), conv_bias=r(c["inner"]))


def run_decode_layer(dev, step_factory, label):
    """tokens/s of a whole Mamba layer's decoding step (in_proj, conv step, x_proj, dt_proj,
    state update, gate, out_proj) at the Mamba-2.8B width, batch 64: `step_factory()`
    returns (step(hidden) -> out, graphable).  Eager and (when graphable) CUDA-graph
    replays, 128 steps each."""
    import torch
    step, graphable = step_factory()
    Bsz = LAYER["batch"]
    g = torch.Generator(device=dev).manual_seed(3)
    hid = [torch.randn(Bsz, LAYER["model"], device=dev, generator=g).to(step.dtype) for _ in range(8)]
    n = 128

    def eager():
        for i in range(n):
            step(hid[i % 8])

    us_eager = _time_steps(eager, 1, 2) * 1e3 / n
    res = {"what": label, "eager_us_per_step": us_eager, "eager_tokens_per_s": Bsz / (us_eager / 1e6)}
    if graphable:
        from ssm_mamba_b200.decode import GraphedStep
        gs = GraphedStep(step, [hid[0]], preserve=step.caches)

        def graphed():
            for i in range(n):
                gs(hid[i % 8])

        us = _time_steps(graphed, 1, 2) * 1e3 / n
        res.update({"graph_us_per_step": us, "graph_tokens_per_s": Bsz / (us / 1e6)})
        del gs
    res["config"] = ("one Mamba layer, model 2560, inner 5120, state 16, rank 160, conv width 4, batch 64, "
                     f"{'bf16' if step.dtype == torch.bfloat16 else 'fp32'} weights and activations")
    return res


def _ours_layer_factory(dev, dtype):
    def make():
        from ssm_mamba_b200.decode import MambaLayerCache, mamba_layer_step
        w = _layer_weights(dev, dtype)
        cache = MambaLayerCache.zeros(w, LAYER["batch"], dtype)

        def step(hidden):
            return mamba_layer_step(w, cache, hidden)

        step.dtype = dtype
        step.caches = [cache.conv_state, cache.ssm_state]
        return step, True
    return make


CFG4 = dict(batch=4, seqlen=2048, model=2560, layers=64, inner=5120, state=16, rank=160, width=4,
            vocab=50288, ids=50280)


def _lm_weights(dev, dtype, seed=3):
    """Random-init Mamba-2.8B-architecture causal LM (models/causal_lm.py:27-98 with the
    modules/block.py and modules/mamba.py:34-79 defaults): every projection, the conv and
    the tied embedding ~ N(0, 0.02) in `dtype`; dt_proj bias from dt ~ logUniform(1e-3, 1e-1);
    A from the S4D-real log_A; D = 1; RMSNorm weights 0 (the norm scales by 1 + weight); no
    biases.  Returns (embedding, [(norm weight, MambaLayerWeights)], final norm weight)."""
    import torch
    MambaLayerWeights = _pure("weights").MambaLayerWeights
    dt_bias_init, s4d_real_A = _pure("workloads").dt_bias_init, _pure("workloads").s4d_real_A
    c = CFG4
    g = torch.Generator(device=dev).manual_seed(seed)
    r = lambda *sh: torch.randn(*sh, device=dev, generator=g, dtype=torch.float32).mul_(0.02).to(dtype)  # noqa: E731
    A, Dv = s4d_real_A(c["inner"], c["state"], dev), torch.ones(c["inner"], device=dev)
    layers = []
    for _ in range(c["layers"]):
        layers.append((torch.zeros(c["model"], device=dev), MambaLayerWeights(
            in_proj_weight=r(2 * c["inner"], c["model"]), conv_weight=r(c["inner"], c["width"]).float(),
            x_proj_weight=r(c["rank"] + 2 * c["state"], c["inner"]), dt_proj_weight=r(c["inner"], c["rank"]),
            dt_proj_bias=dt_bias_init(c["inner"], g, dev), A=A, D=Dv, out_proj_weight=r(c["model"], c["inner"]))))
    return r(c["vocab"], c["model"]), layers, torch.zeros(c["model"], device=dev)


def _rms_norm(x, weight, eps=1e-6):
    # modules/rms_norm.py:17-31: computed in float32, scaled by 1 + weight
    import torch
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + weight)).type_as(x)


def _fused_rms_norm(x, weight, eps=1e-6):
    # the same arithmetic as _rms_norm (float32 normalisation, scaled by 1 + weight, cast
    # back) through torch's fused rms_norm kernel instead of seven elementwise passes
    import torch.nn.functional as F
    return F.rms_norm(x.float(), (x.shape[-1],), weight=1.0 + weight, eps=eps).type_as(x)


def _ref_glue_layer(w, hidden, scan):
    """The reference's Mamba.forward (modules/mamba.py:100-186; no cache, no lengths) in torch
    ops, with its layout copies, around `scan(u, A, B, C, D, delta, delta_bias) -> out`."""
    import torch
    import torch.nn.functional as F
    Bsz, L, _ = hidden.shape
    Dm, R, N = w.inner, w.rank, w.state
    x, gate = torch.chunk(F.linear(hidden, w.in_proj_weight).permute(0, 2, 1).contiguous(), 2, dim=1)
    gate = gate.permute(0, 2, 1).contiguous()
    x = F.silu(F.conv1d(x, w.conv_weight.to(x.dtype)[:, None], None, padding=w.conv_weight.shape[1] - 1,
                        groups=Dm)[..., :L])
    p = F.linear(x.permute(0, 2, 1).contiguous().view(Bsz * L, Dm), w.x_proj_weight)
    delta, Bm, Cm = torch.split(p, [R, N, N], dim=-1)
    delta = (w.dt_proj_weight @ delta.t()).view(Dm, Bsz, L).permute(1, 0, 2).contiguous()
    Bm = Bm.reshape(Bsz, L, N).permute(0, 2, 1).contiguous()
    Cm = Cm.reshape(Bsz, L, N).permute(0, 2, 1).contiguous()
    out = scan(x, w.A, Bm, Cm, w.D, delta, w.dt_proj_bias)
    out = out.permute(0, 2, 1).contiguous() * F.silu(gate)
    return F.linear(out, w.out_proj_weight)


def run_prefill_lm(dev, dtype, variants, reps=3, pg=None, world=1, rank=0, norm=None):
    """Config 4: prefill forward of the random-init Mamba-2.8B-architecture causal LM
    (CausalLM.forward, models/causal_lm.py:79-98: embedding, 64 x (RMSNorm, Mamba layer,
    residual), RMSNorm, tied lm_head) on batch 4 x 2048 token ids (seed 3 + rank), timed with
    CUDA events over `reps` forwards after one warm-up.  Data-parallel over ranks (weak
    scaling: every rank runs its own batch of 4, no collective); the time is the slowest
    rank's.  `variants` maps a label to layer(weights, normed hidden) -> layer output;
    `norm` is the RMSNorm (default: the reference module's torch ops, _rms_norm).  Returns
    ms and whole-job tokens/s per label."""
    import torch
    import torch.nn.functional as F
    c = CFG4
    norm = norm or _rms_norm
    emb, layers, norm_w = _lm_weights(dev, dtype)
    g = torch.Generator(device=dev).manual_seed(3 + rank)
    ids = torch.randint(0, c["ids"], (c["batch"], c["seqlen"]), device=dev, generator=g)
    tokens = c["batch"] * c["seqlen"] * world
    res = {}
    with torch.no_grad():
        for label, layer in variants.items():
            def fwd():
                h = F.embedding(ids, emb)
                for nw, w in layers:
                    h = h + layer(w, norm(h, nw))
                return F.linear(norm(h, norm_w), emb)
            err = None
            barrier(pg)
            try:
                ms = _time_steps(fwd, 1, reps)
            except Exception as e:  # one variant failing must not hide the others
                ms, err = 1e30, str(e)[:200]
            ms = max_over_ranks(ms, pg)   # every rank takes this collective, failed or not
            if err is not None or ms >= 1e29:
                res[label] = {"error": err or "failed on another rank"}
            else:
                res[label] = {"ms_per_forward": ms, "tokens_per_s": tokens / (ms / 1e3)}
            torch.cuda.empty_cache()
    res["config"] = (f"config 4: Mamba-2.8B-architecture causal LM prefill forward, batch {c['batch']} per GPU x "
                     f"{world} GPU(s) (data-parallel, no collective), seqlen {c['seqlen']}, {c['layers']} layers, "
                     f"model {c['model']}, vocab {c['vocab']}, "
                     f"{'bf16' if dtype == torch.bfloat16 else 'fp32'} random-init weights, eval (no dropout); "
                     f"RMSNorm: {'torch fused rms_norm' if norm is _fused_rms_norm else 'the module torch ops'}")
    del emb, layers
    torch.cuda.empty_cache()
    return res


TRAIN = dict(batch=8, seqlen=2048, model=768, inner=1536, state=16, rank=48, width=4)


def run_train_layer(dev, dtype, variants, reps=10, graph=False):
    """One Mamba-130M-shape layer (the config-2 scan inside it: batch 8, seqlen 2048, model
    768, d_inner 1536, d_state 16, dt_rank 48, conv width 4) trained for one step: the
    layer's forward and backward with every weight a leaf (modules/mamba.py:100-186 and its
    autograd), random weights ~ N(0, 0.02) (seed 13).  `variants` maps a label to
    layer(weights, hidden) -> output.  With `graph`, the first variant's step is also
    captured once in a CUDA graph and replayed."""
    import torch
    MambaLayerWeights = _pure("weights").MambaLayerWeights
    dt_bias_init, s4d_real_A = _pure("workloads").dt_bias_init, _pure("workloads").s4d_real_A
    c = TRAIN
    g = torch.Generator(device=dev).manual_seed(13)
    r = lambda *sh: torch.randn(*sh, device=dev, generator=g, dtype=torch.float32).mul_(0.02).to(dtype)  # noqa: E731
    w = MambaLayerWeights(
        in_proj_weight=r(2 * c["inner"], c["model"]), conv_weight=r(c["inner"], c["width"]).float() * 10,
        x_proj_weight=r(c["rank"] + 2 * c["state"], c["inner"]), dt_proj_weight=r(c["inner"], c["rank"]) * 5,
        dt_proj_bias=dt_bias_init(c["inner"], g, dev), A=s4d_real_A(c["inner"], c["state"], dev),
        D=torch.ones(c["inner"], device=dev), out_proj_weight=r(c["model"], c["inner"]))
    leaves = [w.in_proj_weight, w.conv_weight, w.x_proj_weight, w.dt_proj_weight, w.dt_proj_bias, w.D,
              w.out_proj_weight]
    for t in leaves:
        t.requires_grad_()
    hid = torch.randn(c["batch"], c["seqlen"], c["model"], device=dev, generator=g).to(dtype).requires_grad_()
    dout = torch.randn(c["batch"], c["seqlen"], c["model"], device=dev, generator=g).to(dtype)
    res = {}
    for label, layer in variants.items():
        def step():
            layer(w, hid).backward(dout)
            for t in leaves + [hid]:
                t.grad = None
        try:
            ms = _time_steps(step, 2, reps)
            res[label] = {"ms_per_step": ms, "tokens_per_s": c["batch"] * c["seqlen"] / (ms / 1e3)}
            if graph and label == next(iter(variants)):
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    step()
                torch.cuda.current_stream().wait_stream(s)
                cg = torch.cuda.CUDAGraph()
                with torch.cuda.graph(cg):
                    step()
                gms = _time_steps(cg.replay, 2, reps)
                res[label].update({"graph_ms_per_step": gms,
                                   "graph_tokens_per_s": c["batch"] * c["seqlen"] / (gms / 1e3)})
                del cg
        except Exception as e:  # one variant failing must not hide the others
            res[label] = {"error": str(e)[:200]}
        torch.cuda.empty_cache()
    res["config"] = (f"one Mamba-130M-shape layer, forward + backward, batch {c['batch']}, seqlen {c['seqlen']}, "
                     f"model {c['model']}, d_inner {c['inner']}, d_state {c['state']}, dt_rank {c['rank']}, "
                     f"{'bf16' if dtype == torch.bfloat16 else 'fp32'} weights and activations")
    return res


def _ours_prefill_variants():
    from ssm_mamba_b200 import SelectiveScanFn
    from ssm_mamba_b200.layer import mamba_layer_forward
    return {"ssm_mamba_b200.layer.mamba_layer_forward (no layout copies, fused gate)":
            lambda w, x: mamba_layer_forward(w, x)[0],
            "reference module glue + ssm_mamba_b200.SelectiveScanFn (ops swapped only)":
            lambda w, x: _ref_glue_layer(w, x, lambda *a: SelectiveScanFn.apply(*a)[0])}


def _ours_conv_fwd_bwd(x, w, b, dout):
    # the extension's entry points (what causal_conv1d_fn's forward and backward call)
    from ssm_mamba_b200._ext import _C
    _C.conv1d_fwd(x, w, b, True, None, False)
    _C.conv1d_bwd(x, w, b, True, dout)


def _ours_conv_step(x, state, w, b):
    from ssm_mamba_b200 import causal_conv1d_update
    causal_conv1d_update(x, state, w, b)


def _ours_fwd_bwd(inp):
    from ssm_mamba_b200 import SelectiveScanFn
    leaves = [t.requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta, inp.delta_bias)]
    out, _ = SelectiveScanFn.apply(*leaves)
    out.backward(inp.dout)
    for t in leaves:
        t.grad = None


def _ours_update(x, A, B, C, D, dt, bias, h):
    from ssm_mamba_b200 import SelectiveUpdateFn
    return SelectiveUpdateFn.apply(x, A, B, C, D, dt, bias, h)


def run_ours(args, world, rank, local, pg):
    import torch
    from ssm_mamba_b200._ext import _C
    from ssm_mamba_b200 import selective_scan_fn, selective_state_update
    scan_inputs = _pure("workloads").scan_inputs
    dev = torch.device("cuda", local)
    if args.decode_only:
        return {"decode": run_decode(args, world, rank, local, pg, measured_peaks()[0])}
    if args.decode_layer_only:
        return {"decode_layer": {"bf16": run_decode_layer(dev, _ours_layer_factory(dev, torch.bfloat16),
                                                          "ssm_mamba_b200.decode.mamba_layer_step (+ GraphedStep)")}}
    if args.prefill_only:
        v = dict(list(_ours_prefill_variants().items())[:1])     # mamba_layer_forward only
        return {"prefill_lm": {"bf16": run_prefill_lm(dev, torch.bfloat16, v, norm=_fused_rms_norm)}}
    B, D, L, N = CFG2["batch"], CFG2["dim"], CFG2["seqlen"], CFG2["dstate"]
    inp = scan_inputs(B, D, L, N, torch.bfloat16, seed=1 + rank, device=dev, with_z=True)
    fwd_bytes, bwd_bytes = scan_bytes(B, D, L, N)

    def step():
        out, y, ck, _ = _C.scan_fwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias, None,
                                    None, True, True, True, 1, False)
        ev_mid = torch.cuda.Event(enable_timing=True)
        ev_mid.record()
        g = _C.scan_bwd(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias, None, None, True,
                        True, y, ck, inp.dout, None)
        return ev_mid, out, g

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(args.warmup):
        step()
    barrier(pg)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = []
    torch.cuda.synchronize()
    barrier(pg)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks.mark("t0")
    t_start.record()
    for i in range(args.steps):
        starts[i].record()
        # keep nothing of the step but its event: the same memory footprint as the warm-up
        # steps, so the caching allocator never has to grow inside the timed region
        mids.append(step()[0])
        ends[i].record()
    t_end.record()
    torch.cuda.synchronize()
    clocks.mark("t1")
    barrier(pg)
    clk = clocks.stop()
    elapsed_ms = t_start.elapsed_time(t_end)
    fwd_each = [starts[i].elapsed_time(mids[i]) for i in range(args.steps)]
    bwd_each = [mids[i].elapsed_time(ends[i]) for i in range(args.steps)]
    fwd_ms, bwd_ms = statistics.mean(fwd_each), statistics.mean(bwd_each)
    step_each = [a + b for a, b in zip(fwd_each, bwd_each)]
    elapsed_ms = max_over_ranks(elapsed_ms, pg)
    total_bytes = (fwd_bytes + bwd_bytes) * args.steps * world
    value = total_bytes / (elapsed_ms / 1e3) / 1e12
    peak, peak_kind = measured_peaks()

    # ---- end to end through the public API: pinned host inputs in, gradients out -------
    # Every step copies its inputs from pinned host memory and its input gradients back.
    # The copies run on their own streams, double-buffered, so step i's host->device copy
    # and step i-1's device->host copy overlap step i's compute (a data pipeline would do
    # the same); the timed region covers all copies of all steps.
    e2e = None
    e2e_steps = 0 if args.no_e2e else min(args.steps, 20)
    # the host side of the end-to-end loop runs on the GPU's own NUMA node (restored after,
    # so the host baselines below keep every core)
    saved_cpus = os.sched_getaffinity(0)
    bound_cpus = bind_host_to_gpu(local) if e2e_steps else None
    f = lambda t: t.detach().to("cpu").pin_memory()  # noqa: E731
    host_in = {k: f(getattr(inp, k)) for k in ("u", "delta", "z", "B", "C", "dout")}
    A = inp.A.clone().requires_grad_()
    Dp = inp.D.clone().requires_grad_()
    bias = inp.delta_bias.clone().requires_grad_()
    grad_keys = ("u", "delta", "z", "B", "C")
    NBUF = 2
    host_out = [{k: torch.empty(host_in[k].shape, dtype=host_in[k].dtype).pin_memory() for k in grad_keys}
                for _ in range(NBUF)]
    dev_in = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in host_in.items()}
              for _ in range(NBUF)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    comp = torch.cuda.current_stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(NBUF)]
    in_free = [torch.cuda.Event() for _ in range(NBUF)]
    used = [False] * NBUF

    def e2e_step(i):
        b = i % NBUF
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(in_free[b])          # the compute that read this buffer is done
            for k, v in host_in.items():
                dev_in[b][k].copy_(v, non_blocking=True)
            in_ready[b].record(s_in)
        comp.wait_event(in_ready[b])
        d = dev_in[b]
        leaves = {k: d[k].detach().requires_grad_() for k in grad_keys}
        o = selective_scan_fn(leaves["u"], leaves["delta"], A, leaves["B"].unsqueeze(1),
                              leaves["C"].unsqueeze(1), Dp, leaves["z"], bias, delta_softplus=True)
        o.backward(d["dout"])
        in_free[b].record(comp)
        used[b] = True
        s_out.wait_stream(comp)
        with torch.cuda.stream(s_out):
            for k in grad_keys:
                g = leaves[k].grad
                host_out[b][k].copy_(g, non_blocking=True)
                g.record_stream(s_out)

    if e2e_steps:
        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier(pg)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        s_in.wait_event(e0)
        s_out.wait_event(e0)
        for i in range(e2e_steps):
            e2e_step(i)
        comp.wait_stream(s_out)
        e1.record(comp)
        torch.cuda.synchronize()
        barrier(pg)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), pg)
        h2d = sum(v.numel() * v.element_size() for v in host_in.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out[0].values())
        e2e = {"value": (fwd_bytes + bwd_bytes) * e2e_steps * world / (e2e_ms / 1e3) / 1e12, "unit": "TB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / e2e_steps,
               "steps": e2e_steps, "host_cpus": len(bound_cpus) if bound_cpus else None,
               "api": "ssm_mamba_b200.selective_scan_fn forward + autograd backward; copies double-buffered "
                      "on separate streams"}
    del host_in, host_out, dev_in
    os.sched_setaffinity(0, saved_cpus)

    decode = None if args.no_decode else run_decode(args, world, rank, local, pg, peak)
    long_seq = None if args.no_long else run_long_seq(args, world, rank, local, pg, peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_sample(target_s=args.cpu_seconds)
    conv = None
    if world == 1 and not args.no_conv:
        conv = run_conv(dev, _ours_conv_fwd_bwd, _ours_conv_step,
                        "ssm_mamba_b200.causal_conv1d_fn / causal_conv1d_update")
    layer = None
    if world == 1 and not args.no_layer:
        layer = {"bf16": run_decode_layer(dev, _ours_layer_factory(dev, torch.bfloat16),
                                          "ssm_mamba_b200.decode.mamba_layer_step (+ GraphedStep)"),
                 "fp32": run_decode_layer(dev, _ours_layer_factory(dev, torch.float32),
                                          "ssm_mamba_b200.decode.mamba_layer_step (+ GraphedStep)")}
    eq = None
    if world == 1 and not args.no_fp32:
        eq = run_equal_precision(dev, _ours_fwd_bwd, _ours_update)
        eq["api"] = "ssm_mamba_b200.SelectiveScanFn / SelectiveUpdateFn (the reference's signatures)"
    train = None
    if world == 1 and not args.no_layer:
        v = _ours_prefill_variants()
        train = {"bf16": run_train_layer(dev, torch.bfloat16, v, graph=True)}
        if not args.no_fp32:
            train["fp32"] = run_train_layer(dev, torch.float32, v, reps=5)
    varlen = None
    if world == 1 and not args.no_fp32:
        varlen = run_varlen(dev, _ours_varlen_fwd_bwd, ("fp32", "bf16"))
        varlen["api"] = "ssm_mamba_b200.SelectiveScanFn with length and padding_size"
    prefill = None
    if not args.no_prefill:
        variants = _ours_prefill_variants()
        if world > 1:   # data-parallel over ranks: the layer only
            variants = dict(list(variants.items())[:1])
        prefill = {"bf16": run_prefill_lm(dev, torch.bfloat16, variants, pg=pg, world=world, rank=rank,
                                          norm=_fused_rms_norm)}
        if world == 1 and not args.no_fp32:
            prefill["fp32"] = run_prefill_lm(dev, torch.float32, _ours_prefill_variants(), reps=2,
                                             norm=_fused_rms_norm)

    bwd_gbs = bwd_bytes / (bwd_ms / 1e3) / 1e9
    fwd_gbs = fwd_bytes / (fwd_ms / 1e3) / 1e9
    # The scan kernels are bound by instruction issue, not HBM: warp instructions per launch
    # (ncu, committed summaries) over the measured duration, against 4 warp instructions per
    # clock per SM at the SM clock sampled during the timed region.
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = (clk or {}).get("sm_mhz") or (clk or {}).get("sm_max_mhz") or 1965.0
    issue_peak = 4.0 * sms * mhz * 1e6
    issue = {"what": "warp instructions issued per second against 4 per clock per SM (the issue limit) "
                     "at the sampled SM clock; instruction counts from ncu (profiles/)",
             "sm_mhz": mhz, "sms": sms, "peak_warp_inst_per_s": issue_peak}
    bwd_kernel = "scan_bwd_split_kernel"   # the backward's main kernel at config 2's 12 288 rows
    for kname, ms_k in ((bwd_kernel, bwd_ms), ("scan_fwd_kernel", fwd_ms)):
        n_inst = traffic_from_profiles(kname, key="warp_instructions_per_launch")
        if n_inst:
            issue[kname] = {"warp_inst_per_launch": n_inst, "achieved_warp_inst_per_s": n_inst / (ms_k / 1e3),
                            "frac": n_inst / (ms_k / 1e3) / issue_peak}
    # The roofs of each scan kernel other than HBM, from its committed per-launch counts over
    # the duration measured here: instruction issue (4 warp instructions per clock per SM), the
    # shared-memory pipe (one 128-byte wavefront or one warp shuffle per clock per SM) and the
    # MUFU pipe (16 exp2 / reciprocal / tanh results per clock per SM: a warp instruction
    # holds it 2 clocks per SM).  `bound` names the highest; none is saturated at config 2
    # (both kernels are latency-bound with ~10 warps per SM), so binding_frac is its fraction.
    sm_hz = mhz * 1e6

    def roofs(kname, ms_k):
        per_s = 1.0 / (ms_k / 1e3) / (sms * sm_hz)
        out = {}
        for roof, key, scale in (("issue", "warp_instructions_per_launch", 0.25),
                                 ("mio", "mio_ops_per_launch", 1.0), ("mufu", "mufu_warp_inst_per_launch", 2.0)):
            n = traffic_from_profiles(kname, key=key)
            if n:
                out[roof] = n * scale * per_s
        return out

    bwd_roofs, fwd_roofs = roofs(bwd_kernel, bwd_ms), roofs("scan_fwd_kernel", fwd_ms)
    bwd_bound = max(bwd_roofs, key=bwd_roofs.get) if bwd_roofs else "latency"
    fwd_bound = max(fwd_roofs, key=fwd_roofs.get) if fwd_roofs else "latency"
    line = {
        "metric": "scan fwd+bwd achieved HBM TB/s (% of peak) at 1/2/4/8 B200; decode tokens/s",
        "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded normal draws, S4D-real A, dt-bias init)",
        "config": {"workload": "config 2: Mamba-130M-shape layer selective_scan fwd+bwd, batch 8 per GPU, "
                               "d_inner 1536, seqlen 2048, d_state 16, bf16 u/delta/z/B/C, z gate, softplus",
                   "global_batch": B * world, "seq_len": L, "parallelism": f"batch-sharded x{world}, no collective",
                   "l2": "inputs larger than L2 (~330 MB read per step)",
                   "frac_of_hbm_peak": value / world * 1e3 / peak},
        "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        "step_ms_min_median_max": [min(step_each), statistics.median(step_each), max(step_each)],
        "slow_steps": [i for i, v in enumerate(step_each) if v > 1.5 * statistics.median(step_each)][:10],
        # `bound` names the roof that binds each kernel per the committed ncu counters (DRAM is
        # 10-20% busy); achieved / peak / frac are the HBM figures of the contract,
        # binding_frac the fraction of the binding roof
        "roofline": {"bound": bwd_bound, "binding_frac": bwd_roofs.get(bwd_bound), "roofs": bwd_roofs,
                     "binding_what": "fractions of the non-HBM roofs from per-launch ncu counts (profiles/) over "
                                     "the duration timed here at the sampled clock: issue (4 warp instructions "
                                     "per clock per SM), mio (one shared-memory wavefront or warp shuffle per "
                                     "clock per SM), mufu (16 results per clock per SM); none saturated: "
                                     "latency-bound at ~10 warps per SM",
                     "kernel": f"ssm_scan_bwd ({bwd_kernel} + scan_reduce_kernel)",
                     "achieved": bwd_gbs, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": bwd_gbs / peak, "traffic": traffic_from_profiles(bwd_kernel),
                     "algorithmic_bytes_per_launch": bwd_bytes},
        "roofline_fwd": {"bound": fwd_bound, "binding_frac": fwd_roofs.get(fwd_bound), "roofs": fwd_roofs,
                         "binding_what": "as for roofline",
                         "kernel": "scan_fwd_kernel", "achieved": fwd_gbs, "peak": peak,
                         "unit": "GB/s", "frac": fwd_gbs / peak, "traffic": traffic_from_profiles("scan_fwd_kernel"),
                         "algorithmic_bytes_per_launch": fwd_bytes},
        "issue_roof": issue,
        "seqpar_parity": (long_seq or {}).get("seqpar_parity"),
        "e2e": e2e, "gpu_launches": 3 * args.steps, "clocks": clk, "decode": decode, "long_seq": long_seq,
        "cpu_baseline": cpu, "fp32_equal_precision": eq, "conv1d": conv, "decode_layer": layer,
        "prefill_lm": prefill, "varlen": varlen, "train_layer": train,
    }
    return line


def run_reference(args, world, rank, local, pg):
    """Reference arm: the reference's math on the host CPU cores (oracle port, bounded
    sample per step), plus the reference's own CUDA kernels on the GPU for context."""
    import torch
    if rank != 0:
        return None
    import numpy as np
    oracle = host_oracle()
    scan_inputs = _pure("workloads").scan_inputs
    L, N = CFG2["seqlen"], CFG2["dstate"]
    sb, sd = 1, 48
    inp = scan_inputs(sb, sd, L, N, torch.bfloat16, seed=1, device="cpu", with_z=True)
    f = lambda t: t.float().numpy()  # noqa: E731
    a = [f(inp.u), f(inp.delta), f(inp.A), f(inp.B), f(inp.C)]
    kw = dict(D=f(inp.D), z=f(inp.z), delta_bias=f(inp.delta_bias), dtype=np.float32)

    def step():
        fw = oracle.scan_fwd(*a, **kw)
        oracle.scan_bwd(*a, f(inp.dout), fwd=fw, **kw)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    fb, bb = scan_bytes(sb, sd, L, N)
    value = (fb + bb) * args.steps / dt / 1e12
    line = {
        "impl": "reference", "metric": "scan fwd+bwd achieved HBM TB/s (% of peak) at 1/2/4/8 B200; decode tokens/s",
        "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config 2 (Mamba-130M layer scan fwd+bwd), bounded sample of "
                               f"{sb}x{sd} channel rows per step, seqlen {L}, d_state {N}",
                   "global_batch": 8, "seq_len": L, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": oracle.num_threads(), "kind": "port",
                         "sample": f"{sb}x{sd} of 8x1536 channel rows per step (reference has no CPU path; "
                                   "C restatement of its kernels, float32, OpenMP)"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    # the other configs' host baselines (the reference has no CPU path; same C restatement)
    if not args.no_cpu:
        line["cpu_cfg3_decode"] = cpu_decode_sample()
        line["cpu_cfg5_long_seq"] = cpu_long_seq_sample()
    # the reference's own CUDA kernels (float32 only) on the GPU, same shapes as the float32
    # set of the other arm, through its pybind functions (what its SelectiveScanFn calls)
    try:
        import build_ref
        if torch.cuda.is_available() and build_ref.available() and not args.no_ref_cuda:
            ref = build_ref.load("ref_selective_scan")
            ref_up = build_ref.load("ref_selective_update")
            dev = torch.device("cuda", local)

            class RefScanFn(torch.autograd.Function):
                """Autograd over the reference's pybind functions, as the reference's
                SelectiveScanFn does (ops/selective_scan_interface.py:9-80): the forward
                returns (out, final state), the backward passes dout and the final state's
                gradient back.  Written here because the reference's Python files are not on
                the GPU box; both arms thus pay the same autograd overhead."""

                @staticmethod
                def forward(ctx, u, A, B, C, D, delta, bias):
                    out, h = ref.forward(u, A, B, C, D, delta, bias, None, None, None)
                    ctx.save_for_backward(u, A, B, C, D, delta, bias, h)
                    return out, h[..., -1, 1::2]

                @staticmethod
                def backward(ctx, dout, dh):
                    u, A, B, C, D, delta, bias, h = ctx.saved_tensors
                    g = ref.backward(u, A, B, C, D, delta, bias, h, None, dout.contiguous(), dh.contiguous(),
                                     None, None)
                    return g[0], g[1], g[2], g[3], g[4], g[5], g[6]

            def fwd_bwd(inp):
                leaves = [t.requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta,
                                                       inp.delta_bias)]
                out, _ = RefScanFn.apply(*leaves)
                out.backward(inp.dout)
                for t in leaves:
                    t.grad = None

            line["ref_cuda_b200"] = run_equal_precision(dev, fwd_bwd, lambda *a: ref_up.apply(*a))

            class RefScanLenFn(torch.autograd.Function):
                """RefScanFn with `length` and the padding side passed to the pybind functions."""

                @staticmethod
                def forward(ctx, u, A, B, C, D, delta, bias, length, pad):
                    out, h = ref.forward(u, A, B, C, D, delta, bias, None, length, pad)
                    ctx.save_for_backward(u, A, B, C, D, delta, bias, h, length)
                    ctx.pad = pad
                    return out, h[..., -1, 1::2]

                @staticmethod
                def backward(ctx, dout, dh):
                    u, A, B, C, D, delta, bias, h, length = ctx.saved_tensors
                    g = ref.backward(u, A, B, C, D, delta, bias, h, None, dout.contiguous(), dh.contiguous(),
                                     length, ctx.pad)
                    return g[0], g[1], g[2], g[3], g[4], g[5], g[6], None, None

            def ref_varlen(inp, length, pad):
                leaves = [t.requires_grad_() for t in (inp.u, inp.A, inp.B, inp.C, inp.D, inp.delta,
                                                       inp.delta_bias)]
                out, _ = RefScanLenFn.apply(*leaves, length, pad)
                out.backward(inp.dout)
                for t in leaves:
                    t.grad = None

            line["ref_varlen_b200"] = run_varlen(dev, ref_varlen)
            line["ref_varlen_b200"]["api"] = "reference CUDA kernels with length and padding_side, float32"

            # the reference module's conv1d + SiLU (modules/mamba.py:137-139, 203-213): torch ops
            import torch.nn.functional as F

            def conv_fwd_bwd(x, w, b, dout):
                xl, wl, bl = x.requires_grad_(), w.requires_grad_(), b.requires_grad_()
                y = F.silu(F.conv1d(xl, wl.to(x.dtype)[:, None, :], bl.to(x.dtype), padding=w.shape[1] - 1,
                                    groups=w.shape[0])[..., :x.shape[-1]])
                y.backward(dout)
                for t in (xl, wl, bl):
                    t.grad = None

            def conv_step(x, state, w, b):
                window = torch.cat([state, x.unsqueeze(-1)], dim=-1)
                state.copy_(window[:, :, 1:])
                F.silu((window * w.to(x.dtype).unsqueeze(0)).sum(dim=-1) + b.to(x.dtype))

            line["ref_conv1d_b200"] = run_conv(dev, conv_fwd_bwd, conv_step,
                                               "reference module's torch ops: nn.Conv1d + F.silu, cat/sum step")

            # the reference module's decoding step (modules/mamba.py:188-241): torch ops with the
            # reference's selective_update extension (float32 only), a new state every step
            def ref_layer_factory():
                w = _layer_weights(dev, torch.float32)
                Bsz = LAYER["batch"]
                st = {"ctx": torch.zeros(Bsz, LAYER["inner"], LAYER["width"] - 1, device=dev),
                      "h": torch.zeros(Bsz, LAYER["inner"], LAYER["state"], device=dev)}

                def step(hidden):
                    xz = F.linear(hidden, w.in_proj_weight)
                    x, gate = xz.chunk(2, dim=-1)
                    window = torch.cat([st["ctx"], x.unsqueeze(-1)], dim=-1)
                    st["ctx"] = window[:, :, 1:]
                    x = F.silu((window * w.conv_weight.unsqueeze(0)).sum(dim=-1) + w.conv_bias)
                    delta, Bm, Cm = torch.split(F.linear(x, w.x_proj_weight), [w.rank, w.state, w.state], dim=-1)
                    delta = (w.dt_proj_weight @ delta.t()).t().contiguous()
                    y, st["h"] = ref_up.apply(x.contiguous(), w.A, Bm.contiguous(), Cm.contiguous(), w.D, delta,
                                              w.dt_proj_bias, st["h"])
                    return F.linear(y * F.silu(gate), w.out_proj_weight)

                step.dtype = torch.float32
                return step, False

            line["ref_decode_layer_b200"] = run_decode_layer(
                dev, ref_layer_factory, "reference module's step: torch ops + its selective_update kernel, fp32")

            # config 4: the reference module's forward (its layout copies, gate after the scan)
            # around its selective_scan kernel, float32 (the kernel's only dtype)
            def ref_scan(u, A, B, C, D, delta, bias):
                return ref.forward(u, A, B, C, D, delta, bias, None, None, None)[0]

            if not args.no_layer:
                def ref_scan_ag(u, A, B, C, D, delta, bias):
                    return RefScanFn.apply(u, A, B, C, D, delta, bias)[0]

                line["ref_train_layer_b200"] = run_train_layer(
                    dev, torch.float32,
                    {"reference module glue + its selective_scan kernels": lambda w, x: _ref_glue_layer(w, x, ref_scan_ag)},
                    reps=5)
            if not args.no_prefill:
                line["ref_prefill_lm_b200"] = run_prefill_lm(
                    dev, torch.float32,
                    {"reference module glue + its selective_scan kernel": lambda w, x: _ref_glue_layer(w, x, ref_scan)},
                    reps=2)
            line["ref_cuda_b200"]["what"] = ("reference CUDA kernels (oracle/_ref, built from its sources), "
                                             "float32, no z gate (the reference has none)")
    except Exception as e:  # context only; never fail the reference arm on it
        line["ref_cuda_b200"] = {"error": str(e)[:200]}
    line["this_library"] = _loaded_library_evidence()
    return line


def _loaded_library_evidence():
    """What of this repository the process has loaded: the ssm_mamba_b200 Python modules and
    every in-tree shared library mapped (/proc/self/maps).  The reference arm loads only the
    pure-torch input generators (ssm_mamba_b200/workloads.py, weights.py) by path, without the
    package, so it must list no module and map no native library of ssm_mamba_b200."""
    mods = sorted(m for m in sys.modules if m == "ssm_mamba_b200" or m.startswith("ssm_mamba_b200."))
    libs = set()
    try:
        with open("/proc/self/maps") as f:
            for row in f:
                path = row.split()[-1] if len(row.split()) >= 6 else ""
                if path.startswith(ROOT) and ".so" in path:
                    libs.add(os.path.relpath(path, ROOT))
    except OSError:
        pass
    return {"python_modules": mods, "native_libraries_mapped": sorted(libs),
            "native_code_of_this_library_loaded": any(p.startswith("ssm_mamba_b200") for p in libs)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ref-cuda", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-long", action="store_true", help="skip the long-sequence (config 5) measurement")
    ap.add_argument("--no-conv", action="store_true", help="skip the conv1d + SiLU measurement")
    ap.add_argument("--no-layer", action="store_true", help="skip the whole-layer decode measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 causal LM prefill measurement")
    ap.add_argument("--long-seqlen", type=int, default=0,
                    help="profiling aid: config 5 at this total seqlen instead of 131072 (a small ncu case)")
    ap.add_argument("--decode-layer-only", action="store_true",
                    help="profiling aid: only the bf16 whole-layer decode step")
    ap.add_argument("--prefill-only", action="store_true",
                    help="profiling aid: only the config-4 prefill through mamba_layer_forward")
    ap.add_argument("--no-fp32", action="store_true",
                    help="skip the float32 workloads timed like the reference's kernels")
    ap.add_argument("--decode-only", action="store_true", help="profiling aid: only the decode loop")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        # rank 0 alone runs the reference arm; the other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if rank != 0:
            return
        line = run_reference(args, world, rank, local, None)
        print(json.dumps(line), flush=True)
        return
    world, rank, local, pg = dist_setup()
    line = run_ours(args, world, rank, local, pg)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
