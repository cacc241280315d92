#!/usr/bin/env python3
"""Benchmark of the NPA rollout hot path: particle-steps/s.

Workloads (--workload, default "cfg2"; seeded synthetic inputs from
burn_automata_b200/workloads.py):
  cfg0  one 2D rollout, 4,096 particles, C=16, MLP 64->128->18
  cfg1  hashgrid build + perception alone, 1,048,576 2D particles, C=32, F=130
  cfg2  256 independent cfg0-architecture rollouts of 4,096 particles, split
        evenly over the GPUs ("scaling": "strong"; 32 rollouts per GPU at 8)
  cfg3  one 3D torus rollout, 16,384 particles, C=32, MLP 160->256->35
  cfg4  one clustered 2D rollout, 4,194,304 particles (64-component mixture)
No collective runs on the step path: each rank steps its own shard.  A
single-rollout configuration does not shard, so at N > 1 each rank runs an
independent replica ("weak"); --strong --rollouts R splits R rollouts over
the ranks (cfg4 x 8), --weak gives every rank a full cfg2 batch.  After the
timed region rank 0 checks every rank's final rollouts bit for bit against a
1-GPU rerun of the same rollouts ("validation").

A bench step is one rollout step (hashgrid -> density -> perception ->
MLP + Euler) over every particle of the shard; for cfg1 it is one hashgrid
build + perception pass (features and density written).  The timed region is
exactly K steps on resident device state, bracketed by barrier + synchronize,
timed with CUDA events on the launching stream; the job time is the max over
ranks.  The per-step working set exceeds the 126 MB L2 for cfg1, cfg2 and
cfg4; cfg0 and cfg3 are small single rollouts that stay L2-resident (stated in
the line's config).

Extra keys:
  roofline       dominant kernel (MLP step kernel; perception for cfg1)
                 against measured HBM bandwidth, from CUDA events around each
                 of its launches in the timed region
  step_roofline  the whole step's algorithmic bytes against HBM bandwidth
  compute_roof   the MLP step kernel against the FP32 pipe (the MLP keeps the
                 reference's multiply-then-add order, so it runs as FP32 ops)
  cpu_baseline   the CPU oracle (a port of the reference's CPU path) on a
                 bounded sample of the same workload, all host threads
  e2e            the same metric through the host-buffer call a drop-in user
                 makes (step_cpu / perceive_with_options): per step, H2D of
                 that step's inputs from pinned memory and D2H of its outputs
--impl reference times the CPU port alone (the reference's own Rust/rayon
path cannot be built here: no cargo / rustc).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "particle-steps/s per rollout step at 1/2/4/8 B200; % of HBM roofline"
DATA = "synthetic (seeded; see burn_automata_b200/workloads.py)"

# rollouts (in total for the batched configuration, per rank otherwise), kind
# of step, default timed steps
WORKLOADS = {
    "cfg0": {"rollouts": 1, "kind": "step", "steps": 200},
    "cfg1": {"rollouts": 1, "kind": "perception", "steps": 50},
    "cfg2": {"rollouts": 256, "kind": "step", "steps": 200, "batched": True},
    "cfg3": {"rollouts": 1, "kind": "step", "steps": 100},
    "cfg4": {"rollouts": 1, "kind": "step", "steps": 5},
}

# DRAM bytes (read + write) of one launch of the dominant kernel, from the
# committed ncu captures, per particle of that launch:
#   profiles/mlp_step_kernel_cfg2.txt: 356.7 MB + 71.1 MB for 1,048,576 rows;
#   profiles/perception_kernel_cfg1.txt: 1306.5 MB + 620.9 MB for 1,048,576 particles.
NCU_TRAFFIC_PER_PARTICLE = {
    ("cfg2", "mlp_step_kernel"): (356.652288e6 + 71.074048e6) / 1048576,
    ("cfg1", "perception_kernel"): (1306.484736e6 + 620.867840e6) / 1048576,
}
NCU_TRAFFIC_SOURCE = {
    ("cfg2", "mlp_step_kernel"): "profiles/mlp_step_kernel_cfg2.txt",
    ("cfg1", "perception_kernel"): "profiles/perception_kernel_cfg1.txt",
}


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def grid_cells(grid) -> int:
    gs = list(grid.grid_size) + [1, 1, 1]
    return int(np.prod(gs[:grid.dim]))


def mlp_kernel_bytes(model) -> int:
    """Algorithmic HBM bytes per particle of the MLP step kernel: feature row
    read (4F), position read + write (32), own state read and next state
    write (8C), permutation read (4)."""
    return 4 * model.perception_dims() + 32 + 8 * model.state_dims + 4


def fused_kernel_bytes(model) -> int:
    """The fused step kernel per particle: the MLP stage's bytes without the
    feature row, plus the perception's own reads: hit list and count (~40),
    own state (4C), volume (4) and record (16)."""
    return 32 + 8 * model.state_dims + 4 + 40 + 4 * model.state_dims + 4 + 16


def step_bytes(w) -> float:
    """Whole rollout step per particle-step: position read + write (32),
    state read + write (8C), density write + read (8), hashgrid key /
    permutation write + read (16), bin offsets 4 (B cells + 1) / (B N)."""
    offsets = 4.0 * (grid_cells(w.grid) * w.batch + 1) / (w.batch * w.n)
    return 32 + 8 * w.state_dims + 8 + 16 + offsets


def perception_kernel_bytes(w, features) -> int:
    """cfg1 perception kernel per particle: own position (16) and state (4C)
    read, volume read (4), feature row write (4F)."""
    return 16 + 4 * w.state_dims + 4 + 4 * features


def mean_neighbours(w) -> float:
    """Mean in-radius neighbours per particle (self included) of a workload's
    positions: r < eps, within each rollout (2D / 3D Euclidean; Grid-mode
    periodic wrap is not modelled -- cfg1 is Particle mode)."""
    from scipy.spatial import cKDTree

    d = w.grid.dim
    counts = []
    for b in range(w.batch):
        p = w.positions[b * w.n:(b + 1) * w.n, :d].astype(np.float64)
        counts.append(cKDTree(p).query_ball_point(p, w.grid.eps, return_length=True))
    return float(np.mean(np.concatenate(counts)))


def perception_flops(w, neighbours) -> float:
    """Algorithmic FP32 operations of one particle's perception with the full
    option set (state and density gradients, hybrid moment, log-normalised;
    forward.rs:249-295, normalize.rs), each multiply, add, square root,
    division and ln_1p counted as one:
      per in-radius neighbour other than itself: 8 per channel (blur 3, state
        gradient 5) + 37 (delta 2, r^2 3, poly6 4, two spiky magnitudes 14,
        gradient vector 2, density gradient 4, moment 8);
      its own pair: 9 + 3 per channel;
      per particle: moment inverse 8 + 19 per channel (correction 8, scale 2,
        log-normalisation 9) + density gradient 11."""
    c = w.state_dims
    return (neighbours - 1.0) * (8 * c + 37) + (9 + 3 * c) + 8 + 19 * c + 11


def perception_step_bytes(w, features) -> float:
    """cfg1 pass per particle: position read (16), state read (4C), density
    write + read (8), hashgrid (16), feature write (4F), offsets."""
    offsets = 4.0 * (grid_cells(w.grid) * w.batch + 1) / (w.batch * w.n)
    return 16 + 4 * w.state_dims + 8 + 16 + 4 * features + offsets


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled DURING the timed
    region.  NVML is polled every few milliseconds from a thread started
    right before the timed region and stopped right after it, on every GPU of
    the job, so even a short region gets samples taken under load; without
    NVML, nvidia-smi at its 100 ms floor.  sm_mhz is the median over the
    samples taken inside the region (the GPU is busy throughout it)."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4),
               ("hw_power_brake_slowdown", 0x80))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_devices, period_s=0.004):
        self.cuda_devices = list(cuda_devices)
        self.period_s = period_s
        self.samples = []
        self.handles = []
        self.nvml = None
        self.proc = None
        self.path = None
        self.thread = None
        self.running = False

    def _nvml_handles(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        handles = []
        for d in self.cuda_devices:
            p = torch.cuda.get_device_properties(d)
            h = None
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{p.uuid}")
            except Exception:
                try:
                    bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                    h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
                except Exception:
                    h = None
            if h is not None:
                handles.append(h)
        return pynvml, handles

    def _poll(self):
        nv = self.nvml
        while self.running:
            for h in self.handles:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(sm), float(mx), int(rs)))
                except Exception:
                    pass
            time.sleep(self.period_s)

    def start(self):
        import threading

        try:
            self.nvml, self.handles = self._nvml_handles()
        except Exception:
            self.nvml, self.handles = None, []
        if self.handles:
            self.running = True
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.running = False
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            sm = [s[0] for s in self.samples]
            names = sorted({n for s in self.samples for n, bit in self.REASONS if s[2] & bit})
            return {"sm_mhz": float(np.median(sm)), "sm_min_mhz": min(sm),
                    "sm_max_mhz": max(s[1] for s in self.samples), "reasons": names,
                    "samples": len(self.samples), "gpus": len(self.handles),
                    "source": "nvml, polled every ~4 ms inside the timed region"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [[p.strip() for p in line.split(",")]
                for line in Path(self.path).read_text().splitlines()]
        os.unlink(self.path)
        rows = [r for r in rows if len(r) >= 9]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        if not sm:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k] == "Active"})
        return {"sm_mhz": float(np.median(sm)), "sm_min_mhz": min(sm),
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi -lms 100 inside the timed region"}


# ---- CPU samples (the oracle: a port of the reference CPU path) ----

class CpuSample:
    """A bounded, per-particle-representative piece of a workload for the CPU
    port: whole rollouts of a batched config, one mixture component of cfg4
    (its particle density), a density-preserving sub-square of cfg1, or the
    single rollout of cfg0 / cfg3."""

    def __init__(self, name, size, seed=0):
        from burn_automata_b200 import workloads

        self.name = name
        if name == "cfg4":
            self.w = workloads.make("cfg4", seed, n=65536, components=1)
            self.desc = "one 65,536-particle component of the cfg4 mixture (sigma 0.02)"
        elif name == "cfg1":
            full = 1 << 20
            n = int(max(4096, min(full, size)))
            half = float(np.sqrt(n / full))
            self.w = workloads.make("cfg1", seed, n=n)
            self.w.positions[:, :2] = workloads.uniform_positions_2d(n, seed, -half, half)[:, :2]
            self.desc = (f"{n:,} cfg1 particles uniform in [-{half:.3f},{half:.3f}]^2 "
                         "(cfg1's particle density)")
        elif name == "cfg2":
            b = int(max(1, min(256, size)))
            self.w = workloads.make("cfg2", seed, batch=b)
            self.desc = f"{b} of the 256 cfg2 rollouts"
        else:
            self.w = workloads.make(name, seed)
            self.desc = f"the {name} rollout"
        self.particles = self.w.batch * self.w.n

    def run(self, pos=None, st=None):
        """One step of the sample; returns (positions, states) after it."""
        import oracle

        w = self.w
        pos = w.positions if pos is None else pos
        st = w.states if st is None else st
        if w.model is None:
            oracle.perceive_with_options(pos, st, w.batch, w.n, w.state_dims, w.grid, w.options)
            return pos, st
        p, s, _ = oracle.rollout(w.model, w.weights, w.grid, pos, st, w.batch, w.n, 1, w.dt)
        return p, s


def calibrated_sample(name, seconds_per_step):
    """The CpuSample whose one step takes about `seconds_per_step` here."""
    probe_size = {"cfg1": 1 << 16, "cfg2": 2}.get(name, 1)
    s = CpuSample(name, probe_size)
    t = time.perf_counter()
    s.run()
    per_particle = (time.perf_counter() - t) / s.particles
    if name == "cfg1":
        return CpuSample(name, seconds_per_step / max(per_particle, 1e-12))
    if name == "cfg2":
        return CpuSample(name, seconds_per_step / max(per_particle * s.w.n, 1e-12))
    return s


def cpu_baseline(name, target_seconds=12.0):
    """The CPU port timed on a bounded sample (about target_seconds)."""
    import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    s = calibrated_sample(name, target_seconds / 4)
    t = time.perf_counter()
    pos, st = s.run()
    one = time.perf_counter() - t
    if one >= target_seconds / 2:  # one step is already a long enough sample
        return {"value": s.particles / one, "unit": "particle-steps/s", "cores": threads,
                "kind": "port", "sample": f"1 step of {s.desc}"}
    steps = int(min(16, max(1, target_seconds / max(one, 1e-6))))
    t = time.perf_counter()
    for _ in range(steps):
        pos, st = s.run(pos, st)
    dt = time.perf_counter() - t
    return {"value": s.particles * steps / dt, "unit": "particle-steps/s", "cores": threads,
            "kind": "port", "sample": f"{steps} step(s) of {s.desc}"}


def run_reference(args, rank, world):
    """CPU port of the reference path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import oracle

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    budget = min(1.0, 150.0 / max(args.steps + args.warmup, 1))
    s = calibrated_sample(args.workload, budget)
    pos = st = None
    for _ in range(args.warmup):
        pos, st = s.run(pos, st)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        pos, st = s.run(pos, st)
        times.append(time.perf_counter() - t)
    total = float(np.sum(times))
    value = s.particles * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "particle-steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
        "scaling": shard_plan(args, world, rank)[2], "vs_baseline": None, "dtype": "f32",
        "data": DATA,
        "config": {"workload": args.workload, "sample": s.desc,
                   "note": "CPU port of the reference path (oracle/npa_oracle.c); the Rust "
                           "reference cannot be built without cargo"},
        "cpu_baseline": {"value": value, "unit": "particle-steps/s", "cores": threads,
                         "kind": "port", "sample": f"per step: {s.desc}"},
        "e2e": {"value": value, "unit": "particle-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- GPU arm ----

def pinned(shape):
    import torch

    return torch.empty(shape, dtype=torch.float32).pin_memory().numpy()


def shard_plan(args, world, rank):
    """(first rollout, rollouts on this rank, scaling) for this rank.

    The batched configuration (cfg2) splits its 256 rollouts over the ranks
    ("strong": 32 rollouts per GPU at 8 GPUs), as the configuration says;
    --weak gives every rank its own full batch instead.  A single-rollout
    configuration does not shard: at N > 1 each rank runs an independent
    replica (rank r draws rollout r; "weak"), unless --strong splits an
    explicit --rollouts over the ranks (cfg4 x 8: --rollouts 8 --strong)."""
    from burn_automata_b200 import multigpu

    spec = WORKLOADS[args.workload]
    total = args.rollouts or spec["rollouts"]
    strong = args.strong or (spec.get("batched", False) and not args.weak)
    first, count = multigpu.shard(total, world, rank, strong)
    return first, count, ("strong" if strong else "weak")


def final_state(args, w, local_rank, steps, stream_ptr):
    """One GPU's result for shard `w` after `steps` bench steps, run from the
    start: the executor's state after `steps` rollout steps (graph replays),
    or one perception pass (cfg1, whose input does not evolve)."""
    import burn_automata_b200 as ba
    import torch

    dev = torch.device("cuda", local_rank)
    if WORKLOADS[args.workload]["kind"] == "perception":
        runner = ba.DevicePerception(w.grid, w.options, w.batch, w.n, w.state_dims, local_rank)
        runner(torch.from_numpy(w.positions).to(dev), torch.from_numpy(w.states).to(dev),
               stream=stream_ptr)
        torch.cuda.synchronize()
        return runner.features.cpu().numpy(), runner.density.cpu().numpy()
    model = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                               w.weights.b2), device=local_rank)
    ex = ba.CudaAutomataExecutor(model, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states)
    ex.step_state_many(steps, w.dt, use_graph=True, stream=stream_ptr)
    out = ex.read_state()
    ex.close()
    model.close()
    return out


def validate_against_one_gpu(args, world, local_rank, plans, gathered, steps, stream_ptr):
    """Rank 0, after the timed region: reruns every rank's rollouts on this
    one GPU from the same seeded inputs for the same number of steps and
    compares the per-rollout digests bit for bit.  Rollouts are independent
    and the kernels deterministic, so a sharded run must reproduce the
    1-GPU run exactly.  Returns the validation record for the JSON line."""
    from burn_automata_b200 import multigpu, workloads

    if world <= 1:
        return {"checked": False, "reason": "1 GPU: nothing sharded"}
    if args.workload == "cfg4":
        return {"checked": False,
                "reason": "a 1-GPU rerun of the 4,194,304-particle rollouts takes minutes"}
    t0 = time.perf_counter()
    expected = {}
    spec = WORKLOADS[args.workload]
    batched = spec.get("batched", False)
    if batched and len({(f, c) for f, c in plans}) == len(plans):
        lo = min(f for f, _ in plans)
        hi = max(f + c for f, c in plans)
        w = workloads.make(args.workload, batch=hi - lo, first=lo)
        expected.update(multigpu.rollout_digests(w.batch, lo, *final_state(args, w, local_rank, steps,
                                                            stream_ptr)))
    else:
        for first, count in sorted(set(plans)):
            w = workloads.make(args.workload, batch=count, first=first)
            expected.update(multigpu.rollout_digests(w.batch, first, *final_state(args, w, local_rank, steps,
                                                                   stream_ptr)))
    checked, mismatched = multigpu.compare_digests(gathered, expected)
    return {"checked": True, "rollouts": checked, "bit_exact": not mismatched,
            "mismatched_rollouts": mismatched[:16],
            "method": "per-rollout blake2b digests of the final positions + states of every "
                      "rank, gathered once after timing, against a 1-GPU rerun of the same "
                      "rollouts for the same number of steps on rank 0",
            "rerun_s": round(time.perf_counter() - t0, 3)}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import burn_automata_b200 as ba
    from burn_automata_b200 import multigpu, workloads

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    multigpu.init("nccl", multigpu.RankInfo(rank, world, local_rank), timeout_s=180, device=dev)
    lib = ba.load_library()
    spec = WORKLOADS[args.workload]
    first, per_rank, scaling = shard_plan(args, world, rank)
    w = workloads.make(args.workload, batch=per_rank, first=first,
                       **({"n": args.particles} if args.particles else {}),
                       **({"components": args.components} if args.components else {}))
    particles_rank = w.batch * w.n
    stream = torch.cuda.Stream(dev)
    sptr = stream.cuda_stream
    perception_only = spec["kind"] == "perception"

    step_groups = None
    if perception_only:
        runner = ba.DevicePerception(w.grid, w.options, w.batch, w.n, w.state_dims, local_rank)
        d_pos = torch.from_numpy(w.positions).to(dev)
        d_st = torch.from_numpy(w.states).to(dev)
        for _ in range(args.warmup):
            runner(d_pos, d_st, stream=sptr)
        features = runner.feature_dims
    else:
        model = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                                   w.weights.b2), device=local_rank)
        ex = ba.CudaAutomataExecutor(model, w.grid, w.batch, w.n)
        ex.create_state(w.positions, w.states)
        if args.fused or args.ws:
            ex.set_fused_step(2 if args.ws else True)
        if args.groups:
            ex.set_step_groups(args.groups)
        step_groups = ex.step_groups
        ex.step_state_many(args.warmup, w.dt, use_graph=True, stream=sptr)
        features = w.model.perception_dims()
    torch.cuda.synchronize()

    sampler = ClockSampler(range(world)) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    launches0 = lib.npa_kernel_launch_count()
    if perception_only:
        phase_ms, total_ms = runner.run_profiled(d_pos, d_st, args.steps, stream=sptr)
        dominant = phase_ms[:, 2]
    else:
        # the step as a user replays it: whole-step graphs, no events inside
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        ex.step_state_many(args.steps, w.dt, use_graph=True, stream=sptr)
        ev1.record(stream)
        ev1.synchronize()
        total_ms = ev0.elapsed_time(ev1)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    launches = lib.npa_kernel_launch_count() - launches0
    extra_steps = 0
    if not perception_only:
        # per-phase times from a separate run with events between the phases
        # (after the timed region: the events add a few microseconds per phase)
        extra_steps = min(args.steps, 50)
        phase_ms, _ = ex.step_state_many_profiled(extra_steps, w.dt, use_graph=True,
                                                  stream=sptr)
        dominant = phase_ms[:, 3]
    if world > 1:
        dist.barrier()
    max_ms, dom_ms = multigpu.max_over_ranks([total_ms, float(dominant.mean())], dev)
    rank_ms = multigpu.gather_floats(total_ms, dev)

    # all ranks' particles (strong scaling may give ranks unequal shares)
    cnt = torch.tensor([float(particles_rank)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(cnt)
    particles_job = int(cnt.item())
    value = particles_job * args.steps / (max_ms / 1000.0)

    # one gather of per-rollout digests of the final states, checked on rank 0
    # against a 1-GPU rerun (validation only, outside the timed region)
    if perception_only:
        fp, fs = runner.features.cpu().numpy(), runner.density.cpu().numpy()
    else:
        fp, fs = ex.read_state()
    digests = multigpu.rollout_digests(w.batch, first, fp, fs)
    gathered = multigpu.gather_objects(digests)
    plans = multigpu.gather_objects((first, per_rank))
    validation = None
    if rank == 0:
        steps_done = args.warmup + args.steps + extra_steps
        validation = validate_against_one_gpu(args, world, local_rank, plans, gathered,
                                              steps_done, sptr)

    # e2e through the host-buffer call of a drop-in user, one call per step
    e2e = None
    if not args.no_e2e:
        if perception_only:
            inp = (pinned((particles_rank, 4)), pinned(particles_rank * w.state_dims))
            inp[0][:] = w.positions
            inp[1][:] = w.states
            out = (pinned(particles_rank * features), pinned(particles_rank))

            def one(k):
                ba.perceive_with_options(inp[0], inp[1], w.batch, w.n, w.state_dims, w.grid,
                                         w.options, outputs=(), out=out)
            h2d = inp[0].nbytes + inp[1].nbytes
            d2h = out[0].nbytes + out[1].nbytes
            api = ("perceive_with_options (C ABI npa_perceive_with_options) with pinned host "
                   "buffers, features + density copied back, one call per step")
        else:
            bufs = [(pinned((particles_rank, 4)), pinned(particles_rank * w.state_dims))
                    for _ in range(2)]
            bufs[0][0][:] = w.positions
            bufs[0][1][:] = w.states

            def one(k):
                src, dst = bufs[k % 2], bufs[(k + 1) % 2]
                model.step(src[0], src[1], w.batch, w.n, w.grid, w.dt, outputs=(), out=dst)
            h2d = d2h = bufs[0][0].nbytes + bufs[0][1].nbytes
            api = ("NpaModel.step (C ABI npa_model_step, the step_cpu drop-in) with pinned "
                   "host buffers, next positions + states copied back, one call per step")
        for k in range(args.warmup):
            one(k)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for k in range(args.steps):
            one(k)
        e2e_s = multigpu.max_over_ranks([time.perf_counter() - t0], dev)[0]
        e2e = {"value": particles_job * args.steps / e2e_s, "unit": "particle-steps/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": api}

    if rank == 0:
        peak, peak_kind = load_peaks()
        if perception_only:
            kernel, kbytes = "perception_kernel", perception_kernel_bytes(w, features)
            sbytes = perception_step_bytes(w, features)
            names = ["hashgrid", "density", "perception"]
        else:
            if args.fused or args.ws:
                kernel = "ws_step_kernel" if args.ws else "fused_step_kernel"
                kbytes = fused_kernel_bytes(w.model)
            else:
                kernel, kbytes = "mlp_step_kernel", mlp_kernel_bytes(w.model)
            sbytes = step_bytes(w)
            names = ["hashgrid", "density", "perception", "mlp_step"]
        achieved = kbytes * particles_rank / (dom_ms / 1000.0) / 1e9
        tr = NCU_TRAFFIC_PER_PARTICLE.get((args.workload, kernel))
        if world == 1:
            parallelism = "1 GPU"
        elif scaling == "strong":
            parallelism = (f"{world} shards of the {args.rollouts or spec['rollouts']} rollouts "
                           "(no step-path collective)")
        else:
            parallelism = f"{world} independent replicas / shards (no step-path collective)"
        line = {
            "metric": METRIC, "value": value, "unit": "particle-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": "f32", "data": DATA,
            "config": {"workload": (args.workload if not (args.particles or args.components)
                                    else f"{args.workload} reduced: {w.n} particles per rollout"
                                         + (f", {args.components} components"
                                            if args.components else "")),
                       "rollouts_per_gpu": per_rank,
                       "rollouts_total": sum(c for _, c in plans),
                       "particles_per_rollout": w.n, "particles_per_gpu": particles_rank,
                       "state_dims": w.state_dims, "features": features,
                       "eps": w.grid.eps, "grid": list(w.grid.grid_size[:w.grid.dim]),
                       "parallelism": parallelism,
                       "step_kernels": ("warp-specialised fused perception + MLP + Euler"
                                        if args.ws else
                                        "fused perception + MLP + Euler" if args.fused
                                        else "perception tiles, then MLP + Euler"),
                       "step_groups": step_groups,
                       "l2": ("no flush: per-step working set exceeds the 126 MB L2"
                              if particles_rank >= (1 << 20) else
                              "no flush: the shard's per-step working set is below the 126 MB "
                              "L2 and stays resident, as a rollout of this size does")},
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": tr * particles_rank if tr else None,
                         "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                            + NCU_TRAFFIC_SOURCE[(args.workload, kernel)]) if tr else None,
                         "bytes_per_particle": kbytes, "avg_launch_ms": dom_ms},
            "step_roofline": {"bound": "hbm", "achieved": sbytes * value / world / 1e9,
                              "peak": peak, "unit": "GB/s",
                              "frac": sbytes * value / world / 1e9 / peak,
                              "bytes_per_particle": sbytes},
            "phase_ms": {k: float(phase_ms[:, i].mean()) for i, k in enumerate(names)},
            "rank_ms_per_step": [t / args.steps for t in rank_ms],
            "gpu_launches": int(launches),
            "clocks": clocks,
            "validation": validation,
        }
        sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * sm_mhz * 1e6 / 1e12
        if perception_only:
            nbr = mean_neighbours(w)
            flops = perception_flops(w, nbr)
            fp32_achieved = flops * particles_rank / (dom_ms / 1000.0) / 1e12
            line["compute_roof"] = {
                "bound": "fp32", "kernel": kernel, "achieved": fp32_achieved, "peak": fp32_peak,
                "frac": fp32_achieved / fp32_peak, "flops_per_particle": flops,
                "mean_neighbours": nbr,
                "unit": "TFLOP/s (algorithmic FP32 operations of the pair sums and the "
                        "per-particle finish, sqrt / division / ln_1p counted as one; peak = 148 SM "
                        "x 128 lanes x median SM clock)"}
        if not perception_only:
            mlp_ops = 2 * (features * w.model.hidden_dims
                           + w.model.hidden_dims * w.model.update_dims())
            fp32_peak = 148 * 128 * sm_mhz * 1e6 / 1e12
            fp32_achieved = mlp_ops * particles_rank / (dom_ms / 1000.0) / 1e12
            line["compute_roof"] = {"bound": "fp32", "kernel": kernel, "achieved": fp32_achieved,
                                    "peak": fp32_peak, "frac": fp32_achieved / fp32_peak,
                                    "unit": "TFLOP/s (FP32 mul + add, reference order; peak = "
                                            "148 SM x 128 lanes x median SM clock)"}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.workload)
        line["cpu_baseline"] = cpu
        line["e2e"] = e2e
        print(json.dumps(line), flush=True)
    if not perception_only:
        ex.close()
        model.close()
    if world > 1:
        dist.barrier()
    multigpu.finish()


def fp32_ceiling():
    """The MLP's layer-1 register tile alone (npa_debug_fp32_tile_rate): 64
    products and 64 sums per k step from shared memory, nothing else.  Its
    rate against 148 SMs x 128 lanes x the sampled clock is the practical FP32
    ceiling of exact-order multiply-add (a rounded multiply, then a rounded
    add)."""
    import ctypes

    import burn_automata_b200 as ba
    import torch

    lib = ba.load_library()
    torch.cuda.init()
    sampler = ClockSampler([0])
    sampler.start()
    rate, ms = ctypes.c_double(0.0), ctypes.c_double(0.0)
    status = lib.npa_debug_fp32_tile_rate(4000, ctypes.byref(rate), ctypes.byref(ms))
    clocks = sampler.stop()
    if status != 0:
        raise SystemExit(f"probe failed: {lib.npa_last_error_message().decode()}")
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    peak = 148 * 128 * mhz * 1e6
    print(json.dumps({"probe": "exact-order FP32 register tile (MLP layer 1 inner loop)",
                      "ops_per_s": rate.value, "kernel_ms": ms.value, "peak_ops_per_s": peak,
                      "frac": rate.value / peak, "clocks": clocks}))


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default per workload: cfg0/cfg2 200, cfg1 50, cfg3 100, "
                         "cfg4 5)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS))
    ap.add_argument("--strong", action="store_true",
                    help="split --rollouts over the ranks (the default for cfg2)")
    ap.add_argument("--weak", action="store_true",
                    help="cfg2: every rank runs its own full batch instead of a share of it")
    ap.add_argument("--rollouts", type=int, default=None,
                    help="rollouts in total (split over the ranks) for cfg2 or with --strong; "
                         "per rank otherwise (default: 256 for cfg2, 1 otherwise)")
    ap.add_argument("--fused", action="store_true",
                    help="executor step as one perception + MLP + Euler kernel after the density "
                         "pass (2D, sparse cells)")
    ap.add_argument("--ws", action="store_true",
                    help="executor step as the warp-specialised fused kernel (perception and MLP "
                         "warps in one block per SM)")
    ap.add_argument("--groups", type=int, default=None,
                    help="replay the shard's rollouts as this many independent chains (1-4; "
                         "default: the executor's choice)")
    ap.add_argument("--particles", type=int, default=None,
                    help="particles per rollout instead of the workload's (reduced cases for "
                         "profiling; the bench line then names a reduced workload)")
    ap.add_argument("--components", type=int, default=None,
                    help="cfg4: mixture components (1 with --particles 65536 is one component at "
                         "the full draw's density)")
    ap.add_argument("--fp32-ceiling", action="store_true",
                    help="print the FP32 pipe rate of the MLP's exact-order register tile alone "
                         "(the ceiling the MLP kernel can approach) and exit")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.strong and args.weak:
        ap.error("--strong and --weak exclude each other")
    if args.steps is None:
        args.steps = WORKLOADS[args.workload]["steps"]
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.fp32_ceiling:
        fp32_ceiling()
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
