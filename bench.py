#!/usr/bin/env python3
"""Benchmark of the NPA rollout step: particle-steps/s.

Workload (default "cfg2"): batched 2D rollouts, 4,096 particles each, the
config-0 architecture (C=16, MLP 64->128->18, eps 0.05, grid 64x64 Particle
hash), one shared seeded MLP.  Each GPU rank runs its own shard of 256
rollouts (1,048,576 particles per step) with no collective on the step path
("scaling": "weak"); --strong instead splits the 256 rollouts over the ranks.

A bench step is one rollout step (hashgrid -> density -> fused perception +
MLP + Euler) over every particle of the shard.  The timed region is exactly K
steps on resident device state, bracketed by barrier + synchronize, timed with
CUDA events on the launching stream; the job time is the max over ranks.

Extra keys:
  roofline      dominant kernel (fused step) against measured HBM bandwidth,
                from CUDA events around each of its launches in the timed region
  compute_roof  the same kernel against the FP32 pipe (the MLP keeps the
                reference's multiply-then-add order, so it runs as FP32 ops)
  cpu_baseline  the CPU oracle (a port of the reference's CPU path) on a
                bounded sample of the same workload, all host threads
  e2e           the same metric through the public rollout API with host
                buffers: H2D of the initial particles from pinned memory, K
                steps, D2H of the final particles
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
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH_TOTAL = 256
PARTICLES = 4096
# Algorithmic HBM bytes of the MLP step kernel per particle (C = 16, F = 64):
# feature row read (4F = 256), position read + write (32), next state write
# (4C = 64), permutation read (4).
FUSED_BYTES_PER_PARTICLE = 356
# Whole rollout step per particle-step (hashgrid keys / permutation and the
# density round trip added): 184 + bin offsets (4 * 4097 / 4096).
STEP_BYTES_PER_PARTICLE = 188
METRIC = "particle-steps/s per rollout step at 1/2/4/8 B200; % of HBM roofline"


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


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def mark(self, which):
        if which == "begin":
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self, gpu_indices):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx in gpu_indices:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k] == "Active"})
        # Samples while the GPU is busy (under load) give the median clock.
        busy = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": float(np.median(busy)) if busy else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def visible_gpu_indices(world):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return [int(x) for x in vis.split(",")][:max(world, 1)]
        except ValueError:
            pass
    return list(range(max(world, 1)))


def cpu_baseline(workload_name, target_seconds=12.0):
    """Times the CPU oracle (port of the reference CPU path) on a bounded sample."""
    import oracle
    from burn_automata_b200 import workloads

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    w = workloads.make(workload_name, batch=4, steps=1)
    t = time.perf_counter()
    oracle.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, 1, w.dt)
    per_ps = (time.perf_counter() - t) / (w.batch * w.n)
    rollouts = int(min(64, max(4, target_seconds / 4 / (per_ps * w.n))))
    steps = int(min(16, max(1, target_seconds / (per_ps * w.n * rollouts))))
    w = workloads.make(workload_name, batch=rollouts, steps=steps)
    t = time.perf_counter()
    oracle.rollout(w.model, w.weights, w.grid, w.positions, w.states, w.batch, w.n, steps, w.dt)
    dt = time.perf_counter() - t
    return {"value": w.batch * w.n * steps / dt, "unit": "particle-steps/s", "cores": threads,
            "kind": "port",
            "sample": f"{rollouts} rollouts x {w.n} particles x {steps} steps of {workload_name}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    import oracle
    from burn_automata_b200 import workloads

    oracle.build()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    per_rank = BATCH_TOTAL // world if args.strong else BATCH_TOTAL
    # Calibrate a per-step sample of rollouts that takes ~1 s on the host.
    probe = workloads.make(args.workload, batch=4, steps=1)
    t = time.perf_counter()
    oracle.rollout(probe.model, probe.weights, probe.grid, probe.positions, probe.states,
                   probe.batch, probe.n, 1, probe.dt)
    per_rollout = (time.perf_counter() - t) / probe.batch
    sample = int(min(per_rank, max(1, 1.0 / max(per_rollout, 1e-6))))
    w = workloads.make(args.workload, batch=sample, steps=1)
    pos, st = w.positions.copy(), w.states.copy()
    for _ in range(args.warmup):
        pos, st, _ = oracle.rollout(w.model, w.weights, w.grid, pos, st, w.batch, w.n, 1, w.dt)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        pos, st, _ = oracle.rollout(w.model, w.weights, w.grid, pos, st, w.batch, w.n, 1, w.dt)
        times.append(time.perf_counter() - t)
    total = float(np.sum(times))
    value = sample * w.n * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "particle-steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; see burn_automata_b200/workloads.py)",
        "config": {"workload": args.workload, "rollouts_per_step_sample": sample,
                   "particles_per_rollout": w.n, "note": "CPU port of the reference path "
                   "(oracle/npa_oracle.c); the Rust reference cannot be built without cargo"},
        "cpu_baseline": {"value": value, "unit": "particle-steps/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{sample} rollouts x {w.n} particles per step"},
        "e2e": {"value": value, "unit": "particle-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import burn_automata_b200 as ba
    from burn_automata_b200 import multigpu, workloads

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    multigpu.init("nccl", multigpu.RankInfo(rank, world, local_rank), timeout_s=180, device=dev)
    lib = ba.load_library()
    total_rollouts = args.rollouts or BATCH_TOTAL
    first, per_rank = multigpu.shard(total_rollouts, world, rank, args.strong)
    w = workloads.make(args.workload, batch=per_rank, first=first)
    model = ba.NpaModel(w.model, ba.NpaWeights(w.weights.w1, w.weights.b1, w.weights.w2,
                                               w.weights.b2), device=local_rank)
    ex = ba.CudaAutomataExecutor(model, w.grid, w.batch, w.n)
    ex.create_state(w.positions, w.states)
    stream = torch.cuda.Stream()
    sptr = stream.cuda_stream
    ex.step_state_many(args.warmup, w.dt, use_graph=True, stream=sptr)
    torch.cuda.synchronize()

    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.npa_kernel_launch_count()
    if sampler:
        sampler.mark("begin")
    phase_ms, total_ms = ex.step_state_many_profiled(args.steps, w.dt, use_graph=True,
                                                     stream=sptr)
    if sampler:
        sampler.mark("end")
    torch.cuda.synchronize()
    launches = lib.npa_kernel_launch_count() - launches0
    if world > 1:
        dist.barrier()
    max_ms, fused_ms = multigpu.max_over_ranks([total_ms, float(phase_ms[:, 3].mean())], dev)
    clocks = sampler.stop(visible_gpu_indices(world)) if sampler else None

    particles_rank = w.batch * w.n
    # all ranks' particles (strong scaling may give ranks unequal shares)
    cnt = torch.tensor([float(particles_rank)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(cnt)
    particles_job = int(cnt.item())
    value = particles_job * args.steps / (max_ms / 1000.0)

    # e2e through the public rollout API with host buffers (rank-local, then max).
    e2e = None
    if not args.no_e2e:
        pin_pos = torch.from_numpy(w.positions).pin_memory()
        pin_st = torch.from_numpy(w.states).pin_memory()
        out_pos = torch.empty_like(pin_pos).pin_memory()
        out_st = torch.empty_like(pin_st).pin_memory()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ex.create_state(pin_pos.numpy(), pin_st.numpy())
        ex.step_state_many(args.steps, w.dt, use_graph=True, stream=sptr)
        p_, s_ = ex.read_state()
        out_pos.numpy()[:] = p_
        out_st.numpy()[:] = s_
        e2e_s = time.perf_counter() - t0
        e2e_s = multigpu.max_over_ranks([e2e_s], dev)[0]
        h2d = w.positions.nbytes + w.states.nbytes
        e2e = {"value": particles_job * args.steps / e2e_s, "unit": "particle-steps/s",
               "h2d_bytes_per_step": h2d / args.steps, "d2h_bytes_per_step": h2d / args.steps,
               "api": "CudaAutomataExecutor create_state + step_state_many + read_state",
               "note": "one upload of the initial particles and one readback of the final "
                       "particles per K-step rollout (per-step bytes are amortised)"}

    # one gather of per-shard checksums of the final states (validation only)
    fp, fs = ex.read_state()
    checksums = multigpu.gather_checksums(multigpu.shard_checksum(fp, fs), dev)

    if rank == 0:
        peak, peak_kind = load_peaks()
        fused_achieved = FUSED_BYTES_PER_PARTICLE * particles_rank / (fused_ms / 1000.0) / 1e9
        sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
        mlp_ops = 2 * (w.model.perception_dims() * w.model.hidden_dims
                       + w.model.hidden_dims * w.model.update_dims())
        fp32_peak = 148 * 128 * sm_mhz * 1e6 / 1e12
        fp32_achieved = mlp_ops * particles_rank / (fused_ms / 1000.0) / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.workload)
        line = {
            "metric": METRIC, "value": value, "unit": "particle-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded; see burn_automata_b200/workloads.py)",
            "config": {"workload": args.workload, "rollouts_per_gpu": per_rank,
                       "particles_per_rollout": w.n, "particles_per_gpu": particles_rank,
                       "state_dims": w.model.state_dims, "mlp": [w.model.perception_dims(),
                                                                 w.model.hidden_dims,
                                                                 w.model.update_dims()],
                       "eps": w.grid.eps, "grid": list(w.grid.grid_size[:2]),
                       "parallelism": f"{world} independent shards (no step-path collective)",
                       "l2": "no flush: per-step working set (~220 MB) exceeds the 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": "mlp_step_kernel",
                         "achieved": fused_achieved, "peak": peak, "unit": "GB/s",
                         "frac": fused_achieved / peak, "peak_source": peak_kind,
                         "traffic": None,
                         "bytes_per_particle": FUSED_BYTES_PER_PARTICLE,
                         "avg_launch_ms": fused_ms},
            "step_roofline": {"bound": "hbm", "achieved":
                              STEP_BYTES_PER_PARTICLE * value / world / 1e9, "peak": peak,
                              "unit": "GB/s",
                              "frac": STEP_BYTES_PER_PARTICLE * value / world / 1e9 / peak},
            "compute_roof": {"bound": "fp32", "achieved": fp32_achieved, "peak": fp32_peak,
                             "unit": "TFLOP/s (FP32 mul + add, reference order)",
                             "frac": fp32_achieved / fp32_peak},
            "phase_ms": {"hashgrid": float(phase_ms[:, 0].mean()),
                         "density": float(phase_ms[:, 1].mean()),
                         "perception": float(phase_ms[:, 2].mean()),
                         "mlp_step": float(phase_ms[:, 3].mean())},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "final_state_checksums": checksums,
        }
        print(json.dumps(line), flush=True)
    ex.close()
    model.close()
    if world > 1:
        dist.barrier()
    multigpu.finish()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2"])
    ap.add_argument("--strong", action="store_true",
                    help="split the 256 rollouts over the ranks instead of 256 per rank")
    ap.add_argument("--rollouts", type=int, default=None,
                    help="rollouts per rank (default: 256, or 256 / ranks with --strong)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
