"""Benchmark of the batched AVBD environment step: the pure-engine step of
the synthetic biped.

Workload: the seed-0 synthetic biped, 4096 environments per GPU, dt 5 ms,
4 substeps per control step, 10 AVBD iterations, fp32, PD targets HOME +
N(0, 0.05 rad) drawn once per environment, no self-contact, kp 20 N m/rad,
torque cap 2 N m.  200 control steps settle the robots (untimed), then W
warm-up steps, then K timed steps.  One step = one `CudaBatch.step` call = one
kernel launch advancing every environment 4 physics steps.

Metric: physics env-steps/s = envs x substeps x K / device seconds (the
reference's formula, scripts/benchmark_engines.py:551), summed over ranks and
divided by the slowest rank's time.  The L2 cache is flushed (256 MiB write)
between timed steps, outside the timed events.  After the K steps the
reference's own method runs beside it (median of 5 trials x 200 steps), then
the end-to-end pass through the public API with host copies every step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...

``--workload config3`` (91-pair self-contact BAM env, 16384 envs per GPU),
``--workload config4`` (PPO rollout and update) and ``--workload config5``
(65536 domain-randomised envs per GPU at 20 iterations) time the larger
workloads (see run_extended and run_ppo); the default, the 4096-env
pure-engine step, is the headline line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ENVS = 4096
SUBSTEPS = 4
ITERATIONS = 10
DT = 0.005
SETTLE = 200
NOISE = 0.05
TRIALS = 5           # the reference's method: median of 5 trials ...
TRIAL_STEPS = 200    # ... of 200 control steps each
FLOP_STEPS = 20      # control steps the flop count follows from the timed states
METRIC = "physics env-steps/s"
UNIT = "env-steps/s"


def workload(args):
    return {
        "workload": "config 2: synthetic biped (seed 0), fixed HOME + N(0,0.05 rad) PD targets, ground contact only",
        "envs_per_gpu": args.envs,
        "substeps_per_step": SUBSTEPS,
        "iterations": ITERATIONS,
        "dt": DT,
        "settle_steps": SETTLE,
        "kp": None,
        "torque_limit": None,
        "l2": "GPU: flushed between timed steps (256 MiB write, outside the timed events); CPU arm: host run",
        "parallelism": f"env shards x{args.gpus}, no physics communication",
    }


def make_model(directory, seed=0):
    from duck_gym_b200 import biped

    path = biped.write(directory, seed=seed)
    meta = json.loads((Path(directory) / "metadata.json").read_text())
    return path, meta


def fixed_targets(meta, envs, seed):
    rng = np.random.default_rng(seed)
    home = np.asarray(meta["home"], np.float32)
    return (home + rng.normal(0, NOISE, (envs, home.size))).astype(np.float32)


REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """SM clock and throttle-reason samples taken while the timed region runs.

    Reads NVML in-process every 5 ms (read-only queries), so even a timed
    region of a few milliseconds holds samples; falls back to an nvidia-smi
    loop at 100 ms where NVML cannot be loaded."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD = 0.005

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.thread = None
        self.running = False
        self.lines = []      # (monotonic time, sm MHz, max MHz, power W, set of reasons)
        self.window = None   # (start, end) of the timed region
        self.source = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        """Start sampling; returns once the first sample has arrived."""
        try:
            nvml, handle = self._nvml_handle()
            bits = {"hw_slowdown": nvml.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nvml.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nvml.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nvml.nvmlClocksEventReasonSwPowerCap}
            sm_max = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))

            def poll():
                while self.running:
                    try:
                        sm = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
                        mask = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        power = nvml.nvmlDeviceGetPowerUsage(handle) / 1e3
                    except Exception:
                        break
                    self.lines.append((time.monotonic(), sm, sm_max, power,
                                       {name for name, bit in bits.items() if mask & bit}))
                    time.sleep(self.PERIOD)

            self.running = True
            self.source = "NVML in-process, every 5 ms"
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
        except Exception:
            self._start_smi()
        deadline = time.monotonic() + 10
        while not self.lines and time.monotonic() < deadline:
            time.sleep(0.01)

    def _start_smi(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi every 100 ms"

            def read():
                for line in self.proc.stdout:
                    parts = [p.strip() for p in line.split(",")]
                    try:
                        self.lines.append((time.monotonic(), float(parts[1]), float(parts[2]), float(parts[3]),
                                           {n for n, f in zip(REASONS, parts[5:9]) if f.lower() == "active"}))
                    except (ValueError, IndexError):
                        continue

            self.thread = threading.Thread(target=read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def stop(self):
        self.running = False
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self, window=None):
        """Samples taken while the timed region (or `window`) ran."""
        sm, reasons, sm_max, power = [], set(), None, []
        start, end = window or self.window or (-1e30, 1e30)
        for when, mhz, top, watts, active in self.lines:
            if start <= when <= end:
                sm.append(mhz)
                sm_max = top
                power.append(watts)
                reasons |= active
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": sm_max, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None, "source": self.source}


def count_flops(model, meta, targets, records, steps):
    """Algorithmic flops per physics env-step, counted by the CPU oracle's
    counting scalar on the states the timed region starts from: `records` are
    the envs' portable records exported right before the timed steps, advanced
    `steps` control steps with the same `targets` [envs, J]."""
    from oracle.oracle import count_ops

    envs = targets.shape[0]
    c = count_ops(model, np.asarray(meta["home"], np.float32), np.repeat(targets[None], steps, axis=0),
                  np.zeros((envs, 3), np.float32), DT, ITERATIONS, SUBSTEPS, meta["kp"], meta["torque_limit"],
                  records=records, threads=min(64, os.cpu_count() or 1))
    flops = c["add"] + c["mul"] + c["div"] + c["sqrt"]
    transcendental = c["sin"] + c["cos"] + c["tan"] + c["atan2"] + c["hypot"] + c["remainder"]
    n = c["physics_steps"]
    return {"flops_per_env_step": flops / n, "transcendentals_per_env_step": transcendental / n,
            "gs_iterations_per_env_step": c["gs_iterations"] / n,
            "sample": f"all {envs} envs from the timed region's starting states x {steps} control steps"}


def reference_batch(model, envs, cores):
    """The reference's own CPU solver (oracle/_ref CpuBatch32), else the CPU
    restatement, with the kind string for the JSON line."""
    from oracle.oracle import OracleBatch, reference_module

    ref = reference_module()
    if ref is not None:
        return ref.CpuBatch32(str(model), envs, DT, ITERATIONS, cores), "reference"
    return OracleBatch(model, envs, DT, ITERATIONS, threads=cores), "port"


def cpu_settled(model, meta, envs, cores, settle=SETTLE):
    """A CPU batch on the bench workload after the same untimed settle steps
    as the GPU arm (HOME start, fixed targets)."""
    batch, kind = reference_batch(model, envs, cores)
    target = fixed_targets(meta, envs, 0)
    forces = np.zeros((envs, 3), np.float32)
    for _ in range(settle):
        batch.step(target, forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
    return batch, kind, target, forces


def cpu_baseline(model, meta, seconds=12.0, envs=1024):
    """The reference's own CPU solver (oracle/_ref CpuBatch32) on this host's
    cores, else the CPU restatement, on a bounded sample of the workload: the
    first `envs` environments' targets, settled like the GPU arm, then timed
    for about `seconds` (median of 5 trials)."""
    cores = min(64, os.cpu_count() or 1)
    batch, kind, target, forces = cpu_settled(model, meta, envs, cores)
    t0 = time.perf_counter()
    batch.step(target, forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
    first = time.perf_counter() - t0
    steps = max(1, min(100, int(seconds / 5 / max(first, 1e-3))))
    values = []
    for _ in range(5):
        t0 = time.perf_counter()
        for _ in range(steps):
            batch.step(target, forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
        values.append(envs * SUBSTEPS * steps / (time.perf_counter() - t0))
    return {"value": statistics.median(values), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{envs} envs after {SETTLE} settle steps, median of 5 trials x {steps} control steps "
                      f"({SUBSTEPS} substeps), wall clock"}


def small_batch(model, meta, device, envs=16, steps=1000):
    """The CPU-runnable workload as written: 16 envs from HOME, HOME + N(0,
    0.1 rad) targets drawn per joint per control step, 1000 control steps of
    4 substeps.  Timed on the reference's CPU solver (one thread per env, as
    many as the host has, wall clock) and on this library (the targets
    already on the device, CUDA events around the 1000 launches): a batch
    this small leaves the GPU launch-bound, which is what the number shows."""
    import torch

    from duck_gym_b200 import CudaBatch

    rng = np.random.default_rng(0)
    home = np.asarray(meta["home"], np.float32)
    targets = (home + rng.normal(0, 0.1, (steps, envs, home.size))).astype(np.float32)
    forces = np.zeros((envs, 3), np.float32)
    q = np.tile(home, (envs, 1))
    cores = min(envs, os.cpu_count() or 1)
    cpu, kind = reference_batch(model, envs, cores)
    cpu.reset(np.ones(envs, bool), q, np.zeros((envs, 6), np.float32))
    t0 = time.perf_counter()
    for k in range(steps):
        cpu.step(targets[k], forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
    cpu_value = envs * SUBSTEPS * steps / (time.perf_counter() - t0)
    gpu = CudaBatch(model, envs, DT, ITERATIONS, device.index)
    gpu.reset(torch.ones(envs, dtype=torch.bool, device=device), torch.from_numpy(q).to(device),
              torch.zeros(envs, 6, device=device))
    dt_targets = torch.from_numpy(targets).to(device)
    df = torch.zeros(envs, 3, device=device)
    for k in range(5):
        gpu.step(dt_targets[k], df, SUBSTEPS, meta["kp"], meta["torque_limit"])
    gpu.reset(torch.ones(envs, dtype=torch.bool, device=device), torch.from_numpy(q).to(device),
              torch.zeros(envs, 6, device=device))
    stream = torch.cuda.current_stream(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    a.record(stream)
    for k in range(steps):
        gpu.step(dt_targets[k], df, SUBSTEPS, meta["kp"], meta["torque_limit"])
    b.record(stream)
    b.synchronize()
    gpu_value = envs * SUBSTEPS * steps / (a.elapsed_time(b) / 1e3)
    return {"workload": f"{envs} envs from HOME, HOME + N(0,0.1 rad) targets per joint per control step, "
                        f"{steps} control steps", "unit": UNIT,
            "cpu": {"value": cpu_value, "cores": cores, "kind": kind, "timing": "wall clock"},
            "gpu": {"value": gpu_value, "timing": "CUDA events, targets resident on the device"}}


def reference_cuda_module():
    """The reference's own CUDA extension rebuilt for sm_100a by
    oracle/build_ref_cuda.py, or None."""
    import importlib.util

    path = ROOT / "oracle" / "_ref" / "cuda" / "_duck_cuda.so"
    if not path.exists():
        return None
    import torch  # noqa: F401  (the extension links libtorch)

    spec = importlib.util.spec_from_file_location("_duck_cuda", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def reference_cuda(model, meta, envs, device, steps=40, trials=5):
    """Context number: the reference's own CUDA step (extension.cu advance,
    one 32-thread block per env) rebuilt for sm_100a and run on this GPU on
    the same workload -- settled 200 steps, then `trials` x `steps` control
    steps timed with CUDA events, L2 flushed between steps, median trial.
    Both of its compact-state variants are timed (state in global memory, and
    the whole state copied to shared memory)."""
    import torch

    ext = reference_cuda_module()
    if ext is None:
        return None
    kp, limit = meta["kp"], meta["torque_limit"]
    target = torch.from_numpy(fixed_targets(meta, envs, 0)).to(device)
    forces = torch.zeros(envs, 3, device=device)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    out = {}
    for shared in (False, True):
        sim = ext.CudaBatch(str(model), envs, DT, ITERATIONS, device.index, False, True, shared)
        for _ in range(SETTLE):
            sim.step(target, forces, SUBSTEPS, kp, limit)
        values = []
        for _ in range(trials):
            total = 0.0
            for _ in range(steps):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                sim.step(target, forces, SUBSTEPS, kp, limit)
                b.record(stream)
                b.synchronize()
                total += a.elapsed_time(b) / 1e3
            values.append(envs * SUBSTEPS * steps / total)
        failed = float((sim.state()[2][:, 5] > 0).float().mean())
        out["shared_memory" if shared else "global_memory"] = {"value": statistics.median(values),
                                                               "failed_env_fraction": failed}
        del sim
    best = max(out.values(), key=lambda v: v["value"])["value"]
    return {"value": best, "unit": UNIT, "variants": out,
            "kernel": "reference extension.cu advance<S,Shared> (specialized compact state), built for sm_100a "
                      "with the reference's flags by oracle/build_ref_cuda.py",
            "sample": f"{envs} envs after {SETTLE} settle steps, median of {trials} trials x {steps} control steps, "
                      "CUDA events, L2 flushed between steps"}


def traffic_from_profile():
    """DRAM bytes per advance launch from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "advance_biped4096.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


def reference_arm(args, rank, world):
    """--impl reference: the reference's CPU solver (oracle/_ref, else the
    oracle port) on all host cores, on the same workload, settled the same
    200 steps, then W warm-up and K timed control steps (wall clock)."""
    if rank != 0:
        return
    with tempfile.TemporaryDirectory() as d:
        model, meta = make_model(d)
        cores = min(64, os.cpu_count() or 1)
        envs = min(args.envs, 4096)
        batch, kind, target, forces = cpu_settled(model, meta, envs, cores)
        for _ in range(args.warmup):
            batch.step(target, forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
        t0 = time.perf_counter()
        for _ in range(args.steps):
            batch.step(target, forces, SUBSTEPS, meta["kp"], meta["torque_limit"])
        elapsed = time.perf_counter() - t0
        value = envs * SUBSTEPS * args.steps / elapsed
        cfg = workload(args)
        cfg.update(kp=meta["kp"], torque_limit=meta["torque_limit"], envs_per_gpu=envs)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded biped, no dataset)",
            "config": cfg,
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{envs} envs after {SETTLE} settle + {args.warmup} warm-up steps, "
                                       f"{args.steps} control steps timed"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)


COMMAND_RANGES = [[-0.3, 0.3], [-0.3, 0.3], [-1.0, 1.0]]


def run_ppo(args, rank, world, local, device):
    """Full RL rollout plus PPO update.  4096 BamEnv envs
    per GPU (the synthetic bundle, dt 5 ms, decimation 4, 10 iterations) on a
    velocity-command task, commands U[-0.3,0.3] m/s in x/y and U[-1,1] rad/s
    in yaw; actor MLP 61-512-256-128-14 ELU under bf16 autocast (the actor
    observation has 51 live entries -- angular velocity, gravity, joint
    positions and velocities, last action, command -- plus the reference's 10
    zero pads; a 48-dim layout does not add up to that list of terms); 24-step
    rollouts, 5 epochs x 4 minibatches; gradients averaged over the ranks by
    bucketed NCCL all-reduces overlapped with backward.  One step = one PPO
    iteration; value = envs x 24 x 4 physics steps per iteration x ranks /
    slowest rank's device seconds."""
    import torch
    import torch.distributed as dist

    from duck_gym_b200 import biped
    from duck_gym_b200.bam_env import BamEnv
    from duck_gym_b200.ppo import PPO, PPOConfig
    from duck_gym_b200.sharding import max_over_ranks, rank_seed

    envs = args.envs
    training = dict(command_ranges=COMMAND_RANGES, command_resample_seconds=5.0, reset_joint_noise=0.01,
                    reset_tilt_noise=0.01, horizontal_velocity_variance=0.1, vertical_velocity_variance=0.1)
    stream = torch.cuda.current_stream(device)
    with tempfile.TemporaryDirectory() as d:
        biped.write_bam(d, seed=0)
        env = BamEnv(d, num_envs=envs, iterations=10, auto_reset=True, reward_enabled=True, device=local,
                     training=training, seed=rank_seed(0, rank), seconds=20.0)
        agent = PPO(env, PPOConfig(), device=device, seed=rank_seed(1, rank))
        for _ in range(args.warmup):
            agent.rollout()
            agent.update()
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        rollout_ms, update_ms = [], []
        clocks = ClockSampler(local)
        clocks.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        t_start = time.monotonic()
        for k in range(args.steps):
            flush.zero_()
            mid = torch.cuda.Event(enable_timing=True)
            starts[k].record(stream)
            agent.rollout()
            mid.record(stream)
            stats = agent.update()
            ends[k].record(stream)
            torch.cuda.synchronize(device)
            rollout_ms.append(starts[k].elapsed_time(mid))
            update_ms.append(mid.elapsed_time(ends[k]))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        clocks.window = (t_start, time.monotonic())
        clocks.stop()
        device_s = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3
        slowest = max_over_ranks(device_s, device)
        physics = envs * agent.cfg.steps_per_env * env.decimation
        value = physics * args.steps * world / slowest
        if rank == 0:
            print(json.dumps({
                "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * slowest / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 physics, bf16 actor/critic",
                "data": "synthetic (seeded biped, no dataset)",
                "config": {"workload": "config 4: PPO rollout (24 steps) + update (5 epochs x 4 minibatches) on the "
                                       "BAM velocity-command task, actor 61-512-256-128-14 ELU bf16",
                           "envs_per_gpu": envs, "substeps_per_step": env.decimation, "iterations": 10, "dt": env.dt,
                           "rollout_ms": statistics.mean(rollout_ms), "update_ms": statistics.mean(update_ms),
                           "samples_per_iteration": envs * agent.cfg.steps_per_env * world,
                           "last_update": stats,
                           "l2": "flushed between timed iterations (256 MiB write, outside the timed events)",
                           "parallelism": f"dp{world}: env shards, NCCL gradient all-reduce"},
                "clocks": clocks.summary()}), flush=True)


def run_extended(args, rank, world, local, device):
    """The self-contact and domain-randomised workloads on the synthetic biped
    (both beyond the reference's envelope: 91 body-collision pairs; per-env
    parameters).

    config3: 16384 envs per GPU, self-contact on (all 91 non-adjacent link
      pairs), the BAM servo of the synthetic bundle (4 N m/rad, 0.1 N m s/rad,
      0.5 N m cap, load-dependent friction), dt 5 ms, decimation 4,
      10 iterations.  A step is one BamEnv.step (CUDA graph: servo, physics
      and bookkeeping per substep, reward and observations) with actions
      N(0, 0.1) fixed per env, auto-reset on.
    config5: 65536 envs per GPU, 20 iterations, per-env link masses
      x U[0.8, 1.2] (inertias alike) and ground friction U[0.4, 1.2]; each
      step 2 % of the envs reset with joint offsets N(0, 0.02 rad) and 2 %
      receive a base push N(0, 0.5 m/s) (a base force m dv / t held over the
      step); PD targets swing the legs through a crouch-and-extend cycle
      (jump-like), dt 5 ms, 4 substeps.
    value = envs x physics substeps x K / device seconds, max over ranks."""
    import torch

    from duck_gym_b200 import CudaBatch, biped
    from duck_gym_b200.sharding import max_over_ranks, rank_seed, weak_shard

    if args.workload == "config4":
        return run_ppo(args, rank, world, local, device)
    per_gpu = args.envs if args.envs != ENVS else (16384 if args.workload == "config3" else 65536)
    envs = weak_shard(per_gpu, rank, world).count   # weak scaling: envs per GPU fixed
    gen = torch.Generator(device=device).manual_seed(rank_seed(0, rank))
    stream = torch.cuda.current_stream(device)
    with tempfile.TemporaryDirectory() as d:
        if args.workload == "config3":
            from duck_gym_b200.bam_env import BamEnv

            biped.write_bam(d, seed=0, self_contacts=True)
            env = BamEnv(d, num_envs=envs, iterations=10, auto_reset=True, reward_enabled=True, device=local,
                         max_pairs=128, seconds=20.0)
            actions = 0.1 * torch.randn(envs, 14, generator=gen, device=device)
            substeps = env.decimation

            def one_step():
                env.step(actions)

            launches = lambda: env.native.launches
            cfg = {"workload": "config 3: synthetic biped (seed 0), 91 self-contact pairs, BAM servo (4 N m/rad, "
                               "0.1 N m s/rad, 0.5 N m), BamEnv step with auto-reset, actions N(0,0.1) fixed",
                   "envs_per_gpu": envs, "substeps_per_step": substeps, "iterations": 10, "dt": env.dt}
        else:
            path = biped.write(d, seed=0)
            meta = json.loads((Path(d) / "metadata.json").read_text())
            text = Path(path).read_text()
            batch = CudaBatch(str(path), envs, DT, 20, local)
            lines = text.splitlines()
            nb, nj, ns = (int(v) for v in lines[0].split()[2:5])
            mass0 = torch.tensor([float(lines[2 + b].split()[1]) for b in range(nb)], device=device)
            inertia0 = torch.tensor([[float(v) for v in lines[2 + b].split()[2:5]] for b in range(nb)], device=device)
            scale = 0.8 + 0.4 * torch.rand(envs, nb, generator=gen, device=device)
            friction = (0.4 + 0.8 * torch.rand(envs, 1, generator=gen, device=device)).expand(envs, ns).contiguous()
            mass = (mass0 * scale).contiguous()
            batch.set_parameters(mass, (inertia0 * scale[..., None]).contiguous(), friction)
            home = torch.tensor(meta["home"], device=device)
            legs = torch.zeros(14, device=device)
            for name, a in (("hip_pitch", -0.4), ("knee", 0.8), ("ankle", -0.4)):
                for j, n in enumerate(meta["joint_names"]):
                    if name in n:
                        legs[j] = a
            phase = 2 * math.pi * torch.rand(envs, 1, generator=gen, device=device)
            kp, limit = meta["kp"], meta["torque_limit"]
            forces = torch.zeros(envs, 3, device=device)
            substeps = SUBSTEPS
            counter = [0]

            def one_step():
                k = counter[0]
                counter[0] += 1
                cycle = 0.5 - 0.5 * torch.cos(phase + 2 * math.pi * k * SUBSTEPS * DT / 0.6)
                target = (home + legs * cycle).contiguous()
                reset = torch.rand(envs, generator=gen, device=device) < 0.02
                q = (home + 0.02 * torch.randn(envs, 14, generator=gen, device=device)).contiguous()
                batch.reset(reset, q, torch.zeros(envs, 6, device=device))
                push = torch.rand(envs, 1, generator=gen, device=device) < 0.02
                dv = 0.5 * torch.randn(envs, 3, generator=gen, device=device)
                torch.where(push, dv * mass[:, 1:2] / (SUBSTEPS * DT), torch.zeros_like(dv), out=forces)
                batch.step(target, forces, SUBSTEPS, kp, limit)

            launches = lambda: batch.launches
            cfg = {"workload": "config 5: synthetic biped (seed 0), per-env masses x U[0.8,1.2] and ground friction "
                               "U[0.4,1.2], 2% resets/step with joint offsets N(0,0.02), 2% base pushes N(0,0.5 m/s), "
                               "crouch-and-extend PD targets",
                   "envs_per_gpu": envs, "substeps_per_step": SUBSTEPS, "iterations": 20, "dt": DT}
        for _ in range(SETTLE // 4 + args.warmup):
            one_step()
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        clocks = ClockSampler(local)
        clocks.start()
        l0 = launches()
        torch.cuda.synchronize(device)
        t_start = time.monotonic()
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            one_step()
            ends[k].record(stream)
        torch.cuda.synchronize(device)
        clocks.window = (t_start, time.monotonic())
        clocks.stop()
        device_s = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3
        slowest = max_over_ranks(device_s, device)
        value = envs * substeps * args.steps * world / slowest
        if rank == 0:
            cfg.update({"l2": "flushed between timed steps (256 MiB write, outside the timed events)",
                        "parallelism": f"env shards x{world}, no physics communication"})
            print(json.dumps({
                "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * slowest / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded biped, no dataset)",
                "config": cfg, "gpu_launches": launches() - l0, "clocks": clocks.summary()}), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--envs", type=int, default=ENVS)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=["config2", "config3", "config4", "config5"], default="config2")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    from duck_gym_b200 import CudaBatch, fp32_peak_tflops
    from duck_gym_b200.sharding import max_over_ranks, rank_seed, weak_shard

    if args.workload != "config2":
        run_extended(args, rank, world, local, device)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    with tempfile.TemporaryDirectory() as d:
        model, meta = make_model(d)
        kp, limit = meta["kp"], meta["torque_limit"]
        envs = weak_shard(args.envs, rank, world).count   # weak scaling: envs per GPU fixed
        batch = CudaBatch(model, envs, DT, ITERATIONS, local)
        target_host = fixed_targets(meta, envs, rank_seed(0, rank))
        target = torch.from_numpy(target_host).to(device)
        forces = torch.zeros(envs, 3, device=device)
        for _ in range(SETTLE):
            batch.step(target, forces, SUBSTEPS, kp, limit)
        for _ in range(args.warmup):
            batch.step(target, forces, SUBSTEPS, kp, limit)
        # The states the timed region starts from, for the flop count.
        start_records = batch.export_records().cpu().numpy() if rank == 0 else None
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)  # 256 MiB > L2
        stream = torch.cuda.current_stream(device)

        def barrier():
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(device)

        def timed(steps):
            """Per-step device times (ms) of `steps` steps, L2 flushed between
            steps outside the events, on the launching stream."""
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            for k in range(steps):
                flush.zero_()
                starts[k].record(stream)
                batch.step(target, forces, SUBSTEPS, kp, limit)
                ends[k].record(stream)
            return starts, ends

        clocks = ClockSampler(local)
        clocks.start()
        launches0 = batch.launches
        barrier()
        wall0 = time.perf_counter()
        t_start = time.monotonic()
        starts, ends = timed(args.steps)
        barrier()
        t_end = time.monotonic()
        wall = time.perf_counter() - wall0
        launches = batch.launches - launches0
        kernel_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        device_s = sum(kernel_ms) / 1e3
        slowest = max_over_ranks(device_s, device)
        total_steps = envs * SUBSTEPS * args.steps * world
        value = total_steps / slowest

        # The reference's own method beside it (benchmark_engines.py:510-551):
        # 5 trials of TRIAL_STEPS steps, median, max over ranks per trial.
        trial_values = []
        for _ in range(TRIALS):
            barrier()
            ts, te = timed(TRIAL_STEPS)
            barrier()
            trial_s = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(ts, te)) / 1e3, device)
            trial_values.append(envs * SUBSTEPS * TRIAL_STEPS * world / trial_s)

        # End to end through the public API, every step: the step's targets
        # and forces copied in from pinned host memory, one step, the full
        # state() snapshot (bodies, joints, diagnostics) copied back to pinned
        # host memory.  The copies run on two side streams (inputs, outputs)
        # ordered by stream waits, so step k + 1 computes while step k's state
        # goes back to the host (state() returns fresh tensors, which step
        # k + 1 does not touch); the host buffers are double-buffered.
        host_in = torch.from_numpy(target_host).pin_memory()
        host_forces = torch.zeros(envs, 3).pin_memory()
        nb, nj = batch.num_bodies, batch.num_joints
        host_out = [(torch.empty(envs, nb, 13).pin_memory(), torch.empty(envs, nj, 2).pin_memory(),
                     torch.empty(envs, 6).pin_memory()) for _ in range(2)]
        inputs, outputs = torch.cuda.Stream(device), torch.cuda.Stream(device)
        e2e_steps = max(10, args.steps)
        # The clock record covers the timed steps and the trials; the sampler
        # stops before the end-to-end pass, whose host thread issues every
        # copy and launch itself.
        clocks.window = (t_start, time.monotonic())
        clocks.stop()

        def e2e_window():
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            inputs.wait_stream(stream)
            outputs.wait_stream(stream)
            for k in range(e2e_steps):
                with torch.cuda.stream(inputs):
                    tin = host_in.to(device, non_blocking=True)
                    fin = host_forces.to(device, non_blocking=True)
                stream.wait_stream(inputs)
                tin.record_stream(stream)
                fin.record_stream(stream)
                batch.step(tin, fin, SUBSTEPS, kp, limit)
                state = batch.state()
                outputs.wait_stream(stream)
                with torch.cuda.stream(outputs):
                    for host, dev in zip(host_out[k % 2], state):
                        host.copy_(dev, non_blocking=True)
                        dev.record_stream(outputs)
            stream.wait_stream(outputs)
            e1.record(stream)
            barrier()
            return envs * SUBSTEPS * e2e_steps * world / max_over_ranks(e0.elapsed_time(e1) / 1e3, device)

        # One untimed window first (the caching allocator grows its pools for
        # the per-step input and state tensors held by the side streams), then
        # three timed windows, median: one window is short enough for a stall
        # of the shared host to dominate it.
        e2e_window()
        e2e_values = [e2e_window() for _ in range(3)]
        host_diag = host_out[(e2e_steps - 1) % 2][2]
        e2e_value = statistics.median(e2e_values)
        failed_fraction = float((host_diag[:, 5] > 0).float().mean())

        line = None
        if rank == 0:
            peak = fp32_peak_tflops(local)
            flops = count_flops(model, meta, target_host, start_records, min(args.steps, FLOP_STEPS))
            mean_kernel_s = statistics.mean(kernel_ms) / 1e3
            achieved = flops["flops_per_env_step"] * envs * SUBSTEPS / mean_kernel_s / 1e12
            state_bytes = batch.record_length * 4  # record read + written per launch (upper bound)
            hbm_algorithmic = envs * (2 * state_bytes) + envs * (14 + 3) * 4
            peaks = {}
            peaks_path = ROOT / "MEASURED_PEAKS.json"
            if peaks_path.exists():
                peaks = json.loads(peaks_path.read_text())
            hbm_peak = peaks.get("hbm_gbs", 6650.0)
            traffic = traffic_from_profile()
            cfg = workload(args)
            cfg.update(kp=kp, torque_limit=limit)
            line = {
                "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * slowest / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded biped, no dataset)",
                "config": cfg,
                "roofline": {
                    "bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic,
                    "kernel": "advanceKernel<float,8,false>",
                    "peak_source": "measured: FP32 FMA probe on this GPU (duck_fp32_peak), 2 flops per FMA",
                    "flops_per_env_step": flops["flops_per_env_step"],
                    "flops_source": "oracle counting scalar (+,-,*,/,sqrt), " + flops["sample"],
                    "transcendentals_per_env_step": flops["transcendentals_per_env_step"],
                    "gs_iterations_per_env_step": flops["gs_iterations_per_env_step"],
                    "hbm": {"algorithmic_bytes_per_launch": hbm_algorithmic,
                            "achieved_gbs": hbm_algorithmic / mean_kernel_s / 1e9, "peak_gbs": hbm_peak,
                            "frac": hbm_algorithmic / mean_kernel_s / 1e9 / hbm_peak,
                            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650 GB/s"},
                },
                "trials": {"count": TRIALS, "steps_each": TRIAL_STEPS, "median": statistics.median(trial_values),
                           "values": trial_values, "method": "per-step CUDA events summed per trial, L2 flushed "
                                                             "between steps, max over ranks"},
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": envs * (nj + 3) * 4,
                        "d2h_bytes_per_step": envs * (nb * 13 + nj * 2 + 6) * 4, "steps": e2e_steps,
                        "windows": e2e_values, "statistic": "median of 3 windows",
                        "path": "CudaBatch.step + CudaBatch.state(): pinned host targets/forces in, bodies, joints "
                                "and diag out, every step; copies on side streams overlap the next step"},
                "gpu_launches": launches,
                "clocks": clocks.summary((t_start, t_end)),
                "clocks_all_regions": clocks.summary(),
                "wall_s": wall,
                "failed_env_fraction": failed_fraction,
            }
            if not args.no_cpu_baseline and world == 1:
                line["cpu_baseline"] = cpu_baseline(model, meta)
                line["small_batch"] = small_batch(model, meta, device)
                ref_gpu = reference_cuda(model, meta, envs, device)
                if ref_gpu is not None:
                    ref_gpu["ours_over_reference"] = value / ref_gpu["value"]
                    line["reference_cuda"] = ref_gpu
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if line is not None:
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
