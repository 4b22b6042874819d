#!/usr/bin/env python3
"""Throughput benchmark: SO3LR force evaluation + NVE step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3|2|1]

One "step" is one MD step of BASELINE.json config 3 by default: a seeded
8,000-molecule (24,000-atom) periodic water box at 0.997 g/cm^3, 300 K
Maxwell-Boltzmann velocities, velocity-Verlet NVE with dt = 0.5 fs, float64.
Each step builds the neighbour lists, evaluates energy, forces and virial
through the CUDA library, and integrates.

Printed JSON line (rank 0):
  value   atom-steps/s of the whole job, positions and velocities resident in HBM
  e2e     the same metric through the C ABI with host buffers: every step copies
          the positions host->device (pinned) and the forces + energy/virial back
  roofline  the pair-filter MLP kernels (the dominant FP64 tensor-core work),
          timed with CUDA events on the library's stream during the timed region,
          against the FP64 DGEMM throughput measured on this GPU before timing
  step_roofline  the whole step's FP64 work (the reference algorithm's FLOP
          count and the FLOP this build executes) against the FP64 peak
  cpu_baseline  the float64 CPU restatement (oracle/) on a bounded sample
  identity  one single-point evaluation of the config-4 box (64,000 H2O,
          192,000 atoms, seed 2026) at every GPU count, outside the timed
          regions: energy and virial as exact hex floats and a SHA-256 of the
          forces, so that runs at 1, 2, 4 and 8 GPUs compare bit for bit
  stats.exchange_ms_per_step  (N > 1) device time per step of each exchange
          phase (position all-gather, halo-list rebuild, feature and adjoint
          halo exchanges, charge/ratio all-gathers, exact-sum all-gathers),
          max over ranks
For N > 1 (torchrun) the box grows with N (N x 8,000 molecules, weak scaling:
24,000 atoms per GPU, 192,000 atoms at N = 8 as in config 4) and is split into
N spatial bricks; each rank owns the atoms of its brick, evaluates their pairs,
and the library exchanges rows with NCCL (all-gathers of positions, charges and
ratios; send/receive of the halo rows of block features and adjoints). The N > 1 runs
are NVT with a Nose-Hoover chain at 300 K (config 4). Times are the max over
ranks.

--impl reference times the reference algorithm's CPU restatement on all host
threads, each step one energy+force evaluation of the same 24,000-atom box the
GPU arm integrates (the reference's own CPU paths cannot be built here: its
kernels require the Kokkos CUDA backend and cuBLAS).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

A100_24K_ATOM_STEPS = 69706.0  # reference, examples/scaling/README.md:60 (1x A100-40GB, 24,000 atoms)
DT_PS = 0.0005

CONFIGS = {
    1: (64, "config1: 64 H2O (192 atoms), periodic cubic box, float64"),
    2: (1000, "config2: NVE MD of 1,000 H2O (3,000 atoms), periodic cubic box, 0.5 fs, float64"),
    3: (8000, "config3: NVE MD of 8,000 H2O (24,000 atoms), periodic cubic box, 0.5 fs, float64"),
}


def workload(config: int, world: int):
    """Molecule count and the `config` record of the timed workload, shared by
    both arms so that their lines describe the same configuration."""
    nmol, desc = CONFIGS[config]
    if world > 1:
        nmol *= world
        desc = (f"config4 (weak-scaled): NVT MD of {nmol:,} H2O ({3 * nmol:,} atoms) on {world} GPUs, "
                f"Nose-Hoover chain (3 thermostats, 300 K, 0.05 ps), spatial bricks, periodic cubic box, "
                f"0.5 fs, float64")
    from so3lr_b200.systems import box_length
    cfg = {"workload": desc, "atoms": 3 * nmol, "atoms_per_gpu": 3 * nmol / world,
           "box_A": float(box_length(nmol, 0.997)),
           "seed": 2026, "timestep_fs": 0.5,
           "parallelism": "single" if world == 1 else
           f"spatial{world} (brick decomposition, NCCL all-gather of owned rows, max over ranks)",
           "l2": "no flush: per-step working set (pair filters, HBM-resident activations) exceeds L2"}
    return nmol, cfg


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None
        self.skip = 0

    def start(self):
        """Start sampling and return once nvidia-smi has written its first row
        (at most 3 s), so that the rows kept by stop() (those after it) all
        fall inside the region timed between start() and stop()."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.skip = 0
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 3.0 and self.proc.poll() is None:
            with open(self.path) as fh:
                lines = fh.read().splitlines()
            if lines:
                self.skip = len(lines)
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        with open(self.path) as fh:
            text = "\n".join(fh.read().splitlines()[self.skip:])
        os.unlink(self.path)
        return summarize_clocks(text)


def summarize_clocks(text: str) -> dict:
    """Median SM clock, maximum SM clock and the throttle reasons seen Active in
    nvidia-smi CSV rows of ClockSampler.FIELDS (noheader, nounits)."""
    rows = []
    for line in text.splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) >= 9:
            rows.append(parts)
    if not rows:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
    sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
    smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower().startswith("active")})
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
            "reasons": reasons, "samples": len(rows)}


def measure_fp64_peak(device: int) -> float:
    """Dense FP64 throughput of cuBLAS DGEMM (torch.matmul float64), TFLOP/s, best of 5."""
    import torch
    n = 8192
    a = torch.randn(n, n, dtype=torch.float64, device=f"cuda:{device}")
    b = torch.randn(n, n, dtype=torch.float64, device=f"cuda:{device}")
    torch.matmul(a, b)
    torch.cuda.synchronize()
    best = 0.0
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        best = max(best, 2.0 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
    del a, b
    torch.cuda.empty_cache()
    return best


def measure_tf32_peak(device: int) -> float:
    """Dense TF32 tensor-core throughput of cuBLAS (torch.matmul float32 with
    TF32 allowed, 8192^3), TFLOP/s, best of 5."""
    import torch
    n = 8192
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn(n, n, dtype=torch.float32, device=f"cuda:{device}")
        b = torch.randn(n, n, dtype=torch.float32, device=f"cuda:{device}")
        torch.matmul(a, b)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            torch.cuda.synchronize()
            best = max(best, 2.0 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
        del a, b
        torch.cuda.empty_cache()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return best


def library_record() -> dict:
    """Which build of libso3lr_b200.so this run loaded: SHA-256 (first 16 hex
    digits) and modification time of the in-tree library, and whether it is
    newer than every source file (built from the sources in this tree)."""
    import hashlib
    from so3lr_b200.build import LIB, headers, sources
    data = LIB.read_bytes()
    newest = max(p.stat().st_mtime for p in [src for src, _ in sources()] + list(headers()))
    return {"path": "so3lr_b200/libso3lr_b200.so", "sha256_16": hashlib.sha256(data).hexdigest()[:16],
            "mtime": LIB.stat().st_mtime, "newer_than_sources": LIB.stat().st_mtime >= newest}


def cpu_model() -> str:
    """The host CPU's model name (lscpu / /proc/cpuinfo), for the baseline record."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_checkpointing(natoms: int) -> bool:
    """Whether the oracle keeps only block inputs for its reverse: about
    2.6 MB per atom held otherwise, 1.4 MB per atom with it (measured on the
    3,000-atom box); chosen when the host's available memory is short."""
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        return True
    return natoms * 2.6e6 * 1.5 > avail


def cpu_baseline(seconds: float = 12.0) -> dict:
    """Oracle (float64 CPU restatement of the reference kernels) on a bounded sample."""
    import torch
    from oracle.so3lr_oracle import OracleModel, System, evaluate
    from so3lr_b200.systems import water_box
    om = OracleModel.load(str(ROOT / "models" / "so3lr.so3lr"))
    w = water_box(216, seed=7)
    s = System(pos=w.pos, z=w.z, cell=w.cell)
    evaluate(om, s)  # warm-up
    t0 = time.perf_counter()
    count = 0
    while True:
        evaluate(om, s)
        count += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": len(w.z) * count / dt, "unit": "atom-steps/s", "cores": torch.get_num_threads(),
            "kind": "port", "cpu": cpu_model(),
            "sample": f"{count} energy+force evaluations of a 648-atom periodic water box (216 H2O) "
                      f"by the float64 CPU restatement in oracle/ (torch CPU, {torch.get_num_threads()} threads)"}


def run_reference(args) -> None:
    """The reference algorithm's float64 CPU restatement (oracle/, torch CPU, all
    host threads) on the workload of our arm. At N = 1 every step is one
    energy+force evaluation of the same 24,000-atom box (same seed) that the GPU
    arm integrates; under torchrun rank 0 alone runs, and each step evaluates
    that 24,000-atom box, which is one GPU's share of the weak-scaled workload
    (the whole 192,000-atom box would take minutes per step on the CPU)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch
    from oracle.so3lr_oracle import OracleModel, System, build_graphs, evaluate
    from so3lr_b200.systems import water_box
    threads = host_threads()
    torch.set_num_threads(threads)
    om = OracleModel.load(str(ROOT / "models" / "so3lr.so3lr"))
    if args.config == 5:
        from so3lr_b200.systems import turbo_batch
        pos, z, off, q, mult = turbo_batch(32, seed=7)
        image = np.repeat(np.arange(len(off) - 1), np.diff(off))
        s = System(pos=pos, z=z, image=image, image_charge=q, image_multiplicity=mult)
        n_sample, what = len(z), "a 32-cluster pack (a bounded sample)"
        n_atoms = int(len(turbo_batch(TURBO_CLUSTERS, seed=7)[1]))
        cfg = {"workload": f"config5: NVE MD of a turbo pack of {TURBO_CLUSTERS} water clusters ({n_atoms} atoms)"}
    else:
        nmol, cfg = workload(args.config, world)
        w = water_box(CONFIGS[args.config][0], seed=2026)
        s = System(pos=w.pos, z=w.z, cell=w.cell)
        n_sample = len(w.z)
        what = (f"the same {n_sample}-atom box the GPU arm integrates (seed 2026)" if world == 1 else
                f"the {n_sample}-atom box of one GPU's share of the {3 * nmol}-atom workload (a bounded sample)")
    ckpt = oracle_checkpointing(n_sample)
    graphs = build_graphs(om, s)  # the reference rebuilds its lists only on reneighbouring steps
    for _ in range(args.warmup):
        evaluate(om, s, graphs=graphs, checkpoint_blocks=ckpt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        evaluate(om, s, graphs=graphs, checkpoint_blocks=ckpt)
    dt = time.perf_counter() - t0
    value = n_sample * args.steps / dt
    sample = (f"each step = one energy+force evaluation of {what} by the float64 CPU restatement of the "
              f"reference kernels (oracle/, torch CPU, {threads} threads"
              f"{', block intermediates recomputed in the reverse' if ckpt else ''}); the reference's "
              f"Kokkos/cuBLAS code has no CPU build")
    line = {
        "impl": "reference", "metric": "atom-steps/s", "value": value, "unit": "atom-steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "atom-steps/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model(), "sample": sample, "sample_atoms": n_sample},
        "e2e": {"value": value, "unit": "atom-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import maxwell_boltzmann, water_box

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    nmol, cfg = workload(args.config, world)
    mixed = args.precision == "mixed"
    if mixed:
        cfg["workload"] += " (mixed float32: pair-filter GEMMs as three-pass TF32 with float32 accumulation)"
    w = water_box(nmol, seed=2026)
    n = len(w.z)
    v0 = maxwell_boltzmann(w.mass, 300.0, seed=11)
    peak = measure_tf32_peak(local) / 3.0 if mixed else measure_fp64_peak(local)

    model = So3lrB200(args.model, local)
    if pathlib.Path(args.model).resolve() != (ROOT / "models" / "so3lr.so3lr").resolve():
        info = model.describe()
        cfg["workload"] += f" with the model file {pathlib.Path(args.model).name} ({info['summary']})"
    if mixed:
        model.set_precision("mixed")
    if world > 1:
        uid = [So3lrB200.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.comm_init(world, rank, uid[0])
    ext = torch.cuda.ExternalStream(model.stream, device=f"cuda:{local}")

    # ---- device-resident MD (value) -----------------------------------------
    model.md_init(w.pos, w.z, w.cell, w.boxlo, v0, w.mass)
    if world > 1:
        model.md_thermostat(300.0, 0.05, 3)  # BASELINE config 4 is NVT
    model.md_run(args.warmup, DT_PS)
    stats = model.stats()
    model.profile(True)
    for k in range(len(PROFILE_KINDS)):
        model.profile_read(k)
    launches0 = model.launch_count()
    clocks = ClockSampler(local)
    clocks.start()  # before the barrier: its wait for nvidia-smi must not skew the ranks' start
    barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(ext)
    model.md_run(args.steps, DT_PS)
    t_end.record(ext)
    torch.cuda.synchronize()
    ms = t_start.elapsed_time(t_end)
    clock_info = clocks.stop()
    launches = model.launch_count() - launches0
    prof_all = [model.profile_read(k) for k in range(len(PROFILE_KINDS))]
    prof = prof_all[:2]
    model.profile(False)
    # per-step device time of each exchange phase, max over ranks (N > 1)
    exchange = None
    if world > 1:
        exchange = {name: max_over_ranks(prof_all[k]["ms"]) / args.steps
                    for k, name in enumerate(PROFILE_KINDS) if k >= 2}
    state = model.md_state(n)
    owned = model.owned_atoms()
    ms_max = max_over_ranks(ms)
    value = n * args.steps / (ms_max * 1e-3)

    # ---- end to end through the C ABI with host buffers (e2e) ---------------
    # one GPU: so3lr_compute with the whole system; several: every rank holds
    # only the atoms of its brick on the host (as a LAMMPS rank does) and calls
    # so3lr_compute_local, the GPUs exchanging the ranks' atoms themselves
    from so3lr_b200.runtime import partition
    mine = np.arange(n) if world == 1 else np.nonzero(partition(state["x"], w.boxlo, w.cell, world) == rank)[0]
    nl = len(mine)
    x_host = torch.empty((nl, 3), dtype=torch.float64, pin_memory=True).numpy()
    v_host = torch.empty((nl, 3), dtype=torch.float64, pin_memory=True).numpy()
    f = torch.empty((nl, 3), dtype=torch.float64, pin_memory=True).numpy()
    x_host[:] = state["x"][mine]
    v_host[:] = state["v"][mine]
    z32 = np.ascontiguousarray(w.z[mine], dtype=np.int32)
    tags = mine + 1

    def evaluate_host():
        if world == 1:
            model.compute(x_host, z32, cell=w.cell, boxlo=w.boxlo, terms=False, forces_out=f)
        else:
            model.compute_local(n, tags, x_host, z32, cell=w.cell, boxlo=w.boxlo, eatom=False, forces_out=f)

    evaluate_host()
    ftm2v = 1.0 / 1.0364269e-4
    dtf = 0.5 * DT_PS * ftm2v
    # velocity-Verlet half kicks and drift in place (no temporaries per step)
    kick = np.ascontiguousarray(np.broadcast_to((dtf / w.mass[mine])[:, None], (nl, 3)))
    tmp = np.empty((nl, 3))
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        np.multiply(f, kick, out=tmp)
        v_host += tmp
        np.multiply(v_host, DT_PS, out=tmp)
        x_host += tmp
        evaluate_host()
        np.multiply(f, kick, out=tmp)
        v_host += tmp
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = n * args.steps / e2e_s

    # ---- roofline of the dominant kernel -----------------------------------
    dom = max(prof, key=lambda p: p["ms"])
    dom_name = "filter_forward" if dom is prof[0] else "filter_reverse"
    achieved = dom["flops"] / (dom["ms"] * 1e-3) / 1e12 if dom["ms"] > 0 else 0.0
    traffic = None
    tfile = ROOT / "profiles" / "filter_traffic.json"
    if tfile.exists():
        try:
            t = json.loads(tfile.read_text())
            per_pair = t.get(dom_name, {}).get("dram_bytes_per_pair")
            if per_pair:
                traffic = per_pair * stats["sr_pairs"]
        except (ValueError, KeyError):
            traffic = None

    # ---- one fixed system at every GPU count (bit-identity across N) ----------
    identity = None if args.no_identity else identity_check(model)

    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu) else None
    if rank == 0:
        steps_per_s = args.steps / (ms_max * 1e-3)
        lr_pairs = count_lr_pairs(w.pos, w.boxlo, w.cell, 12.0)  # host only, after every timed region
        line = {
            "metric": "atom-steps/s", "value": value, "unit": "atom-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / A100_24K_ATOM_STEPS) if (world == 1 and args.config == 3) else None,
            "dtype": "tf32x3+f64" if mixed else "f64", "data": "synthetic",
            "config": cfg,
            "library": library_record(),
            "stats": {"atoms_owned_rank0": owned, "sr_edges_rank0": stats["sr_edges"],
                      "sr_pairs_rank0": stats["sr_pairs"], "ns_per_day": steps_per_s * 0.0432,
                      "exchange_ms_per_step": exchange},
            "identity": identity,
            # one GPU: positions in, forces + energy/virial out; several: each
            # rank's (tag, x, y, z, Z) records in, its forces + energy/virial out
            "e2e": {"value": e2e_value, "unit": "atom-steps/s",
                    "h2d_bytes_per_step": 3 * 8 * n if world == 1 else 5 * 8 * n,
                    "d2h_bytes_per_step": 3 * 8 * n + world * 7 * 8,
                    "call": "so3lr_compute" if world == 1 else "so3lr_compute_local (each rank its brick's atoms)"},
            "roofline": {"bound": "tensor", "kernel": dom_name, "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak if peak else None, "traffic": traffic,
                         "peak_source": ("a third of the cuBLAS TF32 GEMM throughput (torch.matmul float32 "
                                         "8192^3, TF32 allowed) measured on this GPU before the timed region: "
                                         "three TF32 passes per product" if mixed else
                                         "FP64 cuBLAS DGEMM 8192^3 (torch.matmul float64) measured on this GPU "
                                         "before the timed region; MEASURED_PEAKS.json has no FP64 entry"),
                         "launches": dom["launches"], "ms_per_launch": dom["ms"] / max(1, dom["launches"]),
                         "other": {("filter_reverse" if dom is prof[0] else "filter_forward"):
                                   {"ms": (prof[1] if dom is prof[0] else prof[0])["ms"],
                                    "achieved_tflops": ((prof[1] if dom is prof[0] else prof[0])["flops"]
                                                        / max(1e-12, (prof[1] if dom is prof[0] else prof[0])["ms"] * 1e-3)
                                                        / 1e12)},
                                   "filter_share_of_step": (prof[0]["ms"] + prof[1]["ms"]) / ms}},
            # edge and pair counts are this rank's (its own rows and their halo
            # pairs); the work of the other ranks' equal bricks is taken as the same
            "step_roofline": None if mixed else step_roofline(n / world, stats["sr_edges"], stats["sr_pairs"],
                                                              lr_pairs / world, steps_per_s, peak, world),
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "gpu_launches": launches,
            "energy_final": state["energy"],
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


TURBO_CLUSTERS = 4096

# so3lr_profile_read kinds: the pair-filter kernels and the multi-GPU exchange phases
PROFILE_KINDS = ("filter_forward", "filter_reverse", "position_allgather", "halo_list_rebuild",
                 "feature_halo_exchange", "adjoint_halo_exchange", "charge_ratio_allgather", "exact_sum_allgather")


def run_turbo(args) -> None:
    """Config 5: a pack of 4,096 water clusters (4-16 H2O; half neutral, a
    quarter OH-, a quarter H3O+), open boundaries, NVE velocity Verlet at 0.5 fs
    through so3lr_compute_batch with host buffers (the turbo path has no
    device-resident loop, so value and e2e are the same measurement). Under
    torchrun the clusters are dealt to the ranks largest first, round robin;
    the ranks never communicate (the reference gathers every image to one
    coordinator rank instead, mpi_turbo_replica_broker.cpp:130-307)."""
    import torch
    import torch.distributed as dist
    from so3lr_b200 import So3lrB200
    from so3lr_b200.systems import MASS, maxwell_boltzmann, turbo_batch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        tt = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    pos, z, off, q, mult = turbo_batch(TURBO_CLUSTERS, seed=7)
    sizes = np.diff(off)
    mine = deal_clusters(sizes, rank, world)
    x = np.concatenate([pos[off[k]:off[k + 1]] for k in mine])
    zz = np.ascontiguousarray(np.concatenate([z[off[k]:off[k + 1]] for k in mine]), dtype=np.int32)
    my_off = np.concatenate([[0], np.cumsum(sizes[mine])]).astype(np.int64)
    my_q, my_m = q[mine], mult[mine]
    n, n_total = len(zz), int(len(z))
    mass = np.array([MASS[int(v)] for v in zz])
    peak = measure_fp64_peak(local)
    model = So3lrB200(ROOT / "models" / "so3lr.so3lr", local)
    x_host = torch.empty((n, 3), dtype=torch.float64, pin_memory=True).numpy()
    v_host = torch.empty((n, 3), dtype=torch.float64, pin_memory=True).numpy()
    x_host[:] = x
    v_host[:] = maxwell_boltzmann(mass, 300.0, seed=11 + rank)
    kick = np.ascontiguousarray(np.broadcast_to((0.5 * DT_PS / 1.0364269e-4 / mass)[:, None], (n, 3)))
    tmp = np.empty((n, 3))

    def step(f):
        np.multiply(f, kick, out=tmp)
        np.add(v_host, tmp, out=v_host)
        np.multiply(v_host, DT_PS, out=tmp)
        np.add(x_host, tmp, out=x_host)
        f = model.compute_batch(x_host, zz, my_off, my_q, my_m)["forces"]
        np.multiply(f, kick, out=tmp)
        np.add(v_host, tmp, out=v_host)
        return f

    f = model.compute_batch(x_host, zz, my_off, my_q, my_m)["forces"]
    for _ in range(args.warmup):
        f = step(f)
    stats = model.stats()
    model.profile(True)
    for k in (0, 1):
        model.profile_read(k)
    launches0 = model.launch_count()
    clocks = ClockSampler(local)
    clocks.start()  # before the barrier: its wait for nvidia-smi must not skew the ranks' start
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        f = step(f)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    clock_info = clocks.stop()
    launches = model.launch_count() - launches0
    prof = [model.profile_read(k) for k in (0, 1)]
    model.profile(False)
    t_max = max_over_ranks(elapsed)
    value = n_total * args.steps / t_max
    if rank == 0:
        dom = max(prof, key=lambda p_: p_["ms"])
        achieved = dom["flops"] / (dom["ms"] * 1e-3) / 1e12 if dom["ms"] > 0 else 0.0
        line = {
            "metric": "atom-steps/s", "value": value, "unit": "atom-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": f"config5: NVE MD of a turbo pack of {TURBO_CLUSTERS} water clusters "
                                   f"({n_total} atoms; 4-16 H2O, 50% neutral, 25% OH-, 25% H3O+), open boundaries, "
                                   f"0.5 fs, float64, through so3lr_compute_batch with host buffers",
                       "atoms": n_total, "atoms_rank0": n, "images_rank0": int(len(mine)),
                       "sr_edges_rank0": stats["sr_edges"], "sr_pairs_rank0": stats["sr_pairs"],
                       "parallelism": "single" if world == 1 else
                       f"{world} independent GPUs, clusters dealt largest first, no communication",
                       "l2": "no flush: per-step working set exceeds L2"},
            "e2e": {"value": value, "unit": "atom-steps/s", "h2d_bytes_per_step": (3 * 8 + 4) * n_total,
                    "d2h_bytes_per_step": (3 + 1 + 1) * 8 * n_total + 8 * TURBO_CLUSTERS},
            "roofline": {"bound": "tensor", "kernel": "filter_forward" if dom is prof[0] else "filter_reverse",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if peak else None, "traffic": None,
                         "peak_source": "FP64 cuBLAS DGEMM 8192^3 measured on this GPU before the timed region"},
            "cpu_baseline": None,
            "clocks": clock_info,
            "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


IDENTITY_MOLECULES = 64000


def identity_check(model) -> dict:
    """One single-point evaluation of the config-4 box (64,000 H2O, 192,000
    atoms, seed 2026) through so3lr_compute, outside every timed region, at
    whatever GPU count this run has (collective when decomposed). The energy
    and virial as exact hexadecimal floats and a SHA-256 of the force array
    (float64, little-endian, input atom order) let runs at 1, 2, 4 and 8 GPUs
    be compared bit for bit."""
    import hashlib
    from so3lr_b200.systems import water_box
    w = water_box(IDENTITY_MOLECULES, seed=2026)
    r = model.compute(w.pos, w.z, cell=w.cell, boxlo=w.boxlo, terms=False)
    f = np.ascontiguousarray(r["forces"], dtype="<f8")
    return {"system": f"config4 box: {IDENTITY_MOLECULES:,} H2O ({3 * IDENTITY_MOLECULES:,} atoms), seed 2026, "
                      f"single point through so3lr_compute",
            "energy": r["energy"], "energy_hex": float(r["energy"]).hex(),
            "virial_hex": [float(v).hex() for v in r["virial"]],
            "forces_sha256": hashlib.sha256(f.tobytes()).hexdigest()}


def deal_clusters(sizes, rank: int, world: int) -> np.ndarray:
    """The clusters rank `rank` of `world` evaluates: sorted by size, largest
    first (stable), then dealt round robin, so every cluster goes to exactly
    one rank and the ranks' atom counts differ by at most the largest cluster."""
    return np.argsort(-np.asarray(sizes), kind="stable")[rank::world]


def count_lr_pairs(pos, boxlo, cell, cutoff: float) -> int:
    """Unordered atom pairs within the long-range cutoff under the minimum-image
    convention (exact for boxes at least twice the cutoff, as in every bench
    configuration), counted on the host with a k-d tree after the timed
    regions."""
    from scipy.spatial import cKDTree
    x = np.mod(np.asarray(pos) - np.asarray(boxlo), np.asarray(cell))
    tree = cKDTree(x, boxsize=np.asarray(cell))
    return int((tree.count_neighbors(tree, cutoff) - len(x)) // 2)


def step_roofline(n, sr_edges, sr_pairs, lr_pairs, steps_per_s, peak, world):
    """Whole-step FP64 work against the FP64 peak of all GPUs (n, edges, pairs:
    one rank's share). Reference-algorithm FLOP per
    step (filters per directed edge and block: 197,632 forward + reverse, plus
    about 6k for attention, L0 and radial terms; node GEMMs 288 kFLOP per atom
    and block; heads 181 kFLOP per atom; 250 FLOP per long-range half pair) and
    the FLOP this build executes (filters once per pair; each long-range pair
    evaluated from both of its atoms)."""
    ref = world * (3 * sr_edges * 203.6e3 + 3 * n * 288e3 + n * 181e3 + 250 * lr_pairs)
    executed = world * (3 * sr_pairs * 197_632 + 3 * sr_edges * 6.0e3 + 3 * n * 288e3 + n * 181e3
                        + 2 * 250 * lr_pairs)
    return {"reference_flop_per_step": ref, "executed_flop_per_step": executed, "lr_half_pairs": lr_pairs * world,
            "executed_tflops": executed * steps_per_s / 1e12,
            "reference_equivalent_tflops": ref * steps_per_s / 1e12,
            "frac_executed": executed * steps_per_s / 1e12 / (peak * world) if peak else None,
            "peak_tflops_per_gpu": peak, "unit": "TFLOP/s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 5], default=3,
                    help="3 (default): the headline 24,000-atom box; 5: the turbo cluster pack")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--precision", choices=["float64", "mixed"], default="float64",
                    help="mixed: pair-filter GEMMs as three-pass TF32 (the mixed float32 run of config 2)")
    ap.add_argument("--model", default=str(ROOT / "models" / "so3lr.so3lr"),
                    help="model file for configs 1-3 (default: the shipped SO3LR model)")
    ap.add_argument("--no-identity", action="store_true",
                    help="skip the single-point evaluation of the 192,000-atom box (energy and force hash)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.config == 5:
        run_turbo(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
