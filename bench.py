"""Benchmark of the particle hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload sharded16m|dambreak1m|blobs4m|ref65k]

A step is one manifest SPH step of the workload (grid rebuild: cell hash +
stable radix sort + cell table; density; pressure+viscosity; gravity,
integrate, box) on synthetic seeded inputs resident in HBM. The default
workload is cfg3 (16,384,000 particles, 160^3 cells), the config the metric
quotes at 1/2/4/8 GPUs; at N=1 the line also carries the 1M dam-break step
rate and the 2^28-pair radix sort rate under "extra".

--impl reference times the reference's CPU path on the host cores: its own
SPH and module kernels (CUDA C strings) built for the host by
`make -C oracle ref`, or the oracle port of the same step where that build is
absent (the Rust reference itself cannot be built here).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "forge-gpu_b200"))

import numpy as np  # noqa: E402

import workloads  # noqa: E402

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per particle of
# one launch of the dominant kernel, from an ncu capture of
# `bench.py --steps 2 --warmup 3 --no-extra --no-cpu` on a B200 (the kernel's
# traffic grows with the particle count, so it is quoted per particle).
# bench.py cannot read DRAM counters itself; the figure is refreshed with each
# capture of a changed kernel.
NCU_TRAFFIC_B_PER_PARTICLE = {("sharded16m", "force"): 1191.3e6 / 16384000}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# Algorithmic HBM bytes per particle per phase (compulsory traffic; perfect
# neighbour reuse). P = radix passes, C/N = cells per particle.
def alg_bytes(cfg):
    P = (cfg.key_bits + 7) // 8
    cn = (cfg.cells + 1) / cfg.n
    return {
        # hash+histogram: read pos, write key; pass 0: read key, write key+idx;
        # passes 1..P-1: read and write key+idx
        "sort": 12 + 4 + 4 + 8 + 16 * (P - 1),
        # read sorted key + idx, gather pos + vel, write pos4 + vel4 + cell_start
        "cells_gather": 4 + 4 + 12 + 12 + 32 + 4 * cn,
        "density": 16 + 4 + 4 + 4,  # pos4 read, idx read, rho to vel4.w + density_out
        "force": 16 + 16 + 4 + 24,  # pos4, vel4, idx read; pos, vel write
    }


class Clocks:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[4:8]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


PHASES = ("sort", "cells_gather", "density", "force")
WALKS = {"auto": 0, "thread": 1, "group4": 2, "group8": 3, "group16": 4, "rows": 5, "tile": 6}  # forge_grid_set_walk
WALK = 0


def kernels_per_step(cfg):
    """hash + histogram, the sort passes, cell table, chunk fill, density, force."""
    return 1 + (cfg.key_bits + 7) // 8 + 2 + 2


def sharded_kernels_per_step(cfg):
    """Our kernels per step on a rank with two neighbours (the overlapped
    step): grid build (hash + histogram, passes, cell table, chunk fill),
    density, prepare (gather + 3 zone-list kernels), density round (pack,
    scatter), ghost densities, 2 force zones, round 1 (3 selection kernels,
    compaction, halo remap, unpack)."""
    return (1 + (cfg.key_bits + 7) // 8 + 2) + 1 + 4 + 2 + 1 + 2 + 6


def lattice_pairs(cfg):
    """Neighbours within h (self included) of an interior particle of a cubic
    lattice config: the integer offsets with |offset| * spacing < h. None for
    the random workloads."""
    spacing = {"sharded16m": cfg.h / 2, "dambreak1m": cfg.h / 2, "dambreak1m_h025": cfg.h / 5,
               "dambreak65k": cfg.h / 2}.get(cfg.name)
    if spacing is None:
        return None
    m = int(cfg.h / spacing) + 1
    r = np.arange(-m, m + 1)
    d2 = r[:, None, None] ** 2 + r[None, :, None] ** 2 + r[None, None, :] ** 2
    return int((d2 * spacing * spacing < cfg.h * cfg.h * (1 - 1e-9)).sum())


def sph_params(forge_sph, cfg):
    return forge_sph.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)


def step_params(forge_sph, cfg):
    sp = forge_sph.StepParams()
    sp.dt = cfg.dt
    sp.gravity[:] = list(cfg.gravity)
    sp.box_min[:] = list(cfg.box_min)
    sp.box_max[:] = list(cfg.box_max)
    sp.restitution = cfg.restitution
    sp.flags = 7
    return sp


class SphRun:
    """Device-resident state + the step call (forge_sph_step through the C ABI)."""

    def __init__(self, torch, forge_sph, cfg, pos, vel):
        self.t, self.f, self.cfg = torch, forge_sph, cfg
        dev = torch.device("cuda", torch.cuda.current_device())
        self.p = [torch.from_numpy(x).to(dev) for x in pos]
        self.v = [torch.from_numpy(x).to(dev) for x in vel]
        self.rho = torch.empty(cfg.n, dtype=torch.float32, device=dev)
        self.grid = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, dev.index)
        self.grid.set_walk(WALK)
        self.sp = sph_params(forge_sph, cfg)
        self.stp = step_params(forge_sph, cfg)
        self.args = [x.data_ptr() for x in self.p] + [x.data_ptr() for x in self.v] + [self.rho.data_ptr()]
        self.L = forge_sph.lib()

    def step(self):
        st = self.t.cuda.current_stream().cuda_stream
        rc = self.L.forge_sph_step(self.grid.handle, ctypes.byref(self.sp), ctypes.byref(self.stp), *self.args,
                                   self.cfg.n, st)
        self.f.check(rc)


def time_steps(torch, fn, steps):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def time_steps_flushed(torch, fn, steps):
    """Device time of `steps` calls of fn, each preceded (outside its timed
    span) by a 256 MB write that evicts the 126 MB L2: for workloads whose
    state fits in L2."""
    junk = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    for s, e in ev:
        junk.fill_(1.0)
        s.record()
        fn()
        e.record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in ev)


L2_BYTES = 126e6


def state_bytes(cfg):
    """Per-step device state the SPH step touches: caller SoA arrays (28 B) +
    the grid's cell-ordered copies, keys, indices and sort buffers (~68 B)."""
    return cfg.n * 96


def max_over_ranks(torch, dist, v):
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_sph_single(torch, forge_sph, cfg, steps, warmup, rank_dev, clocks=True):
    pos, vel = workloads.particles(cfg)
    run = SphRun(torch, forge_sph, cfg, pos, vel)
    for _ in range(warmup):
        run.step()
    run.grid.check()
    L = forge_sph.lib()
    forge_sph.check(L.forge_grid_profile_enable(run.grid.handle, steps))
    ck = Clocks(rank_dev)
    if clocks:
        ck.start()
        time.sleep(0.3)
    flush = state_bytes(cfg) < 2 * L2_BYTES
    ms = (time_steps_flushed if flush else time_steps)(torch, run.step, steps)
    clk = ck.stop() if clocks else None
    run.grid.check()
    buf = (ctypes.c_float * (4 * steps))()
    got = ctypes.c_uint32(0)
    forge_sph.check(L.forge_grid_profile_read(run.grid.handle, buf, steps, ctypes.byref(got)))
    ph = np.array(buf[:4 * got.value], np.float64).reshape(-1, 4)
    forge_sph.check(L.forge_grid_profile_enable(run.grid.handle, 0))
    phase_ms = {k: float(ph[:, i].mean()) for i, k in enumerate(PHASES)}
    run.l2_flushed = flush
    return run, ms, phase_ms, clk, pos, vel


def e2e_sph(torch, forge_sph, cfg, pos, vel, steps, warmup):
    """Same step through the public API with HOST buffers: every step copies the
    particle state from pinned host memory to the device (forge_io_upload),
    steps, and reads the new state back (forge_io_download, which waits for
    it): pos, vel, 24 B/particle each way."""
    run = SphRun(torch, forge_sph, cfg, pos, vel)
    hp = [torch.from_numpy(x.copy()).pin_memory() for x in pos + vel]
    dv = run.p + run.v
    io = forge_sph.FieldIO(cfg.n, torch.cuda.current_device())
    # The state goes through host memory every step, in chunks: chunk c of
    # step k's result is read back (copy engine D2H) and, as soon as it is
    # on the host, sent again as step k+1's input (copy engine H2D), so the
    # two directions overlap; the step itself waits for every chunk.
    main = torch.cuda.current_stream()
    s_down, s_up = torch.cuda.Stream(), torch.cuda.Stream()
    chunks = 8
    bounds = [cfg.n * c // chunks for c in range(chunks + 1)]
    up_done = torch.cuda.Event()
    io.upload(hp, dv, stream=main)

    def one():
        run.step()
        step_done = torch.cuda.Event()
        step_done.record(main)
        s_down.wait_event(step_done)
        for a, b in zip(bounds[:-1], bounds[1:]):
            io.download([d[a:b] for d in dv], [h[a:b] for h in hp], stream=s_down)  # pinned: asynchronous
            landed = torch.cuda.Event()
            landed.record(s_down)
            s_up.wait_event(landed)
            io.upload([h[a:b] for h in hp], [d[a:b] for d in dv], stream=s_up)
        up_done.record(s_up)
        main.wait_event(up_done)

    for _ in range(warmup):
        one()
    ms = time_steps(torch, one, steps)
    nbytes = sum(x.numel() * 4 for x in hp)
    return ms / steps, nbytes


def sort_rate(torch, forge_sph, kind, n, steps=5, warmup=3):
    keys_np = workloads.sort_keys(kind, n)
    k0 = torch.from_numpy(keys_np.view(np.int32)).cuda()
    keys, vals = k0.clone(), torch.arange(n, dtype=torch.int32, device="cuda")
    s = forge_sph.RadixSorter(n, torch.cuda.current_device())
    bits = 32 if kind == "uniform" else 30

    def one():
        s.sort_pairs(keys, vals, n, 0, bits)

    for _ in range(warmup):
        keys.copy_(k0)
        one()
    s.check()
    total = 0.0
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for _ in range(steps):
        keys.copy_(k0)  # 1 GiB rewrite between sorts also evicts L2
        ev[0].record()
        one()
        ev[1].record()
        torch.cuda.synchronize()
        total += ev[0].elapsed_time(ev[1])
    s.check()
    t = total / steps / 1e3
    passes = (bits + 7) // 8
    gbs = (4 + 16 * passes) * n / t / 1e9  # histogram reads keys; each pass reads+writes key+value
    return {"gkeys_per_s": n / t / 1e9, "ms": t * 1e3, "passes": passes, "achieved_gbs": gbs}


def cpu_sample(cfg, max_particles):
    """Bounded CPU sample of a workload: the first max_particles particles in
    original order (for the lattice configs a bottom slab of the same domain)."""
    pos, vel = workloads.particles(cfg)
    m = min(cfg.n, max_particles)
    return [np.ascontiguousarray(x[:m]) for x in pos], [np.ascontiguousarray(x[:m]) for x in vel], m


def cpu_steps(cfg, pos, vel, steps, threads):
    """Reference algorithm on the host: the oracle port of the manifest step."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    p = oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)
    sp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.step(p, sp, pos, vel, cfg.cell_size, cfg.dims, threads=threads)
        times.append(time.perf_counter() - t0)
    return times


def cpu_threads():
    """Every core this process may run on. Counted from the affinity mask,
    not omp_get_max_threads(): torchrun sets OMP_NUM_THREADS=1 for its ranks,
    and the CPU baseline must not inherit that."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_steps(cfg, pos, vel, steps, threads):
    """The timed CPU reference: the reference's own kernels built for the
    host (oracle/_ref/libref.so: its unfused manifest step, threads in
    parallel) where that library was built, else the oracle port of the same
    step. Returns (per-step seconds, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref
    if not ref.available():
        return cpu_steps(cfg, pos, vel, steps, threads), "port"
    run = ref.ManifestStep(cfg, pos[0].size)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run(pos, vel, threads)
        times.append(time.perf_counter() - t0)
    return times, "reference"


PUBLISHED_DAM_BREAK_L40 = 3.04e8  # `forge run dam-break.toml`, particle-steps/s on an L40 (the reference's README)


def dam_break_manifest(device):
    """The reference's published workload through the `forge run` path
    (manifest.py): 50K-particle dam break, 20,000 steps, timed end to end
    like the reference's CLI (warm-up, graph capture and replays)."""
    try:
        import manifest
        m = manifest.Manifest.from_file(os.path.join(ROOT, "forge-gpu_b200", "examples", "dam_break_50k.toml"))
        r = manifest.run_manifest(m, device=device, seed=0)
        return {"value": r.throughput, "unit": "particle-steps/s", "particles": r.count, "steps": r.steps,
                "seconds": r.elapsed_secs, "published_l40": PUBLISHED_DAM_BREAK_L40,
                "vs_published_l40": r.throughput / PUBLISHED_DAM_BREAK_L40,
                "timing": "wall clock of run_manifest (warm-up + capture + replays), as the reference's CLI"}
    except Exception as e:  # an extra: a failure here must not lose the bench line
        return {"error": repr(e)[:300]}


def cpu_variants(cfg, pos, vel, phase_ms):
    """The reference's own CPU path is single-threaded (HashGrid::build,
    hashgrid.rs:82-125): the oracle step on one thread, and the grid build
    alone (stable counting sort) on one thread over the whole workload, beside
    the GPU's grid build (sort + cell table phases)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    m1 = min(pos[0].size, 131_072)
    p1, v1 = [x[:m1].copy() for x in pos], [x[:m1].copy() for x in vel]
    t1 = min(cpu_steps(cfg, p1, v1, 1, 1))
    full, _ = workloads.particles(cfg)
    t0 = time.perf_counter()
    oracle.grid_build(*full, cfg.cell_size, cfg.dims)
    tg = time.perf_counter() - t0
    gpu_ms = phase_ms["sort"] + phase_ms["cells_gather"]
    return {"single_thread_step": {"value": m1 / t1, "unit": "particle-steps/s", "cores": 1,
                                   "sample": f"first {m1} of {cfg.n} particles, 1 oracle step"},
            "hashgrid_build_single_thread": {"value": cfg.n / tg, "unit": "particles/s", "cores": 1,
                                             "sample": f"all {cfg.n} particles, one build"},
            "hashgrid_build_gpu": {"value": cfg.n / (gpu_ms / 1e3), "unit": "particles/s",
                                   "sample": "sort + cell-table phases of the timed steps"}}


CPU_SAMPLE = {"sharded16m": 1_024_000, "dambreak1m": 262_144, "dambreak1m_h025": 131_072, "blobs4m": 262_144,
              "ref65k": 65_536}


def reference_arm(args, rank, world):
    if rank != 0:
        return
    cfg = workloads.config(args.workload)
    m = CPU_SAMPLE.get(args.workload, 262_144)
    pos, vel, m = cpu_sample(cfg, m)
    th = cpu_threads()
    cpu_reference_steps(cfg, pos, vel, args.warmup, th)
    times, kind = cpu_reference_steps(cfg, pos, vel, args.steps, th)
    t = sum(times) / len(times)
    val = m / t
    what = ("the reference's own kernels (unfused manifest step) built for the host" if kind == "reference"
            else "oracle port of the manifest step")
    sample = f"first {m} of {cfg.n} particles ({cfg.name}), {what}, {th} OpenMP threads on {cpu_model()}"
    line = {"metric": "SPH particle-steps/s", "value": val, "unit": "particle-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": cfg.name, "particles": cfg.n, "cells": cfg.cells, "h": cfg.h},
            "cpu_baseline": {"value": val, "unit": "particle-steps/s", "cores": th, "kind": kind,
                             "cpu": cpu_model(), "sample": sample},
            "e2e": {"value": val, "unit": "particle-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def sharded_roofline(cfg, phase_ms, n_own_max):
    """Roofline of the dominant kernel of a sharded step: the force pass of the
    busiest rank (boundary and interior zones; owned particles only), its
    algorithmic bytes over the rank's force phase time (CUDA events)."""
    fms = phase_ms.get("force")
    if not fms:
        return None
    hbm, peak_kind = peaks()
    achieved = alg_bytes(cfg)["force"] * n_own_max / (fms / 1e3) / 1e9
    return {"bound": "hbm", "kernel": "force (busiest rank)", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "traffic": None, "peak_kind": peak_kind}


def sharded_rate(args, torch, dist, rank, world, local, name, steps, warmup):
    """The sharded step of workload `name` for `steps` timed steps (device
    time, max over ranks): particle-steps/s and ms per step. Skewed
    workloads start at particle-count quantiles and rebalance every 10 steps."""
    import forge_sph
    import slab
    cfg = workloads.config(name)
    pos, vel = workloads.particles(cfg)
    cap = int(cfg.n / world * 1.3) + 4 * (cfg.n // cfg.dims[0]) + 1024
    be = slab.GpuBackend(forge_sph, cfg, cap, local)
    balance = cfg.name == "blobs4m"
    run = slab.SlabRun(dist, rank, world, cfg, pos, vel, be, torch.device("cuda", local), capacity=cap, comm="nccl",
                       forge_sph=forge_sph, balance=balance, halo_width=args.halo_width)
    del pos, vel
    count = [0]

    def step():
        run.step()
        count[0] += 1
        if balance and count[0] % 10 == 0:
            run.rebalance()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    ms = max_over_ranks(torch, dist, time_steps(torch, step, steps))
    be.grid.check()
    return {"value": cfg.n * steps / (ms / 1e3), "unit": "particle-steps/s", "ms_per_step": ms / steps,
            "particles": cfg.n, "steps": steps, "rebalanced_every": 10 if balance else 0}


def run_sharded(args, torch, dist, rank, world, local):
    """N > 1: x-slab decomposition of the workload over `world` GPUs (strong
    scaling: the total particle count is fixed). Halo, ghost-density and
    migration exchanges go rank to rank over NCCL send/recv; the timed region
    is bracketed by barriers and the max over ranks is reported."""
    import forge_sph
    import slab
    cfg = workloads.config(args.workload)
    pos, vel = workloads.particles(cfg)
    cap = int(cfg.n / world * 1.3) + 4 * (cfg.n // cfg.dims[0]) + 1024
    dev = torch.device("cuda", local)
    be = slab.GpuBackend(forge_sph, cfg, cap, local, walk=WALK)
    # skewed workloads: bounds at particle-count quantiles, rebalanced every k steps
    balance = args.rebalance_every > 0 if args.rebalance_every is not None else cfg.name == "blobs4m"
    every = (args.rebalance_every or 10) if balance else 0
    run = slab.SlabRun(dist, rank, world, cfg, pos, vel, be, dev, capacity=cap, comm="nccl", forge_sph=forge_sph,
                       balance=balance, halo_width=args.halo_width)
    del pos, vel
    count = [0]

    def step():
        run.step()
        count[0] += 1
        if every and count[0] % every == 0:
            run.rebalance()

    for _ in range(args.warmup):
        step()
    be.grid.check()
    torch.cuda.synchronize()
    dist.barrier()
    ck = Clocks(local)
    ck.start()
    time.sleep(0.3)
    dist.barrier()
    ms = time_steps(torch, step, args.steps)
    clk = ck.stop()
    be.grid.check()
    ms_max = max_over_ranks(torch, dist, ms)
    n_min = -max_over_ranks(torch, dist, -float(run.n_own))
    n_max = max_over_ranks(torch, dist, float(run.n_own))
    halo = max_over_ranks(torch, dist, float(run.last_halo))
    # phase breakdown on a few extra (untimed) steps
    run.timing = []
    run.timing_side = []
    for _ in range(3):
        run.step()
    torch.cuda.synchronize()
    phase_ms = {}
    ev = run.timing
    for (a, ea), (b, eb) in zip(ev[:-1], ev[1:]):
        if b != "start":
            phase_ms[b] = phase_ms.get(b, 0.0) + ea.elapsed_time(eb) / 3
    side_ms = {}  # overlapped rounds: side-stream progress after the prepare step
    for name, e, ref in run.timing_side:
        side_ms[name] = side_ms.get(name, 0.0) + ref.elapsed_time(e) / 3
    run.timing = None
    phase_ms = {k: max_over_ranks(torch, dist, v) for k, v in sorted(phase_ms.items())}
    side_ms = {k: max_over_ranks(torch, dist, v) for k, v in sorted(side_ms.items())}

    # e2e: the same sharded step with the rank's particle state read from and
    # written back to pinned host memory every step.
    hbuf = torch.empty((run.cols.shape[0], cap), dtype=torch.float32).pin_memory()
    io = forge_sph.FieldIO(cap, local)
    cur = run.n
    for k in range(hbuf.shape[0]):
        hbuf[k, :cur].copy_(run.cols[k, :cur])
    moved = [0]

    def one():
        nonlocal cur
        rows = range(hbuf.shape[0])
        for r0 in (0, 6):  # forge_io_upload: pinned host rows -> device columns (6 per call)
            io.upload([hbuf[k, :cur] for k in rows[r0:r0 + 6]], [run.cols[k, :cur] for k in rows[r0:r0 + 6]])
        run.n = cur
        step()
        cur = run.n
        for r0 in (0, 6):  # forge_io_download: back to the host (returns when there)
            io.download([run.cols[k, :cur] for k in rows[r0:r0 + 6]], [hbuf[k, :cur] for k in rows[r0:r0 + 6]])
        moved[0] += cur * hbuf.shape[0] * 4

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_steps = max(3, args.steps // 2)
    moved[0] = 0
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(e2e_steps):
        one()
    e_ev.record()
    torch.cuda.synchronize()
    nbytes = moved[0]
    e2e_ms = max_over_ranks(torch, dist, s_ev.elapsed_time(e_ev))
    tot_bytes = max_over_ranks(torch, dist, float(nbytes)) * world / e2e_steps
    if rank == 0:
        line = {"metric": "SPH particle-steps/s", "value": cfg.n * args.steps / (ms_max / 1e3),
                "unit": "particle-steps/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": cfg.name, "particles": cfg.n, "cells": cfg.cells, "h": cfg.h,
                           "inputs_exceed_l2": True, "parallelism": f"x-slab over {world} GPUs (NCCL send/recv in the library)",
                           "max_halo_particles_per_rank": halo, "halo_width_h": args.halo_width,
                           "slab_bounds": "initial particle-count quantiles, rebalanced on the density-weighted x-histogram every %d steps"
                           % every if every
                           else "uniform", "owned_per_rank_min_max": [n_min, n_max]},
                "phases_ms_max_over_ranks": phase_ms,
                "roofline": sharded_roofline(cfg, phase_ms, n_max),
                "overlap_ms_after_prepare_max_over_ranks": side_ms,
                "e2e": {"value": cfg.n * e2e_steps / (e2e_ms / 1e3), "unit": "particle-steps/s",
                        "h2d_bytes_per_step": tot_bytes, "d2h_bytes_per_step": tot_bytes},
                "gpu_launches": sharded_kernels_per_step(cfg) * args.steps * world,
                "clocks": clk}
    if not args.no_extra and cfg.name != "blobs4m":
        # cfg4 (skewed blobs) at this GPU count as well
        torch.cuda.empty_cache()
        ex = sharded_rate(args, torch, dist, rank, world, local, "blobs4m", 10, 3)
        if rank == 0:
            line["extra"] = {"blobs4m": ex}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="sharded16m",
                    choices=["sharded16m", "dambreak1m", "dambreak1m_h025", "dambreak65k", "blobs4m", "ref65k"])
    ap.add_argument("--no-extra", action="store_true", help="skip the 1M dam-break and 2^28 sort extras")
    ap.add_argument("--walk", choices=list(WALKS), default="auto",
                    help="neighbour-pass kernel family (auto: row walks below 2^18 particles)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--sort-only", type=int, default=None, metavar="LOG2N",
                    help="time only the standalone key/value sort of 2^LOG2N uniform pairs (for profiling)")
    ap.add_argument("--rebalance-every", type=int, default=None,
                    help="N>1: slab bounds at particle-count quantiles, rebalanced every K steps (0: uniform "
                         "slabs; default: 10 for blobs4m, uniform otherwise)")
    ap.add_argument("--halo-width", type=float, choices=[1.0, 2.0], default=1.0,
                    help="N>1: halo of h with a ghost-density round, or of 2h with ghost densities computed locally")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    global WALK
    WALK = WALKS[args.walk]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    import forge_sph
    torch.cuda.set_device(local)
    if args.sort_only is not None:
        r = sort_rate(torch, forge_sph, "uniform", 1 << args.sort_only, steps=args.steps, warmup=args.warmup)
        print(json.dumps({"sort_only": f"2^{args.sort_only} uniform u32 pairs", **r}), flush=True)
        return
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        run_sharded(args, torch, dist, rank, world, local)
        dist.destroy_process_group()
        return

    cfg = workloads.config(args.workload)
    hbm, peak_kind = peaks()
    run, ms, phase_ms, clk, pos, vel = run_sph_single(torch, forge_sph, cfg, args.steps, args.warmup, local)
    flushed = run.l2_flushed
    ms_step = ms / args.steps
    value = cfg.n / (ms_step / 1e3)
    ab = alg_bytes(cfg)
    dom = max(PHASES, key=lambda k: phase_ms[k])
    achieved = ab[dom] * cfg.n / (phase_ms[dom] / 1e3) / 1e9
    traffic = None
    if (cfg.name, dom) in NCU_TRAFFIC_B_PER_PARTICLE:
        traffic = NCU_TRAFFIC_B_PER_PARTICLE[(cfg.name, dom)] * cfg.n
    pairs = lattice_pairs(cfg)
    phases = {k: {"ms": phase_ms[k], "alg_bytes_per_particle": ab[k],
                  "achieved_gbs": ab[k] * cfg.n / (phase_ms[k] / 1e3) / 1e9,
                  "frac_of_hbm": ab[k] * cfg.n / (phase_ms[k] / 1e3) / 1e9 / hbm} for k in PHASES}
    del run
    torch.cuda.empty_cache()
    e2e_ms, e2e_bytes = e2e_sph(torch, forge_sph, cfg, pos, vel, max(3, args.steps // 2), 3)

    line = {"metric": "SPH particle-steps/s", "value": value, "unit": "particle-steps/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg.name, "particles": cfg.n, "cells": cfg.cells, "h": cfg.h,
                       "key_bits": cfg.key_bits, "inputs_exceed_l2": state_bytes(cfg) >= 2 * L2_BYTES,
                       "l2_flushed_between_steps": flushed,
                       "parallelism": "single GPU"},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind},
            "phases": phases,
            "e2e": {"value": cfg.n / (e2e_ms / 1e3), "unit": "particle-steps/s",
                    "h2d_bytes_per_step": e2e_bytes, "d2h_bytes_per_step": e2e_bytes},
            "gpu_launches": kernels_per_step(cfg) * args.steps,
            "clocks": clk}
    if pairs is not None:  # the pair-evaluation rate of the neighbour passes (interior lattice particles)
        line["neighbour_pairs"] = {
            "within_h_per_particle_incl_self": pairs,
            "density_pair_terms_per_s": pairs * cfg.n / (phase_ms["density"] / 1e3),
            "force_pair_terms_per_s": (pairs - 1) * cfg.n / (phase_ms["force"] / 1e3)}
    if not args.no_cpu:
        m = CPU_SAMPLE.get(cfg.name, 262_144)
        cp, cv, m = cpu_sample(cfg, m)
        th = cpu_threads()
        times, kind = cpu_reference_steps(cfg, cp, cv, 2, th)
        t = min(times)
        what = "reference kernels built for the host" if kind == "reference" else "oracle port"
        line["cpu_baseline"] = {"value": m / t, "unit": "particle-steps/s", "cores": th, "kind": kind,
                                "cpu": cpu_model(),
                                "sample": f"first {m} of {cfg.n} particles, 2 steps ({what}), best of 2"}
        line["cpu_baseline_variants"] = cpu_variants(cfg, cp, cv, phase_ms)
    if not args.no_extra and cfg.name != "dambreak1m":
        extra = {}
        c1 = workloads.config("dambreak1m")
        r1, ms1, ph1, _, _, _ = run_sph_single(torch, forge_sph, c1, 50, 5, local, clocks=False)
        extra["dambreak1m"] = {"value": c1.n / (ms1 / 50 / 1e3), "unit": "particle-steps/s",
                               "ms_per_step": ms1 / 50, "phases_ms": ph1, "l2_flushed_between_steps": r1.l2_flushed,
                               "h": c1.h, "particles_per_cell": 8}
        del r1
        torch.cuda.empty_cache()
        c2 = workloads.config("dambreak1m_h025")
        r2, ms2, ph2, _, _, _ = run_sph_single(torch, forge_sph, c2, 20, 3, local, clocks=False)
        extra["dambreak1m_h025"] = {"value": c2.n / (ms2 / 20 / 1e3), "unit": "particle-steps/s",
                                    "ms_per_step": ms2 / 20, "phases_ms": ph2,
                                    "l2_flushed_between_steps": r2.l2_flushed, "h": c2.h, "particles_per_cell": 125}
        del r2
        torch.cuda.empty_cache()
        c3 = workloads.config("blobs4m")
        r3, ms3, ph3, _, _, _ = run_sph_single(torch, forge_sph, c3, 10, 3, local, clocks=False)
        extra["blobs4m"] = {"value": c3.n / (ms3 / 10 / 1e3), "unit": "particle-steps/s", "ms_per_step": ms3 / 10,
                            "phases_ms": ph3, "l2_flushed_between_steps": r3.l2_flushed, "h": c3.h}
        del r3
        torch.cuda.empty_cache()
        extra["dam_break_50k_manifest"] = dam_break_manifest(local)
        torch.cuda.empty_cache()
        for kind in ("uniform", "morton"):
            extra["radix_sort_2^28_" + kind] = sort_rate(torch, forge_sph, kind, 1 << 28)
            extra["radix_sort_2^28_" + kind]["frac_of_hbm"] = extra["radix_sort_2^28_" + kind]["achieved_gbs"] / hbm
            torch.cuda.empty_cache()
        line["extra"] = extra
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
