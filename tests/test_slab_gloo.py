"""CPU test of the x-slab decomposition (forge-gpu_b200/slab.py) with gloo
ranks: halo exchange, ghost-density exchange and migration must reproduce the
single-process step exactly. The per-rank compute is the oracle (a CPU
stand-in for the GPU backend), local arrays are kept in particle-id order, so
every particle sees its neighbours in the same order as in the unsharded run
and the trajectories must match bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import slab
import slab_cpu
import workloads

STEPS = 8


def _cfg():
    cfg = workloads.small("ref65k", 6000, (20, 20, 20))
    cfg.dt = 1e-3  # fast particles: several cross slab faces within STEPS
    return cfg


def _inputs(cfg):
    pos, vel = workloads.uniform_particles(cfg.n, seed=31, vsigma=1.0)
    return pos, vel


class OracleBackend:
    """CPU backend with the GpuBackend interface (density, force_step)."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.p = oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)

    classify = staticmethod(slab_cpu.torch_classify)
    compact = staticmethod(slab_cpu.torch_compact)
    x_hist = staticmethod(slab_cpu.torch_x_hist)

    def density(self, pos, n):
        c = self.cfg
        p = [x.numpy() for x in pos]
        _, self.si, self.cs = oracle.grid_build(*p, c.cell_size, c.dims)
        return torch.from_numpy(oracle.density(self.p, *p, c.cell_size, c.dims, self.cs, self.si))

    def force_step(self, cols, rho, n, n_update):
        c = self.cfg
        a = [x.numpy() for x in cols]  # views: updated in place
        v, _ = oracle.force(self.p, 3, *a[:3], *a[3:], rho.numpy(), c.cell_size, c.dims, self.cs, self.si,
                            np.float32(c.dt))
        dt = np.float32(c.dt)
        e = np.float32(c.restitution)
        for k in range(3):  # gravity.rs:31-34, integrate.rs:16-31, box_collider.rs:36-46 (float32, in order)
            u = (v[k][:n_update] + np.float32(c.gravity[k]) * dt).astype(np.float32)
            u = np.where(np.isfinite(u), u, np.float32(0)).astype(np.float32)
            x = (a[k][:n_update] + u * dt).astype(np.float32)
            lo, hi = np.float32(c.box_min[k]), np.float32(c.box_max[k])
            below = x < lo
            x = np.where(below, lo, x)
            u = np.where(below, np.abs(u) * e, u)
            above = x > hi
            x = np.where(above, hi, x)
            u = np.where(above, -np.abs(u) * e, u)
            a[k][:n_update] = x
            a[3 + k][:n_update] = u


def _rank_main(rank, world, port, out_path, halo_width=1.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        pos, vel = _inputs(cfg)
        run = slab.SlabRun(dist, rank, world, cfg, pos, vel, OracleBackend(cfg), torch.device("cpu"),
                           order_by_id=True, halo_width=halo_width,
                           comm=lambda r: slab_cpu.PyComm(r, dist))
        first_owner = run.ids().clone()
        halo = 0
        for _ in range(STEPS):
            run.step()
            halo += run.last_halo
        moved = int((~torch.isin(run.ids(), first_owner)).sum())
        states = [None] * world
        dist.all_gather_object(states, (run.state.numpy().copy(), moved, halo))
        if rank == 0:
            np.save(out_path, np.array(states, dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,halo_width", [(2, 1.0), (3, 1.0), (3, 2.0)])
def test_sharded_step_matches_single_process(tmp_path, world, halo_width):
    """halo_width 2: a 2h halo, ghost densities computed locally (no density
    round) -- the same trajectory bit for bit."""
    out = str(tmp_path / "states.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), out, halo_width), nprocs=world, join=True,
                       start_method="spawn")
    states = np.load(out, allow_pickle=True)
    rows = np.concatenate([s[0] for s in states])
    assert sum(s[1] for s in states) > 0, "no particle migrated: the test does not exercise migration"
    assert all(s[2] > 0 for s in states), "a rank received no halo"
    ids = rows[:, 6].copy().view(np.int32)
    cfg = _cfg()
    assert np.array_equal(np.sort(ids), np.arange(cfg.n)), "particles lost or duplicated"
    order = np.argsort(ids)
    got = rows[order, :6]
    pos, vel = _inputs(cfg)
    sp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    p = oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)
    for _ in range(STEPS):
        oracle.step(p, sp, pos, vel, cfg.cell_size, cfg.dims)
    want = np.stack(pos + vel, axis=1)
    assert np.array_equal(got, want)


def _skewed_inputs(cfg):
    """Two dense clumps in x (a cfg4-like skew): uniform slabs are imbalanced."""
    rng = np.random.Generator(np.random.PCG64(77))
    n = cfg.n
    x = np.where(np.arange(n) % 3 == 0, rng.normal(0.2, 0.04, n), rng.normal(0.7, 0.06, n))
    pos = [np.clip(x, 0.0, 0.999).astype(np.float32), rng.random(n, dtype=np.float32),
           rng.random(n, dtype=np.float32)]
    vel = [(rng.normal(0.0, 1.0, n)).astype(np.float32) for _ in range(3)]
    return pos, vel


def _balanced_rank_main(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        pos, vel = _skewed_inputs(cfg)
        run = slab.SlabRun(dist, rank, world, cfg, pos, vel, OracleBackend(cfg), torch.device("cpu"),
                           order_by_id=True, balance=True, hist_bins=256,
                           comm=lambda r: slab_cpu.PyComm(r, dist))
        first = list(run.geo.bounds)
        loads = [run.n_own]
        moved = 0
        for s in range(STEPS):
            run.step()
            if s % 2 == 1:
                moved += int(run.rebalance())
            loads.append(run.n_own)
        states = [None] * world
        dist.all_gather_object(states, (run.state.numpy().copy(), first, list(run.geo.bounds), loads, moved))
        if rank == 0:
            np.save(out_path, np.array(states, dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_balanced_slabs_with_rebalancing_match_single_process(tmp_path):
    """The partition for skewed inputs: initial bounds at particle-count
    quantiles, rebalanced every 2 steps from an all-reduced work histogram
    (x weighted by density), each bound kept between its old neighbours;
    the trajectory is still the single-process one bit for bit and the
    loads stay balanced."""
    world = 3
    out = str(tmp_path / "states.npy")
    mp.start_processes(_balanced_rank_main, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    states = np.load(out, allow_pickle=True)
    cfg = _cfg()
    first = states[0][1]
    assert all(s[1] == first for s in states), "ranks disagree on the bounds"
    assert abs(first[1] - 1 / 3) > 0.02, "initial bounds are not the quantiles"
    assert sum(s[4] for s in states) > 0, "no rebalancing moved a bound"
    for k in range(STEPS + 1):
        loads = [s[3][k] for s in states]
        assert max(loads) < 1.25 * cfg.n / world, loads
    rows = np.concatenate([s[0] for s in states])
    ids = rows[:, 6].copy().view(np.int32)
    assert np.array_equal(np.sort(ids), np.arange(cfg.n)), "particles lost or duplicated"
    got = rows[np.argsort(ids), :6]
    pos, vel = _skewed_inputs(cfg)
    sp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    p = oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)
    for _ in range(STEPS):
        oracle.step(p, sp, pos, vel, cfg.cell_size, cfg.dims)
    assert np.array_equal(got, np.stack(pos + vel, axis=1))
