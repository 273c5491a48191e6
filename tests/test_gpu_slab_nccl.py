"""GPU test of the library's NCCL slab exchange (forge_slab_exchange /
forge_slab_exchange_rho): two ranks on two GPUs must reproduce the single-GPU
forge_sph_step trajectory bit for bit (local arrays in particle-id order).
Needs two visible GPUs; skipped on one."""
import ctypes
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import forge_sph
import slab
import workloads

pytestmark = pytest.mark.gpu
STEPS = 6


def _cfg():
    cfg = workloads.small("ref65k", 40_000, (24, 24, 24))
    cfg.dt = 5e-4
    return cfg


def _inputs(cfg):
    return workloads.uniform_particles(cfg.n, seed=43, vsigma=1.0)


def _skewed(cfg):
    rng = np.random.Generator(np.random.PCG64(5))
    n = cfg.n
    x = np.where(np.arange(n) % 4 == 0, rng.normal(0.25, 0.05, n), rng.normal(0.75, 0.08, n))
    pos = [np.clip(x, 0.0, 0.999).astype(np.float32), rng.random(n, dtype=np.float32),
           rng.random(n, dtype=np.float32)]
    return pos, [rng.normal(0.0, 1.0, n).astype(np.float32) for _ in range(3)]


def _rank_main(rank, world, port, out_path, order_by_id=True, skewed=False, halo_width=1.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)  # plumbing: the NCCL id broadcast
    try:
        torch.cuda.set_device(rank)
        cfg = _cfg()
        pos, vel = _skewed(cfg) if skewed else _inputs(cfg)
        # test mode compares bit for bit with one GPU: both sides use the
        # per-thread walks, whose per-particle sums do not depend on which
        # particles share a thread (group walks agree to fp32 rounding only)
        be = slab.GpuBackend(forge_sph, cfg, cfg.n, rank, walk=forge_sph.WALK_THREAD if order_by_id else 0)
        run = slab.SlabRun(dist, rank, world, cfg, pos, vel, be, torch.device("cuda", rank), order_by_id=order_by_id,
                           capacity=cfg.n + 8, comm="nccl", forge_sph=forge_sph, balance=skewed, hist_bins=256,
                           halo_width=halo_width)
        for s in range(STEPS):
            run.step()
            if skewed and s % 2 == 1:
                run.rebalance()
        be.grid.check()
        states = [None] * world
        dist.all_gather_object(states, run.state.cpu().numpy().copy())
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


def _sharded_rows(tmp_path, order_by_id, skewed=False, world=2, halo_width=1.0):
    out = str(tmp_path / "states.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), out, order_by_id, skewed, halo_width), nprocs=world, join=True,
                       start_method="spawn")
    rows = np.concatenate(list(np.load(out, allow_pickle=True)))
    ids = rows[:, 6].copy().view(np.int32)
    assert np.array_equal(np.sort(ids), np.arange(_cfg().n)), "particles lost or duplicated"
    return rows[np.argsort(ids), :6]


def _single_gpu_rows(skewed=False, walk=None):
    cfg = _cfg()
    pos, vel = _skewed(cfg) if skewed else _inputs(cfg)
    p = [torch.from_numpy(x.copy()).cuda() for x in pos]
    v = [torch.from_numpy(x.copy()).cuda() for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    g.set_walk(forge_sph.WALK_THREAD if walk is None else walk)
    be = slab.GpuBackend(forge_sph, cfg, 1, 0)
    L = forge_sph.lib()
    for _ in range(STEPS):
        forge_sph.check(L.forge_sph_step(g.handle, ctypes.byref(be.sp), ctypes.byref(be.stp),
                                         *(x.data_ptr() for x in p + v), rho.data_ptr(), cfg.n, None))
    return np.stack([x.cpu().numpy() for x in p + v], axis=1)


two_gpus = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@two_gpus
@pytest.mark.parametrize("halo_width", [1.0, 2.0])
def test_nccl_sharded_step_matches_single_gpu(cuda, tmp_path, halo_width):
    """Test mode (local arrays in particle-id order each step): bit for bit,
    with the 1h halo + ghost-density round and with the 2h halo whose ghost
    densities are computed locally."""
    assert np.array_equal(_sharded_rows(tmp_path, True, halo_width=halo_width), _single_gpu_rows())


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("order_by_id", [True, False])
def test_nccl_four_ranks(cuda, tmp_path, order_by_id):
    """Four ranks: the two middle ones exchange with both neighbours. Test
    mode bit for bit; the overlapped production step within fp32 summation
    order (as in the two-rank test)."""
    got, want = _sharded_rows(tmp_path, order_by_id, world=4), _single_gpu_rows(walk=None if order_by_id else 0)
    if order_by_id:
        assert np.array_equal(got, want)
    else:
        np.testing.assert_allclose(got[:, :3], want[:, :3], rtol=0, atol=1e-5)
        np.testing.assert_allclose(got[:, 3:], want[:, 3:], rtol=0, atol=1e-3)


@two_gpus
@pytest.mark.parametrize("halo_width", [1.0, 2.0])
def test_nccl_overlapped_step_close_to_single_gpu(cuda, tmp_path, halo_width):
    """The production path (both exchange rounds overlapped with the interior
    force on a second stream, local arrays in exchange order): the same
    particles, and trajectories equal up to fp32 summation order (neighbour
    order differs from the single-GPU run): |dx| <= 1e-5, |dv| <= 1e-3."""
    got, want = _sharded_rows(tmp_path, False, halo_width=halo_width), _single_gpu_rows(walk=0)
    np.testing.assert_allclose(got[:, :3], want[:, :3], rtol=0, atol=1e-5)
    np.testing.assert_allclose(got[:, 3:], want[:, 3:], rtol=0, atol=1e-3)


@two_gpus
def test_nccl_balanced_rebalanced_step_matches_single_gpu(cuda, tmp_path):
    """Skewed x distribution: slab bounds at particle-count quantiles,
    rebalanced every 2 steps (forge_slab_comm_set_bounds + a migrating round
    1); test mode, so bit for bit."""
    assert np.array_equal(_sharded_rows(tmp_path, True, skewed=True), _single_gpu_rows(skewed=True))


def _dead_neighbour_main(rank, world, port, out_path):
    """Rank 1 leaves between steps (no kernel or NCCL call in flight); rank
    0's next exchange must fail with FORGE_ERR_TIMEOUT after its 2 s
    deadline instead of hanging, with its communicator aborted."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    cfg = _cfg()
    pos, vel = _inputs(cfg)
    be = slab.GpuBackend(forge_sph, cfg, cfg.n, rank)
    run = slab.SlabRun(dist, rank, world, cfg, pos, vel, be, torch.device("cuda", rank), capacity=cfg.n + 8,
                       comm="nccl", forge_sph=forge_sph)
    forge_sph.check(forge_sph.lib().forge_slab_comm_set_timeout(run.comm.h, 2.0))
    run.step()
    torch.cuda.synchronize()
    dist.barrier()  # both finished step 1
    if rank == 1:
        time.sleep(8.0)  # gone: never joins step 2
        os._exit(0)
    t0 = time.monotonic()
    try:
        run.step()
        torch.cuda.synchronize()
        res = "no error"
    except forge_sph.ForgeError as e:
        res = f"{e.code}|{e}"
    took = time.monotonic() - t0
    again = ""
    try:
        run.comm.exchange_rho(torch.zeros(8, device="cuda"))
    except forge_sph.ForgeError as e:
        again = str(e)
    with open(out_path, "w") as f:
        f.write(f"{res}\n{took}\n{again}\n")
    os._exit(0)


@two_gpus
def test_nccl_dead_neighbour_times_out(cuda, tmp_path):
    out = str(tmp_path / "result.txt")
    mp.start_processes(_dead_neighbour_main, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    res, took, again = open(out).read().split("\n")[:3]
    assert res.startswith(f"{forge_sph.FORGE_ERR_TIMEOUT}|"), res
    assert "aborted" in res
    assert 1.5 < float(took) < 30.0
    assert "aborted" in again
