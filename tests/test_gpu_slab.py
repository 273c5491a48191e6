"""GPU test of the sharded SPH step: two ranks (processes) on one B200 run
the x-slab decomposition with the library's kernels (forge_sph_density +
forge_sph_force_step) and gloo exchanges staged through host memory; with
local arrays in particle-id order the result must equal the single-GPU
forge_sph_step run bit for bit."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import forge_sph
import slab
import slab_cpu
import workloads

pytestmark = pytest.mark.gpu
STEPS = 6


def _cfg():
    cfg = workloads.small("ref65k", 40_000, (24, 24, 24))
    cfg.dt = 5e-4
    return cfg


def _inputs(cfg):
    return workloads.uniform_particles(cfg.n, seed=41, vsigma=1.0)


def _rank_main(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(0)
        cfg = _cfg()
        pos, vel = _inputs(cfg)
        # per-thread walks on both sides: bit-for-bit comparison (see
        # test_gpu_slab_nccl.py)
        be = slab.GpuBackend(forge_sph, cfg, cfg.n, 0, walk=forge_sph.WALK_THREAD)
        run = slab.SlabRun(dist, rank, world, cfg, pos, vel, be, torch.device("cuda", 0), order_by_id=True,
                           comm=lambda r: slab_cpu.PyComm(r, dist, comm_device="cpu"))
        for _ in range(STEPS):
            run.step()
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


def test_two_rank_sharded_step_matches_single_gpu(cuda, tmp_path):
    out = str(tmp_path / "states.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    rows = np.concatenate(list(np.load(out, allow_pickle=True)))
    ids = rows[:, 6].copy().view(np.int32)
    cfg = _cfg()
    assert np.array_equal(np.sort(ids), np.arange(cfg.n))
    got = rows[np.argsort(ids), :6]
    # single GPU, same steps
    pos, vel = _inputs(cfg)
    p = [torch.from_numpy(x.copy()).cuda() for x in pos]
    v = [torch.from_numpy(x.copy()).cuda() for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    g.set_walk(forge_sph.WALK_THREAD)
    be = slab.GpuBackend(forge_sph, cfg, 1, 0)
    L = forge_sph.lib()
    for _ in range(STEPS):
        forge_sph.check(L.forge_sph_step(g.handle, ctypes.byref(be.sp), ctypes.byref(be.stp),
                                         *(x.data_ptr() for x in p + v), rho.data_ptr(), cfg.n, None))
    want = np.stack([x.cpu().numpy() for x in p + v], axis=1)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [0, 1, 4095, 4097, 300_000])
def test_slab_classify_and_compact_match_torch(cuda, n):
    torch_ = cuda
    g = torch_.Generator().manual_seed(n)
    x = (torch_.rand(n, generator=g) * 1.2 - 0.1).cuda()
    cfg = _cfg()
    be = slab.GpuBackend(forge_sph, cfg, max(n, 1), 0)
    for flags in (1, 2, 3, 5, 6, 7, 13, 14, 15):
        got = be.classify(x, n, 0.25, 0.75, 0.05, flags)
        want = slab_cpu.torch_classify(x, n, 0.25, 0.75, 0.05, flags)
        for a, b in zip(got, want):
            assert torch_.equal(a, b), flags
    mig = slab_cpu.torch_classify(x, n, 0.25, 0.75, 0.05, 3)[0]
    cols = torch_.rand((7, n + 5), generator=g).cuda()
    ref = cols.clone()
    be.compact(cols, n, mig)
    slab_cpu.torch_compact(ref, n, mig)
    keep = n - mig.numel()
    assert torch_.equal(cols[:, :keep], ref[:, :keep])


@pytest.mark.parametrize("n", [0, 1, 1000, 300_001])
def test_x_hist_matches_torch_and_is_deterministic(cuda, n):
    """forge_slab_x_hist (the load-balancing histogram): counts equal the
    torch restatement exactly; density weights within the 2^-16 fixed-point
    quantisation; two runs give the same bits."""
    g = cuda.Generator().manual_seed(n + 1)
    x = (cuda.rand(n, generator=g) * 1.4 - 0.2).cuda()
    w = (cuda.rand(n, generator=g) * 2000.0).cuda()
    be = slab.GpuBackend(forge_sph, _cfg(), max(n, 1), 0)
    c = be.x_hist(x, None, 0.0, 1.0, 256)
    assert cuda.equal(c.cpu(), slab_cpu.torch_x_hist(x.cpu(), None, 0.0, 1.0, 256))
    h1 = be.x_hist(x, w, 0.0, 1.0, 4096)
    h2 = be.x_hist(x, w, 0.0, 1.0, 4096)
    assert cuda.equal(h1, h2)
    want = slab_cpu.torch_x_hist(x.cpu(), w.cpu(), 0.0, 1.0, 4096)
    assert cuda.allclose(h1.cpu(), want, rtol=1e-6, atol=1e-3)
