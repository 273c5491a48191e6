"""GPU parity of every neighbour-pass kernel family (forge_grid_set_walk:
per-thread walks; warp-cooperative group walks of 4, 8 and 16 particles per
warp; row-parallel walks, nine threads per particle; cell-block CTAs over
rows staged in shared memory) against the oracle, on sparse, lattice, dense, skewed, ragged and
out-of-grid inputs and with cell size < h (no shared walk across cells).

Tolerances as in test_gpu_sph.py: density 1e-5 relative; accelerations
|a_gpu - a_cpu| <= 1e-4 * sum_j |term_j| / rho_i."""
import ctypes

import numpy as np
import pytest

import forge_sph
import oracle
import workloads
from _util import assert_force_close, dev, host_f32

pytestmark = pytest.mark.gpu


def _case(name):
    if name == "sparse":  # ~1 particle per cell, positions outside the grid
        cfg = workloads.small("ref65k", 20_000, (28, 28, 28))
        pos, vel = workloads.uniform_particles(cfg.n, seed=5, lo=-0.03, hi=1.03)
    elif name == "lattice":  # 8 per cell, cell-aligned groups
        cfg = workloads.config("dambreak65k")
        pos, _ = workloads.particles(cfg)
        vel = list(workloads.uniform_particles(cfg.n, seed=6)[1])
    elif name == "dense":  # ~24 per cell, random
        cfg = workloads.small("ref65k", 24_000, (10, 10, 10))
        pos, vel = workloads.uniform_particles(cfg.n, seed=7, lo=-0.02, hi=1.02)
    elif name == "blobs":  # hot cells of several hundred particles
        cfg = workloads.small("ref65k", 30_000, (20, 20, 20))
        rng = np.random.Generator(np.random.PCG64(8))
        c = rng.uniform(0.2, 0.8, (6, 3))
        xyz = c[np.arange(cfg.n) % 6] + rng.normal(0, 0.02, (cfg.n, 3))
        pos = [np.ascontiguousarray(xyz[:, k], dtype=np.float32) for k in range(3)]
        vel = [rng.normal(0, 0.1, cfg.n).astype(np.float32) for _ in range(3)]
    elif name == "ragged":  # n not a multiple of any group size, tiny degenerate grid
        cfg = workloads.small("ref65k", 1_003, (3, 2, 5))
        pos, vel = workloads.uniform_particles(cfg.n, seed=9, lo=-0.1, hi=1.1)
    elif name == "small_cells":  # cell size h/2: members must share their cell
        cfg = workloads.small("ref65k", 20_000, (24, 24, 24))
        cfg.h = 2.0 / 24
        pos, vel = workloads.uniform_particles(cfg.n, seed=10)
    else:
        raise KeyError(name)
    return cfg, pos, vel


CASES = ["sparse", "lattice", "dense", "blobs", "ragged", "small_cells"]
WALKS = {"auto": forge_sph.WALK_AUTO, "thread": forge_sph.WALK_THREAD, "group4": forge_sph.WALK_GROUP4,
         "group8": forge_sph.WALK_GROUP8, "group16": forge_sph.WALK_GROUP16, "rows": forge_sph.WALK_ROWS,
         "tile": forge_sph.WALK_TILE}


def _params(mod, cfg):
    return mod.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)


def _oracle(cfg, pos, vel, terms):
    ci, si, cst = oracle.grid_build(*pos, cfg.cell_size, cfg.dims)
    th = oracle.max_threads()
    p = _params(oracle, cfg)
    rho = oracle.density(p, *pos, cfg.cell_size, cfg.dims, cst, si, th)
    args = (*pos, *vel, rho, cfg.cell_size, cfg.dims, cst, si, 1e-4)
    _, a = oracle.force(p, terms, *args, threads=th)
    _, scale = oracle.force(p, terms | 4, *args, threads=th)
    return rho, a, scale


def _gpu(torch, cfg, pos, vel, terms, walk=forge_sph.WALK_AUTO):
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    g.set_walk(walk)
    d, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    L = forge_sph.lib()
    sp = _params(forge_sph, cfg)
    forge_sph.check(L.forge_sph_density(g.handle, ctypes.byref(sp), *(x.data_ptr() for x in d), cfg.n,
                                        rho.data_ptr(), None))
    vo = [torch.empty_like(x) for x in v]
    a = [torch.empty_like(x) for x in v]
    forge_sph.check(L.forge_sph_force(g.handle, ctypes.byref(sp), terms, *(x.data_ptr() for x in d),
                                      *(x.data_ptr() for x in v), rho.data_ptr(), cfg.n, 1e-4,
                                      *(x.data_ptr() for x in vo), *(x.data_ptr() for x in a), None))
    g.check()
    return host_f32(rho), [host_f32(x) for x in a]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("walk", list(WALKS))
def test_density_and_force_vs_oracle(cuda, case, walk):
    cfg, pos, vel = _case(case)
    rho, a, scale = _oracle(cfg, pos, vel, 3)
    rg, ag = _gpu(cuda, cfg, pos, vel, 3, WALKS[walk])
    np.testing.assert_allclose(rg, rho, rtol=1e-5, atol=0)
    assert_force_close(ag, a, scale)


@pytest.mark.parametrize("terms", [1, 2])
@pytest.mark.parametrize("case", ["dense", "blobs"])
@pytest.mark.parametrize("walk", ["thread", "group8", "rows"])
def test_single_terms(cuda, terms, case, walk):
    cfg, pos, vel = _case(case)
    _, a, scale = _oracle(cfg, pos, vel, terms)
    _, ag = _gpu(cuda, cfg, pos, vel, terms, WALKS[walk])
    assert_force_close(ag, a, scale)


@pytest.mark.parametrize("case", ["lattice", "blobs"])
@pytest.mark.parametrize("walk", ["thread", "group8", "rows"])
def test_passes_are_deterministic(cuda, case, walk):
    cfg, pos, vel = _case(case)
    r1, a1 = _gpu(cuda, cfg, pos, vel, 3, WALKS[walk])
    r2, a2 = _gpu(cuda, cfg, pos, vel, 3, WALKS[walk])
    assert np.array_equal(r1, r2)
    for x, y in zip(a1, a2):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("case", CASES)
def test_tile_density_equals_thread_walk(cuda, case):
    """The cell-block density pass walks the same candidates in the same
    order as the per-thread walk, from staged shared memory (or from global
    memory where a segment's rows exceed the staging capacity: the dense and
    blob cases): bit-identical densities."""
    cfg, pos, vel = _case(case)
    rt, _ = _gpu(cuda, cfg, pos, vel, 3, forge_sph.WALK_THREAD)
    rs, _ = _gpu(cuda, cfg, pos, vel, 3, forge_sph.WALK_TILE)
    assert np.array_equal(rt, rs)


@pytest.mark.parametrize("case", ["dense", "blobs"])
def test_fused_step_vs_oracle(cuda, case):
    """forge_sph_step (density, force, gravity/integrate/box) on dense and
    skewed inputs, against the oracle's step."""
    cfg, pos, vel = _case(case)
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    p, v = [dev(cuda, x) for x in pos], [dev(cuda, x) for x in vel]
    rho = cuda.empty(cfg.n, dtype=cuda.float32, device="cuda")
    sp = forge_sph.StepParams()
    sp.dt = cfg.dt
    sp.gravity[:] = list(cfg.gravity)
    sp.box_min[:] = list(cfg.box_min)
    sp.box_max[:] = list(cfg.box_max)
    sp.restitution = cfg.restitution
    sp.flags = 7
    forge_sph.check(forge_sph.lib().forge_sph_step(g.handle, ctypes.byref(_params(forge_sph, cfg)), ctypes.byref(sp),
                                                   *(x.data_ptr() for x in p + v), rho.data_ptr(), cfg.n, None))
    g.check()
    po, vo = [x.copy() for x in pos], [x.copy() for x in vel]
    osp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    ro = oracle.step(_params(oracle, cfg), osp, po, vo, cfg.cell_size, cfg.dims, threads=oracle.max_threads(),
                     want_density=True)
    np.testing.assert_allclose(host_f32(rho), ro, rtol=1e-5)
    for k in range(3):
        np.testing.assert_allclose(host_f32(p[k]), po[k], rtol=0, atol=1e-6)
        np.testing.assert_allclose(host_f32(v[k]), vo[k], rtol=1e-4, atol=1e-6)


def test_x_window_step_equals_whole_grid(cuda):
    """A grid restricted to an x-window (a shard's slab) gives the same step
    bit for bit as the whole grid when every particle lies inside it: cells
    are assigned globally and then shifted, so rows, windows and candidate
    order are unchanged."""
    cfg = workloads.small("ref65k", 30_000, (40, 40, 40))
    rng = np.random.Generator(np.random.PCG64(12))
    pos = [rng.uniform(0.3, 0.6, cfg.n).astype(np.float32), rng.random(cfg.n, dtype=np.float32),
           rng.random(cfg.n, dtype=np.float32)]
    vel = [rng.normal(0, 0.05, cfg.n).astype(np.float32) for _ in range(3)]

    def run(window):
        g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
        if window:
            g.set_x_window(10, 16)  # cells [10, 26) cover x in [0.25, 0.65)
        p, v = [dev(cuda, x) for x in pos], [dev(cuda, x) for x in vel]
        rho = cuda.empty(cfg.n, dtype=cuda.float32, device="cuda")
        sp = forge_sph.StepParams()
        sp.dt = 1e-4
        sp.flags = 3  # gravity + integrate (no box)
        sp.gravity[:] = [0.0, -9.81, 0.0]
        for _ in range(3):
            forge_sph.check(forge_sph.lib().forge_sph_step(g.handle, ctypes.byref(_params(forge_sph, cfg)),
                                                           ctypes.byref(sp), *(x.data_ptr() for x in p + v),
                                                           rho.data_ptr(), cfg.n, None))
        g.check()
        return [host_f32(x) for x in p + v + [rho]]

    for a, b in zip(run(True), run(False)):
        assert np.array_equal(a, b)


def test_x_window_rejects_cells_outside_the_grid(cuda):
    g = forge_sph.HashGrid(0.1, (10, 10, 10), (0, 0, 0), 16, 0)
    with pytest.raises(forge_sph.ForgeError, match="outside"):
        g.set_x_window(5, 6)
    g.set_x_window(5, 5)
