"""GPU parity: SPH density, pressure/viscosity forces, the fused step and
100-step trajectories, against the oracle.

Tolerances (fp32; the GPU fuses multiply-adds, the oracle rounds every op):
  density  |rho_gpu - rho_cpu| <= 1e-5 * rho_cpu            (per particle)
  accel    |a_gpu - a_cpu|     <= 1e-4 * sum_j |term_j|/rho_i (per component)
  trajectory (100 steps, cfg0) |x_gpu - x_cpu| <= 1e-5 (positions in [0,1]);
             |v_gpu - v_cpu| <= 3e-5 for every particle and <= 1e-4 |v_cpu|
             for all but 0.1% of them (fp32 rounding differences grow
             chaotically over 100 steps; measured worst case 1.3e-5)
"""
import ctypes

import numpy as np
import pytest

import forge_sph
import oracle
import workloads
from _util import assert_force_close, dev, host_f32

pytestmark = pytest.mark.gpu
RHO_TOL = 1e-5


def oparams(cfg):
    return oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)


def gparams(cfg):
    return forge_sph.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)


def run_density(torch, cfg, pos):
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    d = [dev(torch, p) for p in pos]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    forge_sph.check(forge_sph.lib().forge_sph_density(g.handle, ctypes.byref(gparams(cfg)), *(x.data_ptr() for x in d),
                                                      cfg.n, rho.data_ptr(), None))
    g.check()
    return g, d, rho


def oracle_density(cfg, pos, threads=None):
    ci, si, cst = oracle.grid_build(*pos, cfg.cell_size, cfg.dims)
    rho = oracle.density(oparams(cfg), *pos, cfg.cell_size, cfg.dims, cst, si,
                         threads or oracle.max_threads())
    return rho, si, cst


def check_density(cfg, pos, rho_gpu):
    rho, si, cst = oracle_density(cfg, pos)
    np.testing.assert_allclose(host_f32(rho_gpu), rho, rtol=RHO_TOL, atol=0)
    return rho, si, cst


def test_density_cfg0(cuda):
    cfg = workloads.config("ref65k")
    pos, _ = workloads.particles(cfg)
    _, _, rho = run_density(cuda, cfg, pos)
    check_density(cfg, pos, rho)


@pytest.mark.parametrize("n,dims", [(1, (4, 4, 4)), (5, (3, 2, 1)), (4097, (1, 1, 1)), (30_000, (25, 7, 3))])
def test_density_ragged_and_degenerate_grids(cuda, n, dims):
    cfg = workloads.small("ref65k", n, dims)
    pos, _ = workloads.uniform_particles(n, seed=n, lo=-0.05, hi=1.05)
    _, _, rho = run_density(cuda, cfg, pos)
    check_density(cfg, pos, rho)


def test_density_dense_cells_dambreak65k(cuda):
    cfg = workloads.config("dambreak65k")
    pos, _ = workloads.particles(cfg)
    _, _, rho = run_density(cuda, cfg, pos)
    check_density(cfg, pos, rho)


def run_force(torch, cfg, pos, vel, terms, dt=1e-4):
    g, d, rho = run_density(torch, cfg, pos)
    v = [dev(torch, x) for x in vel]
    vo = [torch.empty_like(x) for x in v]
    a = [torch.empty_like(x) for x in v]
    forge_sph.check(forge_sph.lib().forge_sph_force(
        g.handle, ctypes.byref(gparams(cfg)), terms, *(x.data_ptr() for x in d), *(x.data_ptr() for x in v),
        rho.data_ptr(), cfg.n, dt, *(x.data_ptr() for x in vo), *(x.data_ptr() for x in a), None))
    g.check()
    return rho, [host_f32(x) for x in vo], [host_f32(x) for x in a]


@pytest.mark.parametrize("terms", [1, 2, 3])
def test_force_terms_cfg0(cuda, terms):
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    rho_g, vo_g, a_g = run_force(cuda, cfg, pos, vel, terms)
    rho, si, cst = check_density(cfg, pos, rho_g)
    p = oparams(cfg)
    args = (*pos, *vel, rho, cfg.cell_size, cfg.dims, cst, si, 1e-4)
    th = oracle.max_threads()
    vo, a = oracle.force(p, terms, *args, threads=th)
    _, scale = oracle.force(p, terms | 4, *args, threads=th)
    assert_force_close(a_g, a, scale)
    for k in range(3):
        np.testing.assert_allclose(vo_g[k], vo[k], rtol=1e-5, atol=1e-4 * 1e-4 * scale[k].max())


def test_force_dense_lattice_dambreak65k(cuda):
    cfg = workloads.config("dambreak65k")
    pos, vel = workloads.particles(cfg)
    vel = [np.asarray(workloads.uniform_particles(cfg.n, seed=4)[1][k]) for k in range(3)]
    rho_g, _, a_g = run_force(cuda, cfg, pos, vel, 3)
    rho, si, cst = oracle_density(cfg, pos)
    args = (*pos, *vel, rho, cfg.cell_size, cfg.dims, cst, si, 1e-4)
    _, a = oracle.force(oparams(cfg), 3, *args, threads=oracle.max_threads())
    _, scale = oracle.force(oparams(cfg), 7, *args, threads=oracle.max_threads())
    assert_force_close(a_g, a, scale)


@pytest.mark.parametrize("terms", [1, 2, 3])
def test_force_dense_cells_single_particle_path(cuda, terms):
    """>= 8 particles per cell on average selects the one-particle-per-thread
    force kernel; it must agree with the oracle like the two-particle one."""
    cfg = workloads.small("ref65k", 24_000, (10, 10, 10))
    pos, vel = workloads.uniform_particles(cfg.n, seed=77, lo=-0.02, hi=1.02)
    rho_g, _, a_g = run_force(cuda, cfg, pos, vel, terms)
    rho, si, cst = check_density(cfg, pos, rho_g)
    args = (*pos, *vel, rho, cfg.cell_size, cfg.dims, cst, si, 1e-4)
    _, a = oracle.force(oparams(cfg), terms, *args, threads=oracle.max_threads())
    _, scale = oracle.force(oparams(cfg), terms | 4, *args, threads=oracle.max_threads())
    assert_force_close(a_g, a, scale)


def make_step(cfg):
    sp = forge_sph.StepParams()
    sp.dt = cfg.dt
    sp.gravity[:] = list(cfg.gravity)
    sp.box_min[:] = list(cfg.box_min)
    sp.box_max[:] = list(cfg.box_max)
    sp.restitution = cfg.restitution
    sp.flags = 7
    osp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    return sp, osp


def gpu_steps(torch, cfg, pos, vel, steps):
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    p, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    sp, _ = make_step(cfg)
    L = forge_sph.lib()
    for _ in range(steps):
        forge_sph.check(L.forge_sph_step(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp),
                                         *(x.data_ptr() for x in p), *(x.data_ptr() for x in v), rho.data_ptr(),
                                         cfg.n, None))
    g.check()
    return [host_f32(x) for x in p], [host_f32(x) for x in v], host_f32(rho)


def test_single_step_vs_oracle(cuda):
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    pg, vg, rg = gpu_steps(cuda, cfg, pos, vel, 1)
    po, vo = [x.copy() for x in pos], [x.copy() for x in vel]
    _, osp = make_step(cfg)
    ro = oracle.step(oparams(cfg), osp, po, vo, cfg.cell_size, cfg.dims, threads=oracle.max_threads(),
                     want_density=True)
    np.testing.assert_allclose(rg, ro, rtol=RHO_TOL)
    for k in range(3):
        np.testing.assert_allclose(pg[k], po[k], rtol=0, atol=1e-6)
        np.testing.assert_allclose(vg[k], vo[k], rtol=1e-4, atol=1e-6)


def test_trajectory_100_steps_cfg0(cuda):
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    pg, vg, _ = gpu_steps(cuda, cfg, pos, vel, 100)
    po, vo = [x.copy() for x in pos], [x.copy() for x in vel]
    _, osp = make_step(cfg)
    for _ in range(100):
        oracle.step(oparams(cfg), osp, po, vo, cfg.cell_size, cfg.dims, threads=oracle.max_threads())
    for k in range(3):
        np.testing.assert_allclose(pg[k], po[k], rtol=0, atol=1e-5)
        np.testing.assert_allclose(vg[k], vo[k], rtol=0, atol=3e-5)
        loose = np.abs(vg[k] - vo[k]) > 1e-4 * np.abs(vo[k]) + 1e-9
        assert loose.mean() <= 1e-3, loose.sum()


def test_step_is_deterministic(cuda):
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    a = gpu_steps(cuda, cfg, pos, vel, 5)
    b = gpu_steps(cuda, cfg, pos, vel, 5)
    for x, y in zip(a[0] + a[1], b[0] + b[1]):
        assert np.array_equal(x, y)


def test_pipeline_modules_match_fused_step(cuda):
    """Pipeline(SphFused, Gravity, Integrate, BoxCollider) takes the fused
    forge_sph_step path; the same modules run one by one must agree."""
    torch = cuda
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)

    def fields():
        f = forge_sph.FieldSet(cfg.n, 0)
        for a, x in zip("xyz", pos):
            f.add_f32("pos_" + a, x)
        for a, x in zip("xyz", vel):
            f.add_f32("vel_" + a, x)
        return f

    mods = [forge_sph.SphFusedModule(cfg.h, cfg.cell_size, cfg.dims, cfg.mass, cfg.gas_constant, cfg.rest_density,
                                     cfg.viscosity),
            forge_sph.GravityModule(*cfg.gravity), forge_sph.IntegrateModule(),
            forge_sph.BoxColliderModule(*cfg.box_min, *cfg.box_max, cfg.restitution)]
    fused = forge_sph.Pipeline()
    for m in mods:
        fused.add(m)
    f1 = fields()
    for _ in range(3):
        fused.step(f1, cfg.dt)
    f2 = fields()
    for _ in range(3):
        for m in mods:
            m.execute(f2, cfg.dt)
    torch.cuda.synchronize()
    for k in ("pos_x", "pos_y", "pos_z", "vel_x", "vel_y", "vel_z"):
        np.testing.assert_allclose(host_f32(f1.f32_fields[k]), host_f32(f2.f32_fields[k]), rtol=1e-5, atol=1e-7)


def test_unfused_modules_sequence(cuda):
    """SphDensity -> SphPressure -> SphViscosity (manifest_runner.rs:405-497):
    viscosity sees the pressure-updated velocities."""
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    f = forge_sph.FieldSet(cfg.n, 0)
    for a, x in zip("xyz", pos):
        f.add_f32("pos_" + a, x)
    for a, x in zip("xyz", vel):
        f.add_f32("vel_" + a, x)
    pipe = forge_sph.Pipeline()
    pipe.add(forge_sph.SphDensityModule(cfg.h, cfg.cell_size, cfg.dims, cfg.mass))
    pipe.add(forge_sph.SphPressureModule(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density))
    pipe.add(forge_sph.SphViscosityModule(cfg.h, cfg.mass, cfg.viscosity))
    pipe.step(f, cfg.dt)
    rho, si, cst = oracle_density(cfg, pos)
    p = oparams(cfg)
    th = oracle.max_threads()
    v1, _ = oracle.force(p, 1, *pos, *vel, rho, cfg.cell_size, cfg.dims, cst, si, cfg.dt, threads=th)
    v2, _ = oracle.force(p, 2, *pos, *v1, rho, cfg.cell_size, cfg.dims, cst, si, cfg.dt, threads=th)
    for k, a in enumerate("xyz"):
        np.testing.assert_allclose(host_f32(f.f32_fields["vel_" + a]), v2[k], rtol=1e-4, atol=1e-6)


def test_step_is_capture_safe_in_a_cuda_graph(cuda):
    """forge_sph_step only enqueues work (no allocation, no host sync), so a
    captured step replayed K times equals K eager steps bit for bit -- the way
    run_manifest drives the step (manifest_runner.rs:53-77)."""
    torch = cuda
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    eager = gpu_steps(torch, cfg, pos, vel, 4)
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    p, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    sp, _ = make_step(cfg)
    L = forge_sph.lib()
    args = [x.data_ptr() for x in p + v] + [rho.data_ptr()]
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        forge_sph.check(L.forge_sph_step(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp), *args, cfg.n,
                                         side.cuda_stream))
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    g.check()
    for x, y in zip([host_f32(t) for t in p + v], eager[0] + eager[1]):
        assert np.array_equal(x, y)


def _all_ops_modules(cfg):
    return [forge_sph.SphFusedModule(cfg.h, cfg.cell_size, cfg.dims, cfg.mass, cfg.gas_constant, cfg.rest_density,
                                     cfg.viscosity),
            forge_sph.GravityModule(0.0, -9.81, 0.0), forge_sph.DragModule(2.0), forge_sph.IntegrateModule(),
            forge_sph.GroundPlaneModule(0.05, 0.3), forge_sph.SphereColliderModule(0.5, 0.4, 0.5, 0.15, 0.6),
            forge_sph.BoxColliderModule(0, 0, 0, 1, 1, 1, 0.8)]


def test_fused_epilogue_ops_vs_oracle(cuda):
    """SphFused + gravity, drag, integrate, ground plane, sphere and box
    colliders (the waterfall / tsunami module mix) as one fused step, against
    the oracle applying the same modules in order."""
    cfg = workloads.config("ref65k")
    cfg.dt = 2e-3  # large enough that the ground and the sphere are hit
    pos, vel = workloads.uniform_particles(cfg.n, seed=91, vsigma=0.5)
    pipe = forge_sph.Pipeline()
    for m in _all_ops_modules(cfg):
        pipe.add(m)
    sp = pipe._fused_plan()
    assert sp is not None and sp.n_ops == 6
    f = forge_sph.FieldSet(cfg.n, 0)
    for a, x in zip("xyz", pos):
        f.add_f32("pos_" + a, x)
    for a, x in zip("xyz", vel):
        f.add_f32("vel_" + a, x)
    pipe.step(f, cfg.dt)
    osp = oracle.StepParams()
    osp.dt = cfg.dt
    osp.n_ops = sp.n_ops
    for k in range(sp.n_ops):
        osp.ops[k].kind = sp.ops[k].kind
        for q in range(7):
            osp.ops[k].p[q] = sp.ops[k].p[q]
    po, vo = [x.copy() for x in pos], [x.copy() for x in vel]
    oracle.step(oparams(cfg), osp, po, vo, cfg.cell_size, cfg.dims, threads=oracle.max_threads())
    inside = 0
    for k, a in enumerate("xyz"):
        gp, gv = host_f32(f.f32_fields["pos_" + a]), host_f32(f.f32_fields["vel_" + a])
        np.testing.assert_allclose(gp, po[k], rtol=0, atol=2e-6)
        np.testing.assert_allclose(gv, vo[k], rtol=1e-4, atol=2e-5)
    d = np.sqrt((po[0] - 0.5) ** 2 + (po[1] - 0.4) ** 2 + (po[2] - 0.5) ** 2)
    assert (np.abs(d - 0.15) < 1e-5).sum() > 0, "no particle was pushed onto the sphere"
    assert (po[1] == np.float32(0.05)).sum() > 0, "no particle hit the ground plane"


def _force_step_run(torch, cfg, pos, vel, n_update, zones, walk=forge_sph.WALK_THREAD):
    """forge_sph_density + forge_sph_force_step (zones None) or the split
    forge_sph_force_step_zone calls (zones = [(mode, inner_lo, inner_hi,
    guard_lo, guard_hi), ...])."""
    L = forge_sph.lib()
    sp, _ = make_step(cfg)
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    g.set_walk(walk)
    p, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
    rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
    forge_sph.check(L.forge_sph_density(g.handle, ctypes.byref(gparams(cfg)), *(x.data_ptr() for x in p), cfg.n,
                                        rho.data_ptr(), None))
    args = [x.data_ptr() for x in p + v] + [rho.data_ptr(), cfg.n, n_update]
    if zones is None:
        forge_sph.check(L.forge_sph_force_step(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp), *args, None))
    else:
        for z in zones:
            forge_sph.check(L.forge_sph_force_step_zone(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp), *args,
                                                        ctypes.byref(forge_sph.ForceZone(*z)), None))
    return g, [host_f32(t) for t in p + v]


@pytest.mark.parametrize("name,walk", [("ref65k", forge_sph.WALK_THREAD), ("dambreak65k", forge_sph.WALK_THREAD),
                                       ("dambreak65k", forge_sph.WALK_GROUP8), ("dambreak65k", forge_sph.WALK_ROWS)])
def test_zoned_force_step_equals_whole_pass(cuda, name, walk):
    """Boundary zone then interior zone (the split a sharded step overlaps
    its exchange with) updates every particle exactly once, ghosts
    (i >= n_update) untouched. Per-thread walks (pair and single-particle
    force kernels) and row-parallel walks (a particle's sum involves no other
    particle) equal the single forge_sph_force_step bit for bit; a group
    walk splits a particle's candidates over lanes by the particles that
    share its warp, which differ between a zone list and the whole cell
    order, so it agrees to fp32 rounding."""
    cfg = workloads.config(name)
    pos, vel = workloads.particles(cfg)
    n_upd = cfg.n - 1000
    zones = (0.31, 0.59, 0.25, 0.65)  # interior: x-slices 50..93 (cs/4 = 0.00625 wide) inside [0.31, 0.59)
    g0, want = _force_step_run(cuda, cfg, pos, vel, n_upd, None, walk)
    g1, got = _force_step_run(cuda, cfg, pos, vel, n_upd, [(1,) + zones, (2,) + zones], walk)
    g1.check()
    for a, b in zip(got, want):
        if walk in (forge_sph.WALK_THREAD, forge_sph.WALK_ROWS):
            assert np.array_equal(a, b)
        else:
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-7)
    for a, b in zip(got, pos + vel):
        assert np.array_equal(a[n_upd:], b[n_upd:])
    if walk != forge_sph.WALK_THREAD:
        return
    # the boundary pass alone leaves the interior particles as they were
    _, half = _force_step_run(cuda, cfg, pos, vel, n_upd, [(1,) + zones], walk)
    fx = pos[0] / np.float32(cfg.cell_size)  # the kernels' slice of x: cell * 4 + floor(4 * frac)
    cx = np.clip(np.floor(fx), 0, cfg.dims[0] - 1)
    k = cx * 4 + np.clip(np.floor((fx - cx.astype(np.float32)) * np.float32(4)), 0, 3)
    inner = (k >= 50) & (k < 94)
    inner[n_upd:] = False
    assert inner.sum() > 1000
    outer = ~inner
    outer[n_upd:] = False
    for a, b, c in zip(half, pos + vel, want):
        assert np.array_equal(a[inner], b[inner])
        assert np.array_equal(a[outer], c[outer])


def test_zoned_force_step_guard_and_order(cuda):
    """An interior particle that ends outside [guard_lo, guard_hi) sets
    FORGE_DEV_ZONE (reported by forge_grid_check); an interior pass without a
    boundary pass of the same build is refused."""
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    g, _ = _force_step_run(cuda, cfg, pos, vel, cfg.n, [(1, 0.3, 0.6, 0.25, 0.65), (2, 0.3, 0.6, 0.45, 0.46)])
    with pytest.raises(forge_sph.ForgeError, match="0x8"):
        g.check()
    with pytest.raises(forge_sph.ForgeError, match="interior pass must follow"):
        _force_step_run(cuda, cfg, pos, vel, cfg.n, [(2, 0.3, 0.6, 0.25, 0.65)])


def test_zoned_prepare_then_late_ghost_densities(cuda):
    """The overlapped sharded order: prepare (gather + lists) with stale ghost
    densities, the ghosts' exact densities written afterwards, then the
    boundary pass (which re-reads them) and the interior pass on a second
    stream -- equal to one forge_sph_force_step on the exact densities."""
    torch = cuda
    cfg = workloads.config("ref65k")
    pos, vel = workloads.particles(cfg)
    n_own = cfg.n - 5000  # the last 5000 play the ghosts
    L = forge_sph.lib()
    sp, _ = make_step(cfg)
    zones = (0.31, 0.59, 0.25, 0.65)

    def run(split):
        g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
        g.set_walk(forge_sph.WALK_THREAD)  # bit-for-bit comparison (see the zoned test above)
        p, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
        rho = torch.empty(cfg.n, dtype=torch.float32, device="cuda")
        forge_sph.check(L.forge_sph_density(g.handle, ctypes.byref(gparams(cfg)), *(x.data_ptr() for x in p), cfg.n,
                                            rho.data_ptr(), None))
        args = [x.data_ptr() for x in p + v] + [rho.data_ptr(), cfg.n, n_own]
        if not split:
            forge_sph.check(L.forge_sph_force_step(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp), *args,
                                                   None))
        else:
            exact = rho[n_own:].clone()
            rho[n_own:] *= 1.5  # stale ghost densities at prepare time

            def zone(mode, stream):
                forge_sph.check(L.forge_sph_force_step_zone(g.handle, ctypes.byref(gparams(cfg)), ctypes.byref(sp),
                                                            *args, ctypes.byref(forge_sph.ForceZone(mode, *zones)),
                                                            stream.cuda_stream))
            main = torch.cuda.current_stream()
            zone(forge_sph.ZONE_PREPARE, main)
            side = torch.cuda.Stream(priority=-1)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                rho[n_own:] = exact  # the density round
                zone(forge_sph.ZONE_BOUNDARY, side)
            zone(forge_sph.ZONE_INTERIOR, main)
            main.wait_stream(side)
        torch.cuda.synchronize()
        g.check()
        return [host_f32(t) for t in p + v]

    want, got = run(False), run(True)
    for a, b in zip(got, want):
        assert np.array_equal(a, b)


def test_apply_ops_unfused_modules_vs_oracle(cuda):
    """forge_apply_ops (the per-particle modules of an unfused pipeline) on
    every particle, against the oracle applying the same op list."""
    torch = cuda
    n = 50_000
    pos, vel = workloads.uniform_particles(n, seed=17, vsigma=0.5)
    ops = [(forge_sph.OP_GRAVITY, [0.0, -9.81, 0.0]), (forge_sph.OP_DRAG, [2.0]), (forge_sph.OP_INTEGRATE, []),
           (forge_sph.OP_GROUND, [0.05, 0.3]), (forge_sph.OP_SPHERE, [0.5, 0.4, 0.5, 0.15, 0.6]),
           (forge_sph.OP_BOX, [0.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.8])]
    sp, osp = forge_sph.StepParams(), oracle.StepParams()
    for s in (sp, osp):
        s.dt = 0.05  # large: particles reach the ground, the sphere and the walls
        s.n_ops = len(ops)
        for k, (kind, prm) in enumerate(ops):
            s.ops[k].kind = kind
            for q, val in enumerate(prm):
                s.ops[k].p[q] = val
    p, v = [dev(torch, x) for x in pos], [dev(torch, x) for x in vel]
    forge_sph.check(forge_sph.lib().forge_apply_ops(ctypes.byref(sp), *(x.data_ptr() for x in p + v), n, 0, None))
    torch.cuda.synchronize()
    po, vo = [x.copy() for x in pos], [x.copy() for x in vel]
    oracle.apply_ops(osp, po, vo)
    for k in range(3):
        np.testing.assert_allclose(host_f32(p[k]), po[k], rtol=0, atol=2e-6)
        np.testing.assert_allclose(host_f32(v[k]), vo[k], rtol=1e-4, atol=2e-5)
    assert (po[1] == np.float32(0.05)).sum() > 0, "no particle hit the ground plane"
