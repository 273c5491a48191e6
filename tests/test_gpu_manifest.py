"""GPU run of a TOML manifest (manifest.run_manifest): the fused pipeline
captured as one CUDA graph of `substeps` forge_sph_step calls and replayed,
against the same steps run eagerly."""
import numpy as np
import pytest

import manifest
from test_manifest import DAM

pytestmark = pytest.mark.gpu


def test_captured_manifest_run_equals_eager_run(cuda):
    m = manifest.Manifest.from_toml(DAM)
    a = manifest.run_manifest(m, seed=3, capture=True, steps=6)
    b = manifest.run_manifest(m, seed=3, capture=False, steps=6)
    assert a.steps == b.steps == 6 * 4
    assert a.pipeline == ["sph_fused", "gravity", "integrate", "ground_plane", "box_collider"]
    assert np.array_equal(a.positions, b.positions)
    p = a.positions
    assert np.isfinite(p).all()
    assert (p >= 0.0).all() and (p <= 1.0).all() and (p[:, 1] >= np.float32(0.02)).all()
    start = manifest.initial_fields(m, seed=3)
    assert not np.array_equal(p[:, 1], start["pos_y"])  # it moved (gravity)
    assert a.throughput > 0


def test_manifest_run_vs_oracle(cuda):
    """The `forge run` path end to end (manifest.run_manifest: TOML ->
    fields -> fused pipeline -> captured graph replays,
    manifest_runner.rs:43-78) against the oracle stepping the same initial
    fields with the same module list (SPH, gravity, integrate, ground plane,
    box) for the same 20 steps: positions within 1e-5 (fp32 summation order
    differs, as in the 100-step trajectory test)."""
    import oracle
    m = manifest.Manifest.from_toml(DAM)
    got = manifest.run_manifest(m, seed=3, capture=True, steps=5)
    assert got.steps == 20
    pipe = manifest.build_pipeline(m)
    sph, sp = pipe.modules[0], pipe._fused_plan()
    osp = oracle.StepParams()
    osp.dt = float(np.float32(m.simulation["dt"]))
    osp.n_ops = sp.n_ops
    for k in range(sp.n_ops):
        osp.ops[k].kind = sp.ops[k].kind
        for q in range(7):
            osp.ops[k].p[q] = sp.ops[k].p[q]
    op = oracle.SphParams(sph.smoothing_radius, sph.particle_mass, sph.gas_constant, sph.rest_density,
                          sph.viscosity_coefficient)
    f = manifest.initial_fields(m, seed=3)
    pos = [f["pos_" + a].copy() for a in "xyz"]
    vel = [f["vel_" + a].copy() for a in "xyz"]
    for _ in range(got.steps):
        oracle.step(op, osp, pos, vel, sph.cell_size, tuple(sph.grid_dims), threads=oracle.max_threads())
    want = np.stack(pos, axis=1)
    np.testing.assert_allclose(got.positions, want, rtol=0, atol=1e-5)
    assert np.abs(want - np.stack([f["pos_" + a] for a in "xyz"], axis=1)).max() > 1e-5  # the particles moved
