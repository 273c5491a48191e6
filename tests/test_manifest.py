"""Manifest runner host logic (forge-gpu_b200/manifest.py): schema defaults,
validation, field initialisation, pipeline construction and fusion. The
captured run itself is a GPU test."""
import numpy as np
import pytest

import forge_sph
import manifest

DAM = """
[simulation]
name = "dam"
dt = 0.0001
substeps = 4
duration = 0.01
count = 3000

[[fields]]
name = "position"
init = { type = "random", min = [0.0, 0.0, 0.0], max = [0.4, 0.8, 0.4] }

[[fields]]
name = "velocity"
init = { type = "zero" }

[spatial]
cell_size = 0.05
grid_dims = [20, 20, 20]

[[forces]]
type = "sph_density"
smoothing_radius = 0.05

[[forces]]
type = "sph_pressure"
gas_constant = 3.0
rest_density = 1000.0

[[forces]]
type = "sph_viscosity"
coefficient = 0.1

[[forces]]
type = "gravity"

[[constraints]]
type = "ground_plane"
y = 0.02

[[constraints]]
type = "box"
min = [0.0, 0.0, 0.0]
max = [1.0, 1.0, 1.0]
restitution = 0.3
"""


def test_schema_defaults_and_counts():
    m = manifest.Manifest.from_toml(DAM)
    assert m.particle_count() == 3000
    assert m.total_steps() == 25  # (0.01 / 1e-4) / 4
    assert m.forces[3]["value"] == [0.0, -9.81, 0.0]
    assert m.constraints[0]["restitution"] == 0.5 and m.constraints[1]["restitution"] == 0.3
    bare = manifest.Manifest.from_toml('[simulation]\nname = "x"\n[[fields]]\nname = "p"\ncount = 7\n')
    assert (bare.simulation["dt"], bare.simulation["substeps"], bare.simulation["duration"]) == (0.001, 1, 1.0)
    assert bare.particle_count() == 7
    assert manifest.Manifest.from_toml('[simulation]\nname = "x"\n').particle_count() == 1000


@pytest.mark.parametrize("text,msg", [
    ('[simulation]\nname = "x"\ndt = 0.0\n', "dt must be > 0"),
    ('[simulation]\nname = "x"\nduration = -1.0\n', "duration must be > 0"),
    ('[simulation]\nname = "x"\ncount = 0\n', "count > 0"),
    ('[simulation]\nname = "x"\n[[forces]]\ntype = "gravity"\nvalue = [0.0, 1.0]\n', "3 components"),
    ('[simulation]\nname = "x"\n[[constraints]]\ntype = "sphere"\ncenter = [0.0]\nradius = 1.0\n', "3 components"),
])
def test_validation_errors(text, msg):
    errs = manifest.validate(manifest.Manifest.from_toml(text))
    assert any(msg in e for e in errs), errs


@pytest.mark.parametrize("text", [
    "not toml [",
    '[simulation]\ndt = 1.0\n',
    '[simulation]\nname = "x"\n[[forces]]\ntype = "magnet"\n',
    '[simulation]\nname = "x"\n[[forces]]\ntype = "sph_density"\n',
    '[simulation]\nname = "x"\n[[constraints]]\ntype = "box"\nmin = [0, 0, 0]\n',
    '[simulation]\nname = "x"\n[[fields]]\nname = "p"\ninit = { type = "spiral" }\n',
])
def test_parse_errors(text):
    with pytest.raises(manifest.ManifestError):
        manifest.Manifest.from_toml(text)


def test_initial_fields():
    m = manifest.Manifest.from_toml(DAM)
    f = manifest.initial_fields(m, seed=5)
    assert set(f) == {"pos_x", "pos_y", "pos_z", "vel_x", "vel_y", "vel_z"}
    assert all(a.dtype == np.float32 and a.size == 3000 for a in f.values())
    assert f["pos_y"].min() >= 0.0 and f["pos_y"].max() < 0.8 and f["pos_x"].max() < 0.4
    assert not f["vel_x"].any()
    g = manifest.initial_fields(m, seed=5)
    assert all(np.array_equal(f[k], g[k]) for k in f)  # seeded
    grid = manifest.Manifest.from_toml('[simulation]\nname = "c"\ncount = 10\n[[fields]]\nname = "pos"\n'
                                       'init = { type = "grid", spacing = 0.5, origin = [1.0, 2.0, 3.0] }\n'
                                       '[[fields]]\nname = "mass"\ntype = "f32"\n'
                                       'init = { type = "constant", value = [2.5] }\n')
    f = manifest.initial_fields(grid)
    side = 4  # ceil(sqrt(10))
    assert np.array_equal(f["pos_x"], (1.0 + (np.arange(10) % side) * 0.5).astype(np.float32))
    assert np.array_equal(f["pos_z"], (3.0 + (np.arange(10) // side) * 0.5).astype(np.float32))
    assert (f["pos_y"] == 2.0).all() and (f["mass"] == 2.5).all()
    assert not f["vel_z"].any()  # velocity added as zeros


def test_fused_pipeline_and_its_step_plan():
    m = manifest.Manifest.from_toml(DAM)
    p = manifest.build_pipeline(m)
    assert [x.name() for x in p.modules] == ["sph_fused", "gravity", "integrate", "ground_plane", "box_collider"]
    sph = p.modules[0]
    assert sph.particle_mass == float(np.float32(1000.0) / np.float32(3000) * np.float32(0.001))
    assert (sph.cell_size, tuple(sph.grid_dims), sph.gas_constant, sph.viscosity_coefficient) == \
        (0.05, (20, 20, 20), 3.0, 0.1)
    sp = p._fused_plan()
    assert sp is not None and sp.n_ops == 4
    assert [sp.ops[k].kind for k in range(4)] == [forge_sph.OP_GRAVITY, forge_sph.OP_INTEGRATE,
                                                   forge_sph.OP_GROUND, forge_sph.OP_BOX]


def test_unfused_pipeline_order_and_rejections():
    text = DAM.replace('[[forces]]\ntype = "sph_viscosity"\ncoefficient = 0.1\n', "")
    p = manifest.build_pipeline(manifest.Manifest.from_toml(text))
    assert [x.name() for x in p.modules] == ["sph_density", "sph_pressure", "gravity", "integrate", "ground_plane",
                                             "box_collider"]
    assert p._fused_plan() is None
    with pytest.raises(manifest.ManifestError, match="custom"):
        manifest.build_pipeline(manifest.Manifest.from_toml(DAM + '\n[[forces]]\ntype = "custom"\nexpr = "v"\n'))
    with pytest.raises(manifest.ManifestError, match="springs"):
        manifest.build_pipeline(manifest.Manifest.from_toml(DAM + '\n[springs]\nstiffness = 1.0\ndamping = 0.1\n'))


def test_example_dam_break_manifest():
    """The shipped example (the reference's published 50K dam-break workload)
    parses, validates and fuses into one forge_sph_step per substep."""
    import os
    path = os.path.join(os.path.dirname(manifest.__file__), "examples", "dam_break_50k.toml")
    m = manifest.Manifest.from_file(path)
    assert manifest.validate(m) == []
    assert m.particle_count() == 50000 and m.total_steps() == 2000 and m.simulation["substeps"] == 10
    p = manifest.build_pipeline(m)
    assert [x.name() for x in p.modules] == ["sph_fused", "gravity", "integrate", "box_collider"]
    assert p._fused_plan() is not None
    sph = p.modules[0]
    assert (sph.smoothing_radius, sph.cell_size, tuple(sph.grid_dims)) == (0.025, 0.05, (40, 60, 20))
