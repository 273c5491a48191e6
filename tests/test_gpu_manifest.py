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
